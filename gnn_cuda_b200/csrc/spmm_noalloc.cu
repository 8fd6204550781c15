// GCN aggregation for callers that cannot hand the library a scratch buffer.
//
// gnn_spmm_gcn_forward needs a caller-provided workspace (the per-call list of
// long rows and its counters). Some callers have no way to provide one: a
// plugin host or FFI binding that owns every device allocation and only passes
// input/output buffers in; a process running at a fixed device-memory budget;
// or a latency-sensitive path that must not call cudaMalloc/cudaFree, which can
// block until the whole device is idle. gnn_spmm_gcn_forward_noalloc serves
// them: it runs exactly what gnn_spmm_gcn_forward runs when given the minimum
// workspace (gnn_spmm_workspace_bytes), with the same results, and takes that
// workspace from the fixed-size array below, which the CUDA runtime places in
// device memory when this module is loaded on a device and which stays there
// until the process exits. Nothing is allocated per call.
//
// Because only the minimum workspace is used, the per-row kernel takes rows in
// row-id order: the degree-ordered row schedule needs another 4 bytes per node
// (18,102,528 bytes in all for a 2,449,029-node, 64,308,169-entry graph, more
// than the array holds), so it never runs here. On power-law graphs that costs
// time, not accuracy (every row is summed the same way in either order).
//
// Limits and sharing rules (also in include/gnn_b200.h):
//   * the array holds kNoAllocScratchBytes (8 MiB); problems whose
//     gnn_spmm_workspace_bytes(num_nodes, num_edges) is larger are rejected
//     with GNN_ERR_UNSUPPORTED before any work is queued;
//   * there is one array per device, shared by every call on that device:
//     calls whose executions overlap on the GPU (different streams, or
//     different host threads) race on it and give wrong results — serialise
//     them, for example by using one stream;
//   * each call clears the counters it needs (the 256-byte header) on its own
//     stream before its kernels read them, so leftovers of the previous call
//     do not matter; the rest of the array is written before it is read;
//   * the first call on each device looks the array's device address up
//     (cudaGetSymbolAddress); make that first call before any stream capture
//     on that device. The address is kept for the life of the process, so a
//     cudaDeviceReset of that device after the first call is not supported
//     (the module is reloaded and the array may move).
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr int kMaxDevices = 64;

// Device-resident scratch. In host code this name is only a handle for the
// runtime, not a device address: the address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Looks the scratch address up once per device, with that device current.
int scratch_for_current_device(void** out) {
  int dev = -1;
  GNN_CUDA_TRY(cudaGetDevice(&dev), "gnn_spmm_gcn_forward_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    return gnnb200::fail(GNN_ERR_DEVICE, "gnn_spmm_gcn_forward_noalloc: device index out of range");
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    GNN_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                 "gnn_spmm_gcn_forward_noalloc: cudaGetSymbolAddress of the built-in scratch");
    if (p == nullptr) {
      return gnnb200::fail(GNN_ERR_CUDA, "gnn_spmm_gcn_forward_noalloc: built-in scratch has no device address");
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return GNN_OK;
}

}  // namespace

extern "C" int gnn_spmm_gcn_forward_noalloc(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                            const float* deg_inv_sqrt, const float* x, float* out,
                                            int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                                            gnn_stream_t stream) {
  if (num_nodes < 0 || num_edges < 0 || feat_dim < 0) {
    return gnnb200::fail(GNN_ERR_INVALID_ARGUMENT, "num_nodes, num_edges and feat_dim must be >= 0");
  }
  const size_t need = gnn_spmm_workspace_bytes(num_nodes, num_edges);
  if (need > kNoAllocScratchBytes) {
    return gnnb200::fail(GNN_ERR_UNSUPPORTED,
                         "gnn_spmm_gcn_forward_noalloc: this graph needs " + std::to_string(need) +
                             " bytes of scratch but the built-in scratch holds " +
                             std::to_string(kNoAllocScratchBytes) +
                             " bytes; call gnn_spmm_gcn_forward with a workspace instead");
  }
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != GNN_OK) return rc;
  // exactly the minimum workspace: the same launches as gnn_spmm_gcn_forward given need bytes
  return gnn_spmm_gcn_forward(row_ptr, row_ptr_type, col_ind, deg_inv_sqrt, x, out, num_nodes, num_edges,
                              feat_dim, scratch, need, stream);
}
