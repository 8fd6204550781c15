// Peer memory for the multi-GPU row exchange: exportable device buffers,
// CUDA IPC handles, and copy-engine copies into a peer's buffer.
//
// The reference runs on one GPU and has no counterpart; these entry points
// serve the row-partitioned mode. After each row piece of a layer's output is
// written into this rank's slice of the next layer's input, the host pushes
// that slice into every peer's copy of the same buffer with one
// cudaMemcpyAsync per peer. The copy engines move the bytes over NVLink, so
// no SM is taken away from the aggregation kernel of the next piece, which
// runs at the same time.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "common.cuh"

using namespace gnnb200;

namespace {

struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
    else cudaGetLastError();
  }
  ~DeviceGuard() {
    if (ok && prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int gnn_peer_alloc(size_t bytes, int device, void** ptr) {
  GNN_REQUIRE(ptr != nullptr, GNN_ERR_NULL_POINTER, "ptr must not be NULL");
  GNN_REQUIRE(device >= 0, GNN_ERR_INVALID_ARGUMENT, "device must be >= 0");
  GNN_REQUIRE(bytes > 0, GNN_ERR_INVALID_ARGUMENT, "bytes must be > 0");
  *ptr = nullptr;
  DeviceGuard g(device);
  GNN_REQUIRE(g.ok, GNN_ERR_DEVICE, "cannot select CUDA device " + std::to_string(device));
  GNN_CUDA_TRY(cudaMalloc(ptr, bytes), "cudaMalloc");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_peer_free(void* ptr, int device) {
  if (ptr == nullptr) {
    clear_error();
    return GNN_OK;
  }
  DeviceGuard g(device);
  GNN_REQUIRE(g.ok, GNN_ERR_DEVICE, "cannot select CUDA device " + std::to_string(device));
  GNN_CUDA_TRY(cudaFree(ptr), "cudaFree");
  clear_error();
  return GNN_OK;
}

extern "C" size_t gnn_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int gnn_ipc_get_handle(const void* ptr, void* handle, size_t handle_bytes) {
  GNN_REQUIRE(ptr != nullptr && handle != nullptr, GNN_ERR_NULL_POINTER, "ptr and handle must not be NULL");
  GNN_REQUIRE(handle_bytes >= sizeof(cudaIpcMemHandle_t), GNN_ERR_INVALID_ARGUMENT,
              "handle buffer smaller than " + std::to_string(sizeof(cudaIpcMemHandle_t)) + " bytes");
  cudaIpcMemHandle_t h;
  GNN_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_ipc_open(const void* handle, size_t handle_bytes, int device, void** ptr) {
  GNN_REQUIRE(handle != nullptr && ptr != nullptr, GNN_ERR_NULL_POINTER, "handle and ptr must not be NULL");
  GNN_REQUIRE(handle_bytes >= sizeof(cudaIpcMemHandle_t), GNN_ERR_INVALID_ARGUMENT,
              "handle smaller than " + std::to_string(sizeof(cudaIpcMemHandle_t)) + " bytes");
  *ptr = nullptr;
  DeviceGuard g(device);
  GNN_REQUIRE(g.ok, GNN_ERR_DEVICE, "cannot select CUDA device " + std::to_string(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  GNN_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_ipc_close(void* ptr, int device) {
  if (ptr == nullptr) {
    clear_error();
    return GNN_OK;
  }
  DeviceGuard g(device);
  GNN_REQUIRE(g.ok, GNN_ERR_DEVICE, "cannot select CUDA device " + std::to_string(device));
  GNN_CUDA_TRY(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_can_access_peer(int device, int peer, int* can) {
  GNN_REQUIRE(can != nullptr, GNN_ERR_NULL_POINTER, "can must not be NULL");
  *can = 0;
  GNN_CUDA_TRY(cudaDeviceCanAccessPeer(can, device, peer), "cudaDeviceCanAccessPeer");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_copy_async(void* dst, const void* src, size_t bytes, gnn_stream_t stream) {
  if (bytes == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(dst != nullptr && src != nullptr, GNN_ERR_NULL_POINTER, "dst and src must not be NULL");
  GNN_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
               "cudaMemcpyAsync");
  clear_error();
  return GNN_OK;
}

namespace {

constexpr int kMaxPeers = 8;

struct PeerTargets {
  char* dst[kMaxPeers];
};

// Reads each 16-byte word of src once and stores it into every target (peer
// buffers mapped through CUDA IPC): the SMs drive the NVLink writes.
__global__ void __launch_bounds__(512) push_rows_kernel(const int4* __restrict__ src, PeerTargets t, int ntargets,
                                                        int64_t words) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < words; i += stride) {
    const int4 v = __ldg(src + i);
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p) {
      if (p < ntargets) reinterpret_cast<int4*>(t.dst[p])[i] = v;
    }
  }
}

}  // namespace

extern "C" int gnn_peer_push(const void* src, void* const* dsts, int ndst, size_t bytes, int ctas,
                             gnn_stream_t stream) {
  if (bytes == 0 || ndst == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(src != nullptr && dsts != nullptr, GNN_ERR_NULL_POINTER, "src and dsts must not be NULL");
  GNN_REQUIRE(ndst > 0 && ndst <= kMaxPeers, GNN_ERR_INVALID_ARGUMENT,
              "ndst must be in 1.." + std::to_string(kMaxPeers));
  GNN_REQUIRE(bytes % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0, GNN_ERR_INVALID_ARGUMENT,
              "bytes and src must be multiples of 16");
  PeerTargets t{};
  for (int p = 0; p < ndst; ++p) {
    GNN_REQUIRE(dsts[p] != nullptr && reinterpret_cast<uintptr_t>(dsts[p]) % 16 == 0, GNN_ERR_INVALID_ARGUMENT,
                "every destination must be a 16-byte aligned, non-NULL pointer");
    t.dst[p] = static_cast<char*>(dsts[p]);
  }
  const int64_t words = static_cast<int64_t>(bytes / 16);
  const int64_t want = (words + 511) / 512;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, ctas > 0 ? ctas : 4 * sm_count())));
  push_rows_kernel<<<grid, 512, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const int4*>(src), t, ndst,
                                                                       words);
  GNN_LAUNCH_CHECK("peer push kernel launch");
  clear_error();
  return GNN_OK;
}

namespace {

struct ListedTargets {
  char* dst[kMaxPeers];
  int64_t off[kMaxPeers + 1];  // rows [off[q], off[q+1]) of the id list go to dst[q]
};

// One warp per listed row: copies row ids[e] (row_bytes, 16-byte words) from
// src to the same row of the destination that owns list entry e. Every
// destination shares src's row layout, so the row offset is the same on both
// sides. Ids outside [0, max_rows) are skipped (the host validated them).
// Work item w goes to destination w % ntargets, entry w / ntargets of that
// destination's list: every destination is written at the same time. Walking
// the lists destination after destination instead made every rank write to the
// same peer at once (all ranks' lists share the peer order), so one GPU's
// incoming links carried the traffic of seven senders while the others idled.
__global__ void __launch_bounds__(512) push_listed_rows_kernel(const char* __restrict__ src, ListedTargets t,
                                                               int ntargets, const int32_t* __restrict__ ids,
                                                               int64_t row_words, int64_t max_rows,
                                                               int64_t max_count) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t items = max_count * ntargets;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < items;
       w += warps) {
    const int q = static_cast<int>(w % ntargets);
    const int64_t j = w / ntargets;
    const int64_t e = t.off[q] + j;
    if (e >= t.off[q + 1]) continue;  // this destination's list is shorter
    const int64_t row = ids[e];
    if (row < 0 || row >= max_rows) continue;
    const int4* s = reinterpret_cast<const int4*>(src) + row * row_words;
    int4* d = reinterpret_cast<int4*>(t.dst[q]) + row * row_words;
    for (int64_t k = lane; k < row_words; k += 32) d[k] = __ldg(s + k);
  }
}

}  // namespace

extern "C" int gnn_peer_push_rows(const void* src, void* const* dsts, int ndst, const int32_t* row_ids,
                                  const int64_t* row_offsets, int64_t row_bytes, int64_t max_rows, int ctas,
                                  gnn_stream_t stream) {
  GNN_REQUIRE(ndst >= 0 && ndst <= kMaxPeers, GNN_ERR_INVALID_ARGUMENT,
              "ndst must be in 0.." + std::to_string(kMaxPeers));
  if (ndst == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(dsts != nullptr && row_offsets != nullptr, GNN_ERR_NULL_POINTER,
              "dsts and row_offsets must not be NULL");
  ListedTargets t{};
  t.off[0] = row_offsets[0];
  GNN_REQUIRE(row_offsets[0] == 0, GNN_ERR_INVALID_ARGUMENT, "row_offsets must start at 0");
  for (int p = 0; p < ndst; ++p) {
    GNN_REQUIRE(row_offsets[p + 1] >= row_offsets[p], GNN_ERR_INVALID_ARGUMENT, "row_offsets must not decrease");
    t.off[p + 1] = row_offsets[p + 1];
  }
  for (int p = ndst + 1; p <= kMaxPeers; ++p) t.off[p] = t.off[ndst];
  const int64_t total = t.off[ndst];
  if (total == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(src != nullptr && row_ids != nullptr, GNN_ERR_NULL_POINTER, "src and row_ids must not be NULL");
  GNN_REQUIRE(row_bytes > 0 && row_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0,
              GNN_ERR_INVALID_ARGUMENT, "row_bytes and src must be multiples of 16");
  GNN_REQUIRE(max_rows > 0, GNN_ERR_INVALID_ARGUMENT, "max_rows must be > 0");
  for (int p = 0; p < ndst; ++p) {
    GNN_REQUIRE(dsts[p] != nullptr && reinterpret_cast<uintptr_t>(dsts[p]) % 16 == 0, GNN_ERR_INVALID_ARGUMENT,
                "every destination must be a 16-byte aligned, non-NULL pointer");
    t.dst[p] = static_cast<char*>(dsts[p]);
  }
  int64_t max_count = 0;
  for (int p = 0; p < ndst; ++p) max_count = std::max<int64_t>(max_count, t.off[p + 1] - t.off[p]);
  // Default grid: one CTA per SM. Measured on 8 B200s (products-shaped graph, halo push beside
  // the next piece's aggregation): 2.17 ms per step against 3.18 ms with four CTAs per SM,
  // whose push CTAs held every SM while the peers waited at the layer boundary.
  const int64_t want = (max_count * ndst + 15) / 16;  // 16 warps per 512-thread CTA
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, ctas > 0 ? ctas : sm_count())));
  push_listed_rows_kernel<<<grid, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const char*>(src), t, ndst, row_ids, row_bytes / 16, max_rows, max_count);
  GNN_LAUNCH_CHECK("peer row-list push kernel launch");
  clear_error();
  return GNN_OK;
}
