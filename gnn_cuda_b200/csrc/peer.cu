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
