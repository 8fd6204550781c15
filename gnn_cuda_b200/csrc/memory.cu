// Unified / host memory entry points: the allocator family of the C ABI.
//
// Replaces GNN_cuda_common/native/uvm_allocator.cu:93-269 and the pointer
// resolution of tensor_access.cuh:25-64. Differences from the reference, all
// deliberate: prefetches take the caller's stream (the reference always used
// the device's default stream), and pointer information is returned as a plain
// struct that the Python layer turns into the reference's dict.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "common.cuh"

using namespace gnnb200;

namespace {

int pageable_access(int device) {
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrPageableMemoryAccess, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return v != 0;
}

int current_pageable_access() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return pageable_access(dev);
}

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

int advise(void* ptr, size_t bytes, cudaMemoryAdvise what, int location, int device) {
  const int target = (location == 0) ? device : location;
#if CUDART_VERSION >= 13000
  cudaMemLocation loc{};
  loc.type = target < 0 ? cudaMemLocationTypeHost : cudaMemLocationTypeDevice;
  loc.id = target < 0 ? 0 : target;
  GNN_CUDA_TRY(cudaMemAdvise(ptr, bytes, what, loc), "cudaMemAdvise");
#else
  GNN_CUDA_TRY(cudaMemAdvise(ptr, bytes, what, target), "cudaMemAdvise");
#endif
  return GNN_OK;
}

}  // namespace

extern "C" int gnn_managed_alloc(size_t bytes, int device, void** ptr) {
  GNN_REQUIRE(ptr != nullptr, GNN_ERR_NULL_POINTER, "ptr must not be NULL");
  GNN_REQUIRE(device >= 0, GNN_ERR_INVALID_ARGUMENT, "device_index must be >= 0");
  *ptr = nullptr;
  if (bytes == 0) {
    clear_error();
    return GNN_OK;
  }
  DeviceGuard g(device);
  GNN_REQUIRE(g.ok, GNN_ERR_DEVICE, "cannot select CUDA device " + std::to_string(device));
  GNN_CUDA_TRY(cudaMallocManaged(ptr, bytes, cudaMemAttachGlobal), "cudaMallocManaged");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_managed_free(void* ptr, int device) {
  if (ptr == nullptr) {
    clear_error();
    return GNN_OK;
  }
  DeviceGuard g(device);
  GNN_CUDA_TRY(cudaFree(ptr), "cudaFree");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_hmm_supported(int device, int* supported) {
  GNN_REQUIRE(supported != nullptr, GNN_ERR_NULL_POINTER, "supported must not be NULL");
  GNN_REQUIRE(device >= 0, GNN_ERR_INVALID_ARGUMENT, "device_index must be >= 0");
  int v = 0;
  GNN_CUDA_TRY(cudaDeviceGetAttribute(&v, cudaDevAttrPageableMemoryAccess, device),
               "cudaDeviceGetAttribute(PageableMemoryAccess)");
  *supported = v != 0;
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_copy_host_to_managed(void* dst, const void* src, size_t bytes) {
  if (bytes == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(dst != nullptr && src != nullptr, GNN_ERR_NULL_POINTER, "dst and src must not be NULL");
  cudaPointerAttributes attrs{};
  GNN_CUDA_TRY(cudaPointerGetAttributes(&attrs, dst), "cudaPointerGetAttributes");
  GNN_REQUIRE(attrs.type == cudaMemoryTypeManaged, GNN_ERR_INVALID_ARGUMENT,
              "Destination pointer is not cudaMallocManaged memory");
  std::memcpy(dst, src, bytes);
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_prefetch(void* ptr, size_t offset, size_t bytes, size_t total_bytes, int location,
                            int device, gnn_stream_t stream) {
  GNN_REQUIRE(device >= 0, GNN_ERR_INVALID_ARGUMENT, "device_index must be >= 0");
  GNN_REQUIRE(offset <= total_bytes, GNN_ERR_INVALID_ARGUMENT, "offset_bytes exceeds tensor byte size");
  GNN_REQUIRE(bytes <= total_bytes - offset, GNN_ERR_INVALID_ARGUMENT,
              "prefetch byte range exceeds tensor byte size");
  if (bytes == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(ptr != nullptr, GNN_ERR_NULL_POINTER, "ptr must not be NULL");
  DeviceGuard g(device);
  GNN_REQUIRE(g.ok, GNN_ERR_DEVICE, "cannot select CUDA device " + std::to_string(device));
  char* base = static_cast<char*>(ptr) + offset;
#if CUDART_VERSION >= 13000
  cudaMemLocation loc{};
  loc.type = location < 0 ? cudaMemLocationTypeHost : cudaMemLocationTypeDevice;
  loc.id = location < 0 ? 0 : location;
  GNN_CUDA_TRY(cudaMemPrefetchAsync(base, bytes, loc, 0, reinterpret_cast<cudaStream_t>(stream)),
               "cudaMemPrefetchAsync");
#else
  GNN_CUDA_TRY(cudaMemPrefetchAsync(base, bytes, location < 0 ? cudaCpuDeviceId : location,
                                    reinterpret_cast<cudaStream_t>(stream)),
               "cudaMemPrefetchAsync");
#endif
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_advise_preferred_location(void* ptr, size_t bytes, int location, int device) {
  if (bytes == 0) {
    clear_error();
    return GNN_OK;
  }
  DeviceGuard g(device);
  int rc = advise(ptr, bytes, cudaMemAdviseSetPreferredLocation, location < 0 ? cudaCpuDeviceId : location,
                  device);
  if (rc == GNN_OK) clear_error();
  return rc;
}

extern "C" int gnn_advise_accessed_by(void* ptr, size_t bytes, int location, int device) {
  if (bytes == 0) {
    clear_error();
    return GNN_OK;
  }
  DeviceGuard g(device);
  int rc = advise(ptr, bytes, cudaMemAdviseSetAccessedBy, location < 0 ? cudaCpuDeviceId : location,
                  device);
  if (rc == GNN_OK) clear_error();
  return rc;
}

extern "C" int gnn_advise_read_mostly(void* ptr, size_t bytes, int enabled, int device) {
  if (bytes == 0) {
    clear_error();
    return GNN_OK;
  }
  DeviceGuard g(device);
  int rc = advise(ptr, bytes, enabled ? cudaMemAdviseSetReadMostly : cudaMemAdviseUnsetReadMostly,
                  device, device);
  if (rc == GNN_OK) clear_error();
  return rc;
}

extern "C" int gnn_pointer_info_query(const void* ptr, gnn_pointer_info* info) {
  GNN_REQUIRE(info != nullptr, GNN_ERR_NULL_POINTER, "info must not be NULL");
  std::memset(info, 0, sizeof(*info));
  info->device = -1;
  info->pageable_access = current_pageable_access();
  cudaPointerAttributes attrs{};
  if (ptr == nullptr || cudaPointerGetAttributes(&attrs, ptr) != cudaSuccess) {
    cudaGetLastError();
    info->memory_type = -1;
    clear_error();
    return GNN_OK;
  }
  switch (attrs.type) {
    case cudaMemoryTypeHost: info->memory_type = 1; break;
    case cudaMemoryTypeDevice: info->memory_type = 2; break;
    case cudaMemoryTypeManaged: info->memory_type = 3; break;
    default: info->memory_type = 0; break;
  }
  info->device = attrs.device;
  info->is_managed = attrs.type == cudaMemoryTypeManaged;
  info->is_host_mapped = attrs.type == cudaMemoryTypeHost && attrs.devicePointer != nullptr;
  info->device_pointer = attrs.devicePointer;
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_device_accessible_ptr(const void* host_ptr, void** device_ptr) {
  GNN_REQUIRE(device_ptr != nullptr, GNN_ERR_NULL_POINTER, "device_ptr must not be NULL");
  *device_ptr = nullptr;
  if (host_ptr == nullptr) {
    clear_error();
    return GNN_OK;
  }
  cudaPointerAttributes attrs{};
  const cudaError_t st = cudaPointerGetAttributes(&attrs, host_ptr);
  if (st == cudaSuccess) {
    if (attrs.type == cudaMemoryTypeHost && attrs.devicePointer != nullptr) {
      *device_ptr = attrs.devicePointer;
      clear_error();
      return GNN_OK;
    }
    if (attrs.type == cudaMemoryTypeDevice || attrs.type == cudaMemoryTypeManaged) {
      *device_ptr = const_cast<void*>(host_ptr);
      clear_error();
      return GNN_OK;
    }
    if (attrs.type == cudaMemoryTypeUnregistered && current_pageable_access()) {
      *device_ptr = const_cast<void*>(host_ptr);
      clear_error();
      return GNN_OK;
    }
  } else {
    cudaGetLastError();
    if (current_pageable_access()) {
      *device_ptr = const_cast<void*>(host_ptr);
      clear_error();
      return GNN_OK;
    }
  }
  void* alias = nullptr;
  if (cudaHostGetDevicePointer(&alias, const_cast<void*>(host_ptr), 0) != cudaSuccess || alias == nullptr) {
    cudaGetLastError();
    return fail(GNN_ERR_DEVICE, "Failed to obtain a device alias for CPU mapped memory");
  }
  *device_ptr = alias;
  clear_error();
  return GNN_OK;
}
