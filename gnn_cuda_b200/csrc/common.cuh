// Shared internals of libgnnb200.so: status/error plumbing, tuning knobs and
// small device helpers. Nothing here is part of the public C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/gnn_b200.h"

namespace gnnb200 {

// ---- error reporting ---------------------------------------------------------
void set_error(const std::string& msg);
void clear_error();

// Returns `status` after recording `msg` as the thread's last error.
inline int fail(int status, const std::string& msg) {
  set_error(msg);
  return status;
}

// Checks the result of a CUDA runtime call; on failure records
// "<what>: <cuda error string>" and returns GNN_ERR_CUDA from the caller.
#define GNN_CUDA_TRY(expr, what)                                                   \
  do {                                                                             \
    cudaError_t err__ = (expr);                                                    \
    if (err__ != cudaSuccess) {                                                    \
      return ::gnnb200::fail(GNN_ERR_CUDA, std::string(what) + ": " +              \
                                               cudaGetErrorString(err__));         \
    }                                                                              \
  } while (0)

// Process-wide count of kernels launched by this library.
void count_launch();

// After a kernel launch: surfaces launch-configuration errors immediately, as
// the reference does with C10_CUDA_CHECK(cudaGetLastError()), and counts it.
#define GNN_LAUNCH_CHECK(what)                 \
  do {                                         \
    GNN_CUDA_TRY(cudaGetLastError(), what);    \
    ::gnnb200::count_launch();                 \
  } while (0)

#define GNN_REQUIRE(cond, status, msg)   \
  do {                                   \
    if (!(cond)) {                       \
      return ::gnnb200::fail(status, msg); \
    }                                    \
  } while (0)

// ---- tuning knobs ---------------------------------------------------------------
struct Config {
  std::atomic<int64_t> long_row_threshold{0};  // 0 = automatic
  std::atomic<int64_t> long_row_warps{16};
  std::atomic<int64_t> spmm_kernel{1};  // 0 packed stream, 1 one warp per row (default), 2 cp.async staging
  std::atomic<int64_t> gemm_stages{0};  // tcgen05 GEMM X-tile ring depth; 0 = as deep as shared memory allows
  // per-row kernel row order: 0 id order, 1 windowed degree, 2 global degree, 3 automatic (global below
  // a mean degree of 64 entries per row, windowed above)
  std::atomic<int64_t> spmm_schedule{3};
  std::atomic<int64_t> spmm_schedule_window{2048};  // rows per window of the windowed degree order
};
Config& config();

// Number of SMs of the current device (cached per device).
int sm_count();

// ---- device helpers ---------------------------------------------------------------
__device__ __forceinline__ float4 ldg_f4(const float4* p) { return __ldg(p); }

// Streaming (read-once) loads for index/weight arrays: do not keep them in L1
// (and, with GNN_STREAM_EVICT_FIRST, mark their L2 lines first to go).
#ifndef GNN_STREAM_EVICT_FIRST
#define GNN_STREAM_EVICT_FIRST 0
#endif
__device__ __forceinline__ int ld_stream_i32(const int32_t* p) {
  int v;
#if GNN_STREAM_EVICT_FIRST
  asm volatile(
      "{\n\t.reg .b64 pol;\n\t"
      "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
      "ld.global.nc.L1::no_allocate.L2::cache_hint.b32 %0, [%1], pol;\n\t}"
      : "=r"(v)
      : "l"(p));
#else
  asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
#endif
  return v;
}

// Aggregation output rows are written once per launch; with GNN_SPMM_STORE_CS
// they are stored with the streaming (evict-first) cache operator.
#ifndef GNN_SPMM_STORE_CS
#define GNN_SPMM_STORE_CS 0
#endif
__device__ __forceinline__ void st_out_f4(float4* p, float4 v) {
#if GNN_SPMM_STORE_CS
  __stcs(p, v);
#else
  *p = v;
#endif
}
__device__ __forceinline__ float ld_stream_f32(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float4 fma4(float w, float4 v, float4 acc) {
  acc.x = __fmaf_rn(w, v.x, acc.x);
  acc.y = __fmaf_rn(w, v.y, acc.y);
  acc.z = __fmaf_rn(w, v.z, acc.z);
  acc.w = __fmaf_rn(w, v.w, acc.w);
  return acc;
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  a.x = __fadd_rn(a.x, b.x);
  a.y = __fadd_rn(a.y, b.y);
  a.z = __fadd_rn(a.z, b.z);
  a.w = __fadd_rn(a.w, b.w);
  return a;
}

}  // namespace gnnb200
