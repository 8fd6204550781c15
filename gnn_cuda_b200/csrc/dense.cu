// Dense transform and elementwise epilogues.
//
//   gnn_gemm_forward / gnn_linear_forward  — replace gemm_forward_cuda_ /
//     linear_forward_cuda_ (GNN_cuda_common/native/agg_ops.cu:343-391). The
//     reference creates and destroys a cuBLAS handle per call and runs full
//     FP32 cublasSgemm; here GNN_PRECISION_FP32 is a register-tiled FFMA
//     kernel (k accumulated in increasing order) and GNN_PRECISION_TF32 runs on
//     the tcgen05 tensor cores (gemm_tc.cu). Bias and ReLU are fused into the
//     epilogue instead of a second pass over the output.
//   gnn_bias_relu_forward / gnn_tensor_add_inplace / gnn_relu_inplace —
//     replace the kernels of agg_ops.cu:132-166 with the same per-element
//     arithmetic (add then clamp; one fused multiply-add; compare-to-zero).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

namespace gnnb200 {

int gemm_tc_tf32(const float* x, const float* w, const float* bias, float* out, int64_t m,
                 int64_t k, int64_t n, bool relu, cudaStream_t stream, bool* handled);

namespace {

constexpr int BM = 128, BN = 128, BK = 8;

// 256 threads; thread (ty, tx) owns rows {ty*4+i, 64+ty*4+i} and columns
// {tx*4+j, 64+tx*4+j}, i, j < 4.
__global__ void __launch_bounds__(256) sgemm_kernel(const float* __restrict__ A,
                                                     const float* __restrict__ B,
                                                     const float* __restrict__ bias,
                                                     float* __restrict__ C, int64_t M, int64_t K,
                                                     int64_t N, int relu) {
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int t = threadIdx.x;
  const int tx = t & 15, ty = t >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * BM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * BN;

  // global -> register staging coordinates
  const int a_m = t >> 1, a_k = (t & 1) * 4;   // A tile: 128 x 8
  const int b_k = t >> 5, b_n = (t & 31) * 4;  // B tile: 8 x 128

  float ra[4], rb[4];
  auto load_tile = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gm = m0 + a_m, gk = k0 + a_k + i;
      ra[i] = (gm < M && gk < K) ? __ldg(A + gm * K + gk) : 0.0f;
      const int64_t bk = k0 + b_k, bn = n0 + b_n + i;
      rb[i] = (bk < K && bn < N) ? __ldg(B + bk * N + bn) : 0.0f;
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      As[buf][a_k + i][a_m] = ra[i];
      Bs[buf][b_k][b_n + i] = rb[i];
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  const int64_t ktiles = (K + BK - 1) / BK;
  load_tile(0);
  store_tile(0);
  __syncthreads();
  for (int64_t kt = 0; kt < ktiles; ++kt) {
    const int buf = static_cast<int>(kt & 1);
    if (kt + 1 < ktiles) load_tile((kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) {
      store_tile(buf ^ 1);
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias != nullptr) v = __fadd_rn(v, __ldg(bias + gn));
      if (relu && v < 0.0f) v = 0.0f;
      C[gm * N + gn] = v;
    }
  }
}

__global__ void bias_relu_kernel(float* __restrict__ out, const float* __restrict__ bias,
                                 int64_t rows, int64_t cols, int relu) {
  const int64_t count = rows * cols;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    float v = out[i];
    if (bias != nullptr) v = __fadd_rn(v, __ldg(bias + (i % cols)));
    if (relu && v < 0.0f) v = 0.0f;
    out[i] = v;
  }
}

// cols % 4 == 0 and 16-byte aligned pointers.
__global__ void bias_relu_vec_kernel(float4* __restrict__ out, const float4* __restrict__ bias,
                                     int64_t count4, int64_t cols4, int relu) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count4;
       i += stride) {
    float4 v = out[i];
    if (bias != nullptr) v = add4(v, __ldg(bias + (i % cols4)));
    if (relu) {
      if (v.x < 0.0f) v.x = 0.0f;
      if (v.y < 0.0f) v.y = 0.0f;
      if (v.z < 0.0f) v.z = 0.0f;
      if (v.w < 0.0f) v.w = 0.0f;
    }
    out[i] = v;
  }
}

__global__ void add_inplace_kernel(float* __restrict__ dst, const float* __restrict__ src,
                                   float alpha, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
  if (vec) {
    const int64_t count4 = count >> 2;
    float4* d4 = reinterpret_cast<float4*>(dst);
    const float4* s4 = reinterpret_cast<const float4*>(src);
    for (int64_t j = i; j < count4; j += stride) {
      float4 d = d4[j];
      const float4 s = __ldg(s4 + j);
      d.x = __fmaf_rn(alpha, s.x, d.x);
      d.y = __fmaf_rn(alpha, s.y, d.y);
      d.z = __fmaf_rn(alpha, s.z, d.z);
      d.w = __fmaf_rn(alpha, s.w, d.w);
      d4[j] = d;
    }
    for (int64_t j = count4 * 4 + (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
         j < count; j += stride) {
      dst[j] = __fmaf_rn(alpha, src[j], dst[j]);
    }
    return;
  }
  for (; i < count; i += stride) dst[i] = __fmaf_rn(alpha, src[i], dst[i]);
}

__global__ void relu_inplace_kernel(float* __restrict__ t, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    if (t[i] < 0.0f) t[i] = 0.0f;
  }
}

int grid_for(int64_t count, int threads) {
  const int64_t want = (count + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 32LL * sm_count())));
}

int gemm_common(const float* x, const float* w, const float* bias, float* out, int64_t m,
                int64_t k, int64_t n, bool relu, int precision, cudaStream_t stream) {
  GNN_REQUIRE(m >= 0 && k >= 0 && n >= 0, GNN_ERR_INVALID_ARGUMENT, "GEMM sizes must be >= 0");
  GNN_REQUIRE(precision == GNN_PRECISION_TF32 || precision == GNN_PRECISION_FP32,
              GNN_ERR_INVALID_ARGUMENT, "precision must be GNN_PRECISION_TF32 or GNN_PRECISION_FP32");
  if (m == 0 || n == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(out != nullptr, GNN_ERR_NULL_POINTER, "out must not be NULL");
  if (k > 0) GNN_REQUIRE(x != nullptr && w != nullptr, GNN_ERR_NULL_POINTER, "x and weight must not be NULL");
  if (precision == GNN_PRECISION_TF32 && k > 0) {
    bool handled = false;
    int rc = gemm_tc_tf32(x, w, bias, out, m, k, n, relu, stream, &handled);
    if (rc != GNN_OK) return rc;
    if (handled) {
      clear_error();
      return GNN_OK;
    }
  }
  const int64_t gm = (m + BM - 1) / BM, gn = (n + BN - 1) / BN;
  GNN_REQUIRE(gm <= 0x7fffffffLL && gn <= 65535, GNN_ERR_UNSUPPORTED, "GEMM too large");
  sgemm_kernel<<<dim3(static_cast<unsigned>(gm), static_cast<unsigned>(gn)), 256, 0, stream>>>(
      x, w, bias, out, m, k, n, relu ? 1 : 0);
  GNN_LAUNCH_CHECK("gemm kernel launch");
  clear_error();
  return GNN_OK;
}

}  // namespace
}  // namespace gnnb200

using namespace gnnb200;

extern "C" int gnn_gemm_forward(const float* x, const float* weight, float* out, int64_t m,
                                int64_t k, int64_t n, int precision, gnn_stream_t stream) {
  return gemm_common(x, weight, nullptr, out, m, k, n, false, precision,
                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_linear_forward(const float* x, const float* weight, const float* bias, float* out,
                                  int64_t m, int64_t k, int64_t n, int relu, int precision,
                                  gnn_stream_t stream) {
  return gemm_common(x, weight, bias, out, m, k, n, relu != 0, precision,
                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_bias_relu_forward(float* out, const float* bias, int64_t rows, int64_t cols,
                                     int relu, gnn_stream_t stream) {
  GNN_REQUIRE(rows >= 0 && cols >= 0, GNN_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  const int64_t count = rows * cols;
  if (count == 0 || (bias == nullptr && !relu)) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(out != nullptr, GNN_ERR_NULL_POINTER, "out must not be NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = (cols % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(bias)) & 15) == 0;
  if (vec) {
    bias_relu_vec_kernel<<<grid_for(count / 4, 256), 256, 0, s>>>(
        reinterpret_cast<float4*>(out), reinterpret_cast<const float4*>(bias), count / 4, cols / 4,
        relu ? 1 : 0);
  } else {
    bias_relu_kernel<<<grid_for(count, 256), 256, 0, s>>>(out, bias, rows, cols, relu ? 1 : 0);
  }
  GNN_LAUNCH_CHECK("bias_relu launch");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_tensor_add_inplace(float* dst, const float* src, float alpha, int64_t count,
                                      gnn_stream_t stream) {
  GNN_REQUIRE(count >= 0, GNN_ERR_INVALID_ARGUMENT, "count must be >= 0");
  if (count == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(dst != nullptr && src != nullptr, GNN_ERR_NULL_POINTER, "dst and src must not be NULL");
  add_inplace_kernel<<<grid_for(count / 4 + 1, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      dst, src, alpha, count);
  GNN_LAUNCH_CHECK("tensor_add_inplace launch");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_relu_inplace(float* t, int64_t count, gnn_stream_t stream) {
  GNN_REQUIRE(count >= 0, GNN_ERR_INVALID_ARGUMENT, "count must be >= 0");
  if (count == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(t != nullptr, GNN_ERR_NULL_POINTER, "tensor must not be NULL");
  relu_inplace_kernel<<<grid_for(count, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(t, count);
  GNN_LAUNCH_CHECK("relu_inplace launch");
  clear_error();
  return GNN_OK;
}
