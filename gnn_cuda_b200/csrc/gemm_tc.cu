// tcgen05 (5th-generation tensor core) TF32 GEMM for the dense transform X·W.
// Placeholder hook: until the tensor-core kernel is in place every request is
// reported as not handled, and gemm_common runs the FFMA kernel.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace gnnb200 {

int gemm_tc_tf32(const float* x, const float* w, const float* bias, float* out, int64_t m,
                 int64_t k, int64_t n, bool relu, cudaStream_t stream, bool* handled) {
  (void)x; (void)w; (void)bias; (void)out; (void)m; (void)k; (void)n; (void)relu; (void)stream;
  *handled = false;
  return GNN_OK;
}

}  // namespace gnnb200

extern "C" int gnn_gemm_uses_tensor_cores(int64_t m, int64_t k, int64_t n) {
  (void)m; (void)k; (void)n;
  return 0;
}
