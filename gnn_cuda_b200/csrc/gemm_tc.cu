// tcgen05 (5th-generation tensor core) TF32 GEMM for the dense transform
//   out[M, N] = relu?(X[M, K] · W[K, N] + bias)
// replacing the reference's cublasSgemm call (GNN_cuda_common/native/agg_ops.cu:369-391)
// plus its separate bias/ReLU pass (agg_ops.cu:132-147).
//
// Shape of the problem: M = number of nodes (millions), K = N = 128..256. At these
// widths the GEMM is bound by HBM (read X once, write out once; 32-64 flop/B),
// so the design keeps every byte moving once:
//   * persistent CTAs, one per SM; each CTA owns one 128-column slice of W for
//     the whole launch (staged once into shared memory, transposed to the
//     K-major 128-byte-swizzled layout the MMA reads) and walks 128-row tiles of X;
//   * warp 0 streams X tiles in 32-column (128-byte) swizzled chunks with TMA
//     into a ring of up to 8 stages; warp 1 issues tcgen05.mma (kind::tf32, M=128, N=BN,
//     K=8 per instruction) into one of two TMEM accumulators; warps 2-5 drain
//     the other accumulator (tcgen05.ld), add bias, apply ReLU, write 32x32
//     blocks into swizzled shared buffers (two per warp) and hand each block to
//     a TMA bulk store, so the output leaves as whole 128-byte lines — loads,
//     MMAs, the epilogue and the stores of consecutive tiles overlap;
//   * every mbarrier wait is bounded by a clock deadline; on expiry the kernel
//     records an error code in a device status word, stops issuing work, waits
//     (bounded) for its in-flight copies and MMAs, frees its TMEM and returns.
// Accuracy: inputs are consumed as TF32 (10-bit mantissa), products accumulate
// in fp32 — within a relative error of 2e-3 of the float64 product (scaled by sum_k |x_ik * w_kj|).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "tc_core.cuh"

namespace gnnb200 {
namespace {

using namespace tc;

constexpr int BM = 128;             // rows per tile (TMEM lanes)
constexpr int KCHUNK = 32;          // tf32 elements per 128-byte swizzle row
constexpr int MAX_STAGES = 8;       // X chunk ring depth: runtime, up to this many 16 KiB stages
constexpr size_t kSmemLimit = 227 * 1024;
constexpr int A_STAGE_BYTES = BM * KCHUNK * 4;  // 16 KiB
constexpr int kThreads = 192;       // warp0 TMA, warp1 MMA/TMEM, warps 2-5 epilogue
constexpr int OUT_BLOCK_BYTES = 32 * 32 * 4;              // one 32-row x 32-column fp32 output block
constexpr int OUT_STAGING_BYTES = 4 * 2 * OUT_BLOCK_BYTES;  // 4 epilogue warps x 2 buffers = 32 KiB

// device status word: 0 ok, otherwise the role that gave up waiting
__device__ int g_tc_status = 0;

constexpr int kMaxPeers = 8;  // destinations of the fused halo push

struct TcParams {
  int64_t m, k, n;
  int64_t m_tiles;
  int n_tiles;
  const float* bias;
  float* out;
  int relu;
  int stages;  // X chunk ring depth (2..MAX_STAGES)
  // fused halo push (PUSH instantiation only): output row i also goes to row i of
  // peer_out[q] for every bit q set in peer_mask[i]
  const uint8_t* peer_mask;
  float* peer_out[kMaxPeers];
  int npeers;
};

__device__ __forceinline__ void record_timeout(int code) { atomicCAS(&g_tc_status, 0, code); }

template <int BN, bool PUSH>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_out,
                        const float* __restrict__ w, TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int K = static_cast<int>(p.k);
  const int kchunks = K / KCHUNK;
  const uint32_t w_bytes = static_cast<uint32_t>(BN) * K * 4;
  uint8_t* sW = smem;                                  // K/32 blocks of [BN rows x 128 B], K-major
  const int S = p.stages;
  uint8_t* sA = smem + ((w_bytes + 1023) & ~1023u);    // S x 16 KiB
  uint8_t* sOut = sA + S * A_STAGE_BYTES;             // 4 warps x 2 x [32 rows x 128 B], swizzled
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + OUT_STAGING_BYTES);
  uint64_t* full = bars;                 // [S]
  uint64_t* empty = bars + S;            // [S]
  uint64_t* acc_full = bars + 2 * S;     // [2]
  uint64_t* acc_empty = bars + 2 * S + 2; // [2]
  uint64_t* drain = bars + 2 * S + 5;    // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 6);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x % p.n_tiles;
  const int64_t m_first = blockIdx.x / p.n_tiles;
  const int64_t m_step = gridDim.x / p.n_tiles;
  constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators; BN in {32, 64, 128}

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Stage this CTA's W slice (columns [n_tile*BN, +BN), all K rows) transposed
  // into the K-major swizzled layout the MMA reads: row n of the operand is
  // column n of W. Global reads are coalesced along n; the slice stays resident.
  {
    const float* wsrc = w + static_cast<int64_t>(n_tile) * BN;
    for (int idx = threadIdx.x; idx < K * BN; idx += kThreads) {
      const int k = idx / BN;
      const int nn = idx - k * BN;
      const float v = __ldg(wsrc + static_cast<int64_t>(k) * p.n + nn);
      *reinterpret_cast<float*>(sW + kmajor_sw128_offset(nn, k, BN)) = v;
    }
    // generic-proxy smem writes -> visible to the tensor core (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_x) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int64_t mt = m_first; mt < p.m_tiles && ok; mt += m_step) {
        for (int kc = 0; kc < kchunks; ++kc) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            record_timeout(1);
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], A_STAGE_BYTES);
          tma_load_2d(sA + stage * A_STAGE_BYTES, &tmap_x, &full[stage], kc * KCHUNK, static_cast<int>(mt * BM));
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // drain: the last min(issued, S) copies must have landed before exit
      const int64_t pending = std::min<int64_t>(issued, S);
      for (int64_t i = 0; i < pending; ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1;
        }
        if (!mbar_wait(&full[stage], phase)) record_timeout(5);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      const uint32_t sw_base = smem_u32(sW);
      const uint32_t sa_base = smem_u32(sA);
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int64_t mt = m_first; mt < p.m_tiles && ok; mt += m_step) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) {
          record_timeout(2);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kc = 0; kc < kchunks; ++kc) {
          if (!mbar_wait(&full[stage], phase)) {
            record_timeout(2);
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < KCHUNK / 8; ++kk) {
            // both operands K-major: 8 K values = 32 bytes along the 128-byte swizzled row
            const uint64_t a_desc = sw128_desc(sa_base + stage * A_STAGE_BYTES + kk * 32, 16, 1024);
            const uint64_t b_desc = sw128_desc(sw_base + kc * BN * 128 + kk * 32, 16, 1024);
            mma_tf32(d_tmem, a_desc, b_desc, idesc, (kc | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // all MMAs issued by this thread complete before TMEM is released
      mma_commit(drain);
      if (!mbar_wait(drain, 0)) record_timeout(6);
    }
  } else {
    // ---------------- epilogue: warps 2..5 ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // this warp's two staging buffers; lane L fills row L of a 32x32 block, its
    // 16-byte chunk c at chunk c ^ (L % 8) (the TMA 128-byte swizzle), so the
    // eight lanes of each shared-store phase hit eight different bank groups
    uint8_t* staging = sOut + (warp - 2) * (2 * OUT_BLOCK_BYTES);
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t blocks = 0;  // stores this warp has committed
    const int ncol0 = n_tile * BN;
    for (int64_t mt = m_first; mt < p.m_tiles; mt += m_step) {
      // warp-uniform decision: the tcgen05.ld below is .sync.aligned
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase))) {
        if (lane == 0) record_timeout(3);
        break;
      }
      tc_fence_after();
      const int64_t row0 = mt * BM + 32 * q;  // first row of this warp's lane quarter
      const bool has_rows = row0 < p.m;        // rows past m are clipped by the store
      // PUSH: the peers that read this lane's row (none for rows past m)
      uint32_t my_mask = 0;
      if (PUSH && row0 + lane < p.m) my_mask = __ldg(p.peer_mask + row0 + lane);
      const bool any_push = PUSH && __any_sync(0xffffffffu, my_mask != 0);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + static_cast<uint32_t>(acc * BN + c0) + (static_cast<uint32_t>(32 * q) << 16), r);
        if (has_rows) {
          uint8_t* buf = staging + (blocks & 1) * OUT_BLOCK_BYTES;
          // the store committed two blocks ago read this buffer: it must be done reading
          if (lane == 0) bulk_wait_read_1();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                   __uint_as_float(r[j + 3]));
            if (p.bias != nullptr) v = add4(v, __ldg(reinterpret_cast<const float4*>(p.bias + ncol0 + c0 + j)));
            if (p.relu) {
              v.x = v.x < 0.0f ? 0.0f : v.x;
              v.y = v.y < 0.0f ? 0.0f : v.y;
              v.z = v.z < 0.0f ? 0.0f : v.z;
              v.w = v.w < 0.0f ? 0.0f : v.w;
            }
            *reinterpret_cast<float4*>(buf + lane * 128 + ((((j >> 2) ^ (lane & 7))) << 4)) = v;
          }
          // generic-proxy shared writes -> visible to the TMA unit (async proxy)
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, buf, ncol0 + c0, static_cast<int>(row0));
            bulk_commit();
          }
          if (any_push) {
            // the block's rows that peers read, back out of the staging buffer in row
            // order: 8 lanes per row (its 128 bytes of this column block), 4 rows a pass,
            // each stored to every peer whose bit is set (plain stores over NVLink)
            const int c = lane & 7;
#pragma unroll 1
            for (int pass = 0; pass < 8; ++pass) {
              const int j = pass * 4 + (lane >> 3);
              const uint32_t mj = __shfl_sync(0xffffffffu, my_mask, j);
              if (mj != 0) {
                const float4 v = *reinterpret_cast<const float4*>(buf + j * 128 + ((c ^ (j & 7)) << 4));
                const int64_t off = (row0 + j) * p.n + ncol0 + c0 + c * 4;
#pragma unroll
                for (int d = 0; d < kMaxPeers; ++d) {
                  if (d < p.npeers && ((mj >> d) & 1u)) *reinterpret_cast<float4*>(p.peer_out[d] + off) = v;
                }
              }
            }
          }
          ++blocks;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // shared staging must outlive the stores reading it; the writes land before exit
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}

bool device_is_sm100() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

int pick_bn(int64_t n) {
  if (n % 128 == 0) return 128;
  if (n == 64) return 64;
  if (n == 32) return 32;
  return 0;
}

bool shape_ok(int64_t m, int64_t k, int64_t n) {
  return m >= 1 && m <= (int64_t(1) << 31) - BM && k >= KCHUNK && k <= 256 && k % KCHUNK == 0 && pick_bn(n) != 0 &&
         n <= 65536;
}

size_t smem_bytes_for(int bn, int64_t k, int stages) {
  const size_t w = ((static_cast<size_t>(bn) * k * 4) + 1023) & ~size_t(1023);
  return 1024 /* alignment slack */ + w + static_cast<size_t>(stages) * A_STAGE_BYTES + OUT_STAGING_BYTES +
         256 /* barriers + TMEM slot */;
}

// Ring depth: gemm.stages when set (and it fits), else as many stages as the
// shared memory left beside the resident W slice holds, up to MAX_STAGES. More
// stages keep more X bytes in flight per SM, which is what bounds this
// HBM-bound transform. 0 when not even two stages fit.
int stages_for(int bn, int64_t k) {
  const int want = static_cast<int>(config().gemm_stages.load());
  int s = want > 0 ? want : MAX_STAGES;
  while (s >= 2 && smem_bytes_for(bn, k, s) > kSmemLimit) --s;
  return s >= 2 ? s : 0;
}

size_t smem_bytes(int bn, int64_t k) {
  const int s = stages_for(bn, k);
  return s ? smem_bytes_for(bn, k, s) : kSmemLimit + 1;
}

template <int BN, bool PUSH>
int launch_bn(const float* x, const float* w, const float* bias, float* out, int64_t m, int64_t k, int64_t n,
              bool relu, const uint8_t* peer_mask, float* const* peer_out, int npeers, cudaStream_t stream) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(GNN_ERR_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
  CUtensorMap tx{};
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(m)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 4};
    cuuint32_t box[2] = {KCHUNK, BM};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GNN_ERR_CUDA, "cuTensorMapEncodeTiled(x) failed: " + std::to_string(r));
  }
  // output [m, n] row-major, written in 32-row x 32-column blocks (x = column, a multiple of 32)
  CUtensorMap to{};
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(n) * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GNN_ERR_CUDA, "cuTensorMapEncodeTiled(out) failed: " + std::to_string(r));
  }
  const size_t smem = smem_bytes(BN, k);
  // the opt-in is a per-device function attribute; remember the largest size set per device
  static int configured_smem[64][6] = {};
  static std::mutex mu;
  int dev = 0;
  GNN_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  const int slot = (BN == 128 ? 0 : (BN == 64 ? 1 : 2)) + (PUSH ? 3 : 0);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || configured_smem[dev][slot] < static_cast<int>(smem)) {
      GNN_CUDA_TRY(cudaFuncSetAttribute(gemm_tf32_tc_kernel<BN, PUSH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)),
                   "gemm_tf32_tc_kernel: shared memory opt-in");
      if (dev >= 0 && dev < 64) configured_smem[dev][slot] = static_cast<int>(smem);
    }
  }
  TcParams p{};
  p.m = m;
  p.k = k;
  p.n = n;
  p.m_tiles = (m + BM - 1) / BM;
  p.n_tiles = static_cast<int>(n / BN);
  p.bias = bias;
  p.out = out;
  p.relu = relu ? 1 : 0;
  p.stages = stages_for(BN, k);
  if (p.stages < 2) return fail(GNN_ERR_UNSUPPORTED, "gemm_tf32_tc_kernel: shared memory too small for K");
  p.peer_mask = peer_mask;
  p.npeers = PUSH ? npeers : 0;
  for (int d = 0; d < kMaxPeers; ++d) p.peer_out[d] = (PUSH && d < npeers) ? peer_out[d] : nullptr;
  const int64_t tiles = p.m_tiles * p.n_tiles;
  int64_t ctas = std::min<int64_t>(tiles, sm_count());
  ctas = std::max<int64_t>(p.n_tiles, (ctas / p.n_tiles) * p.n_tiles);
  gemm_tf32_tc_kernel<BN, PUSH><<<static_cast<unsigned>(ctas), kThreads, smem, stream>>>(tx, to, w, p);
  GNN_LAUNCH_CHECK("gemm_tf32_tc_kernel launch");
  return GNN_OK;
}

}  // namespace

bool gemm_tc_eligible(const float* x, const float* w, const float* bias, const float* out, int64_t m, int64_t k,
                      int64_t n) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
                      reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(bias);
  return shape_ok(m, k, n) && (a % 16 == 0) && device_is_sm100() && encode_fn() != nullptr &&
         smem_bytes(pick_bn(n), k) <= kSmemLimit;
}

int gemm_tc_tf32(const float* x, const float* w, const float* bias, float* out, int64_t m, int64_t k, int64_t n,
                 bool relu, cudaStream_t stream, bool* handled) {
  *handled = false;
  if (!gemm_tc_eligible(x, w, bias, out, m, k, n)) return GNN_OK;
  int rc;
  switch (pick_bn(n)) {
    case 128: rc = launch_bn<128, false>(x, w, bias, out, m, k, n, relu, nullptr, nullptr, 0, stream); break;
    case 64: rc = launch_bn<64, false>(x, w, bias, out, m, k, n, relu, nullptr, nullptr, 0, stream); break;
    default: rc = launch_bn<32, false>(x, w, bias, out, m, k, n, relu, nullptr, nullptr, 0, stream); break;
  }
  if (rc == GNN_OK) *handled = true;
  return rc;
}

int gemm_tc_tf32_push(const float* x, const float* w, const float* bias, float* out, int64_t m, int64_t k, int64_t n,
                      bool relu, const uint8_t* peer_mask, float* const* peer_out, int npeers, cudaStream_t stream) {
  switch (pick_bn(n)) {
    case 128: return launch_bn<128, true>(x, w, bias, out, m, k, n, relu, peer_mask, peer_out, npeers, stream);
    case 64: return launch_bn<64, true>(x, w, bias, out, m, k, n, relu, peer_mask, peer_out, npeers, stream);
    default: return launch_bn<32, true>(x, w, bias, out, m, k, n, relu, peer_mask, peer_out, npeers, stream);
  }
}

int tc_status_read(int reset, int* status) {
  GNN_CUDA_TRY(cudaMemcpyFromSymbol(status, g_tc_status, sizeof(int)), "read tensor-core status word");
  if (reset) {
    const int zero = 0;
    GNN_CUDA_TRY(cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int)), "reset tensor-core status word");
  }
  return GNN_OK;
}

}  // namespace gnnb200

namespace gnnb200 {
int spmm_status_read(int reset, int* status);  // spmm.cu
}

extern "C" int gnn_device_status(int reset, int* status) {
  GNN_REQUIRE(status != nullptr, GNN_ERR_NULL_POINTER, "status must not be NULL");
  int tc = 0, sp = 0;
  int rc = gnnb200::tc_status_read(reset, &tc);
  if (rc == GNN_OK) rc = gnnb200::spmm_status_read(reset, &sp);
  if (rc != GNN_OK) return rc;
  *status = tc != 0 ? tc : sp;
  gnnb200::clear_error();
  return GNN_OK;
}

extern "C" int gnn_linear_push_forward(const float* x, const float* weight, const float* bias, float* out,
                                       int64_t m, int64_t k, int64_t n, int relu, const uint8_t* peer_mask,
                                       float* const* peer_out, int npeers, gnn_stream_t stream) {
  GNN_REQUIRE(m >= 0 && k >= 0 && n >= 0, GNN_ERR_INVALID_ARGUMENT, "m, k and n must be >= 0");
  GNN_REQUIRE(npeers >= 0 && npeers <= gnnb200::kMaxPeers, GNN_ERR_INVALID_ARGUMENT,
              "npeers must be in [0, 8]");
  if (m == 0) {
    gnnb200::clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(x != nullptr && weight != nullptr && out != nullptr, GNN_ERR_NULL_POINTER,
              "x, weight and out must not be NULL");
  GNN_REQUIRE(npeers == 0 || (peer_mask != nullptr && peer_out != nullptr), GNN_ERR_NULL_POINTER,
              "peer_mask and peer_out must not be NULL when npeers > 0");
  uintptr_t a = 0;
  for (int d = 0; d < npeers; ++d) {
    GNN_REQUIRE(peer_out[d] != nullptr, GNN_ERR_NULL_POINTER, "peer_out entries must not be NULL");
    a |= reinterpret_cast<uintptr_t>(peer_out[d]);
  }
  GNN_REQUIRE(a % 16 == 0 && (n * 4) % 16 == 0, GNN_ERR_INVALID_ARGUMENT,
              "peer rows must be 16-byte aligned");
  if (!gnnb200::gemm_tc_eligible(x, weight, bias, out, m, k, n)) {
    return gnnb200::fail(GNN_ERR_UNSUPPORTED,
                         "linear push: needs the TF32 tensor-core GEMM (sm_100, K a multiple of 32 up to 256, "
                         "N in {32, 64} or a multiple of 128, 16-byte aligned operands)");
  }
  int rc;
  if (npeers == 0) {  // nothing to push: the plain instantiation (the mask is never read)
    bool handled = false;
    rc = gnnb200::gemm_tc_tf32(x, weight, bias, out, m, k, n, relu != 0, reinterpret_cast<cudaStream_t>(stream),
                               &handled);
    if (rc == GNN_OK && !handled) rc = gnnb200::fail(GNN_ERR_UNSUPPORTED, "linear push: tensor-core GEMM not taken");
  } else {
    rc = gnnb200::gemm_tc_tf32_push(x, weight, bias, out, m, k, n, relu != 0, peer_mask, peer_out, npeers,
                                    reinterpret_cast<cudaStream_t>(stream));
  }
  if (rc == GNN_OK) gnnb200::clear_error();
  return rc;
}

extern "C" int gnn_gemm_uses_tensor_cores(int64_t m, int64_t k, int64_t n) {
  return (gnnb200::shape_ok(m, k, n) && gnnb200::device_is_sm100() && gnnb200::encode_fn() != nullptr) ? 1 : 0;
}
