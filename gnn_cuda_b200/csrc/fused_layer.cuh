// Fused aggregation and dense transform: one GNN layer without an [N, F]
// aggregate in HBM.
//
//   GCN   out = relu?( Â·X·W + b )                       (gcn_inference.py:534-600)
//   GIN   out = relu?( relu(((1+eps)·x + Σx)·W1 + b1)·W2 + b2 )  (gin_inference.py:317-359)
//   mean  out = relu?( mean(X)·W + b )                   (the neighbour half of graphsage_inference.py:310-354)
//
// The reference runs each layer as separate kernels with an [N, F] buffer
// between them (agg_buffer / out_buffer, gcn_inference.py:127-128): the
// aggregate is written to HBM, read back by cublasSgemm, and the result is
// read and written again by the bias/ReLU pass. Here a persistent CTA per SM
// builds a 128-row tile of the aggregate directly in shared memory, in the
// K-major 128-byte-swizzled layout tcgen05.mma reads, multiplies it by the
// resident weight slice into TMEM, and writes only the layer output:
//
//   warps 0..15   gather: each takes 8 rows of the tile and sums their
//                 neighbour rows exactly as spmm_vec_kernel does (one warp per
//                 row, CSR order, 128-bit gathers), then stores the row into
//                 the tile (and, for GIN, adds (1+eps)·x[row] first); warp 0
//                 also owns TMEM and, from lane 0, issues the tile's MMAs
//                 (every gather warp waits for them before its next tile anyway);
//   warps 16..19  epilogue: TMEM -> registers, + bias, ReLU, out rows (GIN:
//                 the hidden layer goes back into the tile as the second MMA's
//                 A operand, then the second epilogue writes out).
//
// Tiles are 128 consecutive positions of the global descending-degree row
// order, so the rows of a tile have about the same degree and the sixteen
// gather warps finish together. Rows above the long-row threshold (power-law
// hubs) are summed beforehand by spmm_long_kernel into their own row of `out`
// (which therefore needs at least K columns) and a second launch of this
// kernel, on the side stream, transforms those rows in place.
//
// Results are bit-identical to the unfused sequence (aggregation, then
// gnn_linear_forward on the tcgen05 path): every row is summed in the same
// order, and the tile is multiplied by the same MMA instructions, in the same
// order, on the same operand bits as the standalone GEMM.
//
// Included at the end of spmm.cu: it shares that file's aggregation helpers,
// long-row kernel, row-order schedule and device status word.

#include "tc_core.cuh"

namespace gnnb200 {
namespace {

#ifndef GNN_FUSED_U
// neighbour rows in flight per gather warp. Measured on B200 (GCN layer of the
// 2.45M-node products-shaped graph): 4 rows 7.4 ms, 8 rows 7.7 ms; rows of up
// to 32 entries interleaved four at a time (8 or 16 in flight) 9.0-9.7 ms.
#define GNN_FUSED_U 4
#endif
constexpr int kFzGather = 16;                    // gather warps
constexpr int kFzMmaWarp = 0;                    // the gather warp that also issues the MMAs and owns TMEM
constexpr int kFzEpi0 = kFzGather;               // first of the four epilogue warps
constexpr int kFzThreads = (kFzGather + 4) * 32;  // 640: 20 warps, 96 registers per thread
constexpr int kFzBM = 128;                       // tile rows = TMEM lanes = MMA M
constexpr int kFzRowsPerWarp = kFzBM / kFzGather;
constexpr int kFzStaging = 4 * 32 * 128;         // per epilogue warp: 32 rows x 128 B
constexpr int kFzTmemCols = 256;                 // two 128-column accumulators
constexpr int kFzTimeout = 18;                   // status code: a fused-kernel wait gave up
static_assert(kFzBM % kFzGather == 0 && kFzRowsPerWarp <= 32, "tile rows must split evenly over gather warps");

struct FusedArgs {
  SpmmArgs a;                 // aggregation inputs; a.f = K (<= 128), long rows already summed into out
  const uint32_t* order;      // row order: position -> row id
  const uint32_t* pos_begin;  // device word: first position of this launch (nullptr: 0)
  const uint32_t* pos_end;    // device word: end position (nullptr: num_end)
  int64_t num_end;
  int copy;                   // 1: the tile rows are out[row][0:K] (pre-summed), else aggregated here
  int has_self;               // GIN: row = fma(self_scale, x[row], row) after the sum
  float self_scale;
  int n1, n2;                 // widths of the first / second transform (n2 = 0: one transform)
  const float* b1;
  const float* b2;
  int relu1, relu2;
  float* out;
  int64_t ldo;                // out row stride (= n2 ? n2 : n1)
  int64_t x_row0;             // x row of local row 0 (a row shard's first global row)
};

__device__ __forceinline__ void fz_fail() { atomicCAS(&g_spmm_status, 0, kFzTimeout); }

__device__ __forceinline__ float4 relu4(float4 v) {
  v.x = v.x < 0.0f ? 0.0f : v.x;
  v.y = v.y < 0.0f ? 0.0f : v.y;
  v.z = v.z < 0.0f ? 0.0f : v.z;
  v.w = v.w < 0.0f ? 0.0f : v.w;
  return v;
}

// The warp's eight rows of the tile, one at a time, exactly as spmm_vec_kernel
// sums them (32-edge chunks, GNN_FUSED_U neighbour rows in flight, the next
// row's first chunk of columns loaded while the current row is gathered).
template <int WM, int MEAN, class IdxT>
__device__ __forceinline__ void gather_rows_one_by_one(const FusedArgs& p, int lane, int warp, int my_row,
                                                       IdxT my_beg, IdxT my_end, float my_rs, bool valid_lane,
                                                       uint8_t* sA) {
  const SpmmArgs& a = p.a;
  const int K = static_cast<int>(a.f);
  const int64_t col0 = lane;
  const bool valid[1] = {valid_lane};
  auto first_chunk = [&](int i, int& c, float& w) {
    const IdxT beg = __shfl_sync(kFull, my_beg, i);
    const IdxT end = __shfl_sync(kFull, my_end, i);
    const float rs = __shfl_sync(kFull, my_rs, i);
    const int64_t deg = static_cast<int64_t>(end - beg);
    c = 0;
    w = 0.0f;
    if (lane < deg) {
      c = ld_stream_i32(a.col + beg + lane);
      w = edge_weight<WM>(a, rs, c, static_cast<int64_t>(beg) + lane);
    }
  };
  int c_next = 0;
  float w_next = 0.0f;
  first_chunk(0, c_next, w_next);
#pragma unroll 1
  for (int i = 0; i < kFzRowsPerWarp; ++i) {
    const int r = __shfl_sync(kFull, my_row, i);
    const IdxT beg = __shfl_sync(kFull, my_beg, i);
    const IdxT end = __shfl_sync(kFull, my_end, i);
    const float rs = __shfl_sync(kFull, my_rs, i);
    const int c_cur = c_next;
    const float w_cur = w_next;
    if (i + 1 < kFzRowsPerWarp) first_chunk(i + 1, c_next, w_next);
    float4 acc[1] = {make_float4(0.f, 0.f, 0.f, 0.f)};
    if (r >= 0) {
      accumulate_edges<WM, false, 1, GNN_FUSED_U, IdxT>(a, beg, end, rs, lane, col0, valid, acc, true, c_cur, w_cur);
      acc[0] = finish<MEAN>(acc[0], static_cast<int64_t>(end - beg));
      if (p.has_self && valid_lane) {
        const float4 xv =
            ldg_f4(reinterpret_cast<const float4*>(a.x + (p.x_row0 + static_cast<int64_t>(r)) * K) + col0);
        acc[0] = fma4(p.self_scale, xv, acc[0]);
      }
    }
    if (valid_lane) *reinterpret_cast<float4*>(sA + tc::kmajor_sw128_offset(warp + i * kFzGather, 4 * lane, kFzBM)) = acc[0];
  }
}

// Issues the MMAs of one tile (one thread): the tile times W1 into an
// accumulator, and with two transforms, once the epilogue has written the
// hidden tile back over sA, the hidden tile times W2. Returns false after a
// wait ran out. The instruction sequence is the standalone GEMM's.
template <bool TWO>
__device__ __forceinline__ bool fz_issue_mma(uint32_t tmem_base, uint32_t sa, uint32_t sw1, uint32_t sw2, int K,
                                             int n1, int n2, uint64_t* a_free, uint64_t* acc_full,
                                             uint64_t* acc_empty, uint64_t* h_full, int buf,
                                             uint32_t (&empty_phase)[2], uint32_t& h_phase) {
  using namespace tc;
  if constexpr (!TWO) {
    // the epilogue has drained this accumulator (two accumulators alternate)
    if (!mbar_wait(&acc_empty[buf], empty_phase[buf] ^ 1)) return false;
    empty_phase[buf] ^= 1;
  }
  // (with two transforms accumulator 0 is free: the epilogue read it before the
  // hidden tile was complete, and this tile was gathered after that)
  tc_fence_after();
  const uint32_t idesc1 = idesc_tf32(kFzBM, n1);
  const uint32_t d1 = tmem_base + static_cast<uint32_t>(buf * 128);
  for (int kc = 0; kc < K / 32; ++kc) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t ad = sw128_desc(sa + kc * (kFzBM * 128) + kk * 32, 16, 1024);
      const uint64_t bd = sw128_desc(sw1 + kc * (n1 * 128) + kk * 32, 16, 1024);
      mma_tf32(d1, ad, bd, idesc1, (kc | kk) != 0 ? 1u : 0u);
    }
  }
  if constexpr (!TWO) {
    mma_commit(a_free);
    mma_commit(&acc_full[buf]);
    return true;
  } else {
    mma_commit(&acc_full[0]);
    if (!mbar_wait(h_full, h_phase)) return false;
    h_phase ^= 1;
    if (!mbar_wait(&acc_empty[1], empty_phase[1] ^ 1)) return false;
    empty_phase[1] ^= 1;
    tc_fence_after();
    const uint32_t idesc2 = idesc_tf32(kFzBM, n2);
    const uint32_t d2 = tmem_base + 128u;
    for (int kc = 0; kc < n1 / 32; ++kc) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = sw128_desc(sa + kc * (kFzBM * 128) + kk * 32, 16, 1024);
        const uint64_t bd = sw128_desc(sw2 + kc * (n2 * 128) + kk * 32, 16, 1024);
        mma_tf32(d2, ad, bd, idesc2, (kc | kk) != 0 ? 1u : 0u);
      }
    }
    mma_commit(a_free);
    mma_commit(&acc_full[1]);
    return true;
  }
}

template <int WM, int MEAN, class IdxT, bool TWO>
__global__ void __launch_bounds__(kFzThreads, 1)
    fused_layer_kernel(const __grid_constant__ FusedArgs p, const float* __restrict__ w1,
                       const float* __restrict__ w2) {
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SpmmArgs& a = p.a;
  const int K = static_cast<int>(a.f);
  const int n1 = p.n1, n2 = p.n2;
  // the tile: K/32 blocks of [128 rows x 128 B]; with two transforms it also
  // holds the hidden tile (n1/32 blocks), so it is max(K, n1) columns wide
  const int a_cols = TWO ? (K > n1 ? K : n1) : K;
  uint8_t* sA = smem;
  uint8_t* sW1 = sA + kFzBM * a_cols * 4;                  // K/32 blocks of [n1 rows x 128 B]
  uint8_t* sW2 = sW1 + n1 * K * 4;                         // n1/32 blocks of [n2 rows x 128 B]
  uint8_t* sStage = sW2 + (TWO ? n2 * n1 * 4 : 0);         // 4 epilogue warps x 4 KiB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + kFzStaging);
  uint64_t* a_full = bars + 0;     // gather warps -> MMA (count kFzGather)
  uint64_t* a_free = bars + 1;     // MMA done reading the tile (commit)
  uint64_t* acc_full = bars + 2;   // [2] commit -> epilogue
  uint64_t* acc_empty = bars + 4;  // [2] epilogue -> MMA (count 4)
  uint64_t* h_full = bars + 6;     // TWO: hidden tile written (count 4)
  uint64_t* drain = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(a_full, kFzGather);
    mbar_init(a_free, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(h_full, 4);
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == kFzMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kFzTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Weights, transposed into the K-major swizzled layout the MMA reads (row n of
  // the operand = column n of W), exactly as the standalone GEMM stages them.
  for (int idx = threadIdx.x; idx < K * n1; idx += kFzThreads) {
    const int k = idx / n1;
    const int nn = idx - k * n1;
    *reinterpret_cast<float*>(sW1 + kmajor_sw128_offset(nn, k, n1)) = __ldg(w1 + idx);
  }
  if constexpr (TWO) {
    for (int idx = threadIdx.x; idx < n1 * n2; idx += kFzThreads) {
      const int k = idx / n2;
      const int nn = idx - k * n2;
      *reinterpret_cast<float*>(sW2 + kmajor_sw128_offset(nn, k, n2)) = __ldg(w2 + idx);
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int64_t pb = p.pos_begin ? static_cast<int64_t>(*p.pos_begin) : 0;
  const int64_t pe = p.pos_end ? static_cast<int64_t>(*p.pos_end) : p.num_end;
  const int64_t ntiles = pe > pb ? (pe - pb + kFzBM - 1) / kFzBM : 0;

  if (warp < kFzGather) {
    // ---------------- gather warps: build the aggregate tile ----------------
    const IdxT* __restrict__ rp = static_cast<const IdxT*>(a.row_ptr);
    const int64_t col0 = lane;  // this lane's float4 column (K <= 128: one per lane)
    const bool valid = col0 < (K >> 2);
    uint32_t free_phase = 0;
    // warp 0, lane 0 also issues the tile's MMAs (its own state)
    const uint32_t sa = smem_u32(sA), sw1 = smem_u32(sW1), sw2 = smem_u32(sW2);
    uint32_t full_phase = 0, h_phase = 0;
    uint32_t empty_phase[2] = {0, 0};
    int buf = 0;
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
      // the previous tile's MMAs have read sA (warp-uniform decision: shuffles follow)
      if (!__all_sync(kFull, mbar_wait(a_free, free_phase ^ 1))) {
        if (lane == 0) fz_fail();
        break;
      }
      free_phase ^= 1;
      const int64_t p0 = pb + t * kFzBM;
      // lane i < kFzRowsPerWarp: tile row warp + i * kFzGather
      int my_row = -1;
      IdxT my_beg = 0, my_end = 0;
      float my_rs = 1.0f;
      if (lane < kFzRowsPerWarp) {
        const int64_t pos = p0 + warp + lane * kFzGather;
        if (pos < pe) {
          my_row = static_cast<int>(p.order[pos]);
          if (!p.copy) {
            my_beg = rp[my_row];
            my_end = rp[my_row + 1];
            if (WM == kGcn) my_rs = __ldg(a.dis_row + my_row);
          }
        }
      }
      if (!p.copy) {
        gather_rows_one_by_one<WM, MEAN, IdxT>(p, lane, warp, my_row, my_beg, my_end, my_rs, valid, sA);
      } else {
        // the rows were summed beforehand into their own rows of out
#pragma unroll 1
        for (int i = 0; i < kFzRowsPerWarp; ++i) {
          const int tr = warp + i * kFzGather;  // tile row
          const int r = __shfl_sync(kFull, my_row, i);
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (r >= 0 && valid) {
            v = __ldcg(reinterpret_cast<const float4*>(p.out + static_cast<int64_t>(r) * p.ldo) + col0);
            if (p.has_self) {
              const float4 xv =
                  ldg_f4(reinterpret_cast<const float4*>(a.x + (p.x_row0 + static_cast<int64_t>(r)) * K) + col0);
              v = fma4(p.self_scale, xv, v);
            }
          }
          if (valid) *reinterpret_cast<float4*>(sA + kmajor_sw128_offset(tr, 4 * lane, kFzBM)) = v;
        }
      }
      // generic-proxy shared writes -> visible to the tensor core (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full);
      if (warp == kFzMmaWarp) {
        // every gather warp waits for this tile's MMAs (a_free) before the next
        // tile anyway, so issuing them from here costs no gather time
        int ok = 1;
        if (lane == 0) {
          ok = mbar_wait(a_full, full_phase) ? 1 : 0;
          full_phase ^= 1;
          if (ok) {
            ok = fz_issue_mma<TWO>(tmem_base, sa, sw1, sw2, K, n1, n2, a_free, acc_full, acc_empty, h_full, buf,
                                   empty_phase, h_phase) ? 1 : 0;
          }
          if (!ok) fz_fail();
        }
        if (!__shfl_sync(kFull, ok, 0)) break;
        if constexpr (!TWO) buf ^= 1;
      }
    }
    if (warp == kFzMmaWarp) {
      // every MMA issued here completes before TMEM is released
      if (lane == 0) {
        mma_commit(drain);
        if (!mbar_wait(drain, 0)) fz_fail();
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue warps ----------------
    const int q = warp & 3;  // TMEM lane quarter: tile rows 32q .. 32q + 31
    uint8_t* stg = sStage + (warp - kFzEpi0) * 4096;
    uint32_t full_phase[2] = {0, 0};
    int acc = 0;
    // Writes this warp's 32 rows x 32 columns (r, lane L = row 32q + L) to out
    // through the staging buffer, so that every store instruction writes four
    // whole 128-byte row segments.
    auto store_block = [&](const uint32_t (&r)[32], const float* bias, int relu, int c0, int rid) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                               __uint_as_float(r[j + 3]));
        if (bias != nullptr) v = add4(v, __ldg(reinterpret_cast<const float4*>(bias + c0 + j)));
        if (relu) v = relu4(v);
        *reinterpret_cast<float4*>(stg + lane * 128 + ((((j >> 2) ^ (lane & 7))) << 4)) = v;
      }
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int jr = it * 4 + (lane >> 3);
        const int c = lane & 7;
        const int rj = __shfl_sync(kFull, rid, jr);
        const float4 v = *reinterpret_cast<const float4*>(stg + jr * 128 + ((c ^ (jr & 7)) << 4));
        if (rj >= 0) *reinterpret_cast<float4*>(p.out + static_cast<int64_t>(rj) * p.ldo + c0 + 4 * c) = v;
      }
      __syncwarp();
    };
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const int64_t pos = pb + t * kFzBM + 32 * q + lane;
      const int rid = pos < pe ? static_cast<int>(p.order[pos]) : -1;
      const int buf = TWO ? 0 : acc;
      if (!__all_sync(kFull, mbar_wait(&acc_full[buf], full_phase[buf]))) {
        if (lane == 0) fz_fail();
        break;
      }
      full_phase[buf] ^= 1;
      tc_fence_after();
      const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
      if constexpr (!TWO) {
#pragma unroll 1
        for (int c0 = 0; c0 < n1; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(lane_base + static_cast<uint32_t>(buf * 128 + c0), r);
          store_block(r, p.b1, p.relu1, c0, rid);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        acc ^= 1;
      } else {
        // hidden = relu1(acc0 + b1) -> the A tile of the second MMA (row 32q + lane)
        const int row = 32 * q + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < n1; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(lane_base + static_cast<uint32_t>(c0), r);
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                   __uint_as_float(r[j + 3]));
            if (p.b1 != nullptr) v = add4(v, __ldg(reinterpret_cast<const float4*>(p.b1 + c0 + j)));
            if (p.relu1) v = relu4(v);
            *reinterpret_cast<float4*>(sA + kmajor_sw128_offset(row, c0 + j, kFzBM)) = v;
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(h_full);
        if (!__all_sync(kFull, mbar_wait(&acc_full[1], full_phase[1]))) {
          if (lane == 0) fz_fail();
          break;
        }
        full_phase[1] ^= 1;
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < n2; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(lane_base + static_cast<uint32_t>(128 + c0), r);
          store_block(r, p.b2, p.relu2, c0, rid);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[1]);
      }
    }
  }

  __syncthreads();
  if (warp == kFzMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kFzTmemCols)
                 : "memory");
  }
}

// Shared memory of one CTA: the tile (as wide as the wider of K and, with two
// transforms, n1), the resident weights, the epilogue staging, the barriers.
size_t fused_smem_bytes(int64_t k, int64_t n1, int64_t n2) {
  const int64_t a_cols = n2 ? std::max(k, n1) : k;
  return 1024 /* alignment slack */ + static_cast<size_t>(kFzBM) * a_cols * 4 + static_cast<size_t>(n1) * k * 4 +
         static_cast<size_t>(n2) * n1 * 4 + kFzStaging + 128 /* barriers + TMEM slot */;
}

bool fused_device_ok() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return major == 10 && minor == 0;
}

bool fused_shape_ok(int64_t k, int64_t n1, int64_t n2) {
  auto width_ok = [](int64_t v) { return v == 32 || v == 64 || v == 128; };
  if (!(k >= 32 && k <= 128 && k % 32 == 0) || !width_ok(n1)) return false;
  if (n2 != 0 && !width_ok(n2)) return false;
  const int64_t out_dim = n2 ? n2 : n1;
  return out_dim >= k && fused_smem_bytes(k, n1, n2) <= 227 * 1024;
}

struct FusedRequest {
  SpmmRequest agg;  // row_ptr, col, dis, x, n, nnz, f = K, row_begin, workspace
  int mean;         // kNoMean / kMeanDiv / kMeanRcp
  int has_self;
  float self_scale;
  const float *w1, *b1, *w2, *b2;
  int64_t n1, n2;
  int relu1, relu2;
  float* out;
};

template <int WM, int MEAN, class IdxT, bool TWO>
int launch_fused(const FusedArgs& fa, const float* w1, const float* w2, int64_t max_rows, cudaStream_t stream) {
  const size_t smem = fused_smem_bytes(fa.a.f, fa.n1, TWO ? fa.n2 : 0);
  static int configured[64] = {};
  static std::mutex mu;
  int dev = 0;
  GNN_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || configured[dev] < static_cast<int>(smem)) {
      GNN_CUDA_TRY(cudaFuncSetAttribute(fused_layer_kernel<WM, MEAN, IdxT, TWO>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
                   "fused_layer_kernel: shared memory opt-in");
      if (dev >= 0 && dev < 64) configured[dev] = static_cast<int>(smem);
    }
  }
  const int64_t tiles = (max_rows + kFzBM - 1) / kFzBM;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, sm_count())));
  fused_layer_kernel<WM, MEAN, IdxT, TWO><<<grid, kFzThreads, smem, stream>>>(fa, w1, w2);
  GNN_LAUNCH_CHECK("fused_layer_kernel launch");
  return GNN_OK;
}

template <int WM, int MEAN, class IdxT, bool TWO>
int run_fused_typed(const FusedRequest& q, cudaStream_t stream) {
  const SpmmRequest& g = q.agg;
  SpmmArgs a{};
  a.row_ptr = g.row_ptr;
  a.col = g.col;
  a.dis = g.dis;
  a.dis_row = g.dis != nullptr ? g.dis + g.row_begin : nullptr;
  a.x = g.x;
  a.n = g.n;
  a.f = g.f;
  a.out = q.out;
  a.ldo = TWO ? q.n2 : q.n1;
  a.long_thr = std::min<int64_t>(resolve_long_threshold(g.n, g.nnz), int64_t(1) << 25);
  a.long_cap = std::min<int64_t>(long_capacity(g.n, g.nnz), g.nnz / (a.long_thr + 1) + 1);
  a.long_split = static_cast<int>(config().long_row_warps.load());
  a.seg_len = static_cast<int64_t>(a.long_split) * kSegEdgesPerWarp;
  a.rows_per_warp = kRowsPerWarp;
  a.tiles = 1;
  if (g.nnz <= a.long_thr) a.long_cap = 0;
  const WsLayout lay = ws_layout(g.n, g.nnz);
  const size_t need = lay.total + sched_bytes(g.n);
  if (g.ws == nullptr || g.ws_bytes < need) {
    return fail(GNN_ERR_WORKSPACE, "fused layer: workspace missing or smaller than gnn_spmm_schedule_workspace_bytes()");
  }
  char* ws = static_cast<char*>(g.ws);
  a.counters = reinterpret_cast<uint32_t*>(ws);
  a.long_list = reinterpret_cast<uint32_t*>(ws + lay.list_off);
  a.seg_items = reinterpret_cast<uint2*>(ws + lay.seg_off);
  a.seg_cap = a.long_cap > 0 ? lay.seg_cap : 0;
  GNN_CUDA_TRY(cudaMemsetAsync(g.ws, 0, kWsHeader, stream), "fused layer: workspace reset");
  const IdxT* rp = static_cast<const IdxT*>(g.row_ptr);
  if (a.long_cap > 0) {
    const int threads = 256;
    const int64_t want = (g.n + threads - 1) / threads;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 8LL * sm_count())));
    plan_long_rows_kernel<IdxT><<<blocks, threads, 0, stream>>>(rp, g.n, a.long_thr, a.seg_len, a.counters,
                                                               a.long_list, a.long_cap, a.seg_items, a.seg_cap);
    GNN_LAUNCH_CHECK("fused layer: plan kernel launch");
  } else {
    a.long_thr = INT64_MAX;
  }
  // global descending-degree order; rows above the threshold form its last class
  uint32_t* counts = reinterpret_cast<uint32_t*>(ws + lay.total);
  uint32_t* cursor = counts + kSchedBins;
  uint32_t* order =
      reinterpret_cast<uint32_t*>(ws + lay.total + ((2 * kSchedBins * sizeof(uint32_t) + 255) & ~size_t(255)));
  {
    GNN_CUDA_TRY(cudaMemsetAsync(counts, 0, kSchedBins * sizeof(uint32_t), stream), "fused layer: schedule reset");
    const int64_t want = (g.n + 255) / 256;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 4LL * sm_count())));
    sched_hist_kernel<IdxT><<<blocks, 256, 0, stream>>>(rp, g.n, a.long_thr, counts);
    GNN_LAUNCH_CHECK("fused layer: schedule histogram");
    sched_scan_kernel<<<1, 1024, 0, stream>>>(counts, cursor);
    GNN_LAUNCH_CHECK("fused layer: schedule scan");
    const int64_t chunk = (g.n + blocks - 1) / blocks;
    sched_scatter_kernel<IdxT><<<blocks, 256, 0, stream>>>(rp, g.n, a.long_thr, chunk, cursor, order);
    GNN_LAUNCH_CHECK("fused layer: schedule scatter");
  }
  // after the scatter, cursor[0] is the end of the last degree class: the number of short rows
  FusedArgs fa{};
  fa.a = a;
  fa.order = order;
  fa.num_end = g.n;
  fa.has_self = q.has_self;
  fa.self_scale = q.self_scale;
  fa.n1 = static_cast<int>(q.n1);
  fa.n2 = static_cast<int>(q.n2);
  fa.b1 = q.b1;
  fa.b2 = q.b2;
  fa.relu1 = q.relu1;
  fa.relu2 = q.relu2;
  fa.out = q.out;
  fa.ldo = a.ldo;
  fa.x_row0 = g.row_begin;

  SideStream* side = nullptr;
  if (a.long_cap > 0) {
    // long rows: summed by spmm_long_kernel into their own rows of out, then
    // transformed in place by a copy-mode launch, all on the side stream
    int rc = side_stream(&side);
    if (rc != GNN_OK) return rc;
    side->mu.lock();
    cudaError_t e = cudaEventRecord(side->fork, stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side->stream, side->fork, 0);
    if (e == cudaSuccess) {
      const int long_blocks = static_cast<int>(
          std::min<int64_t>(a.long_cap + a.seg_cap, static_cast<int64_t>(GNN_SPMM_LONG_CTAS_PER_SM) * sm_count()));
      const size_t long_smem = static_cast<size_t>(a.long_split) * 32 * sizeof(float4);
      spmm_long_kernel<WM, MEAN, false, 1, IdxT>
          <<<dim3(static_cast<unsigned>(long_blocks), 1u), a.long_split * 32, long_smem, side->stream>>>(a);
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
      side->mu.unlock();
      return fail(GNN_ERR_CUDA, std::string("fused layer: long-row launch: ") + cudaGetErrorString(e));
    }
    count_launch();
    FusedArgs fl = fa;
    fl.copy = 1;
    fl.pos_begin = cursor;  // positions [short rows, n): the long rows
    fl.pos_end = nullptr;
    rc = launch_fused<WM, MEAN, IdxT, TWO>(fl, q.w1, q.w2, a.long_cap, side->stream);
    if (rc == GNN_OK) {
      e = cudaEventRecord(side->join, side->stream);
      if (e != cudaSuccess) rc = fail(GNN_ERR_CUDA, std::string("fused layer: join record: ") + cudaGetErrorString(e));
    }
    if (rc != GNN_OK) {
      side->mu.unlock();
      return rc;
    }
  }
  FusedArgs fs = fa;
  fs.copy = 0;
  fs.pos_begin = nullptr;
  fs.pos_end = cursor;  // positions [0, short rows)
  int rc = launch_fused<WM, MEAN, IdxT, TWO>(fs, q.w1, q.w2, g.n, stream);
  if (side != nullptr) {
    const cudaError_t e = cudaStreamWaitEvent(stream, side->join, 0);
    side->mu.unlock();
    if (e != cudaSuccess && rc == GNN_OK) {
      rc = fail(GNN_ERR_CUDA, std::string("fused layer: join side stream: ") + cudaGetErrorString(e));
    }
  }
  return rc;
}

template <int WM, int MEAN>
int run_fused(const FusedRequest& q, cudaStream_t stream) {
  const SpmmRequest& g = q.agg;
  if (g.n < 0 || g.nnz < 0 || g.f < 0 || q.n1 < 0 || q.n2 < 0) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "num_nodes, num_edges and the widths must be >= 0");
  }
  if (g.row_ptr_type != GNN_INDEX_INT32 && g.row_ptr_type != GNN_INDEX_INT64) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "row_ptr must be int32 or int64");
  }
  if (g.row_ptr_type == GNN_INDEX_INT32 && g.nnz > INT32_MAX) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "num_edges exceeds int32 row_ptr range; use int64 row_ptr");
  }
  if (g.n > INT32_MAX) return fail(GNN_ERR_INVALID_ARGUMENT, "num_nodes must fit int32 column ids");
  if (!fused_shape_ok(g.f, q.n1, q.n2)) {
    return fail(GNN_ERR_UNSUPPORTED,
                "fused layer: feat_dim must be 32, 64, 96 or 128, the widths 32, 64 or 128, and the output at least "
                "feat_dim wide");
  }
  if (!fused_device_ok()) return fail(GNN_ERR_DEVICE, "fused layer: needs an sm_100 device");
  if (g.n == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(g.row_ptr != nullptr && g.x != nullptr && q.out != nullptr && q.w1 != nullptr, GNN_ERR_NULL_POINTER,
              "row_ptr, x, weight and out must not be NULL");
  if (g.nnz > 0) GNN_REQUIRE(g.col != nullptr, GNN_ERR_NULL_POINTER, "col_ind must not be NULL");
  if (WM == kGcn) GNN_REQUIRE(g.dis != nullptr, GNN_ERR_NULL_POINTER, "deg_inv_sqrt must not be NULL");
  if (q.n2 > 0) GNN_REQUIRE(q.w2 != nullptr, GNN_ERR_NULL_POINTER, "the second weight must not be NULL");
  const uintptr_t al = reinterpret_cast<uintptr_t>(g.x) | reinterpret_cast<uintptr_t>(q.out) |
                       reinterpret_cast<uintptr_t>(q.w1) | reinterpret_cast<uintptr_t>(q.w2) |
                       reinterpret_cast<uintptr_t>(q.b1) | reinterpret_cast<uintptr_t>(q.b2);
  GNN_REQUIRE(al % 16 == 0, GNN_ERR_INVALID_ARGUMENT, "fused layer: x, out, weights and biases must be 16-byte aligned");
  GNN_REQUIRE(static_cast<const void*>(g.x) != static_cast<const void*>(q.out), GNN_ERR_INVALID_ARGUMENT,
              "fused layer: out must not alias x");
  int rc;
  const bool two = q.n2 > 0;
  if (g.row_ptr_type == GNN_INDEX_INT64) {
    rc = two ? run_fused_typed<WM, MEAN, int64_t, true>(q, stream) : run_fused_typed<WM, MEAN, int64_t, false>(q, stream);
  } else {
    rc = two ? run_fused_typed<WM, MEAN, int32_t, true>(q, stream) : run_fused_typed<WM, MEAN, int32_t, false>(q, stream);
  }
  if (rc == GNN_OK) clear_error();
  return rc;
}

}  // namespace
}  // namespace gnnb200

using gnnb200::FusedRequest;

extern "C" int gnn_fused_layer_supported(int64_t feat_dim, int64_t width1, int64_t width2) {
  return (gnnb200::fused_shape_ok(feat_dim, width1, width2) && gnnb200::fused_device_ok()) ? 1 : 0;
}

extern "C" int gnn_fused_aggregate_linear(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                          const float* deg_inv_sqrt, int aggregation, int64_t row_begin,
                                          const float* x, int64_t num_rows, int64_t num_cols, int64_t num_edges,
                                          int64_t feat_dim, float self_scale, int add_self, const float* weight1,
                                          const float* bias1, int64_t width1, int relu1, const float* weight2,
                                          const float* bias2, int64_t width2, int relu2, float* out,
                                          void* workspace, size_t workspace_bytes, gnn_stream_t stream) {
  using namespace gnnb200;
  GNN_REQUIRE(row_begin >= 0 && num_rows >= 0 && row_begin + num_rows <= num_cols, GNN_ERR_INVALID_ARGUMENT,
              "rows [row_begin, row_begin + num_rows) must lie inside [0, num_cols)");
  GNN_REQUIRE(num_cols <= INT32_MAX, GNN_ERR_INVALID_ARGUMENT, "num_cols must fit int32 column ids");
  FusedRequest q{};
  q.agg.row_ptr = row_ptr;
  q.agg.row_ptr_type = row_ptr_type;
  q.agg.col = col_ind;
  q.agg.dis = deg_inv_sqrt;
  q.agg.x = x;
  q.agg.n = num_rows;
  q.agg.nnz = num_edges;
  q.agg.f = feat_dim;
  q.agg.row_begin = row_begin;
  q.agg.ws = workspace;
  q.agg.ws_bytes = workspace_bytes;
  q.has_self = add_self ? 1 : 0;
  q.self_scale = self_scale;
  q.w1 = weight1;
  q.b1 = bias1;
  q.n1 = width1;
  q.relu1 = relu1 ? 1 : 0;
  q.w2 = weight2;
  q.b2 = bias2;
  q.n2 = width2;
  q.relu2 = relu2 ? 1 : 0;
  q.out = out;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (aggregation) {
    case GNN_AGG_GCN: return run_fused<kGcn, kNoMean>(q, s);
    case GNN_AGG_SUM: return run_fused<kUnit, kNoMean>(q, s);
    case GNN_AGG_MEAN: return run_fused<kUnit, kMeanDiv>(q, s);
    case GNN_AGG_MEAN_RECIPROCAL: return run_fused<kUnit, kMeanRcp>(q, s);
    default: return fail(GNN_ERR_INVALID_ARGUMENT, "aggregation must be GNN_AGG_GCN, _SUM, _MEAN or _MEAN_RECIPROCAL");
  }
}
