// CSR aggregation (SpMM) engine for GCN / PyG-weighted GCN / sum / mean.
//
// One engine serves every aggregation entry point of the reference
// (GNN_cuda_common/native/gcn_ops.cu:16-194, pyg_gcn_ops.cu:16-192,
// agg_ops.cu:23-130). The per-edge arithmetic is the reference's:
//   GCN     acc = fma(dis[r] * dis[c], x[c], acc)      (gcn_ops.cu:68-75)
//   PyG     acc = fma(edge_weight[e], x[c], acc)       (pyg_gcn_ops.cu:71-74)
//   sum     acc = acc + x[c]                           (agg_ops.cu:83-86)
//   mean    sum, then acc / deg or acc * (1 / deg)     (agg_ops.cu:40-45, :102-111)
// accumulated edge by edge in CSR order, so rows handled by a single warp give
// the same bits as the reference kernels.
//
// B200 mapping
//   * Normal rows: one warp per row. Each pass over a 32-edge chunk loads the 32
//     column indices (and weights) with one coalesced streaming load, then the
//     warp gathers U neighbour rows at a time with 128-bit loads (lane l owns
//     float4 columns l, l+32, ...), so U x 512 B per warp are in flight before
//     the first FMA. Output rows are written with one coalesced 128-bit store
//     per lane.
//   * Long rows (degree > threshold, the power-law hubs): a per-call plan
//     kernel lists them in the caller's workspace; the first CTAs of the main
//     grid pull them from that list with an atomic ticket and split each one
//     into contiguous per-warp edge ranges. The warp partials are added in warp
//     order through shared memory: deterministic, no float atomics. A row
//     longer than one CTA's segment (warps x 512 entries) is cut into
//     segments that separate CTAs take in ticket order; segment k adds its
//     partial to the row after segment k-1 has stored its own (a bounded wait
//     on a per-row counter), so a 10^5-entry hub costs ~512 dependent gathers
//     per warp instead of deg/16, and the sum order stays fixed.
//   * Feature widths that are not a multiple of 4 (or unaligned bases) use a
//     scalar warp-per-row kernel in plain CSR order.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"

namespace gnnb200 {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kBlockThreads = 512;       // 16 warps
#ifndef GNN_SPMM_ROWS_PER_WARP
#define GNN_SPMM_ROWS_PER_WARP 4
#endif
constexpr int kRowsPerWarp = GNN_SPMM_ROWS_PER_WARP;  // rows a warp takes per block (<= 32)
constexpr int kTileF4 = 128;             // float4 columns per feature tile (512 floats)
constexpr int kMaxTiles = 30;            // per-tile tickets live in the workspace header
constexpr size_t kWsHeader = 256;        // uint32 counters, see below
// Workspace header (uint32 words): [0] single-segment long rows listed,
// [1] segments of multi-segment rows listed, [2] long-work ticket (shared by
// all feature tiles), [32+t] work-item ticket of tile t.
constexpr int kHdrLongCount = 0;
constexpr int kHdrSegCount = 1;
constexpr int kHdrLongTicket = 2;
constexpr int kItemTicket = 32;
constexpr int64_t kMinLongThreshold = 32;
// A long row is summed by one CTA in segments of long_split * kSegEdgesPerWarp
// entries: each warp of the CTA takes at most this many entries of a segment.
constexpr int64_t kSegEdgesPerWarp = 512;
constexpr int64_t kMinSegLen = 4 * kSegEdgesPerWarp;  // spmm.long_row_warps >= 4
constexpr int kChainTimeout = 16;  // status code: a segment gave up waiting for its predecessor
constexpr int kPlanOverflow = 17;  // status code: long-row lists overflowed (num_edges too small)
constexpr uint32_t kSegTag = 0x80000000u;

// Neighbour rows a warp gathers per round (rows in flight per warp) and the
// number of 512-thread blocks kept resident per SM. Measured on B200: a few
// rows in flight per warp across many warps beats deep per-warp unrolling —
// too many outstanding gathers per SM congest the memory path.
#ifndef GNN_SPMM_U_NV1
#define GNN_SPMM_U_NV1 4
#endif
#ifndef GNN_SPMM_U_NV2
#define GNN_SPMM_U_NV2 4
#endif
#ifndef GNN_SPMM_U_NV34
#define GNN_SPMM_U_NV34 2
#endif
#ifndef GNN_SPMM_LONG_SERIAL
// 0: the long-row kernel runs on a side stream beside the per-row kernel; 1: before it, on the caller's stream
#define GNN_SPMM_LONG_SERIAL 0
#endif
#ifndef GNN_SPMM_PREFETCH_FIRST
// per-row kernel: load the next row's first 32 columns while the current row is gathered
#define GNN_SPMM_PREFETCH_FIRST 1
#endif
#ifndef GNN_SPMM_MIN_BLOCKS
// at F <= 128 (one float4 per lane); wider rows keep 2. Measured on B200 with the
// degree-ordered rows: 4 blocks (32 registers) 3.06 ms vs 3 blocks (40) 3.26 ms per
// aggregation of the products-shaped graph.
#define GNN_SPMM_MIN_BLOCKS 4
#endif
// Long-row kernel (spmm_long_kernel): register budget, grid and gather depth.
// Measured on B200 (products-shaped graph, F = 128): 64 registers and one
// full wave of long CTAs (2 per SM) beat 40 registers or 1 CTA per SM by 12-30 %.
#ifndef GNN_SPMM_LONG_MIN_BLOCKS
#define GNN_SPMM_LONG_MIN_BLOCKS 2  // register budget: 64 per thread at 512 threads
#endif
#ifndef GNN_SPMM_LONG_CTAS_PER_SM
#define GNN_SPMM_LONG_CTAS_PER_SM 2  // grid size: one full wave; per-row CTAs fill SMs as long CTAs finish
#endif
#ifndef GNN_SPMM_LONG_U
#define GNN_SPMM_LONG_U 4  // neighbour rows in flight per warp in the long-row kernel (F <= 128)
#endif
template <int NV>
__host__ __device__ constexpr int gather_depth() {
  return NV == 1 ? GNN_SPMM_U_NV1 : (NV == 2 ? GNN_SPMM_U_NV2 : GNN_SPMM_U_NV34);
}
template <int NV>
__host__ __device__ constexpr int resident_blocks() {
  return NV == 1 ? GNN_SPMM_MIN_BLOCKS : 2;
}

enum WeightMode : int { kUnit = 0, kGcn = 1, kEdge = 2 };
enum MeanMode : int { kNoMean = 0, kMeanDiv = 1, kMeanRcp = 2 };

struct SpmmArgs {
  const void* row_ptr;
  const int32_t* col;
  const float* dis;        // GCN normalisation vector, indexed by (global) column id
  const float* dis_row;    // GCN row scale base: dis_row[r] for local row r
  const float* ew;         // PyG edge weights
  const float* x;
  const float* hot;        // optimized mode: device copy of rows [0, hot_cutoff)
  int64_t hot_cutoff;
  const int64_t* sched;    // optional row schedule (slot -> row)
  const uint32_t* sched32; // engine-built degree order (slot -> row), per-row kernel only
  float* out;
  int64_t ldo;             // output row stride in floats (f, or wider when out has more columns)
  int64_t n;
  int64_t f;
  int64_t long_thr;
  uint32_t* counters;
  uint32_t* long_list;      // single-segment long rows
  int64_t long_cap;
  // Segments of multi-segment rows, one uint2 each: .x = row; .y = k | kSegTag
  // for segment k > 0, and for segment 0 (.y tag bit clear) the row's chain
  // counter: the number of (segment, tile) units of the row already stored.
  uint2* seg_items;
  int64_t seg_cap;
  int64_t seg_len;          // entries per segment (long_split * kSegEdgesPerWarp)
  int tiles;                // feature tiles (grid.y)
  int long_split;           // warps per segment (spmm.long_row_warps)
  int rows_per_warp;        // per-row kernel: rows a warp takes per block (2 or 4)
};

// Set by a segment whose bounded wait for its predecessor ran out (the row is
// then wrong); read and cleared through gnn_device_status.
__device__ int g_spmm_status = 0;

template <int WM>
__device__ __forceinline__ float edge_weight(const SpmmArgs& a, float rs, int c, int64_t e) {
  if constexpr (WM == kGcn) {
    return __fmul_rn(rs, __ldg(a.dis + c));
  } else if constexpr (WM == kEdge) {
    return ld_stream_f32(a.ew + e);
  } else {
    return 1.0f;
  }
}

template <bool HOT>
__device__ __forceinline__ const float* feature_row(const SpmmArgs& a, int c) {
  if constexpr (HOT) {
    if (c < a.hot_cutoff) return a.hot + static_cast<int64_t>(c) * a.f;
  }
  return a.x + static_cast<int64_t>(c) * a.f;
}

// This lane's float4 slice of feature row c: the row base is a 32x32->64-bit
// multiply-add off a per-lane base pointer (x + col0), one instruction.
template <bool HOT>
__device__ __forceinline__ const float4* gather_row(const SpmmArgs& a, int c, int64_t col0) {
  const uint32_t row_bytes = static_cast<uint32_t>(a.f) * 4u;
  const float* base = a.x;
  if constexpr (HOT) {
    if (c < a.hot_cutoff) base = a.hot;
  }
  const char* lane_base = reinterpret_cast<const char*>(base + col0 * 4);
  return reinterpret_cast<const float4*>(lane_base +
                                         static_cast<uint64_t>(static_cast<uint32_t>(c)) * row_bytes);
}

// Accumulates edges [beg, end) of one row into acc, edge by edge in CSR order.
// All 32 lanes of the warp must call this with the same arguments. When
// `have_first` is set, (c_first, w_first) already hold the first 32-edge chunk's
// column and weight for this lane (prefetched by the caller).
template <int WM, bool HOT, int NV, int U, class IdxT>
__device__ __forceinline__ void accumulate_edges(const SpmmArgs& a, IdxT beg, IdxT end, float rs,
                                                 int lane, int64_t col0, const bool (&valid)[NV],
                                                 float4 (&acc)[NV], bool have_first = false,
                                                 int c_first = 0, float w_first = 0.0f) {
  static_assert(32 % U == 0, "U must divide the warp size");
  for (IdxT base = beg; base < end; base += 32) {
    const int cnt = static_cast<int>(min(static_cast<IdxT>(32), static_cast<IdxT>(end - base)));
    int c = 0;
    float w = 0.0f;
    if (have_first && base == beg) {
      c = c_first;
      w = w_first;
    } else if (lane < cnt) {
      c = ld_stream_i32(a.col + base + lane);
      w = edge_weight<WM>(a, rs, c, static_cast<int64_t>(base) + lane);
    }
    // full groups of U edges: no per-edge guards
    int j = 0;
    for (; j + U <= cnt; j += U) {
      float4 v[U][NV];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const float4* row = gather_row<HOT>(a, __shfl_sync(kFull, c, j + k), col0);
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          if (valid[q]) v[k][q] = ldg_f4(row + 32 * q);
        }
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const float wk = __shfl_sync(kFull, w, j + k);
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          if (valid[q]) {
            if constexpr (WM == kUnit) {
              acc[q] = add4(acc[q], v[k][q]);
            } else {
              acc[q] = fma4(wk, v[k][q], acc[q]);
            }
          }
        }
      }
    }
    // the remaining cnt % U edges, one at a time
    for (; j < cnt; ++j) {
      const float4* row = gather_row<HOT>(a, __shfl_sync(kFull, c, j), col0);
      const float wk = __shfl_sync(kFull, w, j);
#pragma unroll
      for (int q = 0; q < NV; ++q) {
        if (valid[q]) {
          const float4 v = ldg_f4(row + 32 * q);
          if constexpr (WM == kUnit) {
            acc[q] = add4(acc[q], v);
          } else {
            acc[q] = fma4(wk, v, acc[q]);
          }
        }
      }
    }
  }
}

template <int MEAN>
__device__ __forceinline__ float4 finish(float4 acc, int64_t deg) {
  if constexpr (MEAN == kMeanDiv) {
    if (deg > 0) {
      const float d = static_cast<float>(deg);
      acc.x = __fdiv_rn(acc.x, d);
      acc.y = __fdiv_rn(acc.y, d);
      acc.z = __fdiv_rn(acc.z, d);
      acc.w = __fdiv_rn(acc.w, d);
    }
  } else if constexpr (MEAN == kMeanRcp) {
    if (deg > 0) {
      const float inv = __fdiv_rn(1.0f, static_cast<float>(deg));
      acc.x = __fmul_rn(acc.x, inv);
      acc.y = __fmul_rn(acc.y, inv);
      acc.z = __fmul_rn(acc.z, inv);
      acc.w = __fmul_rn(acc.w, inv);
    }
  }
  return acc;
}

// Lists the rows whose degree exceeds the long-row threshold: rows that fit
// one segment go to `list`; a longer row reserves ceil(deg / seg_len)
// consecutive segment slots and writes (row, 0) into the first (its chain
// counter starts at 0) and (row, k | kSegTag) into the others.
template <class IdxT>
__global__ void plan_long_rows_kernel(const IdxT* __restrict__ row_ptr, int64_t n, int64_t thr,
                                      int64_t seg_len, uint32_t* __restrict__ counters,
                                      uint32_t* __restrict__ list, int64_t cap,
                                      uint2* __restrict__ seg_items, int64_t seg_cap) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < n;
       r += stride) {
    const int64_t deg = static_cast<int64_t>(row_ptr[r + 1]) - static_cast<int64_t>(row_ptr[r]);
    if (deg <= thr) continue;
    if (deg <= seg_len) {
      const uint32_t i = atomicAdd(&counters[kHdrLongCount], 1u);
      if (i < cap) list[i] = static_cast<uint32_t>(r);
    } else {
      const int64_t nk = (deg + seg_len - 1) / seg_len;
      const uint32_t base = atomicAdd(&counters[kHdrSegCount], static_cast<uint32_t>(nk));
      if (static_cast<int64_t>(base) + nk <= seg_cap) {
        for (int64_t k = 0; k < nk; ++k) {
          const uint32_t tag = k == 0 ? 0u : (static_cast<uint32_t>(k) | kSegTag);
          seg_items[base + k] = make_uint2(static_cast<uint32_t>(r), tag);
        }
      }
    }
  }
}

// Thread-level bounded wait until *p >= target (acquire). ~2 s at most.
__device__ __forceinline__ bool wait_at_least(const uint32_t* p, uint32_t target) {
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    __nanosleep(128);
  }
  return false;
}

// Long-row phase shared by every vector kernel. Work units, taken with one
// atomic ticket in this order: the segments of multi-segment rows (segment
// major, feature tile minor), then the single-segment long rows. A unit is
// summed by the whole CTA: its segment is cut into long_split contiguous
// chunks (warp w takes chunks w, w + nwarps, ...), each summed edge by edge in
// CSR order, and the chunk partials are added in chunk order through shared
// memory. Segment k > 0 then waits until every tile of segments 0..k-1 has
// stored, and adds its partial to the stored prefix: row = ((s0 + s1) + s2)...
// Tickets are handed out in unit order, so a waiting segment's predecessors
// were taken earlier by CTAs that are running; the wait always ends.
// Inlined by default. Measured on B200 (products-shaped graph, F = 128): out of
// line, the phase gets its own register allocation but the call costs the
// per-row path more (5.65 vs 5.45 ms per aggregation). The kernels take their
// arguments as __grid_constant__, so an out-of-line phase reads them in place
// through a reference instead of from a per-thread local copy.
#ifndef GNN_SPMM_LONG_NOINLINE
#define GNN_SPMM_LONG_NOINLINE 0
#endif
#ifndef GNN_SPMM_GRID_CONST
#define GNN_SPMM_GRID_CONST 1
#endif
#if GNN_SPMM_GRID_CONST
#define GNN_KPARAM const __grid_constant__
#else
#define GNN_KPARAM
#endif
#if GNN_SPMM_LONG_NOINLINE
#define GNN_LONG_PHASE_INLINE __noinline__
#else
#define GNN_LONG_PHASE_INLINE __forceinline__
#endif
template <int WM, int MEAN, bool HOT, int NV, class IdxT>
__device__ GNN_LONG_PHASE_INLINE void long_rows_phase(const SpmmArgs& a, float4* s_part, uint32_t* s_ticket) {
  constexpr int U = NV == 1 ? GNN_SPMM_LONG_U : gather_depth<NV>();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int split = a.long_split;
  const int64_t f4 = a.f >> 2;
  const IdxT* __restrict__ rp = static_cast<const IdxT*>(a.row_ptr);
  const uint32_t tiles = static_cast<uint32_t>(a.tiles);
  uint32_t nseg = __ldcg(&a.counters[kHdrSegCount]);
  uint32_t nlong = __ldcg(&a.counters[kHdrLongCount]);
  if (nseg > a.seg_cap || nlong > a.long_cap) {
    // only possible when num_edges understates the entries row_ptr spans:
    // the lists are incomplete, so their rows are not computed and this is flagged
    if (threadIdx.x == 0) atomicCAS(&g_spmm_status, 0, kPlanOverflow);
    nseg = 0;
    nlong = 0;
  }
  const uint64_t total = static_cast<uint64_t>(nseg + nlong) * tiles;
  while (true) {
    if (threadIdx.x == 0) *s_ticket = atomicAdd(&a.counters[kHdrLongTicket], 1u);
    __syncthreads();
    const uint32_t t = *s_ticket;
    __syncthreads();
    if (t >= total) break;
    const uint32_t unit = t / tiles;
    const int tile = static_cast<int>(t - unit * tiles);
    // Index arithmetic stays in the row_ptr type (32-bit for int32 row_ptr):
    // this phase shares the kernel's register budget with the per-row path.
    int r;  // row ids fit int32 (num_nodes is limited to int32 column ids)
    uint32_t k = 0, head = unit;
    if (unit < nseg) {
      const uint2 it = __ldcg(a.seg_items + unit);  // a head's .y may already count stored units
      r = static_cast<int>(it.x);
      k = (it.y & kSegTag) ? (it.y & ~kSegTag) : 0u;
      head = unit - k;
    } else {
      r = static_cast<int>(a.long_list[unit - nseg]);
    }
    const IdxT beg = rp[r];
    const IdxT end = rp[r + 1];
    const IdxT seg = static_cast<IdxT>(a.seg_len);
    const IdxT sb = beg + static_cast<IdxT>(k) * seg;
    const IdxT se = (end - sb > seg) ? static_cast<IdxT>(sb + seg) : end;
    const bool last = se == end;  // the row's final segment (or its only one)
    const IdxT chunk = (se - sb + split - 1) / split;
    const int64_t col0 = static_cast<int64_t>(tile) * kTileF4 + lane;
    bool valid[NV];
#pragma unroll
    for (int q = 0; q < NV; ++q) valid[q] = (col0 + 32 * q) < f4;
    const float rs = (WM == kGcn) ? __ldg(a.dis_row + r) : 1.0f;
    for (int c = warp; c < split; c += nwarps) {
      const IdxT off = static_cast<IdxT>(c) * chunk;
      const IdxT wb = off < se - sb ? static_cast<IdxT>(sb + off) : se;
      const IdxT we = se - wb > chunk ? static_cast<IdxT>(wb + chunk) : se;
      float4 acc[NV];
#pragma unroll
      for (int q = 0; q < NV; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      accumulate_edges<WM, HOT, NV, U, IdxT>(a, wb, we, rs, lane, col0, valid, acc);
#pragma unroll
      for (int q = 0; q < NV; ++q) s_part[c * 32 * NV + q * 32 + lane] = acc[q];
    }
    __syncthreads();
    if (k > 0) {
      if (threadIdx.x == 0 && !wait_at_least(&a.seg_items[head].y, k * tiles)) {
        atomicCAS(&g_spmm_status, 0, kChainTimeout);
      }
      __syncthreads();
    }
    float4* orow = reinterpret_cast<float4*>(a.out + static_cast<int64_t>(r) * a.ldo);
    for (int j = threadIdx.x; j < 32 * NV; j += blockDim.x) {
      const int64_t cj = static_cast<int64_t>(tile) * kTileF4 + j;
      if (cj < f4) {
        float4 s = s_part[j];
        for (int w = 1; w < split; ++w) s = add4(s, s_part[w * 32 * NV + j]);
        if (k > 0) s = add4(__ldcg(orow + cj), s);
        if (last) s = finish<MEAN>(s, static_cast<int64_t>(end - beg));
        st_out_f4(orow + cj, s);
      }
    }
    if (!last) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) atomicAdd(&a.seg_items[head].y, 1u);
    }
    __syncthreads();
  }
}

// Long rows of the per-row path, in a kernel of their own: it runs beside
// spmm_vec_kernel (forked onto a side stream and joined back), so the hubs
// are summed while the short rows stream, and neither kernel's register
// allocation is shaped by the other's code.
template <int WM, int MEAN, bool HOT, int NV, class IdxT>
__global__ void __launch_bounds__(kBlockThreads, GNN_SPMM_LONG_MIN_BLOCKS)
    spmm_long_kernel(GNN_KPARAM SpmmArgs a) {
  extern __shared__ float4 s_part[];  // [long_split][32 * NV]
  __shared__ uint32_t s_ticket;
  long_rows_phase<WM, MEAN, HOT, NV, IdxT>(a, s_part, &s_ticket);
}

// Per-row vector kernel: RPW rows per warp, skipping long rows
// (spmm_long_kernel's). RPW = 4 by default; 2 for dense graphs (mean degree of
// 64 entries and more), where a warp's rows are long enough that fewer rows per
// warp and more warps per row set win (measured on B200, Reddit-shaped graph:
// 5.77 vs 6.33 ms per aggregation; products shape: 3.40 vs 3.26 ms the other way).
template <int WM, int MEAN, bool HOT, int NV, class IdxT, int RPW>
__global__ void __launch_bounds__(kBlockThreads, resident_blocks<NV>())
    spmm_vec_kernel(GNN_KPARAM SpmmArgs a) {
  constexpr int kRowsPerWarp = RPW;
  constexpr int U = gather_depth<NV>();

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int tile = blockIdx.y;
  const int64_t f4 = a.f >> 2;
  const int64_t col0 = static_cast<int64_t>(tile) * kTileF4 + lane;
  bool valid[NV];
#pragma unroll
  for (int q = 0; q < NV; ++q) valid[q] = (col0 + 32 * q) < f4;
  const IdxT* __restrict__ rp = static_cast<const IdxT*>(a.row_ptr);

  // ---- normal rows ----
  // Lane i (< kRowsPerWarp) fetches row i's bounds and scale once; the first
  // 32-edge chunk (columns + weights) of row i+1 is loaded while row i's
  // neighbour rows are being gathered, so a row does not start with a
  // row_ptr -> col_ind -> gather chain of dependent loads.
  const int64_t blk = blockIdx.x;
  int my_row = -1;  // row ids fit int32 (num_nodes is limited to int32 column ids)
  IdxT my_beg = 0, my_end = 0;
  float my_rs = 1.0f;
  if (lane < kRowsPerWarp) {
    const int64_t slot = (blk * kRowsPerWarp + lane) * nwarps + warp;
    if (slot < a.n) {
      my_row = static_cast<int>(a.sched ? a.sched[slot] : (a.sched32 ? a.sched32[slot] : slot));
      my_beg = rp[my_row];
      my_end = rp[my_row + 1];
      if (WM == kGcn) my_rs = __ldg(a.dis_row + my_row);
    }
  }
  // first chunk of row i for this lane (no load for long rows: they are skipped)
  auto first_chunk = [&](int i, int& c, float& w) {
    const IdxT beg = __shfl_sync(kFull, my_beg, i);
    const IdxT end = __shfl_sync(kFull, my_end, i);
    const float rs = __shfl_sync(kFull, my_rs, i);
    const int64_t deg = static_cast<int64_t>(end - beg);
    c = 0;
    w = 0.0f;
    if (deg <= a.long_thr && lane < deg) {
      c = ld_stream_i32(a.col + beg + lane);
      w = edge_weight<WM>(a, rs, c, static_cast<int64_t>(beg) + lane);
    }
  };
  int c_next = 0;
  float w_next = 0.0f;
  if (GNN_SPMM_PREFETCH_FIRST) first_chunk(0, c_next, w_next);
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int64_t r = __shfl_sync(kFull, my_row, i);  // widened for the output offset
    if (r < 0) break;
    const IdxT beg = __shfl_sync(kFull, my_beg, i);
    const IdxT end = __shfl_sync(kFull, my_end, i);
    const float rs = __shfl_sync(kFull, my_rs, i);
    const int c_cur = c_next;
    const float w_cur = w_next;
    if (GNN_SPMM_PREFETCH_FIRST && i + 1 < kRowsPerWarp) first_chunk(i + 1, c_next, w_next);
    const int64_t deg = static_cast<int64_t>(end - beg);
    if (deg > a.long_thr) continue;  // owned by a long-row CTA
    float4 acc[NV];
#pragma unroll
    for (int q = 0; q < NV; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    accumulate_edges<WM, HOT, NV, U, IdxT>(a, beg, end, rs, lane, col0, valid, acc, GNN_SPMM_PREFETCH_FIRST != 0,
                                           c_cur, w_cur);
    float4* orow = reinterpret_cast<float4*>(a.out + r * a.ldo);
#pragma unroll
    for (int q = 0; q < NV; ++q) {
      if (valid[q]) st_out_f4(orow + col0 + 32 * q, finish<MEAN>(acc[q], deg));
    }
  }
}

// Persistent packed-stream kernel (the default vector path).
//
// Phase 1 — whole blocks take long rows from the plan list (atomic ticket) and
// split each over all warps, partials added in warp order (same as above).
// Phase 2 — every warp independently takes work items of 32 consecutive row
// slots (atomic ticket). For an item it prefix-sums the 32 row degrees (long
// rows count as 0) and walks the item's edges as one packed stream in batches
// of 32: lane l handles stream position v0 + l, finds its row by a 5-step
// shuffle binary search over the prefix sums, and loads that edge's column
// (and weight) — coalesced, because consecutive positions are consecutive CSR
// entries. The warp then gathers the batch's neighbour rows U at a time and
// accumulates them in stream order, writing each row when the stream moves
// past it. Every short row is still summed edge by edge in CSR order by one
// warp, so results are identical to the per-row kernel; what changes is that
// low-degree rows no longer leave lanes idle or serialise a row_ptr -> col ->
// gather latency chain per row, and no warp waits for slower rows of its block.
template <int WM, int MEAN, bool HOT, int NV, class IdxT>
__global__ void __launch_bounds__(kBlockThreads, resident_blocks<NV>()) spmm_stream_kernel(GNN_KPARAM SpmmArgs a) {
  constexpr int U = gather_depth<NV>();
  extern __shared__ float4 s_part[];  // [nwarps][32 * NV] (long rows only)
  __shared__ uint32_t s_ticket;

  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.y;
  const int64_t f4 = a.f >> 2;
  const int64_t col0 = static_cast<int64_t>(tile) * kTileF4 + lane;
  bool valid[NV];
#pragma unroll
  for (int q = 0; q < NV; ++q) valid[q] = (col0 + 32 * q) < f4;
  const IdxT* __restrict__ rp = static_cast<const IdxT*>(a.row_ptr);

  // ---------------- phase 1: long rows ----------------
  if (a.long_cap > 0) long_rows_phase<WM, MEAN, HOT, NV, IdxT>(a, s_part, &s_ticket);

  // ---------------- phase 2: packed streams of short rows ----------------
  const int64_t items = (a.n + 31) >> 5;
  while (true) {
    uint32_t item = 0;
    if (lane == 0) item = atomicAdd(&a.counters[kItemTicket + tile], 1u);
    item = __shfl_sync(kFull, item, 0);
    if (static_cast<int64_t>(item) >= items) break;
    const int64_t s0 = static_cast<int64_t>(item) << 5;

    // this lane's row of the item
    int64_t row = 0;
    IdxT rbeg = 0;
    int deg = 0;        // degree counted in the stream (0 for long rows)
    int true_deg = 0;   // for the mean
    bool live = false;  // a row this warp must write
    float rs = 1.0f;
    if (s0 + lane < a.n) {
      row = a.sched ? a.sched[s0 + lane] : s0 + lane;
      rbeg = rp[row];
      const int64_t d = static_cast<int64_t>(rp[row + 1]) - static_cast<int64_t>(rbeg);
      live = d <= a.long_thr;
      deg = live ? static_cast<int>(d) : 0;
      true_deg = deg;
      if (WM == kGcn) rs = __ldg(a.dis_row + row);
    }
    // exclusive prefix sum of the stream degrees
    int off = deg;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(kFull, off, d);
      if (lane >= d) off += t;
    }
    const int total = __shfl_sync(kFull, off, 31);
    off -= deg;

    float4 acc[NV];
#pragma unroll
    for (int q = 0; q < NV; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    int cur = 0;  // item-local row being accumulated

    // writes row `cur` (if this warp owns it) and clears the accumulator
    auto flush = [&]() {
      const int64_t orow_id = __shfl_sync(kFull, row, cur);
      const int is_live = __shfl_sync(kFull, static_cast<int>(live), cur);
      const int d = __shfl_sync(kFull, true_deg, cur);
      if (is_live) {
        float4* orow = reinterpret_cast<float4*>(a.out + orow_id * a.ldo);
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          if (valid[q]) st_out_f4(orow + col0 + 32 * q, finish<MEAN>(acc[q], d));
        }
      }
#pragma unroll
      for (int q = 0; q < NV; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    };

    for (int v0 = 0; v0 < total; v0 += 32) {
      const int cnt = min(32, total - v0);
      // stream position v -> item row (largest i with off_i <= v)
      const int v = v0 + lane;
      int ri = 0;
#pragma unroll
      for (int step = 16; step >= 1; step >>= 1) {
        const int oc = __shfl_sync(kFull, off, ri + step);
        if (oc <= v) ri += step;
      }
      const IdxT rb_i = __shfl_sync(kFull, rbeg, ri);
      const int off_i = __shfl_sync(kFull, off, ri);
      const float rs_i = __shfl_sync(kFull, rs, ri);
      int c = 0;
      float w = 0.0f;
      if (lane < cnt) {
        const IdxT e = rb_i + static_cast<IdxT>(v - off_i);
        c = ld_stream_i32(a.col + e);
        w = edge_weight<WM>(a, rs_i, c, static_cast<int64_t>(e));
      }
      for (int j = 0; j < cnt; j += U) {
        float4 vals[U][NV];
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int ck = __shfl_sync(kFull, c, (j + k) & 31);
          if (j + k < cnt) {
            const float4* xr = reinterpret_cast<const float4*>(feature_row<HOT>(a, ck));
#pragma unroll
            for (int q = 0; q < NV; ++q) {
              if (valid[q]) vals[k][q] = ldg_f4(xr + col0 + 32 * q);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int rk = __shfl_sync(kFull, ri, (j + k) & 31);
          const float wk = __shfl_sync(kFull, w, (j + k) & 31);
          if (j + k < cnt) {
            while (cur < rk) {  // the stream moved past row `cur`
              flush();
              ++cur;
            }
#pragma unroll
            for (int q = 0; q < NV; ++q) {
              if (valid[q]) {
                if constexpr (WM == kUnit) {
                  acc[q] = add4(acc[q], vals[k][q]);
                } else {
                  acc[q] = fma4(wk, vals[k][q], acc[q]);
                }
              }
            }
          }
        }
      }
    }
    // rows after the last edge of the item (and the last row itself)
    while (cur < 32 && s0 + cur < a.n) {
      flush();
      ++cur;
    }
  }
}

// ---------------------------------------------------------------------------
// Asynchronous-staging variant of the packed-stream kernel.
//
// Same work decomposition and per-row arithmetic as spmm_stream_kernel, but the
// neighbour rows are not gathered into registers: each lane copies its 16-byte
// slices of a batch of kAsyncBatch rows straight into a per-warp shared-memory
// ring with cp.async (L1-bypassing), commits the batch, and only then consumes
// the previous batch from shared memory. Two batches are in flight per warp
// while it computes, and no registers are tied up by outstanding loads, so
// bytes in flight per SM are bounded by shared memory (~190 KB) instead of by
// the register file. Every lane reads back only the bytes it copied itself, so
// per-thread cp.async.wait_group is the only synchronisation needed.
// ---------------------------------------------------------------------------
constexpr int kAsyncBatch = 16;   // edges per stage
constexpr int kAsyncStages = 2;

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int WM, int MEAN, bool HOT, int NV, class IdxT>
__global__ void __launch_bounds__(384, 1) spmm_async_kernel(GNN_KPARAM SpmmArgs a) {
  extern __shared__ float4 s_dyn[];
  __shared__ uint32_t s_ticket;
  constexpr int kRowF4 = 32 * NV;                                 // float4 slots per staged row
  constexpr int kWarpF4 = kAsyncStages * kAsyncBatch * kRowF4;    // per-warp ring

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int tile = blockIdx.y;
  const int64_t f4 = a.f >> 2;
  const int64_t col0 = static_cast<int64_t>(tile) * kTileF4 + lane;
  bool valid[NV];
#pragma unroll
  for (int q = 0; q < NV; ++q) valid[q] = (col0 + 32 * q) < f4;
  const IdxT* __restrict__ rp = static_cast<const IdxT*>(a.row_ptr);
  float4* ring = s_dyn + warp * kWarpF4;  // also reused as [nwarps][32*NV] partials for long rows
  const uint32_t ring_addr = static_cast<uint32_t>(__cvta_generic_to_shared(ring));

  // ---------------- phase 1: long rows (register gathers) ----------------
  // The same segments and chunk cut as the other kernels, whatever this
  // block's warp count: warp w sums chunks w, w + nwarps, ... into their own
  // shared-memory slots (the ring), which are then added in chunk order.
  if (a.long_cap > 0) long_rows_phase<WM, MEAN, HOT, NV, IdxT>(a, s_dyn, &s_ticket);

  // ---------------- phase 2: packed streams with cp.async staging ----------------
  const int64_t items = (a.n + 31) >> 5;
  while (true) {
    uint32_t item = 0;
    if (lane == 0) item = atomicAdd(&a.counters[kItemTicket + tile], 1u);
    item = __shfl_sync(kFull, item, 0);
    if (static_cast<int64_t>(item) >= items) break;
    const int64_t s0 = static_cast<int64_t>(item) << 5;

    int64_t row = 0;
    IdxT rbeg = 0;
    int deg = 0;
    int true_deg = 0;
    bool live = false;
    float rs = 1.0f;
    if (s0 + lane < a.n) {
      row = a.sched ? a.sched[s0 + lane] : s0 + lane;
      rbeg = rp[row];
      const int64_t d = static_cast<int64_t>(rp[row + 1]) - static_cast<int64_t>(rbeg);
      live = d <= a.long_thr;
      deg = live ? static_cast<int>(d) : 0;
      true_deg = deg;
      if (WM == kGcn) rs = __ldg(a.dis_row + row);
    }
    int off = deg;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(kFull, off, d);
      if (lane >= d) off += t;
    }
    const int total = __shfl_sync(kFull, off, 31);
    off -= deg;

    float4 acc[NV];
#pragma unroll
    for (int q = 0; q < NV; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    int cur = 0;
    auto flush = [&]() {
      const int64_t orow_id = __shfl_sync(kFull, row, cur);
      const int is_live = __shfl_sync(kFull, static_cast<int>(live), cur);
      const int d = __shfl_sync(kFull, true_deg, cur);
      if (is_live) {
        float4* orow = reinterpret_cast<float4*>(a.out + orow_id * a.ldo);
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          if (valid[q]) st_out_f4(orow + col0 + 32 * q, finish<MEAN>(acc[q], d));
        }
      }
#pragma unroll
      for (int q = 0; q < NV; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    };

    // previous batch, waiting in the ring: its weights / rows live in lanes 0..prev_cnt-1
    int prev_cnt = 0;
    int prev_ri = 0;
    float prev_w = 0.0f;
    int stage = 0;
    const int nbatches = (total + kAsyncBatch - 1) / kAsyncBatch;
    for (int b = 0; b <= nbatches; ++b) {
      int cnt = 0;
      int ri = 0;
      float w = 0.0f;
      if (b < nbatches) {
        // ---- prepare and issue batch b ----
        const int v0 = b * kAsyncBatch;
        cnt = min(kAsyncBatch, total - v0);
        const int v = v0 + lane;
#pragma unroll
        for (int step = 16; step >= 1; step >>= 1) {
          const int oc = __shfl_sync(kFull, off, ri + step);
          if (oc <= v) ri += step;
        }
        const IdxT rb_i = __shfl_sync(kFull, rbeg, ri);
        const int off_i = __shfl_sync(kFull, off, ri);
        const float rs_i = __shfl_sync(kFull, rs, ri);
        int c = 0;
        if (lane < cnt) {
          const IdxT e = rb_i + static_cast<IdxT>(v - off_i);
          c = ld_stream_i32(a.col + e);
          w = edge_weight<WM>(a, rs_i, c, static_cast<int64_t>(e));
        }
        const uint32_t stage_addr = ring_addr + static_cast<uint32_t>(stage * kAsyncBatch * kRowF4 * 16);
        for (int j = 0; j < cnt; ++j) {
          const int cj = __shfl_sync(kFull, c, j);
          const float* xr = feature_row<HOT>(a, cj);
#pragma unroll
          for (int q = 0; q < NV; ++q) {
            if (valid[q]) {
              cp_async16(stage_addr + static_cast<uint32_t>((j * kRowF4 + q * 32 + lane) * 16),
                         xr + (col0 + 32 * q) * 4);
            }
          }
        }
        cp_async_commit();
      }
      if (b > 0) {
        // ---- consume batch b-1 (issued one stage ago) ----
        if (b < nbatches) {
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
        const int pstage = stage ^ 1;
        const float4* pring = ring + pstage * kAsyncBatch * kRowF4;
        for (int j = 0; j < prev_cnt; ++j) {
          const int rk = __shfl_sync(kFull, prev_ri, j);
          const float wk = __shfl_sync(kFull, prev_w, j);
          while (cur < rk) {
            flush();
            ++cur;
          }
#pragma unroll
          for (int q = 0; q < NV; ++q) {
            if (valid[q]) {
              const float4 val = pring[j * kRowF4 + q * 32 + lane];
              if constexpr (WM == kUnit) {
                acc[q] = add4(acc[q], val);
              } else {
                acc[q] = fma4(wk, val, acc[q]);
              }
            }
          }
        }
      }
      prev_cnt = cnt;
      prev_ri = ri;
      prev_w = w;
      stage ^= 1;
    }
    while (cur < 32 && s0 + cur < a.n) {
      flush();
      ++cur;
    }
  }
}

// Scalar kernel for feature widths that are not a multiple of 4 (or unaligned
// pointers): one warp per row, lane l owns features l, l+32, l+64, l+96 of the
// block's 128-feature tile; plain CSR order for every row.
template <int WM, int MEAN, bool HOT, class IdxT>
__global__ void __launch_bounds__(256) spmm_scalar_kernel(SpmmArgs a) {
  constexpr int SV = 4;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int64_t fbase = static_cast<int64_t>(blockIdx.y) * 32 * SV + lane;
  const IdxT* __restrict__ rp = static_cast<const IdxT*>(a.row_ptr);
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * nwarps + warp;
  if (slot >= a.n) return;
  const int64_t r = a.sched ? a.sched[slot] : slot;
  const IdxT beg = rp[r];
  const IdxT end = rp[r + 1];
  const float rs = (WM == kGcn) ? __ldg(a.dis_row + r) : 1.0f;
  float acc[SV] = {0.f, 0.f, 0.f, 0.f};
  for (IdxT base = beg; base < end; base += 32) {
    const int cnt = static_cast<int>(min(static_cast<IdxT>(32), static_cast<IdxT>(end - base)));
    int c = 0;
    float w = 0.0f;
    if (lane < cnt) {
      c = ld_stream_i32(a.col + base + lane);
      w = edge_weight<WM>(a, rs, c, static_cast<int64_t>(base) + lane);
    }
    for (int j = 0; j < cnt; ++j) {
      const int cj = __shfl_sync(kFull, c, j);
      const float wj = __shfl_sync(kFull, w, j);
      const float* row = feature_row<HOT>(a, cj);
#pragma unroll
      for (int s = 0; s < SV; ++s) {
        const int64_t fi = fbase + 32 * s;
        if (fi < a.f) {
          const float v = __ldg(row + fi);
          acc[s] = (WM == kUnit) ? __fadd_rn(acc[s], v) : __fmaf_rn(wj, v, acc[s]);
        }
      }
    }
  }
  const int64_t deg = static_cast<int64_t>(end - beg);
#pragma unroll
  for (int s = 0; s < SV; ++s) {
    const int64_t fi = fbase + 32 * s;
    if (fi < a.f) {
      float v = acc[s];
      if (MEAN == kMeanDiv && deg > 0) v = __fdiv_rn(v, static_cast<float>(deg));
      if (MEAN == kMeanRcp && deg > 0) v = __fmul_rn(v, __fdiv_rn(1.0f, static_cast<float>(deg)));
      a.out[r * a.ldo + fi] = v;
    }
  }
}

int64_t long_capacity(int64_t n, int64_t nnz) {
  return std::max<int64_t>(0, std::min<int64_t>(n, nnz / (kMinLongThreshold + 1) + 1));
}

// Segments of multi-segment rows: a row longer than one segment (> seg_len >=
// kMinSegLen entries) has ceil(deg / seg_len) < 2 deg / seg_len of them.
int64_t segment_capacity(int64_t nnz) { return nnz > kMinSegLen ? 2 * (nnz / kMinSegLen) + 1 : 0; }

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Workspace layout: header | long_list u32[cap] | seg_items uint2[seg_cap].
// ---- degree-ordered row schedule ---------------------------------------------
// The per-row kernel takes rows in descending degree order when the caller's
// workspace has room for the order (gnn_spmm_schedule_workspace_bytes). Warps
// and blocks then hold rows of about the same length, so a block no longer
// waits for one slow warp, and the heaviest rows start first. Measured on B200
// (products-shaped graph, F = 128): 3.3 ms against 4.5 ms per aggregation in
// row-id order. Every row is still summed by one warp in CSR order: the order
// of rows changes nothing in the results. The order is a counting sort into
// kDegBuckets classes (exact degree below kDegBuckets - 1, longer rows in the
// last class, long-row-kernel rows after everything), built per call in
// O(num_nodes): a shared-memory histogram, one scan, one scatter with
// warp-aggregated atomics (rows of one class in any order).
constexpr int kDegBuckets = 1024;           // classes 0..1022 = degree, 1023 = degree >= 1023
constexpr int kSchedBins = kDegBuckets + 1; // + one class for rows the long-row kernel owns
constexpr int64_t kSchedMinRows = 1 << 16;  // below this the three launches cost more than they save

__device__ __forceinline__ int sched_bin(int64_t deg, int64_t long_thr) {
  if (deg > long_thr) return kDegBuckets;  // owned by spmm_long_kernel: scheduled last
  if (deg < 0) deg = 0;                    // a decreasing row_ptr must not index outside the bins
  return static_cast<int>(deg < kDegBuckets - 1 ? deg : kDegBuckets - 1);
}

template <class IdxT>
__global__ void __launch_bounds__(256) sched_hist_kernel(const IdxT* __restrict__ rp, int64_t n, int64_t long_thr,
                                                         uint32_t* __restrict__ counts) {
  __shared__ uint32_t h[kSchedBins];
  for (int i = threadIdx.x; i < kSchedBins; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < n; r += stride) {
    const int64_t deg = static_cast<int64_t>(rp[r + 1]) - static_cast<int64_t>(rp[r]);
    atomicAdd(&h[sched_bin(deg, long_thr)], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kSchedBins; i += blockDim.x) {
    if (h[i]) atomicAdd(&counts[i], h[i]);
  }
}

// cursor[b] = number of rows in classes scheduled before b: degree classes
// from the highest down, then the long-row class. One block of 1024 threads.
__global__ void __launch_bounds__(1024) sched_scan_kernel(const uint32_t* __restrict__ counts,
                                                          uint32_t* __restrict__ cursor) {
  __shared__ uint32_t part[1024];
  const int t = threadIdx.x;
  // thread t owns degree class kDegBuckets - 1 - t (descending order)
  const uint32_t mine = counts[kDegBuckets - 1 - t];
  part[t] = mine;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const uint32_t v = t >= off ? part[t - off] : 0u;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  cursor[kDegBuckets - 1 - t] = part[t] - mine;  // exclusive prefix in descending order
  if (t == 1023) cursor[kDegBuckets] = part[t];  // the long-row class comes after all of them
}

// Global order, last step. Each block takes a contiguous chunk of rows, counts
// its rows per class in shared memory, reserves one contiguous range per class
// with a single global atomic, and places its rows inside its ranges (shared
// atomics): global atomics scale with blocks x classes, not with rows.
template <class IdxT>
__global__ void __launch_bounds__(256) sched_scatter_kernel(const IdxT* __restrict__ rp, int64_t n, int64_t long_thr,
                                                            int64_t chunk, uint32_t* __restrict__ cursor,
                                                            uint32_t* __restrict__ order) {
  __shared__ uint32_t cnt[kSchedBins];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * chunk;
  const int64_t r1 = r0 + chunk < n ? r0 + chunk : n;
  for (int i = threadIdx.x; i < kSchedBins; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    atomicAdd(&cnt[sched_bin(static_cast<int64_t>(rp[r + 1]) - static_cast<int64_t>(rp[r]), long_thr)], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kSchedBins; i += blockDim.x) {
    if (cnt[i]) cnt[i] = atomicAdd(&cursor[i], cnt[i]);  // this block's first position in class i
  }
  __syncthreads();
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    const int b = sched_bin(static_cast<int64_t>(rp[r + 1]) - static_cast<int64_t>(rp[r]), long_thr);
    order[atomicAdd(&cnt[b], 1u)] = static_cast<uint32_t>(r);
  }
}

// Windowed order: one block sorts one window of `window` consecutive rows by
// class (highest degree first, the long-row kernel's rows last) into the same
// window of the order. Rows keep their neighbourhood in id order — graphs
// numbered by community keep their gather locality — while the rows that
// share a block of the per-row kernel have about the same degree.
template <class IdxT>
__global__ void __launch_bounds__(1024) sched_window_kernel(const IdxT* __restrict__ rp, int64_t n, int64_t long_thr,
                                                            int64_t window, uint32_t* __restrict__ order) {
  __shared__ uint32_t cnt[kSchedBins];
  __shared__ uint32_t part[1024];
  const int t = threadIdx.x;
  const int64_t w0 = static_cast<int64_t>(blockIdx.x) * window;
  const int64_t w1 = w0 + window < n ? w0 + window : n;
  for (int i = t; i < kSchedBins; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int64_t r = w0 + t; r < w1; r += blockDim.x) {
    atomicAdd(&cnt[sched_bin(static_cast<int64_t>(rp[r + 1]) - static_cast<int64_t>(rp[r]), long_thr)], 1u);
  }
  __syncthreads();
  // exclusive prefix over degree classes in descending order; thread t owns class kDegBuckets-1-t
  const uint32_t mine = cnt[kDegBuckets - 1 - t];
  part[t] = mine;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const uint32_t v = t >= off ? part[t - off] : 0u;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  const uint32_t base = static_cast<uint32_t>(w0);
  cnt[kDegBuckets - 1 - t] = base + part[t] - mine;
  if (t == 1023) cnt[kDegBuckets] = base + part[t];
  __syncthreads();
  for (int64_t r = w0 + t; r < w1; r += blockDim.x) {
    const int b = sched_bin(static_cast<int64_t>(rp[r + 1]) - static_cast<int64_t>(rp[r]), long_thr);
    order[atomicAdd(&cnt[b], 1u)] = static_cast<uint32_t>(r);
  }
}

size_t sched_bytes(int64_t n) {
  // counts + cursors (2 x kSchedBins uint32, rounded) + the order itself
  return ((2 * kSchedBins * sizeof(uint32_t) + 255) & ~size_t(255)) + ((static_cast<size_t>(n) * 4 + 255) & ~size_t(255));
}

struct WsLayout {
  size_t list_off, seg_off, total;
  int64_t cap, seg_cap;
};
WsLayout ws_layout(int64_t n, int64_t nnz) {
  WsLayout w{};
  w.cap = (n > 0 && nnz >= 0) ? long_capacity(n, nnz) : 0;
  w.seg_cap = (n > 0 && nnz >= 0) ? segment_capacity(nnz) : 0;
  w.list_off = kWsHeader;
  w.seg_off = w.list_off + align256(static_cast<size_t>(w.cap) * sizeof(uint32_t));
  w.total = w.seg_off + align256(static_cast<size_t>(w.seg_cap) * sizeof(uint2));
  return w;
}

int64_t resolve_long_threshold(int64_t n, int64_t nnz) {
  int64_t thr = config().long_row_threshold.load();
  if (thr <= 0) {
    // A row is "long" when one warp would spend more than ~1/8 of the average
    // per-warp share of the whole launch on it (148 SMs x 32 resident warps).
    const int64_t warps = static_cast<int64_t>(sm_count()) * 32;
    thr = nnz / std::max<int64_t>(1, warps * 8);
    thr = std::min<int64_t>(8192, std::max<int64_t>(256, thr));
  }
  return std::max(thr, kMinLongThreshold);
}

// Per-device side stream (non-blocking, so it never synchronises implicitly
// with the legacy default stream) and the fork / join events of the long-row
// kernel. The mutex keeps one call's record / wait pairs together when several
// host threads use the same device.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex mu;
};

int side_stream(SideStream** out) {
  static SideStream table[64];
  static std::mutex init_mu;
  int dev = 0;
  GNN_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(GNN_ERR_UNSUPPORTED, "spmm: device index above 63");
  SideStream& s = table[dev];
  std::lock_guard<std::mutex> g(init_mu);
  if (s.stream == nullptr) {
    GNN_CUDA_TRY(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking), "spmm: create side stream");
    GNN_CUDA_TRY(cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming), "spmm: create fork event");
    GNN_CUDA_TRY(cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming), "spmm: create join event");
  }
  *out = &s;
  return GNN_OK;
}

template <int WM, int MEAN, bool HOT, class IdxT>
int launch_vec(SpmmArgs a, cudaStream_t stream) {
  const int64_t f4 = a.f >> 2;
  const int64_t tiles = (f4 + kTileF4 - 1) / kTileF4;
  const int64_t lanes_f4 = std::min<int64_t>(f4, kTileF4);
  const int nv = static_cast<int>((lanes_f4 + 31) / 32);
  const int nwarps = static_cast<int>(config().long_row_warps.load());
  const int threads = nwarps * 32;
  const int rpw = a.rows_per_warp == 2 ? 2 : kRowsPerWarp;
  const int64_t rows_per_block = static_cast<int64_t>(nwarps) * (config().spmm_kernel.load() == 1 ? rpw : kRowsPerWarp);
  const int64_t normal_blocks = (a.n + rows_per_block - 1) / rows_per_block;

  const size_t smem = static_cast<size_t>(nwarps) * 32 * nv * sizeof(float4);
  dim3 block(threads);

  if (config().spmm_kernel.load() == 1) {
    // per-row kernel: one warp per row, blocks of consecutive rows; long rows
    // in spmm_long_kernel on the device's side stream, forked from and joined
    // back to `stream`
    const int64_t gx = normal_blocks;
    if (gx > 0x7fffffffLL) return fail(GNN_ERR_UNSUPPORTED, "spmm: too many rows for one launch");
    SideStream* side = nullptr;
    if (a.long_cap > 0 && GNN_SPMM_LONG_SERIAL) {
      // long rows first, on the caller's stream (no fork / join)
      const int long_blocks = static_cast<int>(
          std::min<int64_t>(a.long_cap + a.seg_cap, static_cast<int64_t>(GNN_SPMM_LONG_CTAS_PER_SM) * sm_count()));
      const size_t long_smem = static_cast<size_t>(a.long_split) * 32 * nv * sizeof(float4);
      dim3 lgrid(static_cast<unsigned>(long_blocks), static_cast<unsigned>(tiles));
#define GNN_LAUNCH_NV(NVV) spmm_long_kernel<WM, MEAN, HOT, NVV, IdxT><<<lgrid, block, long_smem, stream>>>(a)
      switch (nv) {
        case 1: GNN_LAUNCH_NV(1); break;
        case 2: GNN_LAUNCH_NV(2); break;
        case 3: GNN_LAUNCH_NV(3); break;
        default: GNN_LAUNCH_NV(4); break;
      }
#undef GNN_LAUNCH_NV
      GNN_LAUNCH_CHECK("spmm long-row kernel launch");
    } else if (a.long_cap > 0) {
      int rc = side_stream(&side);
      if (rc != GNN_OK) return rc;
      side->mu.lock();
      const int long_blocks = static_cast<int>(
          std::min<int64_t>(a.long_cap + a.seg_cap, static_cast<int64_t>(GNN_SPMM_LONG_CTAS_PER_SM) * sm_count()));
      const size_t long_smem = static_cast<size_t>(a.long_split) * 32 * nv * sizeof(float4);
      cudaError_t e = cudaEventRecord(side->fork, stream);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(side->stream, side->fork, 0);
      if (e != cudaSuccess) {
        side->mu.unlock();
        return fail(GNN_ERR_CUDA, std::string("spmm: fork to side stream: ") + cudaGetErrorString(e));
      }
      dim3 lgrid(static_cast<unsigned>(long_blocks), static_cast<unsigned>(tiles));
#define GNN_LAUNCH_NV(NVV) \
  spmm_long_kernel<WM, MEAN, HOT, NVV, IdxT><<<lgrid, block, long_smem, side->stream>>>(a)
      switch (nv) {
        case 1: GNN_LAUNCH_NV(1); break;
        case 2: GNN_LAUNCH_NV(2); break;
        case 3: GNN_LAUNCH_NV(3); break;
        default: GNN_LAUNCH_NV(4); break;
      }
#undef GNN_LAUNCH_NV
      e = cudaGetLastError();
      if (e == cudaSuccess) e = cudaEventRecord(side->join, side->stream);
      if (e != cudaSuccess) {
        side->mu.unlock();
        return fail(GNN_ERR_CUDA, std::string("spmm long-row kernel launch: ") + cudaGetErrorString(e));
      }
      count_launch();
    }
    int rc = GNN_OK;
    if (gx > 0) {
      dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(tiles));
#define GNN_LAUNCH_NV(NVV)                                                          \
  do {                                                                              \
    if (rpw == 2) spmm_vec_kernel<WM, MEAN, HOT, NVV, IdxT, 2><<<grid, block, 0, stream>>>(a); \
    else spmm_vec_kernel<WM, MEAN, HOT, NVV, IdxT, kRowsPerWarp><<<grid, block, 0, stream>>>(a); \
  } while (0)
      switch (nv) {
        case 1: GNN_LAUNCH_NV(1); break;
        case 2: GNN_LAUNCH_NV(2); break;
        case 3: GNN_LAUNCH_NV(3); break;
        default: GNN_LAUNCH_NV(4); break;
      }
#undef GNN_LAUNCH_NV
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) rc = fail(GNN_ERR_CUDA, std::string("spmm kernel launch: ") + cudaGetErrorString(e));
      else count_launch();
    }
    if (side != nullptr) {
      const cudaError_t e = cudaStreamWaitEvent(stream, side->join, 0);  // join, also on the error path
      side->mu.unlock();
      if (e != cudaSuccess && rc == GNN_OK) {
        rc = fail(GNN_ERR_CUDA, std::string("spmm: join side stream: ") + cudaGetErrorString(e));
      }
    }
    return rc;
  }

  if (config().spmm_kernel.load() == 2) {
    // asynchronous-staging kernel: one block per SM, 192 KiB of ring per block
    const int warps = std::min(12, 12 / nv);
    const size_t ring = static_cast<size_t>(warps) * kAsyncStages * kAsyncBatch * 32 * nv * sizeof(float4);
    const int64_t items_a = (a.n + 31) / 32;
    int64_t gxa = std::max<int64_t>((items_a + warps - 1) / warps,
                                    a.long_cap > 0 ? std::min<int64_t>(a.long_cap, sm_count()) : 1);
    gxa = std::max<int64_t>(1, std::min<int64_t>(gxa, sm_count()));
    dim3 grid_a(static_cast<unsigned>(gxa), static_cast<unsigned>(tiles));
    static int configured[64][4] = {};
    int dev = 0;
    GNN_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
#define GNN_LAUNCH_NV(NVV)                                                                                   \
  do {                                                                                                       \
    if (dev < 0 || dev >= 64 || !configured[dev][NVV - 1]) {                                                 \
      GNN_CUDA_TRY(cudaFuncSetAttribute(spmm_async_kernel<WM, MEAN, HOT, NVV, IdxT>,                         \
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ring)), \
                   "spmm_async_kernel: shared memory opt-in");                                               \
      if (dev >= 0 && dev < 64) configured[dev][NVV - 1] = 1;                                                \
    }                                                                                                        \
    spmm_async_kernel<WM, MEAN, HOT, NVV, IdxT><<<grid_a, warps * 32, ring, stream>>>(a);                    \
  } while (0)
    switch (nv) {
      case 1: GNN_LAUNCH_NV(1); break;
      case 2: GNN_LAUNCH_NV(2); break;
      case 3: GNN_LAUNCH_NV(3); break;
      default: GNN_LAUNCH_NV(4); break;
    }
#undef GNN_LAUNCH_NV
    GNN_LAUNCH_CHECK("spmm async kernel launch");
    return GNN_OK;
  }

  // persistent packed-stream kernel: as many blocks as are resident at once,
  // fewer for small graphs
  const int64_t items = (a.n + 31) / 32;
  const int64_t resident = static_cast<int64_t>(nv == 1 ? resident_blocks<1>() : resident_blocks<2>()) * sm_count();
  int64_t gx = std::max<int64_t>((items + nwarps - 1) / nwarps, a.long_cap > 0 ? std::min(a.long_cap, resident) : 1);
  gx = std::max<int64_t>(1, std::min(gx, resident));
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(tiles));
#define GNN_LAUNCH_NV(NVV) spmm_stream_kernel<WM, MEAN, HOT, NVV, IdxT><<<grid, block, smem, stream>>>(a)
  switch (nv) {
    case 1: GNN_LAUNCH_NV(1); break;
    case 2: GNN_LAUNCH_NV(2); break;
    case 3: GNN_LAUNCH_NV(3); break;
    default: GNN_LAUNCH_NV(4); break;
  }
#undef GNN_LAUNCH_NV
  GNN_LAUNCH_CHECK("spmm kernel launch");
  return GNN_OK;
}

template <int WM, int MEAN, bool HOT, class IdxT>
int launch_scalar(SpmmArgs a, cudaStream_t stream) {
  const int threads = 256;
  const int64_t rows_per_block = threads / 32;
  const int64_t gx = (a.n + rows_per_block - 1) / rows_per_block;
  const int64_t tiles = (a.f + 127) / 128;
  if (gx > 0x7fffffffLL) return fail(GNN_ERR_UNSUPPORTED, "spmm: too many rows for one launch");
  spmm_scalar_kernel<WM, MEAN, HOT, IdxT>
      <<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(tiles)), threads, 0, stream>>>(a);
  GNN_LAUNCH_CHECK("spmm scalar kernel launch");
  return GNN_OK;
}

struct SpmmRequest {
  const void* row_ptr;
  int row_ptr_type;
  const int32_t* col;
  const float* dis;
  const float* ew;
  const float* x;
  const float* hot;
  int64_t hot_cutoff;
  const int64_t* sched;
  float* out;
  int64_t n, nnz, f;
  int64_t row_begin;
  void* ws;
  size_t ws_bytes;
};

template <int WM, int MEAN, bool HOT, class IdxT>
int run_typed(const SpmmRequest& q, cudaStream_t stream) {
  SpmmArgs a{};
  a.row_ptr = q.row_ptr;
  a.col = q.col;
  a.dis = q.dis;
  a.dis_row = q.dis != nullptr ? q.dis + q.row_begin : nullptr;
  a.ew = q.ew;
  a.x = q.x;
  a.hot = q.hot;
  a.hot_cutoff = q.hot_cutoff;
  a.sched = q.sched;
  a.out = q.out;
  a.ldo = q.f;
  a.n = q.n;
  a.f = q.f;

  const uintptr_t align = reinterpret_cast<uintptr_t>(q.x) | reinterpret_cast<uintptr_t>(q.out) |
                          reinterpret_cast<uintptr_t>(q.hot);
  const bool vec = (q.f % 4 == 0) && (align % 16 == 0);
  if (!vec) return launch_scalar<WM, MEAN, HOT, IdxT>(a, stream);

  const int64_t tiles = ((q.f >> 2) + kTileF4 - 1) / kTileF4;
  if (tiles > kMaxTiles) {
    return fail(GNN_ERR_UNSUPPORTED, "spmm: feat_dim above " + std::to_string(kMaxTiles * 512) +
                                         " is not supported");
  }
  // Stream degrees are summed in 32-bit over 32 rows, so the threshold is capped at 2^25.
  a.long_thr = std::min<int64_t>(resolve_long_threshold(q.n, q.nnz), int64_t(1) << 25);
  a.long_cap = std::min<int64_t>(long_capacity(q.n, q.nnz), q.nnz / (a.long_thr + 1) + 1);
  a.long_split = static_cast<int>(config().long_row_warps.load());
  a.seg_len = static_cast<int64_t>(a.long_split) * kSegEdgesPerWarp;
  a.rows_per_warp = q.nnz >= 64 * q.n ? 2 : kRowsPerWarp;
  a.tiles = static_cast<int>(tiles);
  if (q.nnz <= a.long_thr) a.long_cap = 0;  // no row can be long
  // the workspace holds the work tickets (and the long-row lists when needed)
  const WsLayout lay = ws_layout(q.n, q.nnz);
  if (q.ws == nullptr || q.ws_bytes < lay.total) {
    return fail(GNN_ERR_WORKSPACE, "spmm: workspace missing or smaller than gnn_spmm_workspace_bytes()");
  }
  char* ws = static_cast<char*>(q.ws);
  a.counters = reinterpret_cast<uint32_t*>(ws);
  a.long_list = reinterpret_cast<uint32_t*>(ws + lay.list_off);
  a.seg_items = reinterpret_cast<uint2*>(ws + lay.seg_off);
  a.seg_cap = a.long_cap > 0 ? lay.seg_cap : 0;
  GNN_CUDA_TRY(cudaMemsetAsync(q.ws, 0, kWsHeader, stream), "spmm: workspace reset");
  if (a.long_cap > 0) {
    const int threads = 256;
    const int64_t want = (q.n + threads - 1) / threads;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 8LL * sm_count())));
    plan_long_rows_kernel<IdxT><<<blocks, threads, 0, stream>>>(
        static_cast<const IdxT*>(q.row_ptr), q.n, a.long_thr, a.seg_len, a.counters, a.long_list, a.long_cap,
        a.seg_items, a.seg_cap);
    GNN_LAUNCH_CHECK("spmm plan kernel launch");
  } else {
    a.long_thr = INT64_MAX;
  }
  // degree-ordered schedule for the per-row kernel, when the workspace holds it
  // Automatic choice, from measurements on B200: sparse power-law graphs (products
  // shape, mean degree 26) gain most from the global order (heaviest rows first,
  // 3.27 vs 3.63 ms windowed, 4.66 ms id order); dense community-numbered graphs
  // (Reddit shape, mean degree 492) keep their gather locality only in windows
  // (6.53 ms with 2,048-row windows, 7.05 ms id order, 8.65 ms global).
  int64_t sched_mode = config().spmm_schedule.load();
  if (sched_mode == 3) sched_mode = q.nnz < 64 * q.n ? 2 : 1;
  if (q.sched == nullptr && sched_mode != 0 && config().spmm_kernel.load() == 1 && q.n >= kSchedMinRows &&
      q.n <= UINT32_MAX && q.ws_bytes >= lay.total + sched_bytes(q.n)) {
    uint32_t* counts = reinterpret_cast<uint32_t*>(ws + lay.total);
    uint32_t* cursor = counts + kSchedBins;
    uint32_t* order = reinterpret_cast<uint32_t*>(ws + lay.total + ((2 * kSchedBins * sizeof(uint32_t) + 255) &
                                                                     ~size_t(255)));
    const IdxT* rp = static_cast<const IdxT*>(q.row_ptr);
    const int64_t window = config().spmm_schedule_window.load();
    if (sched_mode == 1) {
      const int64_t blocks = (q.n + window - 1) / window;
      sched_window_kernel<IdxT><<<static_cast<unsigned>(blocks), 1024, 0, stream>>>(rp, q.n, a.long_thr, window,
                                                                                    order);
      GNN_LAUNCH_CHECK("spmm schedule (windowed)");
    } else {
      GNN_CUDA_TRY(cudaMemsetAsync(counts, 0, kSchedBins * sizeof(uint32_t), stream), "spmm: schedule reset");
      const int64_t want = (q.n + 255) / 256;
      const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 4LL * sm_count())));
      sched_hist_kernel<IdxT><<<blocks, 256, 0, stream>>>(rp, q.n, a.long_thr, counts);
      GNN_LAUNCH_CHECK("spmm schedule histogram");
      sched_scan_kernel<<<1, 1024, 0, stream>>>(counts, cursor);
      GNN_LAUNCH_CHECK("spmm schedule scan");
      const int64_t chunk = (q.n + blocks - 1) / blocks;
      sched_scatter_kernel<IdxT><<<blocks, 256, 0, stream>>>(rp, q.n, a.long_thr, chunk, cursor, order);
      GNN_LAUNCH_CHECK("spmm schedule scatter");
    }
    a.sched32 = order;
  }
  return launch_vec<WM, MEAN, HOT, IdxT>(a, stream);
}

template <int WM, int MEAN>
int run(const SpmmRequest& q, cudaStream_t stream) {
  if (q.n < 0 || q.nnz < 0 || q.f < 0) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "num_nodes, num_edges and feat_dim must be >= 0");
  }
  if (q.row_ptr_type != GNN_INDEX_INT32 && q.row_ptr_type != GNN_INDEX_INT64) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "row_ptr must be int32 or int64");
  }
  if (q.row_ptr_type == GNN_INDEX_INT32 && q.nnz > INT32_MAX) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "num_edges exceeds int32 row_ptr range; use int64 row_ptr");
  }
  if (q.n > INT32_MAX) return fail(GNN_ERR_INVALID_ARGUMENT, "num_nodes must fit int32 column ids");
  if (q.n == 0 || q.f == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(q.row_ptr != nullptr, GNN_ERR_NULL_POINTER, "row_ptr must not be NULL");
  GNN_REQUIRE(q.x != nullptr && q.out != nullptr, GNN_ERR_NULL_POINTER, "x and out must not be NULL");
  if (q.nnz > 0) {
    GNN_REQUIRE(q.col != nullptr, GNN_ERR_NULL_POINTER, "col_ind must not be NULL");
    if (WM == kGcn) GNN_REQUIRE(q.dis != nullptr, GNN_ERR_NULL_POINTER, "deg_inv_sqrt must not be NULL");
    if (WM == kEdge) GNN_REQUIRE(q.ew != nullptr, GNN_ERR_NULL_POINTER, "edge_weight must not be NULL");
  }
  if (WM == kGcn) GNN_REQUIRE(q.dis != nullptr, GNN_ERR_NULL_POINTER, "deg_inv_sqrt must not be NULL");
  int rc;
  const bool hot = q.hot != nullptr;
  if (q.row_ptr_type == GNN_INDEX_INT64) {
    rc = hot ? run_typed<WM, MEAN, true, int64_t>(q, stream) : run_typed<WM, MEAN, false, int64_t>(q, stream);
  } else {
    rc = hot ? run_typed<WM, MEAN, true, int32_t>(q, stream) : run_typed<WM, MEAN, false, int32_t>(q, stream);
  }
  if (rc == GNN_OK) clear_error();
  return rc;
}

int check_optimized(const int64_t* sched, const float* hot, int64_t cutoff, int64_t n) {
  GNN_REQUIRE(sched != nullptr, GNN_ERR_NULL_POINTER, "row_schedule must be CUDA");
  GNN_REQUIRE(hot != nullptr, GNN_ERR_NULL_POINTER, "hot_feature_cache must be CUDA");
  GNN_REQUIRE(cutoff >= 1, GNN_ERR_INVALID_ARGUMENT, "hot_node_cutoff must be >= 1");
  GNN_REQUIRE(cutoff <= n, GNN_ERR_INVALID_ARGUMENT, "hot_node_cutoff must be <= num_nodes");
  return GNN_OK;
}

__global__ void stage_pages_kernel(const int64_t* __restrict__ page_ids, const float* __restrict__ x,
                                   float* __restrict__ out, int64_t total_rows, int64_t rows_per_page,
                                   int64_t f, int64_t n) {
  const int64_t count = total_rows * f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    const int64_t cached_row = i / f;
    const int64_t feat = i - cached_row * f;
    const int64_t page_slot = cached_row / rows_per_page;
    const int64_t node = page_ids[page_slot] * rows_per_page + (cached_row - page_slot * rows_per_page);
    out[i] = (node >= 0 && node < n) ? x[node * f + feat] : 0.0f;
  }
}

__global__ void copy_rows_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    out[i] = x[i];
  }
}

}  // namespace
}  // namespace gnnb200

using namespace gnnb200;

extern "C" size_t gnn_spmm_workspace_bytes(int64_t num_nodes, int64_t num_edges) {
  if (num_nodes <= 0 || num_edges < 0) return kWsHeader;
  return ws_layout(num_nodes, num_edges).total;
}

extern "C" int64_t gnn_spmm_long_row_threshold(int64_t num_nodes, int64_t num_edges) {
  if (num_nodes <= 0 || num_edges < 0) return kMinLongThreshold;
  return std::min<int64_t>(resolve_long_threshold(num_nodes, num_edges), int64_t(1) << 25);
}

extern "C" size_t gnn_spmm_schedule_workspace_bytes(int64_t num_nodes, int64_t num_edges) {
  if (num_nodes <= 0 || num_edges < 0) return kWsHeader;
  return ws_layout(num_nodes, num_edges).total + sched_bytes(num_nodes);
}

namespace gnnb200 {
int spmm_status_read(int reset, int* status) {
  GNN_CUDA_TRY(cudaMemcpyFromSymbol(status, g_spmm_status, sizeof(int)), "read spmm status word");
  if (reset) {
    const int zero = 0;
    GNN_CUDA_TRY(cudaMemcpyToSymbol(g_spmm_status, &zero, sizeof(int)), "reset spmm status word");
  }
  return GNN_OK;
}
}  // namespace gnnb200

static SpmmRequest make_req(const void* rp, int rpt, const int32_t* col, const float* dis,
                            const float* ew, const float* x, float* out, int64_t n, int64_t nnz,
                            int64_t f, void* ws, size_t wsb) {
  SpmmRequest q{};
  q.row_ptr = rp;
  q.row_ptr_type = rpt;
  q.col = col;
  q.dis = dis;
  q.ew = ew;
  q.x = x;
  q.out = out;
  q.n = n;
  q.nnz = nnz;
  q.f = f;
  q.ws = ws;
  q.ws_bytes = wsb;
  return q;
}

extern "C" int gnn_spmm_gcn_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                    const float* deg_inv_sqrt, const float* x, float* out,
                                    int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                                    void* workspace, size_t workspace_bytes, gnn_stream_t stream) {
  auto q = make_req(row_ptr, row_ptr_type, col_ind, deg_inv_sqrt, nullptr, x, out, num_nodes,
                    num_edges, feat_dim, workspace, workspace_bytes);
  return run<kGcn, kNoMean>(q, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_spmm_gcn_partition_forward(const void* row_ptr, int row_ptr_type,
                                              const int32_t* col_ind, const float* deg_inv_sqrt,
                                              int64_t row_begin, const float* x, float* out,
                                              int64_t num_rows, int64_t num_cols, int64_t num_edges,
                                              int64_t feat_dim, void* workspace, size_t workspace_bytes,
                                              gnn_stream_t stream) {
  GNN_REQUIRE(row_begin >= 0 && num_rows >= 0 && row_begin + num_rows <= num_cols, GNN_ERR_INVALID_ARGUMENT,
              "shard rows [row_begin, row_begin + num_rows) must lie inside [0, num_cols)");
  GNN_REQUIRE(num_cols <= INT32_MAX, GNN_ERR_INVALID_ARGUMENT, "num_cols must fit int32 column ids");
  auto q = make_req(row_ptr, row_ptr_type, col_ind, deg_inv_sqrt, nullptr, x, out, num_rows,
                    num_edges, feat_dim, workspace, workspace_bytes);
  q.row_begin = row_begin;
  return run<kGcn, kNoMean>(q, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_spmm_gcn_hmm_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                        const float* deg_inv_sqrt, const float* x, float* out,
                                        int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                                        void* workspace, size_t workspace_bytes, gnn_stream_t stream) {
  return gnn_spmm_gcn_forward(row_ptr, row_ptr_type, col_ind, deg_inv_sqrt, x, out, num_nodes,
                              num_edges, feat_dim, workspace, workspace_bytes, stream);
}

extern "C" int gnn_spmm_gcn_hmm_optimized_forward(
    const void* row_ptr, int row_ptr_type, const int32_t* col_ind, const float* deg_inv_sqrt,
    const float* x, const int64_t* row_schedule, const float* hot_feature_cache,
    int64_t hot_node_cutoff, float* out, int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
    void* workspace, size_t workspace_bytes, gnn_stream_t stream) {
  int rc = check_optimized(row_schedule, hot_feature_cache, hot_node_cutoff, num_nodes);
  if (rc != GNN_OK) return rc;
  auto q = make_req(row_ptr, row_ptr_type, col_ind, deg_inv_sqrt, nullptr, x, out, num_nodes,
                    num_edges, feat_dim, workspace, workspace_bytes);
  q.sched = row_schedule;
  q.hot = hot_feature_cache;
  q.hot_cutoff = hot_node_cutoff;
  return run<kGcn, kNoMean>(q, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_spmm_pyg_gcn_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                        const float* edge_weight, const float* x, float* out,
                                        int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                                        void* workspace, size_t workspace_bytes, gnn_stream_t stream) {
  auto q = make_req(row_ptr, row_ptr_type, col_ind, nullptr, edge_weight, x, out, num_nodes,
                    num_edges, feat_dim, workspace, workspace_bytes);
  return run<kEdge, kNoMean>(q, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_spmm_pyg_gcn_plain_forward(const void* row_ptr, int row_ptr_type,
                                              const int32_t* col_ind, const float* edge_weight,
                                              const float* x, float* out, int64_t num_nodes,
                                              int64_t num_edges, int64_t feat_dim, void* workspace,
                                              size_t workspace_bytes, gnn_stream_t stream) {
  return gnn_spmm_pyg_gcn_forward(row_ptr, row_ptr_type, col_ind, edge_weight, x, out, num_nodes,
                                  num_edges, feat_dim, workspace, workspace_bytes, stream);
}

extern "C" int gnn_spmm_pyg_gcn_optimized_forward(
    const void* row_ptr, int row_ptr_type, const int32_t* col_ind, const float* edge_weight,
    const float* x, const int64_t* row_schedule, const float* hot_feature_cache,
    int64_t hot_node_cutoff, float* out, int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
    void* workspace, size_t workspace_bytes, gnn_stream_t stream) {
  int rc = check_optimized(row_schedule, hot_feature_cache, hot_node_cutoff, num_nodes);
  if (rc != GNN_OK) return rc;
  auto q = make_req(row_ptr, row_ptr_type, col_ind, nullptr, edge_weight, x, out, num_nodes,
                    num_edges, feat_dim, workspace, workspace_bytes);
  q.sched = row_schedule;
  q.hot = hot_feature_cache;
  q.hot_cutoff = hot_node_cutoff;
  return run<kEdge, kNoMean>(q, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_spmm_sum_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                    const float* x, float* out, int64_t num_nodes, int64_t num_edges,
                                    int64_t feat_dim, void* workspace, size_t workspace_bytes,
                                    gnn_stream_t stream) {
  auto q = make_req(row_ptr, row_ptr_type, col_ind, nullptr, nullptr, x, out, num_nodes, num_edges,
                    feat_dim, workspace, workspace_bytes);
  return run<kUnit, kNoMean>(q, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_spmm_mean_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                     const float* x, float* out, int64_t num_nodes, int64_t num_edges,
                                     int64_t feat_dim, int reciprocal, void* workspace,
                                     size_t workspace_bytes, gnn_stream_t stream) {
  auto q = make_req(row_ptr, row_ptr_type, col_ind, nullptr, nullptr, x, out, num_nodes, num_edges,
                    feat_dim, workspace, workspace_bytes);
  if (reciprocal) return run<kUnit, kMeanRcp>(q, reinterpret_cast<cudaStream_t>(stream));
  return run<kUnit, kMeanDiv>(q, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gnn_stage_feature_pages(const int64_t* page_ids, int64_t num_pages, const float* x,
                                       int64_t num_nodes, float* out, int64_t rows_per_page,
                                       int64_t feat_dim, gnn_stream_t stream) {
  GNN_REQUIRE(rows_per_page >= 1, GNN_ERR_INVALID_ARGUMENT, "rows_per_page must be >= 1");
  GNN_REQUIRE(num_pages >= 0 && feat_dim >= 0 && num_nodes >= 0, GNN_ERR_INVALID_ARGUMENT,
              "sizes must be >= 0");
  const int64_t total_rows = num_pages * rows_per_page;
  const int64_t count = total_rows * feat_dim;
  if (count == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(page_ids && x && out, GNN_ERR_NULL_POINTER, "page_ids, x and out must not be NULL");
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>((count + threads - 1) / threads, 16LL * sm_count()));
  stage_pages_kernel<<<blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      page_ids, x, out, total_rows, rows_per_page, feat_dim, num_nodes);
  GNN_LAUNCH_CHECK("stage_feature_pages launch");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_stage_feature_rows(const float* x, int64_t x_rows, float* out, int64_t out_rows,
                                      int64_t feat_dim, gnn_stream_t stream) {
  GNN_REQUIRE(out_rows <= x_rows, GNN_ERR_INVALID_ARGUMENT,
              "out rows must be <= x rows for staged prefix copies");
  GNN_REQUIRE(out_rows >= 0 && feat_dim >= 0, GNN_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  const int64_t count = out_rows * feat_dim;
  if (count == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(x && out, GNN_ERR_NULL_POINTER, "x and out must not be NULL");
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>((count + threads - 1) / threads, 16LL * sm_count()));
  copy_rows_kernel<<<blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, out, count);
  GNN_LAUNCH_CHECK("stage_feature_rows launch");
  clear_error();
  return GNN_OK;
}

// One GNN layer (aggregation + dense transform) in one kernel; shares this file's helpers.
#include "fused_layer.cuh"
