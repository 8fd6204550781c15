// UVM locality preprocessing on the device: the row schedule, page metadata,
// co-access node order and hot-prefix partition that feed the row-scheduled
// ("optimized") aggregation under managed memory.
//
// Restates the reference's host implementation (GNN_cuda_common/graph_utils.py:
// 174-241 build_hot_partition_feature_permutation, :244-372
// build_page_reuse_schedule_metadata, :375-446 build_coaccess_feature_permutation),
// which walks rows, blocks and windows in Python loops. Every order it produces
// is an integer order with explicit tie-breaks, so the same arrays come out bit
// for bit from whole-array radix sorts (CUB, stable):
//   * argsort(-x, stable): one descending key/value sort of x with the identity;
//   * np.lexsort(keys): a chain of stable sorts of the running order, least
//     significant key first (the identity needs no pass);
//   * "the k items a segment touches most, ties by a secondary key": one sort
//     of (segment, item) keys with the item already replaced by its tie rank, a
//     run-length pass that counts each pair, and a stable sort of the runs by
//     (segment, count descending); the first k runs of each segment are the
//     answer, and stability keeps equal counts in tie-rank order.
// The device computes no floating point. The float64 ratios the reference
// reports are formed on the host from the integer totals read back, with the
// same IEEE operations, so they match bit for bit too.
//
// Every index read from caller memory is range-checked before it addresses
// anything; a bad row_ptr, column, schedule or id list is reported as an error
// and never dereferenced.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_run_length_encode.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "common.cuh"

namespace gnnb200 {
namespace {

constexpr int kThreads = 256;
constexpr int64_t kMaxTopK = 4096;  // largest signature_topk / window_cache_pages accepted

// device error word bits
constexpr unsigned kBadRowPtr = 1u, kBadCol = 2u, kBadId = 4u, kNotPerm = 8u;

size_t a256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

int grid_for(int64_t items) {
  const int64_t want = (items + kThreads - 1) / kThreads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 32LL * sm_count())));
}

// Bits needed to hold every value in [0, max_value].
int bits_for(uint64_t max_value) {
  int b = 1;
  while (b < 64 && (max_value >> b) != 0) ++b;
  return b;
}

#define GRID_LOOP(i, n)                                                                       \
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (n); \
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)

// ---- small kernels ---------------------------------------------------------------

__global__ void iota_kernel(int64_t* __restrict__ v, int64_t n) {
  GRID_LOOP(i, n) v[i] = i;
}

__global__ void fill_kernel(int64_t* __restrict__ v, int64_t n, int64_t value) {
  GRID_LOOP(i, n) v[i] = value;
}

__global__ void copy_u64_kernel(const int64_t* __restrict__ src, uint64_t* __restrict__ dst, int64_t n) {
  GRID_LOOP(i, n) dst[i] = static_cast<uint64_t>(src[i]);
}

// inv[perm[i]] = i; perm is known to be a permutation of [0, n).
__global__ void invert_kernel(const int64_t* __restrict__ perm, int64_t* __restrict__ inv, int64_t n) {
  GRID_LOOP(i, n) inv[perm[i]] = i;
}

// Flags values outside [0, n) and repeated values; seen[] must start at zero.
__global__ void check_perm_kernel(const int64_t* __restrict__ p, int64_t n, unsigned* __restrict__ seen,
                                  unsigned* __restrict__ bad) {
  unsigned f = 0;
  GRID_LOOP(i, n) {
    const int64_t v = p[i];
    if (v < 0 || v >= n) {
      f |= kNotPerm;
    } else if (atomicExch(&seen[v], 1u) != 0u) {
      f |= kNotPerm;
    }
  }
  if (f) atomicOr(bad, f);
}

// row_ptr must start at 0, end at num_entries and never decrease.
template <class IdxT>
__global__ void check_row_ptr_kernel(const IdxT* __restrict__ rp, int64_t n, int64_t e, unsigned* __restrict__ bad) {
  unsigned f = 0;
  GRID_LOOP(i, n + 1) {
    const int64_t v = static_cast<int64_t>(rp[i]);
    if (v < 0 || v > e) f |= kBadRowPtr;
    if (i == 0 && v != 0) f |= kBadRowPtr;
    if (i == n && v != e) f |= kBadRowPtr;
    if (i < n && static_cast<int64_t>(rp[i + 1]) < v) f |= kBadRowPtr;
  }
  if (f) atomicOr(bad, f);
}

__global__ void check_cols_kernel(const int32_t* __restrict__ col, int64_t e, int64_t n, unsigned* __restrict__ bad) {
  unsigned f = 0;
  GRID_LOOP(i, e) {
    const int32_t c = col[i];
    if (c < 0 || c >= n) f |= kBadCol;
  }
  if (f) atomicOr(bad, f);
}

template <class IdxT>
__global__ void degree_kernel(const IdxT* __restrict__ rp, int64_t n, int64_t* __restrict__ deg) {
  GRID_LOOP(r, n) deg[r] = static_cast<int64_t>(rp[r + 1]) - static_cast<int64_t>(rp[r]);
}

// page_hist[col / rpp] += 1 for every CSR entry (columns already checked)
__global__ void page_hist_kernel(const int32_t* __restrict__ col, int64_t e, int64_t rpp,
                                 unsigned long long* __restrict__ hist) {
  GRID_LOOP(i, e) atomicAdd(&hist[col[i] / rpp], 1ull);
}

__global__ void max_kernel(const int64_t* __restrict__ v, int64_t n, unsigned long long* __restrict__ out) {
  unsigned long long m = 0;
  GRID_LOOP(i, n) m = max(m, static_cast<unsigned long long>(v[i]));
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m) atomicMax(out, m);
}

// sum of hist[idx[i]] over i < n
__global__ void gather_sum_kernel(const int64_t* __restrict__ hist, const int64_t* __restrict__ idx, int64_t n,
                                  unsigned long long* __restrict__ out) {
  unsigned long long s = 0;
  GRID_LOOP(i, n) s += static_cast<unsigned long long>(hist[idx[i]]);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0 && s) atomicAdd(out, s);
}

// rank[order[i]] = i
__global__ void rank_kernel(const int64_t* __restrict__ order, int64_t n, int64_t* __restrict__ rank) {
  GRID_LOOP(i, n) rank[order[i]] = i;
}

// hist[v] += 1 for 1 <= v < len (np.bincount of the nonzero values)
__global__ void count_hist_kernel(const int64_t* __restrict__ v, int64_t n, int64_t len,
                                  unsigned long long* __restrict__ hist) {
  GRID_LOOP(i, n) {
    const int64_t x = v[i];
    if (x >= 1 && x < len) atomicAdd(&hist[x], 1ull);
  }
}

// Segment keys of every CSR entry: key = seg(r) * num_items + item(col), one warp per row.
//   kind 0: seg = r,                 item = rank[col / rpp]     (row signatures)
//   kind 1: seg = slot[r] / div,     item = rank[col / rpp]     (block / window pages)
//   kind 2: seg = col,               item = slot[r] / div       (node windows)
template <class IdxT, int kKind>
__global__ void entry_keys_kernel(const IdxT* __restrict__ rp, const int32_t* __restrict__ col, int64_t n,
                                  int64_t rpp, const int64_t* __restrict__ rank, const int64_t* __restrict__ slot,
                                  int64_t div, uint64_t num_items, uint64_t* __restrict__ keys) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += warps) {
    const int64_t b = static_cast<int64_t>(rp[r]);
    const int64_t end = static_cast<int64_t>(rp[r + 1]);
    uint64_t row_part = 0;
    if (kKind == 0) row_part = static_cast<uint64_t>(r);
    if (kKind != 0) row_part = static_cast<uint64_t>(slot[r] / div);
    for (int64_t e = b + lane; e < end; e += 32) {
      const int64_t c = col[e];
      if (kKind == 2) {
        keys[e] = static_cast<uint64_t>(c) * num_items + row_part;
      } else {
        keys[e] = row_part * num_items + static_cast<uint64_t>(rank[c / rpp]);
      }
    }
  }
}

// Run (unique key, count) -> composite sort key (segment asc, count desc) and the item.
__global__ void composite_kernel(const uint64_t* __restrict__ ukeys, const uint32_t* __restrict__ counts, int64_t u,
                                 uint64_t num_items, int cbits, uint64_t* __restrict__ comp,
                                 uint32_t* __restrict__ item) {
  const uint64_t cmask = (cbits >= 64) ? ~0ull : ((1ull << cbits) - 1);
  GRID_LOOP(i, u) {
    const uint64_t k = ukeys[i];
    const uint64_t seg = k / num_items;
    comp[i] = (seg << cbits) | (cmask - static_cast<uint64_t>(counts[i]));
    item[i] = static_cast<uint32_t>(k - seg * num_items);
  }
}

// Runs sorted by (segment, count desc, tie rank): first[seg] = index of the
// segment's first run.
__global__ void segment_heads_kernel(const uint64_t* __restrict__ comp, int64_t u, int cbits, int64_t num_segments,
                                     int64_t* __restrict__ first) {
  GRID_LOOP(i, u) {
    const uint64_t seg = comp[i] >> cbits;
    if (seg < static_cast<uint64_t>(num_segments) && (i == 0 || (comp[i - 1] >> cbits) != seg)) first[seg] = i;
  }
}

// A run is among its segment's first k when fewer than k runs of the same
// segment precede it.
__global__ void topk_extract_kernel(const uint64_t* __restrict__ comp, const uint32_t* __restrict__ item, int64_t u,
                                    int cbits, int64_t k, int64_t num_segments, const int64_t* __restrict__ first,
                                    const int64_t* __restrict__ item_map, int64_t* __restrict__ out_items,
                                    int64_t* __restrict__ out_counts, unsigned long long* __restrict__ totals,
                                    unsigned long long* __restrict__ covered, unsigned* __restrict__ bad) {
  const uint64_t cmask = (1ull << cbits) - 1;
  GRID_LOOP(i, u) {
    const uint64_t c = comp[i];
    const uint64_t seg = c >> cbits;
    if (seg >= static_cast<uint64_t>(num_segments)) {
      atomicOr(bad, kBadId);
      continue;
    }
    const uint64_t cnt = cmask - (c & cmask);
    const int64_t pos = i - first[seg];
    if (totals) atomicAdd(&totals[seg], static_cast<unsigned long long>(cnt));
    if (pos < k) {
      const int64_t it = item_map ? item_map[item[i]] : static_cast<int64_t>(item[i]);
      out_items[seg * k + pos] = it;
      if (out_counts) out_counts[seg * k + pos] = static_cast<int64_t>(cnt);
      if (covered) atomicAdd(&covered[seg], static_cast<unsigned long long>(cnt));
    }
  }
}

// keys[i] = src[perm[i] * stride + off] — one lexsort key in the running order
__global__ void gather_key_kernel(const int64_t* __restrict__ src, int64_t stride, int64_t off,
                                  const int64_t* __restrict__ perm, int64_t n, uint64_t* __restrict__ keys) {
  GRID_LOOP(i, n) keys[i] = static_cast<uint64_t>(src[perm[i] * stride + off]);
}

// access[src[i]] += 1 (ids checked), plus 1 per node for self-loops (access pre-filled)
__global__ void access_count_kernel(const int64_t* __restrict__ src, int64_t e, int64_t n,
                                    unsigned long long* __restrict__ access, unsigned* __restrict__ bad) {
  unsigned f = 0;
  GRID_LOOP(i, e) {
    const int64_t s = src[i];
    if (s < 0 || s >= n) {
      f |= kBadId;
    } else {
      atomicAdd(&access[s], 1ull);
    }
  }
  if (f) atomicOr(bad, f);
}

__global__ void col_access_kernel(const int32_t* __restrict__ col, int64_t e, unsigned long long* __restrict__ access) {
  GRID_LOOP(i, e) atomicAdd(&access[col[i]], 1ull);
}

// prefix input: v[i] = access[order[i]]
__global__ void gather_u64_kernel(const int64_t* __restrict__ access, const int64_t* __restrict__ order, int64_t n,
                                  uint64_t* __restrict__ out) {
  GRID_LOOP(i, n) out[i] = static_cast<uint64_t>(access[order[i]]);
}

// first index i with prefix[i] >= target (n if none): np.searchsorted(prefix, target, side="left")
__global__ void lower_bound_kernel(const uint64_t* __restrict__ prefix, int64_t n, uint64_t target,
                                   int64_t* __restrict__ out) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (prefix[mid] < target) lo = mid + 1;
    else hi = mid;
  }
  *out = lo;
}

// hot[order[i]] = (i < cutoff)
__global__ void hot_mask_kernel(const int64_t* __restrict__ order, int64_t n, int64_t cutoff,
                                int64_t* __restrict__ hot) {
  GRID_LOOP(i, n) hot[order[i]] = (i < cutoff) ? 1 : 0;
}

__global__ void base_flags_kernel(const int64_t* __restrict__ base, const int64_t* __restrict__ hot, int64_t n,
                                  int64_t* __restrict__ flags) {
  GRID_LOOP(i, n) flags[i] = hot[base[i]];
}

// stable partition: hot entries of base first (in base order), then the cold ones
__global__ void partition_scatter_kernel(const int64_t* __restrict__ base, const int64_t* __restrict__ flags,
                                         const int64_t* __restrict__ excl, int64_t n, int64_t num_hot,
                                         int64_t* __restrict__ perm) {
  GRID_LOOP(i, n) {
    const int64_t before = excl[i];
    perm[flags[i] ? before : num_hot + (i - before)] = base[i];
  }
}

__global__ void permute_edges_kernel(const int64_t* __restrict__ src, const int64_t* __restrict__ dst, int64_t e,
                                     const int64_t* __restrict__ inv, int64_t n, int64_t* __restrict__ so,
                                     int64_t* __restrict__ dout, unsigned* __restrict__ bad) {
  unsigned f = 0;
  GRID_LOOP(i, e) {
    const int64_t s = src[i], d = dst[i];
    if (s < 0 || s >= n || d < 0 || d >= n) {
      f |= kBadId;
      so[i] = -1;
      dout[i] = -1;
    } else {
      so[i] = inv[s];
      dout[i] = inv[d];
    }
  }
  if (f) atomicOr(bad, f);
}

// ---- workspace layout ---------------------------------------------------------------
// One layout serves every entry point for a given (num_nodes, num_entries, max_k):
//   entry-sized: ka, kb (u64), c, v (u32)         — the segment top-k sorts
//   node-sized:  n0..n3 (i64), sa, sb (u64), pa, pb (i64) — orders, lexsort passes
//   topk-sized:  t0, t1 (i64, num_nodes * max_k)   — signatures / node windows
//   words (256 B), CUB temp
struct Layout {
  size_t ka, kb, c, v, n0, n1, n2, n3, sa, sb, pa, pb, t0, t1, words, temp, temp_bytes, total;
};

int plan_layout(int64_t n, int64_t e, int64_t max_k, Layout* out) {
  const int64_t E = std::max<int64_t>(e, 1);
  const int64_t M = std::max<int64_t>(n, 1) + 1;
  const int64_t T = std::max<int64_t>(n, 1) * std::max<int64_t>(max_k, 1);
  size_t t_sort_e = 0, t_rle = 0, t_pairs_e = 0, t_pairs_m = 0, t_scan = 0, t_iscan = 0;
  {
    cub::DoubleBuffer<uint64_t> k(nullptr, nullptr);
    cub::DoubleBuffer<uint32_t> v(nullptr, nullptr);
    cub::DoubleBuffer<int64_t> p(nullptr, nullptr);
    GNN_CUDA_TRY(cub::DeviceRadixSort::SortKeys(nullptr, t_sort_e, k, E, 0, 64), "locality: sort size query");
    GNN_CUDA_TRY(cub::DeviceRunLengthEncode::Encode(nullptr, t_rle, static_cast<const uint64_t*>(nullptr),
                                                    static_cast<uint64_t*>(nullptr), static_cast<uint32_t*>(nullptr),
                                                    static_cast<int64_t*>(nullptr), E),
                 "locality: run-length size query");
    GNN_CUDA_TRY(cub::DeviceRadixSort::SortPairs(nullptr, t_pairs_e, k, v, E, 0, 64), "locality: sort size query");
    GNN_CUDA_TRY(cub::DeviceRadixSort::SortPairs(nullptr, t_pairs_m, k, p, M, 0, 64), "locality: sort size query");
    GNN_CUDA_TRY(cub::DeviceScan::ExclusiveSum(nullptr, t_scan, static_cast<const int64_t*>(nullptr),
                                               static_cast<int64_t*>(nullptr), M),
                 "locality: scan size query");
    GNN_CUDA_TRY(cub::DeviceScan::InclusiveSum(nullptr, t_iscan, static_cast<const uint64_t*>(nullptr),
                                               static_cast<uint64_t*>(nullptr), M),
                 "locality: scan size query");
  }
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += a256(bytes);
    return at;
  };
  L.ka = take(sizeof(uint64_t) * E);
  L.kb = take(sizeof(uint64_t) * E);
  L.c = take(sizeof(uint32_t) * E);
  L.v = take(sizeof(uint32_t) * E);
  L.n0 = take(sizeof(int64_t) * M);
  L.n1 = take(sizeof(int64_t) * M);
  L.n2 = take(sizeof(int64_t) * M);
  L.n3 = take(sizeof(int64_t) * M);
  L.sa = take(sizeof(uint64_t) * M);
  L.sb = take(sizeof(uint64_t) * M);
  L.pa = take(sizeof(int64_t) * M);
  L.pb = take(sizeof(int64_t) * M);
  L.t0 = take(sizeof(int64_t) * T);
  L.t1 = take(sizeof(int64_t) * T);
  L.words = take(256);
  L.temp_bytes = std::max({t_sort_e, t_rle, t_pairs_e, t_pairs_m, t_scan, t_iscan});
  L.temp = take(L.temp_bytes);
  L.total = off;
  *out = L;
  return GNN_OK;
}

struct Ctx {
  char* ws;
  Layout L;
  cudaStream_t s;
  template <class T>
  T* at(size_t off) const { return reinterpret_cast<T*>(ws + off); }
  unsigned* bad() const { return at<unsigned>(L.words); }
  // words: [0] error bits, [1] run count, [2] max page count, [3] hot page accesses, [4] search result
  unsigned long long* word(int i) const { return at<unsigned long long>(L.words + 8 * i); }
  void* temp() const { return ws + L.temp; }
};

int reset_words(const Ctx& C) {
  GNN_CUDA_TRY(cudaMemsetAsync(C.ws + C.L.words, 0, 256, C.s), "locality: reset counters");
  return GNN_OK;
}

int read_back(const Ctx& C, void* host, const void* dev, size_t bytes, const char* what) {
  GNN_CUDA_TRY(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, C.s), what);
  GNN_CUDA_TRY(cudaStreamSynchronize(C.s), what);
  return GNN_OK;
}

int read_bad(const Ctx& C, unsigned* bad) { return read_back(C, bad, C.bad(), sizeof(unsigned), "locality: read flags"); }

// Stable argsort of int64 values, descending (argsort(-x, kind="stable")); the
// order lands in `order` (n entries). Uses sa/sb/pa/pb.
int argsort_desc(const Ctx& C, const int64_t* values, int64_t n, int bits, int64_t* order) {
  if (n == 0) return GNN_OK;
  uint64_t* sa = C.at<uint64_t>(C.L.sa);
  uint64_t* sb = C.at<uint64_t>(C.L.sb);
  int64_t* pa = C.at<int64_t>(C.L.pa);
  int64_t* pb = C.at<int64_t>(C.L.pb);
  copy_u64_kernel<<<grid_for(n), kThreads, 0, C.s>>>(values, sa, n);
  GNN_LAUNCH_CHECK("locality: keys");
  iota_kernel<<<grid_for(n), kThreads, 0, C.s>>>(pa, n);
  GNN_LAUNCH_CHECK("locality: iota");
  cub::DoubleBuffer<uint64_t> k(sa, sb);
  cub::DoubleBuffer<int64_t> v(pa, pb);
  size_t tb = C.L.temp_bytes;
  GNN_CUDA_TRY(cub::DeviceRadixSort::SortPairsDescending(C.temp(), tb, k, v, n, 0, bits, C.s), "locality: sort");
  GNN_CUDA_TRY(cudaMemcpyAsync(order, v.Current(), sizeof(int64_t) * n, cudaMemcpyDeviceToDevice, C.s),
               "locality: copy order");
  return GNN_OK;
}

// np.lexsort with the identity as least significant key. Keys are int64
// columns key_j[i] = src_j[i * stride_j + off_j] >= 0, listed least significant
// first, each ascending or descending. Result in `order` (n entries).
struct LexKey {
  const int64_t* src;
  int64_t stride, off;
  int bits;
  bool descending;
};

int lexsort(const Ctx& C, const std::vector<LexKey>& keys, int64_t n, int64_t* order) {
  if (n == 0) return GNN_OK;
  uint64_t* sa = C.at<uint64_t>(C.L.sa);
  uint64_t* sb = C.at<uint64_t>(C.L.sb);
  int64_t* pa = C.at<int64_t>(C.L.pa);
  int64_t* pb = C.at<int64_t>(C.L.pb);
  iota_kernel<<<grid_for(n), kThreads, 0, C.s>>>(pa, n);
  GNN_LAUNCH_CHECK("locality: iota");
  cub::DoubleBuffer<int64_t> v(pa, pb);
  for (const LexKey& k : keys) {
    cub::DoubleBuffer<uint64_t> kk(sa, sb);
    gather_key_kernel<<<grid_for(n), kThreads, 0, C.s>>>(k.src, k.stride, k.off, v.Current(), n, sa);
    GNN_LAUNCH_CHECK("locality: lexsort key");
    size_t tb = C.L.temp_bytes;
    if (k.descending) {
      GNN_CUDA_TRY(cub::DeviceRadixSort::SortPairsDescending(C.temp(), tb, kk, v, n, 0, k.bits, C.s),
                   "locality: lexsort pass");
    } else {
      GNN_CUDA_TRY(cub::DeviceRadixSort::SortPairs(C.temp(), tb, kk, v, n, 0, k.bits, C.s), "locality: lexsort pass");
    }
  }
  GNN_CUDA_TRY(cudaMemcpyAsync(order, v.Current(), sizeof(int64_t) * n, cudaMemcpyDeviceToDevice, C.s),
               "locality: copy order");
  return GNN_OK;
}

// Segment top-k over the e keys in ka (key = segment * num_items + item, with the
// item numbered in tie order). See the file comment. out_items[seg * k + pos]
// receives item_map[item] (or the item), out_counts the count; totals/covered
// (optional) accumulate every run's count / the chosen runs' counts per segment.
int segment_topk(const Ctx& C, int64_t e, uint64_t num_items, int key_bits, int64_t num_segments, int64_t k,
                 const int64_t* item_map, int64_t* out_items, int64_t* out_counts, unsigned long long* totals,
                 unsigned long long* covered) {
  if (e == 0) return GNN_OK;
  uint64_t* ka = C.at<uint64_t>(C.L.ka);
  uint64_t* kb = C.at<uint64_t>(C.L.kb);
  uint32_t* cnt = C.at<uint32_t>(C.L.c);
  uint32_t* item = C.at<uint32_t>(C.L.v);
  int64_t* d_runs = reinterpret_cast<int64_t*>(C.word(1));
  cub::DoubleBuffer<uint64_t> kk(ka, kb);
  size_t tb = C.L.temp_bytes;
  GNN_CUDA_TRY(cub::DeviceRadixSort::SortKeys(C.temp(), tb, kk, e, 0, key_bits, C.s), "locality: sort keys");
  uint64_t* sorted = kk.Current();
  uint64_t* uniq = kk.Alternate();
  tb = C.L.temp_bytes;
  GNN_CUDA_TRY(cub::DeviceRunLengthEncode::Encode(C.temp(), tb, sorted, uniq, cnt, d_runs, e, C.s),
               "locality: run-length");
  int64_t u = 0;
  int rc = read_back(C, &u, d_runs, sizeof(u), "locality: read runs");
  if (rc != GNN_OK) return rc;
  const int cbits = bits_for(static_cast<uint64_t>(e));
  const int sbits = bits_for(static_cast<uint64_t>(std::max<int64_t>(num_segments, 1)));
  if (cbits + sbits > 64) return fail(GNN_ERR_UNSUPPORTED, "locality: segment and count ids exceed 64 bits");
  // composite keys overwrite the sorted keys; items go to `item`
  composite_kernel<<<grid_for(u), kThreads, 0, C.s>>>(uniq, cnt, u, num_items, cbits, sorted, item);
  GNN_LAUNCH_CHECK("locality: composite keys");
  cub::DoubleBuffer<uint64_t> ck(sorted, uniq);
  cub::DoubleBuffer<uint32_t> cv(item, cnt);
  tb = C.L.temp_bytes;
  GNN_CUDA_TRY(cub::DeviceRadixSort::SortPairs(C.temp(), tb, ck, cv, u, 0, cbits + sbits, C.s),
               "locality: sort runs");
  int64_t* first = C.at<int64_t>(C.L.pa);  // free outside lexsort/argsort; num_segments <= num_nodes
  segment_heads_kernel<<<grid_for(u), kThreads, 0, C.s>>>(ck.Current(), u, cbits, num_segments, first);
  GNN_LAUNCH_CHECK("locality: segment heads");
  topk_extract_kernel<<<grid_for(u), kThreads, 0, C.s>>>(ck.Current(), cv.Current(), u, cbits, k, num_segments,
                                                         first, item_map, out_items, out_counts, totals, covered,
                                                         C.bad());
  GNN_LAUNCH_CHECK("locality: top-k");
  return GNN_OK;
}

template <class IdxT>
int check_csr(const Ctx& C, const IdxT* rp, const int32_t* col, int64_t n, int64_t e) {
  check_row_ptr_kernel<IdxT><<<grid_for(n + 1), kThreads, 0, C.s>>>(rp, n, e, C.bad());
  GNN_LAUNCH_CHECK("locality: check row_ptr");
  if (e > 0) {
    check_cols_kernel<<<grid_for(e), kThreads, 0, C.s>>>(col, e, n, C.bad());
    GNN_LAUNCH_CHECK("locality: check col_ind");
  }
  unsigned bad = 0;
  int rc = read_bad(C, &bad);
  if (rc != GNN_OK) return rc;
  if (bad & kBadRowPtr) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "row_ptr must start at 0, end at num_entries and never decrease");
  }
  if (bad & kBadCol) return fail(GNN_ERR_INVALID_ARGUMENT, "col_ind holds a column outside [0, num_nodes)");
  return GNN_OK;
}

int row_grid(int64_t n) {
  const int64_t warps = (n + (kThreads / 32) - 1) / (kThreads / 32);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(warps, 32LL * sm_count())));
}

template <class IdxT>
int page_schedule_typed(const Ctx& C, const IdxT* rp, const int32_t* col, int64_t n, int64_t e, int64_t rpp,
                        int64_t rbs, int64_t wnb, int64_t wcp, int64_t hcp, int64_t k, int64_t* page_hist,
                        int64_t* hot_pages, int64_t* row_schedule, int64_t* block_hot, int64_t* window_hot,
                        int64_t* max_page_count, double* hot_coverage, double* avg_window_cov) {
  int rc = check_csr<IdxT>(C, rp, col, n, e);
  if (rc != GNN_OK) return rc;
  const int64_t P = (n + rpp - 1) / rpp;
  const int64_t NB = (n + rbs - 1) / rbs;
  const int64_t rpw = rbs * wnb;
  const int64_t NW = (n + rpw - 1) / rpw;
  int64_t* hot_order = C.at<int64_t>(C.L.n0);
  int64_t* rank = C.at<int64_t>(C.L.n1);
  int64_t* degree = C.at<int64_t>(C.L.n2);
  int64_t* slot = C.at<int64_t>(C.L.n3);
  int64_t* sig = C.at<int64_t>(C.L.t0);
  unsigned long long* totals = C.at<unsigned long long>(C.L.t0);  // windows reuse t0/t1 after the signatures
  unsigned long long* covered = C.at<unsigned long long>(C.L.t1);

  // page histogram (graph_utils.py:269-272) and its maximum
  GNN_CUDA_TRY(cudaMemsetAsync(page_hist, 0, sizeof(int64_t) * P, C.s), "locality: clear page histogram");
  if (e > 0) {
    page_hist_kernel<<<grid_for(e), kThreads, 0, C.s>>>(col, e, rpp, reinterpret_cast<unsigned long long*>(page_hist));
    GNN_LAUNCH_CHECK("locality: page histogram");
  }
  max_kernel<<<grid_for(P), kThreads, 0, C.s>>>(page_hist, P, C.word(2));
  GNN_LAUNCH_CHECK("locality: max page count");
  // hot page order and ranks (:281-290)
  rc = argsort_desc(C, page_hist, P, bits_for(static_cast<uint64_t>(std::max<int64_t>(e, 1))), hot_order);
  if (rc != GNN_OK) return rc;
  rank_kernel<<<grid_for(P), kThreads, 0, C.s>>>(hot_order, P, rank);
  GNN_LAUNCH_CHECK("locality: page ranks");
  const int64_t nhot = std::max<int64_t>(0, std::min<int64_t>(hcp, P));
  if (nhot > 0) {
    GNN_CUDA_TRY(cudaMemcpyAsync(hot_pages, hot_order, sizeof(int64_t) * nhot, cudaMemcpyDeviceToDevice, C.s),
                 "locality: hot pages");
    gather_sum_kernel<<<grid_for(nhot), kThreads, 0, C.s>>>(page_hist, hot_order, nhot, C.word(3));
    GNN_LAUNCH_CHECK("locality: hot page accesses");
  }
  degree_kernel<IdxT><<<grid_for(n), kThreads, 0, C.s>>>(rp, n, degree);
  GNN_LAUNCH_CHECK("locality: degrees");

  // row signatures: each row's k pages by (entries desc, page rank asc), padded with P (:292-306)
  fill_kernel<<<grid_for(n * k), kThreads, 0, C.s>>>(sig, n * k, P);
  GNN_LAUNCH_CHECK("locality: fill signatures");
  const int page_bits = bits_for(static_cast<uint64_t>(P));
  if (e > 0) {
    entry_keys_kernel<IdxT, 0><<<row_grid(n), kThreads, 0, C.s>>>(rp, col, n, rpp, rank, nullptr, 1,
                                                                  static_cast<uint64_t>(P), C.at<uint64_t>(C.L.ka));
    GNN_LAUNCH_CHECK("locality: signature keys");
    rc = segment_topk(C, e, static_cast<uint64_t>(P), bits_for(static_cast<uint64_t>(n) * P), n, k, hot_order, sig,
                      nullptr, nullptr, nullptr);
    if (rc != GNN_OK) return rc;
  }
  // row schedule = lexsort((arange, -degree, sig[:, k-1], ..., sig[:, 0])) (:308-311)
  std::vector<LexKey> keys;
  keys.push_back({degree, 1, 0, bits_for(static_cast<uint64_t>(std::max<int64_t>(n, 1))), true});
  for (int64_t j = k - 1; j >= 0; --j) keys.push_back({sig, k, j, page_bits, false});
  rc = lexsort(C, keys, n, row_schedule);
  if (rc != GNN_OK) return rc;
  rank_kernel<<<grid_for(n), kThreads, 0, C.s>>>(row_schedule, n, slot);
  GNN_LAUNCH_CHECK("locality: schedule slots");

  // block hot pages: top k pages of each row_block_size scheduled rows (:313-334)
  fill_kernel<<<grid_for(NB * k), kThreads, 0, C.s>>>(block_hot, NB * k, P);
  GNN_LAUNCH_CHECK("locality: fill block pages");
  if (e > 0) {
    entry_keys_kernel<IdxT, 1><<<row_grid(n), kThreads, 0, C.s>>>(rp, col, n, rpp, rank, slot, rbs,
                                                                  static_cast<uint64_t>(P), C.at<uint64_t>(C.L.ka));
    GNN_LAUNCH_CHECK("locality: block keys");
    rc = segment_topk(C, e, static_cast<uint64_t>(P), bits_for(static_cast<uint64_t>(NB) * P), NB, k, hot_order,
                      block_hot, nullptr, nullptr, nullptr);
    if (rc != GNN_OK) return rc;
  }
  // window hot pages and per-window coverage (:336-356)
  fill_kernel<<<grid_for(NW * wcp), kThreads, 0, C.s>>>(window_hot, NW * wcp, P);
  GNN_LAUNCH_CHECK("locality: fill window pages");
  GNN_CUDA_TRY(cudaMemsetAsync(totals, 0, sizeof(unsigned long long) * NW, C.s), "locality: clear window totals");
  GNN_CUDA_TRY(cudaMemsetAsync(covered, 0, sizeof(unsigned long long) * NW, C.s), "locality: clear window totals");
  if (e > 0) {
    entry_keys_kernel<IdxT, 1><<<row_grid(n), kThreads, 0, C.s>>>(rp, col, n, rpp, rank, slot, rpw,
                                                                  static_cast<uint64_t>(P), C.at<uint64_t>(C.L.ka));
    GNN_LAUNCH_CHECK("locality: window keys");
    rc = segment_topk(C, e, static_cast<uint64_t>(P), bits_for(static_cast<uint64_t>(NW) * P), NW, wcp, hot_order,
                      window_hot, nullptr, totals, covered);
    if (rc != GNN_OK) return rc;
  }
  // host: scalars and the window-by-window float64 coverage sum
  std::vector<unsigned long long> tot(NW), cov(NW);
  unsigned long long words[4] = {0, 0, 0, 0};
  GNN_CUDA_TRY(cudaMemcpyAsync(tot.data(), totals, sizeof(unsigned long long) * NW, cudaMemcpyDeviceToHost, C.s),
               "locality: read window totals");
  GNN_CUDA_TRY(cudaMemcpyAsync(cov.data(), covered, sizeof(unsigned long long) * NW, cudaMemcpyDeviceToHost, C.s),
               "locality: read window coverage");
  GNN_CUDA_TRY(cudaMemcpyAsync(words, C.ws + C.L.words, sizeof(words), cudaMemcpyDeviceToHost, C.s),
               "locality: read counters");
  GNN_CUDA_TRY(cudaStreamSynchronize(C.s), "locality: synchronize");
  if (words[0] & (kBadId | kBadCol | kBadRowPtr)) return fail(GNN_ERR_INVALID_ARGUMENT, "locality: bad index data");
  double sum = 0.0;
  for (int64_t w = 0; w < NW; ++w) {
    if (tot[w] > 0) sum += static_cast<double>(cov[w]) / static_cast<double>(tot[w]);
  }
  *avg_window_cov = sum / static_cast<double>(std::max<int64_t>(1, NW));
  *max_page_count = static_cast<int64_t>(words[2]);
  *hot_coverage = (nhot > 0 && e > 0) ? static_cast<double>(words[3]) / static_cast<double>(e) : 0.0;
  return GNN_OK;
}

template <class IdxT>
int coaccess_typed(const Ctx& C, const IdxT* rp, const int32_t* col, int64_t n, int64_t e,
                   const int64_t* row_schedule, int64_t rpw, int64_t k, int64_t* perm, int64_t* inv_perm) {
  int rc = check_csr<IdxT>(C, rp, col, n, e);
  if (rc != GNN_OK) return rc;
  // the schedule must be a permutation: slots index it
  unsigned* seen = C.at<unsigned>(C.L.n0);
  GNN_CUDA_TRY(cudaMemsetAsync(seen, 0, sizeof(unsigned) * n, C.s), "locality: clear seen");
  check_perm_kernel<<<grid_for(n), kThreads, 0, C.s>>>(row_schedule, n, seen, C.bad());
  GNN_LAUNCH_CHECK("locality: check schedule");
  unsigned bad = 0;
  rc = read_bad(C, &bad);
  if (rc != GNN_OK) return rc;
  if (bad & kNotPerm) return fail(GNN_ERR_INVALID_ARGUMENT, "row_schedule must be a permutation of [0, num_nodes)");
  const int64_t NW = (n + rpw - 1) / rpw;
  int64_t* slot = C.at<int64_t>(C.L.n1);
  int64_t* access = C.at<int64_t>(C.L.n2);
  int64_t* top_w = C.at<int64_t>(C.L.t0);
  int64_t* top_c = C.at<int64_t>(C.L.t1);
  rank_kernel<<<grid_for(n), kThreads, 0, C.s>>>(row_schedule, n, slot);
  GNN_LAUNCH_CHECK("locality: schedule slots");
  GNN_CUDA_TRY(cudaMemsetAsync(access, 0, sizeof(int64_t) * n, C.s), "locality: clear access counts");
  fill_kernel<<<grid_for(n * k), kThreads, 0, C.s>>>(top_w, n * k, NW);
  GNN_LAUNCH_CHECK("locality: fill windows");
  GNN_CUDA_TRY(cudaMemsetAsync(top_c, 0, sizeof(int64_t) * n * k, C.s), "locality: clear window counts");
  if (e > 0) {
    col_access_kernel<<<grid_for(e), kThreads, 0, C.s>>>(col, e, reinterpret_cast<unsigned long long*>(access));
    GNN_LAUNCH_CHECK("locality: access counts");
    // per node: the k windows reading it most, ties by smaller window (graph_utils.py:400-425)
    entry_keys_kernel<IdxT, 2><<<row_grid(n), kThreads, 0, C.s>>>(rp, col, n, 1, nullptr, slot, rpw,
                                                                  static_cast<uint64_t>(NW), C.at<uint64_t>(C.L.ka));
    GNN_LAUNCH_CHECK("locality: node window keys");
    rc = segment_topk(C, e, static_cast<uint64_t>(NW), bits_for(static_cast<uint64_t>(n) * NW), n, k, nullptr, top_w,
                      top_c, nullptr, nullptr);
    if (rc != GNN_OK) return rc;
  }
  // perm = lexsort((arange, -access, -top_c[:, k-1], top_w[:, k-1], ..., -top_c[:, 0], top_w[:, 0])) (:427-432)
  const int cbits = bits_for(static_cast<uint64_t>(std::max<int64_t>(e, 1)));
  const int wbits = bits_for(static_cast<uint64_t>(NW));
  std::vector<LexKey> keys;
  keys.push_back({access, 1, 0, cbits, true});
  for (int64_t j = k - 1; j >= 0; --j) {
    keys.push_back({top_c, k, j, cbits, true});
    keys.push_back({top_w, k, j, wbits, false});
  }
  rc = lexsort(C, keys, n, perm);
  if (rc != GNN_OK) return rc;
  invert_kernel<<<grid_for(n), kThreads, 0, C.s>>>(perm, inv_perm, n);
  GNN_LAUNCH_CHECK("locality: inverse order");
  rc = read_bad(C, &bad);
  if (rc != GNN_OK) return rc;
  if (bad) return fail(GNN_ERR_INVALID_ARGUMENT, "locality: bad index data");
  return GNN_OK;
}

int check_layout(int64_t n, int64_t e, int64_t max_k, void* workspace, size_t workspace_bytes, Layout* L) {
  int rc = plan_layout(n, e, max_k, L);
  if (rc != GNN_OK) return rc;
  if (workspace == nullptr || workspace_bytes < L->total) {
    return fail(GNN_ERR_WORKSPACE, "locality: workspace missing or smaller than gnn_locality_workspace_bytes()");
  }
  return GNN_OK;
}

}  // namespace
}  // namespace gnnb200

using namespace gnnb200;

extern "C" size_t gnn_locality_workspace_bytes(int64_t num_nodes, int64_t num_entries, int64_t max_k) {
  if (num_nodes < 0 || num_entries < 0 || max_k < 0 || max_k > kMaxTopK) return 0;
  Layout L{};
  if (plan_layout(num_nodes, num_entries, max_k, &L) != GNN_OK) return 0;
  clear_error();
  return L.total;
}

extern "C" int gnn_locality_page_schedule(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                          int64_t num_nodes, int64_t num_entries, int64_t rows_per_page,
                                          int64_t row_block_size, int64_t window_num_blocks,
                                          int64_t window_cache_pages, int64_t hot_cache_pages, int64_t signature_topk,
                                          int64_t* page_histogram, int64_t* hot_pages, int64_t* row_schedule,
                                          int64_t* block_hot_pages, int64_t* window_hot_pages,
                                          int64_t* max_page_count, double* hot_coverage,
                                          double* avg_window_hot_coverage, void* workspace, size_t workspace_bytes,
                                          gnn_stream_t stream) {
  GNN_REQUIRE(num_nodes >= 1 && num_nodes <= INT32_MAX, GNN_ERR_INVALID_ARGUMENT,
              "num_nodes must be in [1, 2^31 - 1]");
  GNN_REQUIRE(num_entries >= 0 && num_entries < (int64_t(1) << 32), GNN_ERR_INVALID_ARGUMENT,
              "num_entries must be in [0, 2^32)");
  GNN_REQUIRE(rows_per_page >= 1 && row_block_size >= 1 && window_num_blocks >= 1, GNN_ERR_INVALID_ARGUMENT,
              "rows_per_page, row_block_size and window_num_blocks must be >= 1");
  GNN_REQUIRE(signature_topk >= 1 && signature_topk <= kMaxTopK && window_cache_pages >= 1 &&
                  window_cache_pages <= kMaxTopK,
              GNN_ERR_INVALID_ARGUMENT, "signature_topk and window_cache_pages must be in [1, 4096]");
  GNN_REQUIRE(row_ptr_type == GNN_INDEX_INT32 || row_ptr_type == GNN_INDEX_INT64, GNN_ERR_INVALID_ARGUMENT,
              "row_ptr must be int32 or int64");
  GNN_REQUIRE(row_ptr && page_histogram && row_schedule && block_hot_pages && window_hot_pages && max_page_count &&
                  hot_coverage && avg_window_hot_coverage && (num_entries == 0 || col_ind) &&
                  (hot_cache_pages <= 0 || hot_pages),
              GNN_ERR_NULL_POINTER, "locality: a required pointer is NULL");
  Layout L{};
  int rc = check_layout(num_nodes, num_entries, std::max(signature_topk, window_cache_pages), workspace,
                        workspace_bytes, &L);
  if (rc != GNN_OK) return rc;
  Ctx C{static_cast<char*>(workspace), L, reinterpret_cast<cudaStream_t>(stream)};
  rc = reset_words(C);
  if (rc != GNN_OK) return rc;
  if (row_ptr_type == GNN_INDEX_INT64) {
    rc = page_schedule_typed<int64_t>(C, static_cast<const int64_t*>(row_ptr), col_ind, num_nodes, num_entries,
                                      rows_per_page, row_block_size, window_num_blocks, window_cache_pages,
                                      hot_cache_pages, signature_topk, page_histogram, hot_pages, row_schedule,
                                      block_hot_pages, window_hot_pages, max_page_count, hot_coverage,
                                      avg_window_hot_coverage);
  } else {
    rc = page_schedule_typed<int32_t>(C, static_cast<const int32_t*>(row_ptr), col_ind, num_nodes, num_entries,
                                      rows_per_page, row_block_size, window_num_blocks, window_cache_pages,
                                      hot_cache_pages, signature_topk, page_histogram, hot_pages, row_schedule,
                                      block_hot_pages, window_hot_pages, max_page_count, hot_coverage,
                                      avg_window_hot_coverage);
  }
  if (rc == GNN_OK) clear_error();
  return rc;
}

extern "C" int gnn_locality_count_histogram(const int64_t* values, int64_t count, int64_t* hist, int64_t hist_len,
                                            gnn_stream_t stream) {
  GNN_REQUIRE(count >= 0 && hist_len >= 1, GNN_ERR_INVALID_ARGUMENT, "count must be >= 0 and hist_len >= 1");
  GNN_REQUIRE(hist != nullptr && (count == 0 || values != nullptr), GNN_ERR_NULL_POINTER,
              "values and hist must not be NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  GNN_CUDA_TRY(cudaMemsetAsync(hist, 0, sizeof(int64_t) * hist_len, s), "count histogram: clear");
  if (count > 0) {
    count_hist_kernel<<<grid_for(count), kThreads, 0, s>>>(values, count, hist_len,
                                                           reinterpret_cast<unsigned long long*>(hist));
    GNN_LAUNCH_CHECK("count histogram");
  }
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_locality_coaccess_permutation(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                                 int64_t num_nodes, int64_t num_entries, const int64_t* row_schedule,
                                                 int64_t rows_per_window, int64_t signature_topk, int64_t* perm,
                                                 int64_t* inv_perm, void* workspace, size_t workspace_bytes,
                                                 gnn_stream_t stream) {
  GNN_REQUIRE(num_nodes >= 1 && num_nodes <= INT32_MAX, GNN_ERR_INVALID_ARGUMENT,
              "num_nodes must be in [1, 2^31 - 1]");
  GNN_REQUIRE(num_entries >= 0 && num_entries < (int64_t(1) << 32), GNN_ERR_INVALID_ARGUMENT,
              "num_entries must be in [0, 2^32)");
  GNN_REQUIRE(rows_per_window >= 1, GNN_ERR_INVALID_ARGUMENT, "rows_per_window must be >= 1");
  GNN_REQUIRE(signature_topk >= 1 && signature_topk <= kMaxTopK, GNN_ERR_INVALID_ARGUMENT,
              "signature_topk must be in [1, 4096]");
  GNN_REQUIRE(row_ptr_type == GNN_INDEX_INT32 || row_ptr_type == GNN_INDEX_INT64, GNN_ERR_INVALID_ARGUMENT,
              "row_ptr must be int32 or int64");
  GNN_REQUIRE(row_ptr && row_schedule && perm && inv_perm && (num_entries == 0 || col_ind), GNN_ERR_NULL_POINTER,
              "locality: a required pointer is NULL");
  Layout L{};
  int rc = check_layout(num_nodes, num_entries, signature_topk, workspace, workspace_bytes, &L);
  if (rc != GNN_OK) return rc;
  Ctx C{static_cast<char*>(workspace), L, reinterpret_cast<cudaStream_t>(stream)};
  rc = reset_words(C);
  if (rc != GNN_OK) return rc;
  if (row_ptr_type == GNN_INDEX_INT64) {
    rc = coaccess_typed<int64_t>(C, static_cast<const int64_t*>(row_ptr), col_ind, num_nodes, num_entries,
                                 row_schedule, rows_per_window, signature_topk, perm, inv_perm);
  } else {
    rc = coaccess_typed<int32_t>(C, static_cast<const int32_t*>(row_ptr), col_ind, num_nodes, num_entries,
                                 row_schedule, rows_per_window, signature_topk, perm, inv_perm);
  }
  if (rc == GNN_OK) clear_error();
  return rc;
}

extern "C" int gnn_locality_hot_partition(const int64_t* src, int64_t num_entries, int64_t num_nodes,
                                          int add_self_loops, const int64_t* base_order, double hot_access_coverage,
                                          double hot_max_ratio, int64_t hot_min_nodes, int64_t* access_count,
                                          int64_t* sorted_nodes, int64_t* perm, int64_t* inv_perm,
                                          int64_t* hot_node_cutoff, int64_t* min_nodes_used, int64_t* total_access,
                                          int64_t* hot_access, void* workspace, size_t workspace_bytes,
                                          gnn_stream_t stream) {
  GNN_REQUIRE(num_nodes >= 1, GNN_ERR_INVALID_ARGUMENT, "num_nodes must be >= 1");
  GNN_REQUIRE(num_entries >= 0, GNN_ERR_INVALID_ARGUMENT, "num_entries must be >= 0");
  GNN_REQUIRE(access_count && sorted_nodes && perm && inv_perm && hot_node_cutoff && min_nodes_used &&
                  total_access && hot_access && (num_entries == 0 || src),
              GNN_ERR_NULL_POINTER, "locality: a required pointer is NULL");
  Layout L{};
  int rc = check_layout(num_nodes, 0, 1, workspace, workspace_bytes, &L);
  if (rc != GNN_OK) return rc;
  Ctx C{static_cast<char*>(workspace), L, reinterpret_cast<cudaStream_t>(stream)};
  rc = reset_words(C);
  if (rc != GNN_OK) return rc;
  const int64_t n = num_nodes;
  // access counts (graph_utils.py:184-187)
  fill_kernel<<<grid_for(n), kThreads, 0, C.s>>>(access_count, n, add_self_loops ? 1 : 0);
  GNN_LAUNCH_CHECK("hot partition: fill");
  if (num_entries > 0) {
    access_count_kernel<<<grid_for(num_entries), kThreads, 0, C.s>>>(
        src, num_entries, n, reinterpret_cast<unsigned long long*>(access_count), C.bad());
    GNN_LAUNCH_CHECK("hot partition: access counts");
  }
  if (base_order != nullptr) {
    unsigned* seen = C.at<unsigned>(C.L.n3);
    GNN_CUDA_TRY(cudaMemsetAsync(seen, 0, sizeof(unsigned) * n, C.s), "hot partition: clear seen");
    check_perm_kernel<<<grid_for(n), kThreads, 0, C.s>>>(base_order, n, seen, C.bad());
    GNN_LAUNCH_CHECK("hot partition: check base order");
  }
  unsigned bad = 0;
  rc = read_bad(C, &bad);
  if (rc != GNN_OK) return rc;
  if (bad & kBadId) return fail(GNN_ERR_INVALID_ARGUMENT, "src holds a node id outside [0, num_nodes)");
  if (bad & kNotPerm) return fail(GNN_ERR_INVALID_ARGUMENT, "base_order must be a permutation of [0, num_nodes)");
  const int64_t total = num_entries + (add_self_loops ? n : 0);
  // sorted_nodes = argsort(access, descending, stable) (:188)
  rc = argsort_desc(C, access_count, n, bits_for(static_cast<uint64_t>(std::max<int64_t>(total, 1))), sorted_nodes);
  if (rc != GNN_OK) return rc;
  // cutoff (:191-207), host arithmetic in float64 as numpy does it
  const double cov = std::max(0.0, std::min(1.0, hot_access_coverage));
  const int64_t max_nodes =
      hot_max_ratio <= 0.0 ? n : std::max<int64_t>(1, std::min<int64_t>(n, static_cast<int64_t>(std::ceil(hot_max_ratio * static_cast<double>(n)))));
  int64_t min_nodes = std::max<int64_t>(0, std::min<int64_t>(hot_min_nodes, n));
  min_nodes = std::min(min_nodes, max_nodes);
  int64_t cutoff = min_nodes;
  uint64_t* prefix = C.at<uint64_t>(C.L.sa);
  uint64_t* scanned = C.at<uint64_t>(C.L.sb);
  gather_u64_kernel<<<grid_for(n), kThreads, 0, C.s>>>(access_count, sorted_nodes, n, prefix);
  GNN_LAUNCH_CHECK("hot partition: gather counts");
  size_t tb = L.temp_bytes;
  GNN_CUDA_TRY(cub::DeviceScan::InclusiveSum(C.temp(), tb, prefix, scanned, n, C.s), "hot partition: prefix sum");
  if (total > 0 && cov > 0.0) {
    const uint64_t target = static_cast<uint64_t>(std::ceil(static_cast<double>(total) * cov));
    int64_t* d_lb = reinterpret_cast<int64_t*>(C.word(4));
    lower_bound_kernel<<<1, 32, 0, C.s>>>(scanned, n, target, d_lb);
    GNN_LAUNCH_CHECK("hot partition: search");
    int64_t lb = 0;
    rc = read_back(C, &lb, d_lb, sizeof(lb), "hot partition: read search");
    if (rc != GNN_OK) return rc;
    cutoff = std::max(cutoff, lb + 1);
  } else if (total > 0) {
    cutoff = std::max<int64_t>(cutoff, 1);
  }
  cutoff = std::max(min_nodes, std::min({n, cutoff, max_nodes}));
  uint64_t hot_sum = 0;
  if (cutoff > 0) {
    rc = read_back(C, &hot_sum, scanned + (cutoff - 1), sizeof(hot_sum), "hot partition: read hot accesses");
    if (rc != GNN_OK) return rc;
  }
  // perm: hot prefix of base_order then its cold suffix, or the sorted order (:209-226)
  if (base_order == nullptr) {
    GNN_CUDA_TRY(cudaMemcpyAsync(perm, sorted_nodes, sizeof(int64_t) * n, cudaMemcpyDeviceToDevice, C.s),
                 "hot partition: copy order");
  } else {
    int64_t* hot = C.at<int64_t>(C.L.n0);
    int64_t* flags = C.at<int64_t>(C.L.n1);
    int64_t* excl = C.at<int64_t>(C.L.n2);
    hot_mask_kernel<<<grid_for(n), kThreads, 0, C.s>>>(sorted_nodes, n, cutoff, hot);
    GNN_LAUNCH_CHECK("hot partition: mask");
    base_flags_kernel<<<grid_for(n), kThreads, 0, C.s>>>(base_order, hot, n, flags);
    GNN_LAUNCH_CHECK("hot partition: flags");
    tb = L.temp_bytes;
    GNN_CUDA_TRY(cub::DeviceScan::ExclusiveSum(C.temp(), tb, flags, excl, n, C.s), "hot partition: scan");
    partition_scatter_kernel<<<grid_for(n), kThreads, 0, C.s>>>(base_order, flags, excl, n, cutoff, perm);
    GNN_LAUNCH_CHECK("hot partition: scatter");
  }
  invert_kernel<<<grid_for(n), kThreads, 0, C.s>>>(perm, inv_perm, n);
  GNN_LAUNCH_CHECK("hot partition: inverse order");
  GNN_CUDA_TRY(cudaStreamSynchronize(C.s), "hot partition: synchronize");
  *hot_node_cutoff = cutoff;
  *min_nodes_used = min_nodes;
  *total_access = total;
  *hot_access = static_cast<int64_t>(hot_sum);
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_permute_edges(const int64_t* src, const int64_t* dst, int64_t num_entries, const int64_t* inv_perm,
                                 int64_t num_nodes, int64_t* src_out, int64_t* dst_out, void* workspace,
                                 size_t workspace_bytes, gnn_stream_t stream) {
  GNN_REQUIRE(num_entries >= 0 && num_nodes >= 1, GNN_ERR_INVALID_ARGUMENT,
              "num_entries must be >= 0 and num_nodes >= 1");
  if (num_entries == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(src && dst && inv_perm && src_out && dst_out, GNN_ERR_NULL_POINTER,
              "permute edges: a required pointer is NULL");
  GNN_REQUIRE(workspace != nullptr && workspace_bytes >= 256, GNN_ERR_WORKSPACE,
              "permute edges: workspace must hold at least 256 bytes");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned* d_bad = static_cast<unsigned*>(workspace);
  GNN_CUDA_TRY(cudaMemsetAsync(d_bad, 0, sizeof(unsigned), s), "permute edges: clear flag");
  permute_edges_kernel<<<grid_for(num_entries), kThreads, 0, s>>>(src, dst, num_entries, inv_perm, num_nodes, src_out,
                                                                   dst_out, d_bad);
  GNN_LAUNCH_CHECK("permute edges");
  unsigned bad = 0;
  GNN_CUDA_TRY(cudaMemcpyAsync(&bad, d_bad, sizeof(bad), cudaMemcpyDeviceToHost, s), "permute edges: read flag");
  GNN_CUDA_TRY(cudaStreamSynchronize(s), "permute edges: synchronize");
  if (bad) return fail(GNN_ERR_INVALID_ARGUMENT, "edge list holds a node id outside [0, num_nodes)");
  clear_error();
  return GNN_OK;
}
