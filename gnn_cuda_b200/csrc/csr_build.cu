// Device CSR builder: the aggregation kernels' input, built on the GPU.
//
// Restates the reference's host builders (GNN_cuda_common/graph_utils.py:449-535:
// build_gcn_normalized_csr, build_pyg_gcn_weighted_csr, build_plain_csr). There,
// scipy's coo_matrix(...).tocsr() + sort_indices() turn (row, col) pairs into a
// CSR whose rows hold their distinct columns in increasing order (duplicate
// pairs merge), and deg_inv_sqrt = clip(deg, 1)^-0.5 is numpy's float32 power.
// Here the same CSR comes out of one radix sort of 64-bit (row << colbits | col)
// keys (CUB, only the bits the ids occupy), a unique pass, a lower-bound
// search per row for row_ptr and a mask for col_ind — the same arrays bit for
// bit. deg_inv_sqrt is a lookup into a table of numpy's float32 values that the
// caller computes on the host for 0..max_degree, so it matches bit for bit too;
// PyG edge weights are the float32 product dis[row] * dis[col].
#include <cuda_runtime.h>
#include <stdint.h>

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_select.cuh>

#include <algorithm>
#include <string>

#include "common.cuh"

namespace gnnb200 {
namespace {

constexpr int kThreads = 256;
// device word flags set by the key packer for ids outside [0, num_nodes)
constexpr unsigned kNegRow = 1u, kNegCol = 2u, kBigRow = 4u, kBigCol = 8u;

int id_bits(int64_t n) {
  int b = 1;
  while (b < 62 && (int64_t(1) << b) < n) ++b;
  return b;
}

int grid_for(int64_t items) {
  const int64_t want = (items + kThreads - 1) / kThreads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 16LL * sm_count())));
}

__global__ void pack_keys_kernel(const int64_t* __restrict__ rows, const int64_t* __restrict__ cols,
                                 int64_t e, int64_t n, int loops, int colbits, uint64_t* __restrict__ keys,
                                 unsigned* __restrict__ bad) {
  const int64_t total = e + (loops ? n : 0);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  unsigned flags = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t r, c;
    if (i < e) {
      r = rows[i];
      c = cols[i];
    } else {
      r = c = i - e;  // self-loop of node i - e
    }
    unsigned f = 0;
    if (r < 0) f |= kNegRow;
    if (c < 0) f |= kNegCol;
    if (r >= n) f |= kBigRow;
    if (c >= n) f |= kBigCol;
    if (f) {
      flags |= f;
      r = 0;
      c = 0;
    }
    keys[i] = (static_cast<uint64_t>(r) << colbits) | static_cast<uint64_t>(c);
  }
  if (flags) atomicOr(bad, flags);
}

// row_ptr[q] = first unique key whose row is >= q; col_ind[i] = column of key i.
template <class IdxT>
__global__ void segments_kernel(const uint64_t* __restrict__ ukeys, int64_t nu, int64_t n, int colbits,
                                IdxT* __restrict__ row_ptr, int32_t* __restrict__ col) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const uint64_t mask = (uint64_t(1) << colbits) - 1;
  const int64_t span = std::max<int64_t>(nu, n + 1);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < span; i += stride) {
    if (i < nu) col[i] = static_cast<int32_t>(ukeys[i] & mask);
    if (i <= n) {
      const uint64_t target = static_cast<uint64_t>(i) << colbits;
      int64_t lo = 0, hi = nu;
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (ukeys[mid] < target) lo = mid + 1;
        else hi = mid;
      }
      row_ptr[i] = static_cast<IdxT>(lo);
    }
  }
}

template <class IdxT>
__global__ void max_degree_kernel(const IdxT* __restrict__ row_ptr, int64_t n,
                                  unsigned long long* __restrict__ max_deg) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  unsigned long long m = 0;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < n; q += stride) {
    m = max(m, static_cast<unsigned long long>(row_ptr[q + 1] - row_ptr[q]));
  }
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m) atomicMax(max_deg, m);
}

template <class IdxT>
__global__ void dis_kernel(const IdxT* __restrict__ row_ptr, int64_t n, const float* __restrict__ table,
                           int64_t table_len, float* __restrict__ dis) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < n; q += stride) {
    const int64_t deg = static_cast<int64_t>(row_ptr[q + 1] - row_ptr[q]);
    dis[q] = table[std::min<int64_t>(deg, table_len - 1)];
  }
}

// One warp per row: edge_weight[e] = dis[row] * dis[col_ind[e]] (one float32 rounding).
template <class IdxT>
__global__ void edge_weight_kernel(const IdxT* __restrict__ row_ptr, const int32_t* __restrict__ col,
                                   const float* __restrict__ dis, int64_t n, float* __restrict__ ew) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += warps) {
    const float dr = dis[r];
    for (int64_t e = static_cast<int64_t>(row_ptr[r]) + lane; e < static_cast<int64_t>(row_ptr[r + 1]); e += 32) {
      ew[e] = __fmul_rn(dr, dis[col[e]]);
    }
  }
}

struct BuildLayout {
  size_t keys_a, keys_b, words, temp, total;
  size_t temp_bytes;
};

size_t a256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

int build_layout(int64_t cap, int bits, BuildLayout* out) {
  size_t sort_bytes = 0, uniq_bytes = 0;
  cub::DoubleBuffer<uint64_t> db(nullptr, nullptr);
  GNN_CUDA_TRY(cub::DeviceRadixSort::SortKeys(nullptr, sort_bytes, db, cap, 0, bits), "cub sort size query");
  GNN_CUDA_TRY(cub::DeviceSelect::Unique(nullptr, uniq_bytes, static_cast<const uint64_t*>(nullptr),
                                         static_cast<uint64_t*>(nullptr), static_cast<int64_t*>(nullptr), cap),
               "cub unique size query");
  BuildLayout L{};
  L.keys_a = 0;
  L.keys_b = a256(static_cast<size_t>(cap) * sizeof(uint64_t));
  L.words = L.keys_b + a256(static_cast<size_t>(cap) * sizeof(uint64_t));
  L.temp = L.words + 256;
  L.temp_bytes = std::max(sort_bytes, uniq_bytes);
  L.total = L.temp + a256(L.temp_bytes);
  *out = L;
  return GNN_OK;
}

template <class IdxT>
int build_typed(const int64_t* rows, const int64_t* cols, int64_t e, int64_t n, int loops, IdxT* row_ptr,
                int32_t* col_ind, int64_t col_capacity, int64_t* num_unique, int64_t* max_degree, char* ws,
                const BuildLayout& L, int bits, int colbits, cudaStream_t stream) {
  const int64_t cap = e + (loops ? n : 0);
  uint64_t* keys_a = reinterpret_cast<uint64_t*>(ws + L.keys_a);
  uint64_t* keys_b = reinterpret_cast<uint64_t*>(ws + L.keys_b);
  int64_t* d_nu = reinterpret_cast<int64_t*>(ws + L.words);
  unsigned long long* d_maxdeg = reinterpret_cast<unsigned long long*>(ws + L.words + 8);
  unsigned* d_bad = reinterpret_cast<unsigned*>(ws + L.words + 16);
  GNN_CUDA_TRY(cudaMemsetAsync(ws + L.words, 0, 256, stream), "csr build: reset counters");
  int64_t nu = 0;
  const uint64_t* ukeys = keys_a;
  if (cap > 0) {
    pack_keys_kernel<<<grid_for(cap), kThreads, 0, stream>>>(rows, cols, e, n, loops, colbits, keys_a, d_bad);
    GNN_LAUNCH_CHECK("csr build: pack keys");
    cub::DoubleBuffer<uint64_t> db(keys_a, keys_b);
    size_t tb = L.temp_bytes;
    GNN_CUDA_TRY(cub::DeviceRadixSort::SortKeys(ws + L.temp, tb, db, cap, 0, bits, stream), "csr build: sort");
    uint64_t* uniq = db.Current() == keys_a ? keys_b : keys_a;
    tb = L.temp_bytes;
    GNN_CUDA_TRY(cub::DeviceSelect::Unique(ws + L.temp, tb, db.Current(), uniq, d_nu, cap, stream),
                 "csr build: unique");
    ukeys = uniq;
    unsigned bad = 0;
    GNN_CUDA_TRY(cudaMemcpyAsync(&nu, d_nu, sizeof(nu), cudaMemcpyDeviceToHost, stream), "csr build: read count");
    GNN_CUDA_TRY(cudaMemcpyAsync(&bad, d_bad, sizeof(bad), cudaMemcpyDeviceToHost, stream), "csr build: read flags");
    GNN_CUDA_TRY(cudaStreamSynchronize(stream), "csr build: synchronize");
    // the host builder's checks, in its order
    if (bad & kNegRow) return fail(GNN_ERR_INVALID_ARGUMENT, "negative row index found");
    if (bad & kNegCol) return fail(GNN_ERR_INVALID_ARGUMENT, "negative column index found");
    if (bad & kBigRow) return fail(GNN_ERR_INVALID_ARGUMENT, "row index exceeds matrix dimensions");
    if (bad & kBigCol) return fail(GNN_ERR_INVALID_ARGUMENT, "column index exceeds matrix dimensions");
  }
  *num_unique = nu;
  if (sizeof(IdxT) == 4 && nu > INT32_MAX) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "row_ptr exceeds int32 range; use an int64 row_ptr");
  }
  if (nu > col_capacity) {
    return fail(GNN_ERR_INVALID_ARGUMENT, "col_ind holds " + std::to_string(col_capacity) + " entries but the CSR has " +
                                              std::to_string(nu));
  }
  segments_kernel<IdxT><<<grid_for(std::max<int64_t>(nu, n + 1)), kThreads, 0, stream>>>(ukeys, nu, n, colbits,
                                                                                        row_ptr, col_ind);
  GNN_LAUNCH_CHECK("csr build: segments");
  if (n > 0) {
    max_degree_kernel<IdxT><<<grid_for(n), kThreads, 0, stream>>>(row_ptr, n, d_maxdeg);
    GNN_LAUNCH_CHECK("csr build: max degree");
  }
  unsigned long long md = 0;
  GNN_CUDA_TRY(cudaMemcpyAsync(&md, d_maxdeg, sizeof(md), cudaMemcpyDeviceToHost, stream), "csr build: read degree");
  GNN_CUDA_TRY(cudaStreamSynchronize(stream), "csr build: synchronize");
  *max_degree = static_cast<int64_t>(md);
  return GNN_OK;
}

}  // namespace
}  // namespace gnnb200

using namespace gnnb200;

extern "C" size_t gnn_csr_build_workspace_bytes(int64_t num_entries, int64_t num_nodes, int add_self_loops) {
  if (num_entries < 0 || num_nodes < 0) return 0;
  const int64_t cap = num_entries + (add_self_loops ? num_nodes : 0);
  BuildLayout L{};
  if (build_layout(std::max<int64_t>(cap, 1), 2 * id_bits(std::max<int64_t>(num_nodes, 1)), &L) != GNN_OK) {
    return 0;
  }
  clear_error();
  return L.total;
}

extern "C" int gnn_csr_build(const int64_t* row_ids, const int64_t* col_ids, int64_t num_entries,
                             int64_t num_nodes, int add_self_loops, void* row_ptr, int row_ptr_type,
                             int32_t* col_ind, int64_t col_capacity, int64_t* num_unique, int64_t* max_degree,
                             void* workspace, size_t workspace_bytes, gnn_stream_t stream) {
  GNN_REQUIRE(num_entries >= 0 && num_nodes >= 0, GNN_ERR_INVALID_ARGUMENT, "num_entries and num_nodes must be >= 0");
  GNN_REQUIRE(num_nodes <= INT32_MAX, GNN_ERR_INVALID_ARGUMENT, "num_nodes must fit int32 column ids");
  GNN_REQUIRE(row_ptr_type == GNN_INDEX_INT32 || row_ptr_type == GNN_INDEX_INT64, GNN_ERR_INVALID_ARGUMENT,
              "row_ptr must be int32 or int64");
  GNN_REQUIRE(num_unique != nullptr && max_degree != nullptr, GNN_ERR_NULL_POINTER,
              "num_unique and max_degree must not be NULL");
  GNN_REQUIRE(row_ptr != nullptr, GNN_ERR_NULL_POINTER, "row_ptr must not be NULL");
  if (num_entries > 0) {
    GNN_REQUIRE(row_ids != nullptr && col_ids != nullptr, GNN_ERR_NULL_POINTER, "row and column ids must not be NULL");
  }
  const int64_t cap = num_entries + (add_self_loops ? num_nodes : 0);
  if (cap > 0) GNN_REQUIRE(col_ind != nullptr, GNN_ERR_NULL_POINTER, "col_ind must not be NULL");
  const int colbits = id_bits(std::max<int64_t>(num_nodes, 1));
  BuildLayout L{};
  int rc = build_layout(std::max<int64_t>(cap, 1), 2 * colbits, &L);
  if (rc != GNN_OK) return rc;
  if (workspace == nullptr || workspace_bytes < L.total) {
    return fail(GNN_ERR_WORKSPACE, "csr build: workspace missing or smaller than gnn_csr_build_workspace_bytes()");
  }
  *num_unique = 0;
  *max_degree = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  if (row_ptr_type == GNN_INDEX_INT64) {
    rc = build_typed<int64_t>(row_ids, col_ids, num_entries, num_nodes, add_self_loops, static_cast<int64_t*>(row_ptr),
                              col_ind, col_capacity, num_unique, max_degree, ws, L, 2 * colbits, colbits, s);
  } else {
    rc = build_typed<int32_t>(row_ids, col_ids, num_entries, num_nodes, add_self_loops, static_cast<int32_t*>(row_ptr),
                              col_ind, col_capacity, num_unique, max_degree, ws, L, 2 * colbits, colbits, s);
  }
  if (rc == GNN_OK) clear_error();
  return rc;
}

extern "C" int gnn_csr_deg_inv_sqrt(const void* row_ptr, int row_ptr_type, int64_t num_nodes, const float* table,
                                    int64_t table_len, float* deg_inv_sqrt, gnn_stream_t stream) {
  GNN_REQUIRE(num_nodes >= 0, GNN_ERR_INVALID_ARGUMENT, "num_nodes must be >= 0");
  if (num_nodes == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(row_ptr != nullptr && table != nullptr && deg_inv_sqrt != nullptr, GNN_ERR_NULL_POINTER,
              "row_ptr, table and deg_inv_sqrt must not be NULL");
  GNN_REQUIRE(table_len >= 2, GNN_ERR_INVALID_ARGUMENT, "table must cover degrees 0..max_degree (at least 2 entries)");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (row_ptr_type == GNN_INDEX_INT64) {
    dis_kernel<int64_t><<<grid_for(num_nodes), kThreads, 0, s>>>(static_cast<const int64_t*>(row_ptr), num_nodes,
                                                                 table, table_len, deg_inv_sqrt);
  } else {
    dis_kernel<int32_t><<<grid_for(num_nodes), kThreads, 0, s>>>(static_cast<const int32_t*>(row_ptr), num_nodes,
                                                                 table, table_len, deg_inv_sqrt);
  }
  GNN_LAUNCH_CHECK("csr deg_inv_sqrt");
  clear_error();
  return GNN_OK;
}

extern "C" int gnn_csr_edge_weight(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                   const float* deg_inv_sqrt, int64_t num_nodes, float* edge_weight,
                                   gnn_stream_t stream) {
  GNN_REQUIRE(num_nodes >= 0, GNN_ERR_INVALID_ARGUMENT, "num_nodes must be >= 0");
  if (num_nodes == 0) {
    clear_error();
    return GNN_OK;
  }
  GNN_REQUIRE(row_ptr != nullptr && deg_inv_sqrt != nullptr, GNN_ERR_NULL_POINTER,
              "row_ptr and deg_inv_sqrt must not be NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = grid_for(num_nodes * 32);
  if (row_ptr_type == GNN_INDEX_INT64) {
    edge_weight_kernel<int64_t><<<grid, kThreads, 0, s>>>(static_cast<const int64_t*>(row_ptr), col_ind, deg_inv_sqrt,
                                                          num_nodes, edge_weight);
  } else {
    edge_weight_kernel<int32_t><<<grid, kThreads, 0, s>>>(static_cast<const int32_t*>(row_ptr), col_ind, deg_inv_sqrt,
                                                          num_nodes, edge_weight);
  }
  GNN_LAUNCH_CHECK("csr edge weight");
  clear_error();
  return GNN_OK;
}
