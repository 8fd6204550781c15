/*
 * gnn_b200.h — C ABI of libgnnb200.so, the B200 (sm_100a) GNN aggregation engine.
 *
 * Drop-in boundary for the operator surface of jonghyun1215/GNN_cuda. Every
 * entry point replaces one function of the reference's pybind11 tables
 * (GNN_cuda_common/native/{agg_ops,gcn_ops,pyg_gcn_ops,uvm_allocator}.cpp);
 * the comment above each declaration names the reference function (file:line)
 * that it replaces.
 *
 * Conventions
 *   - Plain pointers and sizes only. Device pointers must be readable by the
 *     current CUDA device (device memory, cudaMallocManaged memory, mapped
 *     pinned host memory, or pageable host memory on HMM-capable systems).
 *   - Dense matrices are row-major, contiguous, fp32. Index arrays: row_ptr is
 *     int32 or int64 (see gnn_index_type), col_ind is int32.
 *   - Every call is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) and returns a gnn_status. On failure, gnn_last_error()
 *     returns a thread-local message whose text matches the reference's
 *     TORCH_CHECK messages where the same condition is checked.
 *   - No entry point allocates device memory except the allocator family
 *     (gnn_managed_*). Kernels that need scratch take a caller-provided
 *     workspace whose size is given by the matching *_workspace_bytes query.
 *   - Results are deterministic: no floating-point atomics; every output row
 *     is reduced in a fixed order.
 */
#ifndef GNN_B200_H_
#define GNN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct CUstream_st* gnn_stream_t; /* == cudaStream_t */

typedef enum gnn_status {
  GNN_OK = 0,
  GNN_ERR_INVALID_ARGUMENT = 1, /* shape / size / range check failed          */
  GNN_ERR_NULL_POINTER = 2,     /* a required pointer was NULL                */
  GNN_ERR_UNSUPPORTED = 3,      /* valid request this build does not support  */
  GNN_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed       */
  GNN_ERR_TIMEOUT = 5,          /* a bounded device-side wait gave up         */
  GNN_ERR_DEVICE = 6,           /* no usable CUDA device / capability missing */
  GNN_ERR_WORKSPACE = 7         /* workspace missing or too small             */
} gnn_status;

typedef enum gnn_index_type {
  GNN_INDEX_INT32 = 0,
  GNN_INDEX_INT64 = 1
} gnn_index_type;

/* Precision of the dense transform X·W on the tensor cores. */
typedef enum gnn_precision {
  GNN_PRECISION_TF32 = 0, /* one tf32 tcgen05 pass (relative tolerance 2e-3)     */
  GNN_PRECISION_FP32 = 1  /* fp32 SIMT FFMA, the reference's cublasSgemm numerics */
} gnn_precision;

/* ---- library --------------------------------------------------------------- */
int gnn_version(void);                /* major*10000 + minor*100 + patch */
const char* gnn_last_error(void);     /* thread-local; "" after a success  */
const char* gnn_status_string(int status);
/* Tuning knobs (process-wide). Names: "spmm.long_row_threshold" (edges; 0 =
 * automatic), "spmm.long_row_warps" (4..16), "spmm.kernel" (0 = persistent
 * packed-stream kernel; 1 = one warp per row, the default; 2 = packed stream
 * with cp.async staging through shared memory; all give identical results),
 * "spmm.schedule" (row order of the per-row kernel when the workspace holds a
 * schedule: 0 id order, 1 degree order within windows of "spmm.schedule_window"
 * rows, 2 global degree order, 3 automatic = 2 below a mean degree of 64 else 1;
 * identical results), "gemm.stages" (tcgen05 GEMM ring depth, 0 = automatic).
 * Returns GNN_ERR_INVALID_ARGUMENT
 * for an unknown name or out-of-range value. */
int gnn_config_set_int(const char* name, int64_t value);
int gnn_config_get_int(const char* name, int64_t* value);
/* Number of kernels this library has launched in this process (all devices). */
uint64_t gnn_kernel_launches(void);
/* 1 when GNN_PRECISION_TF32 GEMMs of this shape run on the tcgen05 tensor
 * cores of the current device, 0 when they run on the FFMA kernel
 * (eligible: 32 <= K <= 256, K % 32 == 0, N % 128 == 0 or N in {32, 64},
 * 16-byte aligned operands). */
int gnn_gemm_uses_tensor_cores(int64_t m, int64_t k, int64_t n);
/* Device-side bounded waits (mbarrier spins in the tensor-core kernels, the
 * segment chain of long rows in the aggregation kernels) give up after ~2 s
 * instead of hanging; they then record a non-zero code here (1-6 tensor-core
 * pipeline, 16 aggregation segment chain, 17 aggregation long-row list
 * overflow) and the kernel moves on. Synchronises with the current device,
 * stores the word in *status and clears it when reset != 0. */
int gnn_device_status(int reset, int* status);

/* ---- CSR aggregation (SpMM) ------------------------------------------------
 * All aggregation entry points compute, for every row r of a dst-major CSR,
 *     out[r, :] = epilogue( sum_{e in row r, CSR order} w_e * x[col_ind[e], :] )
 * into a preallocated `out` of the same shape as `x` ([num_nodes, feat_dim]).
 * Rows of degree <= the long-row threshold are accumulated sequentially in CSR
 * order with fused multiply-adds, exactly like the reference kernels; longer
 * rows are cut into segments of long_row_warps * 512 entries, each segment
 * split across the warps of one CTA, and the partial sums are added in a fixed
 * order (chunks within a segment, then segments).
 *
 * `workspace` must hold gnn_spmm_workspace_bytes(num_nodes, num_edges) bytes
 * (256-byte aligned, device memory). Two calls in flight at once on different
 * streams must use different workspaces.
 */
size_t gnn_spmm_workspace_bytes(int64_t num_nodes, int64_t num_edges);
/* The larger workspace with room for a degree-ordered row schedule (no
 * reference counterpart: a scheduling aid of this engine). Given at least this
 * many bytes, the per-row aggregation kernel takes rows in descending degree
 * order, built per call by a counting sort (O(num_nodes), graphs of >= 65,536
 * nodes): faster on skewed graphs, identical results, since every row is still
 * summed alone in CSR order. With gnn_spmm_workspace_bytes() bytes the rows run
 * in id order. */
size_t gnn_spmm_schedule_workspace_bytes(int64_t num_nodes, int64_t num_edges);

/* The degree above which a row of a graph with these sizes is summed in
 * segments (the "spmm.long_row_threshold" knob when set, else the automatic
 * value clamp(num_edges / (SMs * 256), 256, 8192) on the current device). A
 * caller that aggregates a graph in several row pieces sets this value as the
 * knob so that every piece cuts its rows exactly as one whole-graph call
 * would. No counterpart in the reference (its kernels never split a row). */
int64_t gnn_spmm_long_row_threshold(int64_t num_nodes, int64_t num_edges);

/* GCN normalised aggregation, w_e = deg_inv_sqrt[r] * deg_inv_sqrt[col].
 * Replaces spmm_gcn_forward_cuda_ (naive), GNN_cuda_common/native/gcn_ops.cu:327. */
int gnn_spmm_gcn_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                         const float* deg_inv_sqrt, const float* x, float* out,
                         int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                         void* workspace, size_t workspace_bytes, gnn_stream_t stream);

/* Row-partitioned GCN aggregation for one shard of a multi-GPU run (no
 * reference counterpart; the reference is single-GPU). The shard holds rows
 * [row_begin, row_begin + num_rows) of the global CSR: row_ptr/col_ind are the
 * shard's (col_ind keeps global column ids), deg_inv_sqrt and x are global
 * ([num_cols] and [num_cols, feat_dim]), out is [num_rows, feat_dim]. Same
 * arithmetic as gnn_spmm_gcn_forward with dis[row_begin + r] as row scale. */
int gnn_spmm_gcn_partition_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                   const float* deg_inv_sqrt, int64_t row_begin, const float* x,
                                   float* out, int64_t num_rows, int64_t num_cols, int64_t num_edges,
                                   int64_t feat_dim, void* workspace, size_t workspace_bytes,
                                   gnn_stream_t stream);

/* GCN aggregation that allocates nothing and takes no workspace. No
 * counterpart in the reference: it exists for callers that cannot hand the
 * library a scratch buffer or let it call cudaMalloc — a plugin host or FFI
 * binding that owns all device memory and passes only inputs and outputs, a
 * process pinned to a fixed memory budget, or a latency-critical path that
 * cannot afford cudaMalloc/cudaFree (which may wait for the whole device).
 * Same kernels and results as gnn_spmm_gcn_forward given the minimum workspace
 * (gnn_spmm_workspace_bytes): rows run in row-id order, because the
 * degree-ordered row schedule needs 4 more bytes per node than the scratch
 * holds at large sizes (18,102,528 bytes for the 2,449,029-node graph below),
 * which is slower on power-law graphs but gives the same results. The scratch
 * is a built-in 8 MiB (8388608-byte) device array per GPU, held until the
 * process exits.
 * Problems with gnn_spmm_workspace_bytes(num_nodes, num_edges) > 8 MiB are
 * rejected with GNN_ERR_UNSUPPORTED (for example, any graph with at most
 * 1,000,000 nodes and 500,000,000 entries fits, and so does a 2,449,029-node,
 * 64,308,169-entry graph). All calls on a device share that array: calls that
 * overlap on the GPU race and must be serialised (e.g. one stream). Each call
 * clears the counters it reads. The first call on a device looks the array's
 * address up, so make it before any stream capture on that device; that
 * address is kept for the process's life, so a cudaDeviceReset of the device
 * after the first call is not supported. */
int gnn_spmm_gcn_forward_noalloc(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                 const float* deg_inv_sqrt, const float* x, float* out,
                                 int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                                 gnn_stream_t stream);

/* Replaces spmm_gcn_hmm_forward_cuda_ ("plain", the default GCN kernel),
 * GNN_cuda_common/native/gcn_ops.cu:350. Same arithmetic as the naive entry. */
int gnn_spmm_gcn_hmm_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                             const float* deg_inv_sqrt, const float* x, float* out,
                             int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                             void* workspace, size_t workspace_bytes, gnn_stream_t stream);

/* Row-scheduled variant with a device copy of the first `hot_node_cutoff` rows
 * of x: neighbours col < hot_node_cutoff are read from hot_feature_cache.
 * Replaces spmm_gcn_hmm_optimized_forward_cuda_, gcn_ops.cu:381 (checks :260-285). */
int gnn_spmm_gcn_hmm_optimized_forward(const void* row_ptr, int row_ptr_type,
                                       const int32_t* col_ind, const float* deg_inv_sqrt,
                                       const float* x, const int64_t* row_schedule,
                                       const float* hot_feature_cache, int64_t hot_node_cutoff,
                                       float* out, int64_t num_nodes, int64_t num_edges,
                                       int64_t feat_dim, void* workspace, size_t workspace_bytes,
                                       gnn_stream_t stream);

/* out[i, :] = x[page_ids[i / rows_per_page] * rows_per_page + i % rows_per_page, :] or 0
 * past num_nodes. Replaces stage_feature_pages_cuda_, gcn_ops.cu:426. */
int gnn_stage_feature_pages(const int64_t* page_ids, int64_t num_pages, const float* x,
                            int64_t num_nodes, float* out, int64_t rows_per_page,
                            int64_t feat_dim, gnn_stream_t stream);

/* out[:rows] = x[:rows]. Replaces stage_feature_rows_cuda_, gcn_ops.cu:449. */
int gnn_stage_feature_rows(const float* x, int64_t x_rows, float* out, int64_t out_rows,
                           int64_t feat_dim, gnn_stream_t stream);

/* PyG-style weighted aggregation, w_e = edge_weight[e].
 * Replaces spmm_pyg_gcn_forward_cuda_ (naive), pyg_gcn_ops.cu:254. */
int gnn_spmm_pyg_gcn_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                             const float* edge_weight, const float* x, float* out,
                             int64_t num_nodes, int64_t num_edges, int64_t feat_dim,
                             void* workspace, size_t workspace_bytes, gnn_stream_t stream);

/* Replaces spmm_pyg_gcn_plain_forward_cuda_, pyg_gcn_ops.cu:277. */
int gnn_spmm_pyg_gcn_plain_forward(const void* row_ptr, int row_ptr_type,
                                   const int32_t* col_ind, const float* edge_weight,
                                   const float* x, float* out, int64_t num_nodes,
                                   int64_t num_edges, int64_t feat_dim, void* workspace,
                                   size_t workspace_bytes, gnn_stream_t stream);

/* Replaces spmm_pyg_gcn_hmm_optimized_forward_cuda_ (pyg_gcn_ops.cu:353) and
 * spmm_pyg_gcn_uvm_optimized_forward_cuda_ (pyg_gcn_ops.cu:363), which are the
 * same function in the reference. */
int gnn_spmm_pyg_gcn_optimized_forward(const void* row_ptr, int row_ptr_type,
                                       const int32_t* col_ind, const float* edge_weight,
                                       const float* x, const int64_t* row_schedule,
                                       const float* hot_feature_cache, int64_t hot_node_cutoff,
                                       float* out, int64_t num_nodes, int64_t num_edges,
                                       int64_t feat_dim, void* workspace, size_t workspace_bytes,
                                       gnn_stream_t stream);

/* Sum aggregation (GIN). Replaces spmm_sum_forward_cuda_, agg_ops.cu:315, and
 * spmm_sum_hmm_forward_cuda_, agg_ops.cu:329 (identical arithmetic). */
int gnn_spmm_sum_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                         const float* x, float* out, int64_t num_nodes, int64_t num_edges,
                         int64_t feat_dim, void* workspace, size_t workspace_bytes,
                         gnn_stream_t stream);

/* Mean aggregation (GraphSAGE); a row of degree 0 gives 0.
 * reciprocal == 0: acc / deg, as spmm_mean_forward_cuda_, agg_ops.cu:322 (kernel :40-45).
 * reciprocal != 0: acc * (1/deg), as spmm_mean_hmm_forward_cuda_, agg_ops.cu:336 (kernel :102-111). */
int gnn_spmm_mean_forward(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                          const float* x, float* out, int64_t num_nodes, int64_t num_edges,
                          int64_t feat_dim, int reciprocal, void* workspace,
                          size_t workspace_bytes, gnn_stream_t stream);

/* ---- dense transform and epilogues ----------------------------------------- */

/* out[M,N] = x[M,K] · weight[K,N] (weight stored [in, out] = nn.Linear.weight^T).
 * Replaces gemm_forward_cuda_, agg_ops.cu:369 (cublasSgemm). */
int gnn_gemm_forward(const float* x, const float* weight, float* out, int64_t m, int64_t k,
                     int64_t n, int precision, gnn_stream_t stream);

/* out = relu?(x · weight + bias) with bias/ReLU fused into the GEMM epilogue;
 * bias may be NULL. Replaces linear_forward_cuda_, agg_ops.cu:343. */
int gnn_linear_forward(const float* x, const float* weight, const float* bias, float* out,
                       int64_t m, int64_t k, int64_t n, int relu, int precision,
                       gnn_stream_t stream);

/* gnn_linear_forward at GNN_PRECISION_TF32 on the tcgen05 path, fused with the
 * halo push of the multi-GPU forward: output row i is also stored to row i of
 * peer_out[d] (a peer's buffer from gnn_ipc_open, the same [m, n] layout) for
 * every bit d set in peer_mask[i] (one byte per row, device memory), from the
 * GEMM's epilogue while later tiles are still computed. npeers <= 8; peer rows
 * 16-byte aligned. Returns GNN_ERR_UNSUPPORTED (nothing launched) where the
 * tensor-core GEMM does not apply (gnn_gemm_uses_tensor_cores, 16-byte aligned
 * operands); the caller then runs gnn_linear_forward and gnn_peer_push_rows.
 * Replaces, for the multi-GPU mode (no reference counterpart), the pair
 * linear_forward_cuda_ (agg_ops.cu:343) + gnn_peer_push_rows. */
int gnn_linear_push_forward(const float* x, const float* weight, const float* bias, float* out,
                            int64_t m, int64_t k, int64_t n, int relu, const uint8_t* peer_mask,
                            float* const* peer_out, int npeers, gnn_stream_t stream);

/* out[i, j] = relu?(out[i, j] + bias[j]); bias may be NULL.
 * Replaces bias_relu_forward_cuda_, agg_ops.cu:393 (kernel :132-147). */
int gnn_bias_relu_forward(float* out, const float* bias, int64_t rows, int64_t cols, int relu,
                          gnn_stream_t stream);

/* dst += alpha * src (one fused multiply-add per element).
 * Replaces tensor_add_inplace_cuda_, agg_ops.cu:399 (kernel :149-156). */
int gnn_tensor_add_inplace(float* dst, const float* src, float alpha, int64_t count,
                           gnn_stream_t stream);

/* t = max(t, 0) keeping -0 and NaN as they are. Replaces relu_inplace_cuda_, agg_ops.cu:420. */
int gnn_relu_inplace(float* t, int64_t count, gnn_stream_t stream);

/* ---- one layer in one pass: aggregation + dense transform ------------------- */

/* Aggregations for gnn_fused_aggregate_linear. */
typedef enum gnn_aggregation {
  GNN_AGG_GCN = 0,             /* sum of dis[r]·dis[c]·x[c] (spmm_gcn_forward_)                  */
  GNN_AGG_SUM = 1,             /* sum of x[c] (spmm_sum_forward_)                                  */
  GNN_AGG_MEAN = 2,            /* sum / deg (spmm_mean_forward_)                                   */
  GNN_AGG_MEAN_RECIPROCAL = 3  /* sum * (1/deg) (spmm_mean_hmm_forward_)                           */
} gnn_aggregation;

/* 1 when gnn_fused_aggregate_linear supports these widths on the current
 * device (sm_100; feat_dim 32, 64, 96 or 128; width1 / width2 32, 64 or 128,
 * width2 = 0 for a single transform; output width >= feat_dim), else 0. */
int gnn_fused_layer_supported(int64_t feat_dim, int64_t width1, int64_t width2);

/* One GNN layer without the [N, F] aggregate in device memory:
 *   a   = aggregate(x) over rows [row_begin, row_begin + num_rows) of the graph
 *         (GCN / sum / mean, exactly as the aggregation entry points above),
 *         then a = fma(self_scale, x[row], a) when add_self (GIN's (1+eps)·x);
 *   h   = relu1?(a · weight1 + bias1)                 weight1 [feat_dim, width1]
 *   out = relu2?(h · weight2 + bias2)  if width2 > 0  weight2 [width1, width2]
 *   out = h                            otherwise.
 * The reference composes each layer from separate calls with an [N, F] buffer
 * between them: gcn_inference.py:534-600 (spmm_gcn_forward_ -> gemm_forward_ ->
 * bias_relu_forward_), gin_inference.py:317-359 (spmm_sum_forward_ ->
 * tensor_add_inplace_ -> linear_forward_ x 2) and the neighbour half of
 * graphsage_inference.py:310-354. Results are bit-identical to that sequence
 * on this library's tcgen05 TF32 path (the same row sums and the same MMA
 * instructions on the same operand bits). x is [num_cols, feat_dim]; out is
 * [num_rows, width2 ? width2 : width1] and must not alias x; rows above the
 * long-row threshold are summed into their own row of out first, which is why
 * the output must be at least feat_dim wide. biases may be NULL; x, out,
 * weights and biases 16-byte aligned. Workspace:
 * gnn_spmm_schedule_workspace_bytes(num_rows, num_edges). */
int gnn_fused_aggregate_linear(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                               const float* deg_inv_sqrt, int aggregation, int64_t row_begin,
                               const float* x, int64_t num_rows, int64_t num_cols, int64_t num_edges,
                               int64_t feat_dim, float self_scale, int add_self, const float* weight1,
                               const float* bias1, int64_t width1, int relu1, const float* weight2,
                               const float* bias2, int64_t width2, int relu2, float* out,
                               void* workspace, size_t workspace_bytes, gnn_stream_t stream);

/* ---- unified / host memory (allocator family) ------------------------------ */

/* cudaMallocManaged(bytes, cudaMemAttachGlobal) on `device`; *ptr = NULL for 0 bytes.
 * Replaces managed_empty_cuda, uvm_allocator.cu:93. */
int gnn_managed_alloc(size_t bytes, int device, void** ptr);
/* Frees memory from gnn_managed_alloc (deleter of uvm_allocator.cu:107-113). */
int gnn_managed_free(void* ptr, int device);
/* *supported = cudaDevAttrPageableMemoryAccess of `device` (HMM). Replaces the
 * capability check of hmm_empty_cpu, uvm_allocator.cu:45-57 and :120-127. */
int gnn_hmm_supported(int device, int* supported);
/* Host memcpy into managed memory after checking that dst is managed.
 * Replaces copy_cpu_to_managed_cuda_, uvm_allocator.cu:129. */
int gnn_copy_host_to_managed(void* dst, const void* src, size_t bytes);
/* cudaMemPrefetchAsync of [ptr+offset, ptr+offset+bytes) to `location`
 * (-1 = cpu, >=0 = that device) on `stream`. Replaces prefetch_cuda_ (:151)
 * and prefetch_range_cuda_ (:163) of uvm_allocator.cu; the reference always
 * used the default stream, this entry point takes the caller's stream. */
int gnn_prefetch(void* ptr, size_t offset, size_t bytes, size_t total_bytes, int location,
                 int device, gnn_stream_t stream);
/* cudaMemAdvise wrappers. location -1 = cpu, 0 = `device` (the reference's
 * location_code convention, uvm_allocator.cu:189-229). */
int gnn_advise_preferred_location(void* ptr, size_t bytes, int location, int device);
int gnn_advise_accessed_by(void* ptr, size_t bytes, int location, int device);
int gnn_advise_read_mostly(void* ptr, size_t bytes, int enabled, int device);

typedef struct gnn_pointer_info {
  int memory_type;     /* 0 unregistered, 1 host, 2 device, 3 managed, -1 query failed */
  int device;          /* attribute device, -1 if none                                   */
  int is_managed;
  int is_host_mapped;  /* pinned host memory with a device alias                         */
  int pageable_access; /* current device supports HMM pageable access                    */
  void* device_pointer;
} gnn_pointer_info;
/* Replaces pointer_info_cuda, uvm_allocator.cu:231 (the Python layer builds the dict). */
int gnn_pointer_info_query(const void* ptr, gnn_pointer_info* info);
/* Device-usable alias of a host pointer: the mapped alias of pinned memory, the
 * pointer itself under HMM, else GNN_ERR_DEVICE. Replaces
 * get_device_accessible_void_ptr, tensor_access.cuh:25-64. */
int gnn_device_accessible_ptr(const void* host_ptr, void** device_ptr);

/* ---- CSR construction on the device ----------------------------------------
 * Replaces the host builders of GNN_cuda_common/graph_utils.py:449-535
 * (build_gcn_normalized_csr, build_pyg_gcn_weighted_csr, build_plain_csr),
 * which go through scipy's coo_matrix.tocsr() + sort_indices(): rows hold
 * their distinct columns in increasing order, duplicate pairs merge, and
 * self-loops (r, r) are appended first when asked. Same arrays bit for bit. */

/* Scratch for gnn_csr_build (two key buffers of num_entries (+ num_nodes) 8-byte
 * keys plus sort/unique scratch). Queries the current device; 0 on failure. */
size_t gnn_csr_build_workspace_bytes(int64_t num_entries, int64_t num_nodes, int add_self_loops);
/* Builds row_ptr [num_nodes + 1] (int32 or int64) and col_ind [*num_unique]
 * from int64 (row_ids[i], col_ids[i]) pairs, i < num_entries, plus (r, r) for
 * every node when add_self_loops != 0. col_capacity must be >= the number of
 * distinct pairs (num_entries + num_nodes always suffices). Ids outside
 * [0, num_nodes) fail with the host builder's messages ("negative row index
 * found", "row index exceeds matrix dimensions", ...); an int32 row_ptr fails
 * when the CSR has more than 2^31 - 1 entries (the reference's cast would wrap).
 * Synchronises `stream`; *num_unique and *max_degree (largest row length) are
 * host values on return. */
int gnn_csr_build(const int64_t* row_ids, const int64_t* col_ids, int64_t num_entries, int64_t num_nodes,
                  int add_self_loops, void* row_ptr, int row_ptr_type, int32_t* col_ind, int64_t col_capacity,
                  int64_t* num_unique, int64_t* max_degree, void* workspace, size_t workspace_bytes,
                  gnn_stream_t stream);
/* deg_inv_sqrt[r] = table[deg(r)], where table[d] (d = 0..max_degree) holds the
 * float32 value clip(d, 1)^-0.5 exactly as numpy's float32 power computes it
 * (graph_utils.py:463-464); the caller fills the table on the host. */
int gnn_csr_deg_inv_sqrt(const void* row_ptr, int row_ptr_type, int64_t num_nodes, const float* table,
                         int64_t table_len, float* deg_inv_sqrt, gnn_stream_t stream);
/* PyG weights edge_weight[e] = deg_inv_sqrt[row(e)] * deg_inv_sqrt[col_ind[e]]
 * in float32 (graph_utils.py:496-497). */
int gnn_csr_edge_weight(const void* row_ptr, int row_ptr_type, const int32_t* col_ind, const float* deg_inv_sqrt,
                        int64_t num_nodes, float* edge_weight, gnn_stream_t stream);

/* ---- UVM locality preprocessing on the device ------------------------------
 * Replaces the host preprocessing behind spmm_mode="optimized":
 * build_page_reuse_schedule_metadata (GNN_cuda_common/graph_utils.py:244-372),
 * build_coaccess_feature_permutation (:375-446),
 * build_hot_partition_feature_permutation (:174-241) and
 * apply_graph_permutation (:76-85), as chained by run/preprocess_gcn_graph.py:40-120.
 * Same arrays bit for bit (integer orders with the reference's tie-breaks);
 * the float64 ratios are formed on the host from integer totals exactly as
 * numpy forms them. The CSR inputs are the dst-major CSR with self-loops that
 * gnn_csr_build produces (graph_utils.py:258-267 builds the same one). These
 * calls validate their index inputs on the device (a bad id is an error, never
 * an out-of-bounds access), read host scalars back, and so synchronise `stream`.
 * All int64 outputs are device arrays the caller allocates. */

/* Scratch for every gnn_locality_* call on a graph of num_nodes nodes and
 * num_entries CSR entries with top-k lists up to max_k (the larger of
 * signature_topk and window_cache_pages; <= 4096). Queries the current device;
 * 0 on failure. */
size_t gnn_locality_workspace_bytes(int64_t num_nodes, int64_t num_entries, int64_t max_k);

/* Page metadata and row schedule of a CSR (build_page_reuse_schedule_metadata).
 * With P = ceil(num_nodes / rows_per_page), NB = ceil(num_nodes / row_block_size),
 * NW = ceil(num_nodes / (row_block_size * window_num_blocks)), k = signature_topk:
 * page_histogram [P], hot_pages [min(hot_cache_pages, P)], row_schedule
 * [num_nodes], block_hot_pages [NB, k], window_hot_pages [NW, window_cache_pages]
 * (pages padded with P); host outputs: the largest page count (the length - 1
 * of page_reuse_histogram, see gnn_locality_count_histogram), hot_coverage and
 * avg_window_hot_coverage. num_entries < 2^32. */
int gnn_locality_page_schedule(const void* row_ptr, int row_ptr_type, const int32_t* col_ind, int64_t num_nodes,
                               int64_t num_entries, int64_t rows_per_page, int64_t row_block_size,
                               int64_t window_num_blocks, int64_t window_cache_pages, int64_t hot_cache_pages,
                               int64_t signature_topk, int64_t* page_histogram, int64_t* hot_pages,
                               int64_t* row_schedule, int64_t* block_hot_pages, int64_t* window_hot_pages,
                               int64_t* max_page_count, double* hot_coverage, double* avg_window_hot_coverage,
                               void* workspace, size_t workspace_bytes, gnn_stream_t stream);

/* hist[v] = number of i with values[i] == v for 1 <= v < hist_len, hist[0] = 0:
 * np.bincount of the non-zero values (graph_utils.py:273-278, the page reuse
 * histogram, with hist_len = largest page count + 1). */
int gnn_locality_count_histogram(const int64_t* values, int64_t count, int64_t* hist, int64_t hist_len,
                                 gnn_stream_t stream);

/* Node order by co-access windows (build_coaccess_feature_permutation):
 * perm, inv_perm [num_nodes]. row_schedule must be a permutation of
 * [0, num_nodes); rows_per_window = row_block_size * window_num_blocks. */
int gnn_locality_coaccess_permutation(const void* row_ptr, int row_ptr_type, const int32_t* col_ind,
                                      int64_t num_nodes, int64_t num_entries, const int64_t* row_schedule,
                                      int64_t rows_per_window, int64_t signature_topk, int64_t* perm,
                                      int64_t* inv_perm, void* workspace, size_t workspace_bytes,
                                      gnn_stream_t stream);

/* Hot prefix / cold suffix order (build_hot_partition_feature_permutation).
 * src: the int64 source id of every edge (plus one access per node when
 * add_self_loops). Outputs: access_count [num_nodes], sorted_nodes [num_nodes]
 * (stable descending order of access_count; hot_nodes is its first
 * *hot_node_cutoff entries), perm and inv_perm [num_nodes]; host: the cutoff,
 * the hot_min_nodes actually used, total and hot access counts. base_order
 * (NULL for none) must be a permutation of [0, num_nodes) — the reference only
 * checks its length. */
int gnn_locality_hot_partition(const int64_t* src, int64_t num_entries, int64_t num_nodes, int add_self_loops,
                               const int64_t* base_order, double hot_access_coverage, double hot_max_ratio,
                               int64_t hot_min_nodes, int64_t* access_count, int64_t* sorted_nodes, int64_t* perm,
                               int64_t* inv_perm, int64_t* hot_node_cutoff, int64_t* min_nodes_used,
                               int64_t* total_access, int64_t* hot_access, void* workspace,
                               size_t workspace_bytes, gnn_stream_t stream);

/* src_out[i] = inv_perm[src[i]], dst_out[i] = inv_perm[dst[i]]
 * (apply_graph_permutation, graph_utils.py:76-85). workspace: >= 256 bytes of
 * device memory for the error flag. */
int gnn_permute_edges(const int64_t* src, const int64_t* dst, int64_t num_entries, const int64_t* inv_perm,
                      int64_t num_nodes, int64_t* src_out, int64_t* dst_out, void* workspace, size_t workspace_bytes,
                      gnn_stream_t stream);

/* ---- peer memory for the row-partitioned multi-GPU mode -------------------- *
 * No counterpart in the reference, which runs on one GPU. A rank allocates its
 * copy of the next layer's input with gnn_peer_alloc, exports it with
 * gnn_ipc_get_handle, opens every peer's copy with gnn_ipc_open, and pushes
 * each finished row piece into the peers' copies with gnn_copy_async (one
 * copy-engine transfer per peer; no SM is used). */

/* cudaMalloc(bytes) on `device`, exportable through CUDA IPC. */
int gnn_peer_alloc(size_t bytes, int device, void** ptr);
int gnn_peer_free(void* ptr, int device);
/* Size of an IPC handle (sizeof(cudaIpcMemHandle_t), 64). */
size_t gnn_ipc_handle_bytes(void);
/* Writes the IPC handle of a gnn_peer_alloc buffer into `handle`. */
int gnn_ipc_get_handle(const void* ptr, void* handle, size_t handle_bytes);
/* Maps a peer's buffer into this process for `device` (peer access enabled lazily). */
int gnn_ipc_open(const void* handle, size_t handle_bytes, int device, void** ptr);
int gnn_ipc_close(void* ptr, int device);
/* *can = cudaDeviceCanAccessPeer(device, peer). */
int gnn_can_access_peer(int device, int peer, int* can);
/* cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream); 0 bytes is a no-op. */
int gnn_copy_async(void* dst, const void* src, size_t bytes, gnn_stream_t stream);
/* One kernel that reads [src, src + bytes) once and stores it to each of the
 * ndst (<= 8) destinations (peer buffers from gnn_ipc_open): the SMs drive the
 * NVLink writes. ctas limits the grid (0 = 4 per SM). bytes, src and every
 * destination must be 16-byte aligned. */
int gnn_peer_push(const void* src, void* const* dsts, int ndst, size_t bytes, int ctas, gnn_stream_t stream);
/* Halo push: stores only the rows each peer reads. For destination q, rows
 * row_ids[row_offsets[q] .. row_offsets[q+1]) (row_offsets is a HOST array of
 * ndst + 1 entries starting at 0; row_ids is device int32) are copied from src
 * to the same row of dsts[q] (every buffer has the same [max_rows, row_bytes]
 * layout). One warp per listed row, the destinations' rows interleaved so that
 * every peer receives at once; ids outside [0, max_rows) are skipped. ctas
 * limits the grid (0 = 1 per SM, which leaves the other SMs' slots to the
 * aggregation running beside the push). row_bytes, src and every destination
 * must be 16-byte aligned; ndst <= 8. */
int gnn_peer_push_rows(const void* src, void* const* dsts, int ndst, const int32_t* row_ids,
                       const int64_t* row_offsets, int64_t row_bytes, int64_t max_rows, int ctas,
                       gnn_stream_t stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* GNN_B200_H_ */
