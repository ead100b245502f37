/*
 * pkm_b200.h - C ABI of the B200 (sm_100a) product-key-memory kernels.
 *
 * Every entry point takes raw device pointers, int64 sizes, dtype codes and
 * a CUDA stream (as void*, i.e. a cudaStream_t), enqueues its kernels on that
 * stream and returns a pkm_status code.  Nothing here allocates device
 * memory: scratch space is passed in by the caller after a *_workspace query.
 * All tensors are dense row-major (C-contiguous).  Shape, dtype and alignment
 * errors are reported before any launch (the reference raises AssertionError
 * for the same conditions, pkm/xformer_embeddingbag.py:226-233).
 *
 * Indices are int64 as in the reference (fwpkm/xformer_embeddingbag_grad_wrapper.py:94).
 * An index outside [0, num_rows) is skipped (contributes nothing, its
 * per-sample gradient is 0) and sets PKM_DEVERR_INDEX in *dev_err when
 * dev_err is not NULL; the host reads that word when it wants to know.
 *
 * Slot numbering of the product keys follows pkm/memory.py:278-281:
 * slot = i1 * n_keys + i2.  Query rows are token*heads + head; keys are
 * [2*heads*n_keys, k_dim/2] viewed as (heads, 2, n_keys, k_dim/2)
 * (pkm/memory.py:257).
 */
#ifndef PKM_B200_H
#define PKM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PKM_API __attribute__((visibility("default")))
#else
#define PKM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types. */
enum {
  PKM_DT_F32 = 0,
  PKM_DT_BF16 = 1,
  PKM_DT_F16 = 2,
};

/* Return codes. */
enum {
  PKM_OK = 0,
  PKM_ERR_INVALID_ARG = 1, /* shape / dtype / alignment / null pointer */
  PKM_ERR_UNSUPPORTED = 2, /* a size outside what the kernels implement */
  PKM_ERR_CUDA = 3,        /* the CUDA runtime reported an error at launch */
  PKM_ERR_WORKSPACE = 4,   /* workspace smaller than the *_workspace query */
};

/* Bits OR-ed into the optional device error word. */
#define PKM_DEVERR_INDEX 1u   /* an index outside [0, num_rows) was skipped */
#define PKM_DEVERR_TIMEOUT 2u /* a bounded wait inside a kernel gave up */

/* Library version (major*10000 + minor*100 + patch). */
PKM_API int pkm_version(void);
/* Static description of a status code. */
PKM_API const char* pkm_status_string(int status);
/* Detail message of the last failing call on this host thread. */
PKM_API const char* pkm_last_error(void);

/*
 * K3 - weighted embedding-bag forward.
 *   out[b, :] = sum_j psw[b, j] * weight[indices[b, j], :]   (fp32 accumulate)
 * Replaces embedding_bag_k / embedding_bag_triton
 * (pkm/xformer_embeddingbag.py:97-138, fwpkm/xformer_embeddingbag_legacy.py:33-74)
 * and the fwpkm torch gather (fwpkm/xformer_embeddingbag_grad_wrapper.py:99-103).
 * psw may be NULL (all weights 1).  weight rows must be 16-byte multiples and
 * at most 4096 bytes; out_dtype may differ from weight_dtype.
 */
PKM_API int pkm_bag_fwd(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                int weight_dtype, int64_t n_bags, int64_t bag_size, int64_t num_rows, int64_t dim,
                void* out, int out_dtype, uint32_t* dev_err, void* stream);

/*
 * K4 - first-order backward of the bag, atomic-free and deterministic.
 *   grad_weight[k] = sum_{(b,j): idx=k} psw[b,j] * grad_out[b]  (dense; 0 for
 *                    untouched rows; summed in ascending (b, j) order)
 *   grad_psw[b,j]  = <weight[idx[b,j]], grad_out[b]>
 *   row_counts[k]  = number of occurrences of k (optional; the bincount of
 *                    fwpkm/fwpkm.py:343)
 * Replaces embedding_bag_bw_rev_indices (pkm/xformer_embeddingbag.py:331-386,
 * fwpkm/xformer_embeddingbag_legacy.py:170-227).  grad_psw and row_counts may
 * be NULL; weight may be NULL when grad_psw is NULL.  grad_out must have the
 * weight's dtype.  workspace must hold pkm_bag_bwd_workspace() bytes,
 * 256-byte aligned.
 */
PKM_API int pkm_bag_bwd_workspace(int64_t n_bags, int64_t bag_size, int64_t num_rows, int64_t dim,
                          size_t* bytes);
PKM_API int pkm_bag_bwd(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                int64_t num_rows, int64_t dim, void* grad_weight, int grad_weight_dtype,
                void* grad_psw, int grad_psw_dtype, int32_t* row_counts, void* workspace,
                size_t workspace_bytes, uint32_t* dev_err, void* stream);

/*
 * Allocation-free K4.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory (an FFI binding without a device
 * allocator of its own, or a latency-critical loop where a cudaMalloc, which
 * may synchronise the device, is not allowed).  Same arguments and results as
 * pkm_bag_bwd, without the workspace: the scratch is a 16 MiB static device
 * array inside the library, held by every GPU that loads it until exit.
 * Sizes whose pkm_bag_bwd_workspace() exceeds 16 MiB return
 * PKM_ERR_UNSUPPORTED before any launch.  Every call looks up the array's
 * device address (cudaGetSymbolAddress, with the caller's device current), so
 * the address stays right across a device or context reset; the first call on
 * a device also loads the library's device code there, so make that first
 * call before any stream capture.  All calls share the one array, so calls that
 * overlap on the GPU (other streams, other host threads) race; the kernels
 * clear what must start at zero on every call.
 */
PKM_API int pkm_bag_bwd_noalloc(const int64_t* indices, const void* psw, int psw_dtype,
                                const void* weight, int weight_dtype, const void* grad_out,
                                int64_t n_bags, int64_t bag_size, int64_t num_rows, int64_t dim,
                                void* grad_weight, int grad_weight_dtype, void* grad_psw,
                                int grad_psw_dtype, int32_t* row_counts, uint32_t* dev_err,
                                void* stream);

/*
 * K5 - double-backward of the bag's weight gradient.
 *   d_grad_out[b] = sum_j a[b,j] * gbar[idx[b,j]]
 *   d_a[b,j]      = <gbar[idx[b,j]], grad_out[b]>
 * Replaces EmbeddingBagBW.backward
 * (fwpkm/xformer_embeddingbag_grad_wrapper.py:43-74).  a may be NULL (ones;
 * then d_a must be NULL).  grad_out must have gbar's dtype.
 */
PKM_API int pkm_bag_bwd2(const int64_t* indices, const void* a, int a_dtype, const void* gbar,
                 int gbar_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                 int64_t num_rows, int64_t dim, void* d_grad_out, int d_grad_out_dtype, void* d_a,
                 int d_a_dtype, uint32_t* dev_err, void* stream);

/*
 * K1 - sub-key scores for both halves of every (token, head) query.
 *   scores[r, p, m] = score(query[r, p*half:(p+1)*half], keys[(h*2+p)*n + m])
 * with r = token*heads + h.  mode 0: dot product (pkm/memory.py:267-268,
 * fwpkm/fwpkm.py:861); mode 1: idw, -log(1e-3 + |q-k|^2) (fwpkm/fwpkm.py:862-866);
 * mode 2: the distance |q-k| = sqrt(max(|q|^2 - 2 q.k + |k|^2, 1e-30)) that
 * torch.cdist(..., compute_mode="use_mm_for_euclid_dist") returns; mode 3:
 * dot product with the sequential sum below.
 * fp32 inputs (all modes) and mode 3 use a sequential fp32 sum over the half
 * dimension without fused multiply-add (the oracle's definition).  bf16 dot
 * products (mode 0) with half % 64 == 0 and n_keys % 8 == 0 run on the
 * tcgen05 tensor cores (fp32 accumulation, rounded to bf16).
 * query and keys must share a dtype; scores has that dtype.  dev_err may be
 * NULL (see PKM_DEVERR_TIMEOUT).
 */
PKM_API int pkm_subkey_scores(const void* query, const void* keys, int dtype, int64_t n_tokens,
                      int64_t heads, int64_t k_dim, int64_t n_keys, int mode, void* scores,
                      uint32_t* dev_err, void* stream);

/*
 * K2 - product top-k over precomputed sub-key scores [rows, 2, n_keys].
 * Stage 1 keeps the knn best sub-keys of each half, stage 2 the knn best of
 * the knn*knn sums (pkm/memory.py:270-285, fwpkm/fwpkm.py:908-923).  Order:
 * score descending, ties to the lowest index (sub-key index, then slot).
 * Outputs (rows x knn): indices (slot, int64), top_scores (score dtype),
 * optional psw = per-row softmax of top_scores computed in fp32 and stored
 * in the score dtype (pkm/memory.py:218), and optional stage-1 lists
 * sub_indices1/2 (int64, sorted like the stage-1 top-k).
 * knn <= 32, knn <= n_keys <= 1024.
 */
PKM_API int pkm_product_topk(const void* scores, int dtype, int64_t rows, int64_t n_keys, int64_t knn,
                     int64_t* indices, void* top_scores, void* psw, int64_t* sub_indices1,
                     int64_t* sub_indices2, void* stream);

/*
 * Backward of the per-row softmax plus the sub-key bags used by the scoring
 * backward.  For each row r (= token*heads + h) of the product top-k:
 *   ds[r, j] = psw[r,j] * (dpsw[r,j] - sum_i psw[r,i] * dpsw[r,i])  (fp32)
 * and, for both halves p, the sub-key bag
 *   sub_idx[2r+p, j] = (h*2+p)*n_keys + (p ? slot % n_keys : slot / n_keys)
 *   sub_w[2r+p, j]   = ds[r, j]
 * so that d_query = bag_fwd(sub_idx, sub_w, keys) and d_keys =
 * bag_bwd(sub_idx, sub_w, grad_out = query) give the gradients of the
 * cartesian scores (pkm/memory.py:274-285).  group = knn for the PKM
 * per-head softmax.  Set psw NULL to pass dpsw through as ds (scores that
 * were not soft-maxed).
 */
PKM_API int pkm_score_bwd_prep(const int64_t* indices, const void* psw, const void* dpsw, int dtype,
                       int64_t rows, int64_t knn, int64_t heads, int64_t n_keys, int64_t* sub_idx,
                       void* sub_w, void* stream);

/*
 * Dense gradient of the sub-key scores [rows, 2, n_keys] from the gradient of
 * the product top-k outputs: the softmax backward of each row (skipped when
 * psw is NULL), rounded to the score dtype, scattered to the two sub-keys of
 * each selected slot and summed where slots share a sub-key.  This is the
 * gradient the reference's autograd forms through topk/gather/expand
 * (pkm/memory.py:218, 274-285); d_query and d_keys then follow by two dense
 * GEMMs per (head, half).  Every element of d_scores is written.
 */
PKM_API int pkm_score_grad_dense(const int64_t* indices, const void* psw, const void* dpsw, int dtype,
                                 int64_t rows, int64_t knn, int64_t n_keys, void* d_scores, void* stream);

/*
 * Score transform of the fast-weight memory over rows of `width` scores (one
 * token's H*knn top-k scores, jointly over the heads).  Replaces
 * FastWeightProductKeyMemory.score_transform (fwpkm/fwpkm.py:105-115):
 *   x = scores / temperature;  mode 0: out = softmax(x) over the row,
 *   mode 1: out = silu(x),  mode 2: out = relu(x);
 * fp32 arithmetic, out in the scores' dtype.  width <= 512.
 * The backward writes d_scores = d(out)/d(scores)^T grad_out; it reads `out`
 * for the softmax and `scores` for silu / relu (the other may be NULL).
 */
/*
 * Dense bf16 GEMM on the tensor cores (fp32 accumulate):
 *   C[b][m, n] = sum_k A[b][m, k] * B[b][n, k] + bias[n]      (b < batch)
 * Replaces the nn.Linear / matmul calls of the layer: the query projection
 * (pkm/memory.py:317-349), the SwiLU and value projections (:143-149,
 * 226-229) with their data and weight gradients, and the dense scoring
 * backward (:267-268).  A is a row-major bf16 matrix [a_rows, a_cols] with
 * row pitch lda elements, read K-major (A[m, k] at row m, column k) or
 * MN-major (A[m, k] at row k, column m); B likewise with n in place of m.
 * Batch b reads A shifted by (a_batch_x columns, a_batch_y rows), B by
 * (b_batch_x, b_batch_y), and writes C + b * c_batch_stride (row pitch ldc).
 * bias may be NULL.  C is bf16 or fp32.  K must be a multiple of 64 unless
 * it spans the operands' whole K extent (then the tail reads zeros); N a
 * multiple of 8, the column batch offsets multiples of 8, bases and row
 * pitches 16-byte aligned.  When the output tiles cannot fill the GPU the K
 * range is split and summed in a fixed order; pkm_gemm_workspace gives the
 * bytes of fp32 partials that needs (0 otherwise), the caller provides them.
 */
PKM_API int pkm_gemm_workspace(int64_t batch, int64_t M, int64_t N, int64_t K, size_t* bytes);
PKM_API int pkm_gemm_bf16(const void* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda,
                          const void* B, int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb,
                          int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_x, int64_t a_batch_y,
                          int64_t b_batch_x, int64_t b_batch_y, const void* bias, int bias_dtype, void* C,
                          int c_dtype, int64_t ldc, int64_t c_batch_stride, void* workspace,
                          size_t workspace_bytes, uint32_t* dev_err, void* stream);
/*
 * fp32 GEMM on the CUDA cores, same operand views and batching as
 * pkm_gemm_bf16 (no bias, fp32 C, any K, unsplit: no workspace):
 *   C[b][m, n] = sum_k A[b][m, k] * B[b][n, k]
 * Replaces the fp32 einsum / cdist gradients of the fast-weight memory's
 * sub-key scores (fwpkm/fwpkm.py:853-869: dS @ K and dS^T @ Q per (head, half)
 * group) and their second derivatives.  Elements outside the operands' row
 * and column extents read as 0.
 */
PKM_API int pkm_gemm_f32(const float* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda,
                         const float* B, int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb,
                         int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_x, int64_t a_batch_y,
                         int64_t b_batch_x, int64_t b_batch_y, float* C, int64_t ldc, int64_t c_batch_stride,
                         void* stream);
/*
 * The same with a workspace from pkm_gemm_f32_workspace: grids that the
 * tiles alone cannot fill split K into fp32 partials summed in split order
 * (the same results for every split count up to fp32 summation order; a
 * workspace smaller than the query's runs unsplit).
 */
PKM_API int pkm_gemm_f32_workspace(int64_t batch, int64_t M, int64_t N, int64_t K, size_t* bytes);
PKM_API int pkm_gemm_f32_ws(const float* A, int a_mn_major, int64_t a_rows, int64_t a_cols, int64_t lda,
                            const float* B, int b_mn_major, int64_t b_rows, int64_t b_cols, int64_t ldb,
                            int64_t batch, int64_t M, int64_t N, int64_t K, int64_t a_batch_x, int64_t a_batch_y,
                            int64_t b_batch_x, int64_t b_batch_y, float* C, int64_t ldc, int64_t c_batch_stride,
                            void* workspace, size_t workspace_bytes, void* stream);

/*
 * The SwiLU-gated value projection's GEMMs with the gate in their epilogue
 * (pkm/memory.py:226-229, value_proj(output * silu(swilu_projection(input)))):
 *   forward:  h = x @ ws^T + bs  and  z = a * silu(h)     (one GEMM, M x N)
 *   backward: dz = dy @ wv,  da = dz * silu(h),  dh = dz * a * silu'(h)
 * x [M, K] (pitch ldx), ws [N, K], a / h / z / da / dh [M, N] (pitch ld),
 * dy [M, K] (pitch ldy), wv [K, N] (pitch ldw); all bf16, every intermediate
 * rounded to bf16 where torch's eager ops round it (the same values as
 * pkm_gemm_bf16 followed by pkm_swiglu_fwd / pkm_swiglu_bwd).  bs may be
 * NULL; da may be NULL.  The bias gradient of ws is the column sum of dh
 * (pkm_colsum).  Constraints as pkm_gemm_bf16; no workspace.
 */
PKM_API int pkm_gemm_swiglu_fwd(const void* x, int64_t ldx, const void* ws, const void* bs, int bias_dtype,
                                const void* a, int64_t M, int64_t N, int64_t K, void* h, void* z, int64_t ld,
                                uint32_t* dev_err, void* stream);
PKM_API int pkm_gemm_swiglu_bwd(const void* dy, int64_t ldy, const void* wv, int64_t ldw, const void* a,
                                const void* h, int64_t M, int64_t N, int64_t K, void* dh, void* da, int64_t ld,
                                uint32_t* dev_err, void* stream);

/*
 * Test hook, no counterpart in the reference: the number of polls each
 * pipeline wait of pkm_gemm_bf16 may take before it gives up, sets
 * PKM_DEVERR_TIMEOUT in the error word and returns (a negative value
 * restores the default, 2^24; 0 gives up without polling).  Copies and MMAs
 * already in flight are still awaited with the default limit and TMEM is
 * released, so a short limit only ends the kernel early; its output is then
 * undefined.  Read by later launches.
 */
PKM_API int pkm_debug_set_wait_limit(int64_t polls);

/*
 * Test hook, no counterpart in the reference: which form pkm_gemm_bf16 (and
 * the fused SwiGLU GEMMs) run.  -1 (default): CTA pairs (clusters of two
 * CTAs sharing one 256-row MMA tile) when M > 128, single CTAs otherwise;
 * 0: single CTAs always; 1: CTA pairs always.  Both forms give the same
 * results; the split count, and with it pkm_gemm_workspace, may differ.
 * Read by later calls.
 */
PKM_API int pkm_debug_gemm_pair(int mode);

PKM_API int pkm_score_transform_fwd(const void* scores, int dtype, int64_t rows, int64_t width,
                                    double temperature, int mode, void* out, void* stream);
PKM_API int pkm_score_transform_bwd(const void* scores, const void* out, const void* grad_out, int dtype,
                                    int64_t rows, int64_t width, double temperature, int mode, void* grad_scores,
                                    void* stream);

/*
 * Data-parallel bag backward: K4 fused with the reduce-scatter of the table
 * gradient over NVLink.  Rank o owns table rows [o*shard_rows,
 * (o+1)*shard_rows) and holds a receive buffer [world][shard_rows][dim] (dtype
 * grad_weight_dtype) that every rank can store to (IPC or symmetric memory);
 * recv_bases is a HOST array of the world buffers' device addresses.  Instead
 * of writing a local dense gradient, the segment pass stores this rank's
 * gradient of row r into recv_bases[r / shard_rows] at row
 * rank*shard_rows + r % shard_rows while it computes, so the transfer overlaps
 * the pass.  Every other argument is pkm_bag_bwd's; world <= 8 (one NVLink
 * domain).  Replaces embedding_bag_bw_rev_indices
 * (pkm/xformer_embeddingbag.py:331-386) followed by the data-parallel
 * all-reduce of values.weight.grad (its reduce-scatter half).
 */
PKM_API int pkm_bag_bwd_sharded(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                                int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                                int64_t num_rows, int64_t dim, void* const* recv_bases, int world, int rank,
                                int64_t shard_rows, int grad_weight_dtype, void* grad_psw, int grad_psw_dtype,
                                int32_t* row_counts, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                                void* stream);

/*
 * Owner side of the exchange (the all-gather half): sums the world partial
 * copies of this rank's shard in its receive buffer `recv` in source order
 * 0..world-1 (bf16 as packed pairs, each addition rounded to bf16 like a
 * bf16 all-reduce; fp32 in fp32), multiplies by `scale` (1/world averages),
 * and stores the
 * rows into rows [rank*shard_rows, ...) of every rank's gradient
 * grad_bases[d] (HOST array of world peer-writable device addresses).
 * max_blocks > 0 bounds the grid so that the kernel can run beside the rest
 * of the backward on another stream.  The caller orders this after every
 * rank's pkm_bag_bwd_sharded (a barrier), and readers of the gradient after
 * every rank's pkm_grad_shard_reduce (a second barrier).  dtype f32 or bf16.
 */
PKM_API int pkm_grad_shard_reduce(const void* recv, int dtype, int64_t num_rows, int64_t dim, int world, int rank,
                                  int64_t shard_rows, void* const* grad_bases, float scale, int max_blocks,
                                  void* stream);

/*
 * Row-owner optimizer step of a replicated table (reduce-scatter -> owner
 * update -> all-gather of parameters): sums this rank's shard copies in
 * `recv` like pkm_grad_shard_reduce, scales by `scale`, applies SGD
 * without momentum to this rank's rows of the table,
 *   d = g + weight_decay * p (rounded to the table dtype; skipped when 0),
 *   p' = p - lr * d (one fused multiply-add, rounded once),
 * the foreach update of torch.optim.SGD, and stores the new rows into rows
 * [rank*shard_rows, ...) of every rank's table table_bases[d] (HOST array
 * of world peer-writable addresses; table_bases[rank] is read first).
 * Ordering as pkm_grad_shard_reduce: after every rank's
 * pkm_bag_bwd_sharded, and readers of the table after every rank's call.
 * Replaces the all-reduce of values.weight.grad plus every rank's full-table
 * optimizer pass.  dtype f32 or bf16.
 */
PKM_API int pkm_grad_shard_sgd(const void* recv, int dtype, int64_t num_rows, int64_t dim, int world, int rank,
                               int64_t shard_rows, void* const* table_bases, float lr, float weight_decay,
                               float scale, int max_blocks, void* stream);

/*
 * pkm_bag_bwd in phases on one workspace: pkm_bag_bwd_sort runs the keys,
 * scan, radix sort and chunk descriptors (and zeroes grad_psw of invalid
 * indices, fills row_counts); pkm_bag_bwd_rows then runs the segment pass
 * and the partial-row sums for the table rows [row_begin, row_end) only,
 * writing those rows of grad_weight and grad_psw of their occurrences.  Each
 * row range once, after the sort; together they equal pkm_bag_bwd.  Lets a
 * caller start exchanging finished rows while later rows are computed.
 */
PKM_API int pkm_bag_bwd_sort(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                             int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                             int64_t num_rows, int64_t dim, void* grad_psw, int grad_psw_dtype, int32_t* row_counts,
                             void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream);
PKM_API int pkm_bag_bwd_rows(const int64_t* indices, const void* psw, int psw_dtype, const void* weight,
                             int weight_dtype, const void* grad_out, int64_t n_bags, int64_t bag_size,
                             int64_t num_rows, int64_t dim, int64_t row_begin, int64_t row_end, void* grad_weight,
                             int grad_weight_dtype, void* grad_psw, int grad_psw_dtype, void* workspace,
                             size_t workspace_bytes, uint32_t* dev_err, void* stream);

/*
 * Routing around the all-to-all of the row-sharded embedding bag (the
 * reference's bag, pkm/xformer_embeddingbag.py:97-138 and :331-386, with
 * the table split by rows: rank o owns rows [o*shard_rows, (o+1)*shard_rows)).
 * pkm_route_pack: owner = indices[e] / shard_rows for the n = n_bags *
 *   bag_size occurrences; a stable partition by owner.  Writes, per packed
 *   position p: order[p] (the occurrence), local_row[p] (its row inside the
 *   owner's shard), weight[p] (psw as fp32, 1 when psw is NULL), bag[p]
 *   (occurrence / bag_size); send_counts[o] (int64 [world]) = entries for
 *   owner o.  Indices outside [0, world*shard_rows) set PKM_DEVERR_INDEX, are
 *   not counted and sort after the last owner.  world <= 255.
 * pkm_route_segments: entries grouped by group_counts (device int64
 *   [groups]) with bags ascending inside each group (true of a pack's output
 *   and of what the all-to-all delivers); one segment per run of equal bag
 *   inside a group.  Writes seg_of[e], seg_start[s] (int64, with
 *   seg_start[n_seg] = n: the offsets pkm_segment_sum takes), seg_bag[s] and
 *   seg_counts[g] (int64 [groups]).  Arrays sized for n entries / n segments.
 * pkm_route_combine: out[b] (n_bags x dim, out_dtype) = the partial rows
 *   [n_seg, dim] of bag b's segments (at most one per group; segments grouped
 *   by seg_counts) summed in group order in fp32 from zero, rounded once;
 *   bags without segments are zero.
 * Workspaces: the *_workspace sizes, 256-byte aligned.
 */
PKM_API int pkm_route_pack_workspace(int64_t n, size_t* bytes);
PKM_API int pkm_route_pack(const int64_t* indices, const void* psw, int psw_dtype, int64_t n_bags, int64_t bag_size,
                           int64_t shard_rows, int world, int64_t* send_counts, int32_t* order, int32_t* local_row,
                           float* weight, int32_t* bag, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                           void* stream);
PKM_API int pkm_route_segments_workspace(int64_t n, size_t* bytes);
PKM_API int pkm_route_segments(const int32_t* bag, int64_t n, const int64_t* group_counts, int groups,
                               int32_t* seg_of, int64_t* seg_start, int32_t* seg_bag, int64_t* seg_counts,
                               void* workspace, size_t workspace_bytes, void* stream);
PKM_API int pkm_route_combine_workspace(int groups, int64_t n_bags, size_t* bytes);
PKM_API int pkm_route_combine(const void* partial, int dtype, int64_t n_seg, int64_t dim, const int32_t* seg_bag,
                              const int64_t* seg_counts, int groups, int64_t n_bags, void* out, int out_dtype,
                              void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream);

/*
 * Ragged entry lists, for tables sharded by rows over ranks (each owner
 * serves the entries that other ranks route to it):
 * pkm_segment_sum: out[s] = sum over entries e in [seg_offsets[s],
 *   seg_offsets[s+1]) of entry_w[e] * rows[entry_row[e]] (fp32, entry order);
 *   the forward of an embedding bag whose bags have different sizes.
 *   Workspace: pkm_segment_sum_workspace(n_segs) bytes, 256-byte aligned.
 * pkm_bag_bwd_ragged: pkm_bag_bwd where entry e's upstream gradient is row
 *   src_of[e] of grad_rows [n_src, dim] (instead of bag e / bag_size);
 *   row_idx [n_entries] are the table rows.  Workspace:
 *   pkm_bag_bwd_workspace(n_entries, 1, num_rows, dim).
 * Replace the shard-local parts of the row-sharded embedding bag (the
 * reference's bag, pkm/xformer_embeddingbag.py:97-138 and :331-386, with the
 * table split over ranks).
 */
PKM_API int pkm_segment_sum_workspace(int64_t n_segs, size_t* bytes);
PKM_API int pkm_segment_sum(const void* rows, int row_dtype, int64_t num_rows, int64_t dim, const int32_t* entry_row,
                            const float* entry_w, int64_t n_entries, const int64_t* seg_offsets, int64_t n_segs,
                            void* out, int out_dtype, void* workspace, size_t workspace_bytes, uint32_t* dev_err,
                            void* stream);
PKM_API int pkm_bag_bwd_ragged(const int64_t* row_idx, const int32_t* src_of, const void* psw, int psw_dtype,
                               const void* weight, int weight_dtype, const void* grad_rows, int64_t n_entries,
                               int64_t n_src, int64_t num_rows, int64_t dim, void* grad_weight,
                               int grad_weight_dtype, void* grad_psw, int grad_psw_dtype, int32_t* row_counts,
                               void* workspace, size_t workspace_bytes, uint32_t* dev_err, void* stream);

/*
 * In-switch all-reduce of a table gradient over NVLink SHARP (NVLS): every
 * rank's gradient [num_rows, dim] sits in one symmetric buffer whose
 * multicast address is mc_src; the owner of rows [rank*shard_rows, ...)
 * reads each 16-byte vector of them with multimem.ld_reduce (the switch
 * returns the sum over ranks; bf16 accumulated in fp32) and stores it, times
 * `scale`, with multimem.st at the same offset of mc_dst (the multicast
 * address of the gradient buffers), which writes every rank's copy.  Only the
 * rows of its shard inside [row_begin, row_end) (row_end < 0: all), so the
 * table can be exchanged in row ranges.  Called by every rank for its own
 * shard, between two barriers (after every rank's rows of the range are
 * written, before any rank reads the result).  Replaces the data-parallel
 * all-reduce of values.weight.grad.
 */
PKM_API int pkm_grad_multimem_allreduce(const void* mc_src, void* mc_dst, int dtype, int64_t num_rows,
                                        int64_t dim, int world, int rank, int64_t shard_rows, int64_t row_begin,
                                        int64_t row_end, float scale, int max_blocks, void* stream);

/*
 * SwiGLU gate of the memory output (pkm/memory.py:226-229: output *
 * silu(swilu_projection(input))) on row-major [n, c] tensors (f32 or bf16,
 * c a multiple of 8, 16-byte aligned), one pass each way:
 *   pkm_swiglu_fwd: z = a * silu(h)
 *   pkm_swiglu_bwd: da = dz * silu(h) (NULL to skip), dh = silu'(h)-chain of
 *     dz * a, and dbias = column sums of dh (the gate projection's bias
 *     gradient; NULL to skip; needs pkm_colsum_workspace bytes)
 * with every intermediate rounded to the activation dtype where torch's eager
 * ops round it.  pkm_colsum: out[c] = sum over rows (fixed order; the bias
 * gradient of an nn.Linear).
 */
PKM_API int pkm_colsum_workspace(int64_t n, int64_t c, size_t* bytes);
PKM_API int pkm_swiglu_fwd(const void* a, const void* h, int dtype, int64_t n, int64_t c, void* z, void* stream);
PKM_API int pkm_swiglu_bwd(const void* dz, const void* a, const void* h, int dtype, int64_t n, int64_t c, void* da,
                           void* dh, void* dbias, int bias_dtype, void* workspace, size_t workspace_bytes,
                           void* stream);
PKM_API int pkm_colsum(const void* x, int dtype, int64_t n, int64_t c, void* out, int out_dtype, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * Addressing statistics of a batch of slot indices, on the device, replacing
 * Qwen3PKMDecoderLayer.compute_addr_stats (modeling_qwen3pkm.py:447-471)
 * without its .item() synchronisations.  With counts = bincount(indices)
 * over [0, rows), writes four doubles to the device array out:
 *   out[0] = sum of counts[k] over slots with counts[k] > 1  (collided)
 *   out[1] = number of slots with counts[k] > 0              (covered)
 *   out[2] = KL(counts / n_indices || uniform over rows), with the
 *            probabilities clamped to [eps, 1 - eps] inside the logs and
 *            zero-probability terms dropped, as torch.distributions does
 *   out[3] = number of indices counted (n_indices unless some were outside
 *            [0, rows), which also sets PKM_DEVERR_INDEX)
 * so collision_ratio = out[0] / (n_indices + 1e-6) and coverage_ratio =
 * out[1] / rows.  n_indices must be positive (the reference's Categorical
 * rejects an empty histogram).  The workspace (pkm_addr_stats_workspace
 * bytes, 256-byte aligned) holds the int32 bins and per-block partials; the
 * reduction order is fixed, so results are bit-reproducible.
 */
PKM_API int pkm_addr_stats_workspace(int64_t rows, size_t* bytes);
PKM_API int pkm_addr_stats(const int64_t* indices, int64_t n_indices, int64_t rows, double* out, void* workspace,
                           size_t workspace_bytes, uint32_t* dev_err, void* stream);

/*
 * Fused FwPKM value update: one SGD step of the fast-weight inner loop on the
 * value table [rows, dim] (f32 or bf16), replacing the value branch of
 * update_fw (fwpkm/fwpkm.py:274-367, update_fw_param :266-272):
 *   counts = bincount(indices)          (int32 [rows], caller's buffer)
 *   scaled = grad * scale / max(counts, 1)
 *   new    = values - lr * (u + weight_decay * values),
 *   u      = clamp(scaled, -1, 1) if grad_clip else scaled
 * each operation rounded to the table dtype as torch's eager ops round, so
 * f32 results equal the reference's bit for bit.  scaled_grad may be NULL.
 * Indices outside [0, rows) set PKM_DEVERR_INDEX and are not counted.
 * pkm_fw_update_bwd: d_values = d_new * (1 - lr * weight_decay), d_grad =
 * (scale / max(counts, 1)) * (d_scaled - lr * d_new * [|scaled| <= 1 when
 * clipping]); d_scaled_grad, d_values, d_grad may be NULL.
 */
PKM_API int pkm_fw_update(const void* values, const void* grad, int dtype, int64_t rows, int64_t dim,
                          const int64_t* indices, int64_t n_indices, double scale, double lr, double weight_decay,
                          int grad_clip, void* new_values, void* scaled_grad, int32_t* counts, uint32_t* dev_err,
                          void* stream);
PKM_API int pkm_fw_update_bwd(const void* d_new_values, const void* d_scaled_grad, const void* scaled_grad,
                              const int32_t* counts, int dtype, int64_t rows, int64_t dim, double scale,
                              double lr, double weight_decay, int grad_clip, void* d_values, void* d_grad,
                              void* stream);

/*
 * Batch normalisation of the query projection, x [n, c] row-major (rows =
 * tokens, c a multiple of 8, x / out / dy / dx 16-byte aligned; x f32 or
 * bf16).  Replaces the query network's nn.BatchNorm1d(heads * k_dim,
 * eps=1e-6, momentum=0.1) (pkm/memory.py:308-309), i.e. ATen's
 * native_batch_norm (training and evaluation) and
 * native_batch_norm_backward.
 *
 * pkm_batchnorm_fwd, training != 0: batch statistics (biased variance for
 * the normalisation), save_mean / save_rstd [c] fp32 receive the mean and
 * 1/sqrt(var + eps), and running_mean / running_var (either may be NULL) are
 * updated with `momentum` and the unbiased variance.  training == 0: the
 * running statistics normalise, save_* receive them (mean, 1/sqrt(var +
 * eps)), and no workspace is needed.  weight / bias (p_dtype) may be NULL.
 * pkm_batchnorm_bwd: from the saved statistics, dx (NULL to skip), dweight
 * and dbias (p_dtype, NULL to skip).  Both reduce in a fixed order: results
 * are deterministic.
 */
PKM_API int pkm_batchnorm_workspace(int64_t n, int64_t c, size_t* bytes);
PKM_API int pkm_batchnorm_fwd(const void* x, int x_dtype, int64_t n, int64_t c, const void* weight,
                              const void* bias, int p_dtype, void* running_mean, void* running_var,
                              int r_dtype, int training, double momentum, double eps, void* out,
                              float* save_mean, float* save_rstd, void* workspace, size_t workspace_bytes,
                              void* stream);
PKM_API int pkm_batchnorm_bwd(const void* dy, const void* x, int x_dtype, int64_t n, int64_t c,
                              const float* save_mean, const float* save_rstd, const void* weight,
                              int p_dtype, void* dx, void* dweight, void* dbias, void* workspace,
                              size_t workspace_bytes, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* PKM_B200_H */
