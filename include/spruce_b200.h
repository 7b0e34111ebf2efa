/*
 * spruce_b200.h -- C ABI of the B200 (sm_100a) SPRUCE sparse-prefill path.
 *
 * Plain pointers, element strides and sizes; no torch or CUDA types.  All
 * pointers are device pointers unless noted, `stream` is a cudaStream_t (NULL
 * = legacy default stream).  No entry point allocates device memory or
 * synchronises the stream: work is enqueued and the call returns.  Inputs are
 * borrowed; outputs are written in place.
 *
 * Return value: SPRUCE_OK or an SPRUCE_ERR_* code; spruce_last_error() gives
 * the calling thread's message for the last failure.  The Python layer maps
 * SPRUCE_ERR_INVALID / SPRUCE_ERR_UNSUPPORTED to ValueError and the rest to
 * RuntimeError, as the reference raises ValueError for contract violations
 * (kernels/seerattention_direct_index_triton.py:350-372).
 *
 * Shapes follow the reference's tensors: q [B, Hq, T, D], k/v [B, Hkv, T, D]
 * (any strides with a unit last stride, e.g. views of token-major
 * [B, T, H, D] projections), selected_blocks int32 [B, L, G, qb, K] with
 * qb = ceil(T / 64) and G = Hkv (interfaces/selected_blocks_spec.md).
 */
#ifndef SPRUCE_B200_H
#define SPRUCE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPRUCE_OK 0
#define SPRUCE_ERR_INVALID 1     /* argument violates the contract         */
#define SPRUCE_ERR_UNSUPPORTED 2 /* outside the kernels' coverage           */
#define SPRUCE_ERR_CUDA 3        /* CUDA runtime / driver error             */
#define SPRUCE_ERR_WORKSPACE 4   /* workspace smaller than required         */

/* Bits kernels OR into the optional device status word (uint32). */
#define SPRUCE_STATUS_TIMEOUT 1u   /* a bounded pipeline wait ran out       */
#define SPRUCE_STATUS_EMPTY_ROW 2u /* a selected_blocks row had no block    */

#define SPRUCE_DTYPE_F32 0
#define SPRUCE_DTYPE_BF16 1
#define SPRUCE_DTYPE_F16 2

#define SPRUCE_BLOCK 64 /* tokens per block; the reference's kernels require 64 */

#if defined(__GNUC__)
#define SPRUCE_API __attribute__((visibility("default")))
#else
#define SPRUCE_API
#endif

/* Message for the calling thread's last failed call ("" if none). */
SPRUCE_API const char *spruce_last_error(void);

/* ABI version of this library (bumped on any signature change). */
SPRUCE_API int spruce_abi_version(void);

/*
 * _group_avg_tokens, teacher/chunked_extract.py:75-80: average the H/G query
 * heads of each group per token.  x [B, H, T, D] with element strides
 * x_strides[4]; out [B, G, T, D] contiguous, same dtype.  Bit-exact with the
 * reference: fp32 sum over heads in order, fp32 divide, one rounding.
 */
SPRUCE_API int spruce_group_avg_tokens(const void *x, const int64_t x_strides[4], int dtype, int64_t B, int64_t H,
                            int64_t T, int64_t D, int64_t G, void *out, void *stream);

/*
 * _proto_pool_seq, teacher/chunked_extract.py:27-72:
 * x [B, H, T, D] (strided) -> out [B, H, nb, P, D] contiguous, nb =
 * ceil(T / block), block = 64.  Prototype 0 is the block mean, bit-exact with
 * the reference's rounding points (16-row fp32 partial sums, sum rounded to
 * dtype, divided by the real row count of the block); prototypes 1..P-1 are
 * the rows farthest from it (fp32 squared L2, descending, ties to the lower
 * row), the mean where a ragged block has no further row.  1 <= P <= 64.
 */
SPRUCE_API int spruce_proto_pool(const void *x, const int64_t x_strides[4], int dtype, int64_t B, int64_t H, int64_t T,
                      int64_t D, int64_t block, int64_t P, void *out, void *stream);

/*
 * Selector inputs of one layer in one launch: pooled_q = block mean of the
 * group-averaged queries, pooled_k = block mean of the keys, both
 * [B, Hkv, qb, D] contiguous in the input dtype.  Equivalent to
 * _proto_pool_seq(_group_avg_tokens(q, Hkv), 64, 1) and
 * _proto_pool_seq(k, 64, 1) (teacher/chunked_extract.py:170-171).
 */
SPRUCE_API int spruce_pool_qk(const void *q, const int64_t q_strides[4], const void *k, const int64_t k_strides[4],
                   int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, void *pooled_q,
                   void *pooled_k, void *stream);

/*
 * The selector's prototype features with P prototypes per block
 * (teacher/chunked_extract.py:27-72 on _group_avg_tokens(q) and on k):
 * prototype 0 is the block mean (exactly as spruce_pool_qk), prototypes
 * 1..P-1 are the block's rows farthest (fp32 squared L2) from that mean, in
 * descending distance, ties to the lower row; slots a ragged last block cannot
 * fill repeat the mean.  pooled_q / pooled_k [B, Hkv, ceil(T/64), P, D]
 * contiguous in the input dtype.  1 <= P <= 64 (spruce_proto_pool takes the
 * same P for one tensor).
 */
SPRUCE_API int spruce_pool_qk_protos(const void *q, const int64_t q_strides[4], const void *k,
                                     const int64_t k_strides[4], int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                                     int64_t T, int64_t D, int64_t P, void *pooled_q, void *pooled_k, void *stream);

/*
 * FlatGate projection, selector/gate.py:120-127 (project_queries /
 * project_keys) and :47-48: out[n, :] = fp32(x[n, :]) @ W, x [N, D] contiguous
 * in dtype, W [D, P] fp32 contiguous, out [N, P] fp32.  Fixed fma order over D.
 */
SPRUCE_API int spruce_gate_project(const void *x, int dtype, int64_t N, int64_t D, const float *W, int64_t P, float *out,
                        void *stream);

/*
 * FlatGate.forward with one prototype, selector/gate.py:80-101:
 * out[r, i, j] = (qp[r, i, :] . kp[r, j, :]) / sqrt(P) for R score matrices
 * (layers x groups), qp [R, qb, P], kp [R, kb, P], out [R, qb, kb], fp32.
 */
SPRUCE_API int spruce_gate_scores(const float *qp, const float *kp, int64_t R, int64_t qb, int64_t kb, int64_t P,
                       float *out, void *stream);

/*
 * MaxSim gate scores (selector/gate.py:29-101 forward, :104-117 and
 * :132-171 candidate scoring): qp [R, nq, P, pdim], kp [R, nk, P, pdim] fp32
 * projected prototypes (spruce_gate_project of each prototype row);
 *   out[r, q, c] = max over (i, j) of qp[r,q,i,:] . kp[r,key,j,:] / sqrt(pdim)
 * with key = c for every c < nk (ids == NULL, ncols == nk: the full score
 * matrix) or key = ids[r, q, c] clamped to [0, nk) (int64 candidate node ids,
 * ncols per row).  Each dot is one fp32 fma chain in index order; with P = 1
 * the result equals spruce_gate_scores.  1 <= P <= 8.  out fp32 [R, nq, ncols].
 */
SPRUCE_API int spruce_gate_maxsim(const float *qp, const float *kp, const int64_t *ids, int64_t R, int64_t nq,
                                  int64_t nk, int64_t ncols, int64_t P, int64_t pdim, float *out, void *stream);

/*
 * Key tree of the deployed selector (selector/tree.py:80-145): one level up.
 * child [R, nchild, P, d] in dtype -> parent [R, ceil(nchild / radix), P, d]:
 * prototype 0 = mean of the (up to radix) children's prototype 0, formed in
 * dtype as the reference does; prototypes 1..P-1 = the children's prototypes
 * farthest from it (distance in dtype), descending, ties to the lower
 * candidate.  1 <= P <= 8, radix >= 2, radix * P <= 256.
 */
SPRUCE_API int spruce_tree_merge(const void *child, int dtype, int64_t R, int64_t nchild, int64_t P, int64_t d,
                                 int64_t radix, void *parent, void *stream);

/*
 * One traversal level (scripts/eval_tree_traversal.py:83-108): the children
 * of each row's selected nodes.  selected int64 [R, nq, S] (-1 = none),
 * child_starts int64 [nchild] (first leaf block of each child) ->
 * cand int64 [R, nq, S * radix] (ids to score: invalid ones clamped) and
 * valid uint8 (parent selected, child exists, child starts at or before the
 * row's block q).  S * radix <= 256.
 */
SPRUCE_API int spruce_tree_candidates(const int64_t *selected, int64_t R, int64_t nq, int64_t S, int64_t radix,
                                      int64_t nchild, const int64_t *child_starts, int64_t *cand, uint8_t *valid,
                                      void *stream);

/*
 * The level's beam (:105-108): per row, the k best of C candidates by score
 * (invalid ones count as the fp32 minimum), descending, ties to the lower
 * position; out int64 [rows, k] = the candidate id, or -1 where it is
 * invalid.  C <= 256, 1 <= k <= C.
 */
SPRUCE_API int spruce_tree_topk(const float *scores, const uint8_t *valid, const int64_t *cand, int64_t rows,
                                int64_t C, int64_t k, int64_t *out, void *stream);

/*
 * Fused flat-gate selection: scores (as spruce_gate_scores), causal /
 * sink / local-window masking, top-W with W = K - (local_window + 1) -
 * sink_blocks (ties to the lowest block id) and packing to selected_blocks
 * rows, without materialising the score matrix.  Equivalent to
 * topk + selected_ids_to_blocks(ids, K, local_window, key_blocks=qb,
 * sink_blocks) (scripts/route_overrides.py:187-205,
 * scripts/export_selected_blocks.py:80-175).  qp/kp [B, G, qb, P] fp32
 * contiguous; row (b, g, q) is written at out + b*out_strides[0] +
 * g*out_strides[1] + q*out_strides[2] (K contiguous int32).
 */
SPRUCE_API int spruce_gate_select(const float *qp, const float *kp, int64_t B, int64_t G, int64_t qb, int64_t P, int64_t K,
                       int64_t local_window, int64_t sink_blocks, int32_t *out, const int64_t out_strides[3],
                       void *stream);

/*
 * spruce_gate_select restricted to query blocks [q_block_begin, q_block_end):
 * only those rows of `out` are written (a GPU that attends a query-block range
 * of a layer selects just those rows).
 */
SPRUCE_API int spruce_gate_select_rows(const float *qp, const float *kp, int64_t B, int64_t G, int64_t qb, int64_t P,
                                       int64_t K, int64_t local_window, int64_t sink_blocks, int32_t *out,
                                       const int64_t out_strides[3], int64_t q_block_begin, int64_t q_block_end,
                                       void *stream);

/* Bytes of workspace spruce_select_blocks needs for this shape; -1 for an
 * invalid shape or a size that would not fit in int64. */
SPRUCE_API int64_t spruce_select_workspace_bytes(int64_t B, int64_t Hkv, int64_t T, int64_t D, int64_t P, int dtype);

/*
 * Whole flat selector for one layer: spruce_pool_qk -> spruce_gate_project
 * (Wq, Wk [D, P] fp32) -> spruce_gate_select.  Pooled features and
 * projections live in the caller's `workspace` (see
 * spruce_select_workspace_bytes).
 */
SPRUCE_API int spruce_select_blocks(const void *q, const int64_t q_strides[4], const void *k, const int64_t k_strides[4],
                         int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const float *Wq,
                         const float *Wk, int64_t P, int64_t K, int64_t local_window, int64_t sink_blocks,
                         int32_t *out, const int64_t out_strides[3], void *workspace, int64_t workspace_bytes,
                         void *stream);

/*
 * spruce_select_blocks for query blocks [q_block_begin, q_block_end) only:
 * pools just the query blocks of the range and the key blocks before its end,
 * projects those rows and selects those rows of `out` (same workspace size).
 */
SPRUCE_API int spruce_select_blocks_rows(const void *q, const int64_t q_strides[4], const void *k,
                                         const int64_t k_strides[4], int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                                         int64_t T, int64_t D, const float *Wq, const float *Wk, int64_t P, int64_t K,
                                         int64_t local_window, int64_t sink_blocks, int32_t *out,
                                         const int64_t out_strides[3], int64_t q_block_begin, int64_t q_block_end,
                                         void *workspace, int64_t workspace_bytes, void *stream);

/*
 * spruce_select_blocks without a caller workspace; it has no counterpart in
 * the reference.  It exists for callers that cannot allocate device memory for
 * us: hosts that reserve the GPU's memory up front in their own pool (a
 * serving process that hands nearly all HBM to its KV cache at start-up) and
 * plugin bindings that pass only the input and output buffers they own.
 * Scratch comes from one static device array of
 * spruce_select_noalloc_max_scratch_bytes() bytes (16 MiB) that every GPU
 * loading this library holds until the process exits; shapes needing more
 * (spruce_select_workspace_bytes) are rejected with SPRUCE_ERR_UNSUPPORTED.
 * No cudaMalloc, cudaFree or allocating library routine is called.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * All calls share the one array: calls that overlap on the GPU (different
 * streams, or other host threads) race on it; serialise them.  The looked-up
 * address is kept per device for the life of the process, so do not use this
 * entry point across a cudaDeviceReset (which tears down the module that holds
 * the array).  Shapes whose scratch size does not fit in int64 are rejected
 * with SPRUCE_ERR_INVALID before any device work.
 */
SPRUCE_API int spruce_select_blocks_noalloc(const void *q, const int64_t q_strides[4], const void *k,
                                            const int64_t k_strides[4], int dtype, int64_t B, int64_t Hq,
                                            int64_t Hkv, int64_t T, int64_t D, const float *Wq, const float *Wk,
                                            int64_t P, int64_t K, int64_t local_window, int64_t sink_blocks,
                                            int32_t *out, const int64_t out_strides[3], void *stream);

/* Size of the static scratch array spruce_select_blocks_noalloc uses. */
SPRUCE_API int64_t spruce_select_noalloc_max_scratch_bytes(void);

/*
 * selected_ids_to_blocks, scripts/export_selected_blocks.py:80-175:
 * ids [R, qb, C] int64 (R = layers x groups, contiguous) -> out [R, qb, K]
 * int32.  Same policy: forced local window and sink blocks, deduplicated
 * causal nonlocal ids of which the smallest fill the remaining slots,
 * sorted, -1 padded.
 */
SPRUCE_API int spruce_pack_selected_ids(const int64_t *ids, int64_t R, int64_t qb, int64_t C, int64_t K,
                             int64_t local_window, int64_t key_blocks, int64_t sink_blocks, int32_t *out,
                             void *stream);

/*
 * validate_selected_blocks rules, interfaces/validator.py:7-62, on the GPU:
 * sel [B, L, G, qb, K] int32 contiguous.  Writes to result[0] (device int64)
 * the smallest violating row (b, l, g, q) flattened, times 8, plus the first
 * violated rule (1 causal, 2 unsorted, 3 duplicate, 4 missing local block,
 * 5 non-trailing pad), or -1 if the tensor is valid.  The host formats the
 * reference's AssertionError message from that row.
 */
SPRUCE_API int spruce_validate_selected_blocks(const int32_t *sel, int64_t B, int64_t L, int64_t G, int64_t qb, int64_t K,
                                    int64_t local_window, int64_t *result, void *stream);

/*
 * Causal GQA block-sparse attention over selected key blocks,
 * kernels/seerattention_direct_index_triton.py:339-416 (and the math of
 * sparse/attention.py:143-274).  q [B, Hq, T, D], k/v [B, Hkv, T, D] with
 * element strides *_strides[4] (unit last stride); indices [B, Hkv, qb, Kw]
 * int32 with strides idx_strides[4] (unit last stride), -1 = padding;
 * out is written through the LOGICAL [B, Hq, T, D] strides out_strides[4]
 * (pass the strides of a [B, T, Hq, D] tensor viewed as [B, Hq, T, D] to get
 * the reference's token-major output).  scale multiplies q.k (D**-0.5 in the
 * reference).  bf16/fp16 run the tcgen05 kernel (D in {64, 128}); fp32 runs
 * a CUDA-core fp32 kernel.  Block ids < 0 are skipped and ids above the query
 * block contribute nothing (causal mask); a row left empty yields zeros and
 * raises SPRUCE_STATUS_EMPTY_ROW in *status when status is not NULL.
 */
SPRUCE_API int spruce_sparse_attention_fwd(const void *q, const int64_t q_strides[4], const void *k,
                                const int64_t k_strides[4], const void *v, const int64_t v_strides[4],
                                const int32_t *indices, const int64_t idx_strides[4], void *out,
                                const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                                int64_t T, int64_t D, int64_t Kw, float scale, uint32_t *status, void *stream);

/*
 * spruce_sparse_attention_fwd restricted to query blocks [q_block_begin,
 * q_block_end): only those output rows are written.  Used to split one
 * layer's query blocks across GPUs; the block ids keep their absolute values.
 */
SPRUCE_API int spruce_sparse_attention_fwd_rows(const void *q, const int64_t q_strides[4], const void *k,
                                                const int64_t k_strides[4], const void *v,
                                                const int64_t v_strides[4], const int32_t *indices,
                                                const int64_t idx_strides[4], void *out,
                                                const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq,
                                                int64_t Hkv, int64_t T, int64_t D, int64_t Kw, float scale,
                                                int64_t q_block_begin, int64_t q_block_end, uint32_t *status,
                                                void *stream);

/*
 * spruce_sparse_attention_fwd_rows with the output all-gather fused into the
 * kernel's epilogue, for layers whose query heads are split across GPUs (in
 * place of an NCCL all-gather of the per-head outputs: NVLink peer stores made
 * while the attention runs).  Each output row is written to
 * `out` and, at the same element offset, to every `peer_outs[i]` (n_peers <=
 * 7): device pointers of identically laid out tensors on the other GPUs,
 * mapped into this process (CUDA IPC) with peer access.  Plain stores; no
 * multicast.  The caller orders the peers' reads after every rank's kernel
 * (e.g. a collective on the same stream).  bf16/fp16 only.
 */
SPRUCE_API int spruce_sparse_attention_fwd_scatter(const void *q, const int64_t q_strides[4], const void *k,
                                                   const int64_t k_strides[4], const void *v,
                                                   const int64_t v_strides[4], const int32_t *indices,
                                                   const int64_t idx_strides[4], void *out,
                                                   const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq,
                                                   int64_t Hkv, int64_t T, int64_t D, int64_t Kw, float scale,
                                                   int64_t q_block_begin, int64_t q_block_end,
                                                   const void *const *peer_outs, int32_t n_peers, uint32_t *status,
                                                   void *stream);

/*
 * Host-only CUDA IPC plumbing for the fused output all-gather (no counterpart
 * in the reference, which is single-GPU).  spruce_ipc_export writes the
 * 64-byte cudaIpcMemHandle of the allocation holding `ptr` to `handle` and
 * ptr's byte offset in it; spruce_ipc_import opens a peer's handle in the
 * CURRENT device's context with lazy peer access and returns the mapped
 * pointer (base + offset) and the mapping base for spruce_ipc_close.  They map
 * existing memory; nothing is allocated.
 */
SPRUCE_API int spruce_ipc_export(const void *ptr, void *handle, int64_t *offset);
SPRUCE_API int spruce_ipc_import(const void *handle, int64_t offset, void **ptr, void **base);
SPRUCE_API int spruce_ipc_close(void *base);

/*
 * Self-check hook with no counterpart in the reference.  The attention
 * softmax computes part of its exponentials with a polynomial on the FMA pipe
 * (Cody-Waite reduction, a degree-3 polynomial fitted for this library) and the
 * rest with the MUFU ex2.approx instruction.  This evaluates both over x[0..n)
 * (device pointers, fp32) into poly_out / mufu_out, so tests can check the
 * polynomial's error bound and its agreement with MUFU after bf16 rounding.
 */
SPRUCE_API int spruce_exp2_selfcheck(const float *x, int64_t n, float *poly_out, float *mufu_out, void *stream);

/* Maximal residual frontiers (interfaces/residual_summaries.py:122-220, build_residual_summary_nodes
 * and residual_frontier_for_row): for each row of selected [rows, K] (int32, contiguous, -1 padded;
 * row r is query block r % qb) the ID-sorted tree nodes that cover exactly the causal blocks the row
 * leaves out, written to out [rows, S] with -1 padding.  The tree is ResidualTreeLayout's node table:
 * node_starts / node_ends int64 [num_nodes] block ranges and node_parents int32 [num_nodes] (-1 for
 * the root).  out may be NULL for a counting pass: row_counts [rows] (optional) receives each row's
 * frontier size and *max_count (optional, zeroed by the caller) the largest. */
SPRUCE_API int spruce_residual_frontier(const int32_t *selected, int64_t rows, int64_t K, int64_t qb,
                                        const int64_t *node_starts, const int64_t *node_ends,
                                        const int32_t *node_parents, int64_t num_nodes, int32_t *out, int64_t S,
                                        int32_t *row_counts, int32_t *max_count, void *stream);

/* Residual-summary attention (sparse/attention.py:83-274 with residual_summaries=True,
 * replacing its per-(query block, KV group) loop at :178-263): the block-sparse attention of
 * spruce_sparse_attention_fwd, where each row's softmax also covers the summary keys of its
 * residual tree nodes.  nodes: int32 [B, Hkv, qb, S] residual node ids, -1 padded (one layer of
 * residual_summary_nodes, interfaces/residual_summaries.py:158-220), element strides node_strides.
 * The summary table is the output of spruce_kv_summary_table for the same K/V: keys and values
 * fp32 [B, Hkv, num_nodes, prototypes, D], counts and log_counts fp32 [B, num_nodes, prototypes].
 * A prototype with count > 0 adds the score q.key * scale + log_count and its value; prototypes
 * are taken in node-slot order.  S == 0 is plain block-sparse attention.  The workspace
 * (spruce_residual_workspace_bytes) holds the gathered summary keys in the compute dtype, padded to
 * ceil(S * prototypes / 64) blocks of 64 per row. */
SPRUCE_API int64_t spruce_residual_workspace_bytes(int64_t B, int64_t Hkv, int64_t T, int64_t D, int64_t S,
                                                   int64_t prototypes, int dtype);
SPRUCE_API int spruce_residual_sparse_attention_fwd(const void *q, const int64_t q_strides[4], const void *k,
                                                    const int64_t k_strides[4], const void *v,
                                                    const int64_t v_strides[4], const int32_t *indices,
                                                    const int64_t idx_strides[4], const int32_t *nodes,
                                                    const int64_t node_strides[4], int64_t S,
                                                    const float *summary_keys, const float *summary_values,
                                                    const float *summary_counts, const float *summary_log_counts,
                                                    int64_t num_nodes, int64_t prototypes, void *out,
                                                    const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq,
                                                    int64_t Hkv, int64_t T, int64_t D, int64_t Kw, float scale,
                                                    void *workspace, int64_t workspace_bytes, uint32_t *status,
                                                    void *stream);

/*
 * build_kv_summary_table, sparse/summaries.py:52-142 (token ranges of
 * _prototype_token_ranges :29-49): for every node n of a residual tree
 * (block ranges node_starts/node_ends, ResidualTreeLayout.starts/ends of
 * interfaces/residual_summaries.py:20-71) and prototype p < prototypes, the
 * mean of the valid K and V rows in token range
 *   [ts + len*p/P, ts + len*(p+1)/P),  ts/te = start/end * block_size clamped to T,
 * taken as the difference of fp32 prefix sums and divided by max(count, 1),
 * as the reference does.  key/value [B, Hkv, T, D] (unit last stride, equal
 * shapes), valid uint8 [B, T] contiguous or NULL (all tokens valid).
 * Outputs (contiguous fp32): keys/values [B, Hkv, nodes, P, D],
 * counts/log_counts [B, nodes, P] (log_counts = log(count) or -inf);
 * range_starts/range_ends int64 [nodes, P] or NULL.  prototypes must be 1, 2
 * or 4 (sparse/config.py:8); block_size >= 1.  The caller passes a device
 * workspace of spruce_kv_summary_workspace_bytes() bytes, 16-byte aligned.
 */
SPRUCE_API int64_t spruce_kv_summary_workspace_bytes(int64_t B, int64_t Hkv, int64_t T, int64_t D);
SPRUCE_API int spruce_kv_summary_table(const void *key, const int64_t key_strides[4], const void *value,
                                       const int64_t value_strides[4], const uint8_t *valid, int dtype, int64_t B,
                                       int64_t Hkv, int64_t T, int64_t D, int64_t block_size, int64_t prototypes,
                                       const int64_t *node_starts, const int64_t *node_ends, int64_t num_nodes,
                                       float *keys, float *values, float *counts, float *log_counts,
                                       int64_t *range_starts, int64_t *range_ends, void *workspace,
                                       int64_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SPRUCE_B200_H */
