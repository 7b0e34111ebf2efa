// Internal launcher declarations shared by the .cu files and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace spruce {

struct PoolJob {
  const void* x;       // [B, H, T, D] strided
  int64_t sb, sh, st;  // element strides (d stride is 1)
  void* out;           // [B, Hout, nb, protos, D] contiguous
  int rep;             // heads averaged per output row (1 = plain pooling)
  int hout;            // output heads
  int blk0, nblk;      // 64-token blocks [blk0, blk0 + nblk) are pooled
  int protos = 1;      // prototypes per block: the mean, then the protos-1 rows farthest from it
};

template <typename T>
cudaError_t launch_pool(PoolJob j0, PoolJob j1, int njobs, int B, int T_len, int D, cudaStream_t stream);
template <typename T>
cudaError_t launch_group_avg(const void* x, const int64_t* strides, void* out, int B, int H, int T_len, int D,
                             int G, cudaStream_t stream);
template <typename T>
cudaError_t launch_project(const void* x, int64_t N, int D, const float* W, int P, float* out, cudaStream_t stream);
// Rows [row0, row0 + nrows) of each of `groups` consecutive [qb, D] matrices.
template <typename T>
cudaError_t launch_project_rows(const void* x, int64_t groups, int qb, int row0, int nrows, int D, const float* W,
                                int P, float* out, cudaStream_t stream);
// One projection job: rows (n / nrows) * qb + row0 + n % nrows, n < groups * nrows,
// of x [.., D] (dtype T) times W [D, P] fp32 -> out [.., P] fp32.
struct ProjRows {
  const void* x;
  const float* W;
  float* out;
  int64_t groups;
  int qb, row0, nrows;
};
// Up to two projection jobs of the same D and P in one launch.
template <typename T>
cudaError_t launch_project_pair(const ProjRows& a, const ProjRows& b, int njobs, int D, int P, cudaStream_t stream);

// Key tree of the deployed selector (tree.cu).
template <typename T>
cudaError_t launch_tree_merge(const void* child, int64_t R, int nchild, void* parent, int P, int d, int radix,
                              cudaStream_t stream);
cudaError_t launch_tree_candidates(const int64_t* sel, int64_t R, int nq, int S, int radix, int nchild,
                                   const int64_t* child_starts, int64_t* cand, uint8_t* valid, cudaStream_t stream);
cudaError_t launch_tree_topk(const float* scores, const uint8_t* valid, const int64_t* cand, int64_t rows, int C,
                             int k, int64_t* out, cudaStream_t stream);

// MaxSim scores (P prototypes of dimension pdim per row / key): every column
// (ids == null, ncols == nk) or the candidate key ids[r, q, c].
cudaError_t launch_maxsim(const float* qp, const float* kp, const int64_t* ids, int64_t R, int nq, int nk, int ncols,
                          int P, int pdim, float* out, cudaStream_t stream);
cudaError_t launch_scores(const float* qp, const float* kp, int64_t R, int qb, int kb, int P, float* out,
                          cudaStream_t stream);
int select_rows_for(int qb, int P, int64_t tiles16 = -1);
cudaError_t launch_select(const float* qp, const float* kp, int B, int G, int qb, int P, int K, int lw, int sink,
                          int32_t* out, const int64_t* out_strides, int q_begin, int q_end, cudaStream_t stream);
cudaError_t launch_pack_ids(const int64_t* ids, int64_t R, int qb, int C, int K, int lw, int kb, int sink,
                            int32_t* out, cudaStream_t stream);
cudaError_t launch_validate(const int32_t* sel, int64_t rows, int qb, int K, int lw, int64_t* result,
                            cudaStream_t stream);

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  const int64_t* qs;   // element strides [4]
  const int64_t* ks;
  const int64_t* vs;
  const int32_t* idx;
  const int64_t* is;
  void* out;
  const int64_t* os;   // logical [B, Hq, T, D] strides
  int B, Hq, Hkv, T, D, Kw;
  float scale;
  uint32_t* status;
  int q_begin, q_end;  // query-block range to compute
  // Fused output all-gather: every output row is also stored at the same
  // offset in each of these peer buffers (P2P-mapped, identical layout).
  const void* const* peer_out;
  int n_peer;
  // Residual summaries (optional; vk == nullptr: none).  Row (b, g, i) also
  // attends to vcount[(b*Hkv + g)*qb + i] virtual blocks of 64 gathered
  // summary keys: virtual tokens [i*nvb*64, ...) of vk / vv ([B, Hkv, Tv, D],
  // element strides vks / vvs), each with the additive natural-log count bias
  // vbias[(b*Hkv + g)*Tv + token] and no causal mask.
  const void* vk;
  const void* vv;
  const int64_t* vks;
  const int64_t* vvs;
  const float* vbias;
  const int32_t* vcount;
  int Tv, nvb;
};

// Virtual block ids start here in a row's compacted id list.
constexpr int kVirtualBase = 1 << 30;

constexpr int kMaxPeers = 7;

// Residual-summary gather: each row's valid (count > 0) node prototypes, in
// node-then-prototype order, become rows of the virtual K/V (in the compute
// dtype) with their natural-log count bias; rows up to the next multiple of 64
// are zero with bias -inf.  vcount receives the row's virtual block count.
struct ResidualGatherArgs {
  const int32_t* nodes;   // [B, Hkv, qb, S] residual node ids (-1 padded)
  int64_t ns[4];          // their element strides (by value: read on the device)
  int S;
  const float* keys;      // [B, Hkv, NN, P, D] summary table
  const float* values;
  const float* counts;    // [B, NN, P]
  const float* log_counts;
  int NN, P;
  int B, Hkv, qb, D, nvb;
  void* vk;               // [B, Hkv, qb*nvb*64, D]
  void* vv;
  float* vbias;           // [B, Hkv, qb*nvb*64]
  int32_t* vcount;        // [B, Hkv, qb]
};
cudaError_t launch_residual_gather(const ResidualGatherArgs& a, int dtype, cudaStream_t stream);
// Maximal residual frontier of each selected_blocks row (sel [rows, K] contiguous,
// query block = row % qb); out [rows, S] ID-sorted, -1 padded (NULL: counts only).
cudaError_t launch_residual_frontier(const int32_t* sel, int64_t rows, int K, int qb, const int64_t* starts,
                                     const int64_t* ends, const int32_t* parents, int NN, int32_t* out, int S,
                                     int32_t* row_counts, int32_t* max_count, cudaStream_t stream);

// tcgen05 path (bf16 / fp16).  Returns cudaErrorInvalidValue for shapes it
// does not cover (the C ABI checks them first).
cudaError_t launch_attn_sm100(const AttnArgs& a, int dtype, cudaStream_t stream);
// CUDA-core fp32 path.
cudaError_t launch_attn_f32(const AttnArgs& a, cudaStream_t stream);
// Largest row width the tcgen05 kernel accepts for this head dim.
int attn_sm100_max_kw(int D);
// Two selected blocks per step (N = 128 QK MMAs); attn_pair_sm100.cu.
cudaError_t launch_attn_pair(const AttnArgs& a, int dtype, cudaStream_t stream);
int attn_pair_max_kw(int D);
// The pair kernel's FMA-pipe polynomial exp2 and the MUFU exp2 over n values (self-check).
cudaError_t launch_exp2_probe(const float* x, float* poly, float* mufu, int64_t n, cudaStream_t stream);

// K/V summary table of the residual tree (summaries.cu).
struct KvSummaryArgs {
  const void* key;            // [B, H, T, D] strided, unit last stride
  const void* value;
  int64_t ks[3], vs[3];       // element strides b, h, t
  const uint8_t* valid;       // [B, T] or null (every token valid)
  int B, H, T, D, P;
  int seg;                    // tokens per prefix segment
  int64_t block_size;
  const int64_t* node_starts; // [nodes] in blocks
  const int64_t* node_ends;
  int64_t nodes;
  float* out_keys;            // [B, H, nodes, P, D]
  float* out_values;
  float* out_counts;          // [B, nodes, P]
  float* out_log_counts;
  int64_t* range_starts;      // [nodes, P] or null
  int64_t* range_ends;
  double* prefix;             // workspace: [2][B*H][nseg + 1][D]
  int64_t* cprefix;           // workspace: [B][nseg + 1]
};
int64_t kv_summary_segments(int64_t T);
int kv_summary_segment_tokens(int64_t block_size, int P, int64_t vecs_per_row);
int64_t kv_summary_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t D);
template <typename T>
cudaError_t launch_kv_summary(const KvSummaryArgs& a, bool vec, cudaStream_t stream);

}  // namespace spruce
