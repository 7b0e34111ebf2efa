// extern "C" entry points of libspruce_b200.so (declared in include/spruce_b200.h).
//
// Each entry point checks the contract the reference enforces (shape and
// dtype ValueErrors of kernels/seerattention_direct_index_triton.py:350-372,
// scripts/export_selected_blocks.py:98-119), plus the alignment the vector
// loads and TMA need, then enqueues its kernels on `stream`.  Nothing here
// allocates device memory or synchronises.
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SPRUCE_OK;
  return fail(SPRUCE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int elem_size(int dtype) { return dtype == SPRUCE_DTYPE_F32 ? 4 : 2; }

bool valid_dtype(int dtype) {
  return dtype == SPRUCE_DTYPE_F32 || dtype == SPRUCE_DTYPE_BF16 || dtype == SPRUCE_DTYPE_F16;
}

// Strides [b, h, t] (element units) must keep every 16-byte row segment aligned.
bool vec_strides_ok(const int64_t* s, int dtype, int64_t D) {
  const int64_t vn = 16 / elem_size(dtype);
  return s[3] == 1 && s[0] % vn == 0 && s[1] % vn == 0 && s[2] % vn == 0 && D % vn == 0;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {
static int spruce_sparse_attention_fwd_rows_impl(const void* q, const int64_t q_strides[4], const void* k,
                                                 const int64_t k_strides[4], const void* v,
                                                 const int64_t v_strides[4], const int32_t* indices,
                                                 const int64_t idx_strides[4], void* out,
                                                 const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq,
                                                 int64_t Hkv, int64_t T, int64_t D, int64_t Kw, float scale,
                                                 int64_t q_block_begin, int64_t q_block_end,
                                                 const void* const* peer_outs, int n_peers, uint32_t* status,
                                                 void* stream, const spruce::AttnArgs* virt = nullptr);

const char* spruce_last_error(void) { return g_last_error.c_str(); }

int spruce_abi_version(void) { return 1; }

int spruce_group_avg_tokens(const void* x, const int64_t x_strides[4], int dtype, int64_t B, int64_t H, int64_t T,
                            int64_t D, int64_t G, void* out, void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (B < 0 || H < 1 || T < 0 || D < 1 || G < 1) return fail(SPRUCE_ERR_INVALID, "bad shape");
  if (H % G) return fail(SPRUCE_ERR_INVALID, "H=%lld not divisible by G=%lld", (long long)H, (long long)G);
  if (!aligned16(x) || !aligned16(out) || !vec_strides_ok(x_strides, dtype, D))
    return fail(SPRUCE_ERR_UNSUPPORTED, "x must be 16-byte aligned with a unit last stride");
  if (B == 0 || T == 0) return SPRUCE_OK;
  cudaError_t e;
  switch (dtype) {
    case SPRUCE_DTYPE_F32: e = spruce::launch_group_avg<float>(x, x_strides, out, B, H, T, D, G, as_stream(stream)); break;
    case SPRUCE_DTYPE_BF16:
      e = spruce::launch_group_avg<__nv_bfloat16>(x, x_strides, out, B, H, T, D, G, as_stream(stream));
      break;
    default: e = spruce::launch_group_avg<__half>(x, x_strides, out, B, H, T, D, G, as_stream(stream)); break;
  }
  return cuda_status(e, "group_avg launch");
}

static int pool_jobs(spruce::PoolJob j0, spruce::PoolJob j1, int njobs, int dtype, int64_t B, int64_t T, int64_t D,
                     void* stream);

// Pooled Q for blocks [q0, q1) and pooled K for blocks [0, k1) (the rows a
// query-block range of the selector reads); shapes already checked.
static int pool_qk_range(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                         int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, void* pooled_q,
                         void* pooled_k, int q0, int q1, int k1, void* stream, int protos = 1) {
  spruce::PoolJob jq{q, q_strides[0], q_strides[1], q_strides[2], pooled_q, (int)(Hq / Hkv), (int)Hkv, q0, q1 - q0,
                     protos};
  spruce::PoolJob jk{k, k_strides[0], k_strides[1], k_strides[2], pooled_k, 1, (int)Hkv, 0, k1, protos};
  return pool_jobs(jq, jk, 2, dtype, B, T, D, stream);
}

static constexpr int64_t kMaxProtos = SPRUCE_BLOCK;  // the mean plus at most every row of the block

static int pool_jobs(spruce::PoolJob j0, spruce::PoolJob j1, int njobs, int dtype, int64_t B, int64_t T, int64_t D,
                     void* stream) {
  cudaError_t e;
  switch (dtype) {
    case SPRUCE_DTYPE_F32: e = spruce::launch_pool<float>(j0, j1, njobs, B, T, D, as_stream(stream)); break;
    case SPRUCE_DTYPE_BF16: e = spruce::launch_pool<__nv_bfloat16>(j0, j1, njobs, B, T, D, as_stream(stream)); break;
    default: e = spruce::launch_pool<__half>(j0, j1, njobs, B, T, D, as_stream(stream)); break;
  }
  return cuda_status(e, "pool launch");
}

int spruce_proto_pool(const void* x, const int64_t x_strides[4], int dtype, int64_t B, int64_t H, int64_t T,
                      int64_t D, int64_t block, int64_t P, void* out, void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (block != SPRUCE_BLOCK) return fail(SPRUCE_ERR_UNSUPPORTED, "block must be 64, got %lld", (long long)block);
  if (P < 1) return fail(SPRUCE_ERR_INVALID, "P must be >= 1, got %lld", (long long)P);
  if (P > kMaxProtos)
    return fail(SPRUCE_ERR_UNSUPPORTED, "at most %lld prototypes per 64-token block, got P=%lld",
                (long long)kMaxProtos, (long long)P);
  if (B < 0 || H < 1 || T < 0 || D < 1 || D > 256) return fail(SPRUCE_ERR_INVALID, "bad shape");
  if (!aligned16(x) || !aligned16(out) || !vec_strides_ok(x_strides, dtype, D))
    return fail(SPRUCE_ERR_UNSUPPORTED, "x must be 16-byte aligned with a unit last stride");
  if (B == 0 || T == 0) return SPRUCE_OK;
  const int nb = (int)((T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK);
  spruce::PoolJob j{x, x_strides[0], x_strides[1], x_strides[2], out, 1, (int)H, 0, nb, (int)P};
  return pool_jobs(j, j, 1, dtype, B, T, D, stream);
}

int spruce_pool_qk_protos(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                          int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, int64_t P,
                          void* pooled_q, void* pooled_k, void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (B < 0 || Hq < 1 || Hkv < 1 || T < 0 || D < 1 || D > 256) return fail(SPRUCE_ERR_INVALID, "bad shape");
  if (Hq % Hkv) return fail(SPRUCE_ERR_INVALID, "query heads (%lld) must be divisible by KV heads (%lld)",
                            (long long)Hq, (long long)Hkv);
  if (P < 1) return fail(SPRUCE_ERR_INVALID, "P must be >= 1, got %lld", (long long)P);
  if (P > kMaxProtos)
    return fail(SPRUCE_ERR_UNSUPPORTED, "at most %lld prototypes per 64-token block, got P=%lld",
                (long long)kMaxProtos, (long long)P);
  if (!aligned16(q) || !aligned16(k) || !aligned16(pooled_q) || !aligned16(pooled_k) ||
      !vec_strides_ok(q_strides, dtype, D) || !vec_strides_ok(k_strides, dtype, D))
    return fail(SPRUCE_ERR_UNSUPPORTED, "q/k must be 16-byte aligned with a unit last stride");
  if (B == 0 || T == 0) return SPRUCE_OK;
  const int nb = (int)((T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK);
  return pool_qk_range(q, q_strides, k, k_strides, dtype, B, Hq, Hkv, T, D, pooled_q, pooled_k, 0, nb, nb, stream,
                       (int)P);
}

int spruce_pool_qk(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4], int dtype,
                   int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, void* pooled_q, void* pooled_k,
                   void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (B < 0 || Hq < 1 || Hkv < 1 || T < 0 || D < 1 || D > 256) return fail(SPRUCE_ERR_INVALID, "bad shape");
  if (Hq % Hkv) return fail(SPRUCE_ERR_INVALID, "query heads (%lld) must be divisible by KV heads (%lld)",
                            (long long)Hq, (long long)Hkv);
  if (!aligned16(q) || !aligned16(k) || !aligned16(pooled_q) || !aligned16(pooled_k) ||
      !vec_strides_ok(q_strides, dtype, D) || !vec_strides_ok(k_strides, dtype, D))
    return fail(SPRUCE_ERR_UNSUPPORTED, "q/k must be 16-byte aligned with a unit last stride");
  if (B == 0 || T == 0) return SPRUCE_OK;
  const int nb = (int)((T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK);
  return pool_qk_range(q, q_strides, k, k_strides, dtype, B, Hq, Hkv, T, D, pooled_q, pooled_k, 0, nb, nb, stream);
}

int spruce_gate_project(const void* x, int dtype, int64_t N, int64_t D, const float* W, int64_t P, float* out,
                        void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (N < 0 || D < 1 || P < 1 || D > 1024) return fail(SPRUCE_ERR_INVALID, "bad projection shape");
  cudaError_t e;
  switch (dtype) {
    case SPRUCE_DTYPE_F32: e = spruce::launch_project<float>(x, N, D, W, P, out, as_stream(stream)); break;
    case SPRUCE_DTYPE_BF16: e = spruce::launch_project<__nv_bfloat16>(x, N, D, W, P, out, as_stream(stream)); break;
    default: e = spruce::launch_project<__half>(x, N, D, W, P, out, as_stream(stream)); break;
  }
  return cuda_status(e, "projection launch");
}

int spruce_gate_maxsim(const float* qp, const float* kp, const int64_t* ids, int64_t R, int64_t nq, int64_t nk,
                       int64_t ncols, int64_t P, int64_t pdim, float* out, void* stream) {
  if (R < 0 || nq < 0 || nk < 1 || ncols < 0 || pdim < 1 || pdim > 4096)
    return fail(SPRUCE_ERR_INVALID, "bad MaxSim shape");
  if (P < 1 || P > 8) return fail(SPRUCE_ERR_UNSUPPORTED, "MaxSim takes 1 to 8 prototypes, got %lld", (long long)P);
  if (ids == nullptr && ncols != nk)
    return fail(SPRUCE_ERR_INVALID, "without candidate ids every key is a column (ncols == nk)");
  if (R * nq > INT32_MAX || nq > INT32_MAX || nk > INT32_MAX || ncols > INT32_MAX)
    return fail(SPRUCE_ERR_UNSUPPORTED, "MaxSim shape too large");
  return cuda_status(spruce::launch_maxsim(qp, kp, ids, R, (int)nq, (int)nk, (int)ncols, (int)P, (int)pdim, out,
                                           as_stream(stream)),
                     "maxsim launch");
}

int spruce_tree_merge(const void* child, int dtype, int64_t R, int64_t nchild, int64_t P, int64_t d, int64_t radix,
                      void* parent, void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (radix < 2) return fail(SPRUCE_ERR_INVALID, "radix must be >= 2, got %lld", (long long)radix);
  if (R < 0 || nchild < 1 || d < 1 || d > 4096 || nchild > INT32_MAX) return fail(SPRUCE_ERR_INVALID, "bad tree shape");
  if (P < 1 || P > 8 || radix * P > 256)
    return fail(SPRUCE_ERR_UNSUPPORTED, "tree merge takes 1 to 8 prototypes and radix * P <= 256");
  cudaError_t e;
  switch (dtype) {
    case SPRUCE_DTYPE_F32:
      e = spruce::launch_tree_merge<float>(child, R, (int)nchild, parent, (int)P, (int)d, (int)radix, as_stream(stream));
      break;
    case SPRUCE_DTYPE_BF16:
      e = spruce::launch_tree_merge<__nv_bfloat16>(child, R, (int)nchild, parent, (int)P, (int)d, (int)radix,
                                                   as_stream(stream));
      break;
    default:
      e = spruce::launch_tree_merge<__half>(child, R, (int)nchild, parent, (int)P, (int)d, (int)radix,
                                            as_stream(stream));
      break;
  }
  return cuda_status(e, "tree merge launch");
}

int spruce_tree_candidates(const int64_t* selected, int64_t R, int64_t nq, int64_t S, int64_t radix, int64_t nchild,
                           const int64_t* child_starts, int64_t* cand, uint8_t* valid, void* stream) {
  if (radix < 2 || R < 0 || nq < 0 || S < 1 || nchild < 1 || nq > INT32_MAX || nchild > INT32_MAX ||
      S * radix > 256)
    return fail(SPRUCE_ERR_INVALID, "bad traversal shape");
  return cuda_status(spruce::launch_tree_candidates(selected, R, (int)nq, (int)S, (int)radix, (int)nchild,
                                                    child_starts, cand, valid, as_stream(stream)),
                     "tree candidate launch");
}

int spruce_tree_topk(const float* scores, const uint8_t* valid, const int64_t* cand, int64_t rows, int64_t C,
                     int64_t k, int64_t* out, void* stream) {
  if (rows < 0 || C < 1 || C > 256 || k < 1 || k > C) return fail(SPRUCE_ERR_INVALID, "bad traversal top-k shape");
  return cuda_status(spruce::launch_tree_topk(scores, valid, cand, rows, (int)C, (int)k, out, as_stream(stream)),
                     "tree top-k launch");
}

int spruce_gate_scores(const float* qp, const float* kp, int64_t R, int64_t qb, int64_t kb, int64_t P, float* out,
                       void* stream) {
  if (R < 0 || qb < 0 || kb < 0 || P < 1 || P > 1024) return fail(SPRUCE_ERR_INVALID, "bad score shape");
  if (R == 0 || qb == 0 || kb == 0) return SPRUCE_OK;
  return cuda_status(spruce::launch_scores(qp, kp, R, qb, kb, P, out, as_stream(stream)), "score launch");
}

static int check_select_policy(int64_t K, int64_t lw, int64_t sink) {
  if (K < 1) return fail(SPRUCE_ERR_INVALID, "k_selected must be >= 1, got %lld", (long long)K);
  if (lw < 0) return fail(SPRUCE_ERR_INVALID, "local_window must be >= 0, got %lld", (long long)lw);
  if (sink < 0) return fail(SPRUCE_ERR_INVALID, "sink_blocks must be >= 0, got %lld", (long long)sink);
  if (K < lw + 1 + sink)
    return fail(SPRUCE_ERR_INVALID, "k_selected=%lld cannot fit local window size %lld plus %lld sink block(s)",
                (long long)K, (long long)(lw + 1), (long long)sink);
  return SPRUCE_OK;
}

int spruce_gate_select_rows(const float* qp, const float* kp, int64_t B, int64_t G, int64_t qb, int64_t P,
                            int64_t K, int64_t local_window, int64_t sink_blocks, int32_t* out,
                            const int64_t out_strides[3], int64_t q_block_begin, int64_t q_block_end, void* stream) {
  int rc = check_select_policy(K, local_window, sink_blocks);
  if (rc) return rc;
  if (B < 0 || G < 1 || qb < 0 || P < 1 || P > 1024) return fail(SPRUCE_ERR_INVALID, "bad selection shape");
  if (q_block_begin < 0 || q_block_end > qb || q_block_begin > q_block_end)
    return fail(SPRUCE_ERR_INVALID, "query-block range [%lld, %lld) outside [0, %lld)", (long long)q_block_begin,
                (long long)q_block_end, (long long)qb);
  if (B == 0 || qb == 0 || q_block_begin == q_block_end) return SPRUCE_OK;
  if (spruce::select_rows_for((int)qb, (int)P) == 0)
    return fail(SPRUCE_ERR_UNSUPPORTED, "qb=%lld query blocks exceed the selection kernel's shared memory",
                (long long)qb);
  return cuda_status(spruce::launch_select(qp, kp, (int)B, (int)G, (int)qb, (int)P, (int)K, (int)local_window,
                                           (int)sink_blocks, out, out_strides, (int)q_block_begin,
                                           (int)q_block_end, as_stream(stream)),
                     "selection launch");
}

int spruce_gate_select(const float* qp, const float* kp, int64_t B, int64_t G, int64_t qb, int64_t P, int64_t K,
                       int64_t local_window, int64_t sink_blocks, int32_t* out, const int64_t out_strides[3],
                       void* stream) {
  return spruce_gate_select_rows(qp, kp, B, G, qb, P, K, local_window, sink_blocks, out, out_strides, 0,
                                 qb < 0 ? 0 : qb, stream);
}

int64_t spruce_select_workspace_bytes(int64_t B, int64_t Hkv, int64_t T, int64_t D, int64_t P, int dtype) {
  // -1 for a shape the selector rejects anyway, or whose size would not fit in int64:
  // a wrapped product must never pass a workspace-size check.
  if (!valid_dtype(dtype) || B < 0 || Hkv < 1 || T < 0 || D < 1 || D > 256 || P < 1 || P > 1024) return -1;
  const int64_t qb = T / SPRUCE_BLOCK + (T % SPRUCE_BLOCK != 0);
  int64_t rows = 0, feat = 0, proj = 0;
  if (__builtin_mul_overflow(B, Hkv, &rows) || __builtin_mul_overflow(rows, qb, &rows)) return -1;
  if (qb > INT32_MAX || rows > INT32_MAX) return -1;  // the kernels index query blocks and rows with int
  if (__builtin_mul_overflow(rows, D * elem_size(dtype), &feat) || __builtin_mul_overflow(rows, P * 4, &proj))
    return -1;
  if (feat > INT64_MAX / 4 - 256 || proj > INT64_MAX / 4 - 256) return -1;
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  return 2 * up(feat) + 2 * up(proj);
}

int spruce_select_blocks(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                         int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const float* Wq,
                         const float* Wk, int64_t P, int64_t K, int64_t local_window, int64_t sink_blocks,
                         int32_t* out, const int64_t out_strides[3], void* workspace, int64_t workspace_bytes,
                         void* stream) {
  const int64_t qb = (T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK;
  return spruce_select_blocks_rows(q, q_strides, k, k_strides, dtype, B, Hq, Hkv, T, D, Wq, Wk, P, K, local_window,
                                   sink_blocks, out, out_strides, 0, qb < 0 ? 0 : qb, workspace, workspace_bytes,
                                   stream);
}

int spruce_select_blocks_rows(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                              int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const float* Wq,
                              const float* Wk, int64_t P, int64_t K, int64_t local_window, int64_t sink_blocks,
                              int32_t* out, const int64_t out_strides[3], int64_t q_block_begin,
                              int64_t q_block_end, void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_select_policy(K, local_window, sink_blocks);
  if (rc) return rc;
  const int64_t need = spruce_select_workspace_bytes(B, Hkv, T, D, P, dtype);
  if (need < 0)
    return fail(SPRUCE_ERR_INVALID, "bad selector shape (B=%lld, Hkv=%lld, T=%lld, D=%lld, P=%lld, dtype %d)",
                (long long)B, (long long)Hkv, (long long)T, (long long)D, (long long)P, dtype);
  if (workspace_bytes < need)
    return fail(SPRUCE_ERR_WORKSPACE, "workspace of %lld bytes, need %lld", (long long)workspace_bytes,
                (long long)need);
  if (!aligned16(workspace)) return fail(SPRUCE_ERR_INVALID, "workspace must be 16-byte aligned");
  const int64_t qb = (T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK;
  const int64_t rows = B * Hkv * qb;
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* pooled_q = ws;
  void* pooled_k = ws + up(rows * D * elem_size(dtype));
  float* qp = reinterpret_cast<float*>(ws + 2 * up(rows * D * elem_size(dtype)));
  float* kp = reinterpret_cast<float*>(ws + 2 * up(rows * D * elem_size(dtype)) + up(rows * P * 4));
  if (q_block_begin < 0 || q_block_end > qb || q_block_begin > q_block_end)
    return fail(SPRUCE_ERR_INVALID, "query-block range [%lld, %lld) outside [0, %lld)", (long long)q_block_begin,
                (long long)q_block_end, (long long)qb);
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (B < 0 || Hq < 1 || Hkv < 1 || T < 0 || D < 1 || D > 256 || P < 1 || P > 1024)
    return fail(SPRUCE_ERR_INVALID, "bad selector shape");
  if (Hq % Hkv) return fail(SPRUCE_ERR_INVALID, "query heads (%lld) must be divisible by KV heads (%lld)",
                            (long long)Hq, (long long)Hkv);
  if (!aligned16(q) || !aligned16(k) || !vec_strides_ok(q_strides, dtype, D) || !vec_strides_ok(k_strides, dtype, D))
    return fail(SPRUCE_ERR_UNSUPPORTED, "q/k must be 16-byte aligned with a unit last stride");
  if (B == 0 || T == 0 || q_block_begin == q_block_end) return SPRUCE_OK;
  // Only the rows the range reads: queries [i0, i1), keys [0, i1 - local_window).
  const int i0 = (int)q_block_begin, i1 = (int)q_block_end;
  const int k1 = std::max(1, std::min(i1, (int)qb));
  rc = pool_qk_range(q, q_strides, k, k_strides, dtype, B, Hq, Hkv, T, D, pooled_q, pooled_k, i0, i1, k1, stream);
  if (rc) return rc;
  // both projections in one launch: queries [i0, i1) and keys [0, k1) of every (batch, group)
  const spruce::ProjRows pj_q{pooled_q, Wq, qp, B * Hkv, (int)qb, i0, i1 - i0};
  const spruce::ProjRows pj_k{pooled_k, Wk, kp, B * Hkv, (int)qb, 0, k1};
  cudaError_t e;
  switch (dtype) {
    case SPRUCE_DTYPE_F32:
      e = spruce::launch_project_pair<float>(pj_q, pj_k, 2, (int)D, (int)P, as_stream(stream));
      break;
    case SPRUCE_DTYPE_BF16:
      e = spruce::launch_project_pair<__nv_bfloat16>(pj_q, pj_k, 2, (int)D, (int)P, as_stream(stream));
      break;
    default:
      e = spruce::launch_project_pair<__half>(pj_q, pj_k, 2, (int)D, (int)P, as_stream(stream));
      break;
  }
  rc = cuda_status(e, "projection launch");
  if (rc) return rc;
  return spruce_gate_select_rows(qp, kp, B, Hkv, qb, P, K, local_window, sink_blocks, out, out_strides, i0, i1,
                                 stream);
}

}  // extern "C"

// ---------------------------------------------------------------- no-allocation selector
// Scratch for spruce_select_blocks_noalloc: one file-scope device array that
// every GPU loading this library holds until the process exits.  In host code
// `g_select_scratch` is only a host-side stand-in, never a device address; the
// device address is fetched per device with cudaGetSymbolAddress below.
namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_select_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_select_scratch on the current device, looked up once per
// device (the first call on a device does this; it makes no allocation).
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(SPRUCE_ERR_UNSUPPORTED, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_select_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_select_scratch)");
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return SPRUCE_OK;
}

}  // namespace

extern "C" {

int64_t spruce_select_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

int spruce_select_blocks_noalloc(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                                 int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, const float* Wq,
                                 const float* Wk, int64_t P, int64_t K, int64_t local_window, int64_t sink_blocks,
                                 int32_t* out, const int64_t out_strides[3], void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  const int64_t need = spruce_select_workspace_bytes(B, Hkv, T, D, P, dtype);
  if (need < 0)
    return fail(SPRUCE_ERR_INVALID, "bad selector shape (B=%lld, Hkv=%lld, T=%lld, D=%lld, P=%lld)", (long long)B,
                (long long)Hkv, (long long)T, (long long)D, (long long)P);
  if (need > kNoAllocScratchBytes)
    return fail(SPRUCE_ERR_UNSUPPORTED,
                "spruce_select_blocks_noalloc: this shape needs %lld bytes of scratch, more than the %lld-byte "
                "static buffer; use spruce_select_blocks with a caller-provided workspace",
                (long long)need, (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // Every region the selector reads (pooled features, projections) is fully
  // written earlier in the same call, so nothing needs clearing first.
  return spruce_select_blocks(q, q_strides, k, k_strides, dtype, B, Hq, Hkv, T, D, Wq, Wk, P, K, local_window,
                              sink_blocks, out, out_strides, scratch, kNoAllocScratchBytes, stream);
}

// ---------------------------------------------------------------- CUDA IPC plumbing (host only)
using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(ptr);
  }
  return fn;
}

int spruce_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  GetAddressRangeFn range = address_range_fn();
  if (range == nullptr) return fail(SPRUCE_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(SPRUCE_ERR_INVALID, "pointer is not inside a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return SPRUCE_OK;
}

int spruce_ipc_import(const void* handle, int64_t offset, void** ptr, void** base) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcOpenMemHandle");
  *base = b;
  *ptr = static_cast<uint8_t*>(b) + offset;
  return SPRUCE_OK;
}

int spruce_ipc_close(void* base) { return cuda_status(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle"); }

int spruce_pack_selected_ids(const int64_t* ids, int64_t R, int64_t qb, int64_t C, int64_t K, int64_t local_window,
                             int64_t key_blocks, int64_t sink_blocks, int32_t* out, void* stream) {
  int rc = check_select_policy(K, local_window, sink_blocks);
  if (rc) return rc;
  if (key_blocks < 1) return fail(SPRUCE_ERR_INVALID, "key_blocks must be >= 1, got %lld", (long long)key_blocks);
  if (R < 0 || qb < 0 || C < 0) return fail(SPRUCE_ERR_INVALID, "bad ids shape");
  const int64_t span = qb > key_blocks ? qb : key_blocks;
  if (span > (1 << 20)) return fail(SPRUCE_ERR_UNSUPPORTED, "too many blocks (%lld)", (long long)span);
  return cuda_status(spruce::launch_pack_ids(ids, R, (int)qb, (int)C, (int)K, (int)local_window, (int)key_blocks,
                                             (int)sink_blocks, out, as_stream(stream)),
                     "pack launch");
}

int spruce_validate_selected_blocks(const int32_t* sel, int64_t B, int64_t L, int64_t G, int64_t qb, int64_t K,
                                    int64_t local_window, int64_t* result, void* stream) {
  if (local_window < 0) return fail(SPRUCE_ERR_INVALID, "local_window must be >= 0, got %lld", (long long)local_window);
  if (B < 0 || L < 0 || G < 0 || qb < 0 || K < 0) return fail(SPRUCE_ERR_INVALID, "bad shape");
  return cuda_status(spruce::launch_validate(sel, B * L * G * qb, (int)qb, (int)K, (int)local_window, result,
                                             as_stream(stream)),
                     "validate launch");
}

int spruce_sparse_attention_fwd_scatter(const void* q, const int64_t q_strides[4], const void* k,
                                        const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                                        const int32_t* indices, const int64_t idx_strides[4], void* out,
                                        const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq,
                                        int64_t Hkv, int64_t T, int64_t D, int64_t Kw, float scale,
                                        int64_t q_block_begin, int64_t q_block_end, const void* const* peer_outs,
                                        int32_t n_peers, uint32_t* status, void* stream) {
  if (n_peers < 0 || n_peers > spruce::kMaxPeers)
    return fail(SPRUCE_ERR_UNSUPPORTED, "n_peers=%d outside [0, %d]", (int)n_peers, spruce::kMaxPeers);
  if (n_peers > 0 && dtype == SPRUCE_DTYPE_F32)
    return fail(SPRUCE_ERR_UNSUPPORTED, "the fused output all-gather covers the bf16/fp16 kernel only");
  for (int i = 0; i < n_peers; ++i)
    if (peer_outs[i] == nullptr || !aligned16(peer_outs[i]))
      return fail(SPRUCE_ERR_INVALID, "peer output %d must be a 16-byte aligned device pointer", i);
  return spruce_sparse_attention_fwd_rows_impl(q, q_strides, k, k_strides, v, v_strides, indices, idx_strides, out,
                                               out_strides, dtype, B, Hq, Hkv, T, D, Kw, scale, q_block_begin,
                                               q_block_end, peer_outs, n_peers, status, stream);
}

int spruce_sparse_attention_fwd_rows(const void* q, const int64_t q_strides[4], const void* k,
                                     const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                                     const int32_t* indices, const int64_t idx_strides[4], void* out,
                                     const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                                     int64_t T, int64_t D, int64_t Kw, float scale, int64_t q_block_begin,
                                     int64_t q_block_end, uint32_t* status, void* stream) {
  return spruce_sparse_attention_fwd_rows_impl(q, q_strides, k, k_strides, v, v_strides, indices, idx_strides, out,
                                               out_strides, dtype, B, Hq, Hkv, T, D, Kw, scale, q_block_begin,
                                               q_block_end, nullptr, 0, status, stream);
}

static int spruce_sparse_attention_fwd_rows_impl(const void* q, const int64_t q_strides[4], const void* k,
                                     const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                                     const int32_t* indices, const int64_t idx_strides[4], void* out,
                                     const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                                     int64_t T, int64_t D, int64_t Kw, float scale, int64_t q_block_begin,
                                     int64_t q_block_end, const void* const* peer_outs, int n_peers,
                                     uint32_t* status, void* stream, const spruce::AttnArgs* virt) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (D != 64 && D != 128) return fail(SPRUCE_ERR_INVALID, "kernel supports head_dim 64 or 128, got %lld", (long long)D);
  if (B < 0 || Hq < 1 || Hkv < 1 || T < 0 || Kw < 0) return fail(SPRUCE_ERR_INVALID, "bad attention shape");
  if (Hq % Hkv) return fail(SPRUCE_ERR_INVALID, "query heads must be divisible by KV heads");
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || idx_strides[3] != 1 || out_strides[3] != 1)
    return fail(SPRUCE_ERR_INVALID, "q, k, v, and indices must have a contiguous final dimension");
  const int64_t qb = (T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK;
  if (q_block_begin < 0 || q_block_end > qb || q_block_begin > q_block_end)
    return fail(SPRUCE_ERR_INVALID, "query-block range [%lld, %lld) outside [0, %lld)", (long long)q_block_begin,
                (long long)q_block_end, (long long)qb);
  if (B == 0 || T == 0 || q_block_begin == q_block_end) return SPRUCE_OK;
  if (T > (int64_t)1 << 30 || Hkv > 65535 || B > 65535 || qb * 2 > (int64_t)1 << 30)
    return fail(SPRUCE_ERR_UNSUPPORTED, "shape too large for the launch grid");
  spruce::AttnArgs a{q, k, v, q_strides, k_strides, v_strides, indices, idx_strides, out, out_strides,
                     (int)B, (int)Hq, (int)Hkv, (int)T, (int)D, (int)Kw, scale, status,
                     (int)q_block_begin, (int)q_block_end, peer_outs, n_peers};
  if (virt != nullptr) {  // residual summaries: the gathered virtual K/V of every row
    a.vk = virt->vk;
    a.vv = virt->vv;
    a.vks = virt->vks;
    a.vvs = virt->vvs;
    a.vbias = virt->vbias;
    a.vcount = virt->vcount;
    a.Tv = virt->Tv;
    a.nvb = virt->nvb;
  }
  if (dtype == SPRUCE_DTYPE_F32) {
    if (Kw > 8192) return fail(SPRUCE_ERR_UNSUPPORTED, "row width %lld too large", (long long)Kw);
    return cuda_status(spruce::launch_attn_f32(a, as_stream(stream)), "fp32 attention launch");
  }
  // TMA needs 16-byte aligned bases and strides that are multiples of 16 bytes.
  const int64_t* ss[3] = {q_strides, k_strides, v_strides};
  const void* bases[3] = {q, k, v};
  for (int t = 0; t < 3; ++t) {
    if (!aligned16(bases[t]) || ss[t][0] % 8 || ss[t][1] % 8 || ss[t][2] % 8)
      return fail(SPRUCE_ERR_UNSUPPORTED, "q/k/v need 16-byte aligned bases and strides");
  }
  if (!aligned16(out) || out_strides[0] % 8 || out_strides[1] % 8 || out_strides[2] % 8)
    return fail(SPRUCE_ERR_UNSUPPORTED, "out needs 16-byte aligned base and strides");
  const int64_t kw_all = Kw + (virt != nullptr ? virt->nvb : 0);
  if (kw_all > spruce::attn_sm100_max_kw((int)D))
    return fail(SPRUCE_ERR_UNSUPPORTED, "row width %lld exceeds %d", (long long)kw_all,
                spruce::attn_sm100_max_kw((int)D));
  return cuda_status(spruce::launch_attn_sm100(a, dtype, as_stream(stream)), "tcgen05 attention launch");
}

int spruce_exp2_selfcheck(const float* x, int64_t n, float* poly_out, float* mufu_out, void* stream) {
  if (n < 0) return fail(SPRUCE_ERR_INVALID, "n must be >= 0");
  if (n > 0 && (x == nullptr || poly_out == nullptr || mufu_out == nullptr))
    return fail(SPRUCE_ERR_INVALID, "null pointer");
  return cuda_status(spruce::launch_exp2_probe(x, poly_out, mufu_out, n, as_stream(stream)), "exp2 probe launch");
}

int spruce_sparse_attention_fwd(const void* q, const int64_t q_strides[4], const void* k, const int64_t k_strides[4],
                                const void* v, const int64_t v_strides[4], const int32_t* indices,
                                const int64_t idx_strides[4], void* out, const int64_t out_strides[4], int dtype,
                                int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, int64_t Kw, float scale,
                                uint32_t* status, void* stream) {
  const int64_t qb = (T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK;
  return spruce_sparse_attention_fwd_rows(q, q_strides, k, k_strides, v, v_strides, indices, idx_strides, out,
                                          out_strides, dtype, B, Hq, Hkv, T, D, Kw, scale, 0, qb < 0 ? 0 : qb,
                                          status, stream);
}

// Workspace of the residual-summary attention: virtual K and V in the compute
// dtype, their fp32 biases and the per-row virtual block counts.
struct ResidualWorkspace {
  int64_t nvb, Tv, off_vv, off_bias, off_count, total;
};

static ResidualWorkspace residual_workspace(int64_t B, int64_t Hkv, int64_t T, int64_t D, int64_t S, int64_t P,
                                            int dtype) {
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  ResidualWorkspace w;
  const int64_t qb = (T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK;
  w.nvb = (S * P + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK;
  w.Tv = qb * w.nvb * SPRUCE_BLOCK;
  const int64_t kv = up(B * Hkv * w.Tv * D * elem_size(dtype));
  w.off_vv = kv;
  w.off_bias = 2 * kv;
  w.off_count = w.off_bias + up(B * Hkv * w.Tv * 4);
  w.total = w.off_count + up(B * Hkv * qb * 4);
  return w;
}

int64_t spruce_residual_workspace_bytes(int64_t B, int64_t Hkv, int64_t T, int64_t D, int64_t S, int64_t prototypes,
                                        int dtype) {
  if (B < 0 || Hkv < 0 || T < 0 || D < 1 || S < 0 || prototypes < 1 || !valid_dtype(dtype)) return -1;
  return residual_workspace(B, Hkv, T, D, S, prototypes, dtype).total;
}

int spruce_residual_sparse_attention_fwd(const void* q, const int64_t q_strides[4], const void* k,
                                         const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                                         const int32_t* indices, const int64_t idx_strides[4], const int32_t* nodes,
                                         const int64_t node_strides[4], int64_t S, const float* summary_keys,
                                         const float* summary_values, const float* summary_counts,
                                         const float* summary_log_counts, int64_t num_nodes, int64_t prototypes,
                                         void* out, const int64_t out_strides[4], int dtype, int64_t B, int64_t Hq,
                                         int64_t Hkv, int64_t T, int64_t D, int64_t Kw, float scale, void* workspace,
                                         int64_t workspace_bytes, uint32_t* status, void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (S < 0 || prototypes < 1 || prototypes > 64 || num_nodes < 0)
    return fail(SPRUCE_ERR_INVALID, "bad residual summary shape (S=%lld, prototypes=%lld, nodes=%lld)", (long long)S,
                (long long)prototypes, (long long)num_nodes);
  const int64_t qb = (T + SPRUCE_BLOCK - 1) / SPRUCE_BLOCK;
  if (S == 0 || B == 0 || T == 0)  // no residual node anywhere: plain block-sparse attention
    return spruce_sparse_attention_fwd_rows_impl(q, q_strides, k, k_strides, v, v_strides, indices, idx_strides, out,
                                                 out_strides, dtype, B, Hq, Hkv, T, D, Kw, scale, 0, qb, nullptr, 0,
                                                 status, stream);
  if (nodes == nullptr || summary_keys == nullptr || summary_values == nullptr || summary_counts == nullptr ||
      summary_log_counts == nullptr)
    return fail(SPRUCE_ERR_INVALID, "residual summaries need nodes and the summary table");
  if (S * prototypes > 51200)
    return fail(SPRUCE_ERR_UNSUPPORTED, "residual width %lld x %lld prototypes too large", (long long)S,
                (long long)prototypes);
  if (Hkv > 65535 || B > 65535 || qb > 65535 * 64) return fail(SPRUCE_ERR_UNSUPPORTED, "shape too large");
  const ResidualWorkspace w = residual_workspace(B, Hkv, T, D, S, prototypes, dtype);
  if (w.Tv > ((int64_t)1 << 31) - 64) return fail(SPRUCE_ERR_UNSUPPORTED, "too many residual summary keys");
  if (workspace == nullptr || workspace_bytes < w.total)
    return fail(SPRUCE_ERR_WORKSPACE, "residual workspace needs %lld bytes, got %lld", (long long)w.total,
                (long long)workspace_bytes);
  if (!aligned16(workspace)) return fail(SPRUCE_ERR_UNSUPPORTED, "workspace must be 16-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  spruce::ResidualGatherArgs g{nodes, {node_strides[0], node_strides[1], node_strides[2], node_strides[3]}, (int)S,
                               summary_keys, summary_values, summary_counts, summary_log_counts, (int)num_nodes,
                               (int)prototypes, (int)B, (int)Hkv, (int)qb, (int)D, (int)w.nvb, ws, ws + w.off_vv,
                               reinterpret_cast<float*>(ws + w.off_bias), reinterpret_cast<int32_t*>(ws + w.off_count)};
  int rc = cuda_status(spruce::launch_residual_gather(g, dtype, as_stream(stream)), "residual gather launch");
  if (rc != SPRUCE_OK) return rc;
  const int64_t vstr[4] = {Hkv * w.Tv * D, w.Tv * D, D, 1};
  spruce::AttnArgs virt{};
  virt.vk = ws;
  virt.vv = ws + w.off_vv;
  virt.vks = vstr;
  virt.vvs = vstr;
  virt.vbias = reinterpret_cast<const float*>(ws + w.off_bias);
  virt.vcount = reinterpret_cast<const int32_t*>(ws + w.off_count);
  virt.Tv = (int)w.Tv;
  virt.nvb = (int)w.nvb;
  return spruce_sparse_attention_fwd_rows_impl(q, q_strides, k, k_strides, v, v_strides, indices, idx_strides, out,
                                               out_strides, dtype, B, Hq, Hkv, T, D, Kw, scale, 0, qb, nullptr, 0,
                                               status, stream, &virt);
}

int spruce_residual_frontier(const int32_t* selected, int64_t rows, int64_t K, int64_t qb, const int64_t* node_starts,
                             const int64_t* node_ends, const int32_t* node_parents, int64_t num_nodes, int32_t* out,
                             int64_t S, int32_t* row_counts, int32_t* max_count, void* stream) {
  if (rows < 0 || K < 0 || qb < 1 || num_nodes < 1 || S < 0)
    return fail(SPRUCE_ERR_INVALID, "bad frontier shape (rows=%lld, K=%lld, qb=%lld, nodes=%lld, S=%lld)",
                (long long)rows, (long long)K, (long long)qb, (long long)num_nodes, (long long)S);
  if (rows % qb) return fail(SPRUCE_ERR_INVALID, "rows must be a multiple of the query-block count");
  if (qb > 51200 || num_nodes > 2 * qb + 64 || K > 0x7fffffff)
    return fail(SPRUCE_ERR_UNSUPPORTED, "frontier shape too large (qb=%lld)", (long long)qb);
  if (rows == 0) return SPRUCE_OK;
  if (selected == nullptr && K > 0) return fail(SPRUCE_ERR_INVALID, "selected is NULL");
  if (node_starts == nullptr || node_ends == nullptr || node_parents == nullptr)
    return fail(SPRUCE_ERR_INVALID, "tree layout arrays are NULL");
  return cuda_status(spruce::launch_residual_frontier(selected, rows, (int)K, (int)qb, node_starts, node_ends,
                                                      node_parents, (int)num_nodes, out, (int)S, row_counts,
                                                      max_count, as_stream(stream)),
                     "residual frontier launch");
}

int64_t spruce_kv_summary_workspace_bytes(int64_t B, int64_t Hkv, int64_t T, int64_t D) {
  if (B < 0 || Hkv < 0 || T < 0 || D < 0) return -1;
  return spruce::kv_summary_workspace_bytes(B, Hkv, T, D);
}

int spruce_kv_summary_table(const void* key, const int64_t key_strides[4], const void* value,
                            const int64_t value_strides[4], const uint8_t* valid, int dtype, int64_t B, int64_t Hkv,
                            int64_t T, int64_t D, int64_t block_size, int64_t prototypes, const int64_t* node_starts,
                            const int64_t* node_ends, int64_t num_nodes, float* keys, float* values, float* counts,
                            float* log_counts, int64_t* range_starts, int64_t* range_ends, void* workspace,
                            int64_t workspace_bytes, void* stream) {
  if (!valid_dtype(dtype)) return fail(SPRUCE_ERR_INVALID, "unsupported dtype code %d", dtype);
  if (block_size < 1) return fail(SPRUCE_ERR_INVALID, "block_size must be positive, got %lld", (long long)block_size);
  if (prototypes != 1 && prototypes != 2 && prototypes != 4)
    return fail(SPRUCE_ERR_INVALID, "prototypes must be one of (1, 2, 4), got %lld", (long long)prototypes);
  if (B < 0 || Hkv < 0 || T < 1 || D < 1 || num_nodes < 0) return fail(SPRUCE_ERR_INVALID, "bad shape");
  if (key_strides[3] != 1 || value_strides[3] != 1)
    return fail(SPRUCE_ERR_UNSUPPORTED, "key/value need a unit last stride");
  if (B > 65535 || 2 * B * Hkv + B > 65535 || T > (int64_t)INT32_MAX - 16 || D > 65536 ||
      block_size > INT32_MAX || (T / 16 + 1) * D >= (int64_t)INT32_MAX - 256)
    return fail(SPRUCE_ERR_UNSUPPORTED, "summary table shape too large");
  const int64_t need = spruce::kv_summary_workspace_bytes(B, Hkv, T, D);
  if (workspace_bytes < need || (need > 0 && (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 15u))))
    return fail(SPRUCE_ERR_WORKSPACE, "workspace needs %lld bytes (16-byte aligned), got %lld", (long long)need,
                (long long)workspace_bytes);
  if (B == 0 || Hkv == 0 || num_nodes == 0) return SPRUCE_OK;
  spruce::KvSummaryArgs a{};
  a.key = key;
  a.value = value;
  for (int i = 0; i < 3; ++i) {
    a.ks[i] = key_strides[i];
    a.vs[i] = value_strides[i];
  }
  a.valid = valid;
  a.B = (int)B;
  a.H = (int)Hkv;
  a.T = (int)T;
  a.D = (int)D;
  a.P = (int)prototypes;
  a.block_size = block_size;
  a.node_starts = node_starts;
  a.node_ends = node_ends;
  a.nodes = num_nodes;
  a.out_keys = keys;
  a.out_values = values;
  a.out_counts = counts;
  a.out_log_counts = log_counts;
  a.range_starts = range_starts;
  a.range_ends = range_ends;
  a.prefix = static_cast<double*>(workspace);
  a.cprefix = reinterpret_cast<int64_t*>(static_cast<char*>(workspace) +
                                         2 * B * Hkv * (spruce::kv_summary_segments(T) + 1) * D * 8);  // 16-token worst case
  const bool vec = aligned16(key) && aligned16(value) && vec_strides_ok(key_strides, dtype, D) &&
                   vec_strides_ok(value_strides, dtype, D);
  a.seg = spruce::kv_summary_segment_tokens(block_size, (int)prototypes, vec ? D / (16 / elem_size(dtype)) : D);
  cudaError_t e;
  switch (dtype) {
    case SPRUCE_DTYPE_F32: e = spruce::launch_kv_summary<float>(a, vec, as_stream(stream)); break;
    case SPRUCE_DTYPE_BF16: e = spruce::launch_kv_summary<__nv_bfloat16>(a, vec, as_stream(stream)); break;
    default: e = spruce::launch_kv_summary<__half>(a, vec, as_stream(stream)); break;
  }
  return cuda_status(e, "summary table launch");
}

}  // extern "C"
