/*
 * CPU restatement of the SPRUCE sparse-prefill hot path -- TEST INFRASTRUCTURE.
 *
 * This file is the parity checker for the CUDA product path, never part of
 * it: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs load the library built from it.
 *
 * Parity is pinned: tests/golden/make_golden.py runs the reference's own torch
 * functions on seeded inputs and commits their outputs under tests/golden/;
 * tests/test_oracle_golden.py checks this restatement against them (indices
 * bit-exact, pooled features bit-exact, attention within fp32 round-off).
 *
 * Element types: 0 = float32, 1 = bfloat16, 2 = float16 (16-bit values are
 * passed as raw uint16 storage).  Rounding to 16-bit types is round-to-
 * nearest-even, as torch does.
 *
 * Compile with -ffp-contract=off: every rounding point below is deliberate.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

static inline float bf16_bits_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float f16_bits_to_f32(uint16_t h) {
    _Float16 x;
    memcpy(&x, &h, 2);
    return (float)x;
}

static inline uint16_t f32_to_f16_bits(float f) {
    _Float16 x = (_Float16)f;
    uint16_t h;
    memcpy(&h, &x, 2);
    return h;
}

static inline float load_elem(const void *p, int dtype, size_t i) {
    if (dtype == DT_F32) return ((const float *)p)[i];
    if (dtype == DT_BF16) return bf16_bits_to_f32(((const uint16_t *)p)[i]);
    return f16_bits_to_f32(((const uint16_t *)p)[i]);
}

static inline void store_elem(void *p, int dtype, size_t i, float v) {
    if (dtype == DT_F32) ((float *)p)[i] = v;
    else if (dtype == DT_BF16) ((uint16_t *)p)[i] = f32_to_bf16_bits(v);
    else ((uint16_t *)p)[i] = f32_to_f16_bits(v);
}

/* Value of v after a round trip through dtype. */
static inline float round_to(int dtype, float v) {
    if (dtype == DT_F32) return v;
    if (dtype == DT_BF16) return bf16_bits_to_f32(f32_to_bf16_bits(v));
    return f16_bits_to_f32(f32_to_f16_bits(v));
}

/*
 * Group average of query heads, teacher/chunked_extract.py:75-80
 * (_group_avg_tokens: x.view(b, G, H//G, L, d).mean(dim=2)).
 * torch's CPU mean over the head axis sums the H/G heads in order in fp32,
 * divides by H/G in fp32 and rounds once to the input dtype.
 * x: [B, H, T, D] contiguous; out: [B, G, T, D].
 */
void oracle_group_avg(const void *x, int dtype, int64_t B, int64_t H, int64_t T,
                      int64_t D, int64_t G, void *out) {
    const int64_t rep = H / G;
    const float frep = (float)rep;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t g = 0; g < G; ++g)
            for (int64_t t = 0; t < T; ++t)
                for (int64_t d = 0; d < D; ++d) {
                    float acc = 0.0f;
                    for (int64_t h = 0; h < rep; ++h) {
                        size_t src = (((size_t)b * H + g * rep + h) * T + t) * D + d;
                        acc = acc + load_elem(x, dtype, src);
                    }
                    size_t dst = (((size_t)b * G + g) * T + t) * D + d;
                    store_elem(out, dtype, dst, acc / frep);
                }
}

/*
 * Block mean (prototype 0 of _proto_pool_seq), teacher/chunked_extract.py:33-46.
 * The reference zero-pads the ragged tail, multiplies by the validity mask,
 * sums the 64 rows of each block and divides by the real row count:
 *   mean = (xb * vf).sum(dim=3) / counts
 * torch's CPU sum over that (non-innermost) axis accumulates 16 consecutive
 * rows at a time in fp32, then adds the chunk totals in order; the sum is
 * rounded to the input dtype, then divided by the count in fp32 and rounded
 * again.  Verified bit-exact against the reference for fp32, bf16 and fp16.
 * x: [B, H, T, D] contiguous; out: [B, H, nb, D] with nb = ceil(T / block).
 */
void oracle_block_mean(const void *x, int dtype, int64_t B, int64_t H, int64_t T,
                       int64_t D, int64_t block, void *out) {
    const int64_t nb = (T + block - 1) / block;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t i = 0; i < nb; ++i) {
                const int64_t t0 = i * block;
                const int64_t count = (T - t0) < block ? (T - t0) : block;
                for (int64_t d = 0; d < D; ++d) {
                    float total = 0.0f;
                    for (int64_t c = 0; c < block; c += 16) {
                        float chunk = 0.0f;
                        for (int64_t r = c; r < c + 16 && r < block; ++r) {
                            float v = 0.0f;
                            if (r < count)
                                v = load_elem(x, dtype, (((size_t)b * H + h) * T + t0 + r) * D + d);
                            chunk = chunk + v;
                        }
                        total = total + chunk;
                    }
                    float s = round_to(dtype, total);
                    size_t dst = (((size_t)b * H + h) * nb + i) * D + d;
                    store_elem(out, dtype, dst, s / (float)count);
                }
            }
}

/*
 * Gate projection, selector/gate.py:47-48 (einsum "gqid,dp->gqip").
 * Accumulation order is fixed: acc = fma(x[d], W[d][p], acc) for d = 0..D-1,
 * the order the CUDA kernel uses, so the two agree bit for bit.
 * x: [N, D] in dtype (converted to fp32 as selector/targets.py:34 does);
 * W: [D, P] fp32; out: [N, P] fp32.
 */
void oracle_project(const void *x, int dtype, int64_t N, int64_t D, const float *W,
                    int64_t P, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n)
        for (int64_t p = 0; p < P; ++p) {
            float acc = 0.0f;
            for (int64_t d = 0; d < D; ++d)
                acc = fmaf(load_elem(x, dtype, (size_t)n * D + d), W[(size_t)d * P + p], acc);
            out[(size_t)n * P + p] = acc;
        }
}

/*
 * FlatGate score with one prototype, selector/gate.py:57 and :101:
 *   s[i][j] = (qp_i . kp_j) / sqrt(p)
 * dot product as fma over p = 0..P-1; the division is a true fp32 division by
 * (float)sqrt(P) (torch divides by the python float math.sqrt(P)).
 * qp: [nq, P], kp: [nk, P]; out: [nq, nk].
 */
void oracle_scores(const float *qp, int64_t nq, const float *kp, int64_t nk, int64_t P,
                   float *out) {
    const float denom = (float)sqrt((double)P);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < nq; ++i)
        for (int64_t j = 0; j < nk; ++j) {
            float acc = 0.0f;
            for (int64_t p = 0; p < P; ++p)
                acc = fmaf(qp[(size_t)i * P + p], kp[(size_t)j * P + p], acc);
            out[(size_t)i * nk + j] = acc / denom;
        }
}

/* Order-preserving map from fp32 to uint32: a > b  <=>  key(a) > key(b).
 * NaN maps above +inf, as torch.topk treats NaN as the largest value. */
static inline uint32_t order_key(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct { uint32_t key; int32_t idx; } cand_t;

static int cand_cmp(const void *a, const void *b) {
    const cand_t *x = (const cand_t *)a, *y = (const cand_t *)b;
    if (x->key != y->key) return x->key > y->key ? -1 : 1;   /* larger score first */
    return x->idx < y->idx ? -1 : (x->idx > y->idx);          /* then lowest block id */
}

/*
 * Flat-gate top-k selection packed into selected_blocks rows.
 *
 * Restates the composition the reference uses for flat top-k routes
 * (scripts/route_overrides.py:187-205 teacher_topk_routes, with the flat
 * FlatGate scores of benchmarks/compare_dense_sparse_live_tree.py:314-320):
 *   mask future, sink and local-window blocks; ids = topk(W) with
 *   W = K - (local_window + 1) - sink_blocks;
 *   selected_ids_to_blocks(ids, K, local_window, key_blocks=kb, sink_blocks)
 *   (scripts/export_selected_blocks.py:80-175).
 * Per row q this is: sink blocks j < min(sink, kb) with j < q - local_window,
 * local blocks max(0, q - local_window)..q, and the W best-scoring candidates
 * j in [sink, q - local_window) -- ties broken toward the lowest block id,
 * which torch.topk leaves unspecified -- emitted in increasing order and
 * padded with -1 to K.
 * scores: [R, qb, kb] fp32 (R independent score matrices, e.g. KV groups);
 * out: [R, qb, K] int32.  Returns 0, or 1 if K cannot hold the forced blocks.
 */
int oracle_select_rows(const float *scores, int64_t R, int64_t qb, int64_t kb, int64_t K,
                       int64_t local_window, int64_t sink_blocks, int32_t *out) {
    if (K < local_window + 1 + sink_blocks) return 1;
    const int64_t sink = sink_blocks < kb ? sink_blocks : kb;
    int64_t W = K - (local_window + 1) - sink_blocks;
    if (W > kb) W = kb;
    int rc = 0;
#pragma omp parallel
    {
        cand_t *cand = (cand_t *)malloc(sizeof(cand_t) * (size_t)(kb > 0 ? kb : 1));
        unsigned char *keep = (unsigned char *)malloc((size_t)(kb > 0 ? kb : 1));
        if (!cand || !keep) {
#pragma omp atomic write
            rc = 2;
        }
#pragma omp for schedule(dynamic, 16)
        for (int64_t row = 0; row < R * qb; ++row) {
            if (!cand || !keep) continue;
            const int64_t q = row % qb;
            const float *s = scores + (size_t)row * kb;
            int32_t *o = out + (size_t)row * K;
            memset(keep, 0, (size_t)kb);
            int64_t n = 0;
            for (int64_t j = sink; j < q - local_window && j < kb; ++j) {
                cand[n].key = order_key(s[j]);
                cand[n].idx = (int32_t)j;
                ++n;
            }
            if (n > W) qsort(cand, (size_t)n, sizeof(cand_t), cand_cmp);
            const int64_t take = n < W ? n : W;
            for (int64_t c = 0; c < take; ++c) keep[cand[c].idx] = 1;
            for (int64_t j = 0; j < sink && j < q - local_window; ++j) keep[j] = 1;
            for (int64_t j = q - local_window < 0 ? 0 : q - local_window; j <= q && j < kb; ++j)
                keep[j] = 1;
            int64_t w = 0;
            for (int64_t j = 0; j < kb && j <= q && w < K; ++j)
                if (keep[j]) o[w++] = (int32_t)j;
            for (; w < K; ++w) o[w] = -1;
        }
        free(cand);
        free(keep);
    }
    return rc;
}

/*
 * selected_ids_to_blocks restatement, scripts/export_selected_blocks.py:80-175.
 * ids: [R, qb, C] int64 candidate ids (any value; invalid ones are ignored);
 * out: [R, qb, K] int32.  Policy per row q:
 *   nonlocal candidates: 0 <= id < kb, id <= q, id < q - local_window,
 *   id >= sink (export_selected_blocks.py:125-129), deduplicated, and only the
 *   `remaining` SMALLEST kept (:138-146) where
 *   remaining = K - min(q + 1, local_window + 1) - clamp(q - local_window, 0, sink);
 *   plus sink ids j < sink with j < q - local_window (:164-170) and local ids
 *   q - local_window .. q that are >= 0 (:153-158); sorted, first K, -1 pad.
 * Returns 0, or 1 on the argument errors the reference raises ValueError for.
 */
int oracle_pack_ids(const int64_t *ids, int64_t R, int64_t qb, int64_t C, int64_t K,
                    int64_t local_window, int64_t kb, int64_t sink_blocks, int32_t *out) {
    if (K < 1 || local_window < 0 || sink_blocks < 0 || kb < 1) return 1;
    if (K < local_window + 1 + sink_blocks) return 1;
    const int64_t sink = sink_blocks < kb ? sink_blocks : kb;
    const int64_t span = qb > kb ? qb : kb;
    int rc = 0;
#pragma omp parallel
    {
        unsigned char *mark = (unsigned char *)malloc((size_t)span + 1);
        if (!mark) {
#pragma omp atomic write
            rc = 2;
        }
#pragma omp for schedule(static)
        for (int64_t row = 0; row < R * qb; ++row) {
            if (!mark) continue;
            const int64_t q = row % qb;
            const int64_t *r = ids + (size_t)row * C;
            int32_t *o = out + (size_t)row * K;
            memset(mark, 0, (size_t)span + 1);
            for (int64_t c = 0; c < C; ++c) {
                const int64_t id = r[c];
                if (id >= 0 && id < kb && id <= q && id < q - local_window && id >= sink)
                    mark[id] = 1;
            }
            int64_t local_count = q + 1 < local_window + 1 ? q + 1 : local_window + 1;
            int64_t sink_count = q - local_window;
            if (sink_count < 0) sink_count = 0;
            if (sink_count > sink) sink_count = sink;
            int64_t remaining = K - local_count - sink_count;
            int64_t kept = 0;
            for (int64_t j = 0; j < span; ++j)
                if (mark[j]) {
                    if (kept < remaining) ++kept;
                    else mark[j] = 0;
                }
            for (int64_t j = 0; j < sink; ++j)
                if (j < q - local_window) mark[j] = 1;
            for (int64_t j = q - local_window; j <= q; ++j)
                if (j >= 0) mark[j] = 1;
            int64_t w = 0;
            for (int64_t j = 0; j < span && w < K; ++j)
                if (mark[j]) o[w++] = (int32_t)j;
            for (; w < K; ++w) o[w] = -1;
        }
        free(mark);
    }
    return rc;
}

/*
 * Block-sparse causal GQA attention, sparse/attention.py:143-274
 * (sparse_prefill_attention_forward without the HF mask and residual
 * summaries): for each batch, KV group g and query block, the key tokens of
 * the row's non-negative block ids (in row order, tokens >= T dropped,
 * :204-207), fp32 scores q.k / sqrt(D) (:217-219), future tokens masked
 * (:222-224), softmax in fp32 (:266), fp32 P.V (:267-269).  A row whose
 * tokens are all masked gets zeros (the reference would raise on an empty
 * row, :194-199; the direct-index kernels return zeros/NaN).
 * q: [B, Hq, T, D] fp32, k/v: [B, Hkv, T, D] fp32, idx: [B, Hkv, qb, Kw]
 * int32; out: [B, T, Hq, D] fp32 (token-major like the reference's return).
 */
void oracle_sparse_attention_rows(const float *q, const float *k, const float *v,
                                  const int32_t *idx, int64_t B, int64_t Hq, int64_t Hkv,
                                  int64_t T, int64_t D, int64_t Kw, int64_t block, float scale,
                                  int64_t q_begin, int64_t q_end, float *out);

void oracle_sparse_attention(const float *q, const float *k, const float *v,
                             const int32_t *idx, int64_t B, int64_t Hq, int64_t Hkv,
                             int64_t T, int64_t D, int64_t Kw, int64_t block, float scale,
                             float *out) {
    const int64_t qb = (T + block - 1) / block;
    oracle_sparse_attention_rows(q, k, v, idx, B, Hq, Hkv, T, D, Kw, block, scale, 0, qb, out);
}

/* Same, restricted to query blocks [q_begin, q_end) (other output rows untouched). */
void oracle_sparse_attention_rows(const float *q, const float *k, const float *v,
                                  const int32_t *idx, int64_t B, int64_t Hq, int64_t Hkv,
                                  int64_t T, int64_t D, int64_t Kw, int64_t block, float scale,
                                  int64_t q_begin, int64_t q_end, float *out) {
    const int64_t qb = (T + block - 1) / block;
    const int64_t nq = q_end - q_begin;
    const int64_t rep = Hq / Hkv;
#pragma omp parallel
    {
        int64_t *keys = (int64_t *)malloc(sizeof(int64_t) * (size_t)(Kw * block + 1));
        float *s = (float *)malloc(sizeof(float) * (size_t)(Kw * block + 1));
        double *acc = (double *)malloc(sizeof(double) * (size_t)D);
#pragma omp for schedule(dynamic, 1)
        for (int64_t unit = 0; unit < B * Hkv * nq * rep; ++unit) {
            const int64_t hh = unit % rep;
            const int64_t b = unit / (Hkv * nq * rep);
            const int64_t g = (unit / (nq * rep)) % Hkv;
            const int64_t i = q_begin + (unit / rep) % nq;
            const int32_t *row = idx + (((size_t)b * Hkv + g) * qb + i) * Kw;
            int64_t nk = 0;
            for (int64_t c = 0; c < Kw; ++c) {
                if (row[c] < 0) continue;
                for (int64_t t = 0; t < block; ++t) {
                    int64_t key = (int64_t)row[c] * block + t;
                    if (key < T) keys[nk++] = key;
                }
            }
            const float *kg = k + ((size_t)b * Hkv + g) * T * D;
            const float *vg = v + ((size_t)b * Hkv + g) * T * D;
            {
                const int64_t h = g * rep + hh;
                for (int64_t t = i * block; t < (i + 1) * block && t < T; ++t) {
                    const float *qr = q + (((size_t)b * Hq + h) * T + t) * D;
                    float m = -INFINITY;
                    for (int64_t c = 0; c < nk; ++c) {
                        if (keys[c] > t) { s[c] = -INFINITY; continue; }
                        const float *kr = kg + (size_t)keys[c] * D;
                        float dot = 0.0f;
                        for (int64_t d = 0; d < D; ++d) dot += qr[d] * kr[d];
                        s[c] = dot * scale;
                        if (s[c] > m) m = s[c];
                    }
                    float *o = out + (((size_t)b * T + t) * Hq + h) * D;
                    if (m == -INFINITY) {
                        for (int64_t d = 0; d < D; ++d) o[d] = 0.0f;
                        continue;
                    }
                    double l = 0.0;
                    for (int64_t d = 0; d < D; ++d) acc[d] = 0.0;
                    for (int64_t c = 0; c < nk; ++c) {
                        if (s[c] == -INFINITY) continue;
                        const double p = exp((double)s[c] - (double)m);
                        l += p;
                        const float *vr = vg + (size_t)keys[c] * D;
                        for (int64_t d = 0; d < D; ++d) acc[d] += p * (double)vr[d];
                    }
                    for (int64_t d = 0; d < D; ++d) o[d] = (float)(acc[d] / l);
                }
            }
        }
        free(keys);
        free(s);
        free(acc);
    }
}

/*
 * Residual-summary attention, sparse/attention.py:178-265: per (b, g, query
 * block i, head, token) the scores of the selected blocks' causal keys (as
 * in oracle_sparse_attention_rows), then, for each residual node id
 * nodes[b, g, i, s] >= 0 in order and each prototype p with
 * counts[b, node, p] > 0, the summary score q.key * scale + log_counts[b,
 * node, p] (no causal mask), one softmax over both (double sums) and the
 * matching values.  Summary table: keys/values [B, Hkv, NN, P, D],
 * counts/log_counts [B, NN, P]; nodes [B, Hkv, qb, S].
 */
void oracle_residual_attention(const float *q, const float *k, const float *v, const int32_t *idx,
                               const int32_t *nodes, int64_t S, const float *skeys, const float *svalues,
                               const float *scounts, const float *slogc, int64_t NN, int64_t P,
                               int64_t B, int64_t Hq, int64_t Hkv, int64_t T, int64_t D, int64_t Kw,
                               int64_t block, float scale, float *out) {
    const int64_t qb = (T + block - 1) / block;
    const int64_t rep = Hq / Hkv;
    const int64_t cap = Kw * block + S * P + 1;
#pragma omp parallel
    {
        /* key c: >= 0 a token of the sequence, < 0 summary row -(1 + s * P + p) */
        int64_t *keys = (int64_t *)malloc(sizeof(int64_t) * (size_t)cap);
        float *sc = (float *)malloc(sizeof(float) * (size_t)cap);
        double *acc = (double *)malloc(sizeof(double) * (size_t)D);
#pragma omp for schedule(dynamic, 1)
        for (int64_t unit = 0; unit < B * Hkv * qb * rep; ++unit) {
            const int64_t hh = unit % rep;
            const int64_t b = unit / (Hkv * qb * rep);
            const int64_t g = (unit / (qb * rep)) % Hkv;
            const int64_t i = (unit / rep) % qb;
            const int32_t *row = idx + (((size_t)b * Hkv + g) * qb + i) * Kw;
            const int32_t *nrow = nodes + (((size_t)b * Hkv + g) * qb + i) * S;
            int64_t nk = 0;
            for (int64_t c = 0; c < Kw; ++c) {
                if (row[c] < 0) continue;
                for (int64_t t = 0; t < block; ++t) {
                    int64_t key = (int64_t)row[c] * block + t;
                    if (key < T) keys[nk++] = key;
                }
            }
            for (int64_t s = 0; s < S; ++s) {
                const int32_t node = nrow[s];
                if (node < 0 || node >= NN) continue;
                for (int64_t p = 0; p < P; ++p)
                    if (scounts[((size_t)b * NN + node) * P + p] > 0.0f) keys[nk++] = -(1 + s * P + p);
            }
            const float *kg = k + ((size_t)b * Hkv + g) * T * D;
            const float *vg = v + ((size_t)b * Hkv + g) * T * D;
            const int64_t h = g * rep + hh;
            for (int64_t t = i * block; t < (i + 1) * block && t < T; ++t) {
                const float *qr = q + (((size_t)b * Hq + h) * T + t) * D;
                float m = -INFINITY;
                for (int64_t c = 0; c < nk; ++c) {
                    const float *kr;
                    float bias = 0.0f;
                    if (keys[c] >= 0) {
                        if (keys[c] > t) { sc[c] = -INFINITY; continue; }
                        kr = kg + (size_t)keys[c] * D;
                    } else {
                        const int64_t e = -keys[c] - 1, node = nrow[e / P], p = e % P;
                        kr = skeys + ((((size_t)b * Hkv + g) * NN + node) * P + p) * D;
                        bias = slogc[((size_t)b * NN + node) * P + p];
                    }
                    float dot = 0.0f;
                    for (int64_t d = 0; d < D; ++d) dot += qr[d] * kr[d];
                    sc[c] = dot * scale + bias;
                    if (sc[c] > m) m = sc[c];
                }
                float *o = out + (((size_t)b * T + t) * Hq + h) * D;
                if (m == -INFINITY) {
                    for (int64_t d = 0; d < D; ++d) o[d] = 0.0f;
                    continue;
                }
                double l = 0.0;
                for (int64_t d = 0; d < D; ++d) acc[d] = 0.0;
                for (int64_t c = 0; c < nk; ++c) {
                    if (sc[c] == -INFINITY) continue;
                    const double pr = exp((double)sc[c] - (double)m);
                    l += pr;
                    const float *vr;
                    if (keys[c] >= 0) {
                        vr = vg + (size_t)keys[c] * D;
                    } else {
                        const int64_t e = -keys[c] - 1, node = nrow[e / P], p = e % P;
                        vr = svalues + ((((size_t)b * Hkv + g) * NN + node) * P + p) * D;
                    }
                    for (int64_t d = 0; d < D; ++d) acc[d] += pr * (double)vr[d];
                }
                for (int64_t d = 0; d < D; ++d) o[d] = (float)(acc[d] / l);
            }
        }
        free(keys);
        free(sc);
        free(acc);
    }
}

/*
 * build_kv_summary_table, sparse/summaries.py:52-142, with the prototype
 * token ranges of _prototype_token_ranges (:29-49).
 *
 * x [B, H, T, D] contiguous (key, then value), valid uint8 [B, T] or NULL.
 * Node ranges are in blocks (ResidualTreeLayout.starts/ends).  The reference
 * takes an fp32 cumsum of valid-masked rows (:100-114); torch's CPU cumsum
 * accumulates in double and rounds each prefix to float, which is what the
 * running `acc` below does.  Means are fp32 prefix differences divided by
 * max(count, 1) (:127-129); log_counts = log(count) or -inf (:130-134), here
 * the correctly rounded float of the double log.
 */
static void summary_prefix_column(const void *x, int dtype, const uint8_t *valid, int64_t T, int64_t D,
                                  float *prefix) {
    double acc = 0.0;
    prefix[0] = 0.0f;
    for (int64_t t = 0; t < T; ++t) {
        float w = load_elem(x, dtype, (size_t)(t * D));
        if (valid && !valid[t]) w = 0.0f * w;
        acc += (double)w;
        prefix[t + 1] = (float)acc;
    }
}

void oracle_kv_summary_table(const void *key, const void *value, int dtype, const uint8_t *valid, int64_t B,
                             int64_t H, int64_t T, int64_t D, int64_t block_size, int64_t P,
                             const int64_t *node_starts, const int64_t *node_ends, int64_t nodes, float *keys,
                             float *values, float *counts, float *log_counts, int64_t *range_starts,
                             int64_t *range_ends) {
    for (int64_t n = 0; n < nodes; ++n) {
        int64_t ts = node_starts[n] * block_size, te = node_ends[n] * block_size;
        if (ts > T) ts = T;
        if (te > T) te = T;
        const int64_t len = te - ts;
        for (int64_t p = 0; p < P; ++p) {
            range_starts[n * P + p] = ts + len * p / P;
            range_ends[n * P + p] = ts + len * (p + 1) / P;
        }
    }
    const size_t es = dtype == DT_F32 ? 4 : 2;
    for (int64_t b = 0; b < B; ++b) {
        const uint8_t *vb = valid ? valid + b * T : NULL;
        /* count prefix: double cumsum of 0/1 values, exact integers */
        int64_t *cprefix = (int64_t *)malloc((size_t)(T + 1) * sizeof(int64_t));
        cprefix[0] = 0;
        for (int64_t t = 0; t < T; ++t) cprefix[t + 1] = cprefix[t] + (vb ? (vb[t] != 0) : 1);
        for (int64_t i = 0; i < nodes * P; ++i) {
            const float c = (float)(cprefix[range_ends[i]] - cprefix[range_starts[i]]);
            counts[b * nodes * P + i] = c;
            log_counts[b * nodes * P + i] = c > 0.0f ? (float)log((double)c) : -INFINITY;
        }
        free(cprefix);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
        for (int64_t h = 0; h < H; ++h) {
            for (int64_t d = 0; d < D; ++d) {
                float *prefix = (float *)malloc((size_t)(T + 1) * sizeof(float));
                for (int which = 0; which < 2; ++which) {
                    const char *src = (const char *)(which ? value : key) + ((b * H + h) * T * D + d) * es;
                    float *dst = which ? values : keys;
                    summary_prefix_column(src, dtype, vb, T, D, prefix);
                    for (int64_t i = 0; i < nodes * P; ++i) {
                        float c = counts[b * nodes * P + i];
                        if (c < 1.0f) c = 1.0f;
                        const float pooled = prefix[range_ends[i]] - prefix[range_starts[i]];
                        dst[((b * H + h) * nodes * P + i) * D + d] = pooled / c;
                    }
                }
                free(prefix);
            }
        }
    }
}

/*
 * MaxSim gate scores, selector/gate.py:29-101 (forward) and :132-171
 * (candidate scoring): out[r, q, c] = max over (i, j) of
 * qp[r,q,i,:] . kp[r,key,j,:] / sqrt(pdim), key = c or ids[r,q,c] clamped to
 * [0, nk).  The reference takes the dots as einsum / matmul reductions; here
 * each dot is one fmaf chain in index order (the fixed order of the CUDA
 * kernel), so the two agree bit for bit and sit within fp32 rounding of the
 * reference.
 */
void oracle_maxsim(const float *qp, const float *kp, const int64_t *ids, int64_t R, int64_t nq, int64_t nk,
                   int64_t ncols, int64_t P, int64_t pdim, float *out) {
    const float denom = (float)sqrt((double)pdim);
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static)
#endif
    for (int64_t r = 0; r < R; ++r) {
        for (int64_t q = 0; q < nq; ++q) {
            const float *qrow = qp + (r * nq + q) * P * pdim;
            for (int64_t c = 0; c < ncols; ++c) {
                int64_t key = c;
                if (ids) {
                    key = ids[(r * nq + q) * ncols + c];
                    key = key < 0 ? 0 : (key >= nk ? nk - 1 : key);
                }
                const float *krow = kp + (r * nk + key) * P * pdim;
                float best = -INFINITY;
                for (int64_t i = 0; i < P; ++i)
                    for (int64_t j = 0; j < P; ++j) {
                        float acc = 0.0f;
                        for (int64_t x = 0; x < pdim; ++x) acc = fmaf(qrow[i * pdim + x], krow[j * pdim + x], acc);
                        if (acc > best) best = acc;
                    }
                out[(r * nq + q) * ncols + c] = best / denom;
            }
        }
    }
}

/* Number of threads the OpenMP runtime will use (for the CPU-baseline report). */
int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
