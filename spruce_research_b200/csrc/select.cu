// Flat-gate selection: projection, scores, masked top-k and packing into
// selected_blocks rows; plus the reference's id packer and validator.
//
// References: selector/gate.py:47-101 (FlatGate, P = 1),
// scripts/route_overrides.py:187-205 (topk -> selected_ids_to_blocks),
// scripts/export_selected_blocks.py:80-175 (packing policy),
// interfaces/validator.py:7-62 (row rules).
//
// Every score is a fixed-order fp32 fma chain over the projection dim
// followed by a true division by sqrt(P), so the CUDA result equals the CPU
// restatement bit for bit; the top-k is an exact radix select on the
// order-preserving integer image of the scores with ties broken toward the
// lowest block id, so indices are bit-exact too.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace spruce {

// ------------------------------------------------------------------ projection

// Row n of the launch is row (n / nrows) * qb + row0 + n % nrows of x (and of out).
// ROWS rows per 128-thread CTA (4, or 16 when there are many rows so that W
// is read from L2 fewer times): the rows are staged in shared memory, thread
// p keeps one accumulator per row and reads 16 weights at a time.
// Each output is one fma chain over d = 0..D-1 in order.
constexpr int kProjRows = 4;

template <typename T, int ROWS>
__global__ void __launch_bounds__(128) project_kernel(const T* __restrict__ x, int64_t N, int D,
                                                      const float* __restrict__ W, int P, float* __restrict__ out,
                                                      int qb, int row0, int nrows) {
  extern __shared__ float xs[];  // [ROWS][D]
  const int64_t n0 = (int64_t)blockIdx.x * ROWS;
  const int rows = (int)(N - n0 < ROWS ? N - n0 : ROWS);
  auto map_row = [&](int64_t n) { return (n / nrows) * qb + row0 + n % nrows; };
  for (int e = threadIdx.x; e < rows * D; e += blockDim.x) xs[e] = Elem<T>::to_f(x[map_row(n0 + e / D) * D + e % D]);
  for (int e = rows * D + threadIdx.x; e < ROWS * D; e += blockDim.x) xs[e] = 0.0f;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    float acc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
    int d = 0;
    for (; d + 16 <= D; d += 16) {  // 16 weight loads in flight, then the chains in d order
      float w[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) w[u] = __ldg(W + (int64_t)(d + u) * P + p);
#pragma unroll
      for (int u = 0; u < 16; ++u)
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = __fmaf_rn(xs[r * D + d + u], w[u], acc[r]);
    }
    for (; d < D; ++d) {
      const float w = __ldg(W + (int64_t)d * P + p);
#pragma unroll
      for (int r = 0; r < ROWS; ++r) acc[r] = __fmaf_rn(xs[r * D + d], w, acc[r]);
    }
    for (int r = 0; r < rows; ++r) out[map_row(n0 + r) * P + p] = acc[r];
  }
}

// The same projection with one thread per output (row, p), for few rows: a
// row-tiled CTA per 4 rows would leave most SMs idle, while per-output
// threads spread the (tiny) work over every SM.  128-thread blocks along p,
// so a warp shares its row (broadcast loads of x) and reads 32 consecutive
// weights; one fma chain over d = 0..D-1 in order per output.
template <typename T>
__global__ void __launch_bounds__(128) project_out_kernel(const T* __restrict__ x, int64_t N, int D,
                                                          const float* __restrict__ W, int P,
                                                          float* __restrict__ out, int qb, int row0, int nrows) {
  const int64_t idx = (int64_t)blockIdx.x * 128 + threadIdx.x;
  if (idx >= N * P) return;
  const int p = (int)(idx % P);
  const int64_t n = idx / P;
  const int64_t row = (n / nrows) * qb + row0 + n % nrows;
  const T* xr = x + row * D;
  float acc = 0.0f;
  int d = 0;
  for (; d + 8 <= D; d += 8) {  // 16 loads in flight, then the chain in d order
    float xv[8], wv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      xv[u] = Elem<T>::to_f(xr[d + u]);
      wv[u] = __ldg(W + (int64_t)(d + u) * P + p);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fmaf_rn(xv[u], wv[u], acc);
  }
  for (; d < D; ++d) acc = __fmaf_rn(Elem<T>::to_f(xr[d]), __ldg(W + (int64_t)d * P + p), acc);
  out[row * P + p] = acc;
}

// ------------------------------------------------------------------ score tiles
// A CTA of 256 threads scores ROWS query rows against 256 key columns at a
// time: thread t owns column j0 + t and keeps ROWS fp32 accumulators; the
// key projections are staged transposed in shared memory, 32 p at a time.
constexpr int kScoreThreads = 256;
constexpr int kPChunk = 32;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;  // NaN sorts above +inf (torch.topk)
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// qs: [ROWS][P] query projections in smem; kT: [kPChunk][kScoreThreads] staging.
// Writes fp32 scores of columns [j0, j0 + 256) ∩ [0, ncols) via `emit(r, j, s)`.
template <int ROWS, typename Emit>
__device__ __forceinline__ void score_columns(const float* qs, const float* __restrict__ kp, int P, int j0,
                                              int ncols, float* kT, float denom, Emit emit, int qstride = -1) {
  if (qstride < 0) qstride = P;
  const int t = threadIdx.x;
  float acc[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
  for (int p0 = 0; p0 < P; p0 += kPChunk) {
    __syncthreads();
    // Stage kp[j0 .. j0+255][p0 .. p0+31] transposed: coalesced along p.
    for (int e = t; e < kPChunk * kScoreThreads; e += kScoreThreads) {
      const int jj = e / kPChunk;
      const int pp = e % kPChunk;
      const int j = j0 + jj;
      kT[pp * kScoreThreads + jj] = (j < ncols && p0 + pp < P) ? __ldg(kp + (int64_t)j * P + p0 + pp) : 0.0f;
    }
    __syncthreads();
    const int pn = min(kPChunk, P - p0);
    for (int pp = 0; pp < pn; ++pp) {
      const float kv = kT[pp * kScoreThreads + t];
#pragma unroll
      for (int r = 0; r < ROWS; ++r) acc[r] = __fmaf_rn(qs[r * qstride + p0 + pp], kv, acc[r]);
    }
  }
  const int j = j0 + t;
  if (j < ncols) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) emit(r, j, __fdiv_rn(acc[r], denom));
  }
}

// 16 query rows x 256 key columns with 4x4 register micro-tiles: thread t owns
// rows 4*(t/64)..+3 and columns j0 + (t%64) + 64*c, c = 0..3.  Key
// projections are staged 32 p at a time, row-major with a 36-float stride
// (conflict-free 16-byte loads); query rows are read as broadcast float4s.
// Every output is still one fma chain over p = 0..P-1 in order, so scores
// equal score_columns' (and the CPU restatement's) bit for bit.
constexpr int kKStride = 36;

template <typename Emit>
__device__ __forceinline__ void score_tile16(const float* qs, int qstride, const float* __restrict__ kp, int P,
                                             int j0, int ncols, float* ks, float denom, Emit emit) {
  const int t = threadIdx.x;
  const int rg = t >> 6;
  const int cg = t & 63;
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
  for (int p0 = 0; p0 < P; p0 += kPChunk) {
    const int pn = min(kPChunk, P - p0);
    __syncthreads();
    for (int e = t; e < kScoreThreads * kPChunk; e += kScoreThreads) {
      const int jj = e >> 5;
      const int pp = e & 31;
      const int j = j0 + jj;
      ks[jj * kKStride + pp] = (j < ncols && pp < pn) ? __ldg(kp + (int64_t)j * P + p0 + pp) : 0.0f;
    }
    __syncthreads();
    int pp = 0;
    for (; pp + 4 <= pn; pp += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) qv[r] = *reinterpret_cast<const float4*>(qs + (4 * rg + r) * qstride + p0 + pp);
#pragma unroll
      for (int c = 0; c < 4; ++c) kv[c] = *reinterpret_cast<const float4*>(ks + (cg + 64 * c) * kKStride + pp);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          acc[r][c] = __fmaf_rn(qv[r].x, kv[c].x, acc[r][c]);
          acc[r][c] = __fmaf_rn(qv[r].y, kv[c].y, acc[r][c]);
          acc[r][c] = __fmaf_rn(qv[r].z, kv[c].z, acc[r][c]);
          acc[r][c] = __fmaf_rn(qv[r].w, kv[c].w, acc[r][c]);
        }
    }
    for (; pp < pn; ++pp)
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          acc[r][c] = __fmaf_rn(qs[(4 * rg + r) * qstride + p0 + pp], ks[(cg + 64 * c) * kKStride + pp], acc[r][c]);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int j = j0 + cg + 64 * c;
    if (j < ncols)
#pragma unroll
      for (int r = 0; r < 4; ++r) emit(4 * rg + r, j, __fdiv_rn(acc[r][c], denom));
  }
}

// 16-byte asynchronous global->shared copy; src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async16(float* dst, const float* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 4*RM query rows against all column chunks [0, ncols), RM x 4 register
// micro-tiles (thread t: rows RM*(t/64).., columns j0 + t%64 + 64c), with the
// key projections staged by cp.async into two alternating buffers
// (ks2: 2 x [256][kKStride]): the copy of stage s+1 (a 256-column x 32-p
// slab) is in flight while stage s is multiplied.  Every score is one fma
// chain over p = 0..P-1 in order, as in score_tile16 / score_columns, so the
// scores are bit-identical.  Needs P % 4 == 0 (16-byte aligned key rows).
template <int RM, typename Emit>
__device__ __forceinline__ void score_rows_async(const float* qs, int qstride, const float* __restrict__ kp,
                                                 int P, int ncols, float* ks2, float denom, Emit emit) {
  const int t = threadIdx.x;
  const int rg = t >> 6;
  const int cg = t & 63;
  const int npc = (P + kPChunk - 1) / kPChunk;
  const int total = ((ncols + kScoreThreads - 1) / kScoreThreads) * npc;
  if (total == 0) return;
  auto issue = [&](int st) {
    const int j0 = (st / npc) * kScoreThreads, p0 = (st % npc) * kPChunk;
    float* buf = ks2 + (st & 1) * (kScoreThreads * kKStride);
#pragma unroll
    for (int i = 0; i < kPChunk * kScoreThreads / 4 / kScoreThreads; ++i) {
      const int e = t + kScoreThreads * i;
      const int jj = e >> 3, part = e & 7;
      const int j = j0 + jj, p = p0 + part * 4;
      const bool ok = j < ncols && p < P;
      cp_async16(buf + jj * kKStride + part * 4, ok ? kp + (int64_t)j * P + p : kp, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  issue(0);
  float acc[RM][4];
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
  for (int st = 0; st < total; ++st) {
    if (st + 1 < total) {
      issue(st + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* ks = ks2 + (st & 1) * (kScoreThreads * kKStride);
    const int pc = st % npc;
    const int p0 = pc * kPChunk;
    const int pn = P % kPChunk == 0 ? kPChunk : min(kPChunk, P - p0);
#pragma unroll
    for (int pp = 0; pp < pn; pp += 4) {
      float4 qv[RM], kv[4];
#pragma unroll
      for (int r = 0; r < RM; ++r) qv[r] = *reinterpret_cast<const float4*>(qs + (RM * rg + r) * qstride + p0 + pp);
#pragma unroll
      for (int c = 0; c < 4; ++c) kv[c] = *reinterpret_cast<const float4*>(ks + (cg + 64 * c) * kKStride + pp);
      // p = pp, pp+1, pp+2, pp+3 in turn across all RM x 4 accumulators: each chain keeps its order,
      // and consecutive fmas are independent (no wait on the previous one's result)
#pragma unroll
      for (int r = 0; r < RM; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = __fmaf_rn(qv[r].x, kv[c].x, acc[r][c]);
#pragma unroll
      for (int r = 0; r < RM; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = __fmaf_rn(qv[r].y, kv[c].y, acc[r][c]);
#pragma unroll
      for (int r = 0; r < RM; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = __fmaf_rn(qv[r].z, kv[c].z, acc[r][c]);
#pragma unroll
      for (int r = 0; r < RM; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = __fmaf_rn(qv[r].w, kv[c].w, acc[r][c]);
    }
    if (pc == npc - 1) {
      const int j0 = (st / npc) * kScoreThreads;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = j0 + cg + 64 * c;
        if (j < ncols)
#pragma unroll
          for (int r = 0; r < RM; ++r) emit(RM * rg + r, j, __fdiv_rn(acc[r][c], denom));
      }
#pragma unroll
      for (int r = 0; r < RM; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
    }
    __syncthreads();  // buffer st & 1 is refilled by the issue at the top of iteration st + 1
  }
}

// 16 query rows against 512-column slabs with 512 threads: thread t owns rows
// 8*(t/256)..+7 and the columns j0 + t%256 and j0 + t%256 + 256 (an 8 x 2
// register tile).  Key projections are staged 16 p at a time by cp.async into
// two alternating buffers (ks2: 2 x [512][kK16Stride]); query rows are read as
// broadcast float4s (a warp's lanes share their rows).  Per 4-p step and warp:
// 8 (q) + 8 (k) shared-memory wavefronts against 16 FMA issue cycles, and 16
// warps per SM where the 256-thread 4 x 4 tile ran 8 (its 128 KB of keys allow
// one CTA per SM) and stalled on dependent fmas.  Every score is still one fma
// chain over p = 0..P-1 in order, so the scores are bit-identical to
// score_rows_async / score_columns.  Needs P % 4 == 0.
constexpr int kSelThreads16 = 512;
constexpr int kSlab16 = 512;
constexpr int kP16 = 16;
constexpr int kK16Stride = 20;  // 80-byte rows: the 16-byte loads of 8 consecutive lanes cover all 32 banks

template <typename Emit>
__device__ __forceinline__ void score_rows16_async(const float* qs, int qstride, const float* __restrict__ kp, int P,
                                                   int ncols, float* ks2, float denom, Emit emit) {
  const int t = threadIdx.x;
  const int rg = t >> 8;
  const int ct = t & 255;
  const int npc = (P + kP16 - 1) / kP16;
  const int total = ((ncols + kSlab16 - 1) / kSlab16) * npc;
  if (total == 0) return;
  auto issue = [&](int st) {
    const int j0 = (st / npc) * kSlab16, p0 = (st % npc) * kP16;
    float* buf = ks2 + (st & 1) * (kSlab16 * kK16Stride);
#pragma unroll
    for (int i = 0; i < kSlab16 * (kP16 / 4) / kSelThreads16; ++i) {
      const int e = t + kSelThreads16 * i;
      const int jj = e >> 2, part = e & 3;
      const int j = j0 + jj, p = p0 + part * 4;
      const bool ok = j < ncols && p < P;
      cp_async16(buf + jj * kK16Stride + part * 4, ok ? kp + (int64_t)j * P + p : kp, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  issue(0);
  const float* qrow = qs + 8 * rg * qstride;
  float acc[8][2];
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[r][0] = acc[r][1] = 0.0f;
  for (int st = 0; st < total; ++st) {
    if (st + 1 < total) {
      issue(st + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* ks = ks2 + (st & 1) * (kSlab16 * kK16Stride);
    const int pc = st % npc;
    const int p0 = pc * kP16;
    const int pn = P % kP16 == 0 ? kP16 : min(kP16, P - p0);
    // Columns past the tile's causal range are not multiplied: a warp skips each
    // of its two 32-column sets that lies wholly at or past ncols (warp-uniform).
    const int jw = (st / npc) * kSlab16 + (ct & ~31);
    const bool c0 = jw < ncols, c1 = jw + 256 < ncols;
    if (c1) {
#pragma unroll
      for (int pp = 0; pp < pn; pp += 4) {
        const float4 k0 = *reinterpret_cast<const float4*>(ks + ct * kK16Stride + pp);
        const float4 k1 = *reinterpret_cast<const float4*>(ks + (ct + 256) * kK16Stride + pp);
        float4 qv[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) qv[r] = *reinterpret_cast<const float4*>(qrow + r * qstride + p0 + pp);
        // p = pp .. pp+3 in turn across all 16 accumulators: each chain keeps its order, and
        // consecutive fmas are independent
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[r][0] = __fmaf_rn(qv[r].x, k0.x, acc[r][0]);
          acc[r][1] = __fmaf_rn(qv[r].x, k1.x, acc[r][1]);
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[r][0] = __fmaf_rn(qv[r].y, k0.y, acc[r][0]);
          acc[r][1] = __fmaf_rn(qv[r].y, k1.y, acc[r][1]);
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[r][0] = __fmaf_rn(qv[r].z, k0.z, acc[r][0]);
          acc[r][1] = __fmaf_rn(qv[r].z, k1.z, acc[r][1]);
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          acc[r][0] = __fmaf_rn(qv[r].w, k0.w, acc[r][0]);
          acc[r][1] = __fmaf_rn(qv[r].w, k1.w, acc[r][1]);
        }
      }
    } else if (c0) {
#pragma unroll
      for (int pp = 0; pp < pn; pp += 4) {
        const float4 k0 = *reinterpret_cast<const float4*>(ks + ct * kK16Stride + pp);
        float4 qv[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) qv[r] = *reinterpret_cast<const float4*>(qrow + r * qstride + p0 + pp);
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r][0] = __fmaf_rn(qv[r].x, k0.x, acc[r][0]);
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r][0] = __fmaf_rn(qv[r].y, k0.y, acc[r][0]);
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r][0] = __fmaf_rn(qv[r].z, k0.z, acc[r][0]);
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r][0] = __fmaf_rn(qv[r].w, k0.w, acc[r][0]);
      }
    }
    if (pc == npc - 1) {
      const int j0 = (st / npc) * kSlab16;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int j = j0 + ct + 256 * c;
        if (j < ncols)
#pragma unroll
          for (int r = 0; r < 8; ++r) emit(8 * rg + r, j, __fdiv_rn(acc[r][c], denom));
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) acc[r][0] = acc[r][1] = 0.0f;
    }
    __syncthreads();  // buffer st & 1 is refilled by the issue at the top of iteration st + 1
  }
}

// Threads and staging floats of select_kernel: 512 threads and two
// [512][kK16Stride] slabs for 16-row tiles; 256 threads and two [256][kKStride]
// slabs for 8-row tiles, one for smaller tiles.  After the scores the staging
// holds the selection's per-warp histograms ([warps][256] ints).
__host__ __device__ constexpr int select_threads(int rows) { return rows >= 16 ? kSelThreads16 : kScoreThreads; }
__host__ __device__ constexpr int select_stage_floats(int rows) {
  return rows >= 16 ? 2 * kSlab16 * kK16Stride : (rows >= 8 ? 2 : 1) * kScoreThreads * kKStride;
}
static_assert(select_stage_floats(16) >= select_threads(16) / 32 * 256 &&
                  select_stage_floats(4) >= select_threads(4) / 32 * 256,
              "the histograms fit in the staging");

// Full score matrix (FlatGate.forward, P = 1): grid (ceil(qb/ROWS), R).
template <int ROWS>
__global__ void __launch_bounds__(kScoreThreads) scores_kernel(const float* __restrict__ qp,
                                                               const float* __restrict__ kp, int qb, int kb, int P,
                                                               float* __restrict__ out, float denom) {
  static_assert(ROWS == 16, "the full-matrix scorer uses 16-row tiles");
  extern __shared__ float sm[];
  const int qstride = (P + 3) / 4 * 4 + 4;
  float* qs = sm;                   // [16][qstride]
  float* kT = sm + ROWS * qstride;  // [256][kKStride]
  const int r0 = blockIdx.x * ROWS;
  const int64_t mat = blockIdx.y;
  const float* q = qp + mat * qb * P;
  const float* k = kp + mat * kb * P;
  for (int e = threadIdx.x; e < ROWS * qstride; e += kScoreThreads) {
    const int r = e / qstride;
    const int pcol = e % qstride;
    qs[e] = (r0 + r < qb && pcol < P) ? q[(int64_t)(r0 + r) * P + pcol] : 0.0f;
  }
  for (int j0 = 0; j0 < kb; j0 += kScoreThreads) {
    score_tile16(qs, qstride, k, P, j0, kb, kT, denom, [&](int r, int j, float s) {
      if (r0 + r < qb) out[(mat * qb + r0 + r) * kb + j] = s;
    });
  }
}

// ------------------------------------------------------------------ fused select
struct SelectArgs {
  const float* qp;   // [B, G, qb, P]
  const float* kp;   // [B, G, qb, P]
  int B, G, qb, P, K, local_window, sink, W;
  int q_begin, q_end;  // query-block rows [q_begin, q_end) are selected
  int32_t* out;
  int64_t osb, osg, osq;
  float denom;
};

// Radix select of the k-th largest key among keys[lo, hi) (k >= 1, k <= hi-lo)
// by one warp.  Returns the threshold key; *need = how many keys equal to the
// threshold belong to the top k (taken lowest index first).
// After each of the first three 8-bit passes the keys that share the new
// prefix (their number is the chosen digit's count) are copied into the warp's
// list cbuf (capacity ccap) when they fit, and the next pass reads only that
// list; the threshold and *need do not depend on the keys' order.
__device__ __forceinline__ uint32_t warp_radix_select(const uint32_t* keys, int lo, int hi, int k, int* hist,
                                                      uint32_t* cbuf, int ccap, int* need) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0, pmask = 0;
  const uint32_t* src = keys + lo;  // the keys a pass reads: src[0, n)
  int n = hi - lo;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    for (int j = lane; j < n; j += 32) {
      const uint32_t key = src[j];
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
    }
    __syncwarp();
    int local = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) local += hist[lane * 8 + b];
    // Suffix sums over lanes: S_l = sum_{l' >= l} local_{l'}.
    int suffix = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_down_sync(0xffffffffu, suffix, off);
      if (lane + off < 32) suffix += v;
    }
    const unsigned ge = __ballot_sync(0xffffffffu, suffix >= k);
    const int hl = 31 - __clz(ge);  // highest lane whose suffix reaches k
    int digit = 0, above = 0;
    if (lane == hl) {
      above = suffix - local;
      for (int b = 7; b >= 0; --b) {
        const int c = hist[lane * 8 + b];
        if (above + c >= k) { digit = lane * 8 + b; break; }
        above += c;
      }
    }
    digit = __shfl_sync(0xffffffffu, digit, hl);
    above = __shfl_sync(0xffffffffu, above, hl);
    const int cnt = hist[digit];  // keys sharing the new prefix
    prefix |= static_cast<uint32_t>(digit) << shift;
    pmask |= 0xFFu << shift;
    k -= above;
    __syncwarp();
    if (shift > 0 && cnt <= ccap && cnt < n) {
      // In place when src is already cbuf: a chunk's keys are all read before any
      // of them is written, and a key is written at or below its read position.
      int pos = 0;
      for (int j0 = 0; j0 < n; j0 += 32) {
        const int j = j0 + lane;
        const uint32_t key = j < n ? src[j] : 0u;
        const bool keep = j < n && (key & pmask) == prefix;
        const unsigned bm = __ballot_sync(0xffffffffu, keep);
        __syncwarp();
        if (keep) cbuf[pos + __popc(bm & ((1u << lane) - 1u))] = key;
        pos += __popc(bm);
      }
      __syncwarp();
      src = cbuf;
      n = pos;
    }
  }
  *need = k;
  return prefix;
}

// PFIX > 0: the projection width is PFIX at compile time (strides and the
// p loops fold to constants); PFIX = 0: a.P at run time.
template <int ROWS, int PFIX>
__global__ void __launch_bounds__(select_threads(ROWS), ROWS >= 16 ? 1 : 2) select_kernel(SelectArgs a) {
  constexpr int NT = select_threads(ROWS);
  extern __shared__ float sm[];
  const int P = PFIX > 0 ? PFIX : a.P;
  const int qb = a.qb;
  const int qstride = (P + 3) / 4 * 4 + 4;           // padded row stride of qs (16-byte aligned rows)
  float* qs = sm;                                   // [ROWS][qstride]
  float* kT = qs + ROWS * qstride;                  // staging: [256][kKStride] or [kPChunk][256]
  int* hist = reinterpret_cast<int*>(kT);          // [NT / 32 warps][256], once the scores are done
  uint32_t* keys = reinterpret_cast<uint32_t*>(kT + select_stage_floats(ROWS));  // [ROWS][qb]

  const int tiles = (a.q_end - a.q_begin + ROWS - 1) / ROWS;
  const int tile = tiles - 1 - blockIdx.x;          // heavy (late) rows first
  const int g = blockIdx.y, b = blockIdx.z;
  const int r0 = a.q_begin + tile * ROWS;
  const int64_t mat = (int64_t)b * a.G + g;
  const float* q = a.qp + mat * qb * P;
  const float* k = a.kp + mat * qb * P;
  for (int e = threadIdx.x; e < ROWS * qstride; e += NT) {
    const int r = e / qstride;
    const int pcol = e % qstride;
    qs[e] = (r0 + r < a.q_end && pcol < P) ? q[(int64_t)(r0 + r) * P + pcol] : 0.0f;
  }
  // Only candidates j < q - local_window of the tile's last row are needed.
  const int ncols = max(0, min(qb, r0 + ROWS - a.local_window));
  if constexpr (ROWS == 16) {
    // the host launches 16-row tiles only for P % 4 == 0 (select_rows_for)
    __syncthreads();  // qs is complete before the first multiply
    score_rows16_async(qs, qstride, k, P, ncols, kT, a.denom,
                       [&](int r, int j, float s) { keys[r * qb + j] = order_key(s); });
  } else if constexpr (ROWS == 8) {
    if (P % 4 == 0) {
      __syncthreads();  // qs is complete before the first multiply
      score_rows_async<ROWS / 4>(qs, qstride, k, P, ncols, kT, a.denom,
                                 [&](int r, int j, float s) { keys[r * qb + j] = order_key(s); });
    } else {
      for (int j0 = 0; j0 < ncols; j0 += kScoreThreads)
        score_columns<ROWS>(qs, k, P, j0, ncols, kT, a.denom,
                            [&](int r, int j, float s) { keys[r * qb + j] = order_key(s); }, qstride);
    }
  } else {
    for (int j0 = 0; j0 < ncols; j0 += kScoreThreads)
      score_columns<ROWS>(qs, k, P, j0, ncols, kT, a.denom,
                          [&](int r, int j, float s) { keys[r * qb + j] = order_key(s); }, qstride);
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the rest of the staging: one list of keys per warp for the radix select
  constexpr int ccap = (select_stage_floats(ROWS) - NT / 32 * 256) / (NT / 32);
  uint32_t* cbuf = reinterpret_cast<uint32_t*>(hist + NT / 32 * 256);
  for (int r = warp; r < ROWS; r += NT / 32) {
    const int i = r0 + r;
    if (i >= a.q_end) break;
    const uint32_t* kr = keys + r * qb;
    const int lo = a.sink;
    const int hi = min(qb, i - a.local_window);
    const int n = max(0, hi - lo);
    uint32_t thr = 0;
    int need = 0;
    const bool partial = n > a.W;  // more candidates than free slots: top-W only
    if (partial && a.W > 0)
      thr = warp_radix_select(kr, lo, hi, a.W, hist + warp * 256, cbuf + warp * ccap, ccap, &need);
    int32_t* o = a.out + b * a.osb + g * a.osg + (int64_t)i * a.osq;
    int pos = 0, ties = 0;
    for (int j0 = 0; j0 <= i; j0 += 32) {
      const int j = j0 + lane;
      bool keep = false;
      bool tie = false;
      if (j <= i) {
        const bool sink = j < a.sink && j < i - a.local_window;
        const bool local = j >= i - a.local_window;
        bool cand = false;
        if (j >= lo && j < hi) {
          if (!partial) cand = true;
          else if (a.W > 0) {
            const uint32_t key = kr[j];
            cand = key > thr;
            tie = key == thr;
          }
        }
        keep = sink || local || cand;
      }
      const unsigned tmask = __ballot_sync(0xffffffffu, tie);
      if (tie) keep = (ties + __popc(tmask & ((1u << lane) - 1u))) < need;
      ties += __popc(tmask);
      const unsigned kmask = __ballot_sync(0xffffffffu, keep);
      const int slot = pos + __popc(kmask & ((1u << lane) - 1u));
      if (keep && slot < a.K) o[slot] = j;
      pos += __popc(kmask);
    }
    for (int s = pos + lane; s < a.K; s += 32) o[s] = -1;
  }
}

// ------------------------------------------------------------------ id packing
struct PackArgs {
  const int64_t* ids;
  int64_t R;
  int qb, C, K, lw, kb, sink, words;
  int32_t* out;
};

__global__ void __launch_bounds__(256) pack_ids_kernel(PackArgs a) {
  extern __shared__ uint32_t bm_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= a.R * a.qb) return;
  uint32_t* bm = bm_all + warp * a.words;
  const int q = row % a.qb;
  for (int w = lane; w < a.words; w += 32) bm[w] = 0;
  __syncwarp();
  const int64_t* r = a.ids + row * a.C;
  for (int c = lane; c < a.C; c += 32) {
    const int64_t id = r[c];
    if (id >= 0 && id < a.kb && id <= q && id < q - a.lw && id >= a.sink)
      atomicOr(&bm[id >> 5], 1u << (id & 31));
  }
  __syncwarp();
  const int local_count = min(q + 1, a.lw + 1);
  const int sink_count = min(max(q - a.lw, 0), a.sink);
  const int remaining = a.K - local_count - sink_count;
  // Keep only the `remaining` smallest marked ids.
  int running = 0;
  for (int w0 = 0; w0 < a.words; w0 += 32) {
    const int w = w0 + lane;
    uint32_t bits = w < a.words ? bm[w] : 0u;
    const int cnt = __popc(bits);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    const int start = running + incl - cnt;
    if (start >= remaining) bits = 0u;
    else
      for (int extra = start + cnt - remaining; extra > 0; --extra) bits &= ~(1u << (31 - __clz(bits)));
    if (w < a.words) bm[w] = bits;
    running += __shfl_sync(0xffffffffu, incl, 31);
  }
  __syncwarp();
  // Forced sink ids (strictly before the local window) and the local window.
  for (int j = lane; j < a.sink; j += 32)
    if (j < q - a.lw) atomicOr(&bm[j >> 5], 1u << (j & 31));
  for (int j = max(0, q - a.lw) + lane; j <= q; j += 32) atomicOr(&bm[j >> 5], 1u << (j & 31));
  __syncwarp();
  int32_t* o = a.out + row * a.K;
  int pos = 0;
  for (int w0 = 0; w0 < a.words; w0 += 32) {
    const int w = w0 + lane;
    uint32_t bits = w < a.words ? bm[w] : 0u;
    const int cnt = __popc(bits);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int slot = pos + incl - cnt;
    while (bits) {
      const int bit = __ffs(bits) - 1;
      bits &= bits - 1u;
      if (slot < a.K) o[slot] = w * 32 + bit;
      ++slot;
    }
    pos += __shfl_sync(0xffffffffu, incl, 31);
  }
  for (int s = pos + lane; s < a.K; s += 32) o[s] = -1;
}

// ------------------------------------------------------------------ validator
__global__ void validate_init_kernel(unsigned long long* result) { *result = 0xFFFFFFFFFFFFFFFFull; }

__global__ void __launch_bounds__(256) validate_kernel(const int32_t* __restrict__ sel, int64_t rows, int qb, int K,
                                                       int lw, unsigned long long* result) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const int q = row % qb;
  const int32_t* r = sel + row * K;
  int rule = 0;
  // 1: causal (every real id <= q); real ids are the values != -1.
  for (int c = 0; c < K && !rule; ++c)
    if (r[c] != -1 && r[c] > q) rule = 1;
  // 2: sorted (non-decreasing among real ids); 3: no duplicates.
  if (!rule) {
    int prev = 0;
    bool have = false;
    for (int c = 0; c < K; ++c) {
      if (r[c] == -1) continue;
      if (have && r[c] < prev) { rule = 2; break; }
      prev = r[c];
      have = true;
    }
  }
  if (!rule) {
    int prev = 0;
    bool have = false;
    for (int c = 0; c < K; ++c) {
      if (r[c] == -1) continue;
      if (have && r[c] == prev) { rule = 3; break; }
      prev = r[c];
      have = true;
    }
  }
  // 4: local window blocks max(0, q - lw) .. q present.
  if (!rule) {
    for (int need = max(0, q - lw); need <= q && !rule; ++need) {
      bool found = false;
      for (int c = 0; c < K; ++c)
        if (r[c] == need) { found = true; break; }
      if (!found) rule = 4;
    }
  }
  // 5: padding only after all real ids.
  if (!rule) {
    bool pad = false;
    for (int c = 0; c < K; ++c) {
      if (r[c] == -1) pad = true;
      else if (pad) { rule = 5; break; }
    }
  }
  if (rule) atomicMin(result, static_cast<unsigned long long>(row) * 8ull + rule);
}

__global__ void validate_finish_kernel(unsigned long long* result) {
  if (*result == 0xFFFFFFFFFFFFFFFFull) *reinterpret_cast<long long*>(result) = -1;
}

// ------------------------------------------------------------------ launchers
// Projection with W held in shared memory.  The row-tiled project_kernel has
// every CTA read the whole W from L2 in the same d order at the same time, so
// the same few L2 lines serve every SM at once (32.6 us for 8192 rows x 128 x
// 128 at config 2, ~4 us of fma work).  Here each of ~2 CTAs per SM copies W
// into shared memory once, starting at a CTA-dependent 16-byte vector, then
// projects its share of the rows 16 at a time: thread t owns column
// p = t % P and rows t / P + i * (256 / P); x is read as broadcast float4s.
// Each output is still one fma chain over d = 0..D-1 in order (bit-identical
// to project_kernel / project_out_kernel).  Needs P | 256, P % 4 == 0,
// D % 4 == 0 and a 16-byte aligned W.
constexpr int kPwThreads = 256;
constexpr int kPwRows = 16;

template <typename T, int RPT>  // RPT = rows per thread = kPwRows * P / kPwThreads
__global__ void __launch_bounds__(kPwThreads, 2) project_w_kernel(ProjRows j0, ProjRows j1, int ctas0, int D,
                                                                   int P) {
  extern __shared__ __align__(16) float pw_smem[];
  float* Ws = pw_smem;         // [D][P]
  float* xs = Ws + D * P;      // [kPwRows][D] this pass's rows in fp32
  T* raw = reinterpret_cast<T*>(xs + kPwRows * D);  // [2][kPwRows][D] rows as loaded, two passes
  const bool second = static_cast<int>(blockIdx.x) >= ctas0;  // job fields are selected by value
  const int cta = second ? blockIdx.x - ctas0 : blockIdx.x;
  const int nct = second ? gridDim.x - ctas0 : ctas0;
  const T* x = static_cast<const T*>(second ? j1.x : j0.x);
  const float* W = second ? j1.W : j0.W;
  float* out = second ? j1.out : j0.out;
  const int qb = second ? j1.qb : j0.qb, row0 = second ? j1.row0 : j0.row0;
  const int nrows = second ? j1.nrows : j0.nrows;
  const int N = static_cast<int>((second ? j1.groups : j0.groups) * nrows);  // < 2^31 (host check)
  const int lo = static_cast<int>((int64_t)N * cta / nct), hi = static_cast<int>((int64_t)N * (cta + 1) / nct);
  if (lo >= hi) return;  // uniform per CTA
  const int nv = D * P / 4;
  const int start = static_cast<int>((int64_t)cta * 131 % nv);
  for (int e = threadIdx.x; e < nv; e += kPwThreads) {
    int v = e + start;
    if (v >= nv) v -= nv;
    cp_async16(Ws + 4 * v, W + 4 * (int64_t)v, 16);
  }
  cp_async_commit();
  constexpr int H = kPwRows / RPT;  // row lanes: thread t takes rows t / P + i * H
  constexpr int VE = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte chunk
  const int p = threadIdx.x % P, h = threadIdx.x / P;
  const int cpr = D / VE;  // chunks per row
  auto row_of = [&](int n) { return (int64_t)(n / nrows) * qb + row0 + n % nrows; };
  // The next pass's rows are fetched by cp.async while this pass multiplies
  // (rows past the CTA's share are zero-filled).
  auto fetch = [&](int n0, int buf) {
    const int rows = min(kPwRows, hi - n0);
    T* dst = raw + buf * kPwRows * D;
    for (int c = threadIdx.x; c < kPwRows * cpr; c += kPwThreads) {
      const int r = c / cpr, k = c - r * cpr;
      const bool ok = r < rows;
      const T* src = ok ? x + row_of(n0 + r) * D + k * VE : x;
      cp_async16(reinterpret_cast<float*>(dst + c * VE), reinterpret_cast<const float*>(src), ok ? 16 : 0);
    }
    cp_async_commit();
  };
  fetch(lo, 0);
  int buf = 0;
  for (int n0 = lo; n0 < hi; n0 += kPwRows, buf ^= 1) {
    const int rows = min(kPwRows, hi - n0);
    if (n0 + kPwRows < hi) {
      fetch(n0 + kPwRows, buf ^ 1);
      cp_async_wait<1>();  // W and this pass's rows have landed
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // ... for every thread, and the previous pass no longer reads xs
    for (int c = threadIdx.x; c < kPwRows * cpr; c += kPwThreads) {
      const uint4 v = *reinterpret_cast<const uint4*>(raw + buf * kPwRows * D + c * VE);
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int k = 0; k < VE; ++k) xs[c * VE + k] = Elem<T>::to_f(e[k]);
    }
    __syncthreads();
    float acc[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) acc[i] = 0.0f;
    for (int d = 0; d < D; d += 4) {
      const float w0 = Ws[d * P + p], w1 = Ws[(d + 1) * P + p], w2 = Ws[(d + 2) * P + p], w3 = Ws[(d + 3) * P + p];
      float4 xv[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i) xv[i] = *reinterpret_cast<const float4*>(xs + (h + i * H) * D + d);
#pragma unroll
      for (int i = 0; i < RPT; ++i) acc[i] = __fmaf_rn(xv[i].x, w0, acc[i]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) acc[i] = __fmaf_rn(xv[i].y, w1, acc[i]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) acc[i] = __fmaf_rn(xv[i].z, w2, acc[i]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) acc[i] = __fmaf_rn(xv[i].w, w3, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = h + i * H;
      if (r < rows) out[row_of(n0 + r) * P + p] = acc[i];
    }
  }
}

// Shared memory of project_w_kernel: W, the fp32 rows, two passes of rows as loaded.
static size_t project_w_smem(int D, int P, size_t elem) {
  return (size_t)(D * P + kPwRows * D) * sizeof(float) + 2 * (size_t)kPwRows * D * elem;
}

static bool project_w_fits(int D, int P, const float* W) {
  return P >= 16 && P <= kPwThreads && kPwThreads % P == 0 && D % 4 == 0 && (D * 2) % 16 == 0 &&
         project_w_smem(D, P, sizeof(float)) <= 96 * 1024 &&
         (reinterpret_cast<uintptr_t>(W) & 15u) == 0;
}

// project_w_kernel takes the jobs: at least 1024 rows in all (fewer, and the W
// copies would dominate), W, P and D within its limits, and 16-byte aligned
// inputs (its cp.async row copies; rows are 16-byte multiples by
// project_w_fits).  Anything else goes to the scalar-load kernels.
static bool project_w_takes(int64_t na, int64_t nb, int D, int P, const float* Wa, const float* Wb, const void* xa,
                            const void* xb) {
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return na + nb >= 1024 && na <= INT32_MAX && nb <= INT32_MAX && project_w_fits(D, P, Wa) && aligned(xa) &&
         (Wb == nullptr || (project_w_fits(D, P, Wb) && aligned(xb)));
}

template <typename T>
static cudaError_t launch_project_w(const ProjRows& a, const ProjRows& b, int njobs, int D, int P,
                                    cudaStream_t stream);

template <typename T>
cudaError_t launch_project_pair(const ProjRows& a, const ProjRows& b, int njobs, int D, int P, cudaStream_t stream) {
  const int64_t na = a.groups * a.nrows, nb = njobs > 1 ? b.groups * b.nrows : 0;
  if (project_w_takes(na, nb, D, P, a.W, njobs > 1 ? b.W : nullptr, a.x, njobs > 1 ? b.x : nullptr))
    return launch_project_w<T>(a, b, njobs, D, P, stream);
  cudaError_t e = launch_project_rows<T>(a.x, a.groups, a.qb, a.row0, a.nrows, D, a.W, P, a.out, stream);
  if (e == cudaSuccess && njobs > 1)
    e = launch_project_rows<T>(b.x, b.groups, b.qb, b.row0, b.nrows, D, b.W, P, b.out, stream);
  return e;
}

template <typename T>
static cudaError_t launch_project_w(const ProjRows& a, const ProjRows& b, int njobs, int D, int P,
                                    cudaStream_t stream) {
  const int64_t na = a.groups * a.nrows, nb = njobs > 1 ? b.groups * b.nrows : 0;
  // ~2 CTAs per SM, split between the jobs by rows, at least one each, never more than their 16-row passes
  const int64_t total = std::min<int64_t>(2 * 148, (na + nb + kPwRows - 1) / kPwRows);
  int64_t ca = na == 0 ? 0 : std::max<int64_t>(1, total * na / (na + nb));
  int64_t cb = nb == 0 ? 0 : std::max<int64_t>(1, total - ca);
  ca = std::min<int64_t>(ca, (na + kPwRows - 1) / kPwRows);
  cb = std::min<int64_t>(cb, (nb + kPwRows - 1) / kPwRows);
  if (ca + cb == 0) return cudaSuccess;
  if ((D * sizeof(T)) % 16 != 0) return cudaErrorInvalidValue;  // callers pass 16-byte rows
  const size_t smem = project_w_smem(D, P, sizeof(T));
  auto go = [&](auto kernel) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (ca == 0)
      kernel<<<(unsigned)cb, kPwThreads, smem, stream>>>(b, b, 0, D, P);
    else
      kernel<<<(unsigned)(ca + cb), kPwThreads, smem, stream>>>(a, b, (int)ca, D, P);
    return cudaGetLastError();
  };
  switch (kPwRows * P / kPwThreads) {  // rows per thread
    case 1: return go(project_w_kernel<T, 1>);
    case 2: return go(project_w_kernel<T, 2>);
    case 4: return go(project_w_kernel<T, 4>);
    case 8: return go(project_w_kernel<T, 8>);
    default: return go(project_w_kernel<T, 16>);
  }
}

template <typename T>
cudaError_t launch_project_rows(const void* x, int64_t groups, int qb, int row0, int nrows, int D, const float* W,
                                int P, float* out, cudaStream_t stream) {
  const int64_t N = groups * nrows;
  if (N == 0) return cudaSuccess;
  if (project_w_takes(N, 0, D, P, W, nullptr, x, nullptr)) {
    const ProjRows job{x, W, out, groups, qb, row0, nrows};
    return launch_project_w<T>(job, job, 1, D, P, stream);
  }
  if (N * P <= (int64_t)148 * 128 * 16) {  // fewer outputs than 16 per-output threads per SM-lane
    project_out_kernel<T><<<(unsigned)((N * P + 127) / 128), 128, 0, stream>>>(static_cast<const T*>(x), N, D, W, P,
                                                                              out, qb, row0, nrows);
    return cudaGetLastError();
  }
  if (N >= (int64_t)148 * 16 * 8) {  // many rows: 16 per CTA, so W is read from L2 a quarter as often
    const size_t smem = sizeof(float) * 16 * D;
    project_kernel<T, 16><<<(unsigned)((N + 15) / 16), 128, smem, stream>>>(static_cast<const T*>(x), N, D, W, P,
                                                                           out, qb, row0, nrows);
    return cudaGetLastError();
  }
  const size_t smem = sizeof(float) * kProjRows * D;
  project_kernel<T, kProjRows><<<(unsigned)((N + kProjRows - 1) / kProjRows), 128, smem, stream>>>(
      static_cast<const T*>(x), N, D, W, P, out, qb, row0, nrows);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_project(const void* x, int64_t N, int D, const float* W, int P, float* out,
                           cudaStream_t stream) {
  if (N > INT32_MAX) return cudaErrorInvalidValue;
  return launch_project_rows<T>(x, 1, (int)N, 0, (int)N, D, W, P, out, stream);
}

template cudaError_t launch_project_rows<float>(const void*, int64_t, int, int, int, int, const float*, int, float*,
                                                cudaStream_t);
template cudaError_t launch_project_rows<__nv_bfloat16>(const void*, int64_t, int, int, int, int, const float*, int,
                                                        float*, cudaStream_t);
template cudaError_t launch_project_rows<__half>(const void*, int64_t, int, int, int, int, const float*, int, float*,
                                                 cudaStream_t);
template cudaError_t launch_project_pair<float>(const ProjRows&, const ProjRows&, int, int, int, cudaStream_t);
template cudaError_t launch_project_pair<__nv_bfloat16>(const ProjRows&, const ProjRows&, int, int, int,
                                                        cudaStream_t);
template cudaError_t launch_project_pair<__half>(const ProjRows&, const ProjRows&, int, int, int, cudaStream_t);
template cudaError_t launch_project<float>(const void*, int64_t, int, const float*, int, float*, cudaStream_t);
template cudaError_t launch_project<__nv_bfloat16>(const void*, int64_t, int, const float*, int, float*,
                                                   cudaStream_t);
template cudaError_t launch_project<__half>(const void*, int64_t, int, const float*, int, float*, cudaStream_t);

static float gate_denom(int P) { return static_cast<float>(std::sqrt(static_cast<double>(P))); }

cudaError_t launch_scores(const float* qp, const float* kp, int64_t R, int qb, int kb, int P, float* out,
                          cudaStream_t stream) {
  constexpr int ROWS = 16;
  const size_t smem = sizeof(float) * (ROWS * ((P + 3) / 4 * 4 + 4) + kScoreThreads * kKStride);
  cudaError_t e = cudaFuncSetAttribute(scores_kernel<ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((qb + ROWS - 1) / ROWS, (unsigned)R);
  scores_kernel<ROWS><<<grid, kScoreThreads, smem, stream>>>(qp, kp, qb, kb, P, out, gate_denom(P));
  return cudaGetLastError();
}

size_t select_smem_bytes(int rows, int qb, int P) {
  const int qstride = (P + 3) / 4 * 4 + 4;
  return sizeof(float) * (rows * qstride + select_stage_floats(rows)) +
         sizeof(uint32_t) * (size_t)rows * qb;
}

template <int ROWS>
static cudaError_t launch_select_rows(const SelectArgs& a, cudaStream_t stream) {
  const size_t smem = select_smem_bytes(ROWS, a.qb, a.P);
  auto kernel = a.P == 128 ? select_kernel<ROWS, 128> : select_kernel<ROWS, 0>;  // 128: the gate width in use
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (a.q_end <= a.q_begin) return cudaSuccess;
  dim3 grid((a.q_end - a.q_begin + ROWS - 1) / ROWS, a.G, a.B);
  kernel<<<grid, select_threads(ROWS), smem, stream>>>(a);
  return cudaGetLastError();
}

// Largest tile whose keys fit in shared memory; 16-row tiles (P % 4 == 0) only when they
// still give two waves of CTAs (`tiles16` = CTAs at 16 rows, < 0 = unknown),
// else 8-row tiles, which halve the rows per CTA and double the CTAs.
int select_rows_for(int qb, int P, int64_t tiles16) {
  const size_t limit = 227 * 1024;
  if (P % 4 == 0 && select_smem_bytes(16, qb, P) <= limit && (tiles16 < 0 || tiles16 >= 2 * 148)) return 16;
  if (select_smem_bytes(8, qb, P) <= limit) return 8;
  if (select_smem_bytes(4, qb, P) <= limit) return 4;
  return 0;
}

cudaError_t launch_select(const float* qp, const float* kp, int B, int G, int qb, int P, int K, int lw, int sink,
                          int32_t* out, const int64_t* out_strides, int q_begin, int q_end, cudaStream_t stream) {
  SelectArgs a;
  a.q_begin = q_begin;
  a.q_end = q_end;
  a.qp = qp;
  a.kp = kp;
  a.B = B;
  a.G = G;
  a.qb = qb;
  a.P = P;
  a.K = K;
  a.local_window = lw;
  a.sink = std::min(sink, qb);
  a.W = std::min(K - (lw + 1) - sink, qb);
  a.out = out;
  a.osb = out_strides[0];
  a.osg = out_strides[1];
  a.osq = out_strides[2];
  a.denom = gate_denom(P);
  switch (select_rows_for(qb, P, (int64_t)((q_end - q_begin + 15) / 16) * G * B)) {
    case 16: return launch_select_rows<16>(a, stream);
    case 8: return launch_select_rows<8>(a, stream);
    case 4: return launch_select_rows<4>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pack_ids(const int64_t* ids, int64_t R, int qb, int C, int K, int lw, int kb, int sink,
                            int32_t* out, cudaStream_t stream) {
  PackArgs a;
  a.ids = ids;
  a.R = R;
  a.qb = qb;
  a.C = C;
  a.K = K;
  a.lw = lw;
  a.kb = kb;
  a.sink = std::min(sink, kb);
  a.words = (std::max(qb, kb) + 31) / 32;
  a.out = out;
  const int64_t rows = R * qb;
  if (rows == 0) return cudaSuccess;
  const size_t smem = sizeof(uint32_t) * 8 * a.words;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(pack_ids_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  pack_ids_kernel<<<(unsigned)((rows + 7) / 8), 256, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_validate(const int32_t* sel, int64_t rows, int qb, int K, int lw, int64_t* result,
                            cudaStream_t stream) {
  auto* res = reinterpret_cast<unsigned long long*>(result);
  validate_init_kernel<<<1, 1, 0, stream>>>(res);
  if (rows > 0) validate_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(sel, rows, qb, K, lw, res);
  validate_finish_kernel<<<1, 1, 0, stream>>>(res);
  return cudaGetLastError();
}

}  // namespace spruce

// ------------------------------------------------------------------ MaxSim scores
namespace spruce {

// MaxSim gate scores (selector/gate.py:29-101, :104-117, :132-171):
//   s[r, q, c] = max over (i, j) of qp[r, q, i, :] . kp[r, key(c), j, :] / denom
// with key(c) = c (every key column) or ids[r, q, c] clamped to [0, nk) (the
// candidate nodes of a tree level).  Every dot is one fma chain over p in
// order, the max is exact in any order.  One CTA per (r, q): the row's P
// query prototypes and a batch of G = 128 / (P*P) candidates' key prototypes
// are staged in shared memory (rows padded by one float against bank
// conflicts); thread t computes the dot (i, j) = ((t % P^2) / P, t % P) of
// candidate t / P^2, and the first G threads take the max over each
// candidate's P^2 dots.
constexpr int kMaxsimThreads = 128;

__global__ void __launch_bounds__(kMaxsimThreads) maxsim_kernel(const float* __restrict__ qp,
                                                               const float* __restrict__ kp,
                                                               const int64_t* __restrict__ ids, int nq, int nk,
                                                               int ncols, int P, int pdim, float denom,
                                                               float* __restrict__ out) {
  extern __shared__ float msm[];
  const int stride = pdim + 1;
  const int PP = P * P;
  const int G = kMaxsimThreads / PP;
  float* qs = msm;                      // [P][stride]
  float* ks = qs + P * stride;          // [G][P][stride]
  float* dots = ks + G * P * stride;    // [kMaxsimThreads]
  const int64_t rq = blockIdx.x;        // r * nq + q
  const int64_t r = rq / nq;
  for (int e = threadIdx.x; e < P * pdim; e += kMaxsimThreads) qs[(e / pdim) * stride + e % pdim] = qp[rq * P * pdim + e];
  const int slot = threadIdx.x / PP, i = (threadIdx.x % PP) / P, j = threadIdx.x % P;
  for (int c0 = 0; c0 < ncols; c0 += G) {
    __syncthreads();  // qs ready / previous batch's ks and dots consumed
    const int nb = min(G, ncols - c0);
    for (int e = threadIdx.x; e < nb * P * pdim; e += kMaxsimThreads) {
      const int g = e / (P * pdim), rest = e % (P * pdim);
      int64_t key = c0 + g;
      if (ids != nullptr) {
        key = ids[rq * ncols + c0 + g];
        key = key < 0 ? 0 : (key >= nk ? nk - 1 : key);
      }
      ks[(g * P + rest / pdim) * stride + rest % pdim] = __ldg(kp + (r * nk + key) * P * pdim + rest);
    }
    __syncthreads();
    float acc = -INFINITY;
    if (slot < nb) {
      const float* qi = qs + i * stride;
      const float* kj = ks + (slot * P + j) * stride;
      acc = 0.0f;
      for (int x = 0; x < pdim; ++x) acc = __fmaf_rn(qi[x], kj[x], acc);
    }
    if (PP == 64) {  // P = 8: a candidate's dots fill two whole warps
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc = fmaxf(acc, __shfl_xor_sync(0xffffffffu, acc, off));
      if ((threadIdx.x & 31) == 0) dots[threadIdx.x >> 5] = acc;
      __syncthreads();
      if (threadIdx.x < nb)
        out[rq * ncols + c0 + threadIdx.x] = __fdiv_rn(fmaxf(dots[2 * threadIdx.x], dots[2 * threadIdx.x + 1]), denom);
    } else {
      dots[threadIdx.x] = acc;
      __syncthreads();
      if (threadIdx.x < nb) {
        float best = -INFINITY;
        for (int e = 0; e < PP; ++e) best = fmaxf(best, dots[threadIdx.x * PP + e]);
        out[rq * ncols + c0 + threadIdx.x] = __fdiv_rn(best, denom);
      }
    }
  }
}

// MaxSim with one candidate per lane: a one-warp CTA per (r, q) row scores
// 32 candidates at a time, each lane holding all P*P dot products of its
// candidate in registers.  Query prototypes are read as broadcasts, the
// candidates' prototypes are staged by cp.async in chunks of kMsChunk
// elements of p into two alternating buffers (candidate rows padded to
// P*kMsChunk + 4 floats, so a quarter-warp's float4 reads hit distinct
// banks).  Each dot is the same in-order fma chain over p as maxsim_kernel.
constexpr int kMsChunk = 16;

template <int P>
__global__ void __launch_bounds__(32) maxsim_lane_kernel(const float* __restrict__ qp, const float* __restrict__ kp,
                                                         const int64_t* __restrict__ ids, int nq, int nk, int ncols,
                                                         int pdim, float denom, float* __restrict__ out) {
  constexpr int KS = P * kMsChunk + 4;     // floats per staged candidate
  constexpr int QV = P * kMsChunk / 4;     // float4 copies of one query chunk
  constexpr int KV = 32 * P * kMsChunk / 4;  // float4 copies of one candidate chunk
  constexpr int STAGE = 32 * KS + P * kMsChunk;
  extern __shared__ __align__(16) float lsm[];
  const int lane = threadIdx.x;
  // consecutive CTAs take different r, so the few nodes of a narrow tree level
  // are not all read by every resident CTA at once
  const int64_t R = gridDim.x / nq;
  const int64_t r = blockIdx.x % R;
  const int64_t rq = r * nq + blockIdx.x / R;
  const float* qrow = qp + rq * P * pdim;
  const int nch = pdim / kMsChunk;
  for (int c0 = 0; c0 < ncols; c0 += 32) {
    const int nb = min(32, ncols - c0);
    int64_t mykey = c0 + lane;
    if (ids != nullptr && lane < nb) mykey = ids[rq * ncols + c0 + lane];
    mykey = mykey < 0 ? 0 : (mykey >= nk ? nk - 1 : mykey);
    const float* krow = kp + (r * nk + mykey) * P * pdim;
    auto stage = [&](int ch) {
      float* buf = lsm + (ch & 1) * STAGE;
      float* qs = buf + 32 * KS;
      const int x0 = ch * kMsChunk;
      for (int e = lane; e < QV; e += 32) {
        const int i = e / (kMsChunk / 4), v = e % (kMsChunk / 4);
        cp_async16(qs + i * kMsChunk + 4 * v, qrow + (int64_t)i * pdim + x0 + 4 * v, 16);
      }
#pragma unroll 4
      for (int e = lane; e < KV; e += 32) {
        const int c = e / (P * kMsChunk / 4), rest = e % (P * kMsChunk / 4);
        const int j = rest / (kMsChunk / 4), v = rest % (kMsChunk / 4);
        const float* src = reinterpret_cast<const float*>(
            __shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(krow), c));
        if (c < nb) cp_async16(buf + c * KS + j * kMsChunk + 4 * v, src + (int64_t)j * pdim + x0 + 4 * v, 16);
      }
      cp_async_commit();
    };
    float acc[P][P];
#pragma unroll
    for (int i = 0; i < P; ++i)
#pragma unroll
      for (int j = 0; j < P; ++j) acc[i][j] = 0.0f;
    stage(0);
    for (int ch = 0; ch < nch; ++ch) {
      if (ch + 1 < nch) {
        stage(ch + 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();
      const float* buf = lsm + (ch & 1) * STAGE;
      const float* qs = buf + 32 * KS;
      const float* ks = buf + lane * KS;
#pragma unroll
      for (int v = 0; v < kMsChunk / 4; ++v) {
        float4 qv[P];
#pragma unroll
        for (int i = 0; i < P; ++i) qv[i] = *reinterpret_cast<const float4*>(qs + i * kMsChunk + 4 * v);
#pragma unroll
        for (int j = 0; j < P; ++j) {
          const float4 kv = *reinterpret_cast<const float4*>(ks + j * kMsChunk + 4 * v);
#pragma unroll
          for (int i = 0; i < P; ++i) {
            float a = acc[i][j];
            a = __fmaf_rn(qv[i].x, kv.x, a);
            a = __fmaf_rn(qv[i].y, kv.y, a);
            a = __fmaf_rn(qv[i].z, kv.z, a);
            acc[i][j] = __fmaf_rn(qv[i].w, kv.w, a);
          }
        }
      }
      __syncwarp();  // this buffer is restaged two chunks on
    }
    float best = -INFINITY;
#pragma unroll
    for (int i = 0; i < P; ++i)
#pragma unroll
      for (int j = 0; j < P; ++j) best = fmaxf(best, acc[i][j]);
    if (lane < nb) out[rq * ncols + c0 + lane] = __fdiv_rn(best, denom);
  }
}

// MaxSim for a level of at most 32 nodes (the top of the key tree), where
// every query row's candidates come from the same few nodes: a persistent
// CTA stages all nk nodes' prototypes of one r in shared memory once (node
// rows padded to P*p + 4 floats for conflict-free float4 reads) and its warps
// score whole rows, lane = (row slot, node), nkpad = next power of two >= nk
// nodes per row slot.  A row's candidate scores are then shuffled out of the
// lanes that hold the candidates' nodes.  Same in-order fma chain per dot.
template <int P>
__global__ void __launch_bounds__(256) maxsim_nodes_kernel(const float* __restrict__ qp, const float* __restrict__ kp,
                                                           const int64_t* __restrict__ ids, int nq, int nk, int nkpad,
                                                           int ncols, int pdim, float denom, float* __restrict__ out) {
  extern __shared__ __align__(16) float nsm[];
  const int NS = P * pdim + 4;
  const int64_t r = blockIdx.y;
  const float* kr = kp + r * nk * P * pdim;
  for (int e = threadIdx.x; e < nk * P * pdim / 4; e += blockDim.x) {
    const int n = e / (P * pdim / 4), rest = e % (P * pdim / 4);
    cp_async16(nsm + n * NS + 4 * rest, kr + 4 * (int64_t)e, 16);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int rpw = 32 / nkpad, sub = lane / nkpad, n = lane % nkpad;
  const int groups = (nq + rpw - 1) / rpw;
  const float* ks = nsm + min(n, nk - 1) * NS;  // only nk node rows are staged; lanes n >= nk are never read out
  for (int g = blockIdx.x * nwarps + warp; g < groups; g += gridDim.x * nwarps) {  // uniform per warp
    const int q = g * rpw + sub;
    const bool live = q < nq;
    const int64_t rq = r * nq + (live ? q : nq - 1);
    const float* qrow = qp + rq * P * pdim;
    float acc[P][P];
#pragma unroll
    for (int i = 0; i < P; ++i)
#pragma unroll
      for (int j = 0; j < P; ++j) acc[i][j] = 0.0f;
#pragma unroll 2
    for (int v = 0; v < pdim / 4; ++v) {
      float4 qv[P];
#pragma unroll
      for (int i = 0; i < P; ++i) qv[i] = __ldg(reinterpret_cast<const float4*>(qrow + i * pdim) + v);
#pragma unroll
      for (int j = 0; j < P; ++j) {
        const float4 kv = *reinterpret_cast<const float4*>(ks + j * pdim + 4 * v);
#pragma unroll
        for (int i = 0; i < P; ++i) {
          float a = acc[i][j];
          a = __fmaf_rn(qv[i].x, kv.x, a);
          a = __fmaf_rn(qv[i].y, kv.y, a);
          a = __fmaf_rn(qv[i].z, kv.z, a);
          acc[i][j] = __fmaf_rn(qv[i].w, kv.w, a);
        }
      }
    }
    float best = -INFINITY;
#pragma unroll
    for (int i = 0; i < P; ++i)
#pragma unroll
      for (int j = 0; j < P; ++j) best = fmaxf(best, acc[i][j]);
    const float score = __fdiv_rn(best, denom);
    if (ids == nullptr) {
      if (live && n < nk) out[rq * ncols + n] = score;
      continue;
    }
    for (int cb = 0; cb < ncols; cb += nkpad) {  // same trip count in every lane
      const int c = cb + n;
      const bool w = live && c < ncols;
      int64_t key = w ? ids[rq * ncols + c] : 0;
      key = key < 0 ? 0 : (key >= nk ? nk - 1 : key);
      const float s = __shfl_sync(0xffffffffu, score, sub * nkpad + (int)key);
      if (w) out[rq * ncols + c] = s;
    }
  }
}

template <int P>
cudaError_t launch_maxsim_nodes(const float* qp, const float* kp, const int64_t* ids, int64_t R, int nq, int nk,
                                int ncols, int pdim, float denom, float* out, cudaStream_t stream) {
  int nkpad = 1;
  while (nkpad < nk) nkpad <<= 1;
  const size_t smem = sizeof(float) * (size_t)nk * (P * pdim + 4);
  cudaError_t e = cudaFuncSetAttribute(maxsim_nodes_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  const int rows_per_warp = 32 / nkpad;
  const int64_t groups = (nq + rows_per_warp - 1) / rows_per_warp;
  const int64_t per_r = std::max<int64_t>(1, std::min<int64_t>((148 + R - 1) / R, (groups + 7) / 8));
  maxsim_nodes_kernel<P><<<dim3((unsigned)per_r, (unsigned)R), 256, smem, stream>>>(qp, kp, ids, nq, nk, nkpad,
                                                                                    ncols, pdim, denom, out);
  return cudaGetLastError();
}

template <int P>
cudaError_t launch_maxsim_lane(const float* qp, const float* kp, const int64_t* ids, int64_t R, int nq, int nk,
                               int ncols, int pdim, float denom, float* out, cudaStream_t stream) {
  const size_t smem = sizeof(float) * 2 * (32 * (P * kMsChunk + 4) + P * kMsChunk);
  maxsim_lane_kernel<P><<<(unsigned)(R * nq), 32, smem, stream>>>(qp, kp, ids, nq, nk, ncols, pdim, denom, out);
  return cudaGetLastError();
}

cudaError_t launch_maxsim(const float* qp, const float* kp, const int64_t* ids, int64_t R, int nq, int nk, int ncols,
                          int P, int pdim, float* out, cudaStream_t stream) {
  if (R * nq == 0 || ncols == 0) return cudaSuccess;
  if (P < 1 || P > 8) return cudaErrorInvalidValue;
  const float denom = static_cast<float>(std::sqrt(static_cast<double>(pdim)));
  const bool lane_ok = pdim % kMsChunk == 0 && pdim > 0 &&
                       ((reinterpret_cast<uintptr_t>(qp) | reinterpret_cast<uintptr_t>(kp)) & 15) == 0;
  const size_t nodes_smem = sizeof(float) * (size_t)nk * (P * pdim + 4);
  if (lane_ok && P >= 4 && nk <= 32 && nodes_smem <= 227 * 1024 && R <= 65535) {
    switch (P) {
      case 4: return launch_maxsim_nodes<4>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      case 5: return launch_maxsim_nodes<5>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      case 6: return launch_maxsim_nodes<6>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      case 7: return launch_maxsim_nodes<7>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      default: return launch_maxsim_nodes<8>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
    }
  }
  if (lane_ok && P >= 4) {
    switch (P) {
      case 4: return launch_maxsim_lane<4>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      case 5: return launch_maxsim_lane<5>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      case 6: return launch_maxsim_lane<6>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      case 7: return launch_maxsim_lane<7>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
      default: return launch_maxsim_lane<8>(qp, kp, ids, R, nq, nk, ncols, pdim, denom, out, stream);
    }
  }
  const int G = kMaxsimThreads / (P * P);
  const size_t smem = sizeof(float) * ((size_t)(1 + G) * P * (pdim + 1) + kMaxsimThreads);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(maxsim_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  maxsim_kernel<<<(unsigned)(R * nq), kMaxsimThreads, smem, stream>>>(qp, kp, ids, nq, nk, ncols, P, pdim, denom,
                                                                      out);
  return cudaGetLastError();
}

}  // namespace spruce
