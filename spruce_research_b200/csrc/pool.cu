// Block-summary pooling of queries and keys (selector inputs).
//
// Reference: teacher/chunked_extract.py:27-80 (_proto_pool_seq with P = 1,
// _group_avg_tokens).  The rounding points are the reference's, so results
// are bit-identical to its CPU torch path:
//   group average  g[t] = rnd( (x_h0 + x_h1 + ... ) / rep )      fp32, heads in order
//   block mean     m    = rnd( rnd(S) / count ),  S = ((c0 + c1) + c2) + c3
//                  where c_k is the in-order fp32 sum of rows 16k..16k+15
// (torch's CPU sum over the 64-row axis accumulates 16-row chunks).
//
// Layout / roofline: one CTA per (batch, head-or-group, 64-token block) reads
// the block's rows once with 16-byte vector loads (coalesced along D) and
// writes one pooled row.  The kernel is HBM-bound: at config 2 it reads Q
// (0.94 GB) and K (0.13 GB) once and writes 8.4 MB.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace spruce {

constexpr int kPoolThreads = 256;
constexpr int kPoolBlock = 64;

// 16-byte vector of T.
template <typename T> struct Vec16 { static constexpr int N = 16 / sizeof(T); };

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float (&v)[Vec16<T>::N]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int k = 0; k < Vec16<T>::N; ++k) v[k] = Elem<T>::to_f(e[k]);
}

// grid: (nb, Hout, B) for each of up to two jobs stacked along y (job = y / Hout0).
template <typename T>
__global__ void __launch_bounds__(kPoolThreads) pool_block_kernel(PoolJob j0, PoolJob j1, int njobs, int T_len,
                                                                   int D, int nb) {
  constexpr int VN = Vec16<T>::N;
  extern __shared__ float pool_smem[];
  float* rows = pool_smem;                 // [64][D] group-averaged, already rounded to T
  float* part = pool_smem + kPoolBlock * D; // [4][D] 16-row partial sums
  float* meanv = part + 4 * D;              // [D] the mean prototype (rounded to T), protos > 1
  float* dist = meanv + D;                  // [64] squared distances to the mean, protos > 1

  int y = blockIdx.y;
  const PoolJob& job = (njobs > 1 && y >= j0.hout) ? j1 : j0;
  if (njobs > 1 && y >= j0.hout) y -= j0.hout;
  if (static_cast<int>(blockIdx.x) >= job.nblk) return;
  const int i = job.blk0 + blockIdx.x;
  const int b = blockIdx.z;
  const int t0 = i * kPoolBlock;
  const int count = min(kPoolBlock, T_len - t0);
  const int nvec = D / VN;
  const T* x = static_cast<const T*>(job.x);
  const float frep = static_cast<float>(job.rep);

  // Phase 1: per-token group average (rep = 1 copies the row), rounded to T.
  for (int task = threadIdx.x; task < kPoolBlock * nvec; task += kPoolThreads) {
    const int r = task / nvec;
    const int v = task % nvec;
    float acc[VN];
#pragma unroll
    for (int k = 0; k < VN; ++k) acc[k] = 0.0f;
    if (r < count) {
      const T* base = x + b * job.sb + (int64_t)(y * job.rep) * job.sh + (int64_t)(t0 + r) * job.st + v * VN;
      for (int h = 0; h < job.rep; ++h) {
        float e[VN];
        load_vec<T>(base + (int64_t)h * job.sh, e);
#pragma unroll
        for (int k = 0; k < VN; ++k) acc[k] = __fadd_rn(acc[k], e[k]);
      }
#pragma unroll
      for (int k = 0; k < VN; ++k) acc[k] = round_through<T>(__fdiv_rn(acc[k], frep));
    }
#pragma unroll
    for (int k = 0; k < VN; ++k) rows[r * D + v * VN + k] = acc[k];
  }
  __syncthreads();

  // Phase 2: in-order fp32 sums of each 16-row chunk.
  for (int task = threadIdx.x; task < 4 * D; task += kPoolThreads) {
    const int c = task / D;
    const int d = task % D;
    float s = 0.0f;
#pragma unroll
    for (int r = 0; r < 16; ++r) s = __fadd_rn(s, rows[(c * 16 + r) * D + d]);
    part[c * D + d] = s;
  }
  __syncthreads();

  // Phase 3: chunk totals in order, round, divide by the real row count, round.
  const int P = job.protos;
  T* out = static_cast<T*>(job.out) + ((int64_t)(b * job.hout + y) * nb + i) * P * D;
  for (int d = threadIdx.x; d < D; d += kPoolThreads) {
    float total = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) total = __fadd_rn(total, part[c * D + d]);
    const float s = round_through<T>(total);
    const T m = Elem<T>::from_f(__fdiv_rn(s, static_cast<float>(count)));
    out[d] = m;
    meanv[d] = Elem<T>::to_f(m);
  }
  if (P == 1) return;  // uniform per CTA
  __syncthreads();

  // Phase 4 (teacher/chunked_extract.py:53-54): squared L2 distance of each real
  // row to the mean, in fp32, one warp per row; pad rows of a ragged tail are -inf.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < kPoolBlock; r += kPoolThreads / 32) {
    float acc = 0.0f;
    for (int d = lane; d < D; d += 32) {
      const float diff = __fsub_rn(rows[r * D + d], meanv[d]);
      acc = __fadd_rn(acc, __fmul_rn(diff, diff));  // squares rounded, as pow(2) then sum
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) dist[r] = r < count ? acc : -INFINITY;
  }
  __syncthreads();

  // Phase 5 (:55-57): the P-1 largest distances in descending order (ties to the
  // lower row), by one warp: each of the 64 rows is held by lane r % 32.
  __shared__ int pick[kPoolBlock];
  if (warp == 0) {
    float d0 = dist[lane], d1 = dist[lane + 32];
    for (int s = 0; s < P - 1 && s < kPoolBlock; ++s) {
      float best = d0;
      int bi = lane;
      if (d1 > best) {
        best = d1;
        bi = lane + 32;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
      }
      if (lane == 0) pick[s] = (best == -INFINITY) ? -1 : bi;  // only pad rows left: the mean (:62-67)
      // a picked row drops out like a pad row (real distances are >= 0)
      if (bi == lane) d0 = -INFINITY;
      if (bi == lane + 32) d1 = -INFINITY;
    }
  }
  __syncthreads();

  // Phase 6 (:68-72): prototypes 1.. are the picked rows (exact copies), or the
  // mean where the block has no further real row.
  for (int e = threadIdx.x; e < (P - 1) * D; e += kPoolThreads) {
    const int s = e / D, d = e % D;
    const int r = s < kPoolBlock ? pick[s] : -1;
    out[(int64_t)(s + 1) * D + d] = Elem<T>::from_f(r >= 0 ? rows[r * D + d] : meanv[d]);
  }
}

// Plain per-token group average (no pooling): out [B, G, T, D] contiguous.
template <typename T>
__global__ void __launch_bounds__(256) group_avg_kernel(const T* x, int64_t sb, int64_t sh, int64_t st, T* out,
                                                        int B, int G, int rep, int T_len, int D) {
  constexpr int VN = Vec16<T>::N;
  const int nvec = D / VN;
  const int64_t total = (int64_t)B * G * T_len * nvec;
  const float frep = static_cast<float>(rep);
  for (int64_t task = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; task < total;
       task += (int64_t)gridDim.x * blockDim.x) {
    const int v = task % nvec;
    const int64_t rest = task / nvec;
    const int t = rest % T_len;
    const int g = (rest / T_len) % G;
    const int b = rest / ((int64_t)T_len * G);
    const T* base = x + b * sb + (int64_t)(g * rep) * sh + (int64_t)t * st + v * VN;
    float acc[VN];
#pragma unroll
    for (int k = 0; k < VN; ++k) acc[k] = 0.0f;
    for (int h = 0; h < rep; ++h) {
      float e[VN];
      load_vec<T>(base + (int64_t)h * sh, e);
#pragma unroll
      for (int k = 0; k < VN; ++k) acc[k] = __fadd_rn(acc[k], e[k]);
    }
    T res[VN];
#pragma unroll
    for (int k = 0; k < VN; ++k) res[k] = Elem<T>::from_f(__fdiv_rn(acc[k], frep));
    *reinterpret_cast<uint4*>(out + (((int64_t)b * G + g) * T_len + t) * D + v * VN) =
        *reinterpret_cast<const uint4*>(res);
  }
}

template <typename T>
cudaError_t launch_pool(PoolJob j0, PoolJob j1, int njobs, int B, int T_len, int D, cudaStream_t stream) {
  const int nb = (T_len + kPoolBlock - 1) / kPoolBlock;
  const size_t smem = sizeof(float) * (kPoolBlock * D + 4 * D + D + kPoolBlock);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(pool_block_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int gx = njobs > 1 ? std::max(j0.nblk, j1.nblk) : j0.nblk;
  if (gx <= 0) return cudaSuccess;
  dim3 grid(gx, j0.hout + (njobs > 1 ? j1.hout : 0), B);
  pool_block_kernel<T><<<grid, kPoolThreads, smem, stream>>>(j0, j1, njobs, T_len, D, nb);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_group_avg(const void* x, const int64_t* s, void* out, int B, int H, int T_len, int D, int G,
                             cudaStream_t stream) {
  const int64_t total = (int64_t)B * G * T_len * (D / Vec16<T>::N);
  int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  if (grid < 1) grid = 1;
  group_avg_kernel<T><<<grid, 256, 0, stream>>>(static_cast<const T*>(x), s[0], s[1], s[2], static_cast<T*>(out),
                                                B, G, H / G, T_len, D);
  return cudaGetLastError();
}

template cudaError_t launch_pool<float>(PoolJob, PoolJob, int, int, int, int, cudaStream_t);
template cudaError_t launch_pool<__nv_bfloat16>(PoolJob, PoolJob, int, int, int, int, cudaStream_t);
template cudaError_t launch_pool<__half>(PoolJob, PoolJob, int, int, int, int, cudaStream_t);
template cudaError_t launch_group_avg<float>(const void*, const int64_t*, void*, int, int, int, int, int,
                                             cudaStream_t);
template cudaError_t launch_group_avg<__nv_bfloat16>(const void*, const int64_t*, void*, int, int, int, int, int,
                                                     cudaStream_t);
template cudaError_t launch_group_avg<__half>(const void*, const int64_t*, void*, int, int, int, int, int,
                                              cudaStream_t);

}  // namespace spruce
