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
// Layout / roofline: every input row is read once with 16-byte vector loads
// (coalesced along D) and each 64-token block writes one pooled row (P = 1).
// At config 2 that is Q (0.94 GB) and K (0.13 GB) read once and 8.4 MB written:
// an HBM-bound job.  P = 1 runs pool_rows_kernel (one thread per 16-row chunk
// and 16-byte vector, loads staged by cp.async, sums in registers); prototypes
// (P > 1) need every row of the block at once and run pool_block_kernel (rows
// staged in shared memory).
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

// ---------------------------------------------------------------------------
// P = 1 pooling with one thread per (16-row chunk, 16-byte vector) of a block.
//
// A thread sums the group averages of its chunk's rows in registers straight
// from the loads; only the four chunk partials of a block pass through shared
// memory.  The rounding points are pool_block_kernel's (and the reference's):
// the group average rounded to T per element, in-order 16-row chunk sums with
// pad rows adding +0, chunk totals in order, round, divide by the row count.
// Two exact shortcuts drop instructions the kernel was bound by:
//   rep = 1:   x / 1 = x, and x is already a T value (no division, no rounding);
//   rep = 2^k: x / rep = x * 2^-k (both are the correctly rounded image of the
//              same real number).
// Measured before: the per-element division and the 32 KB rows round trip kept
// pool_block_kernel at ~52% issue-active and 3.7 TB/s.

constexpr int kRowsThreads = 256;

// In-order sum over the chunk's 16 rows (rows >= nrows are pad rows and add +0),
// each row's group average formed from register loads of its rep heads.  Used
// for group sizes without a staged instantiation (chunk_sum_staged below).
template <typename T>
__device__ __forceinline__ void chunk_sum(const T* p, int64_t sh, int64_t st, int nrows, int rep,
                                          float (&s)[Vec16<T>::N]) {
  constexpr int VN = Vec16<T>::N;
  const float frep = static_cast<float>(rep);
  for (int r = 0; r < 16; ++r) {
    float g[VN];
#pragma unroll
    for (int k = 0; k < VN; ++k) g[k] = 0.0f;
    if (r < nrows) {
      for (int h = 0; h < rep; ++h) {
        float e[VN];
        load_vec<T>(p + r * st + h * sh, e);
#pragma unroll
        for (int k = 0; k < VN; ++k) g[k] = __fadd_rn(g[k], e[k]);
      }
#pragma unroll
      for (int k = 0; k < VN; ++k) g[k] = round_through<T>(__fdiv_rn(g[k], frep));
    }
#pragma unroll
    for (int k = 0; k < VN; ++k) s[k] = __fadd_rn(s[k], g[k]);
  }
}

// The same in-order chunk sum with the rows' loads staged in shared memory by
// cp.async: the data in flight costs no registers, so a thread keeps
// kStageVecs / REP rows (14-16 16-byte vectors) in flight where the register
// form held one row.  stage[v * stride] is the thread's vector v.  A row's
// slot is refilled only after its values were added (the adds use the data, so
// the slot's shared loads have completed).
constexpr int kStageVecs = 16;

__device__ __forceinline__ void pool_cp16(uint4* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void pool_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pool_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename T, int REP>
__device__ __forceinline__ void chunk_sum_staged(const T* p, int64_t sh, int64_t st, int nrows, uint4* stage,
                                                 int stride, float (&s)[Vec16<T>::N]) {
  constexpr int VN = Vec16<T>::N;
  constexpr int S = kStageVecs / REP;  // rows in flight
  static_assert(S >= 1, "a row must fit in the stage");
  auto issue = [&](int r) {  // one commit group per row, empty past the real rows
    if (r < nrows) {
#pragma unroll
      for (int h = 0; h < REP; ++h) pool_cp16(stage + ((r % S) * REP + h) * stride, p + r * st + h * sh);
    }
    pool_cp_commit();
  };
#pragma unroll
  for (int r = 0; r < S; ++r) issue(r);
#pragma unroll 1
  for (int r = 0; r < 16; ++r) {
    pool_cp_wait<S - 1>();  // row r has landed
    float g[VN];
    if (r < nrows) {
      float acc[VN];
#pragma unroll
      for (int k = 0; k < VN; ++k) acc[k] = 0.0f;
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        const uint4 raw = stage[((r % S) * REP + h) * stride];
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int k = 0; k < VN; ++k) acc[k] = __fadd_rn(acc[k], Elem<T>::to_f(e[k]));
      }
      if constexpr (REP == 1) {
#pragma unroll
        for (int k = 0; k < VN; ++k) g[k] = acc[k];  // 0 + x: the reference's -0 -> +0 is kept
      } else if constexpr ((REP & (REP - 1)) == 0) {
#pragma unroll
        for (int k = 0; k < VN; ++k) g[k] = round_through<T>(__fmul_rn(acc[k], 1.0f / REP));
      } else {
#pragma unroll
        for (int k = 0; k < VN; ++k) g[k] = round_through<T>(__fdiv_rn(acc[k], static_cast<float>(REP)));
      }
    } else {
#pragma unroll
      for (int k = 0; k < VN; ++k) g[k] = 0.0f;
    }
#pragma unroll
    for (int k = 0; k < VN; ++k) s[k] = __fadd_rn(s[k], g[k]);
    issue(r + S);
  }
  pool_cp_wait<0>();
}

// items = (batch, block, slot) with the slots of one block adjacent (slot s <
// j0.hout is job 0's head s, the rest job 1's); each CTA takes `ipc` items of
// 4 * (D / VN) threads.
template <typename T>
__global__ void __launch_bounds__(kRowsThreads, 3) pool_rows_kernel(PoolJob j0, PoolJob j1, int njobs, int T_len,
                                                                  int D, int nb, int nbmax, int slots, int64_t items,
                                                                  int ipc) {
  constexpr int VN = Vec16<T>::N;
  __shared__ __align__(16) float part[kRowsThreads * VN];
  extern __shared__ __align__(16) uint4 pool_stage[];  // [kStageVecs][blockDim.x]
  const int nvec = D / VN;
  const int per_item = 4 * nvec;
  const int t = threadIdx.x;
  const int it = t / per_item;
  const int w = t - it * per_item;
  const int c = w / nvec;
  const int v = w - c * nvec;
  const int64_t item = (int64_t)blockIdx.x * ipc + it;

  bool active = item < items;
  int y = 0, b = 0, i = 0, count = 0;
  bool second = false;  // the item belongs to job 1 (fields are selected by value: no local copy of the jobs)
  float s[VN];
#pragma unroll
  for (int k = 0; k < VN; ++k) s[k] = 0.0f;
  if (active) {
    const int slot = static_cast<int>(item % slots);
    const int64_t rest = item / slots;
    const int il = static_cast<int>(rest % nbmax);
    b = static_cast<int>(rest / nbmax);
    second = njobs > 1 && slot >= j0.hout;
    y = second ? slot - j0.hout : slot;
    active = il < (second ? j1.nblk : j0.nblk);
    if (active) {
      i = (second ? j1.blk0 : j0.blk0) + il;
      const int t0 = i * kPoolBlock;
      count = min(kPoolBlock, T_len - t0);
      const int rep = second ? j1.rep : j0.rep;
      const int64_t sh = second ? j1.sh : j0.sh, st = second ? j1.st : j0.st;
      const int nrows = max(0, min(16, count - 16 * c));
      const T* p = static_cast<const T*>(second ? j1.x : j0.x) + b * (second ? j1.sb : j0.sb) +
                   (int64_t)(y * rep) * sh + (int64_t)(t0 + 16 * c) * st + v * VN;
      uint4* stage = pool_stage + t;
      const int stride = blockDim.x;
      switch (rep) {
        case 1: chunk_sum_staged<T, 1>(p, sh, st, nrows, stage, stride, s); break;
        case 2: chunk_sum_staged<T, 2>(p, sh, st, nrows, stage, stride, s); break;
        case 4: chunk_sum_staged<T, 4>(p, sh, st, nrows, stage, stride, s); break;
        case 7: chunk_sum_staged<T, 7>(p, sh, st, nrows, stage, stride, s); break;
        case 8: chunk_sum_staged<T, 8>(p, sh, st, nrows, stage, stride, s); break;
        default: chunk_sum<T>(p, sh, st, nrows, rep, s); break;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VN; ++k) part[t * VN + k] = s[k];
  __syncthreads();
  if (!active || c != 0) return;
  // chunk totals in order, round, divide by the real row count
  T res[VN];
#pragma unroll
  for (int k = 0; k < VN; ++k) {
    float total = 0.0f;
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) total = __fadd_rn(total, part[(t + cc * nvec) * VN + k]);
    res[k] = Elem<T>::from_f(__fdiv_rn(round_through<T>(total), static_cast<float>(count)));
  }
  T* out = static_cast<T*>(second ? j1.out : j0.out) + ((int64_t)(b * (second ? j1.hout : j0.hout) + y) * nb + i) * D +
           v * VN;
  *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(res);
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
  const int slots = j0.hout + (njobs > 1 ? j1.hout : 0);
  const int per_item = 4 * (D / Vec16<T>::N);
  if (j0.protos == 1 && (njobs == 1 || j1.protos == 1) && per_item <= kRowsThreads) {
    const int ipc = kRowsThreads / per_item;
    const int64_t items = (int64_t)B * gx * slots;
    const int64_t ctas = (items + ipc - 1) / ipc;
    if (ctas > INT32_MAX) return cudaErrorInvalidValue;
    const size_t stage = sizeof(uint4) * kStageVecs * ipc * per_item;
    cudaError_t e = cudaFuncSetAttribute(pool_rows_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)stage);
    if (e != cudaSuccess) return e;
    pool_rows_kernel<T><<<(unsigned)ctas, ipc * per_item, stage, stream>>>(j0, j1, njobs, T_len, D, nb, gx,
                                                                            slots, items, ipc);
    return cudaGetLastError();
  }
  dim3 grid(gx, slots, B);
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
