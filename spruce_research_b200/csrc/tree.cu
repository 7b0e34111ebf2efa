// Key-axis tree of the deployed selector: level construction and the
// per-level steps of the beam traversal.
//
// Reference: selector/tree.py:80-145 (build_key_tree, _merge_level_prototypes)
// and scripts/eval_tree_traversal.py:60-113 (traverse_to_leaf_ids).
//
// Parent node p of a level groups children [p*radix, p*radix + radix) of the
// level below (an odd tail is a smaller parent).  Its prototypes are:
//   0:      the mean of the valid children's prototype 0, formed in the
//           features' dtype as the reference does (sum over children in fp32,
//           rounded; divided by the child count, rounded);
//   1..P-1: the children's prototypes farthest from that mean, where each
//           distance is computed in the features' dtype too (difference
//           rounded, square rounded, fp32 sum over d in order, rounded),
//           descending, ties to the lower candidate (torch.topk leaves tie
//           order open).
// Traversal level step, per (layer*group, query row): candidates are the
// children of the row's current selection (selected*radix + offset); a
// candidate is valid when its parent is, it exists, and it starts at or
// before the row's block; scores are MaxSim (select.cu), invalid ones
// replaced by the fp32 minimum; the best min(beam, C, children) candidates in
// descending score (ties to the lower position) are kept, invalid ones as -1.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace spruce {

namespace {

constexpr int kMergeThreads = 128;
constexpr int kMaxCand = 32 * 8;  // radix * P candidates of one parent

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) tree_merge_kernel(const T* __restrict__ child, int nchild,
                                                                    T* __restrict__ parent, int nparent, int P,
                                                                    int d, int radix) {
  extern __shared__ float msm[];
  float* mean = msm;            // [d]
  float* dist = msm + d;        // [radix * P]
  __shared__ int pick[8];
  const int64_t r = blockIdx.y;
  const int pn = blockIdx.x;
  const int c0 = pn * radix;
  const int nvalid = min(radix, nchild - c0);
  const T* base = child + ((int64_t)r * nchild + c0) * P * d;
  T* out = parent + ((int64_t)r * nparent + pn) * P * d;
  const float cnt = round_through<T>((float)nvalid);
  for (int x = threadIdx.x; x < d; x += kMergeThreads) {
    float s = 0.0f;
    for (int c = 0; c < nvalid; ++c) s = __fadd_rn(s, Elem<T>::to_f(base[(int64_t)c * P * d + x]));
    const T m = Elem<T>::from_f(__fdiv_rn(round_through<T>(s), cnt));
    out[x] = m;
    mean[x] = Elem<T>::to_f(m);
  }
  if (P == 1) return;  // uniform per CTA
  __syncthreads();
  const int ncand = radix * P;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < ncand; c += kMergeThreads) {  // one candidate per thread, d in order
    float acc = 0.0f;
    if (c / P < nvalid) {
      const T* row = base + (int64_t)c * d;
      for (int x = 0; x < d; ++x) {
        const float diff = round_through<T>(__fsub_rn(Elem<T>::to_f(row[x]), mean[x]));
        acc = __fadd_rn(acc, round_through<T>(__fmul_rn(diff, diff)));
      }
    }
    dist[c] = c / P < nvalid ? round_through<T>(acc) : -INFINITY;
  }
  __syncthreads();
  if (warp == 0) {
    // P-1 picks among ncand <= 256 candidates: each lane scans its strided share.
    for (int s = 0; s < P - 1; ++s) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int c = lane; c < ncand; c += 32)
        if (dist[c] > best || (dist[c] == best && c < bi)) {
          best = dist[c];
          bi = c;
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
      if (lane == 0) {
        const bool found = bi < ncand;        // false only when every distance left is NaN
        pick[s] = found ? bi : -1;            // -1: the mean
        if (found) dist[bi] = -INFINITY * 0.0f;  // NaN: compares false, never picked again
      }
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < (P - 1) * d; e += kMergeThreads) {
    const int s = e / d, x = e % d;
    out[(int64_t)(s + 1) * d + x] = pick[s] >= 0 ? base[(int64_t)pick[s] * d + x] : Elem<T>::from_f(mean[x]);
  }
}

// Candidates of one traversal level: cand[r, q, s*radix + o] = sel[r, q, s]*radix + o.
__global__ void tree_candidates_kernel(const int64_t* __restrict__ sel, int S, int nq, int radix, int nchild,
                                       const int64_t* __restrict__ child_starts, int64_t* __restrict__ cand,
                                       uint8_t* __restrict__ valid, int64_t total) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= total) return;
  const int C = S * radix;
  const int64_t rq = e / C;
  const int c = (int)(e % C);
  const int q = (int)(rq % nq);
  const int64_t parent = sel[rq * S + c / radix];
  const int64_t id = parent * radix + c % radix;
  bool ok = parent >= 0 && id < nchild;
  const int64_t safe = id < 0 ? 0 : (id >= nchild ? nchild - 1 : id);
  ok = ok && child_starts[safe] <= q;
  cand[e] = ok ? id : safe;  // the reference scores clamped ids; validity decides
  valid[e] = ok ? 1 : 0;
}

// Best k of each row's C <= 256 candidates by score, invalid ones scored as the
// fp32 minimum; ties to the lower position.  One warp per row.
__global__ void tree_topk_kernel(const float* __restrict__ scores, const uint8_t* __restrict__ valid,
                                 const int64_t* __restrict__ cand, int C, int k, int64_t rows,
                                 int64_t* __restrict__ out) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* s = scores + row * C;
  const uint8_t* v = valid + row * C;
  uint32_t taken[kMaxCand / 32] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int t = 0; t < k; ++t) {
    float best = 0.0f;
    int bi = 0x7fffffff;
    bool have = false;
    for (int c = lane; c < C; c += 32) {
      if (taken[c / 32] & (1u << (c % 32))) continue;
      const float x = v[c] ? s[c] : -3.402823466e38f;
      if (!have || x > best || (x == best && c < bi)) {
        best = x;
        bi = c;
        have = true;
      }
    }
    if (!have) best = -INFINITY;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (bi < C) {
      if (bi % 32 == lane) taken[bi / 32] |= 1u << (bi % 32);  // each lane owns candidates c = lane (mod 32)
      if (lane == 0) out[row * k + t] = v[bi] ? cand[row * C + bi] : -1;
    } else if (lane == 0) {
      out[row * k + t] = -1;
    }
  }
}

// The same selection for rows of at most 32 candidates (every level of a beam-16,
// radix-2 traversal): each lane holds one candidate as a 64-bit key -- the
// order-preserving image of its score (-0 folded into +0) above 31 - position --
// and the warp sorts the keys descending with a bitonic network.  Keys are
// distinct, and their order is the float order of the scores with ties to the
// lower position, so the first k lanes hold exactly what tree_topk_kernel picks
// (for scores that are not NaN).
__device__ __forceinline__ uint32_t float_order_key(float f) {
  const uint32_t u = __float_as_uint(f + 0.0f);  // -0 -> +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void tree_topk32_kernel(const float* __restrict__ scores, const uint8_t* __restrict__ valid,
                                   const int64_t* __restrict__ cand, int C, int k, int64_t rows,
                                   int64_t* __restrict__ out) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // warp-uniform
  uint64_t key = 0;         // below every real candidate
  if (lane < C) {
    const float x = valid[row * C + lane] ? scores[row * C + lane] : -3.402823466e38f;
    key = ((uint64_t)float_order_key(x) << 32) | (uint32_t)(31 - lane);
  }
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
    const bool desc = (lane & size) == 0;  // the last merge (size 32) is descending for every lane
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, key, stride);
      const bool keep_max = ((lane & stride) == 0) == desc;
      key = keep_max ? (key > other ? key : other) : (key < other ? key : other);
    }
  }
  if (lane < k) {
    const int pos = 31 - (int)(key & 0xffffffffu);
    out[row * k + lane] = valid[row * C + pos] ? cand[row * C + pos] : -1;
  }
}

}  // namespace

template <typename T>
cudaError_t launch_tree_merge(const void* child, int64_t R, int nchild, void* parent, int P, int d, int radix,
                              cudaStream_t stream) {
  const int nparent = (nchild + radix - 1) / radix;
  if (R == 0 || nparent == 0) return cudaSuccess;
  if (P > 8 || radix * P > kMaxCand) return cudaErrorInvalidValue;
  const size_t smem = sizeof(float) * ((size_t)d + (size_t)radix * P);
  dim3 grid((unsigned)nparent, (unsigned)R);
  tree_merge_kernel<T><<<grid, kMergeThreads, smem, stream>>>(static_cast<const T*>(child), nchild,
                                                               static_cast<T*>(parent), nparent, P, d, radix);
  return cudaGetLastError();
}

template cudaError_t launch_tree_merge<float>(const void*, int64_t, int, void*, int, int, int, cudaStream_t);
template cudaError_t launch_tree_merge<__nv_bfloat16>(const void*, int64_t, int, void*, int, int, int, cudaStream_t);
template cudaError_t launch_tree_merge<__half>(const void*, int64_t, int, void*, int, int, int, cudaStream_t);

cudaError_t launch_tree_candidates(const int64_t* sel, int64_t R, int nq, int S, int radix, int nchild,
                                   const int64_t* child_starts, int64_t* cand, uint8_t* valid, cudaStream_t stream) {
  const int64_t total = R * nq * S * radix;
  if (total == 0) return cudaSuccess;
  tree_candidates_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(sel, S, nq, radix, nchild,
                                                                             child_starts, cand, valid, total);
  return cudaGetLastError();
}

cudaError_t launch_tree_topk(const float* scores, const uint8_t* valid, const int64_t* cand, int64_t rows, int C,
                             int k, int64_t* out, cudaStream_t stream) {
  if (rows == 0 || k == 0) return cudaSuccess;
  if (C > kMaxCand || k > C) return cudaErrorInvalidValue;
  if (C <= 32) {
    tree_topk32_kernel<<<(unsigned)((rows + 3) / 4), 128, 0, stream>>>(scores, valid, cand, C, k, rows, out);
    return cudaGetLastError();
  }
  tree_topk_kernel<<<(unsigned)((rows + 3) / 4), 128, 0, stream>>>(scores, valid, cand, C, k, rows, out);
  return cudaGetLastError();
}

}  // namespace spruce
