// K/V summary table of the residual tree (build_kv_summary_table).
//
// Reference: sparse/summaries.py:52-142 with the prototype ranges of
// _prototype_token_ranges (:29-49).  For every tree node n (a block range
// [start, end) of ResidualTreeLayout) and prototype p < P the reference takes
//   range   [s, e) = ts + len*p/P .. ts + len*(p+1)/P,  ts/te = block*bs clamped to T
//   pooled  = F[e] - F[s]                       (fp32)
//   mean    = pooled / max(count, 1)            (fp32)
// where F is the fp32 prefix of the valid-masked rows.  Torch's CPU cumsum
// accumulates that prefix in double and rounds each element to float, so
// F[t] = float(sum_{u<t} w_u) with the sum exact whenever it is exact in
// double -- always for bf16/fp16 rows, whose 8/11-bit significands leave
// more than 30 bits of headroom at any realistic length.  The kernels below
// build the same double prefix in a different (parallel) order, which gives
// the same exact sum, and round it only at the range ends: the table is
// bit-identical to the reference's CPU result under that condition.
//
// Three launches, all HBM-bound:
//   1. segments: one thread per (tensor, b, h, 16-token sub-segment, 16-byte
//      vector of D) sums its rows in double, 16 loads in flight; sub-sums of
//      a segment (64/P tokens for 64-token blocks, else 16) are merged in
//      shared memory -> prefix[.., j+1, d]; valid counts per (b, segment)
//      alongside.  Reads K and V once.
//   2. scan: one CTA per (tensor*b*h, 8-column slice) turns the segment sums
//      into an inclusive prefix in place (128 rows of ~nseg/128 segments,
//      then a cross-row offset).  Reads/writes the double workspace.
//   3. nodes: one CTA per (node, b, h), threads along D, reads the prefix at
//      the P + 1 range edges (plus at most 15 rows when an edge is not a
//      multiple of 16 -- only ragged tails or small block sizes) and writes
//      the fp32 means, counts, log counts and ranges.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace spruce {

constexpr int kSumSeg = 16;       // smallest prefix segment (tokens); the workspace is sized for it
constexpr int kSumThreads = 256;  // segment and node kernels
constexpr int kScanLanes = 8;     // columns per scan CTA
constexpr int kScanRows = 128;    // rows of segments per scan CTA
constexpr int kScanBatch = 8;     // segments loaded together per scan step
constexpr int kNodeThreads = 128; // node kernel: threads along D
constexpr int kMaxProto = 4;      // prototypes are 1, 2 or 4

int64_t kv_summary_segments(int64_t T) { return (T + kSumSeg - 1) / kSumSeg; }

// Range edges are ts + len*p/P with ts and len multiples of the block size
// (except at a ragged tail), so with 64-token blocks every edge falls on a
// multiple of 64/P and a segment that long needs no partial rows.
// The segment kernel merges r = seg/16 sub-segments inside one CTA, so a longer
// segment also needs 256 threads to hold whole groups of r * vecs_per_row.
int kv_summary_segment_tokens(int64_t block_size, int P, int64_t vecs_per_row) {
  const int seg = block_size % 64 == 0 ? 64 / P : kSumSeg;
  return kSumThreads % ((seg / kSumSeg) * vecs_per_row) == 0 ? seg : kSumSeg;
}

int64_t kv_summary_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t D) {
  const int64_t nseg = kv_summary_segments(T);
  const int64_t prefix = 2 * B * H * (nseg + 1) * D * (int64_t)sizeof(double);
  const int64_t counts = B * (nseg + 1) * (int64_t)sizeof(int64_t);
  return prefix + ((counts + 255) / 256) * 256;
}

namespace {

template <typename T, int VEC>
__device__ __forceinline__ void load_row(const T* p, float (&v)[VEC]) {
  if constexpr (VEC == 1) {
    v[0] = Elem<T>::to_f(p[0]);
  } else {
    static_assert(VEC * sizeof(T) == 16, "vector loads are 16 bytes");
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = Elem<T>::to_f(e[k]);
  }
}

// w_t = x_t * valid_t as the reference forms it (an invalid row is x * 0, which
// keeps a NaN/inf row poisoning the prefix exactly as torch does).
__device__ __forceinline__ float masked(float x, bool ok) { return ok ? x : x * 0.0f; }

// One thread per (tensor, b*h, 16-token sub-segment, vector of D) loads its
// 16 rows together.  When a segment spans r = seg/16 sub-segments the CTA
// holds whole segments (the host only picks seg > 16 when 256 is a multiple of
// r * D/VEC) and the first thread of each group adds the r partial sums from
// shared memory.
template <typename T, int VEC>
__global__ void __launch_bounds__(kSumThreads) summary_segments_kernel(KvSummaryArgs a, int nseg) {
  __shared__ double part[kSumThreads * VEC];
  __shared__ int part_cnt[kSumThreads];
  const int DV = a.D / VEC;
  const int r = a.seg / kSumSeg;
  const int nsub = (a.T + kSumSeg - 1) / kSumSeg;
  const int idx = blockIdx.x * kSumThreads + threadIdx.x;
  const int dv = idx % DV;
  const int js = idx / DV;
  const int which = blockIdx.y & 1;
  const int bh = blockIdx.y >> 1;
  const int b = bh / a.H, h = bh % a.H;
  const int64_t* s = which ? a.vs : a.ks;
  const T* src = static_cast<const T*>(which ? a.value : a.key) + b * s[0] + h * s[1] + (int64_t)dv * VEC;
  const uint8_t* valid = a.valid ? a.valid + (int64_t)b * a.T : nullptr;

  double acc[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) acc[k] = 0.0;
  int cnt = 0;
  if (js < nsub) {
    const int t0 = js * kSumSeg;
    if (t0 + kSumSeg <= a.T) {  // full sub-segment: all 16 loads in flight together
      float v[kSumSeg][VEC];
#pragma unroll
      for (int u = 0; u < kSumSeg; ++u) load_row<T, VEC>(src + (int64_t)(t0 + u) * s[2], v[u]);
#pragma unroll
      for (int u = 0; u < kSumSeg; ++u) {
        const bool ok = valid == nullptr || valid[t0 + u] != 0;
        cnt += ok;
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] += (double)masked(v[u][k], ok);
      }
    } else {
      for (int t = t0; t < a.T; ++t) {
        float v[VEC];
        load_row<T, VEC>(src + (int64_t)t * s[2], v);
        const bool ok = valid == nullptr || valid[t] != 0;
        cnt += ok;
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] += (double)masked(v[k], ok);
      }
    }
  }
  if (r > 1) {  // uniform: r is a kernel argument
#pragma unroll
    for (int k = 0; k < VEC; ++k) part[threadIdx.x * VEC + k] = acc[k];
    part_cnt[threadIdx.x] = cnt;
    __syncthreads();
    if (js % r != 0) return;
    for (int q = 1; q < r; ++q) {
#pragma unroll
      for (int k = 0; k < VEC; ++k) acc[k] += part[(threadIdx.x + q * DV) * VEC + k];
      cnt += part_cnt[threadIdx.x + q * DV];
    }
  }
  const int j = js / r;
  if (j >= nseg) return;
  double* col = a.prefix + (int64_t)(which * a.B * a.H + bh) * (nseg + 1) * a.D + (int64_t)dv * VEC;
#pragma unroll
  for (int k = 0; k < VEC; ++k) col[(int64_t)(j + 1) * a.D + k] = acc[k];
  if (j == 0) {
#pragma unroll
    for (int k = 0; k < VEC; ++k) col[k] = 0.0;
  }
  if (which == 0 && h == 0 && dv == 0) {
    int64_t* c = a.cprefix + (int64_t)b * (nseg + 1);
    c[j + 1] = cnt;
    if (j == 0) c[0] = 0;
  }
}

// grid (ceil(D / 8), 2*B*H + B), block (8, 128).  y < 2*B*H scans a column
// slice of one (tensor, b, h); the last B rows of the grid scan the counts.
__global__ void __launch_bounds__(kScanLanes * kScanRows) summary_scan_kernel(double* prefix, int64_t* cprefix,
                                                                               int rows_bh, int D, int nseg) {
  __shared__ double tot[kScanRows][kScanLanes];
  const int lane = threadIdx.x, row = threadIdx.y;
  const int per = (nseg + kScanRows - 1) / kScanRows;
  const int j0 = 1 + row * per, j1 = min(j0 + per, nseg + 1);
  const bool counts = (int)blockIdx.y >= rows_bh;
  if (counts && blockIdx.x != 0) return;  // uniform per CTA
  const int d = counts ? lane : (int)blockIdx.x * kScanLanes + lane;
  const bool live = counts ? lane == 0 : d < D;
  double* col = counts ? nullptr : prefix + (int64_t)blockIdx.y * (nseg + 1) * D + d;
  int64_t* ccol = counts ? cprefix + (int64_t)(blockIdx.y - rows_bh) * (nseg + 1) : nullptr;

  double s = 0.0;
  if (live) {
    if (counts) {
      int64_t c = 0;
      for (int j = j0; j < j1; ++j) c += ccol[j];
      s = (double)c;
    } else {
      int j = j0;
      for (; j + kScanBatch <= j1; j += kScanBatch) {
        double v[kScanBatch];
#pragma unroll
        for (int u = 0; u < kScanBatch; ++u) v[u] = col[(int64_t)(j + u) * D];
#pragma unroll
        for (int u = 0; u < kScanBatch; ++u) s += v[u];
      }
      for (; j < j1; ++j) s += col[(int64_t)j * D];
    }
  }
  tot[row][lane] = s;
  __syncthreads();
  if (row == 0) {
    double run = 0.0;
    for (int r = 0; r < kScanRows; ++r) {
      const double v = tot[r][lane];
      tot[r][lane] = run;
      run += v;
    }
  }
  __syncthreads();
  if (!live) return;
  if (counts) {
    int64_t run = (int64_t)tot[row][lane];  // integer counts: exact in double
    for (int j = j0; j < j1; ++j) {
      run += ccol[j];
      ccol[j] = run;
    }
  } else {
    double run = tot[row][lane];
    int j = j0;
    for (; j + kScanBatch <= j1; j += kScanBatch) {
      double v[kScanBatch];
#pragma unroll
      for (int u = 0; u < kScanBatch; ++u) v[u] = col[(int64_t)(j + u) * D];
#pragma unroll
      for (int u = 0; u < kScanBatch; ++u) {
        run += v[u];
        col[(int64_t)(j + u) * D] = run;
      }
    }
    for (; j < j1; ++j) {
      run += col[(int64_t)j * D];
      col[(int64_t)j * D] = run;
    }
  }
}

__device__ __forceinline__ int64_t clamp_tokens(int64_t block, int64_t bs, int64_t T) {
  if (block <= 0) return 0;
  if (block >= T) return T;  // block * bs >= block >= T
  return min(block * bs, T);
}

// grid (nodes, B), block 128 over D: every prototype range of one node for
// one batch item and all its heads.  Threads 0..P first resolve the P + 1
// range edges and their valid counts into shared memory (independent loads,
// one round trip); then each column issues the 2 * (P + 1) prefix loads of a
// head together (consecutive prototypes share an edge).
template <typename T>
__global__ void __launch_bounds__(kNodeThreads) summary_nodes_kernel(KvSummaryArgs a, int nseg) {
  __shared__ int64_t s_edge[kMaxProto + 1];
  __shared__ int64_t s_count[kMaxProto + 1];
  __shared__ float s_denom[kMaxProto];
  const int64_t n = blockIdx.x;
  const int b = blockIdx.y;
  const int P = a.P;
  const uint8_t* valid = a.valid ? a.valid + (int64_t)b * a.T : nullptr;
  if (threadIdx.x <= P) {
    const int p = threadIdx.x;
    const int64_t ts = clamp_tokens(a.node_starts[n], a.block_size, a.T);
    const int64_t len = max(clamp_tokens(a.node_ends[n], a.block_size, a.T), ts) - ts;
    const int64_t e = ts + len * p / P;
    const int64_t j = e / a.seg;
    int64_t c = a.cprefix[(int64_t)b * (nseg + 1) + j];
    for (int64_t u = j * a.seg; u < e; ++u) c += valid == nullptr || valid[u] != 0;
    s_edge[p] = e;
    s_count[p] = c;
  }
  __syncthreads();
  if (threadIdx.x < P) {
    const int p = threadIdx.x;
    const float count = (float)(s_count[p + 1] - s_count[p]);
    s_denom[p] = fmaxf(count, 1.0f);
    const int64_t c = ((int64_t)b * a.nodes + n) * P + p;
    a.out_counts[c] = count;
    a.out_log_counts[c] = count > 0.0f ? (float)log((double)count) : -INFINITY;
    if (b == 0 && a.range_starts != nullptr) {
      a.range_starts[n * P + p] = s_edge[p];
      a.range_ends[n * P + p] = s_edge[p + 1];
    }
  }
  __syncthreads();

  int64_t edge_seg[kMaxProto + 1];
#pragma unroll
  for (int p = 0; p <= kMaxProto; ++p) edge_seg[p] = p <= P ? s_edge[p] / a.seg : 0;
  for (int h = 0; h < a.H; ++h) {
    const int bh = b * a.H + h;
    for (int d = threadIdx.x; d < a.D; d += kNodeThreads) {
      double v[2][kMaxProto + 1];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const double* col = a.prefix + (int64_t)(which * a.B * a.H + bh) * (nseg + 1) * a.D + d;
#pragma unroll
        for (int p = 0; p <= kMaxProto; ++p)
          if (p <= P) v[which][p] = col[edge_seg[p] * a.D];
      }
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const int64_t* s = which ? a.vs : a.ks;
        const T* src = static_cast<const T*>(which ? a.value : a.key) + b * s[0] + h * s[1] + d;
        float* out = (which ? a.out_values : a.out_keys) + ((int64_t)bh * a.nodes + n) * P * a.D + d;
        float f_prev = 0.0f;
#pragma unroll
        for (int p = 0; p <= kMaxProto; ++p) {
          if (p > P) break;
          const int64_t e = s_edge[p];
          for (int64_t u = edge_seg[p] * a.seg; u < e; ++u)  // only at edges inside a segment
            v[which][p] += (double)masked(Elem<T>::to_f(src[u * s[2]]), valid == nullptr || valid[u] != 0);
          const float f = (float)v[which][p];
          if (p > 0) out[(int64_t)(p - 1) * a.D] = __fdiv_rn(__fsub_rn(f, f_prev), s_denom[p - 1]);
          f_prev = f;
        }
      }
    }
  }
}

template <typename T, int VEC>
cudaError_t launch_summary_typed(const KvSummaryArgs& a, cudaStream_t stream) {
  const int nseg = (int)((a.T + a.seg - 1) / a.seg);
  const int64_t seg_threads = kv_summary_segments(a.T) * (a.D / VEC);
  dim3 g1((unsigned)((seg_threads + kSumThreads - 1) / kSumThreads), (unsigned)(2 * a.B * a.H));
  summary_segments_kernel<T, VEC><<<g1, kSumThreads, 0, stream>>>(a, nseg);
  dim3 g2((unsigned)((a.D + kScanLanes - 1) / kScanLanes), (unsigned)(2 * a.B * a.H + a.B));
  summary_scan_kernel<<<g2, dim3(kScanLanes, kScanRows), 0, stream>>>(a.prefix, a.cprefix, 2 * a.B * a.H, a.D,
                                                                      nseg);
  summary_nodes_kernel<T><<<dim3((unsigned)a.nodes, (unsigned)a.B), kNodeThreads, 0, stream>>>(a, nseg);
  return cudaGetLastError();
}

}  // namespace

template <typename T>
cudaError_t launch_kv_summary(const KvSummaryArgs& a, bool vec, cudaStream_t stream) {
  if (vec) return launch_summary_typed<T, (int)(16 / sizeof(T))>(a, stream);
  return launch_summary_typed<T, 1>(a, stream);
}

template cudaError_t launch_kv_summary<float>(const KvSummaryArgs&, bool, cudaStream_t);
template cudaError_t launch_kv_summary<__nv_bfloat16>(const KvSummaryArgs&, bool, cudaStream_t);
template cudaError_t launch_kv_summary<__half>(const KvSummaryArgs&, bool, cudaStream_t);

}  // namespace spruce
