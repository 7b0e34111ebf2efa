// Residual-summary gather: the summary keys each query row attends to besides
// its selected blocks, laid out as "virtual blocks" for the attention kernels.
//
// Reference: sparse/attention.py:224-263.  For row (b, g, i) the residual node
// ids residual_summary_nodes[b, layer, g, i, :] (>= 0) are taken in order, each
// with its P prototypes; a prototype joins the softmax when its token count is
// positive, with key and value from the summary table and the additive bias
// log_counts[b, node, p].  Here those prototypes become consecutive rows of
// the virtual K/V ([B, Hkv, qb * nvb * 64, D], row i's rows starting at
// i * nvb * 64) in the compute dtype, with the bias beside them; the rows up
// to the next multiple of 64 are zero with bias -inf, so a partial virtual
// block adds exactly nothing.  vcount[b, g, i] is the row's number of virtual
// blocks.
//
// One CTA per row: warp 0 compacts the valid (node slot, prototype) pairs in
// order into shared memory; then all 128 threads copy rows along D.
#include <algorithm>

#include "attn_common.cuh"

namespace spruce {

namespace {

constexpr int kGatherThreads = 128;

template <typename T> struct Store4;
template <> struct Store4<float> {
  static __device__ __forceinline__ void put(float* dst, float4 v) { *reinterpret_cast<float4*>(dst) = v; }
};
template <> struct Store4<__nv_bfloat16> {
  static __device__ __forceinline__ void put(__nv_bfloat16* dst, float4 v) {
    uint2 u;
    u.x = Pack2<__nv_bfloat16>::pack(v.x, v.y);
    u.y = Pack2<__nv_bfloat16>::pack(v.z, v.w);
    *reinterpret_cast<uint2*>(dst) = u;
  }
};
template <> struct Store4<__half> {
  static __device__ __forceinline__ void put(__half* dst, float4 v) {
    uint2 u;
    u.x = Pack2<__half>::pack(v.x, v.y);
    u.y = Pack2<__half>::pack(v.z, v.w);
    *reinterpret_cast<uint2*>(dst) = u;
  }
};

template <typename T, int D>
__global__ void __launch_bounds__(kGatherThreads) residual_gather_kernel(const ResidualGatherArgs a) {
  extern __shared__ int picks[];  // (slot * P + prototype) of the row's valid prototypes, in order
  __shared__ int npick;
  const int i = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t* row = a.nodes + b * a.ns[0] + g * a.ns[1] + (int64_t)i * a.ns[2];
  const int total = a.S * a.P;
  if (warp == 0) {
    int count = 0;
    for (int base = 0; base < total; base += 32) {
      const int e = base + lane;
      bool keep = false;
      if (e < total) {
        const int node = row[(e / a.P) * a.ns[3]];
        keep = node >= 0 && node < a.NN && a.counts[((int64_t)b * a.NN + node) * a.P + e % a.P] > 0.0f;
      }
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (keep) picks[count + __popc(m & ((1u << lane) - 1u))] = e;
      count += __popc(m);
    }
    if (lane == 0) npick = count;
  }
  __syncthreads();
  // picks -> table row offsets (in units of D), in place
  const int n = min(npick, a.nvb * 64);
  const int64_t bg = (int64_t)b * a.Hkv + g;
  for (int r = threadIdx.x; r < n; r += kGatherThreads) {
    const int pick = picks[r];
    picks[r] = row[(pick / a.P) * a.ns[3]] * a.P + pick % a.P;  // node * P + prototype
  }
  __syncthreads();
  const int npad = (n + 63) / 64 * 64;
  const int64_t Tv = (int64_t)a.qb * a.nvb * 64;
  const int64_t vrow0 = bg * Tv + (int64_t)i * a.nvb * 64;
  T* vk = static_cast<T*>(a.vk) + vrow0 * D;
  T* vv = static_cast<T*>(a.vv) + vrow0 * D;
  const float* keys = a.keys + bg * a.NN * a.P * D;
  const float* values = a.values + bg * a.NN * a.P * D;
  constexpr int V4 = D / 4;  // float4 chunks per row
  for (int e = threadIdx.x; e < npad * V4; e += kGatherThreads) {
    const int r = e / V4, c = e % V4;  // V4 is a power of two: shifts
    float4 kx = make_float4(0.0f, 0.0f, 0.0f, 0.0f), vx = kx;
    if (r < n) {
      const int64_t src = (int64_t)picks[r] * D + 4 * c;
      kx = __ldg(reinterpret_cast<const float4*>(keys + src));
      vx = __ldg(reinterpret_cast<const float4*>(values + src));
    }
    Store4<T>::put(vk + (int64_t)r * D + 4 * c, kx);
    Store4<T>::put(vv + (int64_t)r * D + 4 * c, vx);
  }
  for (int r = threadIdx.x; r < npad; r += kGatherThreads)
    a.vbias[vrow0 + r] = r < n ? a.log_counts[(int64_t)b * a.NN * a.P + picks[r]] : -INFINITY;
  if (threadIdx.x == 0) a.vcount[bg * a.qb + i] = npad / 64;
}

// Maximal frontier of one selected_blocks row (interfaces/residual_summaries.py:122-155):
// node n is taken when its block range lies inside the causal prefix [0, q] and
// holds no selected block, and its parent's range does not (the reference's
// depth-first visit stops exactly there: a parent that fails the test has an
// ancestor chain that fails it too, since ranges only grow upwards).  Nodes are
// scanned in ID order, so the row comes out ID-sorted like the reference's.
// sel [rows, K] contiguous; a row's query block is row % qb.
constexpr int kFrontierThreads = 256;

__global__ void __launch_bounds__(kFrontierThreads)
    residual_frontier_kernel(const int32_t* __restrict__ sel, int K, int qb, const int64_t* __restrict__ starts,
                             const int64_t* __restrict__ ends, const int32_t* __restrict__ parents, int NN,
                             int32_t* __restrict__ out, int S, int32_t* __restrict__ row_counts,
                             int32_t* __restrict__ max_count) {
  extern __shared__ int pre[];  // [qb + 1]: number of selected blocks below x
  __shared__ int wsum[kFrontierThreads / 32];
  const int64_t r = blockIdx.x;
  const int q = (int)(r % qb);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int x = tid; x <= qb; x += kFrontierThreads) pre[x] = 0;
  __syncthreads();
  for (int c = tid; c < K; c += kFrontierThreads) {
    const int id = sel[r * K + c];
    if (id >= 0 && id < qb) pre[id + 1] = 1;  // duplicates mark once
  }
  __syncthreads();
  // inclusive scan of pre[1..qb]: each thread one contiguous chunk, then a block scan of the chunk sums
  const int per = (qb + kFrontierThreads - 1) / kFrontierThreads;
  const int lo = 1 + tid * per, hi = min(qb + 1, lo + per);
  int run = 0;
  for (int x = lo; x < hi; ++x) run += pre[x];
  int incl = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += wsum[w];
  int acc = base + incl - run;  // exclusive prefix of this thread's chunk
  for (int x = lo; x < hi; ++x) {
    acc += pre[x];
    pre[x] = acc;
  }
  __syncthreads();
  const int limit = q + 1;
  auto empty_causal = [&](int n) {
    const int s = (int)starts[n], e = (int)ends[n];
    return e <= limit && pre[e] - pre[s] == 0;
  };
  int total = 0;
  for (int n0 = 0; n0 < NN; n0 += kFrontierThreads) {  // uniform trip count
    const int n = n0 + tid;
    bool take = false;
    if (n < NN && empty_causal(n)) {
      const int par = parents[n];
      take = par < 0 || !empty_causal(par);
    }
    const unsigned m = __ballot_sync(0xffffffffu, take);
    __syncthreads();  // wsum reuse
    if (lane == 0) wsum[warp] = __popc(m);
    __syncthreads();
    int before = total;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    if (take && out != nullptr) {
      const int pos = before + __popc(m & ((1u << lane) - 1u));
      if (pos < S) out[r * S + pos] = n;
    }
    for (int w = 0; w < kFrontierThreads / 32; ++w) total += wsum[w];
  }
  if (out != nullptr)
    for (int pos = total + tid; pos < S; pos += kFrontierThreads) out[r * S + pos] = -1;
  if (tid == 0) {
    if (row_counts != nullptr) row_counts[r] = total;
    if (max_count != nullptr) atomicMax(max_count, total);
  }
}

}  // namespace

cudaError_t launch_residual_frontier(const int32_t* sel, int64_t rows, int K, int qb, const int64_t* starts,
                                     const int64_t* ends, const int32_t* parents, int NN, int32_t* out, int S,
                                     int32_t* row_counts, int32_t* max_count, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const size_t smem = sizeof(int) * ((size_t)qb + 1);
  if (smem > 200 * 1024 || rows > 0x7fffffff) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(residual_frontier_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  residual_frontier_kernel<<<(unsigned)rows, kFrontierThreads, smem, stream>>>(sel, K, qb, starts, ends, parents, NN,
                                                                              out, S, row_counts, max_count);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t gather_typed(const ResidualGatherArgs& a, size_t smem, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(residual_gather_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)a.qb, (unsigned)a.Hkv, (unsigned)a.B);
  residual_gather_kernel<T, D><<<grid, kGatherThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t gather_d(const ResidualGatherArgs& a, size_t smem, cudaStream_t stream) {
  if (a.D == 128) return gather_typed<T, 128>(a, smem, stream);
  if (a.D == 64) return gather_typed<T, 64>(a, smem, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_residual_gather(const ResidualGatherArgs& a, int dtype, cudaStream_t stream) {
  if (a.B == 0 || a.Hkv == 0 || a.qb == 0) return cudaSuccess;
  const size_t smem = sizeof(int) * (size_t)std::max(1, a.S * a.P);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  switch (dtype) {
    case SPRUCE_DTYPE_F32: return gather_d<float>(a, smem, stream);
    case SPRUCE_DTYPE_BF16: return gather_d<__nv_bfloat16>(a, smem, stream);
    case SPRUCE_DTYPE_F16: return gather_d<__half>(a, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace spruce
