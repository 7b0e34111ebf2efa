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

#include "common.cuh"
#include "kernels.h"

namespace spruce {

namespace {

constexpr int kGatherThreads = 128;

template <typename T>
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
  const int n = min(npick, a.nvb * 64);
  const int npad = (n + 63) / 64 * 64;
  const int64_t Tv = (int64_t)a.qb * a.nvb * 64;
  const int64_t vrow0 = ((int64_t)b * a.Hkv + g) * Tv + (int64_t)i * a.nvb * 64;
  T* vk = static_cast<T*>(a.vk) + vrow0 * a.D;
  T* vv = static_cast<T*>(a.vv) + vrow0 * a.D;
  for (int e = threadIdx.x; e < npad * a.D; e += kGatherThreads) {
    const int r = e / a.D, d = e % a.D;
    float kx = 0.0f, vx = 0.0f;
    if (r < n) {
      const int pick = picks[r];
      const int node = row[(pick / a.P) * a.ns[3]];
      const int64_t src = ((((int64_t)b * a.Hkv + g) * a.NN + node) * a.P + pick % a.P) * a.D + d;
      kx = a.keys[src];
      vx = a.values[src];
    }
    vk[e] = Elem<T>::from_f(kx);
    vv[e] = Elem<T>::from_f(vx);
  }
  for (int r = threadIdx.x; r < npad; r += kGatherThreads) {
    float bias = -INFINITY;
    if (r < n) {
      const int pick = picks[r];
      const int node = row[(pick / a.P) * a.ns[3]];
      bias = a.log_counts[((int64_t)b * a.NN + node) * a.P + pick % a.P];
    }
    a.vbias[vrow0 + r] = bias;
  }
  if (threadIdx.x == 0) a.vcount[((int64_t)b * a.Hkv + g) * a.qb + i] = npad / 64;
}

}  // namespace

cudaError_t launch_residual_gather(const ResidualGatherArgs& a, int dtype, cudaStream_t stream) {
  if (a.B == 0 || a.Hkv == 0 || a.qb == 0) return cudaSuccess;
  const size_t smem = sizeof(int) * (size_t)std::max(1, a.S * a.P);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  dim3 grid((unsigned)a.qb, (unsigned)a.Hkv, (unsigned)a.B);
  switch (dtype) {
    case SPRUCE_DTYPE_F32: {
      cudaError_t e = cudaFuncSetAttribute(residual_gather_kernel<float>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      residual_gather_kernel<float><<<grid, kGatherThreads, smem, stream>>>(a);
      break;
    }
    case SPRUCE_DTYPE_BF16: {
      cudaError_t e = cudaFuncSetAttribute(residual_gather_kernel<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      residual_gather_kernel<__nv_bfloat16><<<grid, kGatherThreads, smem, stream>>>(a);
      break;
    }
    case SPRUCE_DTYPE_F16: {
      cudaError_t e = cudaFuncSetAttribute(residual_gather_kernel<__half>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      residual_gather_kernel<__half><<<grid, kGatherThreads, smem, stream>>>(a);
      break;
    }
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace spruce
