// fp32 block-sparse causal GQA attention on CUDA cores.
//
// The tensor cores have no fp32-exact mode (tf32 rounds operands to 10
// mantissa bits, far outside the 1e-4 fp32 tolerance of the reference's
// torch path, sparse/attention.py:213-219), so fp32 inputs run this kernel:
// one CTA per (batch, query head, query block), 256 threads = 64 rows x 4
// column quarters, K/V tiles of the selected blocks staged in shared memory,
// exact online softmax in fp32 (expf).  Same index semantics as the tcgen05
// kernel: ids < 0 skipped, ids above the query block contribute nothing.
// With residual summaries the row's virtual blocks (gathered summary keys,
// sparse/attention.py:224-263) follow its selected blocks in the same online
// softmax: score = q.k * scale + natural-log count bias, no causal mask.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace spruce {

struct F32Params {
  const float* q;
  const float* k;
  const float* v;
  int64_t qsb, qsh, qst, ksb, ksh, kst, vsb, vsh, vst;
  const int32_t* idx;
  int64_t isb, isg, isq;
  float* out;
  int64_t osb, osh, ost;
  int Hq, Hkv, T, Kw, qb, rep, q_begin, nq;
  float scale;
  uint32_t* status;
  const float* vk;  // residual summaries (nullptr: none), see AttnArgs
  const float* vv;
  int64_t vksb, vksh, vkst, vvsb, vvsh, vvst;
  const float* vbias;
  const int32_t* vcount;
  int Tv, nvb;
};

template <int D>
__global__ void __launch_bounds__(256) attn_fwd_f32_kernel(const F32Params p) {
  constexpr int KP = D + 4;  // padded K rows (float4 reads stay aligned, fewer bank conflicts)
  extern __shared__ float fsm[];
  float* Qs = fsm;                 // [64][D]
  float* Ks = Qs + 64 * D;         // [64][KP]
  float* Vs = Ks + 64 * KP;        // [64][D]
  float* Ps = Vs + 64 * D;         // [64][65]
  int* ids = reinterpret_cast<int*>(Ps + 64 * 65);
  __shared__ int nsel;

  const int i = p.q_begin + p.nq - 1 - blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int g = h / p.rep;
  const int tid = threadIdx.x;
  const int r = tid >> 2, part = tid & 3;
  const int warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    const int32_t* row = p.idx + b * p.isb + g * p.isg + (int64_t)i * p.isq;
    int count = 0;
    for (int base = 0; base < p.Kw; base += 32) {
      const int col = base + lane;
      const int id = col < p.Kw ? row[col] : -1;
      const bool keep = id >= 0 && id <= i;
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (keep) ids[count + __popc(m & ((1u << lane) - 1u))] = id;
      count += __popc(m);
    }
    if (lane == 0) nsel = count;
  }
  __shared__ int nvirt;
  if (tid == 0) nvirt = p.vk != nullptr ? min(p.vcount[((int64_t)b * p.Hkv + g) * p.qb + i], p.nvb) : 0;
  const int qtok0 = i * 64;
  for (int e = tid; e < 64 * D; e += 256) {
    const int rr = e / D, d = e % D;
    const int t = qtok0 + rr;
    Qs[e] = t < p.T ? p.q[b * p.qsb + h * p.qsh + (int64_t)t * p.qst + d] : 0.0f;
  }
  __syncthreads();
  const int n = nsel;
  const int nv = nvirt;

  constexpr int DQ = D / 4;
  float o[DQ];
#pragma unroll
  for (int d = 0; d < DQ; ++d) o[d] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  const int qtok = qtok0 + r;

  for (int j = 0; j < n + nv; ++j) {
    const bool virt = j >= n;  // a virtual block of summary keys
    const int k0 = virt ? (i * p.nvb + (j - n)) * 64 : ids[j] * 64;
    __syncthreads();
    if (!virt) {
      for (int e = tid; e < 64 * D; e += 256) {
        const int rr = e / D, d = e % D;
        const int t = k0 + rr;
        const bool in = t < p.T;
        Ks[rr * KP + d] = in ? p.k[b * p.ksb + g * p.ksh + (int64_t)t * p.kst + d] : 0.0f;
        Vs[rr * D + d] = in ? p.v[b * p.vsb + g * p.vsh + (int64_t)t * p.vst + d] : 0.0f;
      }
    } else {
      for (int e = tid; e < 64 * D; e += 256) {
        const int rr = e / D, d = e % D;
        const int64_t t = k0 + rr;
        Ks[rr * KP + d] = p.vk[b * p.vksb + g * p.vksh + t * p.vkst + d];
        Vs[rr * D + d] = p.vv[b * p.vvsb + g * p.vvsh + t * p.vvst + d];
      }
    }
    __syncthreads();
    const float* vbias = virt ? p.vbias + ((int64_t)b * p.Hkv + g) * p.Tv + k0 : nullptr;
    float s[16];
    float mx = -INFINITY;
#pragma unroll
    for (int cc = 0; cc < 16; ++cc) {
      const int col = part * 16 + cc;
      const float4* qa = reinterpret_cast<const float4*>(Qs + r * D);
      const float4* ka = reinterpret_cast<const float4*>(Ks + col * KP);
      float acc = 0.0f;
#pragma unroll 8
      for (int d4 = 0; d4 < D / 4; ++d4) {
        const float4 x = qa[d4], y = ka[d4];
        acc = fmaf(x.x, y.x, acc);
        acc = fmaf(x.y, y.y, acc);
        acc = fmaf(x.z, y.z, acc);
        acc = fmaf(x.w, y.w, acc);
      }
      float sc = acc * p.scale;
      if (virt)
        sc += vbias[col];  // padding rows carry -inf
      else if (k0 + col > qtok)
        sc = -INFINITY;  // causal (also drops keys >= T for real rows)
      s[cc] = sc;
      mx = fmaxf(mx, sc);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m, mx);
    const float mref = m_new == -INFINITY ? 0.0f : m_new;
    const float alpha = m == -INFINITY ? 0.0f : expf(m - mref);
    float sum = 0.0f;
#pragma unroll
    for (int cc = 0; cc < 16; ++cc) {
      const float pr = s[cc] == -INFINITY ? 0.0f : expf(s[cc] - mref);
      Ps[r * 65 + part * 16 + cc] = pr;
      sum += pr;
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l = l * alpha + sum;
    m = m_new;
    __syncwarp();
#pragma unroll
    for (int d = 0; d < DQ; ++d) o[d] *= alpha;
    for (int col = 0; col < 64; ++col) {
      const float pr = Ps[r * 65 + col];
      const float* vr = Vs + col * D + part * DQ;
#pragma unroll
      for (int d = 0; d < DQ; ++d) o[d] = fmaf(pr, vr[d], o[d]);
    }
  }
  if (n == 0 && tid == 0) raise_status(p.status, SPRUCE_STATUS_EMPTY_ROW);
  if (qtok < p.T) {
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    float* orow = p.out + b * p.osb + h * p.osh + (int64_t)qtok * p.ost + part * DQ;
#pragma unroll
    for (int d = 0; d < DQ; ++d) orow[d] = o[d] * inv;
  }
}

template <int D>
static cudaError_t launch_f32_typed(const AttnArgs& a, cudaStream_t stream) {
  F32Params p;
  p.q = static_cast<const float*>(a.q);
  p.k = static_cast<const float*>(a.k);
  p.v = static_cast<const float*>(a.v);
  p.qsb = a.qs[0]; p.qsh = a.qs[1]; p.qst = a.qs[2];
  p.ksb = a.ks[0]; p.ksh = a.ks[1]; p.kst = a.ks[2];
  p.vsb = a.vs[0]; p.vsh = a.vs[1]; p.vst = a.vs[2];
  p.idx = a.idx;
  p.isb = a.is[0]; p.isg = a.is[1]; p.isq = a.is[2];
  p.out = static_cast<float*>(a.out);
  p.osb = a.os[0]; p.osh = a.os[1]; p.ost = a.os[2];
  p.Hq = a.Hq; p.Hkv = a.Hkv; p.T = a.T; p.Kw = a.Kw;
  p.qb = (a.T + 63) / 64;
  p.rep = a.Hq / a.Hkv;
  p.q_begin = a.q_begin;
  p.nq = a.q_end - a.q_begin;
  p.scale = a.scale;
  p.status = a.status;
  p.vk = static_cast<const float*>(a.vk);
  p.vv = static_cast<const float*>(a.vv);
  if (a.vk != nullptr) {
    p.vksb = a.vks[0]; p.vksh = a.vks[1]; p.vkst = a.vks[2];
    p.vvsb = a.vvs[0]; p.vvsh = a.vvs[1]; p.vvst = a.vvs[2];
  } else {
    p.vksb = p.vksh = p.vkst = p.vvsb = p.vvsh = p.vvst = 0;
  }
  p.vbias = a.vbias;
  p.vcount = a.vcount;
  p.Tv = a.Tv;
  p.nvb = a.nvb;
  const size_t smem = sizeof(float) * (64 * D + 64 * (D + 4) + 64 * D + 64 * 65) + sizeof(int) * (size_t)a.Kw;
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_f32_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (p.nq <= 0) return cudaSuccess;
  dim3 grid(p.nq, a.Hq, a.B);
  attn_fwd_f32_kernel<D><<<grid, 256, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_attn_f32(const AttnArgs& a, cudaStream_t stream) {
  if (a.D == 128) return launch_f32_typed<128>(a, stream);
  if (a.D == 64) return launch_f32_typed<64>(a, stream);
  return cudaErrorInvalidValue;
}

}  // namespace spruce
