// Pieces shared by the sm_100a attention kernels: launch parameters, output
// tensor maps for the fused multi-GPU gather, P packing, the FMA-pipe exp2,
// TMEM-operand MMA and TMEM stores, and the host-side tensor-map encoder.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace spruce {

struct AttnParams {
  const int32_t* idx;
  int64_t isb, isg, isq;
  void* out;
  int64_t osb, osh, ost;
  int Hq, Hkv, T, Kw, qb, rep, n_pair, n_cta;
  int q_begin, nq;  // query blocks [q_begin, q_begin + nq) are computed
  float scale_log2;
  uint32_t* status;
  const float* vbias;     // residual summaries (see AttnArgs); nullptr: none
  const int32_t* vcount;
  int Tv, nvb;
};

// Output tensor maps: [0] this GPU's output, [1..] the peers' outputs for the
// fused all-gather (NVLink peer memory, same layout).  Box (64 dims, 1 head,
// 64 tokens), 128-byte swizzle.
struct OutMaps {
  CUtensorMap m[1 + kMaxPeers];
  int count;
};

template <typename T> struct Pack2;
template <> struct Pack2<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Pack2<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// 2^x on the FMA pipe, to take part of the softmax's exponentials off the
// 16-per-clock MUFU unit.  Range reduction n = round(x) by the 1.5 * 2^23
// rounding trick (Cody-Waite), f = x - n in [-0.5, 0.5], 2^f by a degree-3
// polynomial fitted here (iterated weighted least squares on 20001 points for
// minimal relative error; max relative error 7.6e-5 with fp32 Horner
// evaluation, against 3.9e-3 = the bf16 precision P is rounded to), and
// 2^n applied as 2^(n+1) in the exponent field times 0.5 (the product rounds correctly
// where the result is subnormal, e.g. x = -126, where p(0) < 1 would otherwise land in
// the subnormal encoding).  x is clamped at -126; callers only pass x <= 8 (lazy
// rescale) and never -inf.
__device__ __forceinline__ float poly_exp2(float x) {
  x = fmaxf(x, -126.0f);
  const float kRound = 12582912.0f;  // 1.5 * 2^23
  const float t = x + kRound;
  const float n = t - kRound;
  const float f = x - n;
  const float p =
      fmaf(fmaf(fmaf(0.05517556518316269f, f, 0.24262112379074097f), f, 0.6932611465454102f), f, 0.999927282333374f);
  const int ni = __float_as_int(t) - __float_as_int(kRound);
  return __int_as_float(__float_as_int(p) + ((ni + 1) << 23)) * 0.5f;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: two lanes of fp32 math per
// issue slot, each lane rounded exactly as the scalar instruction).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// poly_exp2 of two values with packed arithmetic: the same reduction and
// polynomial, lane by lane, so each result equals poly_exp2 of its input.
__device__ __forceinline__ void poly_exp2_x2(float x0, float x1, float& e0, float& e1) {
  const float kRound = 12582912.0f;  // 1.5 * 2^23
  const uint64_t x = f2_pack(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t kr = f2_pack(kRound, kRound);
  const uint64_t t = f2_add(x, kr);
  const uint64_t f = f2_sub(x, f2_sub(t, kr));
  uint64_t q = f2_fma(f2_pack(0.05517556518316269f, 0.05517556518316269f), f,
                      f2_pack(0.24262112379074097f, 0.24262112379074097f));
  q = f2_fma(q, f, f2_pack(0.6932611465454102f, 0.6932611465454102f));
  q = f2_fma(q, f, f2_pack(0.999927282333374f, 0.999927282333374f));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  const float s0 = __int_as_float(__float_as_int(q0) + ((__float_as_int(t0) - __float_as_int(kRound) + 1) << 23));
  const float s1 = __int_as_float(__float_as_int(q1) + ((__float_as_int(t1) - __float_as_int(kRound) + 1) << 23));
  f2_unpack(f2_mul(f2_pack(s0, s1), f2_pack(0.5f, 0.5f)), e0, e1);
}

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], kind::f16.  A has M rows = TMEM lanes and K
// packed two 16-bit values per 32-bit column (8 columns per K = 16 step).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 4-D map over [B, H, T, D] (dims innermost first: D, H, T, B), 128-byte swizzle,
// box (64 dims, box_h heads, 64 tokens, 1).  Out-of-range boxes read zeros.
static inline bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int B, int H, int T, int D,
                     const int64_t* s, int box_h) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)s[1] * 2, (cuuint64_t)s[2] * 2, (cuuint64_t)s[0] * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_h, 64, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


// AttnParams of a launch (everything but the kernel-specific layout).
static inline AttnParams attn_params(const AttnArgs& a) {
  AttnParams p;
  p.idx = a.idx;
  p.isb = a.is[0];
  p.isg = a.is[1];
  p.isq = a.is[2];
  p.out = a.out;
  p.osb = a.os[0];
  p.osh = a.os[1];
  p.ost = a.os[2];
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.T = a.T;
  p.Kw = a.Kw;
  p.qb = (a.T + 63) / 64;
  p.q_begin = a.q_begin;
  p.nq = a.q_end - a.q_begin;
  p.rep = a.Hq / a.Hkv;
  p.n_pair = (p.rep + 1) / 2;
  p.n_cta = (p.n_pair + 1) / 2;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.status = a.status;
  p.vbias = a.vbias;
  p.vcount = a.vcount;
  p.Tv = a.Tv;
  p.nvb = a.nvb;
  return p;
}

// Output maps over the LOGICAL [B, Hq, T, D] output strides, one head per box:
// [0] this GPU's output, [1..] the peers' outputs.
static inline bool attn_out_maps(const AttnArgs& a, CUtensorMapDataType dt, int D, OutMaps* om) {
  om->count = 1 + a.n_peer;
  if (!make_map(&om->m[0], a.out, dt, a.B, a.Hq, a.T, D, a.os, 1)) return false;
  for (int pp = 0; pp < a.n_peer; ++pp)
    if (!make_map(&om->m[1 + pp], a.peer_out[pp], dt, a.B, a.Hq, a.T, D, a.os, 1)) return false;
  return true;
}

}  // namespace spruce
