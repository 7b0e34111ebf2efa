// Causal GQA block-sparse attention on sm_100a: TMA gathers of the selected
// K/V blocks, tcgen05 MMAs with TMEM accumulators, online softmax.
//
// Reference semantics: kernels/seerattention_direct_index_triton.py:36-121
// (_single_head_kernel: per query block, loop over the row's selected block
// ids, skip -1, exp2 online softmax with scale*log2(e), causal mask) and
// sparse/attention.py:143-274 (fp32 scores, output [B, T, Hq, D]).
//
// Work unit (one CTA): batch b, KV group g, query block i and up to two
// 128-row M-tiles.  A tile holds two query heads x 64 tokens: the TMA box
// (64 dims, 2 heads, 64 tokens) lands as rows r = token * 2 + head, so the
// 7 heads of a Qwen2.5-7B group take 4 tiles (the last half-filled) in two
// CTAs, and every K/V block a CTA gathers is reused by 2 tiles = 4 heads.
//
// Warp roles (320 threads):
//   warps 0-3  softmax + epilogue of tile 0 (TMEM lanes 0-127)
//   warps 4-7  softmax + epilogue of tile 1
//   warp  8    TMA producer (Q once, then K/V of each selected block, STAGES ring)
//   warp  9    TMEM allocator + single-thread MMA issuer
// Per selected block j and tile t:
//   S_t = Q_t K_j^T      (M=128, N=64, K=D; A, B K-major, 128B swizzle)
//   softmax_t: S -> P (bf16/fp16, swizzled smem), lazy O rescale (only when
//              the running max grows by more than 8 in log2 units)
//   O_t += P_t V_j       (M=128, N=D, K=64; B MN-major)
// The MMA warp interleaves the tiles: PV_0(j), S_0(j+1), PV_1(j), S_1(j+1),
// so one tile's softmax overlaps the other tile's tensor-core work.
//
// TMEM columns: O_0 [0, D), O_1 [D, 2D), S_0 [2D, 2D+64), S_1 [2D+64, 2D+128).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace spruce {

constexpr int kAttnThreads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;

struct AttnParams {
  const int32_t* idx;
  int64_t isb, isg, isq;
  void* out;
  int64_t osb, osh, ost;
  int Hq, Hkv, T, Kw, qb, rep, n_pair, n_cta;
  float scale_log2;
  uint32_t* status;
};

template <int D, int STAGES>
struct AttnLayout {
  static constexpr int NP = D / 64;                  // 128-byte panels along the head dim
  static constexpr int Q_PANEL = 128 * 128;          // 128 rows x 128 B
  static constexpr int KV_PANEL = 64 * 128;          // 64 rows x 128 B
  static constexpr int Q_TILE = NP * Q_PANEL;
  static constexpr int KV_TILE = NP * KV_PANEL;
  static constexpr int P_TILE = 128 * 128;           // 128 rows x 64 keys x 2 B
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * Q_TILE;
  static constexpr int OFF_V = OFF_K + STAGES * KV_TILE;
  static constexpr int OFF_P = OFF_V + STAGES * KV_TILE;
  static constexpr int OFF_BAR = OFF_P + 2 * P_TILE;
  // q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2], o_done[2], drain
  static constexpr int NBAR = 1 + 3 * STAGES + 7;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_IDS = OFF_MISC + 16;
  static constexpr int COL_O0 = 0, COL_O1 = D, COL_S0 = 2 * D, COL_S1 = 2 * D + 64;
  static constexpr uint32_t TMEM_COLS = (2 * D + 128 <= 256) ? 256u : 512u;
  static size_t smem_bytes(int kw) { return 1024 + OFF_IDS + 4 * (size_t)kw; }
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

template <typename T, int D, int STAGES>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const AttnParams p) {
  using L = AttnLayout<D, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int i = p.qb - 1 - static_cast<int>(blockIdx.x) / p.n_cta;  // late (heavy) rows first
  const int c = static_cast<int>(blockIdx.x) % p.n_cta;
  const int g = blockIdx.y;
  const int b = blockIdx.z;
  const int pair0 = 2 * c;
  const int n_tiles = min(2, p.n_pair - pair0);

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  int* nsel_slot = reinterpret_cast<int*>(smem + L::OFF_MISC + 8);
  int* ids = reinterpret_cast<int*>(smem + L::OFF_IDS);

  // ---- setup: compact the row's block ids, init barriers, allocate TMEM
  if (warp == kProducerWarp) {
    const int32_t* row = p.idx + b * p.isb + g * p.isg + (int64_t)i * p.isq;
    int count = 0;
    for (int base = 0; base < p.Kw; base += 32) {
      const int col = base + lane;
      const int id = col < p.Kw ? row[col] : -1;
      const bool keep = id >= 0 && id <= i;  // padding skipped; future blocks are fully masked anyway
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (keep) ids[count + __popc(m & ((1u << lane) - 1u))] = id;
      count += __popc(m);
    }
    if (lane == 0) {
      *nsel_slot = count;
      *abort_flag = 0;
      mbar_init(q_full, 1);
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(&k_full[s], 1);
        mbar_init(&v_full[s], 1);
        mbar_init(&kv_empty[s], 1);
      }
      for (int t = 0; t < 2; ++t) {
        mbar_init(&s_full[t], 1);
        mbar_init(&p_full[t], 128);
        mbar_init(&o_done[t], 1);
      }
      mbar_init(drain, 1);
      fence_barrier_init();
      prefetch_tmap(&tmq);
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n = *nsel_slot;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n > 0) {
      uint8_t* qs = smem + L::OFF_Q;
      mbar_arrive_expect_tx(q_full, n_tiles * L::Q_TILE);
      for (int t = 0; t < n_tiles; ++t) {
        const int h0 = g * p.rep + 2 * (pair0 + t);
        for (int pp = 0; pp < L::NP; ++pp)
          tma_load_4d(qs + t * L::Q_TILE + pp * L::Q_PANEL, &tmq, q_full, pp * 64, h0, i * 64, b);
      }
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES && !mbar_wait(&kv_empty[st], ((j / STAGES) - 1) & 1, p.status, abort_flag)) break;
        const int tok = ids[j] * 64;
        uint8_t* ks = smem + L::OFF_K + st * L::KV_TILE;
        uint8_t* vs = smem + L::OFF_V + st * L::KV_TILE;
        mbar_arrive_expect_tx(&k_full[st], L::KV_TILE);
        for (int pp = 0; pp < L::NP; ++pp) tma_load_4d(ks + pp * L::KV_PANEL, &tmk, &k_full[st], pp * 64, g, tok, b);
        mbar_arrive_expect_tx(&v_full[st], L::KV_TILE);
        for (int pp = 0; pp < L::NP; ++pp) tma_load_4d(vs + pp * L::KV_PANEL, &tmv, &v_full[st], pp * 64, g, tok, b);
        issued = j + 1;
      }
      // No copy may be in flight when the CTA exits: wait for the last loads.
      mbar_wait(q_full, 0, p.status, nullptr);
      for (int j = max(0, issued - STAGES); j < issued; ++j) {
        mbar_wait(&k_full[j % STAGES], (j / STAGES) & 1, p.status, nullptr);
        mbar_wait(&v_full[j % STAGES], (j / STAGES) & 1, p.status, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      constexpr uint32_t fmt = UmmaFormat<T>::value;
      constexpr uint32_t idesc_qk = idesc_f16(fmt, 0, 0, 64, 128);
      constexpr uint32_t idesc_pv = idesc_f16(fmt, 0, 1, D, 128);
      const uint32_t q_base = smem_u32(smem + L::OFF_Q);
      const uint32_t k_base = smem_u32(smem + L::OFF_K);
      const uint32_t v_base = smem_u32(smem + L::OFF_V);
      const uint32_t p_base = smem_u32(smem + L::OFF_P);
      const uint32_t s_col[2] = {tmem + L::COL_S0, tmem + L::COL_S1};
      const uint32_t o_col[2] = {tmem + L::COL_O0, tmem + L::COL_O1};

      auto issue_qk = [&](int t, int st) {
        // S_t = Q_t . K^T over D in steps of 16 (32 bytes inside a 128-byte swizzle row).
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks & 3) * 32;
          const uint64_t a = smem_desc(q_base + t * L::Q_TILE + (ks >> 2) * L::Q_PANEL + off, 16, 1024);
          const uint64_t bb = smem_desc(k_base + st * L::KV_TILE + (ks >> 2) * L::KV_PANEL + off, 16, 1024);
          umma_f16_ss(s_col[t], a, bb, idesc_qk, ks > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int st, bool accumulate) {
        // O_t += P_t . V over the 64 keys in steps of 16 keys (2048 bytes of V).
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t a = smem_desc(p_base + t * L::P_TILE + ks * 32, 16, 1024);
          const uint64_t bb = smem_desc(v_base + st * L::KV_TILE + ks * 2048, L::KV_PANEL, 1024);
          umma_f16_ss(o_col[t], a, bb, idesc_pv, (accumulate || ks > 0) ? 1u : 0u);
        }
      };

      bool ok = mbar_wait(q_full, 0, p.status, abort_flag) && mbar_wait(&k_full[0], 0, p.status, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < n_tiles; ++t) {
          issue_qk(t, 0);
          umma_commit(&s_full[t]);
        }
      }
      for (int j = 0; ok && j < n; ++j) {
        const int st = j % STAGES;
        const int st1 = (j + 1) % STAGES;
        if (!mbar_wait(&v_full[st], (j / STAGES) & 1, p.status, abort_flag)) break;
        if (j + 1 < n && !mbar_wait(&k_full[st1], ((j + 1) / STAGES) & 1, p.status, abort_flag)) break;
        for (int t = 0; t < n_tiles; ++t) {
          if (!mbar_wait(&p_full[t], j & 1, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, st, j > 0);
          umma_commit(&o_done[t]);
          if (t == n_tiles - 1) umma_commit(&kv_empty[st]);
          if (j + 1 < n) {
            issue_qk(t, st1);
            umma_commit(&s_full[t]);
          }
        }
      }
      // No MMA may be in flight when TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, p.status, nullptr);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;
    const int row = (warp & 3) * 32 + lane;  // TMEM lane == tile row
    const int tok = row >> 1;                // token within the query block
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + (t ? L::COL_S1 : L::COL_S0);
    const uint32_t tO = tmem + lane_off + (t ? L::COL_O1 : L::COL_O0);
    uint8_t* Ps = smem + L::OFF_P + t * L::P_TILE;
    if (t < n_tiles) {
      float m_used = -INFINITY;
      float l = 0.0f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, p.status, abort_flag));
        if (!ok) break;
        tc_fence_after();
        float sa[32], sb[32];
        tmem_ld32(tS, sa);
        tmem_ld32(tS + 32, sb);
        tmem_wait_ld();
        float s[64];
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          s[cc] = sa[cc];
          s[cc + 32] = sb[cc];
        }
        const bool diag = ids[j] == i;
        float mx = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < 64; ++cc) {
          float x = s[cc] * p.scale_log2;
          if (diag && cc > tok) x = -INFINITY;
          s[cc] = x;
          mx = fmaxf(mx, x);
        }
        const float m_new = fmaxf(m_used, mx);
        const bool rescale = (j == 0) || (m_new > m_used + 8.0f);
        if (j > 0) {
          // PV(j-1) must be complete before P is overwritten or O is rescaled.
          ok = __all_sync(0xffffffffu, mbar_wait(&o_done[t], (j - 1) & 1, p.status, abort_flag));
          if (!ok) break;
          tc_fence_after();
          if (__any_sync(0xffffffffu, rescale)) {
            const float alpha = rescale ? fast_exp2(m_used - m_new) : 1.0f;
#pragma unroll 1
            for (int cc = 0; cc < D / 32; ++cc) {
              float o[32];
              tmem_ld32(tO + cc * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] *= alpha;
              tmem_st32(tO + cc * 32, o);
            }
            tmem_wait_st();
            l *= alpha;
          }
        }
        if (rescale) m_used = m_new;
        const float mref = (m_used == -INFINITY) ? 0.0f : m_used;
        float sum = 0.0f;
        uint8_t* prow = Ps + row * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          float e[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            e[k] = fast_exp2(s[ch * 8 + k] - mref);
            sum += e[k];
          }
          uint4 v;
          v.x = Pack2<T>::pack(e[0], e[1]);
          v.y = Pack2<T>::pack(e[2], e[3]);
          v.z = Pack2<T>::pack(e[4], e[5]);
          v.w = Pack2<T>::pack(e[6], e[7]);
          *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) = v;
        }
        l += sum;
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
      }
      if (ok && n > 0) ok = __all_sync(0xffffffffu, mbar_wait(&o_done[t], (n - 1) & 1, p.status, abort_flag));
      tc_fence_after();
      // Epilogue: O / l -> T, row (token, head) of the token-major output.
      const int hh = 2 * (pair0 + t) + (row & 1);
      const int token = i * 64 + tok;
      const bool valid = hh < p.rep && token < p.T;
      T* orow = static_cast<T*>(p.out) + b * p.osb + (int64_t)(g * p.rep + hh) * p.osh + (int64_t)token * p.ost;
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      if (n == 0 && row == 0) raise_status(p.status, SPRUCE_STATUS_EMPTY_ROW);
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        if (ok && n > 0) {
          tmem_ld32(tO + cc * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0.0f;
        }
        if (valid) {
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint4 v;
            v.x = Pack2<T>::pack(o[v4 * 8 + 0] * inv, o[v4 * 8 + 1] * inv);
            v.y = Pack2<T>::pack(o[v4 * 8 + 2] * inv, o[v4 * 8 + 3] * inv);
            v.z = Pack2<T>::pack(o[v4 * 8 + 4] * inv, o[v4 * 8 + 5] * inv);
            v.w = Pack2<T>::pack(o[v4 * 8 + 6] * inv, o[v4 * 8 + 7] * inv);
            *reinterpret_cast<uint4*>(orow + cc * 32 + v4 * 8) = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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
static bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int B, int H, int T, int D,
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

template <typename T, int D, int STAGES>
static cudaError_t launch_typed(const AttnArgs& a, CUtensorMapDataType dt, cudaStream_t stream) {
  using L = AttnLayout<D, STAGES>;
  CUtensorMap tmq, tmk, tmv;
  if (!make_map(&tmq, a.q, dt, a.B, a.Hq, a.T, D, a.qs, 2) || !make_map(&tmk, a.k, dt, a.B, a.Hkv, a.T, D, a.ks, 1) ||
      !make_map(&tmv, a.v, dt, a.B, a.Hkv, a.T, D, a.vs, 1))
    return cudaErrorInvalidValue;
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
  p.rep = a.Hq / a.Hkv;
  p.n_pair = (p.rep + 1) / 2;
  p.n_cta = (p.n_pair + 1) / 2;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.status = a.status;
  const size_t smem = L::smem_bytes(a.Kw);
  auto kern = attn_fwd_sm100_kernel<T, D, STAGES>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.qb * p.n_cta, a.Hkv, a.B);
  kern<<<grid, kAttnThreads, smem, stream>>>(tmq, tmk, tmv, p);
  return cudaGetLastError();
}

constexpr size_t kMaxSmem = 227 * 1024;

int attn_sm100_max_kw(int D) {
  const size_t base = D == 128 ? AttnLayout<128, 3>::smem_bytes(0) : AttnLayout<64, 4>::smem_bytes(0);
  return static_cast<int>((kMaxSmem - base) / 4);
}

cudaError_t launch_attn_sm100(const AttnArgs& a, int dtype, cudaStream_t stream) {
  if (a.Kw > attn_sm100_max_kw(a.D)) return cudaErrorInvalidValue;
  if (dtype == SPRUCE_DTYPE_BF16) {
    if (a.D == 128) return launch_typed<__nv_bfloat16, 128, 3>(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
    if (a.D == 64) return launch_typed<__nv_bfloat16, 64, 4>(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
  } else if (dtype == SPRUCE_DTYPE_F16) {
    if (a.D == 128) return launch_typed<__half, 128, 3>(a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
    if (a.D == 64) return launch_typed<__half, 64, 4>(a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace spruce
