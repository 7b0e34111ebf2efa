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
// Warp roles (352 threads):
//   warps 0-3  softmax + epilogue of tile 0 (TMEM lanes 0-127)
//   warps 4-7  softmax + epilogue of tile 1
//   warp  8    TMA producer (Q once, then K/V of each selected block, STAGES ring)
//   warp  9    TMEM allocator + QK^T issuer
//   warp 10    PV issuer
// Two issuing warps: a warp's barrier wait stalls until its own queued MMAs
// have been handed to the tensor core, so with one issuer every wait left the
// tensor core idle; with two, one warp's MMAs run while the other waits.
//
// Per selected block j and tile t:
//   S_t = Q_t K_j^T      (M=128, N=64, K=D; A, B K-major, 128B swizzle)
//   softmax_t: S_t -> registers (then S_t is released, so S_t(j+1) runs on
//              the tensor cores while this block's exponentials are computed)
//              -> P (bf16/fp16) into TMEM buffer P_t[j % 2]; O is rescaled
//              only when the running max grows by more than 8 in log2 units
//              (the final O / l is unaffected by the reference max used).
//   O_t += P_t[j % 2] V_j  (A from TMEM, B = V MN-major in smem, N = D)
// MMA issue order per block: S_0(j+1), S_1(j+1) as soon as each S buffer is
// released, then PV_0(j), PV_1(j).  A P buffer is rewritten only after the PV
// that read it has completed (one completion barrier per P buffer).
//
// TMEM columns: O_t at [t*D, (t+1)*D); S_t at 2D + 64t; P_t[b] at 2D + 128 + 64t + 32b.
#include <algorithm>

#include <cstdlib>
#include <cstring>

#include "attn_common.cuh"

namespace spruce {

constexpr int kAttnThreads = 352;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;   // QK^T issuer, owns the TMEM allocation
constexpr int kPvWarp = 10;   // PV issuer

template <int D, int STAGES>
struct AttnLayout {
  static constexpr int NP = D / 64;                  // 128-byte panels along the head dim
  static constexpr int Q_PANEL = 128 * 128;          // 128 rows x 128 B
  static constexpr int KV_PANEL = 64 * 128;          // 64 rows x 128 B
  static constexpr int Q_TILE = NP * Q_PANEL;
  static constexpr int KV_TILE = NP * KV_PANEL;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * Q_TILE;
  static constexpr int OFF_V = OFF_K + STAGES * KV_TILE;
  static constexpr int OFF_BAR = OFF_V + STAGES * KV_TILE;
  // q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], s_free[2], p_full[2][2], o_done[2][2], drain[2]
  static constexpr int NBAR = 1 + 3 * STAGES + 2 + 2 + 4 + 4 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_IDS = OFF_MISC + 16;
  static constexpr int COL_S = 2 * D;                // S_t at COL_S + 64 t
  static constexpr int COL_P = 2 * D + 128;          // P_t[b] at COL_P + 64 t + 32 b
  static constexpr uint32_t TMEM_COLS = (2 * D + 256 <= 256) ? 256u : 512u;
  static size_t smem_bytes(int kw) { return 1024 + OFF_IDS + 4 * (size_t)kw; }
};

template <typename T, int D, int STAGES>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv, const __grid_constant__ OutMaps om,
                          const AttnParams p) {
  using L = AttnLayout<D, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int i = p.q_begin + p.nq - 1 - static_cast<int>(blockIdx.x) / p.n_cta;  // late (heavy) rows first
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
  uint64_t* s_full = kv_empty + STAGES;  // [tile]
  uint64_t* s_free = s_full + 2;         // [tile]
  uint64_t* p_full = s_free + 2;         // [tile * 2 + P buffer]
  uint64_t* o_done = p_full + 4;         // [tile * 2 + P buffer]: PV that read that buffer is done
  uint64_t* drain = o_done + 4;          // [issuer warp]
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
        mbar_init(&s_free[t], 128);
      }
      for (int x = 0; x < 4; ++x) {
        mbar_init(&p_full[x], 128);
        mbar_init(&o_done[x], 1);
      }
      mbar_init(&drain[0], 1);
      mbar_init(&drain[1], 1);
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
    // The whole warp runs the loop (waits are warp-uniform); one elected lane issues.
    if (n > 0) {
      const bool leader = elect_one();
      uint8_t* qs = smem + L::OFF_Q;
      if (leader) {
        mbar_arrive_expect_tx(q_full, n_tiles * L::Q_TILE);
        for (int t = 0; t < n_tiles; ++t) {
          const int h0 = g * p.rep + 2 * (pair0 + t);
          for (int pp = 0; pp < L::NP; ++pp)
            tma_load_4d(qs + t * L::Q_TILE + pp * L::Q_PANEL, &tmq, q_full, pp * 64, h0, i * 64, b);
        }
      }
      __syncwarp();
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES &&
            !__all_sync(0xffffffffu, mbar_wait(&kv_empty[st], ((j / STAGES) - 1) & 1, p.status, abort_flag)))
          break;
        if (leader) {
          const int tok = ids[j] * 64;
          uint8_t* ks = smem + L::OFF_K + st * L::KV_TILE;
          uint8_t* vs = smem + L::OFF_V + st * L::KV_TILE;
          mbar_arrive_expect_tx(&k_full[st], L::KV_TILE);
          for (int pp = 0; pp < L::NP; ++pp)
            tma_load_4d(ks + pp * L::KV_PANEL, &tmk, &k_full[st], pp * 64, g, tok, b);
          mbar_arrive_expect_tx(&v_full[st], L::KV_TILE);
          for (int pp = 0; pp < L::NP; ++pp)
            tma_load_4d(vs + pp * L::KV_PANEL, &tmv, &v_full[st], pp * 64, g, tok, b);
        }
        __syncwarp();
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
  } else if (warp == kMmaWarp || warp == kPvWarp) {
    // ------------------------------------------------------------ MMA issuers
    // Each issuing warp runs its schedule converged; one elected lane issues.
    if (n > 0) {
      const bool leader = elect_one();
      constexpr uint32_t fmt = UmmaFormat<T>::value;
      constexpr uint32_t idesc_qk = idesc_f16(fmt, 0, 0, 64, 128);
      constexpr uint32_t idesc_pv = idesc_f16(fmt, 0, 1, D, 128);
      // Descriptors are built once; per MMA only the start address (low 14 bits,
      // 16-byte units, no carry: shared memory is < 256 KB) is advanced.
      const uint64_t dq0 = smem_desc(smem_u32(smem + L::OFF_Q), 16, 1024);
      const uint64_t dk0 = smem_desc(smem_u32(smem + L::OFF_K), 16, 1024);
      const uint64_t dv0 = smem_desc(smem_u32(smem + L::OFF_V), L::KV_PANEL, 1024);
      auto commit = [&](uint64_t* bar) {
        if (leader) umma_commit(bar);
        __syncwarp();
      };
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status, abort_flag));
      };
      bool ok = true;
      if (warp == kMmaWarp) {
        auto issue_qk = [&](int t, int st) {
          // S_t = Q_t . K^T over D in steps of 16 (32 bytes inside a 128-byte swizzle row).
          const uint32_t d = tmem + L::COL_S + 64 * t;
          const uint64_t qa = dq0 + (uint64_t)((t * L::Q_TILE) >> 4);
          const uint64_t kb = dk0 + (uint64_t)((st * L::KV_TILE) >> 4);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t offq = ((ks >> 2) * L::Q_PANEL + (ks & 3) * 32) >> 4;
            const uint32_t offk = ((ks >> 2) * L::KV_PANEL + (ks & 3) * 32) >> 4;
            if (leader) umma_f16_ss(d, qa + offq, kb + offk, idesc_qk, ks > 0 ? 1u : 0u);
            __syncwarp();
          }
        };
        ok = wait(q_full, 0);
        for (int j = 0; ok && j < n; ++j) {
          const int st = j % STAGES;
          if (!wait(&k_full[st], (j / STAGES) & 1)) break;
          for (int t = 0; t < n_tiles; ++t) {
            // S_t(j) once the softmax has taken S_t(j-1) into registers.
            if (j > 0 && !wait(&s_free[t], (j - 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk(t, st);
            commit(&s_full[t]);
          }
        }
        commit(&drain[0]);  // no MMA of this warp may be in flight when TMEM is released
        mbar_wait(&drain[0], 0, p.status, nullptr);
      } else {
        auto issue_pv = [&](int t, int st, int buf, bool accumulate) {
          // O_t += P_t[buf] . V over 64 keys in steps of 16 keys (8 TMEM columns of P, 2048 bytes of V).
          const uint32_t a = tmem + L::COL_P + 64 * t + 32 * buf;
          const uint64_t vb = dv0 + (uint64_t)((st * L::KV_TILE) >> 4);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            if (leader)
              umma_f16_ts(tmem + t * D, a + ks * 8, vb + (uint64_t)((ks * 2048) >> 4), idesc_pv,
                          (accumulate || ks > 0) ? 1u : 0u);
            __syncwarp();
          }
        };
        for (int j = 0; ok && j < n; ++j) {
          const int st = j % STAGES;
          const int buf = j & 1;
          if (!wait(&v_full[st], (j / STAGES) & 1)) break;
          for (int t = 0; t < n_tiles; ++t) {
            if (!wait(&p_full[2 * t + buf], (j >> 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, st, buf, j > 0);
            commit(&o_done[2 * t + buf]);
          }
          if (!ok) break;
          // QK(j) finished before softmax(j) began, so PV(j) completing frees stage st.
          commit(&kv_empty[st]);
        }
        commit(&drain[1]);
        mbar_wait(&drain[1], 0, p.status, nullptr);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;
    const int row = (warp & 3) * 32 + lane;  // TMEM lane == tile row
    const int tok = row >> 1;                // token within the query block
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + lane_off + t * D;
    if (t < n_tiles) {
      const float sl2 = p.scale_log2;
      float m_used = -INFINITY;  // reference max (log2 units) the exponentials use
      float l = 0.0f;
      bool ok = true;
      const uint32_t tS = tmem + lane_off + L::COL_S + 64 * t;
      for (int j = 0; j < n; ++j) {
        const int buf = j & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, p.status, abort_flag));
        if (!ok) break;
        tc_fence_after();
        float s[64];
        {
          float sa[32], sb[32];
          tmem_ld32(tS, sa);
          tmem_ld32(tS + 32, sb);
          tmem_wait_ld();
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            s[cc] = sa[cc];
            s[cc + 32] = sb[cc];
          }
        }
        tc_fence_before();
        mbar_arrive(&s_free[t]);  // S_t may now be overwritten by S_t(j+1)
        const bool diag = ids[j] == i;
        if (diag) {               // diagonal block: keys after the row's token are masked
#pragma unroll
          for (int cc = 0; cc < 64; ++cc)
            if (cc > tok) s[cc] = -INFINITY;
        }
        // Row max as a tree (exact in any order).
        float mx8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          mx8[u] = fmaxf(fmaxf(fmaxf(s[u], s[u + 8]), fmaxf(s[u + 16], s[u + 24])),
                         fmaxf(fmaxf(s[u + 32], s[u + 40]), fmaxf(s[u + 48], s[u + 56])));
        }
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float m_new = fmaxf(m_used, mx * sl2);
        const bool rescale = (j == 0) || (m_new > m_used + 8.0f);
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
          // PV(j-1) must be complete before O is rescaled.
          ok = __all_sync(0xffffffffu, mbar_wait(&o_done[2 * t + (buf ^ 1)], ((j - 1) >> 1) & 1, p.status,
                                                 abort_flag));
          if (!ok) break;
          tc_fence_after();
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
        if (rescale) m_used = m_new;
        const float neg_ref = (m_used == -INFINITY) ? 0.0f : -m_used;
        uint32_t pk[32];
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (!diag) {
          // A quarter of the exponentials on the FMA pipe, the rest on MUFU.
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            const float x0 = fmaf(s[2 * cc], sl2, neg_ref);
            const float x1 = fmaf(s[2 * cc + 1], sl2, neg_ref);
            const float e0 = (cc & 3) == 3 ? poly_exp2(x0) : fast_exp2(x0);
            const float e1 = (cc & 3) == 3 ? poly_exp2(x1) : fast_exp2(x1);
            part[cc & 3] += e0 + e1;
            pk[cc] = Pack2<T>::pack(e0, e1);
          }
        } else {
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            const float e0 = fast_exp2(fmaf(s[2 * cc], sl2, neg_ref));
            const float e1 = fast_exp2(fmaf(s[2 * cc + 1], sl2, neg_ref));
            part[cc & 3] += e0 + e1;
            pk[cc] = Pack2<T>::pack(e0, e1);
          }
        }
        l += (part[0] + part[1]) + (part[2] + part[3]);
        // P_t[buf] was last read by PV(j-2): it must be complete before it is overwritten.
        if (j >= 2) {
          ok = __all_sync(0xffffffffu, mbar_wait(&o_done[2 * t + buf], ((j - 2) >> 1) & 1, p.status, abort_flag));
          if (!ok) break;
          tc_fence_after();
        }
        tmem_st32u(tmem + lane_off + L::COL_P + 64 * t + 32 * buf, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[2 * t + buf]);
      }
      if (ok && n > 0)  // PV(n-1) complete (and with it every earlier PV into O_t)
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&o_done[2 * t + ((n - 1) & 1)], ((n - 1) >> 1) & 1, p.status, abort_flag));
      tc_fence_after();
      // Epilogue: O / l -> T staged in this tile's Q region (every QK MMA is complete
      // once PV(n-1) is), laid out [panel][head][token][128 B] with the 128-byte
      // swizzle, then TMA tensor stores to this GPU's output and to each peer's.
      uint8_t* stage = smem + L::OFF_Q + t * L::Q_TILE;
      const int hsub = row & 1;
      const int srow = hsub * 64 + tok;  // staging row: head-major
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
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          uint4 v;
          v.x = Pack2<T>::pack(o[v4 * 8 + 0] * inv, o[v4 * 8 + 1] * inv);
          v.y = Pack2<T>::pack(o[v4 * 8 + 2] * inv, o[v4 * 8 + 3] * inv);
          v.z = Pack2<T>::pack(o[v4 * 8 + 4] * inv, o[v4 * 8 + 5] * inv);
          v.w = Pack2<T>::pack(o[v4 * 8 + 6] * inv, o[v4 * 8 + 7] * inv);
          const int col = cc * 32 + v4 * 8;  // first of the 8 dims in this 16-byte chunk
          const int chunk = (col & 63) >> 3;
          *reinterpret_cast<uint4*>(stage + (col >> 6) * L::Q_PANEL + srow * 128 + ((chunk ^ (srow & 7)) << 4)) = v;
        }
      }
      fence_proxy_async_smem();
      named_barrier_sync(1 + t, 128);
      if ((warp & 3) == 0) {
        if (elect_one()) {
          for (int dst = 0; dst < om.count; ++dst)
            for (int h = 0; h < 2; ++h) {
              const int hh = 2 * (pair0 + t) + h;
              if (hh >= p.rep) continue;  // the half-filled last tile of an odd group
              for (int pp = 0; pp < L::NP; ++pp)
                tma_store_4d(&om.m[dst], stage + pp * L::Q_PANEL + h * 8192, pp * 64, g * p.rep + hh, i * 64, b);
            }
          tma_store_commit();
          tma_store_wait_read();  // shared memory must stay valid until the stores have read it
        }
        __syncwarp();
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
template <typename T, int D, int STAGES>
static cudaError_t launch_typed(const AttnArgs& a, CUtensorMapDataType dt, cudaStream_t stream) {
  using L = AttnLayout<D, STAGES>;
  CUtensorMap tmq, tmk, tmv;
  if (!make_map(&tmq, a.q, dt, a.B, a.Hq, a.T, D, a.qs, 2) || !make_map(&tmk, a.k, dt, a.B, a.Hkv, a.T, D, a.ks, 1) ||
      !make_map(&tmv, a.v, dt, a.B, a.Hkv, a.T, D, a.vs, 1))
    return cudaErrorInvalidValue;
  const AttnParams p = attn_params(a);
  OutMaps om;
  if (!attn_out_maps(a, dt, D, &om)) return cudaErrorInvalidValue;
  const size_t smem = L::smem_bytes(a.Kw);
  auto kern = attn_fwd_sm100_kernel<T, D, STAGES>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (p.nq <= 0) return cudaSuccess;
  dim3 grid(p.nq * p.n_cta, a.Hkv, a.B);
  kern<<<grid, kAttnThreads, smem, stream>>>(tmq, tmk, tmv, om, p);
  return cudaGetLastError();
}

constexpr size_t kMaxSmem = 227 * 1024;

int attn_sm100_max_kw(int D) {
  const size_t base = D == 128 ? AttnLayout<128, 4>::smem_bytes(0) : AttnLayout<64, 4>::smem_bytes(0);
  const int single = static_cast<int>((kMaxSmem - base) / 4);
  return std::min(single, attn_pair_max_kw(D));  // either kernel may run the call
}

// The pair kernel (attn_pair_sm100.cu) is the default; SPRUCE_ATTN_KERNEL=single
// selects this one-block-per-step kernel (for comparison).
static bool use_single_block_kernel() {
  static const int single = [] {
    const char* v = getenv("SPRUCE_ATTN_KERNEL");
    return (v != nullptr && strcmp(v, "single") == 0) ? 1 : 0;
  }();
  return single != 0;
}

cudaError_t launch_attn_sm100(const AttnArgs& a, int dtype, cudaStream_t stream) {
  // residual summaries are served by the pair kernel only
  if (!use_single_block_kernel() || a.vk != nullptr) return launch_attn_pair(a, dtype, stream);
  if (a.Kw > attn_sm100_max_kw(a.D)) return cudaErrorInvalidValue;
  if (dtype == SPRUCE_DTYPE_BF16) {
    if (a.D == 128) return launch_typed<__nv_bfloat16, 128, 4>(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
    if (a.D == 64) return launch_typed<__nv_bfloat16, 64, 4>(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
  } else if (dtype == SPRUCE_DTYPE_F16) {
    if (a.D == 128) return launch_typed<__half, 128, 4>(a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
    if (a.D == 64) return launch_typed<__half, 64, 4>(a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace spruce
