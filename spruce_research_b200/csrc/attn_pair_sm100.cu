// Causal GQA block-sparse attention on sm_100a, two selected blocks per step.
//
// Reference semantics: kernels/seerattention_direct_index_triton.py:36-121
// (per query block, loop over the row's selected block ids, skip -1, exp2
// online softmax with scale*log2(e), causal mask) and sparse/attention.py:
// 143-274 (fp32 scores, output [B, T, Hq, D]).
//
// Work unit, warp roles, TMA gathers and epilogue are those of
// attn_sm100.cu: one CTA per (batch b, KV group g, query block i, two
// 128-row M-tiles of 2 heads x 64 tokens).  The difference is the step: the
// row's selected blocks are taken two at a time.  Blocks ids[2j], ids[2j+1]
// land as token rows 0-63 and 64-127 of one 128-token K/V stage, so
//   S_t = Q_t K^T   is M=128, N=128 per 16 dims   (8 MMAs per step),
//   O_t += P_t V    is M=128, N=D per 16 tokens   (8 MMAs per step),
// where single blocks need N=64 QK MMAs, which reach ~61% of the rate an
// N=128 MMA does.  An odd last block is loaded twice and the second copy's
// scores are -inf, so its P is exactly 0 and it adds nothing.
//
// TMEM (512 columns): O_t at [t*D, (t+1)*D); S_t at 2D + 128t (128 fp32
// columns).  P_t (128 16-bit values per row = 64 columns) is written over the
// first 64 columns of S_t after the softmax has read them, in two halves (the
// keys of the pair's first and second block), each announced on its own
// barrier so PV over the first 64 keys runs while the second half is still
// being exponentiated.  One thread issues all MMAs in the order QK_0(j),
// PV_1(j-1), QK_1(j), PV_0(j), ...; MMAs of a thread execute in issue order,
// so QK_t(j+1) overwrites P_t(j) only after PV_t(j) has read it, and the lazy
// O rescale of softmax_t(j+1) (which starts after QK_t(j+1) completes and is
// done before the first half of P_t(j+1) is announced) never races PV_t(j) or
// PV_t(j+1).  The two tiles ping-pong: while one tile's softmax runs, the
// tensor core executes the other tile's MMAs.  Issuing an MMA blocks its
// thread for about its execution time, so the tensor core idles whenever the
// issuer waits for P: the softmax time is what sets the pace.
//
// Softmax per step and row (thread = row = TMEM lane): the 128 scores are
// loaded into registers at once, masked (only on a diagonal or odd last pair),
// reduced to the row max with 3-input max, scaled and shifted with packed
// f32x2 FMAs, exponentiated (an eighth by the polynomial on the FMA pipe, the
// rest on MUFU), summed with packed adds and stored as 64 packed P columns,
// 16 at a time.  O is rescaled only when the running max grows by more than 8
// (log2 units).
//
// Residual summaries (SUM = true, sparse/attention.py:164-265): after its
// selected blocks, a row takes its virtual blocks -- 64 gathered summary keys
// each, read through a second pair of tensor maps -- as ordinary block slots
// with ids kVirtualBase + i*nvb + j.  The producer stages each virtual half's
// 64 count biases (natural log, times log2(e)) in shared memory before it
// releases the stage's K barrier.  A pair with a virtual half moves all its
// scores into log2 units first (scale*log2(e)*s, plus the bias where virtual;
// no causal mask there), so the one online softmax covers blocks and
// summaries exactly as the reference's concatenated scores.
//
// Warp roles (320 threads):
//   warps 0-3  softmax + epilogue of tile 0 (TMEM lanes 0-127); warps 4-7 tile 1
//   warp  8    TMA producer (Q once, then K/V of each block pair, STAGES ring)
//   warp  9    TMEM allocator + issuer of every MMA (QK^T and PV, interleaved)
// Every wait is bounded (see common.cuh): a timeout raises
// SPRUCE_STATUS_TIMEOUT and a shared abort flag, and every role still drains
// its own copies / MMAs before TMEM is released.
#include <algorithm>

#include "attn_common.cuh"

namespace spruce {

constexpr int kPairThreads = 320;
constexpr int kPairProducer = 8;
constexpr int kPairQk = 9;  // MMA issuer, owns the TMEM allocation

template <int D, int STAGES>
struct PairLayout {
  static constexpr int NP = D / 64;          // 128-byte panels along the head dim
  static constexpr int Q_PANEL = 128 * 128;  // 128 rows x 128 B
  static constexpr int KV_PANEL = 128 * 128; // 128 tokens x 128 B
  static constexpr int HALF = 64 * 128;      // one block's 64 tokens in a panel
  static constexpr int Q_TILE = NP * Q_PANEL;
  static constexpr int KV_TILE = NP * KV_PANEL;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * Q_TILE;
  static constexpr int OFF_V = OFF_K + STAGES * KV_TILE;
  static constexpr int OFF_BAR = OFF_V + STAGES * KV_TILE;
  // q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2][2], o_done[2], drain[2]
  static constexpr int NBAR = 1 + 3 * STAGES + 2 + 4 + 2 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_VB = (OFF_MISC + 16 + 15) / 16 * 16;  // [STAGES][128] fp32 virtual-key biases
  static constexpr int OFF_IDS = OFF_VB + STAGES * 128 * 4;
  static constexpr int COL_S = 2 * D;  // S_t (and P_t) at COL_S + 128 t
  static constexpr uint32_t TMEM_COLS = 512u;
  static_assert(2 * D + 256 <= 512, "O and S of both tiles must fit in 512 TMEM columns");
  static size_t smem_bytes(int kw) { return 1024 + OFF_IDS + 4 * (size_t)kw; }
};

template <typename T, int D, int STAGES, bool SUM>
__global__ void __launch_bounds__(kPairThreads, 1)
    attn_pair_sm100_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmvk,
                           const __grid_constant__ CUtensorMap tmvv, const __grid_constant__ OutMaps om,
                           const AttnParams p) {
  using L = PairLayout<D, STAGES>;
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
  uint64_t* s_full = kv_empty + STAGES;  // [tile]: S_t(j) written
  uint64_t* p_full = s_full + 2;         // [tile * 2 + half]: that half of P_t(j) written (128 arrivals)
  uint64_t* o_done = p_full + 4;         // [tile]: PV_t(j) complete
  uint64_t* drain = o_done + 2;          // [issuer warp]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  int* nsel_slot = reinterpret_cast<int*>(smem + L::OFF_MISC + 8);
  int* ids = reinterpret_cast<int*>(smem + L::OFF_IDS);

  // ---- setup: compact the row's block ids, init barriers, allocate TMEM
  if (warp == kPairProducer) {
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
    if constexpr (SUM) {  // then the row's virtual summary blocks
      const int vc = min(p.vcount[((int64_t)b * p.Hkv + g) * p.qb + i], p.nvb);
      for (int j = lane; j < vc; j += 32) ids[count + j] = kVirtualBase + i * p.nvb + j;
      count += vc;
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
        mbar_init(&p_full[2 * t], 128);
        mbar_init(&p_full[2 * t + 1], 128);
        mbar_init(&o_done[t], 1);
      }
      mbar_init(&drain[0], 1);
      mbar_init(&drain[1], 1);
      fence_barrier_init();
      prefetch_tmap(&tmq);
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
    }
    __syncwarp();
  } else if (warp == kPairQk) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n = *nsel_slot;
  const int np = (n + 1) / 2;  // block pairs; an odd last block is paired with itself

  if (warp == kPairProducer) {
    // ------------------------------------------------------------ TMA producer
    if (np > 0) {
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
      for (int j = 0; j < np; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES &&
            !__all_sync(0xffffffffu, mbar_wait(&kv_empty[st], ((j / STAGES) - 1) & 1, p.status, abort_flag)))
          break;
        if constexpr (SUM) {
          // Virtual halves' biases into this stage (released with k_full below).
          float* vb = reinterpret_cast<float*>(smem + L::OFF_VB) + st * 128;
          for (int h = 0; h < 2; ++h) {
            const int id = ids[min(2 * j + h, n - 1)];
            if (id >= kVirtualBase) {
              const float* src = p.vbias + ((int64_t)b * p.Hkv + g) * p.Tv + (int64_t)(id - kVirtualBase) * 64;
              vb[h * 64 + lane] = src[lane] * 1.4426950408889634f;
              vb[h * 64 + 32 + lane] = src[32 + lane] * 1.4426950408889634f;
            }
          }
          __syncwarp();
        }
        if (leader) {
          uint8_t* ks = smem + L::OFF_K + st * L::KV_TILE;
          uint8_t* vs = smem + L::OFF_V + st * L::KV_TILE;
          mbar_arrive_expect_tx(&k_full[st], L::KV_TILE);
          mbar_arrive_expect_tx(&v_full[st], L::KV_TILE);
          for (int h = 0; h < 2; ++h) {
            const int id = ids[min(2 * j + h, n - 1)];
            const bool virt = SUM && id >= kVirtualBase;
            const int tok = (virt ? id - kVirtualBase : id) * 64;
            const CUtensorMap* mk = virt ? &tmvk : &tmk;
            const CUtensorMap* mv = virt ? &tmvv : &tmv;
            for (int pp = 0; pp < L::NP; ++pp)
              tma_load_4d(ks + pp * L::KV_PANEL + h * L::HALF, mk, &k_full[st], pp * 64, g, tok, b);
            for (int pp = 0; pp < L::NP; ++pp)
              tma_load_4d(vs + pp * L::KV_PANEL + h * L::HALF, mv, &v_full[st], pp * 64, g, tok, b);
          }
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
  } else if (warp == kPairQk) {
    // ------------------------------------------------------------ MMA issuers
    if (np > 0) {
      const bool leader = elect_one();
      constexpr uint32_t fmt = UmmaFormat<T>::value;
      constexpr uint32_t idesc_qk = idesc_f16(fmt, 0, 0, 128, 128);
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
      auto issue_qk = [&](int t, int st) {
        // S_t = Q_t . K^T over D in steps of 16 (32 bytes inside a 128-byte swizzle row).
        const uint32_t d = tmem + L::COL_S + 128 * t;
        const uint64_t qa = dq0 + (uint64_t)((t * L::Q_TILE) >> 4);
        const uint64_t kb = dk0 + (uint64_t)((st * L::KV_TILE) >> 4);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t offq = ((ks >> 2) * L::Q_PANEL + (ks & 3) * 32) >> 4;
          const uint32_t offk = ((ks >> 2) * L::KV_PANEL + (ks & 3) * 32) >> 4;
          if (leader) umma_f16_ss(d, qa + offq, kb + offk, idesc_qk, ks > 0 ? 1u : 0u);
          __syncwarp();
        }
        commit(&s_full[t]);
      };
      auto issue_pv_half = [&](int t, int st, int h, bool accumulate) {
        // O_t += P_t . V over keys 64h..64h+63 in steps of 16 keys (8 TMEM columns of P, 2048 bytes of V).
        const uint32_t a = tmem + L::COL_S + 128 * t;
        const uint64_t vb = dv0 + (uint64_t)((st * L::KV_TILE) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int ks = 4 * h + kk;
          if (leader)
            umma_f16_ts(tmem + t * D, a + ks * 8, vb + (uint64_t)((ks * 2048) >> 4), idesc_pv,
                        (accumulate || ks > 0) ? 1u : 0u);
          __syncwarp();
        }
        if (h == 1) commit(&o_done[t]);
      };
      auto pv = [&](int t, int st, int jj) {  // both halves of PV_t(jj), each once its P half is written
        for (int h = 0; h < 2; ++h) {
          if (!wait(&p_full[2 * t + h], jj & 1)) return false;
          tc_fence_after();
          issue_pv_half(t, st, h, jj > 0);
        }
        return true;
      };
      if (warp == kPairQk) {
        // One thread issues every MMA, interleaving the tiles:
        //   QK_0(j) ; PV_1(j-1) ; QK_1(j) ; PV_0(j) ; QK_0(j+1) ; PV_1(j) ; ...
        // tcgen05.mma operations of one thread execute in issue order, so
        // QK_t(j+1) overwrites S_t (= P_t(j)) only after PV_t(j) has read it,
        // and the commit behind QK_t(j+1) also covers PV_t(j): once the
        // softmax sees S_t(j+1), O_t holds PV_t(j) and nothing writes it until
        // PV_t(j+1), which waits for the softmax.
        bool ok = wait(q_full, 0);
        for (int j = 0; ok && j <= np; ++j) {
          const int st = j % STAGES;
          const int sp = (j + STAGES - 1) % STAGES;  // stage of pair j - 1
          if (j < np) {
            if (!wait(&k_full[st], (j / STAGES) & 1)) break;
            tc_fence_after();
            issue_qk(0, st);
          }
          if (j > 0 && n_tiles > 1) {
            if (!pv(1, sp, j - 1)) break;
          }
          if (j > 0) commit(&kv_empty[sp]);  // every MMA reading pair j-1's stage is issued before this
          if (j == np) break;
          if (n_tiles > 1) issue_qk(1, st);
          if (!wait(&v_full[st], (j / STAGES) & 1) || !pv(0, st, j)) break;
        }
        commit(&drain[0]);  // no MMA may be in flight when TMEM is released
        mbar_wait(&drain[0], 0, p.status, nullptr);
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
      const uint32_t tS = tmem + lane_off + L::COL_S + 128 * t;
      for (int j = 0; j < np; ++j) {
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, p.status, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const bool dup1 = 2 * j + 1 >= n;  // odd last block: its repeat (columns 64-127) is masked
        const bool diag0 = ids[2 * j] == i;
        const bool diag1 = !dup1 && ids[2 * j + 1] == i;
        // All 128 scores of the row in registers (one TMEM round trip).
        float s[4][32];  // s[q][c] = column 32q + c
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(tS + 32 * q, s[q]);
        tmem_wait_ld();
        // A pair with a virtual (summary) half: every score to log2 units now,
        // plus the count bias on the virtual half; the scaling below is then 1.
        float sl = sl2;
        if constexpr (SUM) {
          const bool v0 = ids[2 * j] >= kVirtualBase;
          const bool v1 = !dup1 && ids[2 * j + 1] >= kVirtualBase;
          if (v0 || v1) {  // warp-uniform
            // the producer's bias stores are visible once this stage's K phase has completed
            ok = __all_sync(0xffffffffu, mbar_wait(&k_full[j % STAGES], (j / STAGES) & 1, p.status, abort_flag));
            if (!ok) break;
            const float* vb = reinterpret_cast<const float*>(smem + L::OFF_VB) + (j % STAGES) * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (q < 2 ? v0 : v1) {
#pragma unroll
                for (int c4 = 0; c4 < 8; ++c4) {
                  const float4 w = *reinterpret_cast<const float4*>(vb + 32 * q + 4 * c4);
                  s[q][4 * c4 + 0] = fmaf(s[q][4 * c4 + 0], sl2, w.x);
                  s[q][4 * c4 + 1] = fmaf(s[q][4 * c4 + 1], sl2, w.y);
                  s[q][4 * c4 + 2] = fmaf(s[q][4 * c4 + 2], sl2, w.z);
                  s[q][4 * c4 + 3] = fmaf(s[q][4 * c4 + 3], sl2, w.w);
                }
              } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) s[q][c] *= sl2;
              }
            }
            sl = 1.0f;
          }
        }
        // The reference's masks: the diagonal block keeps keys <= the row's token,
        // the repeated odd block none.
        if (dup1 || diag0 || diag1) {  // warp-uniform: only the diagonal pair and an odd last pair
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const bool dup = q >= 2 && dup1;
            const bool diag = q < 2 ? diag0 : diag1;
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (dup || (diag && (q & 1) * 32 + c > tok)) s[q][c] = -INFINITY;
          }
        }
        // Row max: 8 independent chains of 3-input max (exact in any order).
        float mx8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float a = fmax3(s[0][u], s[0][u + 8], s[0][u + 16]);
          a = fmax3(a, s[0][u + 24], s[1][u]);
          a = fmax3(a, s[1][u + 8], s[1][u + 16]);
          a = fmax3(a, s[1][u + 24], s[2][u]);
          a = fmax3(a, s[2][u + 8], s[2][u + 16]);
          a = fmax3(a, s[2][u + 24], s[3][u]);
          a = fmax3(a, s[3][u + 8], s[3][u + 16]);
          mx8[u] = fmaxf(a, s[3][u + 24]);
        }
        const float mx = fmaxf(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], fmax3(mx8[5], mx8[6], mx8[7])));
        const float m_new = fmaxf(m_used, mx * sl);
        const bool rescale = (j == 0) || (m_new > m_used + 8.0f);
        const float alpha = (j > 0 && rescale) ? fast_exp2(m_used - m_new) : 1.0f;
        if (rescale) m_used = m_new;
        const float neg_ref = (m_used == -INFINITY) ? 0.0f : -m_used;
        // Exponentials -> P over S_t's first 64 columns, 16 columns per store.
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        uint64_t sum2[2] = {f2_pack(0.0f, 0.0f), f2_pack(0.0f, 0.0f)};
        const uint64_t sl2x2 = f2_pack(sl, sl), nref2 = f2_pack(neg_ref, neg_ref);
        const bool any_diag = diag0 || diag1;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pk[16];
          if (!any_diag) {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              float x0, x1, e0, e1;
              f2_unpack(f2_fma(f2_pack(s[q][2 * k], s[q][2 * k + 1]), sl2x2, nref2), x0, x1);
              if ((k & 7) == 7) {
                poly_exp2_x2(x0, x1, e0, e1);
              } else {
                e0 = fast_exp2(x0);
                e1 = fast_exp2(x1);
              }
              sum2[k & 1] = f2_add(sum2[k & 1], f2_pack(e0, e1));
              pk[k] = Pack2<T>::pack(e0, e1);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(s[q][2 * k], s[q][2 * k + 1]), sl2x2, nref2), x0, x1);
              const float e0 = fast_exp2(x0);
              const float e1 = fast_exp2(x1);
              sum2[k & 1] = f2_add(sum2[k & 1], f2_pack(e0, e1));
              pk[k] = Pack2<T>::pack(e0, e1);
            }
          }
          tmem_st16u(tS + 16 * q, pk);
          if (q == 1) {
            // First half of P written: rescale O (PV_t(j-1) is complete, PV_t(j) not
            // yet issued), then let the issuer start PV over these 64 keys.
            if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
              for (int cc = 0; cc < D / 32; ++cc) {
                float o[32];
                tmem_ld32(tO + cc * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] *= alpha;
                tmem_st32(tO + cc * 32, o);
              }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[2 * t]);
          }
        }
        f2_unpack(sum2[0], part[0], part[1]);
        f2_unpack(sum2[1], part[2], part[3]);
        l = l * alpha + ((part[0] + part[1]) + (part[2] + part[3]));
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[2 * t + 1]);
      }
      if (ok && np > 0)  // PV_t(np-1) complete (and with it every earlier PV into O_t)
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[t], (np - 1) & 1, p.status, abort_flag));
      tc_fence_after();
      // Epilogue: O / l -> T staged in this tile's Q region (every QK MMA is complete
      // once PV(np-1) is), laid out [panel][head][token][128 B] with the 128-byte
      // swizzle, then TMA tensor stores to this GPU's output and to each peer's.
      uint8_t* stage = smem + L::OFF_Q + t * L::Q_TILE;
      const int hsub = row & 1;
      const int srow = hsub * 64 + tok;  // staging row: head-major
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      if (n == 0 && row == 0) raise_status(p.status, SPRUCE_STATUS_EMPTY_ROW);
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        if (ok && np > 0) {
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
  if (warp == kPairQk) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <typename T, int D, int STAGES>
static cudaError_t launch_pair_typed(const AttnArgs& a, CUtensorMapDataType dt, cudaStream_t stream) {
  using L = PairLayout<D, STAGES>;
  CUtensorMap tmq, tmk, tmv, tmvk, tmvv;
  if (!make_map(&tmq, a.q, dt, a.B, a.Hq, a.T, D, a.qs, 2) || !make_map(&tmk, a.k, dt, a.B, a.Hkv, a.T, D, a.ks, 1) ||
      !make_map(&tmv, a.v, dt, a.B, a.Hkv, a.T, D, a.vs, 1))
    return cudaErrorInvalidValue;
  const bool sum = a.vk != nullptr;
  if (sum) {
    if (!make_map(&tmvk, a.vk, dt, a.B, a.Hkv, a.Tv, D, a.vks, 1) ||
        !make_map(&tmvv, a.vv, dt, a.B, a.Hkv, a.Tv, D, a.vvs, 1))
      return cudaErrorInvalidValue;
  } else {
    tmvk = tmk;
    tmvv = tmv;
  }
  const AttnParams p = attn_params(a);
  OutMaps om;
  if (!attn_out_maps(a, dt, D, &om)) return cudaErrorInvalidValue;
  const size_t smem = L::smem_bytes(a.Kw + (sum ? a.nvb : 0));
  auto kern = sum ? attn_pair_sm100_kernel<T, D, STAGES, true> : attn_pair_sm100_kernel<T, D, STAGES, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (p.nq <= 0) return cudaSuccess;
  dim3 grid(p.nq * p.n_cta, a.Hkv, a.B);
  kern<<<grid, kPairThreads, smem, stream>>>(tmq, tmk, tmv, tmvk, tmvv, om, p);
  return cudaGetLastError();
}

// Self-check of the softmax's two exponentials: poly[i] = poly_exp2_x2 (FMA pipe, as the
// pair kernel evaluates it), mufu[i] = ex2.approx.ftz (MUFU), both over x[i].
__global__ void exp2_probe_kernel(const float* x, float* poly, float* mufu, int64_t n) {
  const int64_t i = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i], x1 = i + 1 < n ? x[i + 1] : 0.0f;
  float e0, e1;
  poly_exp2_x2(x0, x1, e0, e1);
  poly[i] = e0;
  mufu[i] = fast_exp2(x0);
  if (i + 1 < n) {
    poly[i + 1] = e1;
    mufu[i + 1] = fast_exp2(x1);
  }
}

cudaError_t launch_exp2_probe(const float* x, float* poly, float* mufu, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const int64_t pairs = (n + 1) / 2;
  exp2_probe_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, stream>>>(x, poly, mufu, n);
  return cudaGetLastError();
}

constexpr size_t kPairMaxSmem = 227 * 1024;

int attn_pair_max_kw(int D) {
  const size_t base = D == 128 ? PairLayout<128, 2>::smem_bytes(0) : PairLayout<64, 4>::smem_bytes(0);
  return static_cast<int>((kPairMaxSmem - base) / 4);
}

cudaError_t launch_attn_pair(const AttnArgs& a, int dtype, cudaStream_t stream) {
  if (a.Kw + (a.vk != nullptr ? a.nvb : 0) > attn_pair_max_kw(a.D)) return cudaErrorInvalidValue;
  if (dtype == SPRUCE_DTYPE_BF16) {
    if (a.D == 128) return launch_pair_typed<__nv_bfloat16, 128, 2>(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
    if (a.D == 64) return launch_pair_typed<__nv_bfloat16, 64, 4>(a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, stream);
  } else if (dtype == SPRUCE_DTYPE_F16) {
    if (a.D == 128) return launch_pair_typed<__half, 128, 2>(a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
    if (a.D == 64) return launch_pair_typed<__half, 64, 4>(a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace spruce
