"""Generate the golden vectors under tests/golden/ by running the REFERENCE.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/spruce-research

It imports the reference's own torch functions -- _group_avg_tokens,
_proto_pool_seq, FlatGate, selected_ids_to_blocks, validate_selected_blocks,
sparse_prefill_attention_forward, build_kv_summary_table,
build_residual_tree_layout, build_residual_summary_nodes,
residual_attention_density -- feeds them the seeded synthetic inputs of
spruce_research_b200.synthetic and stores their outputs as .npz fixtures.
The tests regenerate the inputs from the stored seeds (checked against the
stored input checksums) and compare the oracle and the CUDA path with the
stored outputs.  Nothing at test time reads the reference checkout.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from spruce_research_b200.synthetic import LayerShape, k_for_density, make_gate_weights, make_layer_inputs  # noqa: E402

# name: (shape, dtype, seed, rope, K (None = 10% density), local_window, sink, stored query blocks)
CASES = {
    # 4/2 heads, d=64, 4096 tokens, fp32, top-8 with sink + diagonal.
    "c0": (LayerShape(1, 4, 2, 4096, 64), torch.float32, 0, None, 8, 0, 1, (0, 1, 2, 17, 40, 63)),
    # config-1 shape (28/4 heads, d=128, bf16, RoPE 1e6) at 2048 tokens, K=8.
    "c1_small": (LayerShape(1, 28, 4, 2048, 128), torch.bfloat16, 1, 1e6, 8, 0, 1, (0, 1, 9, 31)),
    # config-1 shape at 8192 tokens and 10% density (K=7): index parity.
    "c1_8k": (LayerShape(1, 28, 4, 8192, 128), torch.bfloat16, 5, 1e6, None, 0, 1, (127,)),
    # ragged tail (357 tokens), general local window and sink.
    "ragged_bf16": (LayerShape(1, 4, 2, 357, 64), torch.bfloat16, 2, 1e6, 4, 1, 1, None),
    # fp16, 7:1 GQA, no sink.
    "gqa_fp16": (LayerShape(1, 14, 2, 320, 128), torch.float16, 3, 1e6, 3, 1, 0, (0, 4)),
    # batch 2, fp32, d=128.
    "batch2_f32": (LayerShape(2, 4, 1, 256, 128), torch.float32, 4, 1e6, 3, 0, 1, (0, 3)),
}


# The headline configurations in full.  name: (shape, dtype, input seed, gate-weight seed, rope,
# K (None = 10% charged density), local_window, sink, sampled query blocks of the stored attention)
BIG_CASES = {
    # 32768 tokens, 10% density (K = 27).
    "c1_full": (LayerShape(1, 28, 4, 32768, 128), torch.bfloat16, 21, 22, 1e6, None, 0, 1, (0, 1, 256, 510, 511)),
    # 131072 tokens, 10% density (K = 106), with bench.py's default inputs
    # (input seed 0, gate seed 1), so the bench can check its own step against these outputs.
    "c2": (LayerShape(1, 28, 4, 131072, 128), torch.bfloat16, 0, 1, 1e6, None, 0, 1, (0, 1, 1024, 2046, 2047)),
}


def _raw(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy()
    return t.numpy()


class _Module(torch.nn.Module):
    def __init__(self, layer_idx=0):
        super().__init__()
        self.layer_idx = layer_idx


def reference_pipeline(ref, q, k, v, wq, wk, K, local_window, sink):
    """The flat-gate selector + sparse attention, composed from reference functions."""
    B, Hq, T, d = q.shape
    Hkv = k.shape[1]
    qg = ref["group_avg"](q, Hkv)
    pooled_q = ref["proto_pool"](qg, 64, 1)                       # [B, G, qb, 1, d]
    pooled_k = ref["proto_pool"](k, 64, 1)
    qb = pooled_q.shape[2]
    gate = ref["FlatGate"](1, d, d).eval()
    with torch.no_grad():
        gate.Wq.copy_(wq)
        gate.Wk.copy_(wk)
    scores, selected = [], []
    for b in range(B):
        with torch.no_grad():
            s = gate(pooled_q[b].float().unsqueeze(0), pooled_k[b].float().unsqueeze(0))  # [1,G,qb,kb]
        qi = torch.arange(qb)[:, None]
        kj = torch.arange(qb)[None, :]
        forced_or_future = (kj > qi) | (kj >= qi - local_window) | ((kj < sink) & (kj < qi - local_window))
        masked = s.masked_fill(forced_or_future[None, None], torch.finfo(torch.float32).min)
        width = min(K - (local_window + 1) - sink, qb)
        ids = masked.topk(width, dim=-1).indices
        sel = ref["pack"](ids, k_selected=K, local_window=local_window, key_blocks=qb, sink_blocks=sink)
        ref["validate"](sel, local_window=local_window)
        scores.append(s[0])
        selected.append(sel[0, 0])
    selected_blocks = torch.stack(selected)[:, None]                 # [B, 1, G, qb, K]
    out, _ = ref["attention"](_Module(), q, k, v, None, selected_blocks=selected_blocks,
                              block_size=64, validate_selected_blocks_input=False)
    return {
        "pooled_q": pooled_q[:, :, :, 0], "pooled_k": pooled_k[:, :, :, 0],
        "scores": torch.stack(scores), "selected": selected_blocks[:, 0], "out": out,
    }


def big_case(ref, name):
    """One headline configuration in full, through the reference's own functions.

    The gate runs one KV group at a time (the reference's scores are elementwise per
    (group, query block, key block), so this changes no bit and bounds host memory).
    Stored: the whole selected_blocks (int16: ids < 2^15), the score gap at each row's
    selection boundary (the W-th minus the (W+1)-th largest candidate score, +inf when
    the row has no (W+1)-th candidate), SHA-256 digests of the pooled features, and the
    attention output of a few sampled query blocks.
    """
    import hashlib
    import time

    shape, dtype, seed, wseed, rope, K, lw, sink, keep = BIG_CASES[name]
    q, k, v = make_layer_inputs(shape, dtype, seed, rope_theta=rope)
    t0 = time.perf_counter()
    wq, wk = make_gate_weights(1, shape.head_dim, shape.head_dim, wseed)
    qb = shape.query_blocks
    if K is None:
        K = k_for_density(qb, 0.10)
    B, G = shape.batch, shape.kv_heads
    pooled_q = ref["proto_pool"](ref["group_avg"](q, G), 64, 1)        # [B, G, qb, 1, d]
    pooled_k = ref["proto_pool"](k, 64, 1)
    gate = ref["FlatGate"](1, shape.head_dim, shape.head_dim).eval()
    with torch.no_grad():
        gate.Wq.copy_(wq)
        gate.Wk.copy_(wk)
    qi = torch.arange(qb)[:, None]
    kj = torch.arange(qb)[None, :]
    forced_or_future = (kj > qi) | (kj >= qi - lw) | ((kj < sink) & (kj < qi - lw))
    width = min(K - (lw + 1) - sink, qb)
    selected = torch.empty((B, G, qb, K), dtype=torch.int32)
    gap = torch.full((B, G, qb), float("inf"), dtype=torch.float32)
    floor = torch.finfo(torch.float32).min
    t_gap = 0.0
    for b in range(B):
        for g in range(G):
            with torch.no_grad():
                s = gate(pooled_q[b, g:g + 1].float().unsqueeze(0), pooled_k[b, g:g + 1].float().unsqueeze(0))
            masked = s.masked_fill(forced_or_future[None, None], floor)    # [1, 1, qb, kb]
            ids = masked.topk(width, dim=-1).indices
            sel = ref["pack"](ids, k_selected=K, local_window=lw, key_blocks=qb, sink_blocks=sink)
            ref["validate"](sel, local_window=lw)
            selected[b, g] = sel[0, 0, 0]
            tg = time.perf_counter()  # the gap bookkeeping is not part of the reference's path
            top = masked[0, 0].topk(min(width + 1, qb), dim=-1).values     # [qb, width + 1]
            if top.shape[-1] > width:
                real = top[:, width] > floor
                gap[b, g, real] = (top[real, width - 1] - top[real, width])
            t_gap += time.perf_counter() - tg
            del s, masked
    t_sel = time.perf_counter() - t0 - t_gap
    t1 = time.perf_counter()
    out, _ = ref["attention"](_Module(), q, k, v, None, selected_blocks=selected[:, None].contiguous(),
                              block_size=64, validate_selected_blocks_input=False)
    t_attn = time.perf_counter() - t1
    rows = torch.cat([torch.arange(i * 64, min((i + 1) * 64, shape.tokens)) for i in keep])
    digest = {}
    for key, t in (("pooled_q", pooled_q), ("pooled_k", pooled_k)):
        digest[key] = np.frombuffer(hashlib.sha256(_raw(t).tobytes()).digest(), dtype=np.uint8)
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        shape=np.array([shape.batch, shape.q_heads, shape.kv_heads, shape.tokens, shape.head_dim]),
        dtype=np.array([{torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dtype]]),
        seed=np.array([seed]), wseed=np.array([wseed]), rope=np.array([rope if rope is not None else 0.0]),
        policy=np.array([K, lw, sink]),
        checksum=np.array([q.double().sum().item(), k.double().sum().item(), v.double().sum().item()]),
        pooled_q_sha256=digest["pooled_q"], pooled_k_sha256=digest["pooled_k"],
        selected=selected.to(torch.int16).numpy(), gap=gap.numpy(),
        out=_raw(out[:, rows]), out_blocks=np.array(keep, dtype=np.int64),
        # Wall time of the reference's own CPU path on the host that made this fixture:
        # [selector s (pooling, gate, mask / top-k, packing; all KV groups), attention s, torch threads,
        #  os.cpu_count()].  Measured once, inputs already in memory.
        ref_cpu=np.array([t_sel, t_attn, torch.get_num_threads(), os.cpu_count() or 0], dtype=np.float64),
    )
    print(f"{name}: K={K} selector {t_sel:.1f} s, attention {t_attn:.1f} s; "
          f"smallest boundary gap {gap.min().item():.3e}, rows with gap < 1e-6: {(gap < 1e-6).sum().item()}")


# Trained gate weights: the reference's checkpoint (selector_ckpt/<file>, {state_dict, config}),
# loaded through this repository's load_gate; one gate layer's Wq/Wk are stored.
TRAINED = ("flat_gate_trained.pt", 13)


def trained_case(ref, reference_root):
    """The reference's flat (P = 1) and tree (P = 8, beam 16) selectors with trained weights.

    Inputs: the config-1 layer shape at 8192 tokens (seed 41).  P = 1: pooled means,
    FlatGate scores, mask / top-k at 10% density, selected_ids_to_blocks.  P = 8: outlier
    prototypes of the group-averaged queries and of the keys in fp32, build_key_tree
    (radix 2) and traverse_to_leaf_ids (beam 16).
    """
    from spruce_research_b200.selector.gate import load_gate

    ours, cfg = load_gate(os.path.join(reference_root, "selector_ckpt", TRAINED[0]), "cpu")
    layer = TRAINED[1]
    wq, wk = ours.Wq[layer].detach().clone(), ours.Wk[layer].detach().clone()
    shape, seed = LayerShape(1, 28, 4, 8192, 128), 41
    q, k, v = make_layer_inputs(shape, torch.bfloat16, seed, rope_theta=1e6)
    K = k_for_density(shape.query_blocks, 0.10)
    flat = reference_pipeline(ref, q, k, v, wq, wk, K, 0, 1)
    q_feat = ref["proto_pool"](ref["group_avg"](q, shape.kv_heads), 64, 8).float()   # [1, G, qb, 8, d]
    k_feat = ref["proto_pool"](k, 64, 8).float()
    gate = ref["FlatGate"](1, shape.head_dim, shape.head_dim).eval()
    with torch.no_grad():
        gate.Wq.copy_(wq[None])
        gate.Wk.copy_(wk[None])
        levels = ref["build_key_tree"](k_feat, radix=2)
        leaf_ids = ref["traverse"](gate, q_feat, levels, 16, radix=2)
    np.savez_compressed(
        os.path.join(HERE, "trained.npz"),
        checkpoint=np.array([TRAINED[0]]), layer=np.array([layer]),
        config=np.array([cfg["num_layers"], cfg["head_dim"], cfg["proj_dim"]]),
        wq=wq.numpy(), wk=wk.numpy(),
        shape=np.array([shape.batch, shape.q_heads, shape.kv_heads, shape.tokens, shape.head_dim]),
        seed=np.array([seed]), policy=np.array([K, 0, 1]),
        checksum=np.array([q.double().sum().item(), k.double().sum().item(), v.double().sum().item()]),
        selected=flat["selected"].numpy(), leaf_ids=leaf_ids.numpy(),
    )
    print(f"trained: {TRAINED[0]} layer {layer}, P=1 selected {tuple(flat['selected'].shape)}, "
          f"P=8 leaf ids {tuple(leaf_ids.shape)}")


# The whole model at sparse density: a tiny random Qwen2 (tests/golden_cases.py LIVE_MODEL) run
# with the reference's own torch attention backend on fixed routes at ~10% density.
LIVE = dict(model_seed=11, ids_seed=3, tokens=64 * 64 + 17, routes_seed=17)


def live_case(reference_root):
    """Logits of the last token, the final hidden states and every layer's output at sampled
    token rows, from the reference's registered backend (sparse/attention.py:277-291,
    sparse_prefill_attention_forward) in a transformers Qwen2 given selected_blocks."""
    sys.path.insert(0, os.path.join(REPO, "tests"))
    from golden_cases import LIVE_MODEL, live_rows, model_checksum, tiny_qwen2
    from scripts.export_selected_blocks import selected_ids_to_blocks
    from interfaces.validator import validate_selected_blocks
    from sparse.attention import register_sparse_prefill_attention

    T = LIVE["tokens"]
    model = tiny_qwen2(LIVE["model_seed"])
    ids = torch.randint(0, LIVE_MODEL["vocab_size"], (1, T), generator=torch.Generator().manual_seed(LIVE["ids_seed"]))
    L, G = LIVE_MODEL["num_hidden_layers"], LIVE_MODEL["num_key_value_heads"]
    qb = (T + 63) // 64
    K = k_for_density(qb, 0.10)
    cand = torch.randint(0, qb, (L, G, qb, K), generator=torch.Generator().manual_seed(LIVE["routes_seed"]))
    routes = selected_ids_to_blocks(cand, K, local_window=0, key_blocks=qb, sink_blocks=1)   # [1, L, G, qb, K]
    validate_selected_blocks(routes, local_window=0)
    model.set_attn_implementation(register_sparse_prefill_attention())
    with torch.no_grad():
        out = model.base_model(ids, use_cache=False, selected_blocks=routes, block_size=64,
                               validate_selected_blocks_input=False, output_hidden_states=True)
        final = out.last_hidden_state
        logits = model.get_output_embeddings()(final[:, -1:, :])
    rows = live_rows(T)
    layers = torch.stack([h[0, rows] for h in out.hidden_states[1:L]])   # outputs of layers 0 .. L-2
    density = float((routes >= 0).sum()) / (L * G * qb * (qb + 1) / 2)
    np.savez_compressed(
        os.path.join(HERE, "live.npz"),
        seeds=np.array([LIVE["model_seed"], LIVE["ids_seed"], LIVE["routes_seed"]]), tokens=np.array([T]),
        model_checksum=np.array([model_checksum(model)]), routes=routes.to(torch.int16).numpy(),
        logits=logits[0, 0].float().numpy(), final_rows=_raw(final[0, rows]), layer_rows=_raw(layers),
    )
    print(f"live: T={T}, K={K}, charged density {density:.3f}, logits {tuple(logits.shape)}")


def packing_cases(ref):
    gen = torch.Generator().manual_seed(11)
    cases = {}
    for n, (K, lw, sink, C, qb, kb) in enumerate(
            [(5, 1, 0, 6, 40, 40), (6, 1, 1, 9, 40, 40), (4, 0, 2, 12, 33, 33),
             (8, 2, 1, 5, 17, 20), (3, 0, 0, 4, 9, 9), (12, 1, 1, 30, 25, 25)]):
        ids = torch.randint(-3, kb + 4, (2, 2, qb, C), generator=gen)
        out = ref["pack"](ids, k_selected=K, local_window=lw, key_blocks=kb, sink_blocks=sink)
        cases[f"pack{n}_ids"] = ids.numpy()
        cases[f"pack{n}_args"] = np.array([K, lw, kb, sink], dtype=np.int64)
        cases[f"pack{n}_out"] = out.numpy()
    return cases


def proto_cases(ref):
    gen = torch.Generator().manual_seed(12)
    cases = {}
    for n, (H, T, d, dt) in enumerate([(2, 200, 64, torch.bfloat16), (1, 64 * 3 + 5, 128, torch.float32),
                                       (2, 128, 128, torch.float16)]):
        x = torch.randn((1, H, T, d), generator=gen).to(dt)
        cases[f"proto{n}_x"] = _raw(x)
        cases[f"proto{n}_dtype"] = np.array([{torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dt]])
        cases[f"proto{n}_p8"] = _raw(ref["proto_pool"](x, 64, 8))
        cases[f"proto{n}_p1"] = _raw(ref["proto_pool"](x, 64, 1))
    return cases


# name: (shape, dtype, seed, rope, block_size, prototypes, mask kind, stored nodes (None = all))
SUMMARY_CASES = {
    "sum_ragged_bf16": (LayerShape(1, 4, 2, 357, 64), torch.bfloat16, 2, 1e6, 64, 4, None, None),
    "sum_batch2_f32": (LayerShape(2, 4, 1, 256, 128), torch.float32, 4, 1e6, 64, 2, "holes", None),
    "sum_c0_f32": (LayerShape(1, 4, 2, 4096, 64), torch.float32, 0, None, 64, 1, None, None),
    "sum_c1_8k_bf16": (LayerShape(1, 28, 4, 8192, 128), torch.bfloat16, 5, 1e6, 64, 4, None, (0, 1, 127, 200, 254)),
    "sum_gqa_fp16_bs16": (LayerShape(1, 14, 2, 320, 128), torch.float16, 3, 1e6, 16, 4, "right_pad", None),
}


def summary_mask(kind, B, T):
    if kind is None:
        return None
    m = torch.ones((B, T), dtype=torch.bool)
    if kind == "holes":
        m[0, 10:12] = False
        m[0, 100:111] = False
        m[-1, 200:] = False
    else:  # right padding of the last batch item
        m[-1, T - 37:] = False
    return m


def summary_cases(ref):
    import hashlib

    cases = {}
    for name, (shape, dtype, seed, rope, bs, P, mask_kind, keep) in SUMMARY_CASES.items():
        _, k, v = make_layer_inputs(shape, dtype, seed, rope_theta=rope)
        mask = summary_mask(mask_kind, shape.batch, shape.tokens)
        layout = ref["tree_layout"]((shape.tokens + bs - 1) // bs)
        t = ref["summary"](k, v, layout, block_size=bs, prototypes=P, token_mask=mask)
        nodes = np.arange(layout.num_nodes) if keep is None else np.array(keep)
        cases[f"{name}_args"] = np.array([shape.batch, shape.q_heads, shape.kv_heads, shape.tokens, shape.head_dim,
                                          {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dtype], seed,
                                          bs, P], dtype=np.int64)
        cases[f"{name}_rope"] = np.array([rope or 0.0])
        cases[f"{name}_mask"] = np.array([{None: 0, "holes": 1, "right_pad": 2}[mask_kind]])
        cases[f"{name}_nodes"] = nodes
        cases[f"{name}_keys"] = t.keys[:, :, nodes].numpy()
        cases[f"{name}_values"] = t.values[:, :, nodes].numpy()
        cases[f"{name}_counts"] = t.counts.numpy()
        cases[f"{name}_log_counts"] = t.log_counts.numpy()
        cases[f"{name}_range_starts"] = t.range_starts.numpy()
        cases[f"{name}_range_ends"] = t.range_ends.numpy()
        digest = hashlib.sha256()
        for a in (t.keys, t.values, t.counts):
            digest.update(a.contiguous().numpy().tobytes())
        cases[f"{name}_sha256"] = np.frombuffer(digest.digest(), dtype=np.uint8)
        print(f"{name}: nodes={layout.num_nodes} P={P} keys {tuple(t.keys.shape)}")
    # tree layouts and maximal frontiers (interfaces/residual_summaries.py)
    for n in (1, 2, 3, 5, 7, 64, 100):
        lay = ref["tree_layout"](n)
        cases[f"tree{n}"] = np.array([lay.starts, lay.ends, lay.levels, lay.indices], dtype=np.int64)
        cases[f"tree{n}_counts"] = np.array(lay.level_counts, dtype=np.int64)
    c0 = np.load(os.path.join(HERE, "c0.npz"))
    selected = torch.from_numpy(c0["selected"])[:, None].contiguous()    # [B, 1, G, qb, K]
    nodes = ref["summary_nodes"](selected, validate_selected=False)  # c0 routes use local_window=0
    cases["frontier_c0"] = nodes.numpy()
    dens = ref["summary_density"](selected, nodes, seq_len=4096, block_size=64, prototypes=4)
    cases["frontier_c0_density"] = np.array([dens["exact_attention_entries"], dens["summary_prototype_entries"],
                                             dens["maximum_causal_attention_entries"]], dtype=np.int64)
    return cases


def maxsim_cases(ref):
    """The reference FlatGate (MaxSim, P = 8) on its own outlier-prototype features."""
    gen = torch.Generator().manual_seed(13)
    cases = {}
    for n, (G, T, d, p, dt) in enumerate([(2, 64 * 12, 64, 64, torch.bfloat16), (1, 64 * 9 + 20, 128, 96, torch.float32)]):
        q = torch.randn((1, G, T, d), generator=gen).to(dt)
        k = torch.randn((1, G, T, d), generator=gen).to(dt)
        q_feat = ref["proto_pool"](q, 64, 8)           # [1, G, nb, 8, d]
        k_feat = ref["proto_pool"](k, 64, 8)
        torch.manual_seed(100 + n)
        gate = ref["FlatGate"](1, d, p).eval()
        with torch.no_grad():
            s = gate(q_feat.float(), k_feat.float())    # [1, G, nb, nb]
            cand = torch.randint(0, q_feat.shape[2], (1, G, q_feat.shape[2], 5), generator=gen)
            sc = gate.score_candidates(q_feat.float(), k_feat.float(), cand)
        cases[f"ms{n}_q"] = _raw(q)
        cases[f"ms{n}_k"] = _raw(k)
        cases[f"ms{n}_dtype"] = np.array([{torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dt]])
        cases[f"ms{n}_wq"] = gate.Wq.detach().numpy()
        cases[f"ms{n}_wk"] = gate.Wk.detach().numpy()
        cases[f"ms{n}_scores"] = s.numpy()
        cases[f"ms{n}_cand"] = cand.numpy()
        cases[f"ms{n}_cand_scores"] = sc.numpy()
        # key tree (selector/tree.py:116) and beam traversal (scripts/eval_tree_traversal.py:60)
        levels = ref["build_key_tree"](k_feat.float(), radix=2)
        for lvl in levels:
            cases[f"ms{n}_tree{lvl.level}"] = lvl.features.numpy()
            cases[f"ms{n}_tree{lvl.level}_range"] = torch.stack([lvl.starts, lvl.ends]).numpy()
        with torch.no_grad():
            ids = ref["traverse"](gate, q_feat.float(), levels, 4, radix=2)
        cases[f"ms{n}_leaf_ids"] = ids.numpy()
    return cases


# name: (B, Hq, Hkv, T, D, dtype, seed, K, summary prototypes)
RESIDUAL_CASES = {
    "r_bf16": (1, 2, 1, 64 * 7 + 11, 64, torch.bfloat16, 31, 3, (1, 2, 4)),
    "r_f32": (1, 2, 1, 64 * 5 + 5, 64, torch.float32, 32, 2, (4,)),
}


def _routes_with_gaps(B, G, qb, K, gen):
    """int32 [B, 1, G, qb, K]: each row keeps its block and the one before (local window 1)
    plus random earlier blocks, so the residual frontier is not empty."""
    sel = torch.full((B, 1, G, qb, K), -1, dtype=torch.int32)
    for b in range(B):
        for g in range(G):
            for q in range(qb):
                must = {q, q - 1} - {-1}
                rest = [int(x) for x in torch.randperm(max(q - 1, 0), generator=gen)]
                row = sorted(must | set(rest[:max(0, K - len(must))]))
                sel[b, 0, g, q, :len(row)] = torch.tensor(row, dtype=torch.int32)
    return sel


def residual_cases(ref):
    """The reference's residual-summary attention (sparse/attention.py:83-274)."""
    cases = {}
    for name, (B, Hq, Hkv, T, D, dt, seed, K, protos) in RESIDUAL_CASES.items():
        gen = torch.Generator().manual_seed(seed)
        q = torch.randn((B, Hq, T, D), generator=gen).to(dt)
        k = torch.randn((B, Hkv, T, D), generator=gen).to(dt)
        v = torch.randn((B, Hkv, T, D), generator=gen).to(dt)
        qb = (T + 63) // 64
        sel = _routes_with_gaps(B, Hkv, qb, K, gen)
        nodes = ref["summary_nodes"](sel)
        cases[f"{name}_dtype"] = np.array([{torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dt]])
        cases[f"{name}_q"], cases[f"{name}_k"], cases[f"{name}_v"] = _raw(q), _raw(k), _raw(v)
        cases[f"{name}_selected"] = sel.numpy()
        cases[f"{name}_nodes"] = nodes.numpy()
        cases[f"{name}_protos"] = np.array(protos, dtype=np.int64)
        for P in protos:
            with torch.no_grad():
                out, _ = ref["attention"](_Module(0), q, k, v, None, selected_blocks=sel, block_size=64,
                                          residual_summaries=True, residual_summary_nodes=nodes,
                                          summary_prototypes=P)
            cases[f"{name}_out{P}"] = _raw(out)
        print(f"{name}: qb={qb} residual width {nodes.shape[-1]}")
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPRUCE_REFERENCE"),
                    help="path of the reference checkout (or set SPRUCE_REFERENCE)")
    ap.add_argument("--only", choices=["all", "summaries", "maxsim", "residual", "c1_full", "c2", "trained",
                                                   "live"],
                    default="all")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference (or SPRUCE_REFERENCE): the reference checkout to run")
    sys.path.insert(0, args.reference)
    from teacher.chunked_extract import _group_avg_tokens, _proto_pool_seq
    from selector.gate import FlatGate
    from scripts.export_selected_blocks import selected_ids_to_blocks
    from interfaces.validator import validate_selected_blocks
    from sparse.attention import sparse_prefill_attention_forward
    from sparse.summaries import build_kv_summary_table, residual_attention_density
    from interfaces.residual_summaries import build_residual_summary_nodes, build_residual_tree_layout
    ref = {"group_avg": _group_avg_tokens, "proto_pool": _proto_pool_seq, "FlatGate": FlatGate,
           "pack": selected_ids_to_blocks, "validate": validate_selected_blocks,
           "attention": sparse_prefill_attention_forward, "summary": build_kv_summary_table,
           "tree_layout": build_residual_tree_layout, "summary_nodes": build_residual_summary_nodes,
           "summary_density": residual_attention_density}
    from selector.tree import build_key_tree
    from scripts.eval_tree_traversal import traverse_to_leaf_ids
    ref["build_key_tree"] = build_key_tree
    ref["traverse"] = traverse_to_leaf_ids
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if args.only == "summaries":
        np.savez_compressed(os.path.join(HERE, "summaries.npz"), **summary_cases(ref))
        return
    if args.only == "maxsim":
        np.savez_compressed(os.path.join(HERE, "maxsim.npz"), **maxsim_cases(ref))
        return
    if args.only == "residual":
        np.savez_compressed(os.path.join(HERE, "residual.npz"), **residual_cases(ref))
        return
    if args.only in BIG_CASES:
        big_case(ref, args.only)
        return
    if args.only == "trained":
        trained_case(ref, args.reference)
        return
    if args.only == "live":
        live_case(args.reference)
        return

    for name, (shape, dtype, seed, rope, K, lw, sink, keep_blocks) in CASES.items():
        q, k, v = make_layer_inputs(shape, dtype, seed, rope_theta=rope)
        wq, wk = make_gate_weights(1, shape.head_dim, shape.head_dim, seed + 1000)
        if K is None:
            K = k_for_density(shape.query_blocks, 0.10)
        r = reference_pipeline(ref, q, k, v, wq[0], wk[0], K, lw, sink)
        out = r["out"]
        if keep_blocks is not None:
            rows = torch.cat([torch.arange(b * 64, min((b + 1) * 64, shape.tokens)) for b in keep_blocks])
            out = out[:, rows]
            kept = np.array(keep_blocks, dtype=np.int64)
        else:
            kept = np.arange(shape.query_blocks, dtype=np.int64)
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            shape=np.array([shape.batch, shape.q_heads, shape.kv_heads, shape.tokens, shape.head_dim]),
            dtype=np.array([{torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dtype]]),
            seed=np.array([seed]), rope=np.array([rope if rope is not None else 0.0]),
            policy=np.array([K, lw, sink]),
            checksum=np.array([q.double().sum().item(), k.double().sum().item(), v.double().sum().item()]),
            pooled_q=_raw(r["pooled_q"]), pooled_k=_raw(r["pooled_k"]),
            scores=r["scores"].numpy(), selected=r["selected"].numpy(),
            out=_raw(out), out_blocks=kept,
        )
        print(f"{name}: K={K} selected {tuple(r['selected'].shape)} out {tuple(out.shape)}")

    np.savez_compressed(os.path.join(HERE, "packing.npz"), **packing_cases(ref))
    np.savez_compressed(os.path.join(HERE, "proto.npz"), **proto_cases(ref))
    np.savez_compressed(os.path.join(HERE, "summaries.npz"), **summary_cases(ref))
    np.savez_compressed(os.path.join(HERE, "maxsim.npz"), **maxsim_cases(ref))
    np.savez_compressed(os.path.join(HERE, "residual.npz"), **residual_cases(ref))
    for name in BIG_CASES:
        big_case(ref, name)
    trained_case(ref, args.reference)
    live_case(args.reference)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
