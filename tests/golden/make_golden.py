"""Generate the golden vectors under tests/golden/ by running the REFERENCE.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/spruce-research

It imports the reference's own torch functions -- _group_avg_tokens,
_proto_pool_seq, FlatGate, selected_ids_to_blocks, validate_selected_blocks,
sparse_prefill_attention_forward -- feeds them the seeded synthetic inputs of
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPRUCE_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from teacher.chunked_extract import _group_avg_tokens, _proto_pool_seq
    from selector.gate import FlatGate
    from scripts.export_selected_blocks import selected_ids_to_blocks
    from interfaces.validator import validate_selected_blocks
    from sparse.attention import sparse_prefill_attention_forward
    ref = {"group_avg": _group_avg_tokens, "proto_pool": _proto_pool_seq, "FlatGate": FlatGate,
           "pack": selected_ids_to_blocks, "validate": validate_selected_blocks,
           "attention": sparse_prefill_attention_forward}
    torch.set_num_threads(max(1, os.cpu_count() or 1))

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
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
