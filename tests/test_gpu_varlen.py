"""Packed variable-length batches on the GPU.

At 10% density each sequence of a packed batch must select exactly the oracle's
blocks on its own inputs and match the oracle's block-sparse attention on them
(max-abs 2e-2, mean-abs 2e-3 in bf16); at 100% density the result must match
dense causal attention (the reference's all-blocks equivalence gate,
benchmarks/all_blocks_equivalence.py:53-68) within the same tolerance.
"""
import pytest
import torch

from oracle import oracle as O
from spruce_research_b200.synthetic import LayerShape, make_gate_weights, make_layer_inputs
from spruce_research_b200.varlen import VarlenSparsePrefill

pytestmark = pytest.mark.gpu


def _packed(lengths, Hq, Hkv, D, seed):
    qs, ks, vs = [], [], []
    for n, T in enumerate(lengths):
        q, k, v = make_layer_inputs(LayerShape(1, Hq, Hkv, T, D), torch.bfloat16, seed + n)
        qs.append(q[0].transpose(0, 1))
        ks.append(k[0].transpose(0, 1))
        vs.append(v[0].transpose(0, 1))
    cu = [0]
    for T in lengths:
        cu.append(cu[-1] + T)
    return (torch.cat(qs).contiguous().cuda(), torch.cat(ks).contiguous().cuda(), torch.cat(vs).contiguous().cuda(),
            cu)


def test_each_sequence_matches_the_oracle_at_sparse_density():
    lengths = [4096, 1024, 2048 + 37]
    q, k, v, cu = _packed(lengths, 28, 4, 128, seed=40)
    wq, wk = make_gate_weights(1, 128, 128, seed=41, device="cuda")
    out, sel = VarlenSparsePrefill(wq[0], wk[0])(q, k, v, cu, density=0.10)
    for n, (a, b) in enumerate(zip(cu, cu[1:])):
        qs, ks, vs = (x[a:b].unsqueeze(0).transpose(1, 2).cpu() for x in (q, k, v))
        K = sel[n].shape[-1]
        want_sel = O.select_blocks(qs, ks, wq[0].cpu(), wk[0].cpu(), K, 0, 1)["selected"]
        assert torch.equal(sel[n].cpu(), want_sel), f"sequence {n}: selection differs from the oracle"
        want = O.sparse_attention(qs, ks, vs, want_sel, out_dtype=torch.float32)[0]     # [T, Hq, D]
        err = (out[a:b].float().cpu() - want).abs()
        assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, f"sequence {n}: {err.max().item():.3e}"


def test_full_density_matches_dense_causal_attention():
    lengths = [1024, 512 + 64, 640 + 21]
    q, k, v, cu = _packed(lengths, 4, 2, 64, seed=50)
    wq, wk = make_gate_weights(1, 64, 64, seed=51, device="cuda")
    out, sel = VarlenSparsePrefill(wq[0], wk[0])(q, k, v, cu, density=1.0)
    for n, (a, b) in enumerate(zip(cu, cu[1:])):
        qb = (b - a + 63) // 64
        assert sel[n].shape[-1] == qb and (sel[n] >= 0).sum().item() == 2 * qb * (qb + 1) // 2
        qs, ks, vs = (x[a:b].unsqueeze(0).transpose(1, 2).cpu() for x in (q, k, v))
        dense = O.dense_causal_attention(qs, ks, vs)[0]                 # [T, Hq, D]
        err = (out[a:b].float().cpu() - dense).abs()
        assert err.max().item() < 2e-2 and err.mean().item() < 2e-3
