"""Residual-summary attention on the GPU (sparse/attention.py:83-274, residual_summaries=True).

The CUDA path (summary table, gather of each row's valid node prototypes into
virtual blocks, one online softmax over selected blocks and summaries) is
compared with the reference's own outputs (tests/golden/residual.npz, through
the drop-in callback) and with the oracle on generated cases: bf16 / fp16
within max-abs 2e-2 and mean-abs 2e-3, fp32 within 1e-4.  The cases cover
GQA 4:1 and 7:1 (a half-filled last head tile), batch 2, ragged tails, rows
whose summaries span several virtual blocks (odd and even counts), and routes
with no residual node at all (plain block-sparse attention, bit-identical).
"""
import pytest
import torch

from golden_cases import RESIDUAL_CASE_NAMES, load_residual_case
from oracle import oracle as O
from spruce_research_b200 import native
from spruce_research_b200.interfaces.residual_summaries import (build_residual_summary_nodes,
                                                                build_residual_tree_layout)
from spruce_research_b200.sparse.attention import sparse_prefill_attention_forward
from spruce_research_b200.sparse.summaries import build_kv_summary_table

pytestmark = pytest.mark.gpu


class _Layer(torch.nn.Module):
    layer_idx = 0


def _close(got, want, dtype):
    err = (got.float().cpu() - want.float().cpu()).abs()
    if dtype == torch.float32:
        assert err.max().item() < 1e-4, err.max().item()
    else:
        assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, (err.max().item(), err.mean().item())


@pytest.mark.parametrize("name", RESIDUAL_CASE_NAMES)
def test_reference_outputs_through_the_callback(name):
    q, k, v, sel, nodes, outs = load_residual_case(name)
    for P, want in outs.items():
        got, _ = sparse_prefill_attention_forward(_Layer(), q.cuda(), k.cuda(), v.cuda(), None,
                                                  selected_blocks=sel.cuda(), block_size=64,
                                                  residual_summaries=True, residual_summary_nodes=nodes.cuda(),
                                                  summary_prototypes=P)
        assert got.shape == (q.shape[0], q.shape[2], q.shape[1], q.shape[3]) and got.dtype == q.dtype
        _close(got, want, q.dtype)


def _routes(B, G, qb, K, seed):
    gen = torch.Generator().manual_seed(seed)
    sel = torch.full((B, 1, G, qb, K), -1, dtype=torch.int32)
    for b in range(B):
        for g in range(G):
            for q in range(qb):
                must = {q, q - 1} - {-1}
                rest = [int(x) for x in torch.randperm(max(q - 1, 0), generator=gen)]
                row = sorted(must | set(rest[:max(0, K - len(must))]))
                sel[b, 0, g, q, :len(row)] = torch.tensor(row, dtype=torch.int32)
    return sel


def _case(B, Hq, Hkv, T, D, dtype, K, P, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn((B, Hq, T, D), generator=gen).to(dtype)
    k = torch.randn((B, Hkv, T, D), generator=gen).to(dtype)
    v = torch.randn((B, Hkv, T, D), generator=gen).to(dtype)
    qb = (T + 63) // 64
    sel = _routes(B, Hkv, qb, K, seed + 1)
    nodes = build_residual_summary_nodes(sel.cuda()).cpu()
    lay = build_residual_tree_layout(qb)
    table = build_kv_summary_table(k.cuda(), v.cuda(), lay, block_size=64, prototypes=P)
    got = native.residual_sparse_attention(q.cuda(), k.cuda(), v.cuda(), sel[:, 0].cuda(), nodes[:, 0].cuda(), table)
    t = O.kv_summary_table(k, v, lay.starts, lay.ends, 64, P, None)
    want = O.residual_sparse_attention(q, k, v, sel[:, 0], nodes[:, 0], t["keys"], t["values"], t["counts"],
                                       t["log_counts"], out_dtype=torch.float32)
    return got, want, sel, nodes


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("P", [1, 2, 4])
def test_tcgen05_path_matches_oracle(dtype, P):
    got, want, _, nodes = _case(2, 8, 2, 64 * 40 + 17, 128, dtype, 6, P, 70 + P)
    assert nodes.shape[-1] > 0
    _close(got, want, dtype)


def test_odd_group_and_head_dim_64():
    got, want, _, _ = _case(1, 7, 1, 64 * 30 + 3, 64, torch.bfloat16, 5, 2, 81)
    _close(got, want, torch.bfloat16)


def test_fp32_path_matches_oracle():
    got, want, _, _ = _case(1, 4, 2, 64 * 24 + 9, 64, torch.float32, 4, 4, 82)
    _close(got, want, torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_summaries_spanning_several_virtual_blocks(dtype):
    # 256 query blocks with 8 scattered selections per row: frontiers of tens of
    # nodes, x4 prototypes, so rows carry 1 to 5 virtual blocks of summaries
    got, want, sel, nodes = _case(1, 4, 1, 64 * 256, 64, dtype, 8, 4, 83)
    per_row = (nodes[:, 0] >= 0).sum(-1) * 4
    assert per_row.max().item() > 128 and (per_row > 0).any()
    _close(got, want, dtype)


def test_no_residual_nodes_is_plain_sparse_attention():
    gen = torch.Generator().manual_seed(84)
    B, Hq, Hkv, T, D = 1, 4, 2, 64 * 9, 128
    q = torch.randn((B, Hq, T, D), generator=gen).to(torch.bfloat16).cuda()
    k = torch.randn((B, Hkv, T, D), generator=gen).to(torch.bfloat16).cuda()
    v = torch.randn((B, Hkv, T, D), generator=gen).to(torch.bfloat16).cuda()
    qb = T // 64
    sel = torch.full((B, Hkv, qb, qb), -1, dtype=torch.int32)
    for i in range(qb):
        sel[:, :, i, :i + 1] = torch.arange(i + 1, dtype=torch.int32)
    nodes = build_residual_summary_nodes(sel[:, None].cuda()).cpu()
    assert nodes.shape[-1] == 0
    table = build_kv_summary_table(k, v, build_residual_tree_layout(qb), block_size=64, prototypes=1)
    got = native.residual_sparse_attention(q, k, v, sel.cuda(), nodes[:, 0].cuda(), table)
    assert torch.equal(got, native.sparse_attention(q, k, v, sel.cuda()))


def _prefix_mean(v, Hq):
    """Uniform causal attention: out[b, t, h] = mean(v[b, g(h), :t+1]) in fp64, [B, T, Hq, D]."""
    c = torch.cumsum(v.double(), dim=2) / torch.arange(1, v.shape[2] + 1, device=v.device,
                                                        dtype=torch.float64)[None, None, :, None]
    return c.repeat_interleave(Hq // v.shape[1], dim=1).transpose(1, 2)


@pytest.mark.parametrize("P", [1, 2, 4])
def test_identical_keys_give_dense_attention(P):
    # tests/test_summary_pooling.py:100-131 of the reference: with every key equal, a summary
    # prototype weighted by its count stands in exactly for its tokens, so the residual-summary
    # output is dense causal attention -- here uniform over the causal prefix
    gen = torch.Generator().manual_seed(90 + P)
    B, Hq, Hkv, T, D = 1, 8, 2, 64 * 37 + 21, 128
    q = torch.randn((B, Hq, T, D), generator=gen).to(torch.bfloat16).cuda()
    k = torch.randn((B, Hkv, 1, D), generator=gen).to(torch.bfloat16).expand(B, Hkv, T, D).contiguous().cuda()
    v = torch.randn((B, Hkv, T, D), generator=gen).to(torch.bfloat16).cuda()
    sel = _routes(B, Hkv, (T + 63) // 64, 5, 91)
    out, _ = sparse_prefill_attention_forward(_Layer(), q, k, v, None, selected_blocks=sel.cuda(), block_size=64,
                                              residual_summaries=True,
                                              residual_summary_nodes=build_residual_summary_nodes(sel.cuda()),
                                              summary_prototypes=P)
    _close(out, _prefix_mean(v, Hq), torch.bfloat16)


def test_identical_keys_at_config2_shape():
    # the same property at 131072 tokens, 28/4 heads, d=128, routes of the flat selector at 10%
    from spruce_research_b200.pipeline import SparsePrefillLayer
    from spruce_research_b200.synthetic import k_for_density, make_gate_weights

    gen = torch.Generator().manual_seed(95)
    B, Hq, Hkv, T, D = 1, 28, 4, 131072, 128
    q = torch.randn((B, T, Hq, D), generator=gen).to(torch.bfloat16).cuda().transpose(1, 2)
    k = torch.randn((B, Hkv, 1, D), generator=gen).to(torch.bfloat16).cuda().expand(B, Hkv, T, D).contiguous()
    v = torch.randn((B, T, Hkv, D), generator=gen).to(torch.bfloat16).cuda().transpose(1, 2)
    wq, wk = make_gate_weights(1, D, D, 96, device="cuda")
    sel = SparsePrefillLayer(wq[0], wk[0], k_for_density(T // 64, 0.10), 0, 1).select(q, k)
    nodes = build_residual_summary_nodes(sel[:, None], validate_selected=False)[:, 0]
    assert nodes.shape[-1] > 10  # equal scores: the selector keeps the lowest ids, leaving one long gap per row
    table = build_kv_summary_table(k, v, build_residual_tree_layout(T // 64), block_size=64, prototypes=4)
    out = native.residual_sparse_attention(q, k, v, sel, nodes, table)
    want = _prefix_mean(v, Hq)
    err = (out.double() - want).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3, (err.max().item(), err.mean().item())


def test_summaries_disabled_is_identical():
    # tests/test_summary_pooling.py:134-160 of the reference
    q, k, v, sel, nodes, _ = load_residual_case("r_bf16")
    args = dict(selected_blocks=sel.cuda(), block_size=64)
    base, _ = sparse_prefill_attention_forward(_Layer(), q.cuda(), k.cuda(), v.cuda(), None, **args)
    off, _ = sparse_prefill_attention_forward(_Layer(), q.cuda(), k.cuda(), v.cuda(), None, residual_summaries=False,
                                              residual_summary_nodes=nodes.cuda(), summary_prototypes=4, **args)
    assert torch.equal(base, off)
