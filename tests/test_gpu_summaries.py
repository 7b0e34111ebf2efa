"""K/V summary table on the GPU against the reference's outputs and the oracle.

Keys, values, counts and ranges are compared bit for bit (the kernels build
the reference's double-accumulated prefix exactly); log_counts within one
float ulp.  Cases: the reference's known answers (tests/test_summary_pooling.py),
the golden fixtures of summaries.npz, the 128K-token config-2 shape against
the oracle, fp32 with padding masks, and the scalar (unaligned) path.
"""
import math

import pytest
import torch

from golden_cases import SUMMARY_CASE_NAMES, load_summary_case, table_sha256
from oracle import oracle as O
from spruce_research_b200.interfaces.residual_summaries import (build_residual_summary_nodes,
                                                                build_residual_tree_layout)
from spruce_research_b200.sparse.summaries import build_kv_summary_table
from spruce_research_b200.synthetic import LayerShape, make_layer_inputs
from test_summaries import assert_log_counts_close

pytestmark = pytest.mark.gpu


def _check_against_oracle(k, v, mask, bs, P):
    T = k.shape[2]
    lay = build_residual_tree_layout((T + bs - 1) // bs)
    got = build_kv_summary_table(k, v, lay, block_size=bs, prototypes=P, token_mask=mask)
    torch.cuda.synchronize()
    want = O.kv_summary_table(k.cpu(), v.cpu(), lay.starts, lay.ends, bs, P, None if mask is None else mask.cpu())
    for name in ("keys", "values", "counts", "range_starts", "range_ends"):
        g = getattr(got, name).cpu()
        assert torch.equal(g, want[name]), f"{name}: max diff {(g.double() - want[name].double()).abs().max()}"
    assert_log_counts_close(got.log_counts.cpu(), want["log_counts"])
    return got


def test_reference_known_answers_on_gpu():
    key = torch.arange(5, dtype=torch.float32, device="cuda").view(1, 1, 5, 1)
    lay = build_residual_tree_layout(3)
    t = build_kv_summary_table(key, key * 10, lay, block_size=2, prototypes=2)
    assert t.counts[0, 3].tolist() == [2.0, 2.0]
    assert t.keys[0, 0, 3, :, 0].tolist() == [0.5, 2.5]
    assert t.values[0, 0, 3, :, 0].tolist() == [5.0, 25.0]
    torch.testing.assert_close(t.log_counts[0, 3].cpu(), torch.tensor([math.log(2.0)] * 2))
    assert t.counts[0, 2].tolist() == [0.0, 1.0]
    assert torch.isneginf(t.log_counts[0, 2, 0]).item()
    assert t.keys[0, 0, 2, 1, 0].item() == 4.0
    key = torch.tensor([[[[100.0], [100.0], [2.0], [4.0]]]], device="cuda")
    lay = build_residual_tree_layout(2)
    t = build_kv_summary_table(key, key.clone(), lay, block_size=2, prototypes=1,
                               token_mask=torch.tensor([[False, False, True, True]], device="cuda"))
    assert t.counts[0, lay.root_id, 0].item() == 2 and t.keys[0, 0, lay.root_id, 0, 0].item() == 3.0


@pytest.mark.parametrize("name", SUMMARY_CASE_NAMES)
def test_summary_table_matches_reference_golden(name):
    # CUDA == oracle on the inputs this host generates; the CPU suite pins
    # oracle == reference, and where this host reproduces the fixture's inputs
    # exactly (same table hash) the reference's outputs are checked directly.
    case = load_summary_case(name)
    k, v, mask = case.inputs("cuda")
    lay = build_residual_tree_layout((case.shape.tokens + case.block_size - 1) // case.block_size)
    t = build_kv_summary_table(k, v, lay, block_size=case.block_size, prototypes=case.prototypes, token_mask=mask)
    _check_against_oracle(k, v, mask, case.block_size, case.prototypes)
    if table_sha256(*(O.kv_summary_table(k.cpu(), v.cpu(), lay.starts, lay.ends, case.block_size,
                                         case.prototypes, None if mask is None else mask.cpu())[x]
                      for x in ("keys", "values", "counts"))) == case.sha256:
        nodes = case.nodes
        assert torch.equal(t.keys.cpu()[:, :, nodes], case.get("keys"))
        assert torch.equal(t.values.cpu()[:, :, nodes], case.get("values"))
        assert torch.equal(t.counts.cpu(), case.get("counts"))
        assert torch.equal(t.range_starts.cpu(), case.get("range_starts"))
        assert torch.equal(t.range_ends.cpu(), case.get("range_ends"))
        assert table_sha256(t.keys, t.values, t.counts) == case.sha256
        assert_log_counts_close(t.log_counts.cpu(), case.get("log_counts"))


@pytest.mark.parametrize("P", [1, 4])
def test_config2_shape_bit_exact_against_oracle(P):
    # 131072 tokens, 4 KV heads, d=128, bf16 post-RoPE keys: the north-star shape
    shape = LayerShape(1, 28, 4, 131072, 128)
    _, k, v = make_layer_inputs(shape, torch.bfloat16, seed=21)
    k = k.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    v = v.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    t = _check_against_oracle(k, v, None, 64, P)
    lay = build_residual_tree_layout(2048)
    assert t.counts[0, lay.root_id].sum().item() == 131072


def test_fp32_masks_and_ragged_tail_against_oracle():
    shape = LayerShape(2, 8, 2, 32768 + 45, 64)
    _, k, v = make_layer_inputs(shape, torch.float32, seed=22)
    gen = torch.Generator().manual_seed(3)
    mask = torch.rand((2, shape.tokens), generator=gen) > 0.1
    mask[1, 30000:] = False
    _check_against_oracle(k.cuda(), v.cuda(), mask.cuda(), 64, 2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_scalar_path_small_blocks_against_oracle(dtype):
    gen = torch.Generator().manual_seed(5)
    k = torch.randn((2, 3, 101, 3), generator=gen).to(dtype)
    v = torch.randn((2, 3, 101, 3), generator=gen).to(dtype)
    mask = torch.rand((2, 101), generator=gen) > 0.3
    for bs, P in ((2, 4), (3, 2), (7, 1), (1, 4)):
        _check_against_oracle(k.cuda(), v.cuda(), mask.cuda(), bs, P)


def test_residual_nodes_validate_routes_on_gpu():
    sel = torch.full((1, 1, 1, 3, 2), -1, dtype=torch.int32)
    for q in range(3):
        row = torch.arange(max(0, q - 1), q + 1, dtype=torch.int32)
        sel[0, 0, 0, q, :len(row)] = row
    nodes = build_residual_summary_nodes(sel.cuda())
    assert nodes.is_cuda and nodes[0, 0, 0, :, 0].tolist() == [-1, -1, 0]
    bad = sel.clone()
    bad[0, 0, 0, 2] = torch.tensor([2, -1], dtype=torch.int32)
    with pytest.raises(AssertionError, match="Missing local-window"):
        build_residual_summary_nodes(bad.cuda())


def test_frontier_kernel_matches_reference_golden():
    # the c0 routes' frontiers as the reference's build_residual_summary_nodes made them
    from golden_cases import load_npz

    z = load_npz("summaries")
    c0 = load_npz("c0")
    selected = torch.from_numpy(c0["selected"])[:, None].contiguous()
    nodes = build_residual_summary_nodes(selected.cuda(), validate_selected=False)
    assert nodes.is_cuda and torch.equal(nodes.cpu(), torch.from_numpy(z["frontier_c0"]))


@pytest.mark.parametrize("qb,K,seed", [(1, 1, 0), (2, 2, 1), (7, 3, 2), (100, 5, 3), (333, 9, 4), (2048, 24, 5)])
def test_frontier_kernel_matches_host_walk(qb, K, seed):
    # random causal routes (sorted, some rows short) against the reference-mirroring host walk
    gen = torch.Generator().manual_seed(seed)
    sel = torch.full((2, 1, 3, qb, K), -1, dtype=torch.int32)
    for b in range(2):
        for g in range(3):
            for q in range(qb):
                n = int(torch.randint(1, K + 1, (1,), generator=gen))
                ids = sorted(set([q] + [int(x) for x in torch.randint(0, q + 1, (n - 1,), generator=gen)]))
                sel[b, 0, g, q, :len(ids)] = torch.tensor(ids, dtype=torch.int32)
    want = build_residual_summary_nodes(sel, validate_selected=False)
    got = build_residual_summary_nodes(sel.cuda(), validate_selected=False)
    assert got.shape == want.shape and torch.equal(got.cpu(), want)
