"""K/V summary table and residual tree on CPU: the oracle and the host mirror.

The oracle's build_kv_summary_table restatement is pinned to the reference's
outputs (tests/golden/summaries.npz, made by make_golden.py): keys, values
and counts bit-exact (the reference's fp32 cumsum accumulates in double on
CPU, as the oracle does), log_counts within one float ulp (torch's CPU float
log is not correctly rounded for a few integers).  The tree layout, maximal
frontiers, validator messages and density accounting of the host mirror are
checked against the reference's outputs and its tests/test_summary_pooling.py
known answers.
"""
import math

import numpy as np
import pytest
import torch

from golden_cases import SUMMARY_CASE_NAMES, load_npz, load_summary_case, table_sha256
from oracle import oracle as O
from spruce_research_b200.interfaces.residual_summaries import (build_residual_summary_nodes,
                                                                build_residual_tree_layout,
                                                                residual_frontier_for_row,
                                                                validate_residual_summary_nodes)
from spruce_research_b200.sparse.summaries import (_prototype_token_ranges, build_kv_summary_table,
                                                   residual_attention_density, token_validity_from_attention_mask)

LOG_ULP = 2.0 ** -23  # relative: one float ulp of a value in [1, 2) or above


def assert_log_counts_close(got: torch.Tensor, want: torch.Tensor) -> None:
    assert torch.equal(torch.isneginf(got), torch.isneginf(want))
    fin = torch.isfinite(want)
    err = (got[fin].double() - want[fin].double()).abs()
    assert (err <= want[fin].double().abs().clamp_min(1.0) * LOG_ULP).all()


@pytest.mark.parametrize("name", SUMMARY_CASE_NAMES)
def test_oracle_summary_table_matches_reference(name):
    case = load_summary_case(name)
    k, v, mask = case.inputs()
    lay = build_residual_tree_layout((case.shape.tokens + case.block_size - 1) // case.block_size)
    t = O.kv_summary_table(k, v, lay.starts, lay.ends, case.block_size, case.prototypes, mask)
    nodes = case.nodes
    assert torch.equal(t["keys"][:, :, nodes], case.get("keys"))
    assert torch.equal(t["values"][:, :, nodes], case.get("values"))
    assert torch.equal(t["counts"], case.get("counts"))
    assert torch.equal(t["range_starts"], case.get("range_starts"))
    assert torch.equal(t["range_ends"], case.get("range_ends"))
    assert table_sha256(t["keys"], t["values"], t["counts"]) == case.sha256
    assert_log_counts_close(t["log_counts"], case.get("log_counts"))


def test_oracle_reference_known_answers():
    # tests/test_summary_pooling.py:49-70 of the reference
    key = torch.arange(5, dtype=torch.float32).view(1, 1, 5, 1)
    lay = build_residual_tree_layout(3)
    t = O.kv_summary_table(key, key * 10, lay.starts, lay.ends, 2, 2)
    assert t["counts"][0, 3].tolist() == [2.0, 2.0]
    assert t["keys"][0, 0, 3, :, 0].tolist() == [0.5, 2.5]
    assert t["values"][0, 0, 3, :, 0].tolist() == [5.0, 25.0]
    assert t["log_counts"][0, 3].tolist() == [math.log(2.0)] * 2 or torch.allclose(
        t["log_counts"][0, 3], torch.tensor([math.log(2.0)] * 2))
    assert t["counts"][0, 2].tolist() == [0.0, 1.0]
    assert math.isinf(t["log_counts"][0, 2, 0].item()) and t["log_counts"][0, 2, 0].item() < 0
    assert t["keys"][0, 0, 2, 1, 0].item() == 4.0
    # :73-88 padding tokens contribute to neither means nor counts
    key = torch.tensor([[[[100.0], [100.0], [2.0], [4.0]]]])
    lay = build_residual_tree_layout(2)
    t = O.kv_summary_table(key, key.clone(), lay.starts, lay.ends, 2, 1, torch.tensor([[False, False, True, True]]))
    assert t["counts"][0, lay.root_id, 0].item() == 2 and t["keys"][0, 0, lay.root_id, 0, 0].item() == 3.0


def test_tree_layouts_match_reference():
    z = load_npz("summaries")
    for n in (1, 2, 3, 5, 7, 64, 100):
        lay = build_residual_tree_layout(n)
        starts, ends, levels, indices = (tuple(int(x) for x in row) for row in z[f"tree{n}"])
        assert (lay.starts, lay.ends, lay.levels, lay.indices) == (starts, ends, levels, indices)
        assert lay.level_counts == tuple(int(x) for x in z[f"tree{n}_counts"])
        o_starts, o_ends = O.residual_tree_ranges(n)
        assert (tuple(o_starts), tuple(o_ends)) == (starts, ends)
    lay = build_residual_tree_layout(5)
    assert lay.children(lay.root_id) == (lay.node_id(2, 0), lay.node_id(2, 1))
    assert lay.children(lay.node_id(1, 2)) == (lay.node_id(0, 4),)
    with pytest.raises(IndexError):
        lay.range(lay.num_nodes)
    with pytest.raises(ValueError, match="num_leaves must be >= 1"):
        build_residual_tree_layout(0)


def test_frontiers_and_density_match_reference():
    z = load_npz("summaries")
    c0 = load_npz("c0")
    selected = torch.from_numpy(c0["selected"])[:, None].contiguous()
    nodes = build_residual_summary_nodes(selected, validate_selected=False)
    assert torch.equal(nodes, torch.from_numpy(z["frontier_c0"]))
    validate_residual_summary_nodes(selected, nodes, validate_selected=False)
    d = residual_attention_density(selected, nodes, seq_len=4096, block_size=64, prototypes=4)
    want = [int(x) for x in z["frontier_c0_density"]]
    assert [d["exact_attention_entries"], d["summary_prototype_entries"],
            d["maximum_causal_attention_entries"]] == want


def _local_routes(qblocks):
    sel = torch.full((1, 1, 1, qblocks, 2), -1, dtype=torch.int32)
    for q in range(qblocks):
        row = torch.arange(max(0, q - 1), q + 1, dtype=torch.int32)
        sel[0, 0, 0, q, :len(row)] = row
    return sel


def test_frontier_rules_and_validator_messages():
    lay = build_residual_tree_layout(8)
    assert residual_frontier_for_row([0, 7], 7, lay) == sorted(
        [lay.node_id(0, 1), lay.node_id(1, 1), lay.node_id(0, 6), lay.node_id(1, 2)])
    assert residual_frontier_for_row(range(8), 7, lay) == []
    with pytest.raises(ValueError, match="causal"):
        residual_frontier_for_row([3], 2, lay)
    sel = _local_routes(3)
    nodes = build_residual_summary_nodes(sel, validate_selected=False)  # the route validator runs on the GPU
    # reference tests/test_summary_pooling.py:219-233: only query block 2 omits block 0
    assert nodes.shape == (1, 1, 1, 3, 1) and nodes[0, 0, 0, :, 0].tolist() == [-1, -1, 0]
    d = residual_attention_density(sel, nodes, seq_len=5, block_size=2, prototypes=1)
    assert (d["exact_attention_entries"], d["summary_prototype_entries"], d["charged_attention_entries"],
            d["maximum_causal_attention_entries"]) == (10, 1, 11, 12)
    bad = nodes.clone()
    bad[0, 0, 0, 1, 0] = 0  # block 0 now covered twice in row 1
    with pytest.raises(AssertionError, match="disjoint complete causal partition"):
        validate_residual_summary_nodes(sel, bad, validate_selected=False)
    bad = nodes.clone()
    bad[0, 0, 0, 2, 0] = 4  # node 4 = blocks [0, 2): overlaps the exact block 1
    with pytest.raises(AssertionError, match="disjoint complete"):
        validate_residual_summary_nodes(sel, bad, validate_selected=False)
    padded = torch.cat([torch.full_like(nodes, -1), nodes], -1)  # row 2 becomes [-1, 0]
    with pytest.raises(AssertionError, match="padding is not trailing-only"):
        validate_residual_summary_nodes(sel, padded, validate_selected=False)
    with pytest.raises(AssertionError, match="Duplicate residual node IDs"):
        validate_residual_summary_nodes(sel, torch.cat([nodes, nodes], -1), validate_selected=False)


def test_host_ranges_validity_and_argument_errors():
    lay = build_residual_tree_layout(3)
    s, e = _prototype_token_ranges(lay, seq_len=5, block_size=2, prototypes=2, device="cpu")
    assert s[2].tolist() == [4, 4] and e[2].tolist() == [4, 5] and s[3].tolist() == [0, 2]
    floor = torch.finfo(torch.float32).min
    mask = torch.full((1, 1, 5, 5), floor)
    mask[0, 0, 0, 0] = 0
    mask[0, 0, 1, :2] = 0
    mask[0, 0, 2, :3] = 0
    assert token_validity_from_attention_mask(mask, batch=1, seq_len=5).tolist() == [[True, True, True, False,
                                                                                        False]]
    key = torch.zeros(1, 1, 5, 4)
    with pytest.raises(ValueError, match="prototypes must be one of"):
        build_kv_summary_table(key, key, lay, block_size=2, prototypes=3)
    with pytest.raises(ValueError, match="tree has 3 leaves, expected 5"):
        build_kv_summary_table(key, key, lay, block_size=1, prototypes=1)
    with pytest.raises(ValueError, match="shape mismatch"):
        build_kv_summary_table(key, key[:, :, :4], lay, block_size=2, prototypes=1)
    with pytest.raises(RuntimeError, match="CUDA"):
        build_kv_summary_table(key, key, lay, block_size=2, prototypes=1)
