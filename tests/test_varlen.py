"""Packed variable-length batches and the all-blocks route (host logic, CPU).

Reference: benchmarks/all_blocks_equivalence.py:53-68 (every causal block in
the selected_blocks format); config 4's variable-length batch is served by
per-sequence calls of the single-sequence path.
"""
import pytest
import torch

from oracle import oracle as O
from spruce_research_b200.varlen import VarlenSparsePrefill, all_causal_selected_blocks, check_cu_seqlens


def test_all_causal_route_is_every_causal_block():
    sel = all_causal_selected_blocks(num_layers=2, num_kv_groups=3, seq_len=64 * 4 + 5)
    assert sel.shape == (1, 2, 3, 5, 5) and sel.dtype == torch.int32
    assert sel[0, 1, 2].tolist() == [[0, -1, -1, -1, -1], [0, 1, -1, -1, -1], [0, 1, 2, -1, -1],
                                     [0, 1, 2, 3, -1], [0, 1, 2, 3, 4]]
    O.validate_selected_blocks(sel)
    with pytest.raises(ValueError, match="positive"):
        all_causal_selected_blocks(num_layers=0, num_kv_groups=1, seq_len=64)


def test_cu_seqlens_rules():
    assert check_cu_seqlens(torch.tensor([0, 128, 192, 250]), 250) == [0, 128, 192, 250]
    with pytest.raises(ValueError, match="block boundaries"):
        check_cu_seqlens([0, 100, 250], 250)
    with pytest.raises(ValueError, match="from 0 to"):
        check_cu_seqlens([0, 128], 250)
    with pytest.raises(ValueError, match="increasing"):
        check_cu_seqlens([0, 128, 128, 250], 250)
    v = VarlenSparsePrefill(torch.zeros(64, 64), torch.zeros(64, 64))
    with pytest.raises(ValueError, match="exactly one"):
        v.k_for(4096, None, None)
    assert v.k_for(131072, 0.10, None) == 106 and v.k_for(64, None, 1) == 2  # sink + diagonal at least


def test_acceptance_criteria_follow_the_reference_definitions():
    from spruce_research_b200.acceptance import DEFAULT_ACCEPTANCE, logits_error, passes_acceptance, tensor_error

    e = torch.linspace(-3, 3, 512)
    same = logits_error(e.clone(), e)
    assert same["cosine"] > 0.999999 and same["top1_same"] and same["top10_overlap"] == 1.0
    assert tensor_error(e, e)["relative_rmse"] == 0.0
    assert passes_acceptance(same, tensor_error(e, e))
    swapped = e.clone()
    swapped[[-1, 0]] = swapped[[0, -1]]                       # the top-1 token changes
    assert not passes_acceptance(logits_error(swapped, e), tensor_error(e, e))
    assert not passes_acceptance(same, tensor_error(e * 1.05, e))   # 5% relative RMSE > 0.02
    assert DEFAULT_ACCEPTANCE["minimum_logits_cosine"] == 0.999
