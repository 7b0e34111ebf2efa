"""Reference-named drop-ins: host logic and error conventions (CPU).

Mirrors the reference's tests/test_triton_sparse_prefill.py:20-66,
tests/test_sparse_attention.py:73-87 and tests/test_export_selected_blocks.py
error cases; compute paths that need the GPU are in test_gpu_dropin.py.
"""
import pytest
import torch

from spruce_research_b200.export_selected_blocks import selected_ids_to_blocks, selected_mask_to_blocks
from spruce_research_b200.kernels.direct_index import KERNEL_VARIANTS, direct_index_sparse_triton, kernel_runtime_metadata
from spruce_research_b200.kernels.sparse_prefill import (selected_blocks_to_block_mask, selected_blocks_to_head_indices,
                                                         triton_sparse_prefill_attention_forward)
from spruce_research_b200.route_overrides import charged_route_density
from spruce_research_b200.sparse.attention import sparse_prefill_attention_forward


class _Module(torch.nn.Module):
    def __init__(self, layer_idx=0):
        super().__init__()
        self.layer_idx = layer_idx


def _selected(batch=1, layers=1, groups=1, qblocks=2, width=2):
    out = torch.full((batch, layers, groups, qblocks, width), -1, dtype=torch.int32)
    for q in range(qblocks):
        out[:, :, :, q, : q + 1] = torch.arange(q + 1, dtype=torch.int32)
    return out


def test_block_mask_adapter_expands_kv_groups_to_query_heads():
    selected = torch.tensor([[[[[0, -1, -1], [0, 1, -1], [0, 1, 2]],
                               [[0, -1, -1], [1, -1, -1], [0, 2, -1]]]]], dtype=torch.int32)
    mask = selected_blocks_to_block_mask(selected, layer_idx=0, num_query_heads=4)
    assert mask.shape == (1, 4, 3, 3) and mask.dtype == torch.bool
    g0 = torch.tensor([[1, 0, 0], [1, 1, 0], [1, 1, 1]], dtype=torch.bool)
    g1 = torch.tensor([[1, 0, 0], [0, 1, 0], [1, 0, 1]], dtype=torch.bool)
    for h, want in enumerate((g0, g0, g1, g1)):
        assert torch.equal(mask[0, h], want)


def test_head_indices_preserve_compact_rows():
    selected = torch.tensor([[[[[0, -1], [0, 1]]]]], dtype=torch.int32)
    idx = selected_blocks_to_head_indices(selected, layer_idx=0, num_query_heads=2)
    assert idx.shape == (1, 2, 2, 2) and idx[0, 0].tolist() == [[0, -1], [0, 1]]


def test_dense_layer_dispatch_uses_sdpa():
    torch.manual_seed(9)
    q, k, v = (torch.randn(1, 1, 64, 8) for _ in range(3))
    selected = torch.zeros((1, 1, 1, 1, 1), dtype=torch.int32)
    actual, _ = triton_sparse_prefill_attention_forward(_Module(), q, k, v, None, selected_blocks=selected,
                                                        block_size=64, dense_layers=[0])
    expected = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2)
    torch.testing.assert_close(actual, expected.contiguous())


def test_callback_rejects_masks_block_sizes_and_cpu_tensors():
    q = torch.randn(1, 2, 64, 64)
    k = v = torch.randn(1, 1, 64, 64)
    sel = torch.zeros((1, 1, 1, 1, 1), dtype=torch.int32)
    with pytest.raises(ValueError, match="unpadded"):
        triton_sparse_prefill_attention_forward(_Module(), q, k, v, torch.zeros(1), selected_blocks=sel, block_size=64)
    with pytest.raises(ValueError, match="block_size=64"):
        triton_sparse_prefill_attention_forward(_Module(), q, k, v, None, selected_blocks=sel, block_size=32)
    with pytest.raises(RuntimeError, match="CUDA"):
        triton_sparse_prefill_attention_forward(_Module(), q, k, v, None, selected_blocks=sel, block_size=64)
    with pytest.raises(ValueError, match="kernel_variant"):
        direct_index_sparse_triton(q, k, v, sel[0, 0], 0.1, kernel_variant="nope")
    assert kernel_runtime_metadata(KERNEL_VARIANTS[0])["best_config"] is not None


def test_reference_backend_rejects_decode_shape_and_bad_group_count():
    query = torch.randn(1, 2, 2, 4)
    key = value = torch.randn(1, 1, 3, 4)
    with pytest.raises(ValueError, match="prefill-only"):
        sparse_prefill_attention_forward(_Module(), query, key, value, None, selected_blocks=_selected(),
                                         block_size=2)
    query = key = value = torch.randn(1, 2, 4, 4)
    with pytest.raises(ValueError, match="KV groups"):
        sparse_prefill_attention_forward(_Module(), query, key, value, None, selected_blocks=_selected(groups=1),
                                         block_size=2)


def test_packing_argument_errors_follow_reference():
    with pytest.raises(ValueError, match="cannot fit local window"):
        selected_mask_to_blocks(torch.ones((1, 1, 3, 3), dtype=torch.bool), k_selected=1, local_window=1)
    with pytest.raises(ValueError, match="sink block"):
        selected_ids_to_blocks(torch.zeros((1, 1, 4, 2), dtype=torch.long), k_selected=2, local_window=1,
                               key_blocks=4, sink_blocks=1)


def test_charged_density_counts_dense_layers_as_full_triangles():
    row = [[0, -1], [0, 1], [1, 2], [2, 3]]                 # rows keep min(q+1, 2) of q+1 blocks
    sel = torch.tensor([[[row], [row]]], dtype=torch.int32)  # [B=1, L=2, G=1, qb=4, K=2]
    d = charged_route_density(sel, dense_layers=[1])
    assert d["maximum_causal_block_entries"] == 2 * 10
    assert d["charged_block_entries"] == (1 + 2 + 2 + 2) + 10


def test_block_mask_launcher_checks_and_index_conversion():
    from spruce_research_b200.kernels.seerattention import block_mask_to_indices, block_sparse_triton

    mask = torch.zeros((1, 2, 3, 3), dtype=torch.bool)
    mask[0, 0, 0, 0] = mask[0, 0, 2, 0] = mask[0, 0, 2, 2] = True
    mask[0, 1, 1, 1] = mask[0, 1, 1, 2] = True        # a future column is ignored
    ids = block_mask_to_indices(mask)
    assert ids.dtype == torch.int32 and ids.shape == (1, 2, 3, 2)
    assert ids[0, 0].tolist() == [[0, -1], [-1, -1], [0, 2]]
    assert ids[0, 1].tolist() == [[-1, -1], [1, -1], [-1, -1]]
    q = torch.zeros(1, 2, 130, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        block_sparse_triton(q, q, q, mask, 0.1)


def test_residual_summary_keyword_errors_follow_reference():
    # sparse/attention.py:113-141 of the reference: prototype and mode checks, then the residual
    # checks in order (missing nodes, learned mode without / with a checkpoint, node validation),
    # all before any CUDA requirement
    query = torch.randn(1, 2, 4, 4)
    key = value = torch.randn(1, 2, 4, 4)
    sel = _selected(groups=2)
    args = dict(selected_blocks=sel, block_size=2)
    with pytest.raises(ValueError, match="summary_prototypes must be one of"):
        sparse_prefill_attention_forward(_Module(), query, key, value, None, summary_prototypes=3, **args)
    with pytest.raises(ValueError, match="summary_mode must be one of"):
        sparse_prefill_attention_forward(_Module(), query, key, value, None, summary_mode="max", **args)
    with pytest.raises(ValueError, match="requires residual_summary_nodes"):
        sparse_prefill_attention_forward(_Module(), query, key, value, None, residual_summaries=True, **args)
    nodes = torch.full((1, 1, 2, 2, 1), -1, dtype=torch.int32)
    with pytest.raises(ValueError, match="requires summary_checkpoint"):
        sparse_prefill_attention_forward(_Module(), query, key, value, None, residual_summaries=True,
                                         residual_summary_nodes=nodes, summary_mode="learned", **args)
    with pytest.raises(NotImplementedError, match="learned compressor"):
        sparse_prefill_attention_forward(_Module(), query, key, value, None, residual_summaries=True,
                                         residual_summary_nodes=nodes, summary_mode="learned",
                                         summary_checkpoint="ckpt.pt", **args)


def test_load_gate_reads_the_reference_checkpoint_format_without_unpickling_code(tmp_path):
    """{state_dict: {Wq, Wk}, config: {num_layers, head_dim, proj_dim}}, as the reference's
    selector_ckpt/*.pt files hold (scripts/eval_tree_traversal.py:26-32), loaded with
    torch.load(weights_only=True): plain tensors and a dict only."""
    import pickle
    from fractions import Fraction  # an arbitrary class a weights_only load refuses to unpickle

    from spruce_research_b200.selector.gate import load_gate

    wq, wk = torch.randn(2, 8, 4), torch.randn(2, 8, 4)
    path = tmp_path / "gate.pt"
    torch.save({"state_dict": {"Wq": wq, "Wk": wk}, "config": {"num_layers": 2, "head_dim": 8, "proj_dim": 4}}, path)
    gate, cfg = load_gate(str(path), "cpu")
    assert cfg == {"num_layers": 2, "head_dim": 8, "proj_dim": 4}
    assert torch.equal(gate.Wq, wq) and torch.equal(gate.Wk, wk)
    bad = tmp_path / "bad.pt"
    torch.save({"state_dict": {"Wq": wq, "Wk": wk}, "config": Fraction(1, 3)}, bad)
    with pytest.raises(pickle.UnpicklingError):
        load_gate(str(bad), "cpu")
