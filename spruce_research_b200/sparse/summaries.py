"""Live K/V summaries of residual-tree nodes (reference: sparse/summaries.py).

``build_kv_summary_table`` pools the post-RoPE keys and values of every tree
node into ``P`` positional prototypes on the GPU (one C-ABI call,
``spruce_kv_summary_table``: segment sums, prefix scan and node gather, see
csrc/summaries.cu).  The table is bit-identical to the reference's CPU
result for bf16/fp16 inputs and for fp32 inputs whose running sums are exact
in double; ``log_counts`` is the correctly rounded float log, which may
differ from torch's CPU float log by one ulp.

Mirrors sparse/summaries.py:13-27 (``KVSummaryTable``), :29-49
(``_prototype_token_ranges``), :52-142 (``build_kv_summary_table``),
:145-163 (``token_validity_from_attention_mask``) and :166-224
(``residual_attention_density``) with the same argument checks and messages.
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache

import torch

from .. import _lib, native
from ..interfaces.residual_summaries import ResidualTreeLayout, build_residual_tree_layout

SUMMARY_PROTOTYPES = (1, 2, 4)


@dataclass(frozen=True)
class KVSummaryTable:
    """Keys/values ``[B, Hkv, node, P, D]`` fp32; counts/log_counts ``[B, node, P]``;
    range_starts/range_ends ``[node, P]`` token offsets."""

    keys: torch.Tensor
    values: torch.Tensor
    counts: torch.Tensor
    log_counts: torch.Tensor
    range_starts: torch.Tensor
    range_ends: torch.Tensor


def _prototype_token_ranges(layout: ResidualTreeLayout, *, seq_len: int, block_size: int, prototypes: int,
                            device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Token ranges ``[node, P]`` of each prototype: equal shares of the node's clamped span."""
    lo = (torch.tensor(layout.starts, dtype=torch.long) * block_size).clamp_max(seq_len)
    hi = (torch.tensor(layout.ends, dtype=torch.long) * block_size).clamp_max(seq_len)
    span = (hi - lo)[:, None]
    p = torch.arange(prototypes + 1, dtype=torch.long)[None, :]
    edges = lo[:, None] + span * p // prototypes
    return edges[:, :-1].to(device), edges[:, 1:].to(device)


@lru_cache(maxsize=32)
def _node_ranges_on(starts: tuple, ends: tuple, device: str) -> tuple[torch.Tensor, torch.Tensor]:
    """The layout's block ranges as int64 device tensors, uploaded once per layout and device."""
    return (torch.tensor(starts, dtype=torch.int64).to(device), torch.tensor(ends, dtype=torch.int64).to(device))


def build_kv_summary_table(key: torch.Tensor, value: torch.Tensor, layout: ResidualTreeLayout, *, block_size: int,
                           prototypes: int, token_mask: torch.Tensor | None = None) -> KVSummaryTable:
    """Positional means of live K/V per tree node (CUDA; no CPU fallback)."""
    if key.dim() != 4 or value.dim() != 4:
        raise ValueError("key and value must be [batch, kv_heads, tokens, head_dim]")
    if key.shape != value.shape:
        raise ValueError(f"key/value shape mismatch: {key.shape} vs {value.shape}")
    if block_size < 1:
        raise ValueError(f"block_size must be positive, got {block_size}")
    if prototypes not in SUMMARY_PROTOTYPES:
        raise ValueError(f"prototypes must be one of {SUMMARY_PROTOTYPES}, got {prototypes}")
    batch, _, seq_len, _ = key.shape
    leaves = (seq_len + block_size - 1) // block_size
    if layout.num_leaves != leaves:
        raise ValueError(f"tree has {layout.num_leaves} leaves, expected {leaves} "
                         f"for seq_len={seq_len}, block_size={block_size}")
    if token_mask is not None and token_mask.shape != (batch, seq_len):
        raise ValueError(f"token_mask must be {(batch, seq_len)}, got {tuple(token_mask.shape)}")
    dev = key.device
    _lib.require_cuda(key, value)
    starts, ends = _node_ranges_on(layout.starts, layout.ends, str(dev))
    valid = None if token_mask is None else token_mask.to(device=dev, dtype=torch.bool)
    t = native.kv_summary_table(key, value, starts, ends, block_size, prototypes, valid)
    return KVSummaryTable(t["keys"], t["values"], t["counts"], t["log_counts"], t["range_starts"],
                          t["range_ends"])


def token_validity_from_attention_mask(attention_mask: torch.Tensor | None, *, batch: int,
                                       seq_len: int) -> torch.Tensor | None:
    """bool ``[B, T]``: a key is valid when some query row may attend to it."""
    if attention_mask is None:
        return None
    if attention_mask.dim() != 4:
        raise ValueError("residual summaries expect a 4D additive attention mask, "
                         f"got {tuple(attention_mask.shape)}")
    if attention_mask.shape[0] != batch or attention_mask.shape[-1] != seq_len:
        raise ValueError("attention mask batch/key dimensions do not match K/V")
    return (attention_mask[:, 0] >= 0).any(dim=-2)


def residual_attention_density(selected_blocks: torch.Tensor, residual_summary_nodes: torch.Tensor, *,
                               seq_len: int, block_size: int, prototypes: int) -> dict:
    """Attention entries charged to exact blocks (block_size each) and non-empty prototypes (one each)."""
    if selected_blocks.dim() != 5 or residual_summary_nodes.dim() != 5:
        raise ValueError("selected and residual routes must both be 5D")
    if selected_blocks.shape[:4] != residual_summary_nodes.shape[:4]:
        raise ValueError("selected and residual routes must match through Q")
    if prototypes not in SUMMARY_PROTOTYPES:
        raise ValueError(f"prototypes must be one of {SUMMARY_PROTOTYPES}, got {prototypes}")
    B, L, G, Q, _ = selected_blocks.shape
    if Q != (seq_len + block_size - 1) // block_size:
        raise ValueError("sequence length and route query-block count disagree")
    tree = build_residual_tree_layout(Q)
    per_node = torch.tensor([min(prototypes, min(e * block_size, seq_len) - min(s * block_size, seq_len))
                             for s, e in zip(tree.starts, tree.ends)], dtype=torch.int64)
    exact = int((selected_blocks >= 0).sum().item()) * block_size
    ids = residual_summary_nodes.detach().to(device="cpu", dtype=torch.long)
    ids = ids[ids >= 0]
    summary = int(per_node.index_select(0, ids).sum().item()) if ids.numel() else 0
    charged = exact + summary
    maximum = B * L * G * Q * (Q + 1) // 2 * block_size
    fraction = charged / maximum if maximum else 0.0
    return {
        "exact_attention_entries": exact,
        "summary_prototype_entries": summary,
        "charged_attention_entries": charged,
        "maximum_causal_attention_entries": maximum,
        "charged_attention_fraction": fraction,
        "charged_sparsity": 1.0 - fraction,
    }
