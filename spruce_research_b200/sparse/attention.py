"""The reference's block-sparse prefill callback, served by the B200 kernels.

Mirrors sparse/attention.py:83-291 of the reference (the torch "correctness"
backend): same keyword interface, input checks and error messages, the
``selected_blocks`` validator, and the token-major ``[B, T, Hq, D]`` output.
Differences, all raised as errors rather than silently changed results:
block_size must be 64 (the kernels' tile) and the HF additive mask must be
None (the kernel applies the causal mask itself).  Shape errors are reported
before row-rule errors.  With ``residual_summaries=True`` the K/V summary table
is built on the GPU (sparse/summaries.py:52-142) and each row's softmax also
covers its residual nodes' summary keys with the log-count bias
(sparse/attention.py:164-265), in the same kernel launch as the selected blocks.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import native
from ..interfaces.residual_summaries import build_residual_tree_layout, validate_residual_summary_nodes
from ..interfaces.validator import validate_selected_blocks
from .summaries import build_kv_summary_table

SPARSE_PREFILL_ATTENTION = "spruce_sparse_prefill"
SUMMARY_PROTOTYPES = (1, 2, 4)
SUMMARY_MODES = ("mean", "learned")


def _layer_index(module: torch.nn.Module) -> int:
    for name in ("layer_idx", "layer_id"):
        value = getattr(module, name, None)
        if value is not None:
            return int(value)
    raise ValueError("Sparse prefill attention needs module.layer_idx (or module.layer_id) "
                     "to select the correct selected_blocks layer.")


def _validate_inputs(query, key, value, selected_blocks, block_size, layer_idx):
    """The checks of sparse/attention.py:41-80, in the same order."""
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4:
        raise ValueError("query, key, and value must be [batch, heads, tokens, head_dim]")
    if key.shape != value.shape:
        raise ValueError(f"key/value shape mismatch: {tuple(key.shape)} vs {tuple(value.shape)}")
    if query.shape[0] != key.shape[0] or query.shape[-1] != key.shape[-1]:
        raise ValueError("query and key must have the same batch size and head dimension")
    if query.shape[-2] != key.shape[-2]:
        raise ValueError("Stage 3.2 is prefill-only: query and key lengths must match "
                         f"(got {query.shape[-2]} and {key.shape[-2]}).")
    if block_size < 1:
        raise ValueError(f"block_size must be positive, got {block_size}")
    if query.shape[1] % key.shape[1]:
        raise ValueError(f"query heads ({query.shape[1]}) must be divisible by KV heads ({key.shape[1]})")
    if selected_blocks.dim() != 5:
        raise ValueError("selected_blocks must be [batch, layer, kv_head_group, query_block, K]")
    batch, layers, groups, query_blocks, _ = selected_blocks.shape
    expected_blocks = math.ceil(query.shape[-2] / block_size)
    if batch != query.shape[0] or layers <= layer_idx:
        raise ValueError(f"selected_blocks shape {tuple(selected_blocks.shape)} does not cover "
                         f"batch {query.shape[0]} and layer {layer_idx}")
    if groups != key.shape[1]:
        raise ValueError(f"selected_blocks has {groups} KV groups, model has {key.shape[1]} KV heads")
    if query_blocks != expected_blocks:
        raise ValueError(f"selected_blocks has {query_blocks} query blocks; expected {expected_blocks} "
                         f"for seq_len={query.shape[-2]} and block_size={block_size}")


def sparse_prefill_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                                     value: torch.Tensor, attention_mask: Optional[torch.Tensor], *,
                                     selected_blocks: torch.Tensor, block_size: int,
                                     validate_selected_blocks_input: bool = True, residual_summaries: bool = False,
                                     residual_summary_nodes: Optional[torch.Tensor] = None,
                                     summary_prototypes: int = 1, summary_mode: str = "mean",
                                     summary_checkpoint: Optional[str] = None,
                                     validate_residual_summary_nodes_input: bool = True,
                                     **kwargs) -> tuple[torch.Tensor, None]:
    """AttentionInterface implementation for sparse prefill (sparse/attention.py:83-274)."""
    del kwargs
    layer_idx = _layer_index(module)
    _validate_inputs(query, key, value, selected_blocks, block_size, layer_idx)
    if summary_prototypes not in SUMMARY_PROTOTYPES:
        raise ValueError(f"summary_prototypes must be one of {SUMMARY_PROTOTYPES}, got {summary_prototypes}")
    if summary_mode not in SUMMARY_MODES:
        raise ValueError(f"summary_mode must be one of {SUMMARY_MODES}, got {summary_mode!r}")
    if residual_summaries:  # the checks of sparse/attention.py:122-141, in order
        if residual_summary_nodes is None:
            raise ValueError("residual_summaries=True requires residual_summary_nodes; "
                             "construct the complete frontier before model forward")
        if summary_mode == "learned":
            if not summary_checkpoint:
                raise ValueError("summary_mode='learned' requires summary_checkpoint")
            raise NotImplementedError("The learned compressor is gated on deterministic-summary "
                                      "evaluation and is not implemented before that gate passes.")
        if validate_residual_summary_nodes_input:
            validate_residual_summary_nodes(selected_blocks, residual_summary_nodes,
                                            validate_selected=not validate_selected_blocks_input)
    if block_size != 64:
        raise ValueError(f"the B200 kernels use 64-token blocks, got block_size={block_size}")
    if attention_mask is not None:
        raise ValueError("the B200 kernels apply the causal mask themselves; pass attention_mask=None "
                         "(padded batches are not supported)")
    if not query.is_cuda:
        raise RuntimeError("sparse prefill on the B200 path requires CUDA tensors")
    if validate_selected_blocks_input:
        validate_selected_blocks(selected_blocks.to(query.device))
    D = query.shape[-1]
    indices = selected_blocks[:, layer_idx].to(device=query.device, dtype=torch.int32)
    if indices.stride(-1) != 1:
        indices = indices.contiguous()
    if not residual_summaries:
        return native.sparse_attention(query, key, value, indices, scale=1.0 / math.sqrt(D)), None
    if residual_summary_nodes.shape[:4] != selected_blocks.shape[:4]:
        raise ValueError("residual_summary_nodes must match selected_blocks through the query-block dimension")
    nodes = residual_summary_nodes[:, layer_idx].to(device=query.device, dtype=torch.int32)
    layout = build_residual_tree_layout(selected_blocks.shape[3])
    table = build_kv_summary_table(key, value, layout, block_size=block_size, prototypes=summary_prototypes)
    out = native.residual_sparse_attention(query, key, value, indices, nodes, table, scale=1.0 / math.sqrt(D))
    return out, None


def register_sparse_prefill_attention(name: str = SPARSE_PREFILL_ATTENTION) -> str:
    """Register with transformers; decode keeps the SDPA mask (sparse/attention.py:277-291)."""
    try:
        from transformers import AttentionInterface, AttentionMaskInterface
        from transformers.masking_utils import sdpa_mask
    except ImportError as error:
        raise RuntimeError("register_sparse_prefill_attention requires transformers") from error
    AttentionInterface.register(name, sparse_prefill_attention_forward)
    AttentionMaskInterface.register(name, sdpa_mask)
    return name
