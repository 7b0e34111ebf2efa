"""SPRUCE selected-block adapters and the HF attention callback (B200 backend).

Mirrors kernels/sparse_prefill.py of the reference: the same callback
signature, decode and dense-layer dispatch to SDPA, the same checks and the
same index adapters, with the block-sparse path served by the sm_100a kernel.
"""
from __future__ import annotations

import math

import torch

from .direct_index import KERNEL_VARIANTS, direct_index_sparse_triton, kernel_runtime_metadata  # noqa: F401

SPRUCE_TRITON_SPARSE_PREFILL = "spruce_triton_sparse_prefill"
SPRUCE_B200_SPARSE_PREFILL = SPRUCE_TRITON_SPARSE_PREFILL


def selected_blocks_to_block_mask(selected_blocks, *, layer_idx, num_query_heads):
    """``[B, L, Gkv, Qb, K]`` ids -> ``[B, Hq, Qb, Qb]`` bool block mask (kernels/sparse_prefill.py:16-39)."""
    if selected_blocks.dim() != 5:
        raise ValueError("selected_blocks must be [B,L,Gkv,Qb,K]")
    B, L, Gkv, qblocks, _ = selected_blocks.shape
    if not 0 <= layer_idx < L:
        raise ValueError(f"layer_idx {layer_idx} is outside selected_blocks layers={L}")
    if num_query_heads % Gkv:
        raise ValueError("num_query_heads must be divisible by selected KV groups")
    # mask[b, h, i, j] holds when block j is one of row i's ids in head h's KV group; -1 padding
    # and ids outside [0, Qb) equal no block column, so they mark nothing.
    rows = selected_blocks[:, layer_idx].to(torch.long)                        # [B, Gkv, Qb, K]
    blocks = torch.arange(qblocks, device=rows.device)
    mask = (rows[..., :, None] == blocks).any(dim=-2)                          # [B, Gkv, Qb, Qb]
    return mask.repeat_interleave(num_query_heads // Gkv, dim=1).contiguous()


def selected_blocks_to_head_indices(selected_blocks, *, layer_idx, num_query_heads):
    """Expand KV-group rows to query heads (kernels/sparse_prefill.py:42-52)."""
    if selected_blocks.dim() != 5:
        raise ValueError("selected_blocks must be [B,L,Gkv,Qb,K]")
    _, layers, kv_groups, _, _ = selected_blocks.shape
    if not 0 <= layer_idx < layers:
        raise ValueError(f"layer_idx {layer_idx} is outside selected_blocks layers={layers}")
    if num_query_heads % kv_groups:
        raise ValueError("num_query_heads must be divisible by selected KV groups")
    return selected_blocks[:, layer_idx].repeat_interleave(num_query_heads // kv_groups, dim=1).contiguous()


def _sdpa(module, query, key, value, attention_mask, **kwargs):
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    return sdpa_attention_forward(module, query, key, value, attention_mask, **kwargs)


def triton_sparse_prefill_attention_forward(module, query, key, value, attention_mask, *, selected_blocks,
                                            block_size, kernel_variant="single_head", dense_layers=(), **kwargs):
    """Transformers AttentionInterface callback (prefill only), kernels/sparse_prefill.py:55-97.

    Decode calls (q_len != k_len) and ``dense_layers`` go to SDPA exactly as
    in the reference; every other layer runs the block-sparse B200 kernel on
    ``selected_blocks[:, module.layer_idx]``.
    """
    if query.shape[-2] != key.shape[-2]:
        return _sdpa(module, query, key, value, attention_mask, **kwargs)
    if attention_mask is not None:
        raise ValueError("B200 SPRUCE prefill currently supports unpadded batch-size-1 inputs only")
    if key.shape != value.shape:
        raise ValueError("key and value must have matching shapes")
    if block_size != 64:
        raise ValueError("B200 SPRUCE backend currently requires block_size=64")
    layer_idx = int(getattr(module, "layer_idx"))
    if dense_layers and layer_idx in {int(layer) for layer in dense_layers}:
        return _sdpa(module, query, key, value, attention_mask, **kwargs)
    B, Hq, T, D = query.shape
    Hkv = key.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must divide evenly into KV groups")
    if selected_blocks.shape[0] != B or selected_blocks.shape[2] != Hkv:
        raise ValueError("selected_blocks batch/KV-group dimensions do not match Qwen attention")
    if selected_blocks.shape[3] != math.ceil(T / block_size):
        raise ValueError("selected_blocks query-block count does not match sequence length")
    indices = selected_blocks[:, layer_idx]
    if indices.stride(-1) != 1:
        indices = indices.contiguous()
    output = direct_index_sparse_triton(query, key, value, indices, scale=D ** -0.5, block_size=block_size,
                                        kernel_variant=kernel_variant)
    return output, None


b200_sparse_prefill_attention_forward = triton_sparse_prefill_attention_forward


def _sparse_attention_mask(*args, **kwargs):
    """No O(T^2) mask at prefill; SDPA's mask for decode (kernels/sparse_prefill.py:100-107)."""
    q_length = kwargs.get("q_length", args[1] if len(args) > 1 else None)
    kv_length = kwargs.get("kv_length", args[2] if len(args) > 2 else None)
    if q_length == kv_length:
        return None
    from transformers.masking_utils import sdpa_mask

    return sdpa_mask(*args, **kwargs)


def register_triton_sparse_prefill_attention(name=SPRUCE_TRITON_SPARSE_PREFILL):
    """Register the B200 backend with transformers (kernels/sparse_prefill.py:110-121)."""
    try:
        from transformers import AttentionInterface, AttentionMaskInterface
    except ImportError as error:
        raise RuntimeError("registration requires transformers") from error
    AttentionInterface.register(name, triton_sparse_prefill_attention_forward)
    AttentionMaskInterface.register(name, _sparse_attention_mask)
    return name
