"""Direct-index block-sparse attention with the reference kernel's signature.

Mirrors kernels/seerattention_direct_index_triton.py:339-448 of the
reference: same arguments, shapes, checks and error classes, backed by the
sm_100a tcgen05 kernel (bf16/fp16) or the CUDA-core fp32 kernel through the C
ABI.  There is no Triton and one implementation, so ``kernel_variant`` is
validated against the reference's names and otherwise ignored.
"""
from __future__ import annotations

import torch

from .. import native

KERNEL_VARIANTS = (
    "single_head",
    "single_head_causal",
    "single_head_prescale",
    "single_head_qtile",
    "tiled_gqa",
)


def direct_index_sparse_triton(q, k, v, indices, scale, block_size=64, kernel_variant="single_head"):
    """Causal block-sparse attention over exactly the supplied block ids.

    q is ``[B, Hq, T, D]``; k/v and indices keep native KV-group resolution
    ``[B, Hkv, T, D]`` / ``[B, Hkv, ceil(T/64), K]``.  Inputs may be the strided
    views Qwen's projections produce; the output is a fresh contiguous
    ``[B, T, Hq, D]`` (seerattention_direct_index_triton.py:339-416).
    """
    if kernel_variant not in KERNEL_VARIANTS:
        raise ValueError(f"kernel_variant must be one of {KERNEL_VARIANTS}, got {kernel_variant!r}")
    if not q.is_cuda:
        raise RuntimeError("the direct-index B200 backend requires CUDA tensors")
    if block_size != 64:
        raise ValueError("direct-index kernel currently supports block_size=64 only")
    if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:]:
        raise ValueError("q and k/v must match in batch, tokens, and head_dim")
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must be divisible by KV heads")
    qblocks = (T + block_size - 1) // block_size
    if tuple(indices.shape[:3]) != (B, Hkv, qblocks) or indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [B,Hkv,ceil(T/64),K]")
    if D not in (64, 128):
        raise ValueError(f"kernel supports head_dim 64 or 128, got {D}")
    if any(x.stride(-1) != 1 for x in (q, k, v, indices)):
        raise ValueError("q, k, v, and indices must have a contiguous final dimension")
    return native.sparse_attention(q, k, v, indices, scale=scale)


# The B200 name for the same entry point.
direct_index_sparse = direct_index_sparse_triton


def kernel_runtime_metadata(kernel_variant):
    """Which kernel serves a variant (reference: autotune choice, :430-448)."""
    if kernel_variant not in KERNEL_VARIANTS:
        raise ValueError(f"kernel_variant must be one of {KERNEL_VARIANTS}, got {kernel_variant!r}")
    import os

    if os.environ.get("SPRUCE_ATTN_KERNEL") == "single":  # the one-block-per-step kernel, kept for comparison
        cfg = {"kernel": "attn_fwd_sm100_kernel", "tile_rows": 128, "heads_per_tile": 2, "tiles_per_cta": 2,
               "blocks_per_step": 1, "kv_stages": 4, "threads": 352}
    else:  # the default: two selected blocks per step (attn_pair_sm100.cu)
        cfg = {"kernel": "attn_pair_sm100_kernel", "tile_rows": 128, "heads_per_tile": 2, "tiles_per_cta": 2,
               "blocks_per_step": 2, "kv_stages": {64: 4, 128: 2}, "threads": 320}
    cfg["fp32_kernel"] = "attn_fwd_f32_kernel"
    return {"variant": kernel_variant, "best_config": cfg}
