"""Block-mask sparse attention with the reference's legacy launcher signature.

Mirrors ``block_sparse_triton`` (kernels/seerattention_triton.py:71-90 of
the reference): causal 64-token block attention of ``[B, H, T, D]`` q/k/v
(K/V already expanded to the query heads) over a per-head boolean block
mask ``[B, H, ceil(T/64), ceil(T/64)]``, output ``[B, H, T, D]``.  The
reference scans every causal column of the mask; here the mask's causal
true entries become ascending per-row block ids and the same sm_100a
kernels as the direct-index path run them with one query head per group.

One deliberate difference: a row whose mask selects no causal block is
0 / 0 = NaN in the reference; here it is zeros, and the optional ``status``
word receives SPRUCE_STATUS_EMPTY_ROW.
"""
from __future__ import annotations

import torch

from .. import native

PAD = -1


def block_mask_to_indices(block_mask: torch.Tensor) -> torch.Tensor:
    """bool ``[B, H, Qb, Kb]`` -> int32 ``[B, H, Qb, K]`` ascending causal ids, -1 padded.

    Only columns j <= q count (the reference never reads the others, :60-64).
    K is the largest row count (one host read of a scalar).
    """
    B, H, Qb, Kb = block_mask.shape
    cols = torch.arange(Kb, device=block_mask.device)
    causal = cols[None, :] <= torch.arange(Qb, device=block_mask.device)[:, None]
    valid = block_mask.bool() & causal
    width = max(1, int(valid.sum(-1).max().item()))
    key = torch.where(valid, cols.to(torch.int32), torch.full((), Kb, dtype=torch.int32, device=valid.device))
    ids = torch.sort(key, dim=-1).values[..., :width]
    return torch.where(ids >= Kb, torch.full_like(ids, PAD), ids).contiguous()


def block_sparse_triton(q, k, v, block_mask, scale, block_size=64, status=None):
    """Causal block-sparse attention over a per-head block mask (reference :71-90)."""
    if not q.is_cuda:
        raise RuntimeError("the block-mask sparse-prefill backend requires CUDA tensors")
    if block_size != 64:
        raise ValueError("the vendored SeerAttention kernel currently supports block_size=64 only")
    if q.shape != k.shape or q.shape != v.shape or q.shape[2] != k.shape[2]:
        raise ValueError("q, k, and v must have matching [B,H,T,D] shapes")
    if q.shape[-1] not in (64, 128):
        raise ValueError(f"kernel supports head_dim 64 or 128, got {q.shape[-1]}")
    B, H, T, D = q.shape
    qb = (T + block_size - 1) // block_size
    if block_mask.dim() != 4 or tuple(block_mask.shape[:3]) != (B, H, qb) or block_mask.shape[3] < qb:
        raise ValueError(f"block_mask must be [B, H, {qb}, >= {qb}], got {tuple(block_mask.shape)}")
    indices = block_mask_to_indices(block_mask[..., :qb].to(q.device))
    out = torch.empty((B, H, T, D), device=q.device, dtype=q.dtype)
    # the kernel writes through logical [B, H, T, D] strides: give it a [B, T, H, D] view of BHSD storage
    native.sparse_attention(q, k, v, indices, scale=float(scale), out=out.transpose(1, 2), status=status)
    return out
