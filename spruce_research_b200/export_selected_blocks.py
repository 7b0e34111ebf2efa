"""Packing of selector ids into the frozen ``selected_blocks`` format, on the GPU.

Drop-ins for scripts/export_selected_blocks.py:38-175 of the reference, same
policy and argument errors: forced local window (and optional sink) blocks
first, then the smallest causal nonlocal ids that fit, sorted, -1 padded.
"""
from __future__ import annotations

import torch

from . import native


def _check(k_selected, local_window, sink_blocks=0):
    if k_selected < 1:
        raise ValueError(f"k_selected must be >= 1, got {k_selected}")
    if local_window < 0:
        raise ValueError(f"local_window must be >= 0, got {local_window}")
    if sink_blocks < 0:
        raise ValueError(f"sink_blocks must be >= 0, got {sink_blocks}")


@torch.no_grad()
def selected_ids_to_blocks(selected_ids, k_selected, local_window=1, key_blocks=None, sink_blocks=0):
    """``[L, G, qb, C]`` candidate ids -> int32 ``[1, L, G, qb, K]`` (export_selected_blocks.py:80-175)."""
    if selected_ids.dim() != 4:
        raise ValueError(f"selected_ids must be [L,G,qb,C], got {tuple(selected_ids.shape)}")
    _check(k_selected, local_window, sink_blocks)
    if k_selected < local_window + 1 + sink_blocks:
        raise ValueError(f"k_selected={k_selected} cannot fit local window size "
                         f"{local_window + 1} plus {sink_blocks} sink block(s)")
    L, G, qb, C = selected_ids.shape
    kb = qb if key_blocks is None else int(key_blocks)
    if kb < 1:
        raise ValueError(f"key_blocks must be >= 1, got {kb}")
    out = native.pack_selected_ids(selected_ids.reshape(L * G, qb, C), k_selected, local_window, kb,
                                   sink_blocks)
    return out.view(1, L, G, qb, k_selected)


@torch.no_grad()
def selected_mask_to_blocks(selected_mask, k_selected, local_window=1):
    """``[L, G, qb, kb]`` bool mask -> int32 ``[1, L, G, qb, K]`` (export_selected_blocks.py:38-76).

    The mask policy equals id packing of every marked key block with no
    sink (the reference pins this equivalence in its tests), so the mask is
    turned into ids and packed by the same kernel.
    """
    if selected_mask.dim() != 4:
        raise ValueError(f"selected_mask must be [L,G,qb,kb], got {tuple(selected_mask.shape)}")
    _check(k_selected, local_window)
    if k_selected < local_window + 1:
        raise ValueError(f"k_selected={k_selected} cannot fit local window size {local_window + 1}")
    L, G, qb, kb = selected_mask.shape
    ar = torch.arange(kb, device=selected_mask.device, dtype=torch.int64)
    ids = torch.where(selected_mask.bool(), ar, torch.full_like(ar, -1))
    return selected_ids_to_blocks(ids, k_selected, local_window, key_blocks=kb, sink_blocks=0)
