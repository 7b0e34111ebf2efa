"""``selected_blocks`` validation on the GPU (interfaces/validator.py:7-62 of the reference).

One thread per row checks the reference's rules in its order (causal, sorted,
no duplicates, local window present, trailing padding); the host reads back
only the first violating row and raises the reference's AssertionError text.
"""
from __future__ import annotations

import torch

from .. import native

PAD_VALUE = -1
LOCAL_WINDOW = 1


def validate_selected_blocks(t: torch.Tensor, local_window: int = LOCAL_WINDOW) -> None:
    """Raise AssertionError at the first violating row, as the reference does."""
    assert t.dim() == 5, (
        "Expected 5D tensor [batch, layer, kv_head_group, query_block, "
        f"K_selected_blocks], got {t.dim()}D with shape {tuple(t.shape)}")
    assert t.dtype == torch.int32, f"Expected int32, got {t.dtype}"
    assert local_window >= 0, f"local_window must be >= 0, got {local_window}"
    hit = native.validate_first_violation(t, local_window)
    if hit is None:
        return
    flat, rule = hit
    B, L, G, Q, K = t.shape
    b, rest = divmod(flat, L * G * Q)
    l, rest = divmod(rest, G * Q)
    g, q = divmod(rest, Q)
    row = t[b, l, g, q].tolist()
    real = [x for x in row if x != PAD_VALUE]
    where = f"[b={b}, l={l}, g={g}, q={q}]"
    if rule == 1:
        bad = next(x for x in real if x > q)
        raise AssertionError(f"Causal violation at {where}: block {bad} is in the future (q={q})")
    if rule == 2:
        raise AssertionError(f"Not sorted at {where}: {real}")
    if rule == 3:
        raise AssertionError(f"Duplicate block IDs at {where}: {real}")
    if rule == 4:
        missing = [x for x in range(max(0, q - local_window), q + 1) if x not in real]
        raise AssertionError(f"Missing local-window block(s) at {where}: missing {missing}, row={real}")
    raise AssertionError(f"Padding is not trailing-only at {where}: {row}")
