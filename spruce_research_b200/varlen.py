"""Variable-length batches of sparse-prefill sequences (packed, token-major).

The reference runs one sequence per call (its torch and Triton paths take a
padded ``[B, H, T, D]`` batch of one length).  A packed batch here is the
concatenation of the sequences' token-major projections, ``[total, H, D]``,
with ``cu_seqlens`` the ``n + 1`` token offsets; every sequence but the
last starts on a 64-token block boundary, so block ids stay local to each
sequence exactly as in ``selected_blocks``.  Each sequence runs the full
selector + attention on its own slice, one after another on the current
stream, with the K of its own density (``k_for_density``, the charged density
of scripts/route_overrides.py:21-53), so a sequence's result equals the
single-sequence path's.

``all_causal_selected_blocks`` is the reference's 100%-density route
(benchmarks/all_blocks_equivalence.py:53-68): every causal block, which
must reproduce dense causal attention.
"""
from __future__ import annotations

import math

import torch

from .interfaces.validator import PAD_VALUE
from .pipeline import BLOCK, SparsePrefillLayer
from .synthetic import k_for_density


def all_causal_selected_blocks(*, num_layers: int, num_kv_groups: int, seq_len: int,
                               block_size: int = 64) -> torch.Tensor:
    """int32 ``[1, L, G, qb, qb]``: row q lists blocks 0..q, then -1."""
    if min(num_layers, num_kv_groups, seq_len, block_size) < 1:
        raise ValueError("layers, groups, sequence length, and block size must be positive")
    qb = math.ceil(seq_len / block_size)
    cols = torch.arange(qb, dtype=torch.int32)
    rows = torch.where(cols[None, :] <= cols[:, None], cols[None, :].expand(qb, qb),
                       torch.full((qb, qb), PAD_VALUE, dtype=torch.int32))
    return rows[None, None, None].expand(1, num_layers, num_kv_groups, qb, qb).clone()


def check_cu_seqlens(cu_seqlens, total: int) -> list[int]:
    offs = [int(x) for x in (cu_seqlens.tolist() if torch.is_tensor(cu_seqlens) else cu_seqlens)]
    if len(offs) < 2 or offs[0] != 0 or offs[-1] != total:
        raise ValueError(f"cu_seqlens must run from 0 to {total}, got {offs}")
    for a, b in zip(offs, offs[1:]):
        if b <= a:
            raise ValueError(f"cu_seqlens must be strictly increasing, got {offs}")
    if any(o % BLOCK for o in offs[1:-1]):
        raise ValueError(f"sequences must start on {BLOCK}-token block boundaries, got {offs}")
    return offs


class VarlenSparsePrefill:
    """Selector + block-sparse attention over a packed variable-length batch.

    ``wq``/``wk`` are one layer's FlatGate projections; calls take packed
    ``q [total, Hq, D]``, ``k``/``v [total, Hkv, D]`` and ``cu_seqlens`` and
    return the packed output ``[total, Hq, D]`` and the per-sequence
    ``selected_blocks`` rows ``[1, Hkv, qb_s, K_s]``.
    """

    def __init__(self, wq: torch.Tensor, wk: torch.Tensor, local_window: int = 0, sink_blocks: int = 1):
        self.wq, self.wk = wq, wk
        self.local_window, self.sink_blocks = local_window, sink_blocks
        self._layers: dict[int, SparsePrefillLayer] = {}

    def layer(self, k_selected: int) -> SparsePrefillLayer:
        if k_selected not in self._layers:
            self._layers[k_selected] = SparsePrefillLayer(self.wq, self.wk, k_selected, self.local_window,
                                                          self.sink_blocks)
        return self._layers[k_selected]

    def k_for(self, seq_len: int, density: float | None, k_selected: int | None) -> int:
        qb = (seq_len + BLOCK - 1) // BLOCK
        if (density is None) == (k_selected is None):
            raise ValueError("give exactly one of density and k_selected")
        k = k_for_density(qb, density) if density is not None else int(k_selected)
        return max(k, self.local_window + 1 + self.sink_blocks)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens, *,
                 density: float | None = None, k_selected: int | None = None, out: torch.Tensor | None = None):
        if q.dim() != 3 or k.dim() != 3 or v.shape != k.shape or q.shape[0] != k.shape[0]:
            raise ValueError("expected packed q [total, Hq, D] and k/v [total, Hkv, D]")
        total = q.shape[0]
        offs = check_cu_seqlens(cu_seqlens, total)
        if out is None:
            out = torch.empty_like(q)
        selected = []
        for a, b in zip(offs, offs[1:]):
            # [1, H, T, D] views of the token-major slices (the reference's HF layout)
            qs, ks, vs = (x[a:b].unsqueeze(0).transpose(1, 2) for x in (q, k, v))
            layer = self.layer(self.k_for(b - a, density, k_selected))
            _, sel = layer(qs, ks, vs, out=out[a:b].unsqueeze(0))
            selected.append(sel.clone())
        return out, selected
