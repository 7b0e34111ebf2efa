"""One SPRUCE sparse-prefill layer: flat-gate selector + block-sparse attention.

This is the per-layer hot path the benchmarks time: pooled Q/K features,
FlatGate scores, masked top-k packed into ``selected_blocks`` rows, and causal
GQA block-sparse attention over those rows -- five kernel launches, no host
synchronisation, buffers reused across calls.

Reference composition: teacher/chunked_extract.py:164-172 (feature capture),
selector/gate.py:80-101 (scores), scripts/route_overrides.py:187-205 and
scripts/export_selected_blocks.py:80-175 (top-k -> selected_blocks),
kernels/sparse_prefill.py:55-97 (attention callback).
"""
from __future__ import annotations

import torch

from . import native

BLOCK = 64


class SparsePrefillLayer:
    """Selector + attention of one layer with reusable workspace.

    ``wq``/``wk`` are the layer's FlatGate projections ([d, p] fp32 on the GPU).
    Calls return ``(out [B, T, Hq, D], selected [B, Hkv, qb, K] int32)``.
    """

    #: kernels launched per call (pool, 2 projections, select, attention)
    LAUNCHES_PER_CALL = 5

    def __init__(self, wq: torch.Tensor, wk: torch.Tensor, k_selected: int, local_window: int = 0,
                 sink_blocks: int = 1):
        self.wq = wq.detach().float().contiguous()
        self.wk = wk.detach().float().contiguous()
        self.k_selected = int(k_selected)
        self.local_window = int(local_window)
        self.sink_blocks = int(sink_blocks)
        self._workspace = None

    def select(self, q: torch.Tensor, k: torch.Tensor, out: torch.Tensor | None = None,
               q_blocks: tuple[int, int] | None = None) -> torch.Tensor:
        need = native.select_workspace_bytes(q, k, self.wq.shape[1])
        if self._workspace is None or self._workspace.numel() < need or self._workspace.device != q.device:
            self._workspace = torch.empty(max(need, 16), device=q.device, dtype=torch.uint8)
        return native.select_blocks(q, k, self.wq, self.wk, self.k_selected, self.local_window,
                                    self.sink_blocks, out=out, workspace=self._workspace, q_blocks=q_blocks)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None,
                 selected: torch.Tensor | None = None, q_blocks: tuple[int, int] | None = None):
        selected = self.select(q, k, out=selected, q_blocks=q_blocks)
        out = native.sparse_attention(q, k, v, selected, out=out, q_blocks=q_blocks)
        return out, selected


def sparse_prefill_layer(q, k, v, wq, wk, k_selected, local_window=0, sink_blocks=1):
    """Functional form of :class:`SparsePrefillLayer` (allocates its buffers)."""
    return SparsePrefillLayer(wq, wk, k_selected, local_window, sink_blocks)(q, k, v)
