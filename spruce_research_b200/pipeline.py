"""One SPRUCE sparse-prefill layer: flat-gate selector + block-sparse attention.

This is the per-layer hot path the benchmarks time: pooled Q/K features,
FlatGate scores, masked top-k packed into ``selected_blocks`` rows, and causal
GQA block-sparse attention over those rows -- four kernel launches (five when
the projections run separately), no host synchronisation, buffers reused
across calls.

Reference composition: teacher/chunked_extract.py:164-172 (feature capture),
selector/gate.py:80-101 (scores), scripts/route_overrides.py:187-205 and
scripts/export_selected_blocks.py:80-175 (top-k -> selected_blocks),
kernels/sparse_prefill.py:55-97 (attention callback).
"""
from __future__ import annotations

import math

import torch

from . import native

BLOCK = 64


class SparsePrefillLayer:
    """Selector + attention of one layer with reusable workspace.

    ``wq``/``wk`` are the layer's FlatGate projections ([d, p] fp32 on the GPU).
    Calls return ``(out [B, T, Hq, D], selected [B, Hkv, qb, K] int32)``.
    """

    def __init__(self, wq: torch.Tensor, wk: torch.Tensor, k_selected: int, local_window: int = 0,
                 sink_blocks: int = 1):
        self.wq = wq.detach().float().contiguous()
        self.wk = wk.detach().float().contiguous()
        self.k_selected = int(k_selected)
        self.local_window = int(local_window)
        self.sink_blocks = int(sink_blocks)
        self._workspace = None

    def launches_per_call(self, batch: int, groups: int, q_blocks: tuple[int, int]) -> int:
        """Kernels one call launches: pool, the projections, select, attention.

        Both projections share one launch (W in shared memory) when the call
        projects at least 1024 rows and W fits that kernel; otherwise each has
        its own (the rule of ``launch_project_pair`` in ``csrc/select.cu``).
        """
        d, p = self.wq.shape
        i0, i1 = q_blocks
        rows = batch * groups * ((i1 - i0) + max(1, i1))
        fused = (16 <= p <= 256 and 256 % p == 0 and d % 4 == 0 and (d * p + 16 * d) * 4 <= 96 * 1024
                 and rows >= 1024)
        return 4 if fused else 5

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


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def chunk_bounds(r0: int, r1: int, chunks: int, schedule: str = "balanced") -> list[int]:
    """Strictly increasing query-block bounds r0 = b_0 < ... < b_C = r1, C <= chunks.

    "equal": the same number of query blocks per chunk.  "balanced": the same
    causal attention work per chunk (bound c at sqrt(r0^2 + (r1^2 - r0^2) c / C)).
    """
    C = max(1, min(chunks, r1 - r0))
    if schedule == "equal":
        return [r0 + (r1 - r0) * c // C for c in range(C + 1)]
    bounds = [r0]
    for c in range(1, C):
        b = int(round(math.sqrt(r0 * r0 + (r1 * r1 - r0 * r0) * c / C)))
        if bounds[-1] < b < r1:
            bounds.append(b)
    bounds.append(r1)
    return bounds


class HostStreamedLayer:
    """One layer fed from pinned host buffers, pipelined over query-block chunks.

    Chunk c covers query blocks [i0, i1).  Causality means its selection and
    attention read only K/V blocks < i1, i.e. chunks 0..c, so three streams
    overlap the host->device copy of chunk c+1, the selector + attention of
    chunk c and the device->host copy of chunk c-1.  The PCIe copies, not
    the kernels, bound a layer fed from the host (1.2 GB in, 0.94 GB out per
    128K layer), and here they overlap each other and the compute.

    ``after_attention(i0, i1)`` runs on the compute stream after each
    chunk's attention (the multi-GPU fence of the fused output all-gather).

    ``schedule="balanced"`` (default) places the chunk bounds so that every
    chunk holds the same causal attention work (work up to query block i
    grows as i^2, so bound c sits at sqrt(r0^2 + (r1^2 - r0^2) c / C)): the
    last chunk, whose compute and copy-back nobody overlaps, stays short.
    ``schedule="equal"`` gives every chunk the same number of query blocks.
    """

    def __init__(self, layer: SparsePrefillLayer, device, chunks: int = 16, schedule: str = "balanced"):
        if schedule not in ("balanced", "equal"):
            raise ValueError(f"unknown chunk schedule {schedule!r}")
        self.layer = layer
        self.chunks = chunks
        self.schedule = schedule
        self.h2d = torch.cuda.Stream(device)
        self.compute = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self._sel = None

    def __call__(self, hq, hk, hv, dq, dk, dv, dout, hout=None, q_blocks=None, peer_outs=None,
                 after_attention=None, copy_out=True):
        """hq/hk/hv pinned token-major [B, T, H, D]; dq/dk/dv/dout device tensors of the same shapes.

        Only query blocks ``q_blocks`` (default: all) are computed: their
        query rows and the key/value rows up to their end are copied in.
        ``dout`` receives the layer output ([B, T, Hq, D]); with ``hout`` and
        ``copy_out`` those rows are streamed back to the host chunk by chunk.
        The bytes moved are left in ``h2d_bytes`` / ``d2h_bytes``.
        """
        B, T, Hq, D = hq.shape
        Hkv = hk.shape[2]
        qb = (T + BLOCK - 1) // BLOCK
        r0, r1 = (0, qb) if q_blocks is None else q_blocks
        bounds = chunk_bounds(r0, r1, self.chunks, self.schedule)
        C = len(bounds) - 1
        dev = dq.device
        if self._sel is None or self._sel.shape != (B, Hkv, qb, self.layer.k_selected) or self._sel.device != dev:
            self._sel = torch.empty((B, Hkv, qb, self.layer.k_selected), device=dev, dtype=torch.int32)
        cur = torch.cuda.current_stream(dev)
        for s in (self.h2d, self.compute, self.d2h):
            s.wait_stream(cur)
        qv, kv, vv = dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)
        loaded = 0  # K/V tokens already on the device (rows of earlier chunks stay resident)
        self.h2d_bytes = self.d2h_bytes = 0
        for c in range(C):
            i0, i1 = bounds[c], bounds[c + 1]
            t0, t1 = i0 * BLOCK, min(i1 * BLOCK, T)
            h_done = torch.cuda.Event()
            with torch.cuda.stream(self.h2d):
                # this chunk's queries, and every key/value row up to its last token that it may attend
                dq[:, t0:t1].copy_(hq[:, t0:t1], non_blocking=True)
                dk[:, loaded:t1].copy_(hk[:, loaded:t1], non_blocking=True)
                dv[:, loaded:t1].copy_(hv[:, loaded:t1], non_blocking=True)
                h_done.record()
            self.h2d_bytes += _nbytes(hq[:, t0:t1]) + 2 * _nbytes(hk[:, loaded:t1])
            loaded = t1
            c_done = torch.cuda.Event()
            with torch.cuda.stream(self.compute):
                self.compute.wait_event(h_done)
                sel = self.layer.select(qv, kv, out=self._sel, q_blocks=(i0, i1))
                native.sparse_attention(qv, kv, vv, sel, out=dout, q_blocks=(i0, i1), peer_outs=peer_outs)
                if after_attention is not None:
                    after_attention(i0, i1)
                c_done.record()
            if hout is not None and copy_out:
                with torch.cuda.stream(self.d2h):
                    self.d2h.wait_event(c_done)
                    hout[:, t0:t1].copy_(dout[:, t0:t1], non_blocking=True)
                self.d2h_bytes += _nbytes(hout[:, t0:t1])
        for s in (self.h2d, self.compute, self.d2h):
            cur.wait_stream(s)
        return dout
