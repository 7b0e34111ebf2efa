"""Multi-GPU split of one sparse-prefill layer (one process per GPU).

KV-head groups are independent through pooling, gating, top-k and attention,
so a layer shards by group: with N GPUs and Hkv groups, N <= Hkv gives each
rank Hkv/N whole groups; N = m * Hkv gives each group to m ranks, each taking
an equal contiguous range of its query blocks (equal output chunks, so one
NCCL all-gather reassembles the layer; the later half of a causal row range
holds ~5% more selected tiles at config 2).  The only exchange is that
all-gather of the per-rank outputs into the token-major [B, T, Hq, D] tensor
the next layer's output projection reads.

Two forms of that all-gather:
* ``fused`` (default): every rank holds a full [B, T, Hq, D] output tensor,
  the tensors are CUDA-IPC mapped into every other rank, and the attention
  kernel's epilogue stores each output row into all of them over NVLink
  while it runs (plain peer stores, no multicast); one tiny NCCL all-reduce
  afterwards orders the peers' reads after every rank's kernel.
* ``nccl``: NCCL all_gather_into_tensor of the per-rank chunks plus a
  permute into the token-major layout.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import native
from .pipeline import SparsePrefillLayer


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    groups: tuple[int, int]     # KV groups [g0, g1)
    q_blocks: tuple[int, int]   # query blocks [i0, i1)
    parts: int                  # ranks per group (1 = whole groups)


def balanced_cuts(query_blocks: int, parts: int, k_selected: int) -> list[int]:
    """Query-block boundaries giving each part about the same selected tiles.

    Row i holds min(i + 1, K) blocks, so equal row counts leave the later part
    with more work (5.4% more in the second half at config 2).
    """
    work = [min(i + 1, k_selected) for i in range(query_blocks)]
    total = sum(work)
    cuts, acc, p = [0], 0, 1
    for i, w in enumerate(work):
        if p < parts and acc + w / 2 > total * p / parts:
            cuts.append(i)
            p += 1
        acc += w
    while len(cuts) < parts:
        cuts.append(query_blocks)
    return cuts + [query_blocks]


def plan(world: int, rank: int, kv_heads: int, query_blocks: int, k_selected: int | None = None) -> Shard:
    """This rank's KV groups and query-block range.

    With ``k_selected`` the query blocks of a group are split by selected
    tiles (:func:`balanced_cuts`) instead of into equal parts; only the fused
    all-gather accepts such unequal chunks.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if world <= kv_heads:
        if kv_heads % world:
            raise ValueError(f"{kv_heads} KV groups do not split evenly over {world} GPUs")
        per = kv_heads // world
        return Shard(rank, world, (rank * per, (rank + 1) * per), (0, query_blocks), 1)
    if world % kv_heads:
        raise ValueError(f"{world} GPUs is not a multiple of {kv_heads} KV groups")
    parts = world // kv_heads
    g, p = divmod(rank, parts)
    if k_selected is not None:
        cuts = balanced_cuts(query_blocks, parts, k_selected)
        return Shard(rank, world, (g, g + 1), (cuts[p], cuts[p + 1]), parts)
    if query_blocks % parts:
        raise ValueError(f"{query_blocks} query blocks do not split into {parts} equal parts")
    chunk = query_blocks // parts
    return Shard(rank, world, (g, g + 1), (p * chunk, (p + 1) * chunk), parts)


class ShardedSparsePrefill:
    """Runs this rank's share of a layer and all-gathers the full output."""

    def __init__(self, shard: Shard, layer: SparsePrefillLayer, group=None):
        self.shard = shard
        self.layer = layer
        self.group = group
        self._local = None
        self._gathered = None

    def local(self, q, k, v):
        """This rank's selector + attention; returns (local_out_chunk, selected)."""
        s = self.shard
        g0, g1 = s.groups
        rep = q.shape[1] // k.shape[1]
        qs, ks, vs = q[:, g0 * rep:g1 * rep], k[:, g0:g1], v[:, g0:g1]
        B, _, T, D = q.shape
        if self._local is None or self._local.shape != (B, T, (g1 - g0) * rep, D):
            self._local = torch.empty((B, T, (g1 - g0) * rep, D), device=q.device, dtype=q.dtype)
        out, sel = self.layer(qs, ks, vs, out=self._local, q_blocks=s.q_blocks)
        i0, i1 = s.q_blocks
        return out[:, i0 * 64:i1 * 64], sel

    def gather(self, chunk: torch.Tensor, kv_heads: int, tokens: int) -> torch.Tensor:
        """All-gather the per-rank chunks and lay them out as [B, T, Hq, D]."""
        import torch.distributed as dist

        s = self.shard
        world = s.world
        chunk = chunk.contiguous()
        B, Tc, Hr, D = chunk.shape
        if self._gathered is None or self._gathered.shape != (world * B, Tc, Hr, D):
            self._gathered = torch.empty((world * B, Tc, Hr, D), device=chunk.device, dtype=chunk.dtype)
        # rank-major concatenation along dim 0 (the form both NCCL and gloo accept)
        dist.all_gather_into_tensor(self._gathered, chunk, group=self.group)
        gathered = self._gathered.view(world, B, Tc, Hr, D)
        if s.parts == 1:
            # [world, B, T, Hq/world, D] -> [B, T, Hq, D]
            return gathered.permute(1, 2, 0, 3, 4).reshape(B, tokens, world * Hr, D)
        # rank = g * parts + p: [G, parts, B, T/parts, rep, D] -> [B, parts, T/parts, G, rep, D]
        x = gathered.view(kv_heads, s.parts, B, Tc, Hr, D).permute(2, 1, 3, 0, 4, 5)
        return x.reshape(B, tokens, kv_heads * Hr, D)


class PeerOutput:
    """A full output tensor on every rank, mapped into every other rank by CUDA IPC."""

    def __init__(self, shape, dtype, device, group=None):
        import torch.distributed as dist

        self.local = torch.empty(shape, dtype=dtype, device=device)
        handle = native.ipc_export(self.local)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self._bases = []
        self.peer_ptrs = []
        for r, (h, off) in enumerate(handles):
            if r == rank:
                continue
            ptr, base = native.ipc_import(h, off)
            self.peer_ptrs.append(ptr)
            self._bases.append(base)
        self._tick = torch.zeros(1, device=device, dtype=torch.int32)
        self.group = group

    def fence(self):
        """Order later reads of ``local`` after every rank's peer stores (stream-ordered)."""
        import torch.distributed as dist

        dist.all_reduce(self._tick, group=self.group)

    def close(self):
        for base in self._bases:
            native.ipc_close(base)
        self._bases = []
        self.peer_ptrs = []
