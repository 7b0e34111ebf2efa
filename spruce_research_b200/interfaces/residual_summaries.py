"""Residual tree over key blocks (reference: interfaces/residual_summaries.py).

Host-side index bookkeeping for the K/V summary table: a leaf-first binary
tree over the ``qb`` key blocks whose node IDs and block ranges address the
rows of :func:`spruce_research_b200.sparse.summaries.build_kv_summary_table`,
plus the maximal frontier of tree nodes covering the causal blocks a
``selected_blocks`` row leaves out.

Same IDs, ranges, padding and assertion messages as the reference
(``ResidualTreeLayout`` :19-71, ``build_residual_tree_layout`` :73-122,
``residual_frontier_for_row`` :125-160, ``build_residual_summary_nodes``
:163-220, ``validate_residual_summary_nodes`` :223-314).
"""
from __future__ import annotations

from bisect import bisect_left
from dataclasses import dataclass
from typing import Iterable, Sequence

import torch

from .validator import PAD_VALUE, validate_selected_blocks


@dataclass(frozen=True)
class ResidualTreeLayout:
    """Node table of the tree: node ``i`` covers blocks ``[starts[i], ends[i])``.

    Level 0 holds the ``num_leaves`` single blocks; level ``l + 1`` has
    ``ceil(level_counts[l] / 2)`` nodes, node ``j`` joining children ``2j`` and
    ``2j + 1`` (an odd last child is carried up alone).  IDs run level by
    level from the leaves: ``node_id(l, j) = level_offsets[l] + j``.
    """

    num_leaves: int
    level_counts: tuple[int, ...]
    level_offsets: tuple[int, ...]
    starts: tuple[int, ...]
    ends: tuple[int, ...]
    levels: tuple[int, ...]
    indices: tuple[int, ...]

    @property
    def num_nodes(self) -> int:
        return len(self.starts)

    @property
    def root_id(self) -> int:
        return self.level_offsets[-1]

    def node_id(self, level: int, index: int) -> int:
        if not 0 <= level < len(self.level_counts):
            raise IndexError(f"tree level {level} is out of range")
        if not 0 <= index < self.level_counts[level]:
            raise IndexError(f"node index {index} is out of range for level {level}")
        return self.level_offsets[level] + index

    def range(self, node_id: int) -> tuple[int, int]:
        if not 0 <= node_id < self.num_nodes:
            raise IndexError(f"tree node ID {node_id} is out of range")
        return self.starts[node_id], self.ends[node_id]

    def children(self, node_id: int) -> tuple[int, ...]:
        if not 0 <= node_id < self.num_nodes:
            raise IndexError(f"tree node ID {node_id} is out of range")
        level = self.levels[node_id]
        if level == 0:
            return ()
        below = self.level_counts[level - 1]
        first = 2 * self.indices[node_id]
        return tuple(self.level_offsets[level - 1] + j for j in (first, first + 1) if j < below)


def build_residual_tree_layout(num_leaves: int) -> ResidualTreeLayout:
    """The node table for ``num_leaves`` key blocks (2 * num_leaves - 1 nodes or fewer)."""
    if num_leaves < 1:
        raise ValueError(f"num_leaves must be >= 1, got {num_leaves}")
    counts = [int(num_leaves)]
    while counts[-1] > 1:
        counts.append((counts[-1] + 1) // 2)
    offsets = [sum(counts[:i]) for i in range(len(counts))]

    starts: list[int] = list(range(num_leaves))
    ends: list[int] = [i + 1 for i in range(num_leaves)]
    levels: list[int] = [0] * num_leaves
    indices: list[int] = list(range(num_leaves))
    for level in range(1, len(counts)):
        lo, n_below = offsets[level - 1], counts[level - 1]
        for j in range(counts[level]):
            left = lo + 2 * j
            right = lo + min(2 * j + 1, n_below - 1)
            starts.append(starts[left])
            ends.append(ends[right])
            levels.append(level)
            indices.append(j)
    return ResidualTreeLayout(int(num_leaves), tuple(counts), tuple(offsets), tuple(starts), tuple(ends),
                              tuple(levels), tuple(indices))


def residual_frontier_for_row(selected_block_ids: Sequence[int] | Iterable[int], query_block: int,
                              layout: ResidualTreeLayout) -> list[int]:
    """Sorted IDs of the largest nodes that cover the causal blocks the row omits.

    A node is taken whole when it lies inside the causal prefix ``[0, q]`` and
    holds no selected block; otherwise its children are examined.
    """
    if not 0 <= query_block < layout.num_leaves:
        raise ValueError(f"query_block must be in [0, {layout.num_leaves}), got {query_block}")
    chosen = sorted({int(b) for b in selected_block_ids if b >= 0})
    if chosen and chosen[-1] > query_block:
        raise ValueError("selected block IDs must be causal and non-negative")
    limit = query_block + 1
    frontier: list[int] = []
    stack = [layout.root_id]
    while stack:
        node = stack.pop()
        start, end = layout.starts[node], layout.ends[node]
        if start >= limit:
            continue
        i = bisect_left(chosen, start)
        holds_selected = i < len(chosen) and chosen[i] < end
        if end <= limit and not holds_selected:
            frontier.append(node)
        else:
            stack.extend(layout.children(node))
    return sorted(frontier)


def layout_arrays(layout: ResidualTreeLayout, device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The node table on ``device``: starts / ends int64 and parents int32 (-1 for the root)."""
    key = (layout.num_leaves, str(device))
    hit = _LAYOUT_ARRAYS.get(key)
    if hit is None:
        top = len(layout.level_counts) - 1
        parents = [layout.level_offsets[lv + 1] + idx // 2 if lv < top else -1
                   for lv, idx in zip(layout.levels, layout.indices)]
        hit = (torch.tensor(layout.starts, dtype=torch.int64, device=device),
               torch.tensor(layout.ends, dtype=torch.int64, device=device),
               torch.tensor(parents, dtype=torch.int32, device=device))
        _LAYOUT_ARRAYS[key] = hit
    return hit


_LAYOUT_ARRAYS: dict = {}


def _rows(t: torch.Tensor):
    a = t.detach().to(device="cpu")
    B, L, G, Q = a.shape[:4]
    for b in range(B):
        for l in range(L):
            for g in range(G):
                for q in range(Q):
                    yield (b, l, g, q), a[b, l, g, q].tolist()


def build_residual_summary_nodes(selected_blocks: torch.Tensor, *, layout: ResidualTreeLayout | None = None,
                                 validate_selected: bool = True) -> torch.Tensor:
    """int32 ``[B, L, G, Q, S]`` frontiers, -1 padded; S is the longest frontier (0 if none)."""
    if validate_selected:
        validate_selected_blocks(selected_blocks)
    if selected_blocks.dim() != 5:
        raise ValueError("selected_blocks must be [B,L,G,Q,K]")
    if selected_blocks.dtype != torch.int32:
        raise ValueError(f"selected_blocks must be int32, got {selected_blocks.dtype}")
    B, L, G, Q, _ = selected_blocks.shape
    if layout is None:
        layout = build_residual_tree_layout(Q)
    elif layout.num_leaves != Q:
        raise ValueError(f"tree has {layout.num_leaves} leaves but selected_blocks has {Q} query blocks")
    if selected_blocks.is_cuda:  # one GPU launch per pass instead of a Python walk per row
        from .. import native

        starts, ends, parents = layout_arrays(layout, selected_blocks.device)
        return native.residual_frontier(selected_blocks, starts, ends, parents)
    frontiers = {}
    for (b, l, g, q), row in _rows(selected_blocks):
        frontiers[b, l, g, q] = residual_frontier_for_row([x for x in row if x != PAD_VALUE], q, layout)
    width = max((len(f) for f in frontiers.values()), default=0)
    out = torch.full((B, L, G, Q, width), PAD_VALUE, dtype=torch.int32)
    for (b, l, g, q), f in frontiers.items():
        if f:
            out[b, l, g, q, :len(f)] = torch.tensor(f, dtype=torch.int32)
    return out.to(device=selected_blocks.device)


def validate_residual_summary_nodes(selected_blocks: torch.Tensor, residual_summary_nodes: torch.Tensor, *,
                                    require_maximal: bool = True, validate_selected: bool = True) -> None:
    """Exact blocks plus residual nodes must cover each causal prefix exactly once."""
    if validate_selected:
        validate_selected_blocks(selected_blocks)
    assert residual_summary_nodes.dim() == 5, (
        "Expected residual_summary_nodes [batch, layer, kv_head_group, "
        f"query_block, S], got {tuple(residual_summary_nodes.shape)}")
    assert residual_summary_nodes.dtype == torch.int32, (
        f"Expected residual_summary_nodes int32, got {residual_summary_nodes.dtype}")
    assert residual_summary_nodes.shape[:4] == selected_blocks.shape[:4], (
        "selected_blocks and residual_summary_nodes must have identical "
        f"[batch, layer, group, query] dimensions, got {tuple(selected_blocks.shape[:4])} and "
        f"{tuple(residual_summary_nodes.shape[:4])}")
    layout = build_residual_tree_layout(selected_blocks.shape[3])
    residual_rows = dict(_rows(residual_summary_nodes))
    for (b, l, g, q), sel_row in _rows(selected_blocks):
        where = f"b={b}, l={l}, g={g}, q={q}"
        exact = [x for x in sel_row if x != PAD_VALUE]
        padded = residual_rows[b, l, g, q]
        nodes = [x for x in padded if x != PAD_VALUE]
        if PAD_VALUE in padded:
            first = padded.index(PAD_VALUE)
            assert all(x == PAD_VALUE for x in padded[first:]), f"Residual padding is not trailing-only at [{where}]"
        assert nodes == sorted(nodes), f"Residual node IDs are not sorted at [{where}]: {nodes}"
        assert len(nodes) == len(set(nodes)), f"Duplicate residual node IDs at [{where}]: {nodes}"
        coverage = [0] * (q + 1)
        for blk in exact:
            assert 0 <= blk <= q, f"Non-causal exact block {blk} at [{where}]"
            coverage[blk] += 1
        for node in nodes:
            assert 0 <= node < layout.num_nodes, f"Unknown residual node ID {node} at [{where}]"
            start, end = layout.range(node)
            assert end <= q + 1, (
                f"Residual node {node} range [{start}, {end}) is partially or wholly future at [{where}]")
            for blk in range(start, end):
                coverage[blk] += 1
        assert all(c == 1 for c in coverage), (
            "Exact and residual routes do not form a disjoint complete "
            f"causal partition at [{where}]: coverage={coverage}")
        if require_maximal:
            expected = residual_frontier_for_row(exact, q, layout)
            assert nodes == expected, (
                f"Residual frontier is complete but not maximal at [{where}]: expected {expected}, got {nodes}")
