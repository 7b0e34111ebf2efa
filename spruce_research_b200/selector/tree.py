"""Key-axis tree and beam traversal of the deployed selector, on the GPU.

Mirrors selector/tree.py:18-145 (``KeyTreeLevel``, ``build_key_tree``) and
scripts/eval_tree_traversal.py:60-113 (``traverse_to_leaf_ids``) of the
reference: the same levels, node ranges and traversal rules, computed by
csrc/tree.cu (level merge, candidates, beam top-k) and the MaxSim kernel.
Ties (equal prototype distances, equal candidate scores) go to the lower
index; torch.topk leaves their order open.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import native


@dataclass(frozen=True)
class KeyTreeLevel:
    """features ``[L, G, nodes, P, d]``; starts/ends ``[nodes]`` leaf-block ranges."""

    level: int
    features: torch.Tensor
    starts: torch.Tensor
    ends: torch.Tensor


def _level_ranges(kb: int, radix: int) -> list[tuple[list[int], list[int]]]:
    """Leaf-block ranges of every level: parent j spans children j*radix .. (j+1)*radix - 1 (selector/tree.py:116-145)."""
    starts, ends = list(range(kb)), list(range(1, kb + 1))
    out = [(starts, ends)]
    while len(starts) > 1:
        n = len(starts)
        m = (n + radix - 1) // radix
        starts = [starts[j * radix] for j in range(m)]
        ends = [ends[min((j + 1) * radix, n) - 1] for j in range(m)]
        out.append((starts, ends))
    return out


_RANGE_CACHE: dict = {}


def _level_range_tensors(kb: int, radix: int, device) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """The ranges as int64 tensors on ``device``, built once per (kb, radix, device) and shared (read-only)."""
    key = (kb, radix, str(device))
    hit = _RANGE_CACHE.get(key)
    if hit is None:
        ranges = _level_ranges(kb, radix)
        flat = torch.tensor([x for st, en in ranges for x in st + en], dtype=torch.int64).to(device)
        hit, off = [], 0
        for st, en in ranges:
            hit.append((flat[off:off + len(st)], flat[off + len(st):off + 2 * len(st)]))
            off += 2 * len(st)
        _RANGE_CACHE[key] = hit
    return hit


def build_key_tree(k_feat: torch.Tensor, radix: int = 2) -> list[KeyTreeLevel]:
    """Levels leaf-first from leaf key features ``[L, G, kb, P, d]``; odd tails are smaller parents."""
    if radix < 2:
        raise ValueError(f"radix must be >= 2, got {radix}")
    if k_feat.dim() != 5:
        raise ValueError(f"k_feat must be [L,G,kb,P,d], got {tuple(k_feat.shape)}")
    L, G, kb, P, d = k_feat.shape
    ranges = _level_range_tensors(kb, radix, k_feat.device)  # pure functions of kb and radix
    levels = [KeyTreeLevel(0, k_feat, *ranges[0])]
    current = k_feat.reshape(L * G, kb, P, d)
    level = 0
    while current.shape[1] > 1:
        level += 1
        current = native.tree_merge(current, radix)
        levels.append(KeyTreeLevel(level, current.view(L, G, -1, P, d), *ranges[level]))
    return levels


@torch.no_grad()
def traverse_to_leaf_ids(gate, q_feat: torch.Tensor, key_levels: list[KeyTreeLevel], beam: int, radix: int = 2,
                         layer_chunk: int = 1) -> torch.Tensor:
    """Compact selected leaf ids ``[L, G, qb, C]`` (C = min(beam, ...)), -1 in invalid slots."""
    if beam < 1:
        raise ValueError(f"beam must be >= 1, got {beam}")
    if radix < 2:
        raise ValueError(f"radix must be >= 2, got {radix}")
    if layer_chunk < 1:
        raise ValueError(f"layer_chunk must be >= 1, got {layer_chunk}")
    L, G, qb = q_feat.shape[:3]
    if key_levels[-1].features.shape[2] != 1:
        raise ValueError("key tree must end in exactly one root node")
    R = L * G
    selected = torch.zeros((R, qb, 1), dtype=torch.long, device=q_feat.device)
    projected_q = gate.project_queries(q_feat)
    P, p = projected_q.shape[3:]
    qp = projected_q.reshape(R, qb, P, p).float()
    for child_level_idx in range(len(key_levels) - 2, -1, -1):
        child = key_levels[child_level_idx]
        child_count = child.features.shape[2]
        cand, valid = native.tree_candidates(selected, radix, child_count, child.starts)
        kp = gate.project_keys(child.features).reshape(R, child_count, P, p).float()
        scores = native.gate_maxsim(qp, kp, cand)
        k = min(beam, cand.shape[-1], child_count)
        selected = native.tree_topk(scores, valid, cand, k)
    return selected.view(L, G, qb, -1)


@torch.no_grad()
def route_from_features(gate, q_feat: torch.Tensor, k_feat: torch.Tensor, beam: int = 16, radix: int = 2,
                        local_window: int = 1, sink_blocks: int = 0, k_selected: int | None = None) -> torch.Tensor:
    """Tree routes of captured features: int32 ``[L, G, qb, K]``.

    ``q_feat`` / ``k_feat`` are ``[L, G, blocks, P, d]`` prototypes (one row
    of layers per gate layer); the key tree, its beam traversal and
    ``selected_ids_to_blocks`` follow benchmarks/compare_dense_sparse_live_tree.py:131-197
    (K = beam + local_window + 1 unless given).
    """
    L, G, qb = q_feat.shape[:3]
    if k_selected is None:
        k_selected = beam + local_window + 1
    levels = build_key_tree(k_feat, radix)
    ids = traverse_to_leaf_ids(gate, q_feat, levels, beam, radix)          # [L, G, qb, C]
    packed = native.pack_selected_ids(ids.reshape(L * G, qb, -1), k_selected, local_window, k_feat.shape[2],
                                      sink_blocks)
    return packed.view(L, G, qb, k_selected)


@torch.no_grad()
def tree_select_blocks(query: torch.Tensor, key: torch.Tensor, gate, beam: int = 16, radix: int = 2,
                       prototypes: int = 8, local_window: int = 1, sink_blocks: int = 0,
                       k_selected: int | None = None) -> torch.Tensor:
    """The deployed selector for one layer: int32 ``selected_blocks`` rows ``[B, Hkv, qb, K]``.

    Outlier prototypes of the group-averaged queries and of the keys
    (teacher/chunked_extract.py:164-172), the key tree and its beam traversal,
    then ``selected_ids_to_blocks`` (scripts/export_selected_blocks.py:80-175,
    :199-221: K = beam + local_window + 1 unless given).  ``gate`` is a
    one-layer FlatGate.
    """
    from ..teacher.chunked_extract import pool_selector_features

    B, Hkv, T = key.shape[:3]
    qb = (T + 63) // 64
    if k_selected is None:
        k_selected = beam + local_window + 1
    q_feat, k_feat = pool_selector_features(query, key, prototypes)       # [B, Hkv, qb, P, d]
    out = torch.empty((B, Hkv, qb, k_selected), device=query.device, dtype=torch.int32)
    for b in range(B):
        out[b] = route_from_features(gate, q_feat[b][None], k_feat[b][None], beam, radix, local_window,
                                     sink_blocks, k_selected)[0]
    return out
