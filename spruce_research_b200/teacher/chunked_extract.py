"""Block-summary pooling of post-RoPE Q and K on the GPU.

Drop-ins for teacher/chunked_extract.py:27-80 of the reference, bit-exact with
its CPU rounding points (see csrc/pool.cu).  The mean prototype (P = 1) is
what the flat-gate path uses; P > 1 (mean + farthest tokens) is not built.
"""
from __future__ import annotations

import torch

from .. import native

_BLOCK = 64


def _proto_pool_seq(x: torch.Tensor, block: int, P: int) -> torch.Tensor:
    """``[b, H, L, d] -> [b, H, nb, P, d]`` (teacher/chunked_extract.py:27-72), P = 1."""
    return native.proto_pool(x, block, P)


def _group_avg_tokens(x: torch.Tensor, G: int) -> torch.Tensor:
    """``[b, H, L, d] -> [b, G, L, d]`` mean of each group's H/G heads (:75-80)."""
    return native.group_avg_tokens(x, G)


def pool_selector_features(query: torch.Tensor, key: torch.Tensor):
    """The selector inputs the reference's capture hook stores (:164-172), P = 1.

    Returns ``(pooledQ, pooledK)``, each ``[b, Hkv, qb, 1, d]`` in the model
    dtype: block means of the group-averaged queries and of the keys, computed
    in one launch.
    """
    pq, pk = native.pool_qk(query, key)
    return pq[:, :, :, None, :], pk[:, :, :, None, :]
