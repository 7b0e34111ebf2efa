"""Block-summary pooling of post-RoPE Q and K on the GPU.

Drop-ins for teacher/chunked_extract.py:27-80 of the reference, bit-exact with
its CPU rounding points (see csrc/pool.cu).  The mean prototype (P = 1) is
what the flat-gate path uses; P > 1 adds the P-1 rows farthest from the mean
(fp32 squared L2; identical picks unless two distances tie within fp32
rounding), the features of the MaxSim gate.
"""
from __future__ import annotations

import torch

from .. import native

_BLOCK = 64


def _proto_pool_seq(x: torch.Tensor, block: int, P: int) -> torch.Tensor:
    """``[b, H, L, d] -> [b, H, nb, P, d]`` (teacher/chunked_extract.py:27-72)."""
    return native.proto_pool(x, block, P)


def _group_avg_tokens(x: torch.Tensor, G: int) -> torch.Tensor:
    """``[b, H, L, d] -> [b, G, L, d]`` mean of each group's H/G heads (:75-80)."""
    return native.group_avg_tokens(x, G)


def pool_selector_features(query: torch.Tensor, key: torch.Tensor, P: int = 1):
    """The selector inputs the reference's capture hook stores (:164-172).

    Returns ``(pooledQ, pooledK)``, each ``[b, Hkv, qb, P, d]`` in the model
    dtype: the prototypes of the group-averaged queries and of the keys,
    computed in one launch.
    """
    pq, pk = native.pool_qk(query, key, P)
    if P == 1:
        return pq[:, :, :, None, :], pk[:, :, :, None, :]
    return pq, pk
