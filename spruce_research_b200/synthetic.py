"""Seeded synthetic inputs for the SPRUCE sparse-prefill layer.

No public dataset is involved: every benchmark and parity case uses the
planted-affinity construction below, with the shapes of the reference's
configurations (batch 1, 28 query / 4 KV heads, head_dim 128, block 64).

* Q, K, V ~ N(0, 1) in fp32.
* Optional rotary embedding (rotate-half form, base ``rope_theta``) on Q and
  K; the selector consumes post-RoPE features, as the reference's capture
  hook does (teacher/chunked_extract.py:164-172).
* Planted affinity, added after RoPE: for each (batch, KV group, query block)
  a unit vector u is added to the block's queries of every head in the group,
  and 2.0 * u is added to the keys of up to 3 distinct earlier key blocks.
* Cast to the requested dtype last.

The torch generator is seeded explicitly, so a (config, seed, device type)
triple always yields the same tensors.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

BLOCK = 64


@dataclass(frozen=True)
class LayerShape:
    """One attention layer's shape (batch, heads, tokens, head_dim)."""

    batch: int
    q_heads: int
    kv_heads: int
    tokens: int
    head_dim: int

    @property
    def query_blocks(self) -> int:
        return (self.tokens + BLOCK - 1) // BLOCK


def causal_block_entries(query_blocks: int, k_selected: int) -> int:
    """Non-PAD entries of one KV group when every row keeps min(q+1, K) blocks."""
    k = min(k_selected, query_blocks)
    return k * (k + 1) // 2 + (query_blocks - k) * k


def k_for_density(query_blocks: int, density: float) -> int:
    """Smallest row width K whose charged density reaches ``density``.

    Charged density is non-PAD entries over all causal block pairs,
    scripts/route_overrides.py:21-53 (charged_route_density).
    """
    total = query_blocks * (query_blocks + 1) // 2
    for k in range(1, query_blocks + 1):
        if causal_block_entries(query_blocks, k) >= density * total - 1e-9:
            return k
    return query_blocks


def sparse_attention_flops(shape: LayerShape, entries_per_group: int) -> float:
    """Algorithmic FLOPs of block-sparse attention over the selected tiles.

    4 * D * Hq * [(E - qb) * 64 * 64 + qb * 64 * 65 / 2]: every off-diagonal
    selected tile is a full 64x64 QK^T plus PV, every diagonal tile counts its
    causal half (64 * 65 / 2 pairs).  E is per KV group; all groups share it.
    """
    qb = shape.query_blocks
    pairs = (entries_per_group - qb) * BLOCK * BLOCK + qb * BLOCK * (BLOCK + 1) / 2
    return 4.0 * shape.head_dim * shape.q_heads * pairs * shape.batch


def _rope(x: torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half rotary embedding over the token axis of [B, T, H, D]."""
    T, D = x.shape[1], x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device=x.device, dtype=torch.float64) / D))
    ang = torch.arange(T, device=x.device, dtype=torch.float64)[:, None] * inv[None, :]
    cos = ang.cos().float()[None, :, None, :]
    sin = ang.sin().float()[None, :, None, :]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def make_layer_inputs(shape: LayerShape, dtype: torch.dtype, seed: int, device="cpu",
                      rope_theta: float | None = 1e6, plant_blocks: int = 3,
                      plant_scale: float = 2.0):
    """Return (q, k, v) as [B, H, T, D] views of token-major [B, T, H, D] storage.

    That is the layout HF Qwen2 attention hands to the attention callback
    (projection output viewed then transposed), so the kernels are exercised
    on the same strided views the reference's callers produce.
    """
    B, Hq, Hkv, T, D = shape.batch, shape.q_heads, shape.kv_heads, shape.tokens, shape.head_dim
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    q = torch.randn((B, T, Hq, D), generator=gen, device=device, dtype=torch.float32)
    k = torch.randn((B, T, Hkv, D), generator=gen, device=device, dtype=torch.float32)
    v = torch.randn((B, T, Hkv, D), generator=gen, device=device, dtype=torch.float32)
    if rope_theta is not None:
        q = _rope(q, rope_theta)
        k = _rope(k, rope_theta)
    if plant_blocks > 0:
        qb = shape.query_blocks
        rep = Hq // Hkv
        u = torch.randn((B, Hkv, qb, D), generator=gen, device=device, dtype=torch.float32)
        u = u / u.norm(dim=-1, keepdim=True)
        # Up to plant_blocks distinct earlier key blocks per query block.
        draw = torch.rand((B, Hkv, qb, qb), generator=gen, device=device)
        earlier = torch.arange(qb, device=device)[None, :] < torch.arange(qb, device=device)[:, None]
        draw = draw.masked_fill(~earlier, -1.0)
        width = min(plant_blocks, qb)
        top = draw.topk(width, dim=-1)
        chosen = top.indices.masked_fill(top.values < 0, -1)          # [B, Hkv, qb, width]
        # Accumulated on the CPU: scatter_add_ is sequential (deterministic) there, while the
        # CUDA version uses atomics whose order, and so rounding, varies between runs and GPUs.
        k_add = torch.zeros((B, Hkv, qb + 1, D), dtype=torch.float32)
        src = (plant_scale * u.cpu())[:, :, :, None, :].expand(B, Hkv, qb, width, D)
        dst = chosen.cpu().masked_fill(chosen.cpu() < 0, qb)           # dump slot qb
        k_add.scatter_add_(2, dst.reshape(B, Hkv, qb * width, 1).expand(B, Hkv, qb * width, D),
                           src.reshape(B, Hkv, qb * width, D))
        k_add = k_add.to(device)
        q_add = u.repeat_interleave(rep, dim=1)                        # [B, Hq, qb, D]
        q_tok = q_add.repeat_interleave(BLOCK, dim=2)[:, :, :T]        # [B, Hq, T, D]
        k_tok = k_add[:, :, :qb].repeat_interleave(BLOCK, dim=2)[:, :, :T]
        q = q + q_tok.transpose(1, 2)
        k = k + k_tok.transpose(1, 2)
    q = q.to(dtype).contiguous().transpose(1, 2)
    k = k.to(dtype).contiguous().transpose(1, 2)
    v = v.to(dtype).contiguous().transpose(1, 2)
    return q, k, v


def make_gate_weights(num_layers: int, head_dim: int, proj_dim: int, seed: int, device="cpu"):
    """FlatGate-shaped (Wq, Wk), each [L, d, p] fp32, seeded.

    Same distribution as selector/gate.py:23-26 (kaiming_uniform_ with
    a = sqrt(5) on an [L, d, p] tensor, i.e. U(-1/sqrt(d*p), 1/sqrt(d*p))).
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    bound = 1.0 / math.sqrt(head_dim * proj_dim)
    wq = (torch.rand((num_layers, head_dim, proj_dim), generator=gen, device=device) * 2 - 1) * bound
    wk = (torch.rand((num_layers, head_dim, proj_dim), generator=gen, device=device) * 2 - 1) * bound
    return wq, wk
