"""Route accounting (reference: scripts/route_overrides.py:21-53)."""
from __future__ import annotations


def charged_route_density(selected, dense_layers=()):
    """Block-attention density with dense layers charged as their full causal triangle."""
    if selected.dim() != 5:
        raise ValueError(f"selected must be [B,L,G,qb,K], got {tuple(selected.shape)}")
    B, L, G, qb, _ = selected.shape
    layers = sorted({int(layer) for layer in dense_layers})
    if any(layer < 0 or layer >= L for layer in layers):
        raise ValueError(f"dense layer outside [0,{L}): {layers}")
    dense_set = set(layers)
    causal_per_layer = B * G * qb * (qb + 1) // 2
    charged = 0
    for layer in range(L):
        charged += causal_per_layer if layer in dense_set else int((selected[:, layer] >= 0).sum().item())
    maximum = causal_per_layer * L
    fraction = charged / maximum if maximum else 0.0
    return {
        "dense_layers": layers,
        "dense_layer_count": len(layers),
        "dense_layer_fraction": len(layers) / L,
        "charged_block_entries": charged,
        "maximum_causal_block_entries": maximum,
        "charged_attention_fraction": fraction,
        "charged_sparsity": 1.0 - fraction,
    }
