"""SPRUCE sparse prefill of a whole transformers model (Qwen2-style GQA).

Two flows, both on the device end to end:

* two-pass, the reference's live route
  (benchmarks/compare_dense_sparse_live_tree.py:131-219, :453): a dense
  forward whose attention callback stores each layer's selector features
  (teacher/chunked_extract.py:199-215, prototypes of the group-averaged
  queries and of the keys, kept in HBM rather than copied to the host);
  the selector routes every layer at once (``live_route``); a second forward
  runs the block-sparse prefill on those ``selected_blocks`` through the
  registered callback of kernels/sparse_prefill.py:55-97.
* one-pass: the attention callback pools its own post-RoPE Q/K, routes the
  layer and runs the block-sparse kernel in the same call, so no dense
  forward is needed.  Layer l's features then come from the sparse forward's
  hidden states instead of a dense forward's: the flows agree at layer 0 and
  whenever every causal block is selected.

Decode steps (query length != key length) and ``dense_layers`` go to SDPA in
both flows, as in the reference callback.
"""
from __future__ import annotations

import torch

from . import native
from .kernels.direct_index import direct_index_sparse_triton
from .kernels.sparse_prefill import _sdpa, _sparse_attention_mask, register_triton_sparse_prefill_attention
from .selector.gate import FlatGate
from .selector.tree import route_from_features
from .synthetic import k_for_density
from .teacher.chunked_extract import pool_selector_features

SELECTOR_FEATURE_CAPTURE = "spruce_selector_feature_capture"
SPRUCE_LIVE_SPARSE_PREFILL = "spruce_live_sparse_prefill"
BLOCK = 64


def capture_features_attention_forward(module, query, key, value, attention_mask, *, spruce_feature_store,
                                       spruce_prototypes=8, **kwargs):
    """Dense causal attention that also stores the layer's selector features.

    ``spruce_feature_store[layer_idx] = (pooledQ, pooledK)``, each
    ``[B, Hkv, blocks, P, d]`` in the model dtype (teacher/chunked_extract.py:204-206).
    """
    if query.shape[-2] == key.shape[-2]:
        spruce_feature_store[int(module.layer_idx)] = pool_selector_features(query, key, int(spruce_prototypes))
    return _sdpa(module, query, key, value, attention_mask, **kwargs)


def _set_attention(model, name):
    previous = model.config._attn_implementation
    model.set_attn_implementation(name)
    return previous


@torch.no_grad()
def capture_selector_features(model, input_ids, prototypes: int = 8):
    """One dense forward; returns ``{"q_feat", "k_feat"}``, each ``[L, G, blocks, P, d]`` (batch 1).

    The features of benchmarks/compare_dense_sparse_live_tree.py's
    ``load_selector_features``, captured in HBM by one pass over the model.
    """
    if input_ids.shape[0] != 1:
        raise ValueError("feature capture takes one sequence (batch size 1)")
    register_live_sparse_prefill_attention()
    store: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
    previous = _set_attention(model, SELECTOR_FEATURE_CAPTURE)
    try:
        model(input_ids, use_cache=False, logits_to_keep=1, spruce_feature_store=store,
              spruce_prototypes=prototypes)
    finally:
        model.set_attn_implementation(previous)
    order = sorted(store)
    if order != list(range(len(order))):
        raise RuntimeError(f"feature capture saw layers {order}")
    q_feat = torch.stack([store[i][0][0] for i in order])
    k_feat = torch.stack([store[i][1][0] for i in order])
    return {"q_feat": q_feat, "k_feat": k_feat}


class LiveSelector:
    """Per-layer routing policy of a model: a FlatGate and how to use it.

    ``mode="flat"``: one mean prototype per block, FlatGate scores, masked
    top-K packed into rows (scripts/route_overrides.py:187-205); K from
    ``k_selected`` or the charged ``density``.  ``mode="tree"``: ``prototypes``
    outlier prototypes, the key tree and beam traversal
    (scripts/eval_tree_traversal.py:60-113); K = beam + local_window + 1 unless
    given.  ``gate`` holds one layer of Wq/Wk per model layer.
    """

    def __init__(self, gate: FlatGate, *, mode: str = "flat", k_selected: int | None = None,
                 density: float | None = None, local_window: int = 0, sink_blocks: int = 1, beam: int = 16,
                 radix: int = 2, prototypes: int = 8, keep_routes: bool = False):
        if mode not in ("flat", "tree"):
            raise ValueError(f"mode must be 'flat' or 'tree', got {mode!r}")
        if mode == "flat" and (k_selected is None) == (density is None):
            raise ValueError("the flat selector takes exactly one of k_selected and density")
        self.gate = gate
        self.mode = mode
        self.k_selected, self.density = k_selected, density
        self.local_window, self.sink_blocks = int(local_window), int(sink_blocks)
        self.beam, self.radix, self.prototypes = int(beam), int(radix), int(prototypes)
        self.keep_routes = keep_routes
        self.routes: dict[int, torch.Tensor] = {}
        self._layer_gates: dict[int, FlatGate] = {}
        self._wq = gate.Wq.detach().float().contiguous()
        self._wk = gate.Wk.detach().float().contiguous()

    @property
    def num_layers(self) -> int:
        return self._wq.shape[0]

    def width(self, query_blocks: int) -> int:
        if self.mode == "tree":
            return self.k_selected if self.k_selected is not None else self.beam + self.local_window + 1
        if self.k_selected is not None:
            return int(self.k_selected)
        return max(k_for_density(query_blocks, self.density), self.local_window + 1 + self.sink_blocks)

    @torch.no_grad()
    def _layer_gate(self, layer_idx: int) -> FlatGate:
        """A one-layer FlatGate holding this layer's projections (the tree routines index layer 0)."""
        gate = self._layer_gates.get(layer_idx)
        if gate is None:
            gate = FlatGate(1, self._wq.shape[1], self._wq.shape[2]).to(self._wq.device).eval()
            gate.Wq.copy_(self._wq[layer_idx:layer_idx + 1])
            gate.Wk.copy_(self._wk[layer_idx:layer_idx + 1])
            self._layer_gates[layer_idx] = gate
        return gate

    @torch.no_grad()
    def select_layer(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor) -> torch.Tensor:
        """int32 rows ``[B, Hkv, qb, K]`` of one layer from its post-RoPE Q/K."""
        if not 0 <= layer_idx < self.num_layers:
            raise ValueError(f"layer_idx {layer_idx} is outside the gate's {self.num_layers} layers")
        qb = (key.shape[2] + BLOCK - 1) // BLOCK
        K = self.width(qb)
        if self.mode == "flat":
            sel = native.select_blocks(query, key, self._wq[layer_idx], self._wk[layer_idx], K, self.local_window,
                                       self.sink_blocks)
        else:
            q_feat, k_feat = pool_selector_features(query, key, self.prototypes)
            gate = self._layer_gate(layer_idx)
            sel = torch.stack([route_from_features(gate, q_feat[b][None], k_feat[b][None], self.beam, self.radix,
                                                   self.local_window, self.sink_blocks, K)[0]
                               for b in range(key.shape[0])])
        if self.keep_routes:
            self.routes[layer_idx] = sel
        return sel

    @torch.no_grad()
    def route(self, features) -> torch.Tensor:
        """int32 ``selected_blocks`` ``[1, L, G, qb, K]`` for captured features (two-pass flow)."""
        q_feat, k_feat = features["q_feat"], features["k_feat"]
        L, G, qb = q_feat.shape[:3]
        if L != self.num_layers:
            raise ValueError(f"features have {L} layers, the gate {self.num_layers}")
        K = self.width(qb)
        if self.mode == "flat":
            if q_feat.shape[3] != 1:
                raise ValueError("the flat selector routes one prototype per block")
            return self.gate.select_blocks(q_feat, k_feat, K, self.local_window, self.sink_blocks)
        return route_from_features(self.gate, q_feat, k_feat, self.beam, self.radix, self.local_window,
                                   self.sink_blocks, K)[None]

    @property
    def feature_prototypes(self) -> int:
        return 1 if self.mode == "flat" else self.prototypes


def live_route(selector: LiveSelector, features) -> torch.Tensor:
    """Functional form of :meth:`LiveSelector.route` (compare_dense_sparse_live_tree.py:131-219)."""
    return selector.route(features)


def live_sparse_prefill_attention_forward(module, query, key, value, attention_mask, *, spruce_selector,
                                          dense_layers=(), block_size=64, **kwargs):
    """One-pass callback: route this layer from its own Q/K, then block-sparse attention."""
    if query.shape[-2] != key.shape[-2]:
        return _sdpa(module, query, key, value, attention_mask, **kwargs)
    if attention_mask is not None:
        raise ValueError("B200 SPRUCE prefill currently supports unpadded batch-size-1 inputs only")
    if block_size != 64:
        raise ValueError("B200 SPRUCE backend currently requires block_size=64")
    layer_idx = int(getattr(module, "layer_idx"))
    if dense_layers and layer_idx in {int(layer) for layer in dense_layers}:
        return _sdpa(module, query, key, value, attention_mask, **kwargs)
    selected = spruce_selector.select_layer(layer_idx, query, key)
    output = direct_index_sparse_triton(query, key, value, selected, scale=query.shape[-1] ** -0.5,
                                        block_size=block_size)
    return output, None


def register_live_sparse_prefill_attention():
    """Register the capture and one-pass callbacks (and the selected-blocks one)."""
    from transformers import AttentionInterface, AttentionMaskInterface

    register_triton_sparse_prefill_attention()
    AttentionInterface.register(SELECTOR_FEATURE_CAPTURE, capture_features_attention_forward)
    AttentionMaskInterface.register(SELECTOR_FEATURE_CAPTURE, _sparse_attention_mask)
    AttentionInterface.register(SPRUCE_LIVE_SPARSE_PREFILL, live_sparse_prefill_attention_forward)
    AttentionMaskInterface.register(SPRUCE_LIVE_SPARSE_PREFILL, _sparse_attention_mask)
    return SPRUCE_LIVE_SPARSE_PREFILL


@torch.no_grad()
def sparse_prefill(model, input_ids, selector: LiveSelector, *, flow: str = "one_pass", dense_layers=(),
                   use_cache: bool = True):
    """SPRUCE prefill of one sequence; returns ``(model output, selected_blocks or None)``.

    ``flow="two_pass"`` captures features with a dense forward, routes all
    layers and runs the selected-blocks callback; ``flow="one_pass"`` routes
    inside the forward.  Only the last position's logits are computed.
    """
    from .kernels.sparse_prefill import SPRUCE_TRITON_SPARSE_PREFILL

    register_live_sparse_prefill_attention()
    if flow == "two_pass":
        features = capture_selector_features(model, input_ids, selector.feature_prototypes)
        selected = selector.route(features)
        del features
        previous = _set_attention(model, SPRUCE_TRITON_SPARSE_PREFILL)
        try:
            out = model(input_ids, use_cache=use_cache, logits_to_keep=1, selected_blocks=selected, block_size=BLOCK,
                        dense_layers=tuple(dense_layers))
        finally:
            model.set_attn_implementation(previous)
        return out, selected
    if flow != "one_pass":
        raise ValueError(f"flow must be 'one_pass' or 'two_pass', got {flow!r}")
    previous = _set_attention(model, SPRUCE_LIVE_SPARSE_PREFILL)
    try:
        out = model(input_ids, use_cache=use_cache, logits_to_keep=1, spruce_selector=selector,
                    dense_layers=tuple(dense_layers))
    finally:
        model.set_attn_implementation(previous)
    return out, None
