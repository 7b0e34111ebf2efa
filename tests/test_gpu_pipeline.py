"""The per-layer pipeline: SparsePrefillLayer and the host-streamed chunked form.

The streamed layer overlaps host copies with the selector and attention of
earlier query-block chunks; its output must equal the one-shot layer bit for
bit, including selections that depend on keys copied in earlier chunks, and
its last query blocks must match the oracle's attention on the oracle's
selection (max-abs 2e-2, mean-abs 2e-3 in bf16).
"""
import pytest
import torch

from oracle import oracle as O
from spruce_research_b200.pipeline import HostStreamedLayer, SparsePrefillLayer
from spruce_research_b200.synthetic import LayerShape, k_for_density, make_gate_weights, make_layer_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,chunks,schedule", [(8192, 4, "equal"), (8192 + 100, 3, "balanced"),
                                                    (2048, 8, "equal"), (8192, 16, "balanced")])
def test_streamed_layer_equals_one_shot_layer(tokens, chunks, schedule):
    shape = LayerShape(1, 28, 4, tokens, 128)
    K = k_for_density(shape.query_blocks, 0.10)
    q, k, v = make_layer_inputs(shape, torch.bfloat16, seed=21)
    wq, wk = make_gate_weights(1, 128, 128, seed=22)
    layer = SparsePrefillLayer(wq[0].cuda(), wk[0].cuda(), K)
    hq, hk, hv = (t.transpose(1, 2).contiguous().pin_memory() for t in (q, k, v))   # token-major host buffers
    want, sel = layer(*(t.cuda().transpose(1, 2) for t in (hq, hk, hv)))
    dq, dk, dv = (torch.empty_like(t, device="cuda") for t in (hq, hk, hv))
    dout = torch.empty_like(want)
    hout = torch.empty(want.shape, dtype=want.dtype).pin_memory()
    streamed = HostStreamedLayer(layer, torch.device("cuda"), chunks=chunks, schedule=schedule)
    streamed(hq, hk, hv, dq, dk, dv, dout, hout=hout)
    torch.cuda.synchronize()
    assert torch.equal(dout, want)
    assert torch.equal(hout, want.cpu())
    # and against the oracle: its selector bit for bit, its attention on the last query blocks
    ref = O.select_blocks(q, k, wq[0], wk[0], K, 0, 1)
    assert torch.equal(sel.cpu(), ref["selected"])
    qb = shape.query_blocks
    tail = O.sparse_attention(q, k, v, ref["selected"], out_dtype=torch.float32, q_blocks=(qb - 4, qb))
    rows = slice((qb - 4) * 64, tokens)
    err = (hout[:, rows].float() - tail[:, rows]).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3
