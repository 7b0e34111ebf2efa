"""The layer's launch count claim (bench.py's gpu_launches) against the kernels CUPTI sees.

One selector + attention call launches the pooling, the projections (one
launch when at least 1024 rows are projected, else two), the select kernel and
the attention: `SparsePrefillLayer.launches_per_call` must equal the number of
this library's kernels the profiler records for the call.
"""
import pytest
import torch

from spruce_research_b200.pipeline import SparsePrefillLayer
from spruce_research_b200.synthetic import LayerShape, k_for_density, make_gate_weights, make_layer_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens", [8192, 2048])  # 1024 projected rows (fused), 256 (separate)
def test_launches_per_call_matches_the_profiler(tokens):
    shape = LayerShape(1, 28, 4, tokens, 128)
    K = k_for_density(shape.query_blocks, 0.10)
    q, k, v = (t.cuda() for t in make_layer_inputs(shape, torch.bfloat16, seed=5))
    wq, wk = make_gate_weights(1, 128, 128, seed=6)
    layer = SparsePrefillLayer(wq[0].cuda(), wk[0].cuda(), K)
    layer(q, k, v)  # warm-up: workspace, tensor maps, kernel attributes
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        layer(q, k, v)
        torch.cuda.synchronize()
    ours = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
            and "spruce::" in e.name]
    want = layer.launches_per_call(1, shape.kv_heads, (0, shape.query_blocks))
    assert want == (4 if tokens == 8192 else 5)
    assert len(ours) == want, ours
