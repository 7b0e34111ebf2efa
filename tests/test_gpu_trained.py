"""Selection with trained gate weights on the GPU (B200 only).

tests/golden/trained.npz holds one layer of the reference's trained checkpoint
(selector_ckpt/flat_gate_trained.pt, read through this repository's load_gate)
and the reference's own selections with it on seeded config-1-shaped inputs:
the flat P = 1 gate at 10% density and the deployed P = 8 key-tree traversal
(beam 16).  The CUDA path must reproduce both bit for bit.
"""
import pytest
import torch

from spruce_research_b200 import native
from spruce_research_b200.selector.gate import FlatGate
from spruce_research_b200.selector.tree import build_key_tree, traverse_to_leaf_ids
from spruce_research_b200.teacher.chunked_extract import pool_selector_features
from test_oracle_golden import trained_case

pytestmark = pytest.mark.gpu


def test_trained_weights_select_bit_exact_with_reference():
    z, q, k, wq, wk, same = trained_case()
    if not same:
        pytest.skip("this host regenerated other inputs than the reference saw")
    K, lw, sink = (int(x) for x in z["policy"])
    qd, kd = (t.transpose(1, 2).contiguous().cuda().transpose(1, 2) for t in (q, k))
    sel = native.select_blocks(qd, kd, wq.cuda(), wk.cuda(), K, lw, sink)
    torch.cuda.synchronize()
    assert torch.equal(sel.cpu(), torch.from_numpy(z["selected"])), "flat selection differs with trained weights"
    gate = FlatGate(1, wq.shape[0], wq.shape[1]).cuda().eval()
    with torch.no_grad():
        gate.Wq.copy_(wq[None])
        gate.Wk.copy_(wk[None])
    q_feat, k_feat = pool_selector_features(qd, kd, P=8)                # [1, G, qb, 8, d] in bf16
    levels = build_key_tree(k_feat.float(), radix=2)
    ids = traverse_to_leaf_ids(gate, q_feat.float(), levels, 16, radix=2)
    torch.cuda.synchronize()
    assert torch.equal(ids.cpu(), torch.from_numpy(z["leaf_ids"])), "tree leaf ids differ with trained weights"
