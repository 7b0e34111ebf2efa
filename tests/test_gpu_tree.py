"""The deployed selector on the GPU: outlier prototypes, key tree, beam traversal.

CUDA == oracle bit for bit (same rounding points, fma order and tie rules:
equal distances or scores go to the lower index); the CPU suite pins the
oracle's tree levels and traversal to the reference's own outputs
(tests/golden/maxsim.npz, fp32 features).
"""
import pytest
import torch

from golden_cases import load_npz
from oracle import oracle as O
from spruce_research_b200 import native
from spruce_research_b200.selector.gate import FlatGate
from spruce_research_b200.selector.tree import build_key_tree, traverse_to_leaf_ids, tree_select_blocks
from spruce_research_b200.synthetic import LayerShape, make_layer_inputs
from test_oracle_golden import _maxsim_case

pytestmark = pytest.mark.gpu


def _gate(wq, wk):
    gate = FlatGate(1, wq.shape[1], wq.shape[2]).cuda().eval()
    with torch.no_grad():
        gate.Wq.copy_(wq)
        gate.Wk.copy_(wk)
    return gate


def test_tree_and_traversal_match_reference_fixtures():
    z = load_npz("maxsim")
    for n in range(2):
        q, k, wq, wk = _maxsim_case(z, n)
        leaf = torch.from_numpy(z[f"ms{n}_tree0"]).cuda()          # [1, G, nb, 8, d] fp32
        levels = build_key_tree(leaf, radix=2)
        for lvl in levels:
            assert torch.equal(lvl.features.cpu(), torch.from_numpy(z[f"ms{n}_tree{lvl.level}"]))
            rng = torch.from_numpy(z[f"ms{n}_tree{lvl.level}_range"])
            assert torch.equal(lvl.starts.cpu(), rng[0]) and torch.equal(lvl.ends.cpu(), rng[1])
        q_feat = O.proto_pool_seq(q, 64, 8).float().cuda()
        ids = traverse_to_leaf_ids(_gate(wq, wk), q_feat, levels, 4, radix=2)
        assert torch.equal(ids.cpu(), torch.from_numpy(z[f"ms{n}_leaf_ids"]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_tree_levels_in_feature_dtype_match_oracle(dtype):
    gen = torch.Generator().manual_seed(61)
    k_feat = torch.randn((1, 2, 23, 8, 64), generator=gen).to(dtype)
    levels = build_key_tree(k_feat.cuda(), radix=2)
    want = k_feat[0]
    for lvl in levels[1:]:
        want = O.tree_merge(want)
        assert torch.equal(lvl.features[0].cpu(), want), f"level {lvl.level}"
    assert levels[-1].features.shape[2] == 1 and levels[-1].ends.item() == 23


def test_deployed_selector_matches_oracle_composition():
    shape = LayerShape(1, 28, 4, 64 * 40 + 9, 128)
    q, k, v = make_layer_inputs(shape, torch.bfloat16, seed=62)
    gen = torch.Generator().manual_seed(63)
    wq = torch.randn((1, 128, 128), generator=gen) / 11.3
    wk = torch.randn((1, 128, 128), generator=gen) / 11.3
    beam, lw = 6, 1
    qg = q.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    kg = k.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    sel = tree_select_blocks(qg, kg, _gate(wq, wk), beam=beam, local_window=lw)
    # the same composition on the CPU oracle
    qf = O.proto_pool_seq(O.group_avg_tokens(q, 4), 64, 8)[0]
    kf = O.proto_pool_seq(k, 64, 8)[0]
    levels, starts = [kf], [torch.arange(kf.shape[1])]
    while levels[-1].shape[1] > 1:
        n = levels[-1].shape[1]
        levels.append(O.tree_merge(levels[-1]))
        parents = torch.arange(levels[-1].shape[1])
        starts.append(starts[-1][parents * 2])
    ids = O.traverse_to_leaf_ids(O.project(qf, wq[0]), [O.project(x, wk[0]) for x in levels], starts, beam)
    qb = kf.shape[1]
    want = O.selected_ids_to_blocks(ids[None], beam + lw + 1, lw, qb, 0)[0, 0]
    assert torch.equal(sel[0].cpu(), want)
    O.validate_selected_blocks(sel[:, None].cpu().contiguous(), local_window=lw)


@pytest.mark.parametrize("nk", [70, 32, 17, 5, 1])
@pytest.mark.parametrize("P,p", [(8, 64), (5, 48), (4, 16), (3, 64), (8, 40), (1, 32)])
def test_maxsim_shapes_match_oracle(P, p, nk):
    # node-staged kernel (nk <= 32), lane-per-candidate kernel (P >= 4,
    # p % 16 == 0, 16-byte aligned) and the general kernel, over more than one
    # 32-candidate group and clamped ids
    gen = torch.Generator().manual_seed(64 + P * p + nk)
    R, nq, C = 3, 41, 37
    qp = torch.randn((R, nq, P, p), generator=gen)
    kp = torch.randn((R, nk, P, p), generator=gen)
    ids = torch.randint(-2, nk + 2, (R, nq, C), generator=gen)
    assert torch.equal(native.gate_maxsim(qp.cuda(), kp.cuda()).cpu(), O.maxsim(qp, kp))
    assert torch.equal(native.gate_maxsim(qp.cuda(), kp.cuda(), ids.cuda()).cpu(), O.maxsim(qp, kp, ids))
    # a view 4 bytes past an aligned allocation takes the general kernel
    flat = torch.empty(qp.numel() + 1, device="cuda")
    shifted = flat[1:].view(qp.shape)
    shifted.copy_(qp.cuda())
    assert torch.equal(native.gate_maxsim(shifted, kp.cuda(), ids.cuda()).cpu(), O.maxsim(qp, kp, ids))


@pytest.mark.parametrize("C", [1, 5, 17, 32, 33, 64])
def test_tree_topk_matches_stable_sort(C):
    # best k per row by score (invalid slots scored as the fp32 minimum), ties to the lower
    # position: a stable descending sort; C <= 32 takes the bitonic kernel, wider rows the scan
    gen = torch.Generator().manual_seed(70 + C)
    rows = 300
    scores = torch.randn((1, rows, C), generator=gen)
    scores[..., ::3] = torch.round(scores[..., ::3])           # ties
    scores[0, :7, 0] = -0.0
    valid = torch.rand((1, rows, C), generator=gen) > 0.25
    cand = torch.randint(0, 10_000, (1, rows, C), generator=gen)
    for k in sorted({1, max(1, C // 2), C}):
        got = native.tree_topk(scores.cuda(), valid.to(torch.uint8).cuda(), cand.cuda(), k).cpu()
        x = torch.where(valid, scores, torch.full_like(scores, -3.402823466e38))
        order = torch.sort(x, dim=-1, descending=True, stable=True).indices[..., :k]
        want = torch.where(torch.gather(valid, -1, order), torch.gather(cand, -1, order), torch.full_like(order, -1))
        assert torch.equal(got, want), (C, k)
