"""The CPU oracle against the reference's own outputs (tests/golden/, made by make_golden.py).

This pins the oracle: every later GPU parity claim is "CUDA == oracle" plus
"oracle == reference" from here.  Runs on CPU.
"""
import numpy as np
import pytest
import torch

from golden_cases import CASE_NAMES, DT, from_raw, load_case, load_npz
from oracle import oracle as O


@pytest.mark.parametrize("name", CASE_NAMES)
def test_pooled_features_bit_exact(name):
    case = load_case(name)
    q, k, v, wq, wk = case.inputs()
    r = O.select_blocks(q, k, wq, wk, case.K, case.local_window, case.sink)
    assert torch.equal(r["pooled_q"], case.golden("pooled_q"))
    assert torch.equal(r["pooled_k"], case.golden("pooled_k"))


@pytest.mark.parametrize("name", CASE_NAMES)
def test_selected_blocks_bit_exact_and_scores_close(name):
    case = load_case(name)
    q, k, v, wq, wk = case.inputs()
    r = O.select_blocks(q, k, wq, wk, case.K, case.local_window, case.sink)
    # fixed-order fma vs MKL: a few fp32 ulps
    assert (r["scores"] - case.golden("scores")).abs().max().item() < 1e-8
    assert torch.equal(r["selected"], case.golden("selected"))
    O.validate_selected_blocks(r["selected"][:, None].contiguous(), local_window=case.local_window)


@pytest.mark.parametrize("name", CASE_NAMES)
def test_attention_matches_reference(name):
    case = load_case(name)
    q, k, v, wq, wk = case.inputs()
    out = O.sparse_attention(q, k, v, case.golden("selected"), out_dtype=torch.float32)
    rows = case.out_rows()
    err = (out[:, rows] - case.golden("out").float()).abs()
    if case.dtype == torch.float32:
        assert err.max().item() < 1e-5
    else:
        # the golden is rounded to the input dtype: within one ulp of |x| <= 8
        assert err.max().item() < 1.6e-2
        assert err.mean().item() < 1e-3


def test_packing_matches_reference():
    z = load_npz("packing")
    n = 0
    while f"pack{n}_ids" in z:
        K, lw, kb, sink = (int(x) for x in z[f"pack{n}_args"])
        got = O.selected_ids_to_blocks(torch.from_numpy(z[f"pack{n}_ids"]), K, lw, kb, sink)
        assert torch.equal(got, torch.from_numpy(z[f"pack{n}_out"])), f"packing case {n}"
        n += 1
    assert n == 6


def test_mean_prototype_matches_reference():
    z = load_npz("proto")
    for n in range(3):
        dt = DT[int(z[f"proto{n}_dtype"][0])]
        x = from_raw(z[f"proto{n}_x"], dt)
        got = O.proto_pool_seq(x, 64, 1)
        want = from_raw(z[f"proto{n}_p1"], dt)
        assert torch.equal(got, want), f"proto case {n}"


def test_outlier_prototypes_match_reference():
    # _proto_pool_seq(x, 64, 8): the mean plus the 7 rows farthest from it
    z = load_npz("proto")
    for n in range(3):
        dt = DT[int(z[f"proto{n}_dtype"][0])]
        x = from_raw(z[f"proto{n}_x"], dt)
        assert torch.equal(O.proto_pool_seq(x, 64, 8), from_raw(z[f"proto{n}_p8"], dt)), f"proto case {n}"


def test_validator_messages_follow_reference():
    def row(ids, k=4):
        return list(ids) + [-1] * (k - len(ids))

    ok = torch.tensor([[[[row([0]), row([0, 1]), row([0, 1, 2]), row([0, 2, 3])]]]], dtype=torch.int32)
    O.validate_selected_blocks(ok)
    cases = [  # rows of one (batch, layer, group), as in tests/test_validator.py of the reference
        ([row([0, 5])], "future"),
        ([row([0]), row([0, 1, 1])], "Duplicate"),
        ([row([0]), row([0, 1]), row([0, 2, 1])], "Not sorted"),
        ([row([0]), row([1])], "Missing local-window"),
        ([row([0]), [0, -1, 1, -1]], "trailing"),
    ]
    for rows, msg in cases:
        with pytest.raises(AssertionError, match=msg):
            O.validate_selected_blocks(torch.tensor([[[rows]]], dtype=torch.int32))


def test_dense_reference_equals_all_block_oracle():
    # 100% density: the block-sparse oracle must equal dense causal attention.
    from spruce_research_b200.synthetic import LayerShape, make_layer_inputs

    shape = LayerShape(1, 4, 2, 200, 64)
    q, k, v = make_layer_inputs(shape, torch.float32, seed=3)
    qb = shape.query_blocks
    idx = torch.full((1, 2, qb, qb), -1, dtype=torch.int32)
    for i in range(qb):
        idx[0, :, i, : i + 1] = torch.arange(i + 1, dtype=torch.int32)
    sparse = O.sparse_attention(q, k, v, idx, out_dtype=torch.float32)
    dense = O.dense_causal_attention(q, k, v)
    assert (sparse - dense).abs().max().item() < 1e-5


def test_golden_fixtures_are_small():
    import os

    from golden_cases import HERE

    total = sum(os.path.getsize(os.path.join(HERE, f)) for f in os.listdir(HERE) if f.endswith(".npz"))
    # the headline configurations (c1_full, c2) carry their whole selected_blocks and sampled attention rows
    assert total < 12 * 2**20
    assert np.load(os.path.join(HERE, "c0.npz"))["selected"].dtype == np.int32


def _maxsim_case(z, n):
    dt = DT[int(z[f"ms{n}_dtype"][0])]
    q, k = from_raw(z[f"ms{n}_q"], dt), from_raw(z[f"ms{n}_k"], dt)
    wq, wk = torch.from_numpy(z[f"ms{n}_wq"]), torch.from_numpy(z[f"ms{n}_wk"])
    return q, k, wq, wk


def test_maxsim_scores_match_reference():
    # FlatGate with P = 8 prototypes (selector/gate.py:29-101, :132-171) on the
    # reference's own outlier features; MKL einsum vs fixed fma order: fp32 rounding.
    z = load_npz("maxsim")
    for n in range(2):
        q, k, wq, wk = _maxsim_case(z, n)
        qf, kf = O.proto_pool_seq(q, 64, 8)[0], O.proto_pool_seq(k, 64, 8)[0]       # [G, nb, 8, d]
        qp, kp = O.project(qf, wq[0]), O.project(kf, wk[0])                         # [G, nb, 8, p]
        want = torch.from_numpy(z[f"ms{n}_scores"])[0]
        got = O.maxsim(qp, kp)
        assert (got - want).abs().max().item() <= 2e-6 * want.abs().max().item()
        cand = torch.from_numpy(z[f"ms{n}_cand"])[0]
        got_c = O.maxsim(qp, kp, cand)
        want_c = torch.from_numpy(z[f"ms{n}_cand_scores"])[0]
        assert (got_c - want_c).abs().max().item() <= 2e-6 * want_c.abs().max().item()
        assert torch.equal(got_c, torch.gather(got, 2, cand))


def test_key_tree_and_traversal_match_reference():
    # selector/tree.py:116 build_key_tree and scripts/eval_tree_traversal.py:60
    # traverse_to_leaf_ids (beam 4, radix 2) on the reference's fp32 features
    z = load_npz("maxsim")
    for n in range(2):
        q, k, wq, wk = _maxsim_case(z, n)
        qf = O.proto_pool_seq(q, 64, 8)[0].float()          # [G, nb, 8, d]
        level = torch.from_numpy(z[f"ms{n}_tree0"])[0]      # the reference's leaf features (fp32)
        assert torch.equal(level, O.proto_pool_seq(k, 64, 8)[0].float())
        levels, starts = [level], [torch.from_numpy(z[f"ms{n}_tree0_range"])[0]]
        l = 1
        while f"ms{n}_tree{l}" in z:
            level = O.tree_merge(level)
            assert torch.equal(level, torch.from_numpy(z[f"ms{n}_tree{l}"])[0]), f"case {n} level {l}"
            levels.append(level)
            starts.append(torch.from_numpy(z[f"ms{n}_tree{l}_range"])[0])
            l += 1
        assert levels[-1].shape[1] == 1
        proj = [O.project(x, wk[0]) for x in levels]
        ids = O.traverse_to_leaf_ids(O.project(qf, wq[0]), proj, starts, beam=4)
        assert torch.equal(ids, torch.from_numpy(z[f"ms{n}_leaf_ids"])[0])


@pytest.mark.parametrize("name", ["r_bf16", "r_f32"])
def test_residual_attention_oracle_matches_reference(name):
    # sparse/attention.py:83-274 with residual_summaries=True: the oracle's one
    # softmax over selected blocks and residual summary keys, fed the oracle's
    # summary table (bit-exact with build_kv_summary_table), reproduces the
    # reference's outputs.
    from golden_cases import load_residual_case
    from spruce_research_b200.interfaces.residual_summaries import build_residual_tree_layout

    q, k, v, sel, nodes, outs = load_residual_case(name)
    T = q.shape[2]
    lay = build_residual_tree_layout((T + 63) // 64)
    assert nodes.shape[-1] > 0
    for P, want in outs.items():
        t = O.kv_summary_table(k, v, lay.starts, lay.ends, 64, P, None)
        got = O.residual_sparse_attention(q, k, v, sel[:, 0], nodes[:, 0], t["keys"], t["values"], t["counts"],
                                          t["log_counts"], out_dtype=torch.float32)
        err = (got - want.float()).abs().max().item()
        if q.dtype == torch.float32:
            assert err < 2e-6, (P, err)
        else:  # the reference rounds its fp32 result to bf16 once; so does the oracle's caller
            assert (got.to(q.dtype).float() - want.float()).abs().max().item() <= 2 ** -7, (P, err)
    # the summaries matter: without them the output differs
    plain = O.sparse_attention(q, k, v, sel[:, 0], out_dtype=torch.float32)
    assert (plain - outs[max(outs)].float()).abs().max().item() > 1e-2


def test_key_tree_level_ranges_match_reference():
    # selector/tree.py's level ranges, computed once on the host, against the reference's stored levels
    from spruce_research_b200.selector.tree import _level_ranges

    z = load_npz("maxsim")
    for n in range(2):
        kb = z[f"ms{n}_tree0"].shape[2]
        ranges = _level_ranges(kb, 2)
        level = 0
        while f"ms{n}_tree{level}_range" in z:
            want = z[f"ms{n}_tree{level}_range"]
            assert ranges[level] == (want[0].tolist(), want[1].tolist()), (n, level)
            level += 1
        assert level == len(ranges)


# ---------------------------------------------------------------- the headline configurations in full
_BIG = {}


def _big(name):
    """(case, inputs, oracle selector result), computed once per module."""
    from golden_cases import load_big_case

    if name not in _BIG:
        case = load_big_case(name)
        q, k, v, wq, wk = case.inputs()
        assert case.same_inputs(q, k, v), "synthetic generator drifted"
        _BIG[name] = (case, (q, k, v, wq, wk), O.select_blocks(q, k, wq, wk, case.K, case.local_window, case.sink))
    return _BIG[name]


@pytest.mark.parametrize("name", ["c1_full", "c2"])
def test_headline_pooled_features_bit_exact(name):
    from golden_cases import raw_sha256

    case, _, r = _big(name)
    assert raw_sha256(r["pooled_q"]) == case.digest("pooled_q")
    assert raw_sha256(r["pooled_k"]) == case.digest("pooled_k")


@pytest.mark.parametrize("name", ["c1_full", "c2"])
def test_headline_selected_blocks_bit_exact(name):
    """Every row of the reference's selection at config 1 (32K, K=27) and config 2 (128K, K=106)."""
    case, _, r = _big(name)
    differ = (r["selected"] != case.selected).any(-1)
    assert not differ.any(), (f"{int(differ.sum())} of {differ.numel()} rows differ; their boundary score gaps: "
                              f"{case.gap[differ][:8].tolist()}")


@pytest.mark.parametrize("name", ["c1_full", "c2"])
def test_headline_attention_rows_match_reference(name):
    case, (q, k, v, _, _), _ = _big(name)
    out = O.sparse_attention_blocks(q, k, v, case.selected, case.out_blocks)
    err = (out - case.out.float()).abs()
    # the reference's output is rounded to bf16: within one ulp of |x| <= 8
    assert err.max().item() < 1.6e-2
    assert err.mean().item() < 1e-3


# ---------------------------------------------------------------- trained gate weights
def trained_case():
    """(fixture, q, k, wq, wk, same): the reference's selections with one layer of its trained
    checkpoint (tests/golden/trained.npz), the regenerated inputs they were made on, and
    whether this host regenerated exactly those inputs."""
    from spruce_research_b200.synthetic import LayerShape, make_layer_inputs

    z = load_npz("trained")
    B, Hq, Hkv, T, D = (int(x) for x in z["shape"])
    q, k, v = make_layer_inputs(LayerShape(B, Hq, Hkv, T, D), torch.bfloat16, int(z["seed"][0]), rope_theta=1e6)
    cs = np.array([q.double().sum().item(), k.double().sum().item(), v.double().sum().item()])
    return z, q, k, torch.from_numpy(z["wq"]), torch.from_numpy(z["wk"]), bool(np.allclose(cs, z["checksum"]))


def test_trained_gate_flat_selection_matches_reference():
    z, q, k, wq, wk, same = trained_case()
    assert same, "synthetic generator drifted"
    K, lw, sink = (int(x) for x in z["policy"])
    got = O.select_blocks(q, k, wq, wk, K, lw, sink)["selected"]
    assert torch.equal(got, torch.from_numpy(z["selected"]))


def test_trained_gate_tree_traversal_matches_reference():
    from spruce_research_b200.selector.tree import _level_ranges

    z, q, k, wq, wk, same = trained_case()
    assert same, "synthetic generator drifted"
    G = k.shape[1]
    qf = O.proto_pool_seq(O.group_avg_tokens(q, G), 64, 8)[0].float()   # [G, qb, 8, d]
    level = O.proto_pool_seq(k, 64, 8)[0].float()
    levels = [level]
    while level.shape[1] > 1:
        level = O.tree_merge(level)
        levels.append(level)
    starts = [torch.tensor(s) for s, _ in _level_ranges(qf.shape[1], 2)]
    ids = O.traverse_to_leaf_ids(O.project(qf, wq), [O.project(x, wk) for x in levels], starts, beam=16)
    assert torch.equal(ids, torch.from_numpy(z["leaf_ids"])[0])
