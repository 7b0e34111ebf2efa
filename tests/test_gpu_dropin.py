"""Reference-named drop-ins on the GPU, modelled on the reference's own tests.

tests/test_triton_sparse_prefill.py:69-125, tests/test_sparse_attention.py:32-70,
tests/test_gate_maxsim.py, tests/test_proto_pool.py, tests/test_group_avg.py,
tests/test_export_selected_blocks.py and tests/test_validator.py of the
reference, rewritten for 64-token blocks and checked against the oracle or the
reference's golden outputs.
"""

import numpy as np
import pytest
import torch

from golden_cases import DT, from_raw, load_case, load_npz
from oracle import oracle as O
from spruce_research_b200.export_selected_blocks import selected_ids_to_blocks, selected_mask_to_blocks
from spruce_research_b200.interfaces.validator import validate_selected_blocks
from spruce_research_b200.kernels.direct_index import KERNEL_VARIANTS
from spruce_research_b200.kernels.sparse_prefill import triton_sparse_prefill_attention_forward
from spruce_research_b200.selector.gate import FlatGate
from spruce_research_b200.sparse.attention import sparse_prefill_attention_forward
from spruce_research_b200.teacher.chunked_extract import _group_avg_tokens, _proto_pool_seq, pool_selector_features

pytestmark = pytest.mark.gpu


class _Module(torch.nn.Module):
    layer_idx = 0


@pytest.mark.parametrize("kernel_variant", KERNEL_VARIANTS)
def test_callback_matches_reference_attention_fp16_strided(kernel_variant):
    torch.manual_seed(0)
    q = torch.randn(1, 64, 2, 64, device="cuda", dtype=torch.float16).transpose(1, 2)
    k = torch.randn(1, 64, 1, 64, device="cuda", dtype=torch.float16).transpose(1, 2)
    v = torch.randn(1, 64, 1, 64, device="cuda", dtype=torch.float16).transpose(1, 2)
    assert not q.is_contiguous()
    selected = torch.zeros((1, 1, 1, 1, 1), device="cuda", dtype=torch.int32)
    actual, _ = triton_sparse_prefill_attention_forward(_Module(), q, k, v, None, selected_blocks=selected,
                                                        block_size=64, kernel_variant=kernel_variant)
    expected = O.sparse_attention(q, k, v, selected[:, 0], out_dtype=torch.float32)
    torch.testing.assert_close(actual.float().cpu(), expected, atol=2e-2, rtol=2e-2)


def test_callback_matches_reference_across_blocks_gqa():
    torch.manual_seed(4)
    q = torch.randn(1, 128, 4, 64, device="cuda", dtype=torch.float16).transpose(1, 2)
    k = torch.randn(1, 128, 2, 64, device="cuda", dtype=torch.float16).transpose(1, 2)
    v = torch.randn(1, 128, 2, 64, device="cuda", dtype=torch.float16).transpose(1, 2)
    selected = torch.tensor([[[[[0, -1], [0, 1]], [[0, -1], [0, 1]]]]], device="cuda", dtype=torch.int32)
    actual, _ = triton_sparse_prefill_attention_forward(_Module(), q, k, v, None, selected_blocks=selected,
                                                        block_size=64)
    expected = O.sparse_attention(q, k, v, selected[:, 0], out_dtype=torch.float32)
    torch.testing.assert_close(actual.float().cpu(), expected, atol=2e-2, rtol=2e-2)


def _all_causal(qb, groups=1):
    out = torch.full((1, 1, groups, qb, qb), -1, dtype=torch.int32)
    for q in range(qb):
        out[:, :, :, q, : q + 1] = torch.arange(q + 1, dtype=torch.int32)
    return out


def test_reference_backend_all_causal_blocks_equal_dense():
    torch.manual_seed(0)
    query = torch.randn(1, 4, 256, 64, device="cuda")
    key = torch.randn(1, 2, 256, 64, device="cuda")
    value = torch.randn(1, 2, 256, 64, device="cuda")
    out, weights = sparse_prefill_attention_forward(_Module(), query, key, value, None,
                                                    selected_blocks=_all_causal(4, 2).cuda(), block_size=64)
    dense = O.dense_causal_attention(query.cpu(), key.cpu(), value.cpu())
    assert out.shape == (1, 256, 4, 64) and weights is None
    assert (out.cpu() - dense).abs().max().item() < 1e-4


def test_reference_backend_pruned_block_has_no_influence():
    query = torch.ones(1, 1, 192, 64, device="cuda", dtype=torch.bfloat16)
    key = torch.ones(1, 1, 192, 64, device="cuda", dtype=torch.bfloat16)
    value = torch.zeros(1, 1, 192, 64, device="cuda", dtype=torch.bfloat16)
    value[:, :, :64] = 7.0
    # the last query block keeps its local blocks 1 and 2 but drops block 0
    selected = torch.tensor([[[[[0, -1, -1], [0, 1, -1], [1, 2, -1]]]]], device="cuda", dtype=torch.int32)
    out, _ = sparse_prefill_attention_forward(_Module(), query, key, value, None, selected_blocks=selected,
                                              block_size=64)
    assert torch.equal(out[0, 128:].float().cpu(), torch.zeros(64, 1, 64))


def test_fp32_score_accumulation_keeps_fp16_overflow_finite():
    query = torch.full((1, 1, 128, 64), 300.0, device="cuda", dtype=torch.float16)
    key = torch.full((1, 1, 128, 64), 300.0, device="cuda", dtype=torch.float16)
    value = torch.arange(128 * 64, device="cuda", dtype=torch.float16).reshape(1, 1, 128, 64) / 1000
    out, _ = sparse_prefill_attention_forward(_Module(), query, key, value, None,
                                              selected_blocks=_all_causal(2).cuda(), block_size=64)
    assert torch.isfinite(out.float()).all()


def test_flat_gate_scores_and_selection_match_reference():
    case = load_case("c1_8k")
    qc, kc, vc, wqc, wkc = case.inputs("cpu", check=False)
    q, k, v, wq, wk = case.inputs("cuda", check=False)
    ref = O.select_blocks(qc, kc, wqc, wkc, case.K, case.local_window, case.sink)
    pq, pk = pool_selector_features(q, k)
    gate = FlatGate(1, 128, 128).cuda().eval()
    with torch.no_grad():
        gate.Wq.copy_(wq[None])
        gate.Wk.copy_(wk[None])
    s = gate(pq[0][None], pk[0][None])
    assert torch.equal(s[0].cpu(), ref["scores"][0])
    sel = gate.select_blocks(pq[0][None], pk[0][None], case.K, case.local_window, case.sink)
    assert torch.equal(sel[0, 0].cpu(), ref["selected"][0])
    if case.matches_fixture():  # the reference's own outputs for these inputs
        assert (s[0].cpu() - case.golden("scores")[0]).abs().max().item() < 1e-6
        assert torch.equal(sel[0, 0].cpu(), case.golden("selected")[0])


def test_proto_pool_and_group_average_match_reference():
    z = load_npz("proto")
    for n in range(3):
        dt = DT[int(z[f"proto{n}_dtype"][0])]
        x = from_raw(z[f"proto{n}_x"], dt).cuda()
        assert torch.equal(_proto_pool_seq(x, 64, 1).cpu(), from_raw(z[f"proto{n}_p1"], dt))
        assert torch.equal(_proto_pool_seq(x, 64, 8).cpu(), from_raw(z[f"proto{n}_p8"], dt))
    x = torch.randn(1, 12, 70, 64, dtype=torch.bfloat16)
    assert torch.equal(_group_avg_tokens(x.cuda(), 2).cpu(), O.group_avg_tokens(x, 2))
    with pytest.raises(ValueError, match="at most 64 prototypes"):
        _proto_pool_seq(x.cuda(), 64, 65)


@pytest.mark.parametrize("P", [2, 4, 8])
def test_outlier_prototypes_match_oracle_on_selector_features(P):
    # the deployed selector's features: _proto_pool_seq(_group_avg_tokens(q)), _proto_pool_seq(k)
    gen = torch.Generator().manual_seed(30 + P)
    q = torch.randn((2, 28, 64 * 9 + 3, 128), generator=gen).to(torch.bfloat16)
    k = torch.randn((2, 4, 64 * 9 + 3, 128), generator=gen).to(torch.bfloat16)
    pq, pk = pool_selector_features(q.cuda(), k.cuda(), P)
    assert pq.shape == (2, 4, 10, P, 128)
    assert torch.equal(pq.cpu(), O.proto_pool_seq(O.group_avg_tokens(q, 4), 64, P))
    assert torch.equal(pk.cpu(), O.proto_pool_seq(k, 64, P))


def test_packing_drop_ins_match_reference_cases():
    z = load_npz("packing")
    for n in range(6):
        K, lw, kb, sink = (int(x) for x in z[f"pack{n}_args"])
        got = selected_ids_to_blocks(torch.from_numpy(z[f"pack{n}_ids"]).cuda(), K, lw, kb, sink)
        assert torch.equal(got.cpu(), torch.from_numpy(z[f"pack{n}_out"]))
    # tests/test_export_selected_blocks.py:11-28 of the reference
    selected = torch.zeros((2, 2, 4, 4), dtype=torch.bool)
    selected[..., :, 0] = True
    selected[..., 3, 1] = True
    packed = selected_mask_to_blocks(selected.cuda(), k_selected=3, local_window=1).cpu()
    assert packed[0, 0, 0].tolist() == [[0, -1, -1], [0, 1, -1], [0, 1, 2], [0, 2, 3]]
    # sink forcing (tests/test_export_selected_blocks.py:46-59)
    ids = torch.tensor([[[[5, 5], [5, 5], [5, 5], [2, 5], [2, 3], [3, 4]]]], dtype=torch.long).cuda()
    with_sink = selected_ids_to_blocks(ids, k_selected=4, local_window=1, key_blocks=6, sink_blocks=1).cpu()
    assert all(with_sink[0, 0, 0, r, 0].item() == 0 for r in range(6))
    validate_selected_blocks(with_sink.cuda())


def test_gpu_validator_raises_reference_messages():
    def row(ids, k=4):
        return list(ids) + [-1] * (k - len(ids))

    validate_selected_blocks(torch.tensor([[[[row([0]), row([0, 1]), row([0, 1, 2]), row([0, 2, 3])]]]],
                                          dtype=torch.int32, device="cuda"))
    for rows, msg in [([row([0, 5])], "future"), ([row([0]), row([0, 1, 1])], "Duplicate"),
                      ([row([0]), row([0, 1]), row([0, 2, 1])], "Not sorted"),
                      ([row([0]), row([1])], "Missing local-window"),
                      ([row([0]), [0, -1, 1, -1]], "trailing")]:
        t = torch.tensor([[[rows]]], dtype=torch.int32, device="cuda")
        with pytest.raises(AssertionError, match=msg) as gpu_err:
            validate_selected_blocks(t)
        with pytest.raises(AssertionError) as cpu_err:
            O.validate_selected_blocks(t.cpu())
        assert str(gpu_err.value) == str(cpu_err.value)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_block_mask_launcher_matches_oracle_per_head_masks(dtype, D):
    # kernels/seerattention_triton.py:71-90 of the reference: BHSD q/k/v with K/V
    # expanded per head, a per-head bool block mask, output BHSD.
    from spruce_research_b200.kernels.seerattention import block_mask_to_indices, block_sparse_triton

    gen = torch.Generator().manual_seed(21)
    B, H, T = 2, 3, 64 * 5 + 17
    qb = (T + 63) // 64
    q, k, v = (torch.randn((B, H, T, D), generator=gen).to(dtype) for _ in range(3))
    mask = torch.rand((B, H, qb, qb), generator=gen) > 0.5
    mask |= torch.eye(qb, dtype=torch.bool)  # every row keeps its diagonal block
    out = block_sparse_triton(q.cuda(), k.cuda(), v.cuda(), mask.cuda(), D ** -0.5)
    assert out.shape == (B, H, T, D) and out.dtype == dtype
    want = O.sparse_attention(q, k, v, block_mask_to_indices(mask), out_dtype=torch.float32)  # [B, T, H, D]
    err = (out.float().cpu().transpose(1, 2) - want).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3


def test_maxsim_gate_matches_oracle_and_reference():
    # FlatGate.forward / score_candidates with P = 8 (selector/gate.py:29-171)
    from test_oracle_golden import _maxsim_case

    z = load_npz("maxsim")
    for n in range(2):
        q, k, wq, wk = _maxsim_case(z, n)
        qf, kf = _proto_pool_seq(q.cuda(), 64, 8), _proto_pool_seq(k.cuda(), 64, 8)   # [1, G, nb, 8, d]
        gate = FlatGate(1, q.shape[-1], wq.shape[-1]).cuda().eval()
        with torch.no_grad():
            gate.Wq.copy_(wq)
            gate.Wk.copy_(wk)
        s = gate(qf, kf)[0].cpu()
        qp, kp = O.project(qf[0].cpu(), wq[0]), O.project(kf[0].cpu(), wk[0])
        assert torch.equal(s, O.maxsim(qp, kp))
        want = torch.from_numpy(z[f"ms{n}_scores"])[0]
        assert (s - want).abs().max().item() <= 2e-6 * want.abs().max().item()
        cand = torch.from_numpy(z[f"ms{n}_cand"])
        sc = gate.score_candidates(qf, kf, cand.cuda())[0].cpu()
        assert torch.equal(sc, O.maxsim(qp, kp, cand[0]))
    with pytest.raises(ValueError, match="1 to 8 prototypes"):
        gate(torch.zeros(1, 1, 2, 9, q.shape[-1], device="cuda"), torch.zeros(1, 1, 2, 9, q.shape[-1], device="cuda"))
