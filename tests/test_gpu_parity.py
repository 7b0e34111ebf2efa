"""CUDA path vs the CPU oracle and the reference's golden outputs (B200 only).

The chain: the CPU suite pins oracle == reference on the fixtures' inputs;
here CUDA == oracle on the inputs this host regenerates (torch's CPU sampler
can differ in the last bit between CPU models), and CUDA == reference outputs
directly whenever the regenerated inputs equal the fixture's.

Parity bar:
  * pooled features, gate scores and selected block indices: bit-exact;
  * attention: max-abs <= 2e-2 and mean-abs <= 2e-3 for bf16/fp16,
    max-abs <= 1e-4 for fp32, against the reference's block-sparse attention
    on the same indices.
"""
import pytest
import torch

from golden_cases import CASE_NAMES, load_case, load_npz
from oracle import oracle as O
from spruce_research_b200 import native
from spruce_research_b200.synthetic import LayerShape, make_layer_inputs

pytestmark = pytest.mark.gpu

ATOL_MAX_16 = 2e-2
ATOL_MEAN_16 = 2e-3
ATOL_MAX_32 = 1e-4


def assert_attention_close(actual: torch.Tensor, expected: torch.Tensor, dtype: torch.dtype, what: str = ""):
    err = (actual.float().cpu() - expected.float().cpu()).abs()
    assert torch.isfinite(actual.float()).all(), f"{what}: non-finite output"
    if dtype == torch.float32:
        assert err.max().item() <= ATOL_MAX_32, f"{what}: max-abs {err.max().item():.3e}"
    else:
        assert err.max().item() <= ATOL_MAX_16, f"{what}: max-abs {err.max().item():.3e}"
        assert err.mean().item() <= ATOL_MEAN_16, f"{what}: mean-abs {err.mean().item():.3e}"


def _case(name):
    """(case, cpu inputs, cuda inputs, oracle selector result, inputs equal the fixture's)."""
    case = load_case(name)
    cpu = case.inputs("cpu", check=False)
    cuda = case.inputs("cuda", check=False)
    ref = O.select_blocks(cpu[0], cpu[1], cpu[3], cpu[4], case.K, case.local_window, case.sink)
    return case, cpu, cuda, ref, case.matches_fixture()


@pytest.mark.parametrize("name", CASE_NAMES)
def test_pooling_bit_exact_with_reference(name):
    case, cpu, (q, k, v, wq, wk), ref, same = _case(name)
    pq, pk = native.pool_qk(q, k)
    torch.cuda.synchronize()
    assert torch.equal(pq.cpu(), ref["pooled_q"]), "pooled Q differs from the oracle"
    assert torch.equal(pk.cpu(), ref["pooled_k"]), "pooled K differs from the oracle"
    if same:  # the oracle is pinned to these by the CPU suite; check directly too
        assert torch.equal(pq.cpu(), case.golden("pooled_q")), "pooled Q differs from the reference"
        assert torch.equal(pk.cpu(), case.golden("pooled_k")), "pooled K differs from the reference"


# group sizes and head dims the reference fixtures do not cover: the exact
# multiply by 1/8, the run-time group size (3, 5, 6, 16), D = 96 and 256, ragged
# lengths and batch 2
POOL_SHAPES = [
    # (B, Hq, Hkv, T, D, dtype)
    (2, 24, 8, 1000, 128, torch.bfloat16),   # rep 3
    (1, 40, 8, 777, 64, torch.float16),      # rep 5
    (1, 48, 8, 2053, 128, torch.float32),    # rep 6
    (1, 32, 4, 300, 256, torch.bfloat16),    # rep 8, D = 256
    (2, 16, 1, 130, 96, torch.bfloat16),     # rep 16, D = 96 (5 blocks of 48 threads per CTA)
    (1, 8, 2, 200, 256, torch.float32),      # rep 4, D = 256 in fp32 (one block per CTA)
    (1, 4, 4, 65, 128, torch.float16),       # rep 1: queries pooled per head
]


@pytest.mark.parametrize("B,Hq,Hkv,T,D,dtype", POOL_SHAPES)
def test_pooling_group_sizes_bit_exact_with_oracle(B, Hq, Hkv, T, D, dtype):
    q, k, _ = make_layer_inputs(LayerShape(B, Hq, Hkv, T, D), dtype, seed=Hq + T)
    pq, pk = native.pool_qk(q.cuda(), k.cuda())
    torch.cuda.synchronize()
    assert torch.equal(pq.cpu(), O.proto_pool_seq(O.group_avg_tokens(q, Hkv), 64, 1)[:, :, :, 0])
    assert torch.equal(pk.cpu(), O.proto_pool_seq(k, 64, 1)[:, :, :, 0])


@pytest.mark.parametrize("name", CASE_NAMES)
def test_scores_bit_exact_with_oracle(name):
    case, cpu, (q, k, v, wq, wk), ref, same = _case(name)
    pq, pk = native.pool_qk(q, k)
    qp = native.gate_project(pq, wq)
    kp = native.gate_project(pk, wk)
    B, G = pq.shape[:2]
    s = native.gate_scores(qp.flatten(0, 1), kp.flatten(0, 1)).view(B, G, pq.shape[2], pk.shape[2])
    assert torch.equal(qp.cpu(), ref["qp"]), "projection differs from the oracle's fixed fma order"
    assert torch.equal(kp.cpu(), ref["kp"])
    assert torch.equal(s.cpu(), ref["scores"]), "scores differ from the oracle"
    if same:  # and within fp32 round-off of the reference's MKL scores
        assert (s.cpu() - case.golden("scores")).abs().max().item() < 1e-6


@pytest.mark.parametrize("name", CASE_NAMES)
def test_selected_blocks_bit_exact_with_reference(name):
    case, cpu, (q, k, v, wq, wk), ref, same = _case(name)
    sel = native.select_blocks(q, k, wq, wk, case.K, case.local_window, case.sink)
    torch.cuda.synchronize()
    assert torch.equal(sel.cpu(), ref["selected"]), "selected_blocks differ from the oracle"
    if same:
        assert torch.equal(sel.cpu(), case.golden("selected")), "selected_blocks differ from the reference"


@pytest.mark.parametrize("name", CASE_NAMES)
def test_attention_matches_reference(name):
    case, cpu, (q, k, v, wq, wk), ref, same = _case(name)
    idx = ref["selected"]
    out = native.sparse_attention(q, k, v, idx.cuda())
    torch.cuda.synchronize()
    # whole output against the oracle (fp32 math, same indices)
    want = O.sparse_attention(cpu[0], cpu[1], cpu[2], idx, out_dtype=torch.float32)
    assert_attention_close(out, want, case.dtype, name + " vs oracle")
    if same:
        assert_attention_close(out[:, case.out_rows()], case.golden("out"), case.dtype, name)


ATTN_SHAPES = [
    # (B, Hq, Hkv, T, D, dtype, K)
    (1, 28, 4, 1024, 128, torch.bfloat16, 6),
    (1, 28, 4, 1000, 128, torch.bfloat16, 5),     # ragged tail
    (1, 7, 1, 640, 128, torch.float16, 4),
    (2, 4, 2, 448, 64, torch.bfloat16, 3),
    (1, 2, 2, 256, 64, torch.float16, 4),          # MHA (one head per group)
    (1, 12, 2, 70, 128, torch.bfloat16, 2),        # fewer tokens than two blocks
    (1, 6, 2, 320, 64, torch.float32, 3),
]


def _random_rows(B, G, qb, K, seed, dup=False):
    gen = torch.Generator().manual_seed(seed)
    rows = torch.full((B, G, qb, K), -1, dtype=torch.int32)
    for b in range(B):
        for g in range(G):
            for i in range(qb):
                cand = torch.randperm(i + 1, generator=gen)[: K - 1].tolist()
                ids = sorted(set(cand) | {i})[:K]
                rows[b, g, i, : len(ids)] = torch.tensor(ids, dtype=torch.int32)
    return rows


@pytest.mark.parametrize("B,Hq,Hkv,T,D,dtype,K", ATTN_SHAPES)
def test_attention_random_rows_vs_oracle(B, Hq, Hkv, T, D, dtype, K):
    shape = LayerShape(B, Hq, Hkv, T, D)
    q, k, v = make_layer_inputs(shape, dtype, seed=T + D)
    idx = _random_rows(B, Hkv, shape.query_blocks, K, seed=T)
    dev = [t.transpose(1, 2).contiguous().cuda().transpose(1, 2) for t in (q, k, v)]
    out = native.sparse_attention(*dev, idx.cuda())
    ref = O.sparse_attention(q, k, v, idx, out_dtype=torch.float32)
    assert_attention_close(out, ref, dtype, f"{shape}")


def test_attention_contiguous_bhtd_layout_and_padding_skip():
    shape = LayerShape(1, 8, 2, 512, 128)
    q, k, v = make_layer_inputs(shape, torch.bfloat16, seed=5)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()     # [B, H, T, D] storage
    idx = _random_rows(1, 2, 8, 5, seed=3)
    out = native.sparse_attention(q.cuda(), k.cuda(), v.cuda(), idx.cuda())
    ref = O.sparse_attention(q, k, v, idx, out_dtype=torch.float32)
    assert_attention_close(out, ref, torch.bfloat16, "contiguous")


def test_all_causal_blocks_match_dense_attention():
    # 100% density: every causal block selected == dense causal attention.
    shape = LayerShape(1, 14, 2, 640, 128)
    q, k, v = make_layer_inputs(shape, torch.bfloat16, seed=9)
    qb = shape.query_blocks
    idx = torch.full((1, 2, qb, qb), -1, dtype=torch.int32)
    for i in range(qb):
        idx[0, :, i, : i + 1] = torch.arange(i + 1, dtype=torch.int32)
    dev = [t.transpose(1, 2).contiguous().cuda().transpose(1, 2) for t in (q, k, v)]
    out = native.sparse_attention(*dev, idx.cuda())
    ref = O.dense_causal_attention(q, k, v)
    assert_attention_close(out, ref, torch.bfloat16, "all blocks vs dense")


def test_empty_row_gives_zeros_and_status():
    shape = LayerShape(1, 4, 2, 128, 64)
    q, k, v = make_layer_inputs(shape, torch.bfloat16, seed=1)
    idx = torch.tensor([[[[0, -1], [-1, -1]], [[0, -1], [0, 1]]]], dtype=torch.int32)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = [t.transpose(1, 2).contiguous().cuda().transpose(1, 2) for t in (q, k, v)]
    out = native.sparse_attention(*dev, idx.cuda(), status=status)
    torch.cuda.synchronize()
    assert status.item() & 2
    assert torch.equal(out[0, 64:, 0:2].float().cpu(), torch.zeros(64, 2, 64))


def test_pack_selected_ids_matches_reference():
    z = load_npz("packing")
    n = 0
    while f"pack{n}_ids" in z:
        ids = torch.from_numpy(z[f"pack{n}_ids"])
        K, lw, kb, sink = (int(x) for x in z[f"pack{n}_args"])
        L, G, qb, C = ids.shape
        got = native.pack_selected_ids(ids.view(L * G, qb, C).cuda(), K, lw, kb, sink)
        assert torch.equal(got.view(1, L, G, qb, K).cpu(), torch.from_numpy(z[f"pack{n}_out"])), f"case {n}"
        n += 1
    assert n >= 6


def test_projection_of_unaligned_rows_matches_the_aligned_path():
    """Rows that do not start on a 16-byte boundary take the scalar-load projection
    (the shared-W kernel copies rows by 16-byte cp.async), with the same results."""
    g = torch.Generator().manual_seed(3)
    base = torch.randn(2048 * 128 + 1, generator=g).to(torch.bfloat16).cuda()
    x = base[1:].view(2048, 128)  # contiguous, one element into its storage
    assert x.is_contiguous() and x.data_ptr() % 16 != 0
    W = torch.randn(128, 128, generator=g).cuda()
    got = native.gate_project(x, W)
    want = native.gate_project(x.clone(), W)  # 16-byte aligned: the shared-W kernel
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(got.cpu(), O.project(x.cpu(), W.cpu()))
