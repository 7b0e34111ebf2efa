"""Whole-model flows (spruce_research_b200.live) on a tiny random Qwen2.

CPU: argument checks, registration, the decode path (query length != key
length goes to SDPA unchanged) and the loud failure of prefill without CUDA.
GPU: the one-pass and two-pass flows agree where they must (layer 0, every
block selected), dense layers reproduce the SDPA model, routes validate,
and a decode step after a sparse prefill runs on the cache it filled.
"""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from spruce_research_b200.interfaces.validator import validate_selected_blocks  # noqa: E402
from spruce_research_b200.live import (SPRUCE_LIVE_SPARSE_PREFILL, LiveSelector,  # noqa: E402
                                       live_sparse_prefill_attention_forward, register_live_sparse_prefill_attention,
                                       sparse_prefill)
from spruce_research_b200.selector.gate import FlatGate  # noqa: E402


def _tiny_qwen(device, layers=3, seed=0, dtype=torch.bfloat16):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=layers,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=8192,
                      rope_theta=1e6)
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg).to(dtype).eval()
    model.set_attn_implementation("sdpa")
    return model


def _gate(layers, d=64, seed=1, device="cpu"):
    torch.manual_seed(seed)
    return FlatGate(layers, d, d).to(device).eval()


def test_selector_arguments_and_widths():
    gate = _gate(2)
    with pytest.raises(ValueError, match="exactly one"):
        LiveSelector(gate, mode="flat")
    with pytest.raises(ValueError, match="mode"):
        LiveSelector(gate, mode="dense", k_selected=4)
    assert LiveSelector(gate, k_selected=7).width(100) == 7
    assert LiveSelector(gate, density=1.0).width(40) == 40
    assert LiveSelector(gate, density=0.0, local_window=2, sink_blocks=1).width(40) == 4
    assert LiveSelector(gate, mode="tree", beam=6, local_window=1).width(40) == 8
    assert LiveSelector(gate, mode="tree", k_selected=12).width(40) == 12


def test_registration_and_decode_goes_to_sdpa():
    from transformers import AttentionInterface
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    assert register_live_sparse_prefill_attention() == SPRUCE_LIVE_SPARSE_PREFILL
    assert SPRUCE_LIVE_SPARSE_PREFILL in AttentionInterface._global_mapping

    class Layer(torch.nn.Module):
        layer_idx, num_key_value_groups, is_causal = 0, 4, True

    gen = torch.Generator().manual_seed(2)
    q = torch.randn((1, 8, 1, 64), generator=gen)
    k = torch.randn((1, 2, 70, 64), generator=gen)
    v = torch.randn((1, 2, 70, 64), generator=gen)
    got, _ = live_sparse_prefill_attention_forward(Layer(), q, k, v, None, spruce_selector=None, scaling=0.125)
    want, _ = sdpa_attention_forward(Layer(), q, k, v, None, scaling=0.125)
    assert torch.equal(got, want)


def test_prefill_without_cuda_fails_loudly():
    model = _tiny_qwen("cpu", layers=1, dtype=torch.float32)
    sel = LiveSelector(_gate(1), k_selected=4)
    ids = torch.randint(0, 512, (1, 200))
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_prefill(model, ids, sel, flow="one_pass")


def _ids(T, seed=3):
    return torch.randint(0, 512, (1, T), generator=torch.Generator().manual_seed(seed)).cuda()


def _logits(out):
    return out.logits[0, -1].float()


@pytest.mark.gpu
def test_all_blocks_flows_match_each_other_and_dense():
    model = _tiny_qwen("cuda")
    T = 64 * 24 + 17
    qb = (T + 63) // 64
    ids = _ids(T)
    with torch.no_grad():
        dense = _logits(model(ids, use_cache=False, logits_to_keep=1))
    one, _ = sparse_prefill(model, ids, LiveSelector(_gate(3, device="cuda"), k_selected=qb), flow="one_pass",
                            use_cache=False)
    two, selected = sparse_prefill(model, ids, LiveSelector(_gate(3, device="cuda"), k_selected=qb),
                                   flow="two_pass", use_cache=False)
    # every causal block selected: the two flows run identical attention
    assert torch.equal(_logits(one), _logits(two))
    assert ((selected >= 0).sum(-1) == torch.arange(1, qb + 1, device="cuda")).all()
    cos = torch.nn.functional.cosine_similarity(_logits(one), dense, dim=0).item()
    assert cos > 0.9995, cos
    assert (_logits(one) - dense).abs().max().item() <= 0.03 * dense.abs().max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["flat", "tree"])
def test_layer0_routes_agree_between_flows(mode):
    model = _tiny_qwen("cuda", seed=4)
    T = 64 * 40 + 5
    ids = _ids(T, seed=5)
    kw = dict(k_selected=6) if mode == "flat" else dict(beam=4, local_window=1, sink_blocks=0)
    one = LiveSelector(_gate(3, device="cuda"), mode=mode, keep_routes=True, **kw)
    sparse_prefill(model, ids, one, flow="one_pass", use_cache=False)
    _, selected = sparse_prefill(model, ids, LiveSelector(_gate(3, device="cuda"), mode=mode, **kw),
                                 flow="two_pass", use_cache=False)
    assert selected.shape[:3] == (1, 3, 2) and selected.dtype == torch.int32
    # layer 0 sees the same embeddings in both flows
    assert torch.equal(one.routes[0][0], selected[0, 0])
    lw = 0 if mode == "flat" else 1
    validate_selected_blocks(selected, local_window=lw)
    validate_selected_blocks(torch.stack([one.routes[l] for l in range(3)], 1), local_window=lw)


@pytest.mark.gpu
def test_dense_layers_reproduce_sdpa_and_decode_runs():
    model = _tiny_qwen("cuda", seed=6)
    T = 64 * 10 + 33
    ids = _ids(T, seed=7)
    with torch.no_grad():
        dense = model(ids, use_cache=True, logits_to_keep=1)
    sel = LiveSelector(_gate(3, device="cuda"), k_selected=3)
    out, _ = sparse_prefill(model, ids, sel, flow="one_pass", dense_layers=(0, 1, 2))
    torch.testing.assert_close(_logits(out), _logits(dense), atol=1e-2, rtol=1e-2)
    # a sparse prefill, then one decode step on the cache it filled (decode -> SDPA)
    out, _ = sparse_prefill(model, ids, sel, flow="one_pass")
    nxt = out.logits[:, -1:].argmax(-1)
    model.set_attn_implementation(SPRUCE_LIVE_SPARSE_PREFILL)
    try:
        with torch.no_grad():
            step = model(nxt, past_key_values=out.past_key_values, use_cache=True, spruce_selector=sel)
    finally:
        model.set_attn_implementation("sdpa")
    assert step.logits.shape == (1, 1, 512) and torch.isfinite(step.logits).all()
    assert out.past_key_values.get_seq_length() == T + 1


@pytest.mark.gpu
def test_sparse_density_model_passes_the_reference_acceptance_against_its_own_backend():
    """A tiny Qwen2 at ~10% block density (K = 4 of 65 query blocks, sink + diagonal + 2
    routed), on the fixed routes stored with it: this library's drop-in callback against the
    reference's own torch backend run on the CPU (tests/golden/live.npz), judged by the
    reference's acceptance criteria (spruce_research_b200.acceptance) on the last token's
    logits and the final hidden states, and by relative RMSE <= 0.02 on every layer's output."""
    import numpy as np

    from golden_cases import from_raw, live_rows, load_npz, model_checksum, tiny_qwen2
    from spruce_research_b200.acceptance import logits_error, passes_acceptance, tensor_error
    from spruce_research_b200.kernels.sparse_prefill import register_triton_sparse_prefill_attention

    z = load_npz("live")
    model_seed, ids_seed, _ = (int(x) for x in z["seeds"])
    T = int(z["tokens"][0])
    model = tiny_qwen2(model_seed)
    assert abs(model_checksum(model) - float(z["model_checksum"][0])) <= 1e-9 * abs(float(z["model_checksum"][0]))
    model = model.cuda()
    ids = torch.randint(0, 512, (1, T), generator=torch.Generator().manual_seed(ids_seed)).cuda()
    routes = torch.from_numpy(z["routes"].astype(np.int32)).cuda()
    model.set_attn_implementation(register_triton_sparse_prefill_attention())
    try:
        with torch.no_grad():
            out = model.base_model(ids, use_cache=False, selected_blocks=routes, block_size=64,
                                   output_hidden_states=True)
            final = out.last_hidden_state
            logits = model.get_output_embeddings()(final[:, -1:, :])
    finally:
        model.set_attn_implementation("sdpa")
    rows = live_rows(T).cuda()
    lg = logits_error(logits[0, 0].cpu(), torch.from_numpy(z["logits"]))
    fh = tensor_error(final[0, rows].cpu(), from_raw(z["final_rows"], torch.bfloat16))
    assert passes_acceptance(lg, fh), {"logits": lg, "final_hidden": fh}
    want_layers = from_raw(z["layer_rows"], torch.bfloat16)
    for layer, h in enumerate(out.hidden_states[1:1 + want_layers.shape[0]]):
        err = tensor_error(h[0, rows].cpu(), want_layers[layer])
        assert err["relative_rmse"] <= 0.02, (layer, err)
