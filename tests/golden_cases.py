"""Load the golden fixtures made by tests/golden/make_golden.py (reference outputs)."""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np
import torch

from spruce_research_b200.synthetic import LayerShape, make_gate_weights, make_layer_inputs

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DT = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}
CASE_NAMES = ["c0", "c1_small", "c1_8k", "ragged_bf16", "gqa_fp16", "batch2_f32"]


def from_raw(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.view(dtype) if dtype in (torch.bfloat16, torch.float16) else t


@dataclass
class GoldenCase:
    name: str
    shape: LayerShape
    dtype: torch.dtype
    seed: int
    rope: float | None
    K: int
    local_window: int
    sink: int
    z: dict

    def matches_fixture(self) -> bool:
        """True when this host regenerates the exact inputs the reference saw.

        torch's CPU normal sampler has vector paths that depend on the host's
        instruction set, so another CPU model can change the inputs' last bits.
        The CPU suite (run where the fixtures were made) pins oracle == reference;
        GPU tests compare CUDA == oracle on whatever inputs this host makes, and
        also against the fixture outputs when this returns True.
        """
        q, k, v = make_layer_inputs(self.shape, self.dtype, self.seed, rope_theta=self.rope)
        cs = np.array([q.double().sum().item(), k.double().sum().item(), v.double().sum().item()])
        return bool(np.allclose(cs, self.z["checksum"], rtol=1e-12, atol=1e-6))

    def inputs(self, device="cpu", check=True):
        q, k, v = make_layer_inputs(self.shape, self.dtype, self.seed, rope_theta=self.rope)
        cs = np.array([q.double().sum().item(), k.double().sum().item(), v.double().sum().item()])
        if check:
            assert np.allclose(cs, self.z["checksum"], rtol=1e-12, atol=1e-6), "synthetic generator drifted"
        wq, wk = make_gate_weights(1, self.shape.head_dim, self.shape.head_dim, self.seed + 1000)
        if device != "cpu":
            # keep the reference's strided [B, H, T, D] views of token-major storage
            q = q.transpose(1, 2).contiguous().to(device).transpose(1, 2)
            k = k.transpose(1, 2).contiguous().to(device).transpose(1, 2)
            v = v.transpose(1, 2).contiguous().to(device).transpose(1, 2)
            wq, wk = wq.to(device), wk.to(device)
        return q, k, v, wq[0], wk[0]

    def golden(self, key: str) -> torch.Tensor:
        if key in ("pooled_q", "pooled_k", "out"):
            return from_raw(self.z[key], self.dtype)
        return torch.from_numpy(np.ascontiguousarray(self.z[key]))

    def out_rows(self) -> torch.Tensor:
        T = self.shape.tokens
        return torch.cat([torch.arange(b * 64, min((b + 1) * 64, T)) for b in self.z["out_blocks"]])


def load_case(name: str) -> GoldenCase:
    z = dict(np.load(os.path.join(HERE, f"{name}.npz")))
    B, Hq, Hkv, T, D = (int(x) for x in z["shape"])
    K, lw, sink = (int(x) for x in z["policy"])
    rope = float(z["rope"][0]) or None
    return GoldenCase(name, LayerShape(B, Hq, Hkv, T, D), DT[int(z["dtype"][0])], int(z["seed"][0]), rope,
                      K, lw, sink, z)


def load_npz(name: str) -> dict:
    return dict(np.load(os.path.join(HERE, f"{name}.npz")))


SUMMARY_CASE_NAMES = ["sum_ragged_bf16", "sum_batch2_f32", "sum_c0_f32", "sum_c1_8k_bf16", "sum_gqa_fp16_bs16"]


@dataclass
class SummaryCase:
    """One build_kv_summary_table fixture of summaries.npz (reference outputs)."""

    name: str
    shape: LayerShape
    dtype: torch.dtype
    seed: int
    rope: float | None
    block_size: int
    prototypes: int
    mask_kind: int
    z: dict

    def inputs(self, device="cpu"):
        """(key, value, token_mask) as the generator made them; K/V keep the [B, T, H, D] storage."""
        _, k, v = make_layer_inputs(self.shape, self.dtype, self.seed, rope_theta=self.rope)
        mask = None
        if self.mask_kind:
            B, T = self.shape.batch, self.shape.tokens
            mask = torch.ones((B, T), dtype=torch.bool)
            if self.mask_kind == 1:
                mask[0, 10:12] = False
                mask[0, 100:111] = False
                mask[-1, 200:] = False
            else:
                mask[-1, T - 37:] = False
        if device != "cpu":
            k = k.transpose(1, 2).contiguous().to(device).transpose(1, 2)
            v = v.transpose(1, 2).contiguous().to(device).transpose(1, 2)
            mask = None if mask is None else mask.to(device)
        return k, v, mask

    def get(self, key: str) -> torch.Tensor:
        return torch.from_numpy(np.ascontiguousarray(self.z[f"{self.name}_{key}"]))

    @property
    def nodes(self) -> torch.Tensor:
        return self.get("nodes")

    @property
    def sha256(self) -> bytes:
        return bytes(self.z[f"{self.name}_sha256"].tolist())


def load_summary_case(name: str) -> SummaryCase:
    z = load_npz("summaries")
    B, Hq, Hkv, T, D, dt, seed, bs, P = (int(x) for x in z[f"{name}_args"])
    rope = float(z[f"{name}_rope"][0]) or None
    return SummaryCase(name, LayerShape(B, Hq, Hkv, T, D), DT[dt], seed, rope, bs, P,
                       int(z[f"{name}_mask"][0]), z)


def table_sha256(keys: torch.Tensor, values: torch.Tensor, counts: torch.Tensor) -> bytes:
    import hashlib

    h = hashlib.sha256()
    for a in (keys, values, counts):
        h.update(a.detach().cpu().contiguous().numpy().tobytes())
    return h.digest()


RESIDUAL_CASE_NAMES = ("r_bf16", "r_f32")


def load_residual_case(name: str):
    """Inputs, routes, residual nodes and the reference's outputs per summary prototype count."""
    z = load_npz("residual")
    dt = DT[int(z[f"{name}_dtype"][0])]
    q, k, v = (from_raw(z[f"{name}_{x}"], dt) for x in ("q", "k", "v"))
    sel = torch.from_numpy(z[f"{name}_selected"])
    nodes = torch.from_numpy(z[f"{name}_nodes"])
    outs = {int(P): from_raw(z[f"{name}_out{int(P)}"], dt) for P in z[f"{name}_protos"]}
    return q, k, v, sel, nodes, outs


BIG_CASE_NAMES = ("c1_full", "c2")


@dataclass
class BigCase:
    """A headline configuration in full (c1_full: BASELINE config 1, c2: config 2).

    Holds the reference's whole selected_blocks, the score gap at each row's
    selection boundary, digests of its pooled features and the attention output
    of a few sampled query blocks (tests/golden/make_golden.py, big_case).
    """

    name: str
    shape: LayerShape
    dtype: torch.dtype
    seed: int
    wseed: int
    rope: float | None
    K: int
    local_window: int
    sink: int
    z: dict

    def inputs(self):
        """(q, k, v, wq, wk) on the CPU: [B, H, T, D] views of token-major storage, [d, p] weights."""
        q, k, v = make_layer_inputs(self.shape, self.dtype, self.seed, rope_theta=self.rope)
        wq, wk = make_gate_weights(1, self.shape.head_dim, self.shape.head_dim, self.wseed)
        return q, k, v, wq[0], wk[0]

    def same_inputs(self, q, k, v) -> bool:
        """True when these are the inputs the reference saw (see GoldenCase.matches_fixture)."""
        cs = np.array([q.double().sum().item(), k.double().sum().item(), v.double().sum().item()])
        return bool(np.allclose(cs, self.z["checksum"], rtol=1e-12, atol=1e-6))

    @property
    def selected(self) -> torch.Tensor:
        """int32 [B, Hkv, qb, K]."""
        return torch.from_numpy(self.z["selected"].astype(np.int32))

    @property
    def gap(self) -> torch.Tensor:
        return torch.from_numpy(self.z["gap"])

    @property
    def out(self) -> torch.Tensor:
        """The reference's attention output at out_rows(): [B, rows, Hq, D] in the input dtype."""
        return from_raw(self.z["out"], self.dtype)

    @property
    def out_blocks(self) -> list:
        return [int(i) for i in self.z["out_blocks"]]

    def out_rows(self) -> torch.Tensor:
        T = self.shape.tokens
        return torch.cat([torch.arange(b * 64, min((b + 1) * 64, T)) for b in self.out_blocks])

    def digest(self, key: str) -> bytes:
        return bytes(self.z[f"{key}_sha256"].tolist())


def load_big_case(name: str) -> BigCase:
    z = load_npz(name)
    B, Hq, Hkv, T, D = (int(x) for x in z["shape"])
    K, lw, sink = (int(x) for x in z["policy"])
    rope = float(z["rope"][0]) or None
    return BigCase(name, LayerShape(B, Hq, Hkv, T, D), DT[int(z["dtype"][0])], int(z["seed"][0]),
                   int(z["wseed"][0]), rope, K, lw, sink, z)


def raw_sha256(t: torch.Tensor) -> bytes:
    """SHA-256 of a tensor's bytes in its own dtype (bf16/fp16 as their 16-bit patterns)."""
    import hashlib

    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).digest()


# ---------------------------------------------------------------- whole-model case (tests/golden/live.npz)
LIVE_MODEL = dict(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                  num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=8192, rope_theta=1e6)


def tiny_qwen2(seed: int, dtype=torch.bfloat16):
    """A random-init Qwen2 of LIVE_MODEL's shape, initialised on the CPU from `seed` (so every
    host with the same torch builds the same weights); move it to a device afterwards."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    with torch.device("cpu"):
        model = Qwen2ForCausalLM(Qwen2Config(**LIVE_MODEL)).to(dtype).eval()
    return model


def model_checksum(model) -> float:
    return float(sum(p.detach().double().sum().item() for p in model.parameters()))


def live_rows(T: int) -> torch.Tensor:
    """Token rows whose hidden states the fixture stores: the first block and the last two."""
    return torch.cat([torch.arange(0, 64), torch.arange(T - 128, T)])
