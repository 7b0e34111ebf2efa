"""Host-side logic: C-ABI library, argument checks, synthetic workload maths, sharding.

No GPU compute runs here: the library is loaded and exercised only on paths
that reject arguments before touching the device.
"""
import ctypes
import os
import re

import pytest
import torch

from spruce_research_b200 import _lib, native
from spruce_research_b200.sharding import plan
from spruce_research_b200.synthetic import (LayerShape, causal_block_entries, k_for_density, make_gate_weights,
                                            make_layer_inputs, sparse_attention_flops)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "spruce_b200.h")).read()
    return sorted(set(re.findall(r"SPRUCE_API\s+[\w\s\*]*?\b(spruce_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    L = _lib.load()
    names = header_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(L, name), f"{name} declared in include/spruce_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert L.spruce_abi_version() == 1


def test_policy_errors_are_value_errors_before_any_device_work():
    L = _lib.load()
    out3 = _lib.int64s(0, 0, 0)
    rc = L.spruce_gate_select(None, None, 1, 1, 4, 8, 2, 1, 1, None, out3, None)  # K=2 < lw+1+sink=3
    assert rc == _lib.ERR_INVALID
    with pytest.raises(ValueError, match="cannot fit local window size 2 plus 1 sink"):
        _lib.check(rc)
    s4 = _lib.int64s(1, 1, 1, 1)
    rc = L.spruce_sparse_attention_fwd(None, s4, None, s4, None, s4, None, s4, None, s4, 1, 1, 2, 1, 64, 96, 3,
                                       0.1, None, None)
    with pytest.raises(ValueError, match="head_dim 64 or 128"):
        _lib.check(rc)
    rc = L.spruce_pack_selected_ids(None, 1, 4, 2, 3, 1, 0, 0, None, None)
    with pytest.raises(ValueError, match="key_blocks"):
        _lib.check(rc)


def test_selector_sizes_that_would_overflow_are_rejected_before_any_device_work():
    """A shape whose scratch size does not fit in int64 (or whose rows overflow the kernels'
    int indices) gets size -1 and an ERR_INVALID from both selector entry points, so a
    wrapped product can never pass the no-allocation entry point's 16 MiB check."""
    L = _lib.load()
    huge_t = 1 << 62
    assert L.spruce_select_workspace_bytes(1, 4, huge_t, 128, 128, 1) == -1
    assert L.spruce_select_workspace_bytes(1 << 40, 1 << 20, 1 << 20, 128, 128, 1) == -1
    assert L.spruce_select_workspace_bytes(1, 4, 131072, 128, 128, 1) == 12582912   # config 2: 12 MiB
    s4 = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    args = (None, s4, None, s4, 1, 1, 28, 4, huge_t, 128, None, None, 128, 106, 0, 1, None, _lib.int64s(1, 1, 1))
    assert L.spruce_select_blocks_noalloc(*args, None) == _lib.ERR_INVALID
    assert "bad selector shape" in L.spruce_last_error().decode()
    assert L.spruce_select_blocks_rows(*args, 0, 1, None, 1 << 30, None) == _lib.ERR_INVALID


def test_cpu_tensors_are_rejected_without_fallback():
    x = torch.zeros(1, 2, 64, 64, dtype=torch.bfloat16)
    idx = torch.zeros(1, 1, 1, 1, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        native.sparse_attention(x, x[:, :1], x[:, :1], idx)
    with pytest.raises(RuntimeError, match="CUDA"):
        native.pool_qk(x, x[:, :1])


def test_density_k_and_flops_match_the_survey_figures():
    assert k_for_density(512, 0.10) == 27 and causal_block_entries(512, 27) == 13473
    assert k_for_density(2048, 0.10) == 106 and causal_block_entries(2048, 106) == 211523
    assert k_for_density(1024, 0.10) == 53
    assert [k_for_density(2048, d) for d in (0.02, 0.05, 0.25, 0.50, 1.0)] == [21, 52, 275, 600, 2048]
    flops = sparse_attention_flops(LayerShape(1, 28, 4, 131072, 128), 211523)
    assert abs(flops - 12.3615e12) / 12.3615e12 < 1e-3
    assert abs(sparse_attention_flops(LayerShape(1, 28, 4, 32768, 128), 13473) - 0.776e12) < 1e9


def test_synthetic_inputs_are_seeded_and_strided_like_hf():
    shape = LayerShape(1, 4, 2, 130, 64)
    a = make_layer_inputs(shape, torch.bfloat16, seed=5)
    b = make_layer_inputs(shape, torch.bfloat16, seed=5)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
        assert x.shape[2] == 130 and not x.is_contiguous()       # [B, H, T, D] view of [B, T, H, D]
    wq, wk = make_gate_weights(1, 64, 64, seed=1)
    assert wq.abs().max() <= 1 / 64 and wk.shape == (1, 64, 64)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_covers_every_group_and_block_once(world):
    Hkv, qb = 4, 2048
    seen = torch.zeros(Hkv, qb, dtype=torch.int32)
    for r in range(world):
        s = plan(world, r, Hkv, qb)
        g0, g1 = s.groups
        i0, i1 = s.q_blocks
        seen[g0:g1, i0:i1] += 1
    assert torch.equal(seen, torch.ones_like(seen))


def test_shard_plan_rejects_uneven_splits():
    with pytest.raises(ValueError):
        plan(3, 0, 4, 2048)
    with pytest.raises(ValueError):
        plan(8, 0, 4, 2047)


def test_balanced_split_equalises_selected_tiles():
    from spruce_research_b200.sharding import balanced_cuts

    qb, K = 2048, 106
    cuts = balanced_cuts(qb, 2, K)
    work = [min(i + 1, K) for i in range(qb)]
    a, b = sum(work[:cuts[1]]), sum(work[cuts[1]:])
    assert cuts[0] == 0 and cuts[-1] == qb and abs(a - b) <= K
    assert sum(work[1024:]) / sum(work[:1024]) > 1.05        # the equal-rows split is 5% off
    for world in (8, 16):
        seen = torch.zeros(4, qb, dtype=torch.int32)
        for r in range(world):
            s = plan(world, r, 4, qb, k_selected=K)
            seen[s.groups[0]:s.groups[1], s.q_blocks[0]:s.q_blocks[1]] += 1
        assert torch.equal(seen, torch.ones_like(seen))


@pytest.mark.parametrize("r0,r1,chunks", [(0, 2048, 16), (1024, 2048, 16), (0, 3, 16), (5, 6, 4), (7, 300, 9)])
def test_chunk_bounds_cover_the_rows_in_order(r0, r1, chunks):
    from spruce_research_b200.pipeline import chunk_bounds
    for schedule in ("balanced", "equal"):
        b = chunk_bounds(r0, r1, chunks, schedule)
        assert b[0] == r0 and b[-1] == r1 and len(b) - 1 <= chunks
        assert all(x < y for x, y in zip(b, b[1:]))
    # balanced: every chunk carries about the same causal work (sum of its query blocks' key counts)
    b = chunk_bounds(0, 2048, 16)
    work = [(y * y - x * x) for x, y in zip(b, b[1:])]
    assert max(work) / min(work) < 1.02   # bounds are whole query blocks
    with pytest.raises(ValueError):
        from spruce_research_b200.pipeline import HostStreamedLayer
        HostStreamedLayer(None, "cpu", schedule="fifo")


def test_cpulist_parsing_and_affinity_restored():
    from spruce_research_b200 import hostmem
    assert hostmem.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert hostmem.parse_cpulist("") == set()
    before = os.sched_getaffinity(0)
    if torch.cuda.is_available():
        with hostmem.near("cuda:0") as cpus:
            assert not cpus or os.sched_getaffinity(0) == cpus
    assert os.sched_getaffinity(0) == before
