"""spruce_select_blocks_noalloc: the selector entry point that allocates nothing.

Some callers cannot hand this library device memory: a serving process that
reserves nearly all HBM for its own pool at start-up, or a plugin binding that
passes only the input and output buffers it owns.  For them the selector takes
its scratch from one static device array instead of a caller workspace.  These
tests call it through the C ABI and check it against spruce_select_blocks
(which takes a workspace) on two calls in a row, so a stale scratch array from
the first call cannot leak into the second.  The file is named to be
collected last.
"""
import ctypes

import pytest
import torch

from spruce_research_b200 import _lib, native
from spruce_research_b200.synthetic import LayerShape, k_for_density, make_gate_weights, make_layer_inputs

pytestmark = pytest.mark.gpu


def _noalloc(q, k, wq, wk, K, local_window, sink, out=None):
    """One call of the C entry point; `out` (int32 [B, Hkv, qb, K]) and fp32 contiguous
    weights are the caller's buffers, so with them given this makes no allocation at all."""
    L = _lib.load()
    B, Hq, T, d = q.shape
    Hkv = k.shape[1]
    qb = (T + 63) // 64
    if out is None:
        out = torch.full((B, Hkv, qb, K), -7, device=q.device, dtype=torch.int32)
    wq = wq.float().contiguous()
    wk = wk.float().contiguous()
    rc = L.spruce_select_blocks_noalloc(
        q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), _lib.DTYPE_CODE[q.dtype], B, Hq, Hkv, T, d,
        wq.data_ptr(), wk.data_ptr(), wq.shape[1], K, local_window, sink, out.data_ptr(),
        _lib.int64s(*out.stride()[:3]), _lib.stream_of(q))
    _lib.check(rc)
    return out


def _case(T, seed, dtype=torch.bfloat16):
    shape = LayerShape(1, 28, 4, T, 128)
    q, k, _ = make_layer_inputs(shape, dtype, seed, device="cuda")
    wq, wk = make_gate_weights(1, 128, 128, seed + 1, device="cuda")
    return q, k, wq[0], wk[0], k_for_density(shape.query_blocks, 0.10)


def test_noalloc_matches_workspace_entry_point_twice():
    assert _lib.load().spruce_select_noalloc_max_scratch_bytes() == 16 << 20
    for T, seed in ((8192, 11), (6000, 12)):        # two calls in a row, different shapes and inputs
        q, k, wq, wk, K = _case(T, seed)
        got = _noalloc(q, k, wq, wk, K, 0, 1)
        want = native.select_blocks(q, k, wq, wk, K, local_window=0, sink_blocks=1)
        torch.cuda.synchronize()
        assert torch.equal(got.cpu(), want.cpu()), f"noalloc selection differs at T={T}"


def test_noalloc_rejects_shapes_beyond_its_static_scratch():
    L = _lib.load()
    dummy = torch.zeros(16, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(16, device="cuda", dtype=torch.int32)
    s4 = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    # 8 KV groups x 8192 query blocks of d=128 needs ~100 MB of scratch.
    rc = L.spruce_select_blocks_noalloc(dummy.data_ptr(), s4, dummy.data_ptr(), s4, 1, 1, 56, 8, 8192 * 64, 128,
                                        dummy.data_ptr(), dummy.data_ptr(), 128, 16, 0, 1, out.data_ptr(),
                                        _lib.int64s(1, 1, 1), _lib.stream_of(dummy))
    assert rc == _lib.ERR_UNSUPPORTED
    assert "static buffer" in L.spruce_last_error().decode()


def test_noalloc_allocates_nothing_and_serves_config2():
    """At BASELINE config 2's shape (131072 tokens, 12 MiB of scratch, the largest case the
    16 MiB array is documented to hold): same rows as the workspace entry point, and a call
    after the first changes neither the device's free memory nor torch's allocation count."""
    q, k, wq, wk, K = _case(131072, 13)
    want = native.select_blocks(q, k, wq, wk, K, local_window=0, sink_blocks=1)
    B, _, T, _ = q.shape
    out = torch.full((B, k.shape[1], (T + 63) // 64, K), -7, device="cuda", dtype=torch.int32)
    wq32, wk32 = wq.float().contiguous(), wk.float().contiguous()
    _noalloc(q, k, wq32, wk32, K, 0, 1, out=out)  # first call on this device: symbol address lookup
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), want.cpu()), "noalloc selection differs at config 2"
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    out.fill_(-7)
    _noalloc(q, k, wq32, wk32, K, 0, 1, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == alloc0, "torch allocated during the call"
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes during the call"
    assert torch.equal(out.cpu(), want.cpu()), "second noalloc call differs at config 2"
