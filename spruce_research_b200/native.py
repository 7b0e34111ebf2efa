"""Typed torch front end of the C ABI: one function per extern "C" entry point.

Each function takes CUDA tensors, checks dtypes/shapes the way the reference
does, allocates outputs on the input's device through torch's caching
allocator, and enqueues the kernel on the current stream.  The reference-named
drop-ins (FlatGate, _proto_pool_seq, direct_index_sparse_triton, ...) are thin
layers over these.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

BLOCK = 64


def _dt(t: torch.Tensor) -> int:
    try:
        return _lib.DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def _vec_ok(t: torch.Tensor) -> torch.Tensor:
    """A view the 16-byte vector kernels accept (copy only if it is not)."""
    es = t.element_size()
    vn = 16 // es
    if t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and all(s % vn == 0 for s in t.stride()[:-1]):
        return t
    return t.contiguous()


def group_avg_tokens(x: torch.Tensor, G: int) -> torch.Tensor:
    """[b, H, L, d] -> [b, G, L, d] (teacher/chunked_extract.py:75-80)."""
    _lib.require_cuda(x)
    b, H, T, d = x.shape
    if H % G:
        raise AssertionError(f"H={H} not divisible by G={G}")
    x = _vec_ok(x)
    out = torch.empty((b, G, T, d), device=x.device, dtype=x.dtype)
    L = _lib.load()
    _lib.check(L.spruce_group_avg_tokens(x.data_ptr(), _lib.strides(x), _dt(x), b, H, T, d, G, out.data_ptr(),
                                         _lib.stream_of(x)))
    return out


def proto_pool(x: torch.Tensor, block: int = BLOCK, P: int = 1) -> torch.Tensor:
    """[b, H, L, d] -> [b, H, nb, P, d] (teacher/chunked_extract.py:27-72)."""
    _lib.require_cuda(x)
    b, H, T, d = x.shape
    nb = (T + block - 1) // block
    x = _vec_ok(x)
    out = torch.empty((b, H, nb, P, d), device=x.device, dtype=x.dtype)
    L = _lib.load()
    _lib.check(L.spruce_proto_pool(x.data_ptr(), _lib.strides(x), _dt(x), b, H, T, d, block, P, out.data_ptr(),
                                   _lib.stream_of(x)))
    return out


def pool_qk(q: torch.Tensor, k: torch.Tensor, P: int = 1):
    """Selector inputs: (pooled_q, pooled_k), each [B, Hkv, qb, d] (P = 1) or
    [B, Hkv, qb, P, d] (P prototypes: the mean and the P-1 farthest rows)."""
    _lib.require_cuda(q, k)
    B, Hq, T, d = q.shape
    Hkv = k.shape[1]
    if q.dtype != k.dtype:
        raise ValueError("q and k must share a dtype")
    q, k = _vec_ok(q), _vec_ok(k)
    qb = (T + BLOCK - 1) // BLOCK
    shape = (B, Hkv, qb, d) if P == 1 else (B, Hkv, qb, P, d)
    pq = torch.empty(shape, device=q.device, dtype=q.dtype)
    pk = torch.empty(shape, device=q.device, dtype=q.dtype)
    L = _lib.load()
    if P == 1:
        _lib.check(L.spruce_pool_qk(q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), _dt(q), B, Hq, Hkv,
                                    T, d, pq.data_ptr(), pk.data_ptr(), _lib.stream_of(q)))
    else:
        _lib.check(L.spruce_pool_qk_protos(q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), _dt(q), B,
                                           Hq, Hkv, T, d, P, pq.data_ptr(), pk.data_ptr(), _lib.stream_of(q)))
    return pq, pk


def gate_project(x: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    """fp32(x[..., d]) @ W[d, p] with a fixed fma order -> fp32 [..., p]."""
    _lib.require_cuda(x, W)
    d, p = W.shape
    if x.shape[-1] != d:
        raise ValueError(f"feature dim {x.shape[-1]} does not match projection {tuple(W.shape)}")
    xc = x.contiguous()
    Wc = W.detach().float().contiguous()
    out = torch.empty((*x.shape[:-1], p), device=x.device, dtype=torch.float32)
    N = xc.numel() // d if d else 0
    L = _lib.load()
    _lib.check(L.spruce_gate_project(xc.data_ptr(), _dt(xc), N, d, Wc.data_ptr(), p, out.data_ptr(),
                                     _lib.stream_of(x)))
    return out


def gate_maxsim(qp: torch.Tensor, kp: torch.Tensor, ids: torch.Tensor | None = None) -> torch.Tensor:
    """MaxSim scores: qp [R, nq, P, p], kp [R, nk, P, p] fp32 -> [R, nq, nk] (every key)
    or, with int64 candidate ids [R, nq, C], [R, nq, C] (selector/gate.py:29-101, :132-171)."""
    _lib.require_cuda(qp, kp)
    if qp.dtype != torch.float32 or kp.dtype != torch.float32:
        raise ValueError("MaxSim takes fp32 projections")
    R, nq, P, p = qp.shape
    if kp.dim() != 4 or kp.shape[0] != R or kp.shape[2:] != (P, p):
        raise ValueError(f"kp must be [{R}, nk, {P}, {p}], got {tuple(kp.shape)}")
    nk = kp.shape[1]
    qp, kp = qp.contiguous(), kp.contiguous()
    if ids is not None:
        _lib.require_cuda(ids)
        if ids.dim() != 3 or tuple(ids.shape[:2]) != (R, nq):
            raise ValueError(f"ids must be [{R}, {nq}, C], got {tuple(ids.shape)}")
        ids = ids.to(torch.int64).contiguous()
    ncols = nk if ids is None else ids.shape[2]
    out = torch.empty((R, nq, ncols), device=qp.device, dtype=torch.float32)
    _lib.check(_lib.load().spruce_gate_maxsim(qp.data_ptr(), kp.data_ptr(), None if ids is None else ids.data_ptr(),
                                              R, nq, nk, ncols, P, p, out.data_ptr(), _lib.stream_of(qp)))
    return out


def gate_scores(qp: torch.Tensor, kp: torch.Tensor) -> torch.Tensor:
    """qp [R, qb, p], kp [R, kb, p] fp32 -> [R, qb, kb] = qp.kp / sqrt(p)."""
    _lib.require_cuda(qp, kp)
    R, qb, p = qp.shape
    kb = kp.shape[1]
    qp = qp.float().contiguous()
    kp = kp.float().contiguous()
    out = torch.empty((R, qb, kb), device=qp.device, dtype=torch.float32)
    L = _lib.load()
    _lib.check(L.spruce_gate_scores(qp.data_ptr(), kp.data_ptr(), R, qb, kb, p, out.data_ptr(), _lib.stream_of(qp)))
    return out


def gate_select(qp: torch.Tensor, kp: torch.Tensor, k_selected: int, local_window: int = 0, sink_blocks: int = 1,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """qp/kp [B, G, qb, p] fp32 -> selected rows int32 [B, G, qb, K] (or into `out`)."""
    _lib.require_cuda(qp, kp)
    B, G, qb, p = qp.shape
    qp = qp.float().contiguous()
    kp = kp.float().contiguous()
    if out is None:
        out = torch.empty((B, G, qb, k_selected), device=qp.device, dtype=torch.int32)
    _check_rows_out(out, B, G, qb, k_selected)
    L = _lib.load()
    _lib.check(L.spruce_gate_select(qp.data_ptr(), kp.data_ptr(), B, G, qb, p, k_selected, local_window, sink_blocks,
                                    out.data_ptr(), _lib.int64s(*out.stride()[:3]), _lib.stream_of(qp)))
    return out


def _check_rows_out(out: torch.Tensor, B: int, G: int, qb: int, K: int) -> None:
    if out.dtype != torch.int32 or tuple(out.shape) != (B, G, qb, K) or out.stride(-1) != 1:
        raise ValueError(f"selected rows must be int32 [{B}, {G}, {qb}, {K}] with a unit last stride")


def select_workspace_bytes(q: torch.Tensor, k: torch.Tensor, proj_dim: int) -> int:
    B, _, T, d = q.shape
    need = int(_lib.load().spruce_select_workspace_bytes(B, k.shape[1], T, d, proj_dim, _dt(q)))
    if need < 0:
        raise ValueError(f"bad selector shape: q {tuple(q.shape)}, k {tuple(k.shape)}, proj_dim {proj_dim}")
    return need


def select_blocks(q: torch.Tensor, k: torch.Tensor, Wq: torch.Tensor, Wk: torch.Tensor, k_selected: int,
                  local_window: int = 0, sink_blocks: int = 1, out: torch.Tensor | None = None,
                  workspace: torch.Tensor | None = None, q_blocks: tuple[int, int] | None = None) -> torch.Tensor:
    """Whole flat selector of one layer: int32 rows [B, Hkv, qb, K] (or into `out`).

    With ``q_blocks=(i0, i1)`` only rows i0..i1-1 are selected (and only the
    blocks they read are pooled and projected).
    """
    _lib.require_cuda(q, k, Wq, Wk)
    B, Hq, T, d = q.shape
    Hkv = k.shape[1]
    p = Wq.shape[1]
    if q.dtype != k.dtype:
        raise ValueError("q and k must share a dtype")
    if tuple(Wq.shape) != (d, p) or tuple(Wk.shape) != (d, p):
        raise ValueError(f"gate weights must be [{d}, p]")
    q, k = _vec_ok(q), _vec_ok(k)
    Wq = Wq.detach().float().contiguous()
    Wk = Wk.detach().float().contiguous()
    qb = (T + BLOCK - 1) // BLOCK
    if out is None:
        out = torch.empty((B, Hkv, qb, k_selected), device=q.device, dtype=torch.int32)
    _check_rows_out(out, B, Hkv, qb, k_selected)
    need = select_workspace_bytes(q, k, p)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 16), device=q.device, dtype=torch.uint8)
    i0, i1 = (0, qb) if q_blocks is None else q_blocks
    L = _lib.load()
    _lib.check(L.spruce_select_blocks_rows(q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), _dt(q), B,
                                           Hq, Hkv, T, d, Wq.data_ptr(), Wk.data_ptr(), p, k_selected, local_window,
                                           sink_blocks, out.data_ptr(), _lib.int64s(*out.stride()[:3]), i0, i1,
                                           workspace.data_ptr(), workspace.numel() * workspace.element_size(),
                                           _lib.stream_of(q)))
    return out


def pack_selected_ids(ids: torch.Tensor, k_selected: int, local_window: int, key_blocks: int,
                      sink_blocks: int) -> torch.Tensor:
    """ids [R, qb, C] (any int dtype) -> int32 [R, qb, K] with the reference packing policy."""
    _lib.require_cuda(ids)
    R, qb, C = ids.shape
    ids64 = ids.to(torch.int64).contiguous()
    out = torch.empty((R, qb, k_selected), device=ids.device, dtype=torch.int32)
    L = _lib.load()
    _lib.check(L.spruce_pack_selected_ids(ids64.data_ptr(), R, qb, C, k_selected, local_window, key_blocks,
                                          sink_blocks, out.data_ptr(), _lib.stream_of(ids)))
    return out


def validate_first_violation(sel: torch.Tensor, local_window: int) -> tuple[int, int] | None:
    """(flat row, rule) of the first violating row of int32 [B, L, G, qb, K], or None."""
    _lib.require_cuda(sel)
    B, Ln, G, qb, K = sel.shape
    s = sel.contiguous()
    res = torch.empty(1, device=sel.device, dtype=torch.int64)
    L = _lib.load()
    _lib.check(L.spruce_validate_selected_blocks(s.data_ptr(), B, Ln, G, qb, K, local_window, res.data_ptr(),
                                                 _lib.stream_of(sel)))
    v = int(res.item())
    if v < 0:
        return None
    return v // 8, v % 8


def sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                     scale: float | None = None, out: torch.Tensor | None = None,
                     status: torch.Tensor | None = None, q_blocks: tuple[int, int] | None = None,
                     peer_outs: list[int] | None = None) -> torch.Tensor:
    """Block-sparse causal GQA attention -> token-major [B, T, Hq, D].

    q [B, Hq, T, D], k/v [B, Hkv, T, D] (strided views are fine),
    indices int32 [B, Hkv, ceil(T/64), K].  With ``q_blocks=(i0, i1)`` only
    query blocks i0..i1-1 are computed (their rows of ``out``).  With
    ``peer_outs`` (device pointers of other GPUs' identically laid out output
    tensors, mapped into this process) every row is also stored there: the
    output all-gather fused into the kernel.
    """
    _lib.require_cuda(q, k, v, indices)
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = D ** -0.5
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k and v must share a dtype")
    if indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [B,Hkv,ceil(T/64),K]")
    qb = (T + BLOCK - 1) // BLOCK
    if tuple(indices.shape[:3]) != (B, Hkv, qb):
        raise ValueError("indices must be int32 [B,Hkv,ceil(T/64),K]")
    if out is None:
        out = torch.empty((B, T, Hq, D), device=q.device, dtype=q.dtype)
    ostr = _lib.int64s(out.stride(0), out.stride(2), out.stride(1), out.stride(3))
    i0, i1 = (0, qb) if q_blocks is None else q_blocks
    L = _lib.load()
    if peer_outs:
        peers = (ctypes.c_void_p * len(peer_outs))(*peer_outs)
        _lib.check(L.spruce_sparse_attention_fwd_scatter(
            q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(), _lib.strides(v),
            indices.data_ptr(), _lib.strides(indices), out.data_ptr(), ostr, _dt(q), B, Hq, Hkv, T, D,
            indices.shape[-1], float(scale), i0, i1, peers, len(peer_outs),
            status.data_ptr() if status is not None else None, _lib.stream_of(q)))
        return out
    _lib.check(L.spruce_sparse_attention_fwd_rows(
        q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(), _lib.strides(v),
        indices.data_ptr(), _lib.strides(indices), out.data_ptr(), ostr, _dt(q), B, Hq, Hkv, T, D,
        indices.shape[-1], float(scale), i0, i1, status.data_ptr() if status is not None else None,
        _lib.stream_of(q)))
    return out


def residual_frontier(selected: torch.Tensor, starts: torch.Tensor, ends: torch.Tensor,
                      parents: torch.Tensor) -> torch.Tensor:
    """Maximal residual frontiers of selected_blocks rows [..., qb, K] -> int32 [..., qb, S], ID-sorted,
    -1 padded, S the largest frontier (interfaces/residual_summaries.py:122-220).  starts / ends int64
    and parents int32 [num_nodes] are the tree layout on the same device."""
    _lib.require_cuda(selected, starts, ends, parents)
    if selected.dtype != torch.int32 or selected.dim() < 2:
        raise ValueError("selected_blocks must be int32 [..., qb, K]")
    qb, K = selected.shape[-2:]
    sel = selected.contiguous()
    rows = math.prod(sel.shape[:-1])
    L = _lib.load()
    NN = starts.numel()
    stream = _lib.stream_of(sel)
    mx = torch.zeros(1, device=sel.device, dtype=torch.int32)
    _lib.check(L.spruce_residual_frontier(sel.data_ptr(), rows, K, qb, starts.data_ptr(), ends.data_ptr(),
                                          parents.data_ptr(), NN, None, 0, None, mx.data_ptr(), stream))
    S = int(mx.item())
    out = torch.empty((*sel.shape[:-1], S), device=sel.device, dtype=torch.int32)
    if S:
        _lib.check(L.spruce_residual_frontier(sel.data_ptr(), rows, K, qb, starts.data_ptr(), ends.data_ptr(),
                                              parents.data_ptr(), NN, out.data_ptr(), S, None, None, stream))
    return out


def residual_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                              nodes: torch.Tensor, table, scale: float | None = None,
                              out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Block-sparse attention whose softmax also covers each row's residual summary keys
    (sparse/attention.py:164-265) -> token-major [B, T, Hq, D].

    ``nodes`` int32 [B, Hkv, qb, S] residual node ids (-1 padded); ``table`` a
    KVSummaryTable of the same K/V (keys/values fp32 [B, Hkv, nodes, P, D],
    counts/log_counts fp32 [B, nodes, P]).
    """
    _lib.require_cuda(q, k, v, indices, nodes)
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = D ** -0.5
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k and v must share a dtype")
    qb = (T + BLOCK - 1) // BLOCK
    if indices.dtype != torch.int32 or tuple(indices.shape[:3]) != (B, Hkv, qb):
        raise ValueError("indices must be int32 [B,Hkv,ceil(T/64),K]")
    if nodes.dtype != torch.int32 or nodes.dim() != 4 or tuple(nodes.shape[:3]) != (B, Hkv, qb):
        raise ValueError(f"residual nodes must be int32 [{B},{Hkv},{qb},S], got {tuple(nodes.shape)}")
    keys, values = table.keys.float().contiguous(), table.values.float().contiguous()
    counts, log_counts = table.counts.float().contiguous(), table.log_counts.float().contiguous()
    NN, P = keys.shape[2], keys.shape[3]
    if keys.shape != (B, Hkv, NN, P, D) or values.shape != keys.shape or counts.shape != (B, NN, P) \
            or log_counts.shape != counts.shape:
        raise ValueError("summary table shapes do not match q/k/v")
    _lib.require_cuda(keys, values, counts, log_counts)
    S = nodes.shape[3]
    if out is None:
        out = torch.empty((B, T, Hq, D), device=q.device, dtype=q.dtype)
    ostr = _lib.int64s(out.stride(0), out.stride(2), out.stride(1), out.stride(3))
    L = _lib.load()
    need = L.spruce_residual_workspace_bytes(B, Hkv, T, D, S, P, _dt(q))
    if need < 0:
        raise ValueError("bad residual attention shape")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 16), device=q.device, dtype=torch.uint8)
    _lib.check(L.spruce_residual_sparse_attention_fwd(
        q.data_ptr(), _lib.strides(q), k.data_ptr(), _lib.strides(k), v.data_ptr(), _lib.strides(v),
        indices.data_ptr(), _lib.strides(indices), nodes.data_ptr(), _lib.strides(nodes), S, keys.data_ptr(),
        values.data_ptr(), counts.data_ptr(), log_counts.data_ptr(), NN, P, out.data_ptr(), ostr, _dt(q), B, Hq,
        Hkv, T, D, indices.shape[-1], float(scale), workspace.data_ptr(), workspace.numel(),
        status.data_ptr() if status is not None else None, _lib.stream_of(q)))
    return out


def gate_denominator(proj_dim: int) -> float:
    return float(math.sqrt(proj_dim))


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of t's allocation, byte offset of t in it)."""
    _lib.require_cuda(t)
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_int64(0)
    _lib.check(_lib.load().spruce_ipc_export(t.data_ptr(), h, ctypes.byref(off)))
    return h.raw, off.value


def ipc_import(handle: bytes, offset: int) -> tuple[int, int]:
    """Map a peer allocation into the current device's context: (pointer, mapping base)."""
    ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
    buf = ctypes.create_string_buffer(handle, 64)
    _lib.check(_lib.load().spruce_ipc_import(buf, offset, ctypes.byref(ptr), ctypes.byref(base)))
    return ptr.value, base.value


def ipc_close(base: int) -> None:
    _lib.check(_lib.load().spruce_ipc_close(base))


def kv_summary_table(key: torch.Tensor, value: torch.Tensor, node_starts: torch.Tensor, node_ends: torch.Tensor,
                     block_size: int, prototypes: int, valid: torch.Tensor | None = None) -> dict:
    """Per-node prototype means of K and V (sparse/summaries.py:52-142).

    key/value [B, Hkv, T, D] CUDA tensors of one dtype; node_starts/node_ends
    int64 block ranges on the same device; valid bool/uint8 [B, T] or None.
    Returns the fp32 keys/values [B, Hkv, nodes, P, D], counts/log_counts
    [B, nodes, P] and int64 range_starts/range_ends [nodes, P].
    """
    _lib.require_cuda(key, value, node_starts, node_ends)
    if key.dtype != value.dtype:
        raise ValueError(f"key/value dtype mismatch: {key.dtype} vs {value.dtype}")
    B, H, T, D = key.shape
    nodes, P = node_starts.numel(), int(prototypes)
    dev = key.device
    key = key if key.stride(-1) == 1 else key.contiguous()
    value = value if value.stride(-1) == 1 else value.contiguous()
    st = node_starts.to(device=dev, dtype=torch.int64).contiguous()
    en = node_ends.to(device=dev, dtype=torch.int64).contiguous()
    vmask = None if valid is None else valid.to(device=dev, dtype=torch.uint8).contiguous()
    L = _lib.load()
    ws_bytes = int(L.spruce_kv_summary_workspace_bytes(B, H, T, D))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    out = {
        "keys": torch.empty((B, H, nodes, P, D), dtype=torch.float32, device=dev),
        "values": torch.empty((B, H, nodes, P, D), dtype=torch.float32, device=dev),
        "counts": torch.empty((B, nodes, P), dtype=torch.float32, device=dev),
        "log_counts": torch.empty((B, nodes, P), dtype=torch.float32, device=dev),
        "range_starts": torch.empty((nodes, P), dtype=torch.int64, device=dev),
        "range_ends": torch.empty((nodes, P), dtype=torch.int64, device=dev),
    }
    _lib.check(L.spruce_kv_summary_table(
        key.data_ptr(), _lib.strides(key), value.data_ptr(), _lib.strides(value),
        None if vmask is None else vmask.data_ptr(), _dt(key), B, H, T, D, block_size, P,
        st.data_ptr(), en.data_ptr(), nodes, out["keys"].data_ptr(), out["values"].data_ptr(),
        out["counts"].data_ptr(), out["log_counts"].data_ptr(), out["range_starts"].data_ptr(),
        out["range_ends"].data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_of(key)))
    return out


def tree_merge(child: torch.Tensor, radix: int = 2) -> torch.Tensor:
    """One key-tree level up (selector/tree.py:80-112): child [R, n, P, d] -> parent [R, ceil(n / radix), P, d]."""
    _lib.require_cuda(child)
    R, n, P, d = child.shape
    child = child.contiguous()
    out = torch.empty((R, (n + radix - 1) // radix, P, d), device=child.device, dtype=child.dtype)
    _lib.check(_lib.load().spruce_tree_merge(child.data_ptr(), _dt(child), R, n, P, d, radix, out.data_ptr(),
                                             _lib.stream_of(child)))
    return out


def tree_candidates(selected: torch.Tensor, radix: int, child_count: int, child_starts: torch.Tensor):
    """Children of each row's selection: (cand int64 [R, nq, S*radix], valid bool) (eval_tree_traversal.py:83-95)."""
    _lib.require_cuda(selected, child_starts)
    R, nq, S = selected.shape
    selected = selected.to(torch.int64).contiguous()
    starts = child_starts.to(device=selected.device, dtype=torch.int64).contiguous()
    cand = torch.empty((R, nq, S * radix), device=selected.device, dtype=torch.int64)
    valid = torch.empty((R, nq, S * radix), device=selected.device, dtype=torch.uint8)
    _lib.check(_lib.load().spruce_tree_candidates(selected.data_ptr(), R, nq, S, radix, child_count,
                                                  starts.data_ptr(), cand.data_ptr(), valid.data_ptr(),
                                                  _lib.stream_of(selected)))
    return cand, valid


def tree_topk(scores: torch.Tensor, valid: torch.Tensor, cand: torch.Tensor, k: int) -> torch.Tensor:
    """The level's beam: int64 [R, nq, k] candidate ids, -1 where invalid (eval_tree_traversal.py:104-108)."""
    _lib.require_cuda(scores, valid, cand)
    R, nq, C = scores.shape
    out = torch.empty((R, nq, k), device=scores.device, dtype=torch.int64)
    _lib.check(_lib.load().spruce_tree_topk(scores.contiguous().data_ptr(), valid.contiguous().data_ptr(),
                                            cand.contiguous().data_ptr(), R * nq, C, k, out.data_ptr(),
                                            _lib.stream_of(scores)))
    return out
