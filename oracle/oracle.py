"""Python front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Wraps ``oracle/_build/liboracle.so`` (built from ``oracle/oracle.c`` by
``oracle/Makefile``) with numpy/torch-CPU helpers that restate the
reference's sparse-prefill path end to end:

  _group_avg_tokens      teacher/chunked_extract.py:75-80
  _proto_pool_seq (P=1)  teacher/chunked_extract.py:27-46
  FlatGate (P=1)         selector/gate.py:47-57, :101
  flat top-k + packing   scripts/route_overrides.py:187-205 +
                         scripts/export_selected_blocks.py:80-175
  selected_ids_to_blocks scripts/export_selected_blocks.py:80-175
  validate_selected_blocks interfaces/validator.py:7-62
  sparse attention       sparse/attention.py:143-274
  residual tree layout   interfaces/residual_summaries.py:73-122
  K/V summary table      sparse/summaries.py:29-142
  outlier prototypes     teacher/chunked_extract.py:47-72
  MaxSim gate scores     selector/gate.py:29-101, :132-171

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module; the product path never does.  Parity is pinned by the golden
vectors under tests/golden/ (made by running the reference itself).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

DT_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
PAD_VALUE = -1


def build() -> str:
    """Compile the oracle library with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        try:
            build()  # make is incremental: rebuilds only when oracle.c changed
        except (OSError, subprocess.CalledProcessError):
            if not os.path.exists(_LIB_PATH):
                raise
        L = ctypes.CDLL(_LIB_PATH)
        P, I64, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
        L.oracle_group_avg.argtypes = [P, ctypes.c_int, I64, I64, I64, I64, I64, P]
        L.oracle_block_mean.argtypes = [P, ctypes.c_int, I64, I64, I64, I64, I64, P]
        L.oracle_project.argtypes = [P, ctypes.c_int, I64, I64, P, I64, P]
        L.oracle_scores.argtypes = [P, I64, P, I64, I64, P]
        L.oracle_select_rows.argtypes = [P, I64, I64, I64, I64, I64, I64, P]
        L.oracle_select_rows.restype = ctypes.c_int
        L.oracle_pack_ids.argtypes = [P, I64, I64, I64, I64, I64, I64, I64, P]
        L.oracle_pack_ids.restype = ctypes.c_int
        L.oracle_sparse_attention.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, I64, I64, F, P]
        L.oracle_sparse_attention_rows.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, I64, I64, F, I64, I64, P]
        L.oracle_kv_summary_table.argtypes = [P, P, ctypes.c_int, P, I64, I64, I64, I64, I64, I64, P, P, I64,
                                              P, P, P, P, P, P]
        L.oracle_maxsim.argtypes = [P, P, P, I64, I64, I64, I64, I64, I64, P]
        L.oracle_residual_attention.argtypes = [P, P, P, P, P, I64, P, P, P, P, I64, I64, I64, I64, I64, I64,
                                                I64, I64, I64, F, P]
        L.oracle_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _raw(t: torch.Tensor) -> torch.Tensor:
    """Contiguous CPU tensor whose storage the C code reads as raw bits."""
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16)
    return t


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def group_avg_tokens(x: torch.Tensor, G: int) -> torch.Tensor:
    """[b, H, L, d] -> [b, G, L, d] in x's dtype."""
    b, H, T, d = x.shape
    src = _raw(x)
    out = torch.empty((b, G, T, d), dtype=x.dtype)
    lib().oracle_group_avg(_ptr(src), DT_CODE[x.dtype], b, H, T, d, G, _ptr(_raw_view(out)))
    return out


def _raw_view(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int16) if t.dtype in (torch.bfloat16, torch.float16) else t


def block_mean(x: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[b, H, L, d] -> [b, H, nb, d]: prototype 0 of _proto_pool_seq."""
    b, H, T, d = x.shape
    nb = (T + block - 1) // block
    src = _raw(x)
    out = torch.empty((b, H, nb, d), dtype=x.dtype)
    lib().oracle_block_mean(_ptr(src), DT_CODE[x.dtype], b, H, T, d, block, _ptr(_raw_view(out)))
    return out


def proto_pool_seq(x: torch.Tensor, block: int, P: int) -> torch.Tensor:
    """[b, H, L, d] -> [b, H, nb, P, d] (teacher/chunked_extract.py:27-72).

    Prototype 0 is the block mean (oracle_block_mean, bit-exact).  For P > 1
    the next P-1 are the block's real rows with the largest fp32 squared L2
    distance to that mean (:53-57), in descending order with ties to the lower
    row (torch.topk leaves tie order open); slots a ragged block cannot fill
    repeat the mean (:62-72).
    """
    mean = block_mean(x, block)                       # [b, H, nb, d] in x's dtype
    if P == 1:
        return mean[:, :, :, None, :]
    b, H, T, d = x.shape
    nb = mean.shape[2]
    xs = x.detach().cpu()
    out = mean[:, :, :, None, :].repeat(1, 1, 1, P, 1)
    m32 = mean.float().numpy()
    x32 = xs.float().numpy()
    for i in range(nb):
        r0, r1 = i * block, min((i + 1) * block, T)
        rows = x32[:, :, r0:r1, :]                    # [b, H, n, d]
        diff = (rows - m32[:, :, i, None, :]).astype(np.float32)
        dist = (diff * diff).sum(axis=-1, dtype=np.float32)     # [b, H, n]
        for bb in range(b):
            for h in range(H):
                order = np.lexsort((np.arange(r1 - r0), -dist[bb, h]))   # descending, lower row first
                for s, r in enumerate(order[:min(P - 1, block)]):
                    out[bb, h, i, s + 1] = xs[bb, h, r0 + int(r)]
    return out


def project(x: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    """x [..., d] (any float dtype) @ W [d, p] fp32 -> fp32 [..., p]."""
    d, p = W.shape
    src = _raw(x.reshape(-1, d))
    Wc = W.detach().float().cpu().contiguous()
    out = torch.empty((src.shape[0], p), dtype=torch.float32)
    lib().oracle_project(_ptr(src), DT_CODE[x.dtype], src.shape[0], d, _ptr(Wc), p, _ptr(out))
    return out.view(*x.shape[:-1], p)


def scores(qp: torch.Tensor, kp: torch.Tensor) -> torch.Tensor:
    """qp [nq, p], kp [nk, p] fp32 -> [nq, nk] = qp.kp / sqrt(p)."""
    qp = qp.float().contiguous()
    kp = kp.float().contiguous()
    out = torch.empty((qp.shape[0], kp.shape[0]), dtype=torch.float32)
    lib().oracle_scores(_ptr(qp), qp.shape[0], _ptr(kp), kp.shape[0], qp.shape[1], _ptr(out))
    return out


def select_rows(s: torch.Tensor, k_selected: int, local_window: int, sink_blocks: int) -> torch.Tensor:
    """s [R, qb, kb] fp32 -> int32 [R, qb, K] packed rows (flat top-k policy)."""
    R, qb, kb = s.shape
    s = s.float().contiguous()
    out = torch.empty((R, qb, k_selected), dtype=torch.int32)
    rc = lib().oracle_select_rows(_ptr(s), R, qb, kb, k_selected, local_window, sink_blocks, _ptr(out))
    if rc:
        raise ValueError(
            f"k_selected={k_selected} cannot fit local window size {local_window + 1} "
            f"plus {sink_blocks} sink block(s)")
    return out


def selected_ids_to_blocks(selected_ids: torch.Tensor, k_selected: int, local_window: int = 1,
                           key_blocks: int | None = None, sink_blocks: int = 0) -> torch.Tensor:
    """[L, G, qb, C] ids -> int32 [1, L, G, qb, K] (reference packing policy)."""
    L, G, qb, C = selected_ids.shape
    kb = qb if key_blocks is None else int(key_blocks)
    ids = selected_ids.detach().cpu().to(torch.int64).contiguous()
    out = torch.empty((L, G, qb, k_selected), dtype=torch.int32)
    rc = lib().oracle_pack_ids(_ptr(ids), L * G, qb, C, k_selected, local_window, kb, sink_blocks, _ptr(out))
    if rc:
        raise ValueError("invalid packing arguments")
    return out.unsqueeze(0)


def select_blocks(q: torch.Tensor, k: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor,
                  k_selected: int, local_window: int = 0, sink_blocks: int = 1,
                  block: int = 64) -> dict:
    """Full flat selector for one layer.

    q [B, Hq, T, d], k [B, Hkv, T, d] (any strides), wq/wk [d, p] fp32.
    Returns pooled_q/pooled_k [B, Hkv, qb, d] (input dtype), qp/kp fp32,
    scores [B, Hkv, qb, qb] fp32 and selected int32 [B, Hkv, qb, K].
    """
    B, Hq, T, d = q.shape
    Hkv = k.shape[1]
    qg = group_avg_tokens(q, Hkv)
    pooled_q = block_mean(qg, block)
    pooled_k = block_mean(k, block)
    qp = project(pooled_q, wq)
    kp = project(pooled_k, wk)
    qb = pooled_q.shape[2]
    s = torch.stack([scores(qp[b, g], kp[b, g]) for b in range(B) for g in range(Hkv)])
    sel = select_rows(s, k_selected, local_window, sink_blocks)
    return {
        "pooled_q": pooled_q, "pooled_k": pooled_k, "qp": qp, "kp": kp,
        "scores": s.view(B, Hkv, qb, qb), "selected": sel.view(B, Hkv, qb, k_selected),
    }


def sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                     scale: float | None = None, block: int = 64, out_dtype=None,
                     q_blocks: tuple[int, int] | None = None) -> torch.Tensor:
    """q [B, Hq, T, D], k/v [B, Hkv, T, D], indices int32 [B, Hkv, qb, K].

    Returns [B, T, Hq, D] in ``out_dtype`` (default: q's dtype), computed in
    fp32 with double-precision softmax sums.  ``q_blocks=(i0, i1)`` computes
    only those query blocks (other rows are zero).
    """
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = D ** -0.5
    qb = (T + block - 1) // block
    i0, i1 = (0, qb) if q_blocks is None else q_blocks
    qf = q.detach().float().cpu().contiguous()
    kf = k.detach().float().cpu().contiguous()
    vf = v.detach().float().cpu().contiguous()
    idx = indices.detach().cpu().to(torch.int32).contiguous()
    out = torch.zeros((B, T, Hq, D), dtype=torch.float32)
    lib().oracle_sparse_attention_rows(_ptr(qf), _ptr(kf), _ptr(vf), _ptr(idx), B, Hq, Hkv, T, D,
                                       idx.shape[-1], block, float(scale), i0, i1, _ptr(out))
    return out.to(out_dtype or q.dtype)


def sparse_attention_blocks(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                            blocks, scale: float | None = None, block: int = 64) -> torch.Tensor:
    """The rows of the listed query blocks only: [B, rows, Hq, D] fp32, rows in list order.

    Same arithmetic as sparse_attention; the inputs are converted to fp32 once.
    """
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = D ** -0.5
    qf = q.detach().float().cpu().contiguous()
    kf = k.detach().float().cpu().contiguous()
    vf = v.detach().float().cpu().contiguous()
    idx = indices.detach().cpu().to(torch.int32).contiguous()
    out = torch.zeros((B, T, Hq, D), dtype=torch.float32)
    for i in blocks:
        lib().oracle_sparse_attention_rows(_ptr(qf), _ptr(kf), _ptr(vf), _ptr(idx), B, Hq, Hkv, T, D,
                                           idx.shape[-1], block, float(scale), int(i), int(i) + 1, _ptr(out))
    rows = torch.cat([torch.arange(i * block, min((i + 1) * block, T)) for i in blocks])
    return out[:, rows]


def residual_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                              nodes: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, counts: torch.Tensor,
                              log_counts: torch.Tensor, scale: float | None = None, block: int = 64,
                              out_dtype=None) -> torch.Tensor:
    """Selected blocks plus residual summary keys in one softmax (sparse/attention.py:178-265).

    indices int32 [B, Hkv, qb, K], nodes int32 [B, Hkv, qb, S]; summary keys/values
    fp32 [B, Hkv, NN, P, D], counts/log_counts [B, NN, P].  Returns [B, T, Hq, D].
    """
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = D ** -0.5
    f = lambda x: x.detach().float().cpu().contiguous()  # noqa: E731
    qf, kf, vf = f(q), f(k), f(v)
    sk, sv, scnt, slc = f(keys), f(values), f(counts), f(log_counts)
    idx = indices.detach().cpu().to(torch.int32).contiguous()
    nd = nodes.detach().cpu().to(torch.int32).contiguous()
    out = torch.zeros((B, T, Hq, D), dtype=torch.float32)
    lib().oracle_residual_attention(_ptr(qf), _ptr(kf), _ptr(vf), _ptr(idx), _ptr(nd), nd.shape[-1], _ptr(sk),
                                    _ptr(sv), _ptr(scnt), _ptr(slc), sk.shape[2], sk.shape[3], B, Hq, Hkv, T, D,
                                    idx.shape[-1], block, float(scale), _ptr(out))
    return out.to(out_dtype or q.dtype)


def validate_selected_blocks(t: torch.Tensor, local_window: int = 1) -> None:
    """interfaces/validator.py:7-62 restated row by row; raises AssertionError.

    Rows are visited in (b, l, g, q) order and the rules in the reference's
    order (causal, sorted, duplicates, local window, trailing padding), so the
    first violation and its message match the reference's.
    """
    assert t.dim() == 5, (
        "Expected 5D tensor [batch, layer, kv_head_group, query_block, "
        f"K_selected_blocks], got {t.dim()}D with shape {tuple(t.shape)}")
    assert t.dtype == torch.int32, f"Expected int32, got {t.dtype}"
    assert local_window >= 0, f"local_window must be >= 0, got {local_window}"
    a = t.detach().cpu().numpy()
    B, L, G, Q, K = a.shape
    for b in range(B):
        for l in range(L):
            for g in range(G):
                for q in range(Q):
                    row = a[b, l, g, q].tolist()
                    real = [x for x in row if x != PAD_VALUE]
                    where = f"[b={b}, l={l}, g={g}, q={q}]"
                    for block_id in real:
                        assert block_id <= q, (
                            f"Causal violation at {where}: block {block_id} is in the future (q={q})")
                    assert real == sorted(real), f"Not sorted at {where}: {real}"
                    assert len(real) == len(set(real)), f"Duplicate block IDs at {where}: {real}"
                    missing = [x for x in range(max(0, q - local_window), q + 1) if x not in real]
                    assert not missing, (
                        f"Missing local-window block(s) at {where}: missing {missing}, row={real}")
                    if PAD_VALUE in row:
                        first = row.index(PAD_VALUE)
                        assert all(x == PAD_VALUE for x in row[first:]), (
                            f"Padding is not trailing-only at {where}: {row}")


def dense_causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Dense causal GQA attention in fp64 -> [B, T, Hq, D] fp32 (100%-density check)."""
    B, Hq, T, D = q.shape
    rep = Hq // k.shape[1]
    kk = k.double().repeat_interleave(rep, dim=1)
    vv = v.double().repeat_interleave(rep, dim=1)
    s = (q.double() @ kk.transpose(-1, -2)) / math.sqrt(D)
    mask = torch.ones(T, T, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    return (torch.softmax(s, dim=-1) @ vv).transpose(1, 2).float()


def residual_tree_ranges(num_leaves: int) -> tuple[list[int], list[int]]:
    """Leaf-first binary-tree node ranges in blocks (interfaces/residual_summaries.py:73-122).

    Level 0 holds the leaves [i, i+1); each higher level pairs neighbours
    (an odd tail is carried up alone) until one root remains.
    """
    if num_leaves < 1:
        raise ValueError(f"num_leaves must be >= 1, got {num_leaves}")
    level = [(i, i + 1) for i in range(num_leaves)]
    starts, ends = [], []
    while True:
        starts += [a for a, _ in level]
        ends += [b for _, b in level]
        if len(level) == 1:
            return starts, ends
        level = [(level[i][0], level[min(i + 1, len(level) - 1)][1]) for i in range(0, len(level), 2)]


def kv_summary_table(key: torch.Tensor, value: torch.Tensor, starts, ends, block_size: int, prototypes: int,
                     token_mask: torch.Tensor | None = None) -> dict:
    """build_kv_summary_table (sparse/summaries.py:52-142) on CPU.

    key/value [B, H, T, D]; starts/ends: node ranges in blocks.  Returns keys,
    values [B, H, nodes, P, D] fp32, counts/log_counts [B, nodes, P] fp32 and
    range_starts/range_ends [nodes, P] int64.
    """
    B, H, T, D = key.shape
    nodes, P = len(starts), int(prototypes)
    kr, vr = _raw(key), _raw(value)
    valid = None if token_mask is None else token_mask.detach().cpu().to(torch.uint8).contiguous()
    st = torch.tensor(list(starts), dtype=torch.int64)
    en = torch.tensor(list(ends), dtype=torch.int64)
    out = {
        "keys": torch.empty((B, H, nodes, P, D), dtype=torch.float32),
        "values": torch.empty((B, H, nodes, P, D), dtype=torch.float32),
        "counts": torch.empty((B, nodes, P), dtype=torch.float32),
        "log_counts": torch.empty((B, nodes, P), dtype=torch.float32),
        "range_starts": torch.empty((nodes, P), dtype=torch.int64),
        "range_ends": torch.empty((nodes, P), dtype=torch.int64),
    }
    lib().oracle_kv_summary_table(_ptr(kr), _ptr(vr), DT_CODE[key.dtype], None if valid is None else _ptr(valid),
                                  B, H, T, D, block_size, P, _ptr(st), _ptr(en), nodes,
                                  *(_ptr(out[n]) for n in ("keys", "values", "counts", "log_counts",
                                                           "range_starts", "range_ends")))
    return out


def maxsim(qp: torch.Tensor, kp: torch.Tensor, ids: torch.Tensor | None = None) -> torch.Tensor:
    """MaxSim scores of fp32 projections qp [R, nq, P, p], kp [R, nk, P, p]; every key
    column, or the candidate key ids [R, nq, C] (selector/gate.py:29-101, :132-171)."""
    R, nq, P, p = qp.shape
    nk = kp.shape[1]
    qc = qp.detach().cpu().float().contiguous()
    kc = kp.detach().cpu().float().contiguous()
    idc = None if ids is None else ids.detach().cpu().to(torch.int64).contiguous()
    ncols = nk if idc is None else idc.shape[2]
    out = torch.empty((R, nq, ncols), dtype=torch.float32)
    lib().oracle_maxsim(_ptr(qc), _ptr(kc), None if idc is None else _ptr(idc), R, nq, nk, ncols, P, p, _ptr(out))
    return out


def _round_to(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    """fp32 values after a round trip through dtype (round to nearest even)."""
    if dtype == torch.float32:
        return x.astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dtype).float().numpy()


def tree_merge(child: torch.Tensor, radix: int = 2) -> torch.Tensor:
    """One key-tree level up (selector/tree.py:80-112) in the features' dtype.

    Parent prototype 0 = round(round(sum of the valid children's prototype 0 in
    fp32) / round(count)); prototypes 1.. = the children's prototypes with the
    largest distance round(sum_d round(round(x - mean)^2)) (fp32 sum in d
    order), descending, ties to the lower candidate.
    """
    dt = child.dtype
    c = child.detach().cpu().float().numpy()                     # [R, n, P, d]
    R, n, P, d = c.shape
    npar = (n + radix - 1) // radix
    out = np.empty((R, npar, P, d), dtype=np.float32)
    for r in range(R):
        for pn in range(npar):
            kids = c[r, pn * radix:min((pn + 1) * radix, n)]        # [nv, P, d]
            nv = kids.shape[0]
            s = np.zeros(d, dtype=np.float32)
            for k in range(nv):
                s = (s + kids[k, 0]).astype(np.float32)
            mean = _round_to(_round_to(s, dt) / _round_to(np.float32(nv), dt), dt).astype(np.float32)
            out[r, pn, 0] = mean
            if P == 1:
                continue
            cands = kids.reshape(nv * P, d)
            dist = np.full(radix * P, -np.inf, dtype=np.float32)
            for ci in range(nv * P):
                diff = _round_to((cands[ci] - mean).astype(np.float32), dt)
                sq = _round_to((diff * diff).astype(np.float32), dt)
                acc = np.float32(0.0)
                for x in range(d):
                    acc = np.float32(acc + sq[x])
                dist[ci] = _round_to(np.array([acc], dtype=np.float32), dt)[0]
            order = np.lexsort((np.arange(radix * P), -dist))[:P - 1]
            out[r, pn, 1:] = cands[order]
    return torch.from_numpy(out).to(dt)


def traverse_to_leaf_ids(q_proj: torch.Tensor, level_proj: list, level_starts: list, beam: int,
                         radix: int = 2) -> torch.Tensor:
    """scripts/eval_tree_traversal.py:60-113 on projected features.

    q_proj [R, qb, P, p]; level_proj[l] [R, nodes_l, P, p] and level_starts[l]
    [nodes_l] leaf-first.  Candidates are the children of each row's current
    selection; valid when the parent is, the child exists and starts at or
    before the row's block; scores are MaxSim with invalid ones at the fp32
    minimum; the best min(beam, C, children) are kept (ties to the lower
    position), invalid ones as -1.  Returns int64 [R, qb, k].
    """
    R, qb = q_proj.shape[:2]
    sel = torch.zeros((R, qb, 1), dtype=torch.int64)
    for lvl in range(len(level_proj) - 2, -1, -1):
        kp, starts = level_proj[lvl], level_starts[lvl].cpu()
        nchild = kp.shape[1]
        cand = (sel[..., None] * radix + torch.arange(radix)).flatten(-2)
        valid = (sel[..., None] >= 0).expand(*sel.shape, radix).flatten(-2) & (cand < nchild)
        safe = cand.clamp(0, nchild - 1)
        valid &= starts[safe] <= torch.arange(qb)[None, :, None]
        scores = maxsim(q_proj, kp, safe)
        masked = torch.where(valid, scores, torch.full_like(scores, torch.finfo(torch.float32).min))
        k = min(beam, cand.shape[-1], nchild)
        C = cand.shape[-1]
        pos = torch.arange(C).expand_as(masked)
        order = torch.from_numpy(np.lexsort((pos.numpy().reshape(-1, C), -masked.numpy().reshape(-1, C))))
        top = order.view(R, qb, C)[..., :k]
        sel = torch.where(valid.gather(-1, top), safe.gather(-1, top), torch.full_like(top, -1))
    return sel
