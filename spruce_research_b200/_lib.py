"""ctypes binding of libspruce_b200.so (the C ABI in include/spruce_b200.h).

The library is built in-tree by ``spruce_research_b200.build``.  Loading it
needs no GPU (the CUDA runtime is linked statically); every compute entry
point requires CUDA tensors and there is no CPU fallback: a missing library
raises RuntimeError.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import build as _build

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_WORKSPACE = 4

STATUS_TIMEOUT = 1
STATUS_EMPTY_ROW = 2

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

# Every extern "C" symbol of include/spruce_b200.h with its ctypes signature.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "spruce_last_error": ([], ctypes.c_char_p),
    "spruce_abi_version": ([], _INT),
    "spruce_group_avg_tokens": ([_P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_proto_pool": ([_P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_pool_qk": ([_P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P, _P, _P], _INT),
    "spruce_pool_qk_protos": ([_P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P], _INT),
    "spruce_gate_project": ([_P, _INT, _I64, _I64, _P, _I64, _P, _P], _INT),
    "spruce_gate_maxsim": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_tree_merge": ([_P, _INT, _I64, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_tree_candidates": ([_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P], _INT),
    "spruce_tree_topk": ([_P, _P, _P, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_gate_scores": ([_P, _P, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_gate_select": ([_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P], _INT),
    "spruce_gate_select_rows": ([_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _P], _INT),
    "spruce_select_blocks_rows": ([_P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64,
                                   _I64, _P, _P, _I64, _I64, _P, _I64, _P], _INT),
    "spruce_select_workspace_bytes": ([_I64, _I64, _I64, _I64, _I64, _INT], _I64),
    "spruce_select_blocks": ([_P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64,
                              _I64, _P, _P, _P, _I64, _P], _INT),
    "spruce_select_blocks_noalloc": ([_P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64,
                                      _I64, _I64, _P, _P, _P], _INT),
    "spruce_select_noalloc_max_scratch_bytes": ([], _I64),
    "spruce_kv_summary_workspace_bytes": ([_I64, _I64, _I64, _I64], _I64),
    "spruce_kv_summary_table": ([_P, _P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64,
                                 _P, _P, _P, _P, _P, _P, _P, _I64, _P], _INT),
    "spruce_residual_frontier": ([_P, _I64, _I64, _I64, _P, _P, _P, _I64, _P, _I64, _P, _P, _P], _INT),
    "spruce_residual_workspace_bytes": ([_I64, _I64, _I64, _I64, _I64, _I64, _INT], _I64),
    "spruce_residual_sparse_attention_fwd": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _I64,
                                              _I64, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _I64, _F, _P, _I64,
                                              _P, _P], _INT),
    "spruce_ipc_export": ([_P, _P, ctypes.POINTER(ctypes.c_int64)], _INT),
    "spruce_ipc_import": ([_P, _I64, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)], _INT),
    "spruce_ipc_close": ([_P], _INT),
    "spruce_exp2_selfcheck": ([_P, _I64, _P, _P, _P], _INT),
    "spruce_pack_selected_ids": ([_P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_validate_selected_blocks": ([_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "spruce_sparse_attention_fwd": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64,
                                     _I64, _F, _P, _P], _INT),
    "spruce_sparse_attention_fwd_rows": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _INT, _I64, _I64, _I64, _I64,
                                          _I64, _I64, _F, _I64, _I64, _P, _P], _INT),
    "spruce_sparse_attention_fwd_scatter": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _INT, _I64, _I64, _I64,
                                             _I64, _I64, _I64, _F, _I64, _I64, _P, ctypes.c_int32, _P, _P], _INT),
}

_lib = None


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True):
    """Load (building first if needed and possible) and return the library."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.LIB
    if build_if_missing:
        try:
            path = _build.build()
        except RuntimeError:
            if not os.path.exists(path):
                raise
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python -m spruce_research_b200.build` "
            "(there is no CPU fallback for the SPRUCE kernels)")
    lib = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(rc: int) -> None:
    """Map a C-ABI return code to the reference's exception types."""
    if rc == OK:
        return
    msg = load().spruce_last_error().decode()
    if rc in (ERR_INVALID, ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def strides(t: torch.Tensor, n: int = 4):
    return (ctypes.c_int64 * n)(*t.stride()[:n])


def int64s(*vals):
    return (ctypes.c_int64 * len(vals))(*vals)


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor, what: str = "the SPRUCE B200 kernels") -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(f"{what} require CUDA tensors (there is no CPU fallback)")
