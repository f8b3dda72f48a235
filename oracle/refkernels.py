"""ctypes front end of oracle/_ref/libref_moe.so, the reference crate's own CUDA kernels built
from its sources by oracle/build_ref.sh.  TEST INFRASTRUCTURE ONLY (second oracle on the GPU,
generator of tests/golden/ fixtures).

Never call the reference's fused_moe or preprocessing with num_tokens*topk > 65536: that path
(preprocessing.cuh:266-312) scans its counts in place (moe_compute_offsets_kernel is launched
with expert_counts == expert_offsets, :296-298), so the scatter positions it computes are not
trustworthy and could address memory outside the output buffers.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libref_moe.so")
MAX_SAFE_ROWS = 65536
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB_PATH)
        P, I32, I64, U32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32
        L.topk_softmax.argtypes = [P, P, P, P, I32, I64, I32, P]
        L.topk_softmax.restype = None
        L.fused_moe.argtypes = [P, P, P, P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_int, ctypes.c_int, U32, U32, P]
        L.fused_moe.restype = None
        L.ref_preprocessing.argtypes = [P, P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.ref_preprocessing.restype = None
        L.ref_get_last_error.argtypes = []
        L.ref_get_last_error.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _s():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def topk_softmax(logits, k):
    """Reference router on a CUDA f32 tensor [T,E]; returns (w, idx, src) torch tensors."""
    import torch
    T, E = logits.shape
    w = torch.zeros(T, k, device=logits.device)
    idx = torch.zeros(T, k, dtype=torch.int32, device=logits.device)
    src = torch.zeros(T, k, dtype=torch.int32, device=logits.device)
    lib().topk_softmax(_p(logits), _p(w), _p(idx), _p(src), E, T, k, _s())
    return w, idx, src


def preprocessing(idx, w, E):
    """Reference sort/align (launch_preprocessing) for T*k <= 65536 rows."""
    import torch
    T, k = idx.shape
    if T * k > MAX_SAFE_ROWS:
        raise ValueError("the reference's multi-kernel preprocessing path is not run (see module doc)")
    off = torch.zeros(E + 2, dtype=torch.int32, device=idx.device)
    st = torch.zeros(T * k, dtype=torch.int32, device=idx.device)
    sw = torch.zeros(T * k, dtype=torch.float32, device=idx.device)
    lib().ref_preprocessing(_p(idx), _p(w), _p(off), _p(st), _p(sw), T, E, k, _s())
    return off, st, sw


def fused_moe(x, gate, up, down, w, idx, E, k, act, moe_type, dtype_code):
    """Reference fused_moe into a zeroed output; returns (out, cuda_error_code)."""
    import torch
    T, H = x.shape
    I = gate.shape[2]
    if T * k > MAX_SAFE_ROWS:
        raise ValueError("the reference's multi-kernel preprocessing path is not run (see module doc)")
    lib().ref_get_last_error()
    out = torch.zeros(T, H, dtype=x.dtype, device=x.device)
    lib().fused_moe(_p(x), _p(gate), _p(up), _p(down), _p(w), _p(idx), _p(out), T, H, I, E, k,
                    act, moe_type, dtype_code, _s())
    torch.cuda.synchronize()
    return out, lib().ref_get_last_error()
