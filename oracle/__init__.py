"""CPU oracle for the candle-moe hot path -- TEST INFRASTRUCTURE ONLY.

numpy front end over ``oracle/liboracle.so`` (built from ``oracle/oracle.c`` by
``oracle/Makefile``).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import this package, and only as the checker or the timed CPU baseline; the
product library (``candle-moe_b200``) never imports it.

Which reference code each function restates is listed in the header of ``oracle/oracle.c``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

DT_F16, DT_BF16, DT_F32 = 0, 1, 2
DTYPE_CODES = {"f16": DT_F16, "bf16": DT_BF16, "f32": DT_F32}


def build() -> str:
    """Compile oracle/oracle.c (make is incremental)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I, U64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_float, ctypes.c_size_t
        L.oracle_randn.argtypes = [U64, SZ, F, F, I, P, I]
        L.oracle_randn.restype = None
        L.oracle_topk_softmax.argtypes = [P, I, I, I, I, P, P, P, P]
        L.oracle_topk_softmax.restype = None
        L.oracle_route_prep.argtypes = [P, P, I, I, I, P, P, P, P]
        L.oracle_route_prep.restype = None
        L.oracle_moe_forward.argtypes = [P, P, P, P, P, P, I, I, I, I, I, I, I, I, I, I, P]
        L.oracle_moe_forward.restype = I
        L.oracle_moe_forward_ex.argtypes = [P, P, P, P, P, P, I, I, I, I, I, I, I, I, I, I, P, P]
        L.oracle_moe_forward_ex.restype = I
        L.oracle_activation.argtypes = [F, I]
        L.oracle_activation.restype = F
        L.oracle_num_threads.argtypes = []
        L.oracle_num_threads.restype = I
        L.oracle_set_num_threads.argtypes = [I]
        L.oracle_set_num_threads.restype = I
        L.oracle_convert_to_f32.argtypes = [P, I, SZ, P]
        L.oracle_convert_to_f32.restype = None
        L.oracle_convert_from_f32.argtypes = [P, I, SZ, P]
        L.oracle_convert_from_f32.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> int:
    """Use n OpenMP threads from now on (n <= 0: unchanged); returns the resulting count."""
    return lib().oracle_set_num_threads(n)


# ---------------------------------------------------------------------------------------------
# synthetic inputs
# ---------------------------------------------------------------------------------------------

def randn(seed: int, shape, mean: float = 0.0, std: float = 1.0, dtype: str = "f32",
          nthreads: int = 0) -> np.ndarray:
    """Seeded N(mean, std) values (SplitMix64 + Box-Muller), returned as raw storage:
    float32 for "f32", uint16 bit patterns for "bf16"/"f16"."""
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32 if dtype == "f32" else np.uint16)
    lib().oracle_randn(seed, n, mean, std, DTYPE_CODES[dtype], _ptr(out), nthreads)
    return out.reshape(shape)


def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """Raw storage (uint16 bf16/f16 bits or float32) -> float32 copy."""
    a = np.ascontiguousarray(a)
    out = np.empty(a.shape, dtype=np.float32)
    lib().oracle_convert_to_f32(_ptr(a), DTYPE_CODES[dtype], a.size, _ptr(out))
    return out


def from_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> raw storage of `dtype`, round-to-nearest-even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.float32 if dtype == "f32" else np.uint16)
    lib().oracle_convert_from_f32(_ptr(a), DTYPE_CODES[dtype], a.size, _ptr(out))
    return out


# ---------------------------------------------------------------------------------------------
# router
# ---------------------------------------------------------------------------------------------

def topk_softmax(logits: np.ndarray, k: int, renormalize: bool = False):
    """Restates kernels/topk_softmax.cu:136-266.

    Returns (weights [T,k] f32, indices [T,k] i32, token_expert_indices [T,k] i32, near_tie [T]
    bool).  near_tie marks rows whose selection was decided between values within 8 ulps."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    w = np.empty((T, k), np.float32)
    idx = np.empty((T, k), np.int32)
    src = np.empty((T, k), np.int32)
    tie = np.empty((T,), np.uint8)
    if T:
        lib().oracle_topk_softmax(_ptr(logits), T, E, k, int(renormalize), _ptr(w), _ptr(idx),
                                  _ptr(src), _ptr(tie))
    return w, idx, src, tie.astype(bool)


# ---------------------------------------------------------------------------------------------
# route preparation
# ---------------------------------------------------------------------------------------------

def route_prep(indices: np.ndarray, weights: np.ndarray, num_experts: int):
    """Restates kernels/preprocessing.cuh:5-59 with the within-expert order pinned to ascending
    flat index.  Returns (offsets [E+2], sorted_token [rows], sorted_weight [rows],
    sorted_flat [rows])."""
    indices = np.ascontiguousarray(indices).view(np.uint32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    T, k = indices.shape
    E = num_experts
    offsets = np.zeros(E + 2, np.int32)
    valid = int(np.count_nonzero(indices < E))
    st = np.empty(max(valid, 1), np.int32)
    sw = np.empty(max(valid, 1), np.float32)
    sf = np.empty(max(valid, 1), np.int32)
    lib().oracle_route_prep(_ptr(indices), _ptr(weights), T, k, E, _ptr(offsets), _ptr(st),
                            _ptr(sw), _ptr(sf))
    return offsets, st[:valid], sw[:valid], sf[:valid]


# ---------------------------------------------------------------------------------------------
# fused MoE forward
# ---------------------------------------------------------------------------------------------

def moe_forward(x, gate, up, down, routing_weights, indices, *, activation: int, moe_type: int,
                dtype: str, round_dtype: str | None = None, nthreads: int = 0,
                with_max_contrib: bool = False):
    """Restates the reference's fused MoE forward (see oracle/oracle.c).

    x/gate/up/down are raw storage of `dtype` (uint16 bits for bf16/f16).  Returns the f32 output
    [T,H] before the final rounding to `dtype`.  round_dtype defaults to `dtype` for bf16/f16 (the
    reference's GEMM path rounds the intermediate and each weighted contribution) and to none
    for f32.  with_max_contrib: returns (out, max_contrib), max_contrib [T,H] the largest
    |rounded weighted contribution| among each token's slots."""
    x = np.ascontiguousarray(x)
    T, H = x.shape
    E, H2, I = gate.shape
    assert H2 == H
    k = indices.shape[1]
    if round_dtype is None:
        round_dtype = dtype
    out = np.empty((T, H), np.float32)
    mc = np.empty((T, H), np.float32) if with_max_contrib else None
    if T == 0:
        return (out, mc) if with_max_contrib else out
    rc = lib().oracle_moe_forward_ex(
        _ptr(x), _ptr(np.ascontiguousarray(gate)), _ptr(np.ascontiguousarray(up)),
        _ptr(None if down is None else np.ascontiguousarray(down)),
        _ptr(np.ascontiguousarray(routing_weights, dtype=np.float32)),
        _ptr(np.ascontiguousarray(indices).view(np.uint32)),
        T, H, I, E, k, activation, moe_type, DTYPE_CODES[dtype], DTYPE_CODES[round_dtype],
        nthreads, _ptr(out), _ptr(mc))
    if rc != 0:
        raise MemoryError("oracle_moe_forward: allocation failed")
    return (out, mc) if with_max_contrib else out


def activation(x: float, act: int) -> float:
    return lib().oracle_activation(x, act)


def allclose_report(got: np.ndarray, ref: np.ndarray, rtol: float, atol: float):
    """|got-ref| <= atol + rtol*max(|got|,|ref|) (tests/moe_tests.rs:61-91).  Returns
    (ok, max_abs_err, worst_index)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    diff = np.abs(got - ref)
    tol = atol + rtol * np.maximum(np.abs(got), np.abs(ref))
    bad = diff > tol
    worst = int(np.argmax(diff - tol)) if diff.size else 0
    return (not bool(bad.any())), float(diff.max() if diff.size else 0.0), worst
