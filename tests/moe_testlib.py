"""Helpers shared by the tests: seeded inputs (via the oracle's SplitMix64/Box-Muller
generator), host<->torch conversion of raw bf16/f16 storage, and the tolerance rule."""
from __future__ import annotations

import json
import os

import numpy as np

import oracle

TORCH_DTYPES = {}


def torch_dtype(name: str):
    import torch
    return {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[name]


def to_torch(raw: np.ndarray, dtype: str, device="cuda"):
    """Raw oracle storage (float32, or uint16 bit patterns) -> torch tensor of `dtype`."""
    import torch
    if dtype == "f32":
        return torch.from_numpy(np.ascontiguousarray(raw, dtype=np.float32)).to(device)
    t = torch.from_numpy(np.ascontiguousarray(raw).view(np.int16))
    return t.view(torch_dtype(dtype)).to(device)


def from_torch(t, dtype: str) -> np.ndarray:
    """torch tensor -> raw storage (float32 or uint16 bits)."""
    import torch
    t = t.detach().contiguous().cpu()
    if dtype == "f32":
        return t.numpy().astype(np.float32)
    return t.view(torch.int16).numpy().view(np.uint16)


def moe_case(seed: int, T: int, H: int, I: int, E: int, k: int, moe_type: int, dtype: str,
             wstd: float = 0.02, xstd: float = 1.0, bias_std: float = 0.0,
             renormalize: bool = False):
    """Seeded inputs in the API layout (gate/up [E,H,I], down [E,I,H]) and router outputs from
    the oracle router over N(0,1) logits (+ an optional per-expert N(0,bias_std) bias)."""
    x = oracle.randn(seed * 101 + 1, (T, H), std=xstd, dtype=dtype)
    gate = oracle.randn(seed * 101 + 2, (E, H, I), std=wstd, dtype=dtype)
    up = oracle.randn(seed * 101 + 3, (E, H, I), std=wstd, dtype=dtype)
    down = oracle.randn(seed * 101 + 4, (E, I, H), std=wstd, dtype=dtype) if moe_type == 0 else None
    logits = oracle.randn(seed * 101 + 5, (T, E))
    if bias_std:
        logits = logits + oracle.randn(seed * 101 + 6, (E,), std=bias_std)[None, :]
        logits = np.ascontiguousarray(logits, dtype=np.float32)
    w, idx, _, _ = oracle.topk_softmax(logits, k, renormalize=renormalize)
    return dict(x=x, gate=gate, up=up, down=down, logits=logits, w=w, idx=idx)


def rel_tol(dtype: str) -> float:
    """Tolerance of the north-star spec: 1e-4 relative for f32, 1e-2 relative for f16/bf16."""
    return 1e-4 if dtype == "f32" else 1e-2


PARITY_LOG = os.environ.get("CMOE_PARITY_LOG")


def ulp(values: np.ndarray, dtype: str) -> np.ndarray:
    """One unit in the last place of each |value| in `dtype` (0 for f32 and for zeros)."""
    a = np.abs(np.asarray(values, np.float64))
    if dtype == "f32":
        return np.zeros_like(a)
    mant = 7 if dtype == "bf16" else 10
    _, e = np.frexp(a)  # a = f * 2**e, 0.5 <= f < 1
    u = np.ldexp(1.0, e - 1 - mant)
    return np.where(a > 0, u, 0.0)


def oracle_ref(case: dict, act: int, moe_type: int, dtype: str, rows=None):
    """(oracle output [rows, H] before the final rounding, slack [rows, H]) for a moe_case.

    slack = one unit in the last place (of `dtype`) of the element's largest weighted slot
    contribution: the reference rounds every contribution to the operand type before the slots
    are summed (qwen3_moe.cu:637-641), so an f32 accumulation in another order (tensor cores, or
    the reference's own atomics) can land one unit away on a contribution, which may be larger
    than the sum itself."""
    x, w, idx = case["x"], case["w"], case["idx"]
    if rows is not None:
        x, w, idx = x[rows], w[rows], idx[rows]
    ref, mc = oracle.moe_forward(np.ascontiguousarray(x), case["gate"], case["up"], case["down"],
                                 np.ascontiguousarray(w), np.ascontiguousarray(idx),
                                 activation=act, moe_type=moe_type, dtype=dtype,
                                 with_max_contrib=True)
    return ref, ulp(mc, dtype)


def error_report(got: np.ndarray, ref: np.ndarray) -> dict:
    """Error figures of one comparison: max |got-ref| / rms(ref) (the scaled form), and the pure
    element-wise relative error |got-ref| / |ref| -- its maximum over the non-cancelling elements
    (|ref| >= rms(ref), where a relative error is meaningful), and the fraction of ALL elements
    whose pure relative error is within 1e-2 and within 1e-4."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    diff = np.abs(got - ref)
    scale = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    big = np.abs(ref) >= max(scale, 1e-30)
    rel = diff / np.maximum(np.abs(ref), 1e-30)
    return {
        "max_err_of_rms": float(diff.max() / max(scale, 1e-30)) if diff.size else 0.0,
        "max_rel_noncancelling": float(rel[big].max()) if big.any() else 0.0,
        "noncancelling": int(big.sum()),
        "frac_rel_le_1e-2": float(np.mean(rel <= 1e-2)) if rel.size else 1.0,
        "frac_rel_le_1e-4": float(np.mean(rel <= 1e-4)) if rel.size else 1.0,
        "elements": int(ref.size),
    }


def check_close(got: np.ndarray, ref: np.ndarray, rtol: float, what: str = "", slack=None):
    """Element-wise |got-ref| <= rtol*|ref| + rtol*rms(ref) (relative error at the data's
    scale; the rms term keeps cancellation-sized outputs from failing a pure relative test).

    The pure element-wise relative error |got-ref| / |ref| is reported beside it (error_report)
    and bounded by 2*rtol on every non-cancelling element (|ref| >= rms(ref)): for f16/bf16 one
    unit in the last place is 0.4-0.8 % of a value, and a contribution that the reference rounds
    to the operand type before the slots are summed can be larger than the sum itself, so a
    single rounding flip of one contribution can exceed 1e-2 of the sum on its own.

    slack (optional, per element, from oracle_ref): added to the tolerance of each element --
    one unit in the last place of its largest rounded contribution.

    Returns max |got-ref| / rms(ref); with CMOE_PARITY_LOG set, appends one JSON line per
    comparison (the error_report figures) to that file."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    rep = error_report(got, ref)
    if PARITY_LOG:
        with open(PARITY_LOG, "a") as f:
            f.write(json.dumps({"case": what, "rtol": rtol, **rep}) + "\n")
    scale = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    atol = rtol * max(scale, 1e-30)
    diff = np.abs(got - ref)
    tol = atol + rtol * np.abs(ref)
    if slack is not None:
        tol = tol + np.asarray(slack, np.float64)
    bad = diff > tol
    if bad.any():
        i = int(np.argmax(diff - tol))
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} elements out of tolerance (rtol={rtol}); "
            f"worst at flat {i}: got={got.flat[i]:.6g} ref={ref.flat[i]:.6g} "
            f"max_abs={diff.max():.3g} scale={scale:.3g}")
    assert rep["max_rel_noncancelling"] <= 2 * rtol, (
        f"{what}: pure relative error {rep['max_rel_noncancelling']:.3g} > {2 * rtol} on a "
        f"non-cancelling element ({rep})")
    return rep["max_err_of_rms"]
