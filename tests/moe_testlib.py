"""Helpers shared by the tests: seeded inputs (via the oracle's SplitMix64/Box-Muller
generator), host<->torch conversion of raw bf16/f16 storage, and the tolerance rule."""
from __future__ import annotations

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


def check_close(got: np.ndarray, ref: np.ndarray, rtol: float, what: str = ""):
    """Element-wise |got-ref| <= rtol*|ref| + rtol*rms(ref) (relative error at the data's
    scale; the rms term keeps cancellation-sized outputs from failing a pure relative test)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    scale = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    atol = rtol * max(scale, 1e-30)
    diff = np.abs(got - ref)
    bad = diff > atol + rtol * np.abs(ref)
    if bad.any():
        i = int(np.argmax(diff - (atol + rtol * np.abs(ref))))
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} elements out of tolerance (rtol={rtol}); "
            f"worst at flat {i}: got={got.flat[i]:.6g} ref={ref.flat[i]:.6g} "
            f"max_abs={diff.max():.3g} scale={scale:.3g}")
    return float(diff.max() / max(scale, 1e-30)) if diff.size else 0.0
