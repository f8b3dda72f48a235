"""The drop-in symbols exactly as the reference crate's Rust layer calls them.

src/lib.rs:450-469 calls the void `fused_moe` (src/ffi.rs:45-62) with raw device pointers into a
caller-allocated output that it zeroed first (src/lib.rs:296), and src/lib.rs:108-119 calls the
void `topk_softmax` (src/ffi.rs:15-24).  Neither returns a status; this library records one per
thread, read with moe_last_status().  These tests go through ctypes straight to those symbols
(no Python wrapper in between) and check the output against the CPU oracle at the north-star
tolerances (1e-4 relative for f32, 1e-2 for f16/bf16), then the status.
"""
import ctypes

import numpy as np
import pytest
import torch

import candle_moe
import oracle
from moe_testlib import check_close, from_torch, moe_case, oracle_ref, rel_tol, to_torch

pytestmark = pytest.mark.gpu

DT = {"f16": 0, "bf16": 1, "f32": 2}


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call_fused_moe(x, gate, up, down, w, idx, out, T, H, I, E, k, act, moe_type, dtype):
    L = candle_moe.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the argument list of src/lib.rs:450-469, in its order and C types
    L.fused_moe(_p(x), _p(gate), _p(up), _p(down), _p(w), _p(idx), _p(out), T, H, I, E, k, act,
                moe_type, DT[dtype], stream)
    torch.cuda.synchronize()
    return L.moe_last_status()


CASES = [
    # dtype, moe_type, act, T, H, I, E, k   (f32: SIMT; f16/bf16 aligned: tcgen05; k = 1 writes
    # the output rows directly, without the slot combine)
    ("f32", 1, 1, 200, 96, 160, 8, 2),
    ("f32", 0, 0, 64, 128, 256, 8, 1),
    ("bf16", 0, 0, 300, 256, 512, 8, 2),
    ("bf16", 1, 1, 129, 128, 256, 4, 1),
    ("f16", 0, 0, 257, 256, 384, 16, 4),
    ("f16", 0, 2, 100, 256, 256, 8, 1),
    ("bf16", 0, 0, 8, 512, 256, 8, 2),
    ("bf16", 0, 0, 40, 64, 256, 8, 2),  # the reference's own test shapes use H=64 (SIMT path)
]


@pytest.mark.parametrize("dtype,moe_type,act,T,H,I,E,k", CASES)
def test_void_fused_moe_as_the_rust_layer_calls_it(dtype, moe_type, act, T, H, I, E, k):
    case = moe_case(31 + T + k + act, T=T, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype=dtype,
                    renormalize=(moe_type == 0))
    x = to_torch(case["x"], dtype)
    gate, up = to_torch(case["gate"], dtype), to_torch(case["up"], dtype)
    down = None if case["down"] is None else to_torch(case["down"], dtype)
    w = torch.from_numpy(case["w"]).cuda()
    idx = torch.from_numpy(case["idx"].view(np.uint32).view(np.int32)).cuda()
    out = torch.zeros((T, H), dtype=x.dtype, device="cuda")  # src/lib.rs:296: zeroed output
    st = _call_fused_moe(x, gate, up, down, w, idx, out, T, H, I, E, k, act, moe_type, dtype)
    assert st == 0, candle_moe.lib().moe_status_string(st)
    got = oracle.to_f32(from_torch(out, dtype), dtype)
    ref, slack = oracle_ref(case, act, moe_type, dtype)
    check_close(got, ref, rel_tol(dtype), f"fused_moe {dtype} type{moe_type} k{k} T{T}", slack)


def test_void_fused_moe_overwrites_a_dirty_output():
    """The reference accumulates into its output, so its caller must zero it; this library
    overwrites it, which gives the same result for a zeroed output and the exact result for a
    dirty one."""
    T, H, I, E, k = 96, 256, 256, 8, 2
    case = moe_case(5, T=T, H=H, I=I, E=E, k=k, moe_type=0, dtype="bf16")
    args = [to_torch(case["x"], "bf16"), to_torch(case["gate"], "bf16"),
            to_torch(case["up"], "bf16"), to_torch(case["down"], "bf16"),
            torch.from_numpy(case["w"]).cuda(), torch.from_numpy(case["idx"]).cuda()]
    clean = torch.zeros((T, H), dtype=torch.bfloat16, device="cuda")
    dirty = torch.full((T, H), 7.0, dtype=torch.bfloat16, device="cuda")
    assert _call_fused_moe(*args, clean, T, H, I, E, k, 0, 0, "bf16") == 0
    assert _call_fused_moe(*args, dirty, T, H, I, E, k, 0, 0, "bf16") == 0
    assert torch.equal(clean, dirty)


def test_void_fused_moe_reports_errors_through_last_status():
    T, H, I, E, k = 16, 128, 128, 8, 2
    x = torch.zeros((T, H), dtype=torch.bfloat16, device="cuda")
    g = torch.zeros((E, H, I), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((T, k), device="cuda")
    idx = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    out = torch.full((T, H), 3.0, dtype=torch.bfloat16, device="cuda")
    # dtype code 7 does not exist (src/lib.rs:174-182 knows 0, 1, 2)
    L = candle_moe.lib()
    L.fused_moe(_p(x), _p(g), _p(g), _p(g), _p(w), _p(idx), _p(out), T, H, I, E, k, 0, 0, 7,
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    st = L.moe_last_status()
    assert st == candle_moe.MOE_ERR_INVALID_ARG
    # Qwen3 (moe_type 0) without down weights: the reference would dereference NULL
    L.fused_moe(_p(x), _p(g), _p(g), None, _p(w), _p(idx), _p(out), T, H, I, E, k, 0, 0, 1,
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert L.moe_last_status() == candle_moe.MOE_ERR_INVALID_ARG
    # a good call afterwards resets the status
    assert _call_fused_moe(x, g, g, g, w, idx, out, T, H, I, E, k, 0, 0, "bf16") == 0


def test_void_topk_softmax_matches_oracle_and_reports_status():
    T, E, k = 512, 8, 2
    logits = oracle.randn(99, (T, E))
    g = torch.from_numpy(logits).cuda()
    w = torch.empty((T, k), device="cuda")
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    src = torch.empty((T, k), dtype=torch.int32, device="cuda")
    L = candle_moe.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    L.topk_softmax(_p(g), _p(w), _p(idx), _p(src), E, T, k, stream)
    torch.cuda.synchronize()
    assert L.moe_last_status() == 0
    w_ref, idx_ref, src_ref, _ = oracle.topk_softmax(logits, k)
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert np.array_equal(src.cpu().numpy(), src_ref)
    assert np.max(np.abs(w.cpu().numpy() - w_ref)) <= 1e-6
    # 12 experts is not a power of two (src/lib.rs:73-78 rejects it before the FFI call)
    L.topk_softmax(_p(g), _p(w), _p(idx), _p(src), 12, T // 2, k, stream)
    torch.cuda.synchronize()
    assert L.moe_last_status() == candle_moe.MOE_ERR_UNSUPPORTED
