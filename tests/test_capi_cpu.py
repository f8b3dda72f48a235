"""CPU tests of the C-ABI library: it loads, exports exactly what include/candle_moe.h declares,
and rejects bad arguments before touching a GPU.  No kernel runs here."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

import candle_moe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "candle_moe.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", src)) - {"defined"})


def test_header_declares_the_reference_symbols():
    names = declared_functions()
    assert "topk_softmax" in names and "fused_moe" in names


def test_library_exports_every_declared_symbol():
    lib = candle_moe.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", candle_moe.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared_functions()), exported ^ set(declared_functions())


def test_status_strings():
    lib = candle_moe.lib()
    for code, text in [(0, "ok"), (1, "invalid argument"), (2, "unsupported"), (3, "cuda error"),
                       (5, "out of device memory")]:
        assert lib.moe_status_string(code).decode() == text
    assert lib.moe_status_string(99).decode() == "unknown status"


def test_fused_v2_rejects_bad_codes_without_a_gpu():
    lib = candle_moe.lib()
    p = ctypes.c_void_p(16)
    # dtype 7, moe_type 3, negative sizes: rejected before any CUDA call
    assert lib.moe_fused_v2(p, p, p, p, p, p, p, 4, 64, 256, 8, 2, 0, 0, 7, None, 0, None) == 1
    assert lib.moe_fused_v2(p, p, p, p, p, p, p, 4, 64, 256, 8, 2, 0, 3, 1, None, 0, None) == 1
    assert lib.moe_fused_v2(p, p, p, p, p, p, p, -1, 64, 256, 8, 2, 0, 0, 1, None, 0, None) == 1
    # Qwen3 without down weights
    assert lib.moe_fused_v2(p, p, p, None, p, p, p, 4, 64, 256, 8, 2, 0, 0, 1, None, 0, None) == 1
    # zero tokens: nothing to do
    assert lib.moe_fused_v2(p, p, p, p, p, p, p, 0, 64, 256, 8, 2, 0, 0, 1, None, 0, None) == 0
    # too many experts for route preparation
    assert lib.moe_fused_v2(p, p, p, p, p, p, p, 4, 64, 256, 4096, 2, 0, 0, 1, None, 0, None) == 2


def test_router_v2_rejects_bad_expert_counts_without_a_gpu():
    lib = candle_moe.lib()
    p = ctypes.c_void_p(16)
    assert lib.moe_topk_softmax_v2(p, p, p, p, 6, 10, 2, 0, None) == 2   # not a power of two
    assert lib.moe_topk_softmax_v2(p, p, p, p, 512, 10, 2, 0, None) == 2  # > 256
    assert lib.moe_topk_softmax_v2(p, p, p, p, 8, 10, 0, 0, None) == 1   # k = 0
    assert lib.moe_topk_softmax_v2(p, p, p, p, 8, 0, 2, 0, None) == 0    # no tokens


def test_workspace_size_layout():
    ws = candle_moe.workspace_size
    # rows = T*k; intermediate rows*I*elt and slot rows*H*elt dominate
    T, H, I, E, k = 65536, 2048, 768, 128, 8
    rows = T * k
    n = ws(T, H, I, E, k, 0, torch.bfloat16)
    assert n >= rows * I * 2 + rows * H * 2 + 3 * rows * 4
    assert n % 256 == 0
    assert ws(16, 64, 256, 8, 1, 1, torch.float32) >= 16 * 256 * 4  # k = 1: no slot buffer
    assert ws(0, 64, 256, 8, 2, 1, torch.float32) == 0


def test_python_api_validation_matches_reference_messages():
    moe = candle_moe.FusedMoE(8, 2, candle_moe.Activation.Silu)
    x = torch.zeros(4, 16)
    g = torch.zeros(8, 16, 64)
    w = torch.zeros(4, 2)
    i = torch.zeros(4, 2, dtype=torch.int32)
    with pytest.raises(ValueError, match="Number of experts mismatch"):
        moe.forward(x, torch.zeros(7, 16, 64), g, None, w, i, 1)
    with pytest.raises(ValueError, match="Hidden dimension mismatch for gate/up"):
        moe.forward(x, torch.zeros(8, 15, 64), g, None, w, i, 1)
    with pytest.raises(ValueError, match="Intermediate dimension mismatch"):
        moe.forward(x, g, torch.zeros(8, 16, 32), None, w, i, 1)
    with pytest.raises(ValueError, match="Number of tokens mismatch"):
        moe.forward(x, g, g, None, torch.zeros(3, 2), i, 1)
    with pytest.raises(ValueError, match="Number of selected experts mismatch"):
        moe.forward(x, g, g, None, torch.zeros(4, 3), i, 1)
    with pytest.raises(ValueError, match="moe_type must be one of 0 or 1"):
        moe.forward(x, g, g, None, w, i, 2)
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        moe.forward(x, g, g, None, w, i, 1)
    with pytest.raises(ValueError, match="must be a cuda tensor"):
        candle_moe.apply_topk_softmax_inplace(torch.zeros(4, 8), w, i, i)
    assert candle_moe.Activation.Gelu.to_int() == 1 and candle_moe.Activation.Relu.to_int() == 2
    with pytest.raises(TypeError):
        candle_moe.fused_moe_internal_dtype(torch.int8)


def test_exchange_entry_points_reject_bad_arguments_without_a_gpu():
    """The expert-parallel exchange entry points validate before any CUDA call."""
    lib = candle_moe.lib()
    p = ctypes.c_void_p(16)
    two = (ctypes.c_void_p * 2)(16, 32)
    many = (ctypes.c_void_p * 40)(*([16] * 40))
    h = (ctypes.c_uint8 * candle_moe.PEER_HANDLE_BYTES)()
    ptr = ctypes.c_void_p()
    # peer buffers: null outputs, zero size, null handles and pointers
    assert lib.moe_peer_alloc(0, ctypes.byref(ptr), h) == 1
    assert lib.moe_peer_alloc(64, None, h) == 1
    assert lib.moe_peer_open(None, ctypes.byref(ptr)) == 1
    assert lib.moe_peer_close(None) == 1
    assert lib.moe_peer_free(None) == 1
    assert lib.moe_copy_async(None, p, 16, None) == 1
    assert lib.moe_copy_async(p, p, 0, None) == 0  # nothing to copy
    # arrival flags: more than 64 flags, misaligned flags, non-positive timeout
    assert lib.moe_peer_signal(many, 65, 1, None) == 1
    assert lib.moe_peer_signal((ctypes.c_void_p * 1)(18), 1, 1, None) == 1
    assert lib.moe_peer_signal(None, 0, 1, None) == 0
    assert lib.moe_peer_wait(ctypes.c_void_p(18), 1, 1, 1000, None) == 1
    assert lib.moe_peer_wait(p, 65, 1, 1000, None) == 1
    assert lib.moe_peer_wait(p, 1, 1, 0, None) == 1
    # fused push kernels: rank counts beyond 32, null destination tables, inconsistent row maps
    assert lib.moe_ep_push_pairs(p, p, p, p, 0, p, p, 2, 8, 33, 64, 1, many, many, None, 0,
                                 None) == 1
    assert lib.moe_ep_push_pairs(p, p, p, p, 0, p, p, 2, 8, 2, 64, 1, None, two, None, 0,
                                 None) == 1
    assert lib.moe_ep_push_pairs(p, p, p, p, -1, p, p, 2, 8, 2, 64, 1, two, two, None, 0,
                                 None) == 1
    first = (ctypes.c_int64 * 3)(0, 5, 4)  # not ascending
    assert lib.moe_segment_sum_push(p, p, 4, 64, 1, 2, two, first, 0, None) == 1
    first = (ctypes.c_int64 * 3)(0, 2, 3)  # does not end at num_segments
    assert lib.moe_segment_sum_push(p, p, 4, 64, 1, 2, two, first, 0, None) == 1
    assert lib.moe_segment_sum_push(p, p, 0, 64, 1, 2, two, first, 0, None) == 0  # no rows
    # dest groups: assignment counts without a chunk count
    assert lib.moe_ep_dest_groups(p, 4, 2, 8, 2, 2, p, 0, p, None) == 1
