"""Our kernels against the reference crate's own CUDA kernels (oracle/_ref/libref_moe.so, built
from the reference sources for sm_100a) on identical seeded inputs, on the reference paths that
launch.  Also records the reference's failed launches (finding: its large f16/bf16 GEMM kernels
request more than 48 KB of dynamic shared memory without opting in)."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle
from oracle import refkernels
from moe_testlib import check_close, from_torch, moe_case, to_torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refkernels.available(),
                                 reason="oracle/_ref/libref_moe.so not built")]

DT = {"f16": 0, "bf16": 1, "f32": 2}


@pytest.mark.parametrize("E", [1, 2, 4, 8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("k", [1, 2, 8])
def test_router_bit_exact_vs_reference(E, k):
    if k > E:
        pytest.skip("k > E")
    x = torch.from_numpy(oracle.randn(E + 100 * k, (2000, E))).cuda()
    rw, ri, rs = refkernels.topk_softmax(x, k)
    w, i, s = candle_moe.topk_softmax(x, k)
    torch.cuda.synchronize()
    assert torch.equal(i, ri)
    assert torch.equal(s, rs)
    assert torch.equal(w.view(torch.int32), rw.view(torch.int32))  # bit-identical weights


@pytest.mark.parametrize("E", [128, 256])
@pytest.mark.parametrize("k", [3, 16, 32, 33])
@pytest.mark.parametrize("T", [1, 77, 4096])
def test_router_large_expert_counts_many_k_bit_exact_vs_reference(E, k, T):
    """128 and 256 experts (a warp per row), odd and large k, a single token and ragged counts,
    rows with ties: bit-identical to the reference kernel."""
    x = oracle.randn(E * k + T, (T, E))
    x[::5] = np.round(x[::5])  # rows with ties
    x = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    rw, ri, rs = refkernels.topk_softmax(x, k)
    w, i, s = candle_moe.topk_softmax(x, k)
    torch.cuda.synchronize()
    assert torch.equal(i, ri)
    assert torch.equal(s, rs)
    assert torch.equal(w.view(torch.int32), rw.view(torch.int32))


@pytest.mark.parametrize("E", [8, 128, 256])
def test_router_ties_and_non_finite_rows_bit_exact_vs_reference(E):
    """Logits from a 5-value set (ties on every row), plus rows with -inf, +inf and NaN logits:
    the picks (value, then lowest expert) and their bits match the reference kernel, including the
    rows whose probabilities are NaN."""
    k = 8
    g = torch.Generator().manual_seed(E)
    x = torch.randint(-2, 3, (1500, E), generator=g).float()
    x[7, 3] = float("-inf")
    x[11, :E // 2] = float("-inf")
    x[13, 5] = float("inf")
    x[17, E - 1] = float("nan")
    x = x.cuda()
    rw, ri, rs = refkernels.topk_softmax(x, k)
    w, i, s = candle_moe.topk_softmax(x, k)
    torch.cuda.synchronize()
    assert torch.equal(i, ri)
    assert torch.equal(s, rs)
    assert torch.equal(w.view(torch.int32), rw.view(torch.int32))


@pytest.mark.parametrize("T,k,E", [(512, 2, 8), (4096, 8, 16), (8192, 8, 128), (3000, 2, 7)])
def test_route_prep_vs_reference(T, k, E):
    rng = np.random.default_rng(T + k + E)
    idx = torch.from_numpy(rng.integers(0, E, size=(T, k)).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.standard_normal((T, k)).astype(np.float32)).cuda()
    ro, rst, rsw = refkernels.preprocessing(idx, w, E)
    o, st, sw = candle_moe.route_prep(idx, w, E)
    torch.cuda.synchronize()
    assert torch.equal(o, ro)
    o = o.cpu().numpy()
    for e in range(E):
        lo, hi = o[e], o[e + 1]
        a = sorted(zip(st[lo:hi].tolist(), sw[lo:hi].tolist()))
        b = sorted(zip(rst[lo:hi].tolist(), rsw[lo:hi].tolist()))
        assert a == b, e


REF_MOE = [
    # dtype, moe_type, act, T, H, I, E, k  (reference path taken)
    ("f32", 1, 0, 512, 64, 256, 8, 2),     # f32 FFMA
    ("f32", 0, 0, 300, 96, 160, 8, 2),     # f32 FFMA
    ("f32", 1, 1, 100, 32, 128, 8, 2),     # f32 FFMA, GELU
    ("f32", 1, 1, 256, 256, 384, 8, 2),    # f32 FFMA here; ours on the tensor cores (3xTF32)
    ("f32", 0, 0, 200, 128, 256, 8, 2),    # same, Qwen3 SwiGLU
    ("bf16", 0, 0, 8, 256, 512, 8, 2),     # direct (T <= 32)
    ("f16", 1, 2, 32, 128, 256, 8, 2),     # direct, ReLU
    ("f16", 0, 0, 48, 64, 256, 8, 1),      # small wmma GEMM (k=1, 33 <= T <= 64)
]


@pytest.mark.parametrize("dtype,moe_type,act,T,H,I,E,k", REF_MOE)
def test_moe_vs_reference(dtype, moe_type, act, T, H, I, E, k):
    c = moe_case(T + H + act, T=T, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype=dtype, wstd=0.1)
    args = [to_torch(c["x"], dtype), to_torch(c["gate"], dtype), to_torch(c["up"], dtype),
            None if c["down"] is None else to_torch(c["down"], dtype),
            torch.from_numpy(c["w"]).cuda(), torch.from_numpy(c["idx"]).cuda()]
    ref, err = refkernels.fused_moe(*args, E, k, act, moe_type, DT[dtype])
    assert err == 0
    ours = candle_moe.FusedMoE(E, k, candle_moe.Activation(act)).forward(*args, moe_type)
    torch.cuda.synchronize()
    r = oracle.to_f32(from_torch(ref, dtype), dtype)
    o = oracle.to_f32(from_torch(ours, dtype), dtype)
    check_close(o, r, 1e-4 if dtype == "f32" else 1e-2, "ours vs reference")
    orc = oracle.moe_forward(c["x"], c["gate"], c["up"], c["down"], c["w"], c["idx"],
                             activation=act, moe_type=moe_type, dtype=dtype)
    check_close(r, orc, 1e-4 if dtype == "f32" else 1e-2, "reference vs oracle")


def test_reference_large_bf16_gemm_does_not_launch():
    """C3 shape (Nomic bf16, H=768, I=3072, T=4096): the reference selects its 128x128 wmma
    kernels, which ask for 64 KB of dynamic shared memory without the opt-in attribute; the
    launch fails and the output stays zero (nomic_moe.cu:2164-2180)."""
    c = moe_case(3, T=4096, H=768, I=3072, E=8, k=2, moe_type=1, dtype="bf16")
    args = [to_torch(c["x"], "bf16"), to_torch(c["gate"], "bf16"), to_torch(c["up"], "bf16"),
            None, torch.from_numpy(c["w"]).cuda(), torch.from_numpy(c["idx"]).cuda()]
    ref, err = refkernels.fused_moe(*args, 8, 2, 1, 1, 1)
    assert err != 0
    assert float(ref.float().abs().max()) == 0.0
