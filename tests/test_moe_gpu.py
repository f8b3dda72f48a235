"""Fused MoE on the GPU vs the oracle (the reference's naive per-expert path, f16/bf16 rounding
of the intermediate and of each weighted contribution).  Tolerance (north-star spec): 1e-4
relative for f32, 1e-2 relative for f16/bf16, measured at the data's scale (moe_testlib)."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle
from moe_testlib import check_close, from_torch, moe_case, oracle_ref, rel_tol, to_torch

pytestmark = pytest.mark.gpu


def run_gpu(case, E, k, act, moe_type, dtype, path=0):
    prev = candle_moe.set_gemm_path(path)
    try:
        moe = candle_moe.FusedMoE(E, k, candle_moe.Activation(act))
        out = moe.forward(to_torch(case["x"], dtype), to_torch(case["gate"], dtype),
                          to_torch(case["up"], dtype),
                          None if case["down"] is None else to_torch(case["down"], dtype),
                          torch.from_numpy(case["w"]).cuda(),
                          torch.from_numpy(case["idx"].view(np.int32)).cuda(), moe_type)
        torch.cuda.synchronize()
        used = candle_moe.last_gemm_path()
    finally:
        candle_moe.set_gemm_path(prev)
    return oracle.to_f32(from_torch(out, dtype), dtype), used


def check_vs_oracle(got, case, act, moe_type, dtype, what, rows=None, rtol=None):
    """got (rows of the output, f32) against the oracle: the rtol rule plus one unit in the last
    place of each element's largest rounded contribution (moe_testlib.oracle_ref)."""
    ref, slack = oracle_ref(case, act, moe_type, dtype, rows)
    return check_close(got, ref, rel_tol(dtype) if rtol is None else rtol, what, slack)


# the reference's own ten configs (tests/moe_tests.rs:279-397): E=8, I=4H, SiLU, N(0,1) weights
REFERENCE_CASES = [
    ("f32", 1, 16, 16, 2), ("f16", 1, 64, 32, 2), ("f16", 1, 64, 32, 1), ("f32", 0, 64, 32, 2),
    ("f16", 0, 64, 4, 2), ("f16", 0, 64, 32, 2), ("f16", 0, 64, 32, 1), ("bf16", 0, 64, 4, 2),
    ("bf16", 0, 64, 32, 2), ("bf16", 0, 64, 32, 1),
]


@pytest.mark.parametrize("dtype,moe_type,H,T,k", REFERENCE_CASES)
def test_reference_test_configs(dtype, moe_type, H, T, k):
    case = moe_case(H + T + k, T=T, H=H, I=4 * H, E=8, k=k, moe_type=moe_type, dtype=dtype,
                    wstd=1.0)
    got, _ = run_gpu(case, 8, k, 0, moe_type, dtype)
    check_vs_oracle(got, case, 0, moe_type, dtype, "ref config", rtol=rel_tol(dtype))


TC_CASES = [
    # dtype, moe_type, act, T, H, I, E, k
    ("bf16", 0, 0, 300, 256, 512, 8, 2),
    ("f16", 0, 0, 300, 256, 512, 8, 2),
    ("bf16", 1, 1, 300, 256, 512, 8, 2),
    ("f16", 1, 2, 300, 256, 512, 8, 2),
    ("bf16", 1, 1, 129, 128, 256, 4, 1),
    ("bf16", 0, 0, 1, 128, 128, 8, 2),
    ("bf16", 0, 0, 700, 256, 256, 128, 8),
    ("bf16", 1, 0, 257, 384, 640, 16, 4),
    ("f16", 0, 1, 2000, 512, 384, 8, 2),
]


@pytest.mark.parametrize("dtype,moe_type,act,T,H,I,E,k", TC_CASES)
def test_tensor_core_path_vs_oracle(dtype, moe_type, act, T, H, I, E, k):
    case = moe_case(T + H + I + E + k + act, T=T, H=H, I=I, E=E, k=k, moe_type=moe_type,
                    dtype=dtype)
    got, used = run_gpu(case, E, k, act, moe_type, dtype, path=2)
    assert used in (2, 3)  # grouped GEMMs, or the decode kernels for <= 64 tokens
    check_vs_oracle(got, case, act, moe_type, dtype, "tcgen05", rtol=rel_tol(dtype))


@pytest.mark.parametrize("dtype,moe_type,act,T,H,I,E,k", TC_CASES[:4])
def test_simt_path_vs_oracle(dtype, moe_type, act, T, H, I, E, k):
    case = moe_case(T + H + I + E + k + act, T=T, H=H, I=I, E=E, k=k, moe_type=moe_type,
                    dtype=dtype)
    got, used = run_gpu(case, E, k, act, moe_type, dtype, path=1)
    assert used == 1
    check_vs_oracle(got, case, act, moe_type, dtype, "simt", rtol=rel_tol(dtype))


@pytest.mark.parametrize("moe_type,act", [(0, 0), (1, 1), (1, 2), (0, 2)])
def test_f32_path_vs_oracle(moe_type, act):
    case = moe_case(77 + act, T=200, H=96, I=160, E=8, k=2, moe_type=moe_type, dtype="f32")
    got, used = run_gpu(case, 8, 2, act, moe_type, "f32")
    assert used == 1
    check_vs_oracle(got, case, act, moe_type, "f32", "f32", rtol=1e-4)


def test_edge_experts_without_tokens_and_one_hot_routing():
    case = moe_case(5, T=500, H=256, I=256, E=16, k=2, moe_type=0, dtype="bf16")
    case["idx"] = (case["idx"] % 3).astype(np.int32)  # experts 3..15 get no rows
    case["idx"][:, 1] = np.where(case["idx"][:, 0] == case["idx"][:, 1], 2, case["idx"][:, 1])
    got, _ = run_gpu(case, 16, 2, 0, 0, "bf16", path=2)
    check_vs_oracle(got, case, 0, 0, "bf16", "sparse experts", rtol=1e-2)
    case["idx"][:, 0] = 7
    case["idx"][:, 1] = 9
    got, _ = run_gpu(case, 16, 2, 0, 0, "bf16", path=2)
    check_vs_oracle(got, case, 0, 0, "bf16", "two experts", rtol=1e-2)


def test_edge_out_of_range_expert_ids_are_skipped():
    case = moe_case(6, T=64, H=128, I=256, E=8, k=2, moe_type=1, dtype="bf16")
    case["idx"][::3, 1] = 8
    got, _ = run_gpu(case, 8, 2, 0, 1, "bf16", path=2)
    check_vs_oracle(got, case, 0, 1, "bf16", "invalid ids", rtol=1e-2)


def test_paths_agree_and_runs_are_deterministic():
    case = moe_case(8, T=1000, H=256, I=384, E=8, k=2, moe_type=0, dtype="bf16")
    a, _ = run_gpu(case, 8, 2, 0, 0, "bf16", path=2)
    b, _ = run_gpu(case, 8, 2, 0, 0, "bf16", path=2)
    c, _ = run_gpu(case, 8, 2, 0, 0, "bf16", path=1)
    assert np.array_equal(a, b)
    check_close(a, c, 1e-2, "tcgen05 vs simt")


def test_zero_tokens():
    moe = candle_moe.FusedMoE(8, 2)
    x = torch.zeros(0, 128, dtype=torch.bfloat16, device="cuda")
    g = torch.zeros(8, 128, 256, dtype=torch.bfloat16, device="cuda")
    out = moe.forward(x, g, g, g.transpose(1, 2).contiguous(),
                      torch.zeros(0, 2, device="cuda"),
                      torch.zeros(0, 2, dtype=torch.int32, device="cuda"), 0)
    assert out.shape == (0, 128)


# BASELINE-shaped configs at full size, checked on a seeded sample of tokens (each output row
# depends only on its own token, so the oracle runs on the sampled rows alone).
FULL = [
    ("c3-nomic-bf16-T64", "bf16", 1, 1, 64, 768, 3072, 8, 2, 0.0),
    ("c3-nomic-bf16-T4096", "bf16", 1, 1, 4096, 768, 3072, 8, 2, 0.0),
    ("c3-nomic-bf16-T32768", "bf16", 1, 1, 32768, 768, 3072, 8, 2, 0.0),
    ("c4-qwen3-bf16-T8", "bf16", 0, 0, 8, 4096, 1536, 8, 2, 0.0),
    ("c4-qwen3-f16-T8", "f16", 0, 0, 8, 4096, 1536, 8, 2, 0.0),
    ("c4-qwen3-bf16-T64", "bf16", 0, 0, 64, 4096, 1536, 8, 2, 0.0),
    ("c4-qwen3-f16-T64", "f16", 0, 0, 64, 4096, 1536, 8, 2, 0.0),
    ("c4-qwen3-bf16-T32768", "bf16", 0, 0, 32768, 4096, 1536, 8, 2, 0.0),
    ("c4-qwen3-f16-T32768", "f16", 0, 0, 32768, 4096, 1536, 8, 2, 0.0),
    ("c5-qwen3-bf16-T65536", "bf16", 0, 0, 65536, 2048, 768, 128, 8, 0.5),
]


@pytest.mark.parametrize("name,dtype,moe_type,act,T,H,I,E,k,bias", FULL)
def test_baseline_shapes_sampled(name, dtype, moe_type, act, T, H, I, E, k, bias):
    case = moe_case(1, T=T, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype=dtype, bias_std=bias,
                    renormalize=(moe_type == 0))
    got, used = run_gpu(case, E, k, act, moe_type, dtype)
    assert used in (2, 3)  # grouped GEMMs, or the decode kernels for <= 64 tokens
    rows = np.sort(np.random.default_rng(0).choice(T, size=min(T, 48), replace=False))
    check_vs_oracle(got[rows], case, act, moe_type, dtype, name, rows, rtol=rel_tol(dtype))


def test_c2_nomic_f32_full_shape_all_tokens():
    """BASELINE config 2 at its own shape (f32 Nomic, 512 tokens, H768, I3072, 8 experts top-2,
    GELU), every output element against the oracle at the f32 tolerance 1e-4: the tensor-core
    path (three TF32 products) and the FFMA path."""
    case = moe_case(2, T=512, H=768, I=3072, E=8, k=2, moe_type=1, dtype="f32")
    candle_moe.device_error_bits(0, clear=True)
    got, used = run_gpu(case, 8, 2, 1, 1, "f32")
    assert used == 2
    assert candle_moe.device_error_bits(0) == 0
    check_vs_oracle(got, case, 1, 1, "f32", "c2-nomic-f32-T512 3xTF32", rtol=1e-4)
    got, used = run_gpu(case, 8, 2, 1, 1, "f32", path=1)
    assert used == 1
    check_vs_oracle(got, case, 1, 1, "f32", "c2-nomic-f32-T512 FFMA", rtol=1e-4)


@pytest.mark.parametrize("moe_type,act,T,H,I,E,k", [
    (1, 1, 300, 256, 384, 8, 2),    # Nomic GELU, GEMM-2 K-major B in 64-column tiles
    (0, 0, 300, 256, 384, 8, 2),    # Qwen3 SwiGLU: gate|up as one N = 128 MMA, GEMM-2 MN-major
    (0, 2, 77, 2048, 256, 16, 1),   # k = 1 (GEMM-2 writes the output), 128-column GEMM-2 tiles
    (1, 0, 1000, 128, 128, 4, 4),   # one 128-wide GEMM-1 tile per m-tile, many m-tiles
])
def test_f32_tensor_core_path_vs_oracle(moe_type, act, T, H, I, E, k):
    """f32 on the tensor cores (moe_tf32.cu) against the oracle at 1e-4 relative, and against
    the FFMA path on the same inputs."""
    case = moe_case(91 + T + act, T=T, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype="f32",
                    renormalize=(moe_type == 0))
    candle_moe.device_error_bits(0, clear=True)
    got, used = run_gpu(case, E, k, act, moe_type, "f32")
    assert used == 2
    assert candle_moe.device_error_bits(0) == 0
    check_vs_oracle(got, case, act, moe_type, "f32", f"3xTF32 {moe_type} {act}", rtol=1e-4)
    simt, used = run_gpu(case, E, k, act, moe_type, "f32", path=1)
    assert used == 1
    check_close(got, simt, 1e-4, "3xTF32 vs FFMA")
