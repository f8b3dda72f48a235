"""GEMM-2 (default) and GEMM-1 (opt-in path 4) on CTA pairs (cta_group::2) against the oracle and
against the one-CTA kernels (GEMM path 3) on the same inputs: Qwen3 shapes whose hidden
size is a multiple of 256, expert row counts that are not multiples of 256 (half-empty pair
tiles), a k = 1 call, and the config-5 shape on a token sample."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle
from moe_testlib import check_close, from_torch, moe_case, oracle_ref, to_torch

pytestmark = pytest.mark.gpu

CASES = [  # dtype, T, H, I, E, k
    ("bf16", 300, 256, 256, 8, 2),
    ("f16", 1000, 512, 384, 8, 2),
    ("bf16", 96, 256, 128, 4, 1),
    ("bf16", 2048, 2048, 768, 128, 8),
]


def _run(case, dtype, E, k, path):
    prev = candle_moe.set_gemm_path(path)
    try:
        out = candle_moe.FusedMoE(E, k).forward(
            to_torch(case["x"], dtype), to_torch(case["gate"], dtype), to_torch(case["up"], dtype),
            to_torch(case["down"], dtype), torch.from_numpy(case["w"]).cuda(),
            torch.from_numpy(case["idx"]).cuda(), 0)
        torch.cuda.synchronize()
        return out
    finally:
        candle_moe.set_gemm_path(prev)


@pytest.mark.parametrize("path", [0, 4])
@pytest.mark.parametrize("dtype,T,H,I,E,k", CASES)
def test_pair_gemms_match_oracle_and_one_cta_path(dtype, T, H, I, E, k, path):
    """path 0: GEMM-2 on CTA pairs; path 4: GEMM-1 on CTA pairs too."""
    candle_moe.device_error_bits(0, clear=True)
    case = moe_case(77, T=T, H=H, I=I, E=E, k=k, moe_type=0, dtype=dtype, renormalize=True,
                    bias_std=0.5)
    pair = _run(case, dtype, E, k, path)
    assert candle_moe.device_error_bits(0) == 0
    one = _run(case, dtype, E, k, 3)
    got = oracle.to_f32(from_torch(pair, dtype), dtype)
    rows = np.arange(T) if T <= 400 else np.random.default_rng(5).choice(T, 400, replace=False)
    ref, slack = oracle_ref(case, 0, 0, dtype, rows)
    check_close(got[rows], ref, 1e-2, f"pair path {path} {dtype} T={T}", slack)
    diff = (pair.float() - one.float()).abs().max().item()
    assert diff <= 1e-2 * max(one.float().abs().max().item(), 1e-6), diff


@pytest.mark.parametrize("reserve", [24, 127, 128])
def test_large_sm_reserve_still_runs_every_gemm(reserve):
    """moe_set_sm_reserve leaves SMs to concurrent kernels; however few it leaves (the pair
    kernel needs two per cluster), both GEMMs still run and the output is unchanged."""
    dtype, T, H, I, E, k = "bf16", 600, 512, 256, 8, 2
    case = moe_case(91, T=T, H=H, I=I, E=E, k=k, moe_type=0, dtype=dtype, renormalize=True)
    ref = _run(case, dtype, E, k, 0)
    prev = candle_moe.set_sm_reserve(reserve)
    try:
        got = _run(case, dtype, E, k, 0)
    finally:
        candle_moe.set_sm_reserve(prev)
    assert candle_moe.device_error_bits(0) == 0
    assert torch.equal(got, ref)
