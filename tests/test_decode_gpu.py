"""The decode kernels (moe_decode.cu): decode-sized calls (at most 32 tokens by default, any size
with GEMM path 6, which these tests use) with the weights as
the tensor cores' A operand, the work split stream-K across all SMs and the combine fused into
GEMM-2.  They replace the reference's direct kernels (qwen3_moe.cu:85-263, nomic_moe.cu:6-174),
which the reference takes for T <= 32 (moe.cu:481).

Checked against the CPU oracle at every output element (north-star tolerance 1e-2 relative for
f16/bf16, plus one unit of each element's largest rounded contribution), against the grouped
GEMMs on the same inputs (GEMM path 5), for bit-identical repeat runs, and on the routing
shapes that exercise the bookkeeping: units cut between CTAs, experts with more rows than one
chunk, experts without rows, ids >= num_experts, and no routed row at all."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle
from moe_testlib import check_close, from_torch, moe_case, oracle_ref, rel_tol, to_torch

pytestmark = pytest.mark.gpu

DECODE, GROUPED, FORCE_DECODE = 0, 5, 6


def _run(case, E, k, act, moe_type, dtype, path):
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
    return out, used


def _check(case, E, k, act, moe_type, dtype, what, path=FORCE_DECODE):
    candle_moe.device_error_bits(0, clear=True)
    out, used = _run(case, E, k, act, moe_type, dtype, path)
    assert used == 3, f"{what}: the decode kernels did not run (path {used})"
    assert candle_moe.device_error_bits(0) == 0
    got = oracle.to_f32(from_torch(out, dtype), dtype)
    ref, slack = oracle_ref(case, act, moe_type, dtype)
    check_close(got, ref, rel_tol(dtype), what, slack)
    return out


CASES = [
    # name, dtype, moe_type, act, T, H, I, E, k, bias
    ("c4-qwen3-bf16-T8", "bf16", 0, 0, 8, 4096, 1536, 8, 2, 0.0),
    ("c4-qwen3-f16-T8", "f16", 0, 0, 8, 4096, 1536, 8, 2, 0.0),
    ("c4-qwen3-bf16-T64", "bf16", 0, 0, 64, 4096, 1536, 8, 2, 0.0),
    ("c3-nomic-bf16-T64", "bf16", 1, 1, 64, 768, 3072, 8, 2, 0.0),
    ("c5-qwen3-bf16-T8", "bf16", 0, 0, 8, 2048, 768, 128, 8, 0.5),
    ("qwen3-bf16-T1", "bf16", 0, 0, 1, 512, 256, 8, 2, 0.0),
    ("qwen3-f16-T16-k1-relu", "f16", 0, 2, 16, 256, 384, 16, 1, 0.0),
    ("nomic-f16-T17-silu", "f16", 1, 0, 17, 384, 640, 16, 4, 0.0),
    ("nomic-bf16-T33-relu", "bf16", 1, 2, 33, 256, 256, 4, 1, 0.0),
]


@pytest.mark.parametrize("name,dtype,moe_type,act,T,H,I,E,k,bias", CASES)
def test_decode_kernels_vs_oracle_and_grouped_gemms(name, dtype, moe_type, act, T, H, I, E, k,
                                                    bias):
    case = moe_case(11 + T + k, T=T, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype=dtype,
                    bias_std=bias, renormalize=(moe_type == 0))
    a = _check(case, E, k, act, moe_type, dtype, name)
    b = _check(case, E, k, act, moe_type, dtype, name + " (again)")
    assert torch.equal(a, b), "decode kernels are not deterministic"
    grouped, used = _run(case, E, k, act, moe_type, dtype, GROUPED)
    assert used == 2
    check_close(oracle.to_f32(from_torch(a, dtype), dtype),
                oracle.to_f32(from_torch(grouped, dtype), dtype), rel_tol(dtype),
                name + " vs grouped GEMMs",
                slack=oracle_ref(case, act, moe_type, dtype)[1])


def test_decode_experts_with_more_rows_than_a_chunk():
    """All 16 tokens pick expert 3 in both slots: 32 rows of one expert, two 16-row chunks, each
    chunk a separate unit whose pieces are cut between CTAs."""
    T, H, I, E, k = 16, 512, 384, 8, 2
    case = moe_case(3, T=T, H=H, I=I, E=E, k=k, moe_type=0, dtype="bf16", renormalize=True)
    case["idx"][:] = 3
    _check(case, E, k, 0, 0, "bf16", "one expert, two chunks")
    case["idx"][:, 1] = 5
    case["idx"][::2, 0] = 5
    _check(case, E, k, 0, 0, "bf16", "two experts, uneven")


def test_decode_invalid_ids_and_no_routed_rows():
    T, H, I, E, k = 12, 256, 256, 8, 2
    case = moe_case(4, T=T, H=H, I=I, E=E, k=k, moe_type=1, dtype="bf16")
    case["idx"][::3, 1] = 8   # ids >= num_experts are skipped
    case["idx"][5, :] = 9     # a token with no valid slot: its output row is zero
    out = _check(case, E, k, 1, 1, "bf16", "invalid ids")
    assert not out[5].any()
    case["idx"][:] = 8        # nothing routed at all: the whole output is zero
    out, used = _run(case, E, k, 1, 1, "bf16", FORCE_DECODE)
    assert used == 3 and not out.any()


def test_decode_forced_on_a_prefill_sized_call():
    """GEMM path 6 runs the decode kernels at any size: 300 tokens x top-4 over 16 experts, many
    64-row chunks per expert and many more units than SMs."""
    T, H, I, E, k = 300, 256, 384, 16, 4
    case = moe_case(5, T=T, H=H, I=I, E=E, k=k, moe_type=0, dtype="bf16", renormalize=True)
    _check(case, E, k, 0, 0, "bf16", "forced decode T=300", path=FORCE_DECODE)


def test_decode_with_few_sms():
    """An SM reserve leaves the stream-K split fewer CTAs: same output within the tolerance."""
    T, H, I, E, k = 8, 1024, 512, 8, 2
    case = moe_case(6, T=T, H=H, I=I, E=E, k=k, moe_type=0, dtype="bf16", renormalize=True)
    ref, _ = _run(case, E, k, 0, 0, "bf16", FORCE_DECODE)
    prev = candle_moe.set_sm_reserve(128)
    try:
        got = _check(case, E, k, 0, 0, "bf16", "20 SMs")
    finally:
        candle_moe.set_sm_reserve(prev)
    # the split (and so the f32 summation order of cut units) depends on the grid: compare at
    # the tolerance, not bit for bit
    check_close(oracle.to_f32(from_torch(got, "bf16"), "bf16"),
                oracle.to_f32(from_torch(ref, "bf16"), "bf16"), 1e-2, "few SMs vs all SMs",
                slack=oracle_ref(case, 0, 0, "bf16")[1])


@pytest.mark.parametrize("T,expect", [(1, 3), (8, 3), (32, 3), (33, 2), (64, 2)])
def test_automatic_path_takes_the_decode_kernels_up_to_32_tokens(T, expect):
    case = moe_case(7, T=T, H=256, I=256, E=8, k=2, moe_type=0, dtype="bf16", renormalize=True)
    _, used = _run(case, 8, 2, 0, 0, "bf16", DECODE)
    assert used == expect
