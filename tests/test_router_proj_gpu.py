"""The router's gate projection fused with the softmax + top-k (moe_router_project_topk).

The reference's caller computes the router logits with a Linear over the hidden states and
hands them to apply_topk_softmax_inplace (README.md:67-73).  The fused kernel must give the
picks of that two-step path exactly: on the logits it computed (returned for the check), the
drop-in router (topk_softmax, R1) produces bit-identical indices, token-expert indices and
weights.  The logits themselves are checked against an f32 matmul of the same bf16/f16 inputs,
and the picks against the CPU oracle's router on those logits (indices exact outside near-ties,
weights within 1e-6, the north-star router tolerance)."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle

pytestmark = pytest.mark.gpu

CASES = [
    # T, H, E, k, renorm, dtype, bias
    (512, 768, 8, 2, False, torch.bfloat16, 0.0),      # BASELINE config 2/3 router: Linear 768->8
    (300, 4096, 8, 2, True, torch.float16, 0.0),       # config 4 shape (Qwen3, renormalised)
    (4096, 2048, 128, 8, True, torch.bfloat16, 0.5),   # config 5 shape on 4096 tokens, biased
    (1, 256, 256, 4, False, torch.bfloat16, 0.0),
    (129, 128, 16, 16, True, torch.bfloat16, 0.0),
    (77, 512, 64, 3, False, torch.float16, 0.0),
    (200, 64, 1, 1, False, torch.bfloat16, 0.0),
    (200, 192, 4, 2, True, torch.bfloat16, 0.0),
    (1000, 1024, 32, 8, False, torch.bfloat16, 0.0),
]


def _inputs(T, H, E, dtype, bias, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(T, H, generator=g, device="cuda").to(dtype)
    w = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(dtype)
    if bias:
        # a per-expert offset of the logits (BASELINE config 5's load imbalance) through an extra
        # hidden feature that is 1 for every token
        x[:, 0] = 1.0
        w[:, 0] = (torch.randn(E, generator=g, device="cuda") * bias).to(dtype)
    return x, w


@pytest.mark.parametrize("T,H,E,k,renorm,dtype,bias", CASES)
def test_fused_projection_equals_the_two_step_router(T, H, E, k, renorm, dtype, bias):
    x, w = _inputs(T, H, E, dtype, bias, T + H + E + k)
    fw, fi, fs, logits = candle_moe.router_project_topk(x, w, k, renormalize=renorm,
                                                        return_logits=True)
    torch.cuda.synchronize()
    assert candle_moe.device_error_bits(0) == 0
    # the logits: an f32 GEMM of the same inputs
    ref_logits = x.float() @ w.float().t()
    scale = ref_logits.abs().max().item() + 1e-6
    assert (logits - ref_logits).abs().max().item() <= 1e-5 * scale * max(1.0, H / 256)
    # the two-step path on those logits: bit-identical
    rw, ri, rs = candle_moe.topk_softmax(logits, k, renormalize=renorm)
    assert torch.equal(fi, ri)
    assert torch.equal(fs, rs)
    assert torch.equal(fw.view(torch.int32), rw.view(torch.int32))
    # the oracle's router on the same logits
    ow, oi, os_, tie = oracle.topk_softmax(logits.cpu().numpy(), k, renormalize=renorm)
    ok = ~tie
    assert np.array_equal(fi.cpu().numpy()[ok], oi[ok])
    assert np.array_equal(fs.cpu().numpy(), os_)
    assert np.abs(fw.cpu().numpy()[ok] - ow[ok]).max(initial=0.0) <= 1e-6


def test_fused_projection_without_logits_output_and_errors():
    x, w = _inputs(300, 256, 8, torch.bfloat16, 0.0, 5)
    a = candle_moe.router_project_topk(x, w, 2)
    b = candle_moe.router_project_topk(x, w, 2, return_logits=True)
    for u, v in zip(a, b[:3]):
        assert torch.equal(u, v)
    with pytest.raises(candle_moe.MoeError):
        candle_moe.router_project_topk(x, w, 9)  # k > E
    with pytest.raises(candle_moe.MoeError):
        candle_moe.router_project_topk(x[:, :96].contiguous(), w[:, :96].contiguous(), 2)  # H % 64
