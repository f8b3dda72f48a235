"""R1 router on the GPU vs the oracle (kernels/topk_softmax.cu:136-266 restated): indices
bit-exact (rows the oracle marks as near-ties excepted), token_expert_indices exact, weights
within 1e-6."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle

pytestmark = pytest.mark.gpu

W_TOL = 1e-6


def _check(logits, k, renorm=False):
    w_ref, i_ref, s_ref, tie = oracle.topk_softmax(logits, k, renormalize=renorm)
    w, i, s = candle_moe.topk_softmax(torch.from_numpy(logits).cuda(), k, renormalize=renorm)
    w, i, s = w.cpu().numpy(), i.cpu().numpy(), s.cpu().numpy()
    ok = ~tie
    assert np.array_equal(i[ok], i_ref[ok]), np.argwhere(i[ok] != i_ref[ok])[:5]
    # rows decided between values within 8 ulps may legitimately differ (exp() differs between
    # libm and the GPU); they must stay rare
    assert tie.sum() <= max(2, logits.shape[0] // 100), int(tie.sum())
    assert np.array_equal(s, s_ref)
    assert np.abs(w[ok] - w_ref[ok]).max(initial=0) <= W_TOL
    return int(tie.sum())


@pytest.mark.parametrize("E", [1, 2, 4, 8, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_router_all_expert_counts(E, k):
    if k > E:
        pytest.skip("k > E covered separately")
    _check(oracle.randn(E * 10 + k, (1000, E)), k)


@pytest.mark.parametrize("T", [1, 3, 17, 512, 8192, 32768])
def test_router_token_counts(T):
    _check(oracle.randn(T, (T, 8)), 2)


def test_router_c5_shape_with_bias_and_renormalisation():
    logits = oracle.randn(50, (65536, 128)) + oracle.randn(51, (128,), std=0.5)[None, :]
    _check(np.ascontiguousarray(logits, np.float32), 8, renorm=True)


def test_router_k_larger_than_e():
    _check(oracle.randn(7, (64, 2)), 3)


def test_drop_in_apply_topk_softmax_inplace_uint32():
    """The reference's own router test shape (tests/topk_softmax_tests.rs:19-58): T=8, E=4, k=2,
    weights compared after rounding to 3 decimals, indices exactly."""
    logits = torch.from_numpy(oracle.randn(1, (8, 4))).cuda()
    w = torch.zeros(8, 2, device="cuda")
    idx = torch.zeros(8, 2, dtype=torch.uint32, device="cuda")
    src = torch.zeros(8, 2, dtype=torch.uint32, device="cuda")
    candle_moe.apply_topk_softmax_inplace(logits, w, idx, src)
    p = torch.softmax(logits, -1)  # f32, as candle's softmax_last_dim in the reference test
    v, i = torch.topk(p, 2)
    # the reference test rounds both to 3 decimals; a 1-ulp difference can straddle a rounding
    # boundary, so compare the unrounded values at f32 resolution instead
    assert np.abs(w.cpu().numpy() - v.cpu().numpy()).max() <= 1e-6
    assert np.array_equal(idx.cpu().numpy().astype(np.int64), i.cpu().numpy())
    assert np.array_equal(src.cpu().numpy().astype(np.int64),
                          np.arange(2)[None, :] * 8 + np.arange(8)[:, None])


def test_router_rejects_unsupported_expert_count():
    with pytest.raises(candle_moe.MoeError):
        candle_moe.topk_softmax(torch.zeros(4, 6, device="cuda"), 2)


def test_router_is_deterministic():
    x = torch.from_numpy(oracle.randn(3, (4096, 64))).cuda()
    a = candle_moe.topk_softmax(x, 4)
    b = candle_moe.topk_softmax(x, 4)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
