"""CPU tests of the oracle (test infrastructure) against independent restatements in
numpy / torch, and against the golden fixtures produced by the reference's own kernels."""
import glob
import os

import numpy as np
import pytest
import torch

import oracle
from moe_testlib import check_close, moe_case

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("T,E,k", [(8, 4, 2), (512, 8, 2), (300, 16, 4), (257, 128, 8),
                                   (64, 256, 8), (33, 1, 1), (40, 2, 2), (100, 64, 3)])
def test_router_matches_torch_softmax_topk(T, E, k):
    """kernels/topk_softmax.cu:136-266 vs torch softmax + topk (what tests/topk_softmax_tests.rs
    checks with candle's softmax_last_dim + TopKLastDimOp)."""
    logits = oracle.randn(T * 7 + E, (T, E))
    w, idx, src, tie = oracle.topk_softmax(logits, k)
    p = torch.softmax(torch.from_numpy(logits).double(), -1)
    v, i = torch.topk(p, k, dim=-1)
    ok = ~tie
    assert np.array_equal(idx[ok], i.numpy()[ok])
    assert np.abs(w - v.numpy()).max() < 1e-6
    assert np.array_equal(src, (np.arange(k)[None, :] * T + np.arange(T)[:, None]).astype(np.int32))


def test_router_renormalize_and_ties():
    logits = np.zeros((4, 8), np.float32)
    logits[:, 3] = 1.0
    logits[:, 5] = 1.0  # exact tie: lower index first (topk_softmax.cu:240)
    w, idx, _, tie = oracle.topk_softmax(logits, 3)
    assert (idx[:, 0] == 3).all() and (idx[:, 1] == 5).all() and (idx[:, 2] == 0).all()
    assert not tie.any()  # exact ties resolve identically everywhere
    wr, _, _, _ = oracle.topk_softmax(logits, 3, renormalize=True)
    assert np.allclose(wr.sum(1), 1.0, atol=1e-6)
    assert np.allclose(wr, w / w.sum(1, keepdims=True), atol=1e-7)


def test_router_k_larger_than_e_fills_cleared_values():
    # after every expert is taken the cleared value -10000 wins (topk_softmax.cu:256-264)
    w, idx, _, _ = oracle.topk_softmax(np.array([[0.5, 0.1]], np.float32), 3)
    assert idx[0, 0] == 0 and idx[0, 1] == 1 and idx[0, 2] == 0 and w[0, 2] == -10000.0


@pytest.mark.parametrize("T,k,E", [(16, 2, 8), (1000, 2, 8), (513, 8, 128), (77, 3, 5), (1, 1, 1)])
def test_route_prep_is_a_stable_counting_sort(T, k, E):
    rng = np.random.default_rng(T + k + E)
    idx = rng.integers(0, E + 2, size=(T, k)).astype(np.uint32)  # some ids >= E: skipped
    w = rng.standard_normal((T, k)).astype(np.float32)
    off, st, sw, sf = oracle.route_prep(idx, w, E)
    flat = idx.reshape(-1)
    valid = np.nonzero(flat < E)[0]
    order = valid[np.argsort(flat[valid], kind="stable")]
    assert np.array_equal(sf, order)
    assert np.array_equal(st, (order // k).astype(np.int32))
    assert np.array_equal(sw, w.reshape(-1)[order])
    counts = np.bincount(flat[valid], minlength=E)[:E]
    assert np.array_equal(off[:E], np.concatenate([[0], np.cumsum(counts)[:-1]]))
    assert off[E] == len(valid) and off[E + 1] == (counts.max() if E else 0)


def _torch_naive(case, moe_type, act):
    """tests/moe_tests.rs:124-189: per-expert bincount / nonzero / index_select / MLP /
    index_add, in float64."""
    x = torch.from_numpy(case["x"]).double()
    G = torch.from_numpy(case["gate"]).double()
    U = torch.from_numpy(case["up"]).double()
    D = None if case["down"] is None else torch.from_numpy(case["down"]).double()
    idx = torch.from_numpy(case["idx"].astype(np.int64))
    w = torch.from_numpy(case["w"]).double()
    actf = {0: torch.nn.functional.silu,
            1: lambda v: torch.nn.functional.gelu(v, approximate="tanh"),
            2: torch.relu}[act]
    out = torch.zeros_like(x)
    E = G.shape[0]
    for e in range(E):
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        xs = x[tok]
        if moe_type == 0:
            y = (actf(xs @ G[e]) * (xs @ U[e])) @ D[e]
        else:
            y = actf(xs @ G[e]) @ U[e].T
        out.index_add_(0, tok, y * w[tok, slot][:, None])
    return out.numpy()


@pytest.mark.parametrize("moe_type", [0, 1])
@pytest.mark.parametrize("act", [0, 1, 2])
def test_moe_forward_f32_matches_naive_loop(moe_type, act):
    case = moe_case(3 + act, T=40, H=32, I=64, E=8, k=2, moe_type=moe_type, dtype="f32",
                    wstd=0.2)
    got = oracle.moe_forward(case["x"], case["gate"], case["up"], case["down"], case["w"],
                             case["idx"], activation=act, moe_type=moe_type, dtype="f32")
    check_close(got, _torch_naive(case, moe_type, act), 1e-5, "oracle f32")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_moe_forward_rounding_mode_stays_close(dtype):
    case = moe_case(9, T=24, H=64, I=128, E=4, k=2, moe_type=0, dtype=dtype, wstd=0.1)
    rounded = oracle.moe_forward(case["x"], case["gate"], case["up"], case["down"], case["w"],
                                 case["idx"], activation=0, moe_type=0, dtype=dtype)
    exact = oracle.moe_forward(case["x"], case["gate"], case["up"], case["down"], case["w"],
                               case["idx"], activation=0, moe_type=0, dtype=dtype,
                               round_dtype="f32")
    check_close(rounded, exact, 1e-2, "rounded vs unrounded intermediate")


def test_invalid_expert_ids_contribute_nothing():
    case = moe_case(11, T=10, H=16, I=32, E=4, k=2, moe_type=1, dtype="f32", wstd=0.3)
    idx = case["idx"].copy()
    idx[:, 1] = 4  # == E: skipped by preprocessing.cuh:29
    got = oracle.moe_forward(case["x"], case["gate"], case["up"], None, case["w"], idx,
                             activation=0, moe_type=1, dtype="f32")
    case1 = dict(case, idx=idx[:, :1].copy(), w=case["w"][:, :1].copy())
    ref = oracle.moe_forward(case1["x"], case1["gate"], case1["up"], None, case1["w"],
                             case1["idx"], activation=0, moe_type=1, dtype="f32")
    np.testing.assert_array_equal(got, ref)


def test_randn_is_seeded_and_thread_count_independent():
    a = oracle.randn(5, (1000, 37), nthreads=1)
    b = oracle.randn(5, (1000, 37), nthreads=4)
    assert np.array_equal(a, b)
    assert abs(float(a.mean())) < 0.05 and abs(float(a.std()) - 1) < 0.05
    assert not np.array_equal(a, oracle.randn(6, (1000, 37)))


# ---- golden fixtures produced by the reference's own CUDA kernels (tests/golden/) --------------

def _golden(pattern):
    return sorted(glob.glob(os.path.join(GOLDEN, pattern)))


@pytest.mark.parametrize("path", _golden("router_*.npz") or [None])
def test_oracle_router_matches_reference_fixture(path):
    if path is None:
        pytest.skip("no router fixtures")
    f = np.load(path)
    w, idx, src, tie = oracle.topk_softmax(f["logits"], int(f["k"]))
    ok = ~tie
    assert np.array_equal(idx[ok], f["indices"][ok]), path
    assert np.array_equal(src, f["token_expert_indices"]), path
    assert np.abs(w - f["weights"]).max() <= 1e-6, path


@pytest.mark.parametrize("path", _golden("prep_*.npz") or [None])
def test_oracle_route_prep_matches_reference_fixture(path):
    if path is None:
        pytest.skip("no preprocessing fixtures")
    f = np.load(path)
    E = int(f["E"])
    off, st, sw, _ = oracle.route_prep(f["indices"], f["weights"], E)
    assert np.array_equal(off, f["offsets"]), path
    # the reference orders rows within an expert by atomics: compare per-expert multisets
    for e in range(E):
        lo, hi = off[e], off[e + 1]
        a = sorted(zip(st[lo:hi].tolist(), sw[lo:hi].tolist()))
        b = sorted(zip(f["sorted_token_ids"][lo:hi].tolist(), f["sorted_weights"][lo:hi].tolist()))
        assert a == b, (path, e)


@pytest.mark.parametrize("path", _golden("moe_*.npz") or [None])
def test_oracle_moe_matches_reference_fixture(path):
    if path is None:
        pytest.skip("no MoE fixtures")
    f = np.load(path)
    dtype = str(f["dtype"])
    down = f["down"] if int(f["moe_type"]) == 0 else None
    got = oracle.moe_forward(f["x"], f["gate"], f["up"], down, f["w"], f["idx"],
                             activation=int(f["act"]), moe_type=int(f["moe_type"]), dtype=dtype,
                             round_dtype=str(f["round_dtype"]))
    ref = oracle.to_f32(f["out"], dtype)
    check_close(got, ref, float(f["rtol"]), os.path.basename(path))
