"""P1 route preparation on the GPU vs the oracle (kernels/preprocessing.cuh:5-59 restated):
offsets, max count, sorted token ids and weights bit-exact (the order within an expert is pinned
to ascending flat index)."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle

pytestmark = pytest.mark.gpu


def _run(idx, w, E):
    off, st, sw = candle_moe.route_prep(torch.from_numpy(idx.view(np.int32)).cuda(),
                                        torch.from_numpy(w).cuda(), E)
    torch.cuda.synchronize()
    return off.cpu().numpy(), st.cpu().numpy(), sw.cpu().numpy()


def _check(idx, w, E):
    o_ref, s_ref, w_ref, _ = oracle.route_prep(idx, w, E)
    off, st, sw = _run(idx, w, E)
    n = int(o_ref[E])
    assert np.array_equal(off, o_ref)
    assert np.array_equal(st[:n], s_ref)
    assert np.array_equal(sw[:n].view(np.uint32), w_ref.view(np.uint32))


@pytest.mark.parametrize("T,k,E", [(1, 1, 1), (8, 2, 4), (512, 2, 8), (2048, 2, 8),
                                   (2049, 2, 8), (32768, 2, 8), (65536, 8, 128), (5000, 3, 7),
                                   (4096, 8, 256), (3000, 4, 1024)])
def test_route_prep_random(T, k, E):
    rng = np.random.default_rng(T * 31 + k * 7 + E)
    idx = rng.integers(0, E, size=(T, k)).astype(np.uint32)
    w = rng.standard_normal((T, k)).astype(np.float32)
    _check(idx, w, E)


def test_route_prep_skips_out_of_range_ids():
    rng = np.random.default_rng(5)
    idx = rng.integers(0, 10, size=(9000, 2)).astype(np.uint32)
    idx[::7, 1] = 0xFFFFFFFF
    w = rng.standard_normal((9000, 2)).astype(np.float32)
    _check(idx, w, 8)


@pytest.mark.parametrize("T", [100, 40000])
def test_route_prep_all_rows_on_one_expert(T):
    idx = np.full((T, 2), 5, np.uint32)
    w = np.ones((T, 2), np.float32)
    _check(idx, w, 8)


def test_route_prep_biased_c5_routing():
    logits = oracle.randn(50, (65536, 128)) + oracle.randn(51, (128,), std=0.5)[None, :]
    w, idx, _, _ = oracle.topk_softmax(np.ascontiguousarray(logits, np.float32), 8, True)
    _check(idx.view(np.uint32), w, 128)
