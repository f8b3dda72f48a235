"""moe_route_prep_noalloc: route preparation for callers that cannot allocate device memory
during the step (an allocator that owns all of HBM, a plugin handed only its buffers, a graph
being recorded).  Its scratch is a fixed array built into the library instead of the pool.

Checked through the C ABI against the pool-backed moe_route_prep on two calls in a row (the
second call runs over whatever the first left in the shared array), bit-exact as every
route-preparation test is, plus the size limit.  This file sorts last so that a run stopping at
the first failure has run every other test already."""
import ctypes

import numpy as np
import pytest
import torch

import candle_moe

pytestmark = pytest.mark.gpu

MOE_ERR_WORKSPACE = 4


def _bind():
    lib = candle_moe.lib()
    P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    lib.moe_route_prep_noalloc.argtypes = [P, P, I64, I32, I32, P, P, P, P]
    lib.moe_route_prep_noalloc.restype = ctypes.c_int
    lib.moe_route_prep.argtypes = [P, P, I64, I32, I32, P, P, P, P]
    lib.moe_route_prep.restype = ctypes.c_int
    lib.moe_kernel_launches.restype = ctypes.c_int64
    return lib


def _run(fn, idx, w, E):
    T, k = idx.shape
    off = torch.full((E + 2,), -1, dtype=torch.int32, device="cuda")
    st = torch.full((T * k,), -1, dtype=torch.int32, device="cuda")
    sw = torch.full((T * k,), -1.0, dtype=torch.float32, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    status = fn(p(idx), p(w), T, k, E, p(off), p(st), p(sw),
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return status, off.cpu(), st.cpu(), sw.cpu()


@pytest.mark.parametrize("T,k,E", [(20000, 8, 128), (3000, 2, 8), (1500, 2, 2048), (0, 2, 8)])
def test_noalloc_matches_pool_version_on_two_calls_in_a_row(T, k, E):
    lib = _bind()
    for call in range(2):
        rng = np.random.default_rng(1000 * call + T + E)
        idx = torch.from_numpy(rng.integers(0, E, size=(T, k)).astype(np.int32)).cuda()
        w = torch.from_numpy(rng.standard_normal((T, k)).astype(np.float32)).cuda()
        n0 = lib.moe_kernel_launches()
        s_ref, o_ref, t_ref, w_ref = _run(lib.moe_route_prep, idx, w, E)
        n1 = lib.moe_kernel_launches()
        s_new, o_new, t_new, w_new = _run(lib.moe_route_prep_noalloc, idx, w, E)
        assert s_ref == 0 and s_new == 0
        # the same kernels, counted the same way
        assert lib.moe_kernel_launches() - n1 == n1 - n0
        assert torch.equal(o_new, o_ref)
        n = int(o_ref[E])
        assert torch.equal(t_new[:n], t_ref[:n])
        assert torch.equal(w_new[:n].view(torch.int32), w_ref[:n].view(torch.int32))


def test_noalloc_rejects_requests_beyond_its_scratch():
    lib = _bind()
    # 2 * ceil(300*4096 / 4096) * 2048 = 1,228,800 ints > 524,288
    T, k, E = 4096 * 300, 1, 2048
    idx = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((T, k), dtype=torch.float32, device="cuda")
    status, off, _, _ = _run(lib.moe_route_prep_noalloc, idx, w, E)
    assert status == MOE_ERR_WORKSPACE
    assert bool((off == -1).all())  # nothing was launched


_FIRST_CALL = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import candle_moe
lib = candle_moe.lib()
P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
for f in (lib.moe_route_prep_noalloc, lib.moe_route_prep):
    f.argtypes = [P, P, I64, I32, I32, P, P, P, P]
    f.restype = ctypes.c_int
outs = []
rng = np.random.default_rng(7)
# a single-block request (1000 rows) and a multi-block one (80000 rows) at 256 experts
for T, k, E in ((500, 2, 256), (10000, 8, 256)):
    idx = torch.from_numpy(rng.integers(0, E, size=(T, k)).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.standard_normal((T, k)).astype(np.float32)).cuda()
    res = []
    # the no-allocation entry point first: its own set-up runs before any other entry point
    for f in (lib.moe_route_prep_noalloc, lib.moe_route_prep):
        off = torch.full((E + 2,), -1, dtype=torch.int32, device="cuda")
        st = torch.full((T * k,), -1, dtype=torch.int32, device="cuda")
        sw = torch.full((T * k,), -1.0, dtype=torch.float32, device="cuda")
        p = lambda t: ctypes.c_void_p(t.data_ptr())
        assert f(p(idx), p(w), T, k, E, p(off), p(st), p(sw), None) == 0
        torch.cuda.synchronize()
        res.append((off.cpu(), st.cpu(), sw.cpu()))
    (o1, t1, w1), (o2, t2, w2) = res
    n = int(o2[E])
    assert torch.equal(o1, o2) and torch.equal(t1[:n], t2[:n])
    assert torch.equal(w1[:n].view(torch.int32), w2[:n].view(torch.int32))
print("first-call ok")
"""


def test_noalloc_as_the_first_call_of_a_fresh_process():
    """The entry point's own per-device set-up (symbol address, shared-memory attributes) must
    work when nothing else in the library has run yet."""
    import os
    import subprocess
    import sys
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                       "candle-moe_b200")
    r = subprocess.run([sys.executable, "-c", _FIRST_CALL, pkg], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "first-call ok" in r.stdout
