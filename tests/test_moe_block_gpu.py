"""SparseMoeBlock: the layer a model calls (router Linear + softmax top-k + experts, README.md:61-97),
built from the fused router projection and the fused MoE, with an optional (gated) shared expert
as in Qwen2-MoE.  Checked against the CPU oracle composed the same way: the oracle router on the
block's own router logits, the oracle MoE for the routed and the shared experts, summed."""
import numpy as np
import pytest
import torch

import candle_moe
import oracle
from moe_testlib import check_close, from_torch, to_torch, ulp

pytestmark = pytest.mark.gpu


def _w(shape, seed, std, dtype):
    return oracle.randn(seed, shape, std=std, dtype=dtype)


@pytest.mark.parametrize("T,H,I,E,k,moe_type,shared,gated", [
    (300, 512, 256, 16, 4, 0, False, False),
    (200, 256, 384, 8, 2, 0, True, True),
    (8, 512, 256, 16, 2, 0, True, False),     # decode-sized: the decode kernels
    (150, 384, 256, 8, 2, 1, True, True),     # Nomic experts
])
def test_sparse_moe_block_vs_oracle(T, H, I, E, k, moe_type, shared, gated):
    dt = "bf16"
    x = _w((T, H), 1, 1.0, dt)
    wr = _w((E, H), 2, 0.05, dt)
    g, u = _w((E, H, I), 3, 0.02, dt), _w((E, H, I), 4, 0.02, dt)
    d = _w((E, I, H), 5, 0.02, dt) if moe_type == 0 else None
    Is = 256
    sg, su = _w((1, H, Is), 6, 0.02, dt), _w((1, H, Is), 7, 0.02, dt)
    sd = _w((1, Is, H), 8, 0.02, dt) if moe_type == 0 else None
    seg = _w((1, H), 9, 0.05, dt)
    tt = lambda a: None if a is None else to_torch(a, dt)  # noqa: E731
    block = candle_moe.SparseMoeBlock(
        tt(wr), tt(g), tt(u), tt(d), k, norm_topk_prob=(moe_type == 0),
        shared_gate=tt(sg) if shared else None, shared_up=tt(su) if shared else None,
        shared_down=tt(sd) if shared else None, shared_expert_gate=tt(seg) if gated else None)
    out, logits = block.forward(tt(x), return_router_logits=True)
    torch.cuda.synchronize()
    got = oracle.to_f32(from_torch(out, dt), dt)
    w, idx, _, _ = oracle.topk_softmax(logits.cpu().numpy(), k, renormalize=(moe_type == 0))
    ref, mc = oracle.moe_forward(x, g, u, d, w, idx, activation=0, moe_type=moe_type, dtype=dt,
                                 with_max_contrib=True)
    slack = ulp(mc, dt)
    if shared:
        xf = oracle.to_f32(x, dt).astype(np.float64)
        if gated:
            z = xf @ oracle.to_f32(seg, dt).astype(np.float64).T
            sw = (1.0 / (1.0 + np.exp(-z))).astype(np.float32)
        else:
            sw = np.ones((T, 1), np.float32)
        sref, smc = oracle.moe_forward(x, sg, su, sd, sw, np.zeros((T, 1), np.int32),
                                       activation=0, moe_type=moe_type, dtype=dt,
                                       with_max_contrib=True)
        # the block rounds the routed and the shared outputs to bf16 before adding them
        ref = oracle.to_f32(oracle.from_f32(ref, dt), dt) + oracle.to_f32(oracle.from_f32(sref, dt), dt)
        slack = slack + ulp(smc, dt) + ulp(ref, dt)
    check_close(got, ref, 1e-2, f"moe block T{T} type{moe_type} shared{shared}", slack)
