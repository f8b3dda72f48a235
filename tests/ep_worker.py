"""Worker bodies of the expert-parallel tests (spawned ranks)."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist

import oracle
from moe_testlib import moe_case


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class CpuOracleOps:
    """CPU stand-ins for the compute steps (test infrastructure): the oracle's route preparation
    and MoE, torch indexing for row movement."""

    @staticmethod
    def route_prep(dest, w, groups):
        off, st, sw, sf = oracle.route_prep(dest.numpy().astype(np.uint32), w.numpy(), groups)
        n = dest.numel()  # padded to T*k like the CUDA op (entries past off[groups] unused)
        pad = lambda a, v: np.concatenate([a, np.full(n - len(a), v, a.dtype)])  # noqa: E731
        return (torch.from_numpy(off), torch.from_numpy(pad(st, 0)), torch.from_numpy(pad(sw, 0)),
                torch.from_numpy(pad(sf, 0)))

    @staticmethod
    def gather_rows(x, index):
        return x.index_select(0, index.long())

    @staticmethod
    def local_experts(x, gate, up, down, w, e, num_local, k, activation, moe_type):
        if x.shape[0] == 0:
            return torch.zeros_like(x)
        out = oracle.moe_forward(x.numpy(), gate.numpy(), up.numpy(),
                                 None if down is None else down.numpy(), w.numpy(),
                                 e.numpy().astype(np.uint32), activation=activation,
                                 moe_type=moe_type, dtype="f32")
        return torch.from_numpy(out)

    @staticmethod
    def combine_rows(rows, flat, num_tokens, k):
        out = torch.zeros((num_tokens, rows.shape[1]), dtype=torch.float32)
        slots = torch.full((num_tokens * k,), -1, dtype=torch.int64)
        slots[flat.long()] = torch.arange(rows.shape[0])
        for j in range(k):  # slot order
            r = slots.view(num_tokens, k)[:, j]
            m = r >= 0
            out[m] += rows[r[m]]
        return out


def cpu_rank(rank, world, port, T, H, I, E, k, moe_type, result_q):
    import expert_parallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = moe_case(17, T=T * world, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype="f32",
                        wstd=0.1)
        case["idx"][::11, -1] = E  # an out-of-range id: skipped everywhere
        lo, hi = rank * T, (rank + 1) * T
        e0, e1 = expert_parallel.expert_range(E, world, rank)
        layer = expert_parallel.ExpertParallelMoE(E, k, 0, ops=CpuOracleOps(), chunks=3)
        out = layer.forward(torch.from_numpy(case["x"][lo:hi].copy()),
                            torch.from_numpy(case["gate"][e0:e1].copy()),
                            torch.from_numpy(case["up"][e0:e1].copy()),
                            None if case["down"] is None else torch.from_numpy(case["down"][e0:e1].copy()),
                            torch.from_numpy(case["w"][lo:hi].copy()),
                            torch.from_numpy(case["idx"][lo:hi].copy()), moe_type)
        ref = oracle.moe_forward(case["x"][lo:hi].copy(), case["gate"], case["up"], case["down"],
                                 case["w"][lo:hi].copy(), case["idx"][lo:hi].copy(), activation=0,
                                 moe_type=moe_type, dtype="f32")
        scale = float(np.sqrt(np.mean(ref * ref)))
        stats = {k_: int(v) for k_, v in layer.last_stats.items()}
        result_q.put((rank, float(np.abs(out.numpy() - ref).max()) / scale, stats))
    finally:
        dist.destroy_process_group()


def gpu_rank(rank, world, port, T, H, I, E, k, moe_type, dtype, result_q):
    import candle_moe
    import expert_parallel
    from moe_testlib import to_torch
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        case = moe_case(23, T=T * world, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype=dtype,
                        bias_std=0.5, renormalize=True)
        lo, hi = rank * T, (rank + 1) * T
        e0, e1 = expert_parallel.expert_range(E, world, rank)
        x = to_torch(case["x"], dtype)
        G, U = to_torch(case["gate"], dtype), to_torch(case["up"], dtype)
        D = None if case["down"] is None else to_torch(case["down"], dtype)
        w = torch.from_numpy(case["w"]).cuda()
        idx = torch.from_numpy(case["idx"]).cuda()
        layer = expert_parallel.ExpertParallelMoE(E, k, 0)
        out = layer.forward(x[lo:hi].contiguous(), G[e0:e1].contiguous(), U[e0:e1].contiguous(),
                            None if D is None else D[e0:e1].contiguous(), w[lo:hi].contiguous(),
                            idx[lo:hi].contiguous(), moe_type)
        ref = candle_moe.FusedMoE(E, k).forward(x[lo:hi].contiguous(), G, U, D,
                                                w[lo:hi].contiguous(), idx[lo:hi].contiguous(),
                                                moe_type)
        torch.cuda.synchronize()
        o, r = out.float(), ref.float()
        rms = float(r.pow(2).mean().sqrt())
        ok = bool(((o - r).abs() <= 1e-2 * r.abs() + 1e-2 * rms).all())
        diff = float((o - r).abs().max()) / rms
        stats = {k_: int(v) for k_, v in layer.last_stats.items()}
        result_q.put((rank, ok, diff, stats))
    finally:
        dist.destroy_process_group()
