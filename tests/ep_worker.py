"""Worker bodies of the expert-parallel tests (spawned ranks)."""
import ctypes
import mmap
import os
import socket
import time
import uuid

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
    and MoE, torch indexing for row movement and bookkeeping."""

    @staticmethod
    def dest_groups(idx, num_experts, num_ranks, tokens_per_chunk, num_chunks):
        T, k = idx.shape
        El = num_experts // num_ranks
        g = torch.full((T, num_ranks), 0x7FFFFFFF, dtype=torch.int32)  # no group
        asg = torch.zeros((num_chunks, num_ranks), dtype=torch.int64)
        for t in range(T):
            for j in range(k):
                e = int(idx[t, j])
                if 0 <= e < num_experts:
                    d = e // El
                    g[t, d] = (t // tokens_per_chunk) * num_ranks + d
                    asg[t // tokens_per_chunk, d] += 1
        return g, asg

    @staticmethod
    def pack(x, pair_token, pair_flat, idx, w, num_experts, num_ranks, num_pairs_device=None):
        El = num_experts // num_ranks
        k = idx.shape[1]
        U = pair_token.numel() if num_pairs_device is None else int(num_pairs_device[0])
        pair_token, pair_flat = pair_token[:U], pair_flat[:U]
        rows = x[pair_token.long()].clone()
        meta = torch.zeros((U, 2 * k), dtype=torch.int32)
        meta[:, :k] = El
        count = torch.zeros((U,), dtype=torch.int32)
        for r in range(U):
            t, d = int(pair_token[r]), int(pair_flat[r]) % num_ranks
            for j in range(k):
                e = int(idx[t, j])
                if 0 <= e < num_experts and e // El == d:
                    meta[r, j] = e % El
                    meta[r, k + j] = w[t, j:j + 1].view(torch.int32)[0]
                    count[r] += 1
        return rows, meta, count

    @staticmethod
    def entry_flat(pair_token, pair_flat, pair_start, idx, num_experts, num_ranks, n):
        El = num_experts // num_ranks
        k = idx.shape[1]
        flat = torch.zeros((n,), dtype=torch.int32)
        for r in range(pair_token.numel()):
            t, d = int(pair_token[r]), int(pair_flat[r]) % num_ranks
            pos = int(pair_start[r])
            for j in range(k):
                e = int(idx[t, j])
                if 0 <= e < num_experts and e // El == d:
                    flat[pos] = t * k + j
                    pos += 1
        return flat

    @staticmethod
    def segment_sum(rows, start):
        out = torch.zeros((start.numel() - 1, rows.shape[1]), dtype=torch.float32)
        for r in range(start.numel() - 1):
            for i in range(int(start[r]), int(start[r + 1])):
                out[r] += rows[i]
        return out

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
    def local_experts_scatter(x, gate, up, down, w, e, out_row, out, num_local, activation,
                              moe_type):
        k = e.shape[1]
        rows, slots = np.nonzero(e.numpy() < num_local)
        if len(rows) == 0:
            return out
        res = oracle.moe_forward(x.numpy()[rows], gate.numpy(), up.numpy(),
                                 None if down is None else down.numpy(),
                                 np.ascontiguousarray(w.numpy()[rows, slots][:, None]),
                                 np.ascontiguousarray(e.numpy()[rows, slots][:, None]).astype(np.uint32),
                                 activation=activation, moe_type=moe_type, dtype="f32")
        out[torch.from_numpy(out_row.numpy()[rows * k + slots]).long()] = torch.from_numpy(res)
        return out

    @staticmethod
    def set_sm_reserve(sms):
        return 0

    # ---- landing buffers in host shared memory: each landing buffer is a file in /dev/shm that
    # every rank maps; copies are memmoves, flags 32-bit stores and polls (x86 keeps the order)
    _maps = {}

    @classmethod
    def _map(cls, path, nbytes, owner):
        with open(path, "r+b") as f:
            mm = mmap.mmap(f.fileno(), nbytes)
        c = ctypes.c_char.from_buffer(mm)
        addr = ctypes.addressof(c)
        del c
        cls._maps[addr] = (mm, path, owner)
        return addr

    @classmethod
    def peer_alloc(cls, nbytes, device):
        path = f"/dev/shm/cmoe_ep_test_{os.getpid()}_{uuid.uuid4().hex[:16]}"
        with open(path, "wb") as f:
            f.truncate(nbytes)
        addr = cls._map(path, nbytes, True)
        return addr, path.encode().ljust(64, b"\0")

    @classmethod
    def peer_open(cls, handle, device):
        path = handle.rstrip(b"\0").decode()
        return cls._map(path, os.path.getsize(path), False)

    @classmethod
    def peer_close(cls, addr, device):
        mm, _, _ = cls._maps.pop(addr)
        mm.close()

    @classmethod
    def peer_free(cls, addr, device):
        mm, path, _ = cls._maps.pop(addr)
        try:
            mm.close()
        except BufferError:  # a tensor view is still alive; the mapping goes with it
            pass
        os.unlink(path)

    @classmethod
    def device_bytes(cls, addr, nbytes, device):
        return torch.frombuffer(cls._maps[addr][0], dtype=torch.uint8, count=nbytes)

    @staticmethod
    def copy_async(dst, src, nbytes, stream):
        ctypes.memmove(dst, src, nbytes)

    @staticmethod
    def peer_signal(flag_addrs, value, stream):
        for a in flag_addrs:
            ctypes.c_uint32.from_address(a).value = value & 0xFFFFFFFF

    @staticmethod
    def peer_wait(flags, count, value, timeout_s, stream):
        t0 = time.monotonic()
        for i in range(count):
            f = ctypes.c_uint32.from_address(flags + 4 * i)
            while ((f.value - value) & 0xFFFFFFFF) >= 0x80000000:
                if time.monotonic() - t0 > timeout_s:
                    raise TimeoutError(f"flag {i} never reached {value}")
                time.sleep(0.0002)

    @classmethod
    def push_pairs(cls, x, pair_token, pair_flat, off, chunk, idx, w, num_experts, num_ranks,
                   rows_to, meta_to, stream, blocks):
        G = num_ranks
        p0, p1 = int(off[chunk * G]), int(off[chunk * G + G])
        rows, meta, _ = cls.pack(x, pair_token[p0:p1], pair_flat[p0:p1], idx, w, num_experts, G)
        rb, mb = rows.shape[1] * rows.element_size(), meta.shape[1] * 4
        for i in range(p1 - p0):
            d = int(pair_flat[p0 + i]) % G
            pos = p0 + i - int(off[chunk * G + d])
            ctypes.memmove(rows_to[d] + pos * rb, rows[i].data_ptr(), rb)
            ctypes.memmove(meta_to[d] + pos * mb, meta[i].data_ptr(), mb)

    @classmethod
    def segment_sum_push(cls, rows, start, dst, first, stream, blocks):
        y = cls.segment_sum(rows, start).to(rows.dtype).contiguous()
        rb = y.shape[1] * y.element_size()
        for s in range(len(dst)):
            for r in range(first[s], first[s + 1]):
                ctypes.memmove(dst[s] + (r - first[s]) * rb, y[r].data_ptr(), rb)

    @staticmethod
    def num_sms(device):
        return 1

    @staticmethod
    def host_counts(work, gathered):
        work.wait()
        return torch.stack(gathered).numpy()

    @staticmethod
    def new_stream(device):
        return None

    @staticmethod
    def current_stream(device):
        return None

    @staticmethod
    def record(stream):
        return None

    @staticmethod
    def wait(stream, event):
        pass

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


def cpu_rank(rank, world, port, T, H, I, E, k, moe_type, result_q, mode="exact",
             transport="collective", sizes=None, chunks=3, groups=None, placement=None):
    """One CPU rank: forward the rank's tokens (the first n of its T for each n in `sizes`, in
    order, through one layer) and report the worst error against the single-process oracle."""
    import expert_parallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = moe_case(17, T=T * world, H=H, I=I, E=E, k=k, moe_type=moe_type, dtype="f32",
                        wstd=0.1)
        case["idx"][::11, -1] = E  # an out-of-range id: skipped everywhere
        e0, e1 = expert_parallel.expert_range(E, world, rank)
        mine = list(range(e0, e1))
        expert_parallel._Landing.SLACK_ROWS = 0  # let a larger second forward grow the buffers
        layer = expert_parallel.ExpertParallelMoE(E, k, 0, ops=CpuOracleOps(), chunks=chunks,
                                                  mode=mode, transport=transport,
                                                  compute_groups=groups)
        if placement is not None:
            layer.set_placement(placement)
            mine = expert_parallel.local_experts(placement, world, rank)
        worst = 0.0
        for n in sizes or [T]:
            lo, hi = rank * T, rank * T + n
            out = layer.forward(torch.from_numpy(case["x"][lo:hi].copy()),
                                torch.from_numpy(case["gate"][mine].copy()),
                                torch.from_numpy(case["up"][mine].copy()),
                                None if case["down"] is None else
                                torch.from_numpy(case["down"][mine].copy()),
                                torch.from_numpy(case["w"][lo:hi].copy()),
                                torch.from_numpy(case["idx"][lo:hi].copy()), moe_type)
            ref = oracle.moe_forward(case["x"][lo:hi].copy(), case["gate"], case["up"],
                                     case["down"], case["w"][lo:hi].copy(),
                                     case["idx"][lo:hi].copy(), activation=0,
                                     moe_type=moe_type, dtype="f32")
            scale = float(np.sqrt(np.mean(ref * ref)))
            worst = max(worst, float(np.abs(out.numpy() - ref).max()) / scale)
        stats = {k_: int(v) for k_, v in layer.last_stats.items()}
        layer.close()
        result_q.put((rank, worst, stats))
    finally:
        dist.destroy_process_group()


def gpu_rank(rank, world, port, T, H, I, E, k, moe_type, dtype, result_q, mode="exact",
             transport="auto", balance=False):
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
        layer = expert_parallel.ExpertParallelMoE(E, k, 0, mode=mode, transport=transport)
        mine = torch.arange(e0, e1, device="cuda")
        if balance:
            # placement from the expert loads of all ranks' tokens (the biased router's)
            loads = torch.bincount(idx.long().flatten().clamp(max=E), minlength=E + 1)[:E]
            slot = expert_parallel.balanced_placement(loads.tolist(), world)
            layer.set_placement(slot)
            mine = torch.tensor(expert_parallel.local_experts(slot, world, rank), device="cuda")
        Gl, Ul = G[mine].contiguous(), U[mine].contiguous()
        Dl = None if D is None else D[mine].contiguous()
        for _ in range(2):  # the second forward reuses the landing buffers and flag epochs
            out = layer.forward(x[lo:hi].contiguous(), Gl, Ul, Dl,
                                w[lo:hi].contiguous(), idx[lo:hi].contiguous(), moe_type)
        ref = candle_moe.FusedMoE(E, k).forward(x[lo:hi].contiguous(), G, U, D,
                                                w[lo:hi].contiguous(), idx[lo:hi].contiguous(),
                                                moe_type)
        torch.cuda.synchronize()
        o, r_ = out.float(), ref.float()
        rms = float(r_.pow(2).mean().sqrt())
        if mode == "exact":
            same = bool(torch.equal(out, ref))
        else:
            same = bool(((o - r_).abs() <= 1e-2 * r_.abs() + 1e-2 * rms).all())
        diff = float((o - r_).abs().max()) / rms
        stats = {k_: int(v) for k_, v in layer.last_stats.items()}
        stats["error_bits"] = candle_moe.device_error_bits(rank)
        layer.check_errors()  # raises if an arrival wait ran out
        layer.close()
        result_q.put((rank, same and stats["error_bits"] == 0, diff, stats))
    finally:
        dist.destroy_process_group()


class DroppingOps(CpuOracleOps):
    """CPU ops whose rank `drop_rank` goes silent after its first arrival signal (its later
    signals are lost, as when a peer stops), for the failure-detection test.  One lost signal
    followed by a later one is not a failure: a later epoch implies the earlier chunks landed."""
    drop_rank = 1
    rank = 0
    signals = 0

    @classmethod
    def peer_signal(cls, flag_addrs, value, stream):
        cls.signals += 1
        if cls.rank == cls.drop_rank and cls.signals > 1:
            return  # lost
        CpuOracleOps.peer_signal(flag_addrs, value, stream)


def cpu_rank_dropped_signal(rank, world, port, transport, result_q):
    """Rank 1's arrival signals stop after its first; every rank must stop with a timeout of its
    arrival wait (not hang), then release its buffers without a collective step."""
    import time as _time
    import expert_parallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    T, H, I, E, k = 24, 16, 32, 8, 3
    case = moe_case(31, T=T * world, H=H, I=I, E=E, k=k, moe_type=0, dtype="f32", wstd=0.1)
    e0, e1 = expert_parallel.expert_range(E, world, rank)
    DroppingOps.rank = rank
    layer = expert_parallel.ExpertParallelMoE(E, k, 0, ops=DroppingOps(), chunks=3,
                                              transport=transport, wait_timeout_s=1.0)
    lo, hi = rank * T, (rank + 1) * T
    t0 = _time.monotonic()
    outcome = "finished"
    try:
        layer.forward(torch.from_numpy(case["x"][lo:hi].copy()),
                      torch.from_numpy(case["gate"][e0:e1].copy()),
                      torch.from_numpy(case["up"][e0:e1].copy()),
                      torch.from_numpy(case["down"][e0:e1].copy()),
                      torch.from_numpy(case["w"][lo:hi].copy()),
                      torch.from_numpy(case["idx"][lo:hi].copy()), 0)
    except TimeoutError as exc:
        outcome = f"timeout: {exc}"
    finally:
        layer.abandon()
    result_q.put((rank, outcome, _time.monotonic() - t0))
    dist.destroy_process_group()
