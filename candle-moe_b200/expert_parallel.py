"""Expert-parallel MoE layer over NCCL (BASELINE config 5 on 2/4/8 GPUs).

The reference crate has no multi-GPU code; this is the expert-parallel layout its north star asks
for.  With G ranks, rank r owns experts [r*E/G, (r+1)*E/G) and its own tokens.  One forward:

 1. plan: route preparation over (chunk, destination rank) groups, destination = expert //
    (E/G), buckets every (token, slot) row of the local tokens (stable, so rows stay in (token,
    slot) order inside a bucket); rows of one token bound for one rank collapse into one
    "unique" row that carries k slots of (local expert, weight) -- expert ids of other ranks
    become the invalid id E/G there; the token rows are gathered once per (token, rank)
    (moe_gather_rows);
 2. one host synchronisation per forward: the [chunk, rank] row counts, exchanged with one
    all_to_all_single;
 3. per chunk, dispatch rows and slot metadata with all_to_all_single (async on the NCCL stream);
 4. per chunk, run the rank's experts on the received rows as a k-slot fused MoE (invalid slots
    are skipped): one partial output row per received row, the rank's weighted contributions
    summed in slot order in f32 and rounded once;
 5. per chunk, return the partial rows with the reverse all_to_all_single;
 6. combine each token's partial rows in rank order in f32, rounding once (moe_combine_rows).

Dispatch of chunk c+1 and the return of chunk c-1 run on the NCCL stream while chunk c's GEMMs
run on the compute stream.  Compared with the single-GPU path the sum over a token's k slots is
associated per rank (partial sums rounded to the operand type before the final sum); the result
matches it within the bf16 tolerance.  The compute steps are injectable (`ops`) so the exchange
logic can be tested on CPU ranks with gloo; the default ops are the CUDA library's, which have
no CPU fallback.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

import candle_moe


def expert_range(num_experts: int, world: int, rank: int):
    """Experts [start, end) owned by `rank` (E must divide evenly)."""
    if num_experts % world:
        raise ValueError(f"num_experts {num_experts} is not divisible by world size {world}")
    n = num_experts // world
    return rank * n, (rank + 1) * n


class CudaOps:
    """The product's compute steps (CUDA library)."""

    @staticmethod
    def route_prep(groups_of_rows, w, groups):
        return candle_moe.route_prep_ex(groups_of_rows, w, groups)

    @staticmethod
    def gather_rows(x, index):
        return candle_moe.gather_rows(x, index)

    @staticmethod
    def local_experts(x, gate, up, down, w, e, num_local, k, activation, moe_type):
        moe = candle_moe.FusedMoE(num_local, k, candle_moe.Activation(activation))
        return moe.forward(x, gate, up, down, w, e, moe_type)

    @staticmethod
    def combine_rows(rows, flat, num_tokens, k):
        return candle_moe.combine_rows(rows, flat, num_tokens, k)


class ExpertParallelMoE:
    """Expert-parallel counterpart of candle_moe.FusedMoE for one process group."""

    STAGES = ("plan", "exchange", "combine")

    def __init__(self, num_experts: int, num_selected_experts: int,
                 activation=candle_moe.Activation.Silu, group: Optional[dist.ProcessGroup] = None,
                 ops=None, chunks: int = 4):
        self.num_experts = num_experts
        self.k = num_selected_experts
        self.activation = int(activation)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.start, self.end = expert_range(num_experts, self.world, self.rank)
        self.num_local = self.end - self.start
        self.ops = ops or CudaOps()
        self.chunks = max(1, chunks)
        self.last_stats = {}
        self.timing = False          # record CUDA events per stage (benchmark analysis)
        self._events = []

    # ---- benchmark instrumentation -----------------------------------------------------------
    def _mark(self):
        if self.timing:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events.append(e)

    def stage_times(self):
        """Summed milliseconds per stage over the timed forwards (waits for the events)."""
        n = len(self.STAGES) + 1
        tot = {s: 0.0 for s in self.STAGES}
        for i in range(0, len(self._events) - n + 1, n):
            ev = self._events[i:i + n]
            ev[-1].synchronize()
            for j, s in enumerate(self.STAGES):
                tot[s] += ev[j].elapsed_time(ev[j + 1])
        return tot, len(self._events) // n

    # ---- forward -----------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, gate_local: torch.Tensor, up_local: torch.Tensor,
                down_local: Optional[torch.Tensor], routing_weights: torch.Tensor,
                expert_indices: torch.Tensor, moe_type: int) -> torch.Tensor:
        """x [T,H] local tokens; *_local: this rank's experts (gate/up [E/G,H,I], down [E/G,I,H]);
        routing_weights / expert_indices [T,k] with global expert ids.  Returns [T,H]."""
        T, H = x.shape
        k, G, El = self.k, self.world, self.num_local
        C = min(self.chunks, max(T, 1))
        Tc = (T + C - 1) // C
        dev = x.device
        self._mark()

        # 1. plan: bucket (token, slot) rows by (chunk, destination); ids >= E get a group
        #    >= C*G and are skipped by route preparation
        idx = expert_indices.to(torch.int32)
        dest = torch.div(idx, El, rounding_mode="floor")
        chunk_of_token = torch.div(torch.arange(T, device=dev, dtype=torch.int32), Tc,
                                   rounding_mode="floor")
        grp = torch.where(dest < G, chunk_of_token[:, None] * G + dest,
                          torch.full_like(dest, C * G)).to(torch.int32).contiguous()
        off, s_tok, s_w, s_flat = self.ops.route_prep(grp, routing_weights.contiguous(), C * G)
        n_valid = torch.clamp(off[C * G:C * G + 1], min=0)
        # unique (token, destination) rows: first entry of each token within its bucket
        pos = torch.arange(T * k, device=dev)
        valid = pos < n_valid
        flat = torch.where(valid, s_flat[:T * k].long(), torch.zeros_like(pos))
        tok = torch.where(valid, s_tok[:T * k].long(), torch.full_like(pos, -1))
        g_of = torch.where(valid, grp.view(-1)[flat].long(), torch.full_like(pos, -1))
        first = valid.clone()
        first[1:] &= (tok[1:] != tok[:-1]) | (g_of[1:] != g_of[:-1])
        uid = torch.cumsum(first, 0) - 1
        # rows per group without a host round trip (invalid entries count into a spare bin)
        bins = torch.where(valid, g_of, torch.full_like(g_of, C * G))
        u_counts = torch.zeros(C * G + 1, dtype=torch.int64, device=dev)
        u_counts.scatter_add_(0, bins, first.long())
        send_cg = u_counts[:C * G].view(C, G)
        # 2. the one host synchronisation: send counts, the counts peers send here, valid rows
        recv_cg = torch.empty((G, C), dtype=torch.int64, device=dev)     # [G_src, C]
        dist.all_to_all_single(recv_cg, send_cg.t().contiguous(), group=self.group)
        host = torch.cat([send_cg.reshape(-1), recv_cg.reshape(-1), n_valid.long()]).cpu()
        send_cnt = host[:C * G].view(C, G)
        recv_cnt = host[C * G:2 * C * G].view(G, C)
        nv = int(host[-1])
        U = int(send_cnt.sum())
        u_rows = torch.nonzero_static(first, size=U).view(-1)
        u_tok = tok[u_rows]
        u_grp = g_of[u_rows]
        # slot metadata of every unique row: local expert id (El = empty slot) and weight bits
        fv = flat[:nv]
        slot = fv % k
        meta = torch.zeros((U, 2 * k), dtype=torch.int32, device=dev)
        meta[:, :k] = El
        meta[uid[:nv], slot] = torch.remainder(idx.view(-1)[fv], El).to(torch.int32)
        meta[uid[:nv], k + slot] = s_w[:nv].view(torch.int32)
        send_x = self.ops.gather_rows(x, u_tok.to(torch.int32).contiguous())
        self._mark()

        # 3-5. per chunk: dispatch, local experts, return (NCCL async, GEMMs on this stream)
        send_off = [0]
        for c in range(C):
            send_off.append(send_off[-1] + int(send_cnt[c].sum()))
        dispatched = []
        for c in range(C):
            in_splits = send_cnt[c].tolist()
            out_splits = recv_cnt[:, c].tolist()
            R = int(sum(out_splits))
            rx = torch.empty((R, H), dtype=x.dtype, device=dev)
            rm = torch.empty((R, 2 * k), dtype=torch.int32, device=dev)
            sx = send_x[send_off[c]:send_off[c + 1]]
            sm = meta[send_off[c]:send_off[c + 1]]
            h1 = dist.all_to_all_single(rx, sx, out_splits, in_splits, group=self.group,
                                        async_op=True)
            h2 = dist.all_to_all_single(rm, sm, out_splits, in_splits, group=self.group,
                                        async_op=True)
            dispatched.append((rx, rm, h1, h2, in_splits, out_splits))
        back = torch.empty((U, H), dtype=x.dtype, device=dev)
        returned = []
        received = 0
        assignments = torch.zeros((), dtype=torch.int64, device=dev)
        for c, (rx, rm, h1, h2, in_splits, out_splits) in enumerate(dispatched):
            h1.wait()
            h2.wait()
            R = rx.shape[0]
            received += R
            e_loc = rm[:, :k].contiguous()
            w_loc = rm[:, k:].contiguous().view(torch.float32)
            if R:
                y = self.ops.local_experts(rx, gate_local, up_local, down_local, w_loc, e_loc, El,
                                           k, self.activation, moe_type)
            else:
                y = torch.empty((0, H), dtype=x.dtype, device=dev)
            assignments += (e_loc < El).sum()
            h3 = dist.all_to_all_single(back[send_off[c]:send_off[c + 1]], y.contiguous(),
                                        in_splits, out_splits, group=self.group, async_op=True)
            returned.append((h3, y))
        for h3, _ in returned:
            h3.wait()
        self._mark()

        # 6. per token, the partial rows of its destination ranks in rank order
        dest_of_u = torch.remainder(u_grp, G)
        out = self.ops.combine_rows(back, (u_tok * G + dest_of_u).to(torch.int32).contiguous(),
                                    T, G)
        self._mark()
        # assignments_received stays a device tensor: reading it here would synchronise
        self.last_stats = {"unique_rows_sent": U, "rows_received": received, "chunks": C,
                           "assignments_received": assignments}
        return out
