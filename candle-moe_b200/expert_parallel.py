"""Expert-parallel MoE layer over NCCL (BASELINE config 5 on 2/4/8 GPUs).

The reference crate has no multi-GPU code; this is the expert-parallel layout its north star asks
for.  With G ranks, rank r owns experts [r*E/G, (r+1)*E/G) and its own tokens.  One forward:

 1. bucket the local (token, slot) rows by destination rank = expert // (E/G): route preparation
    over G "experts" (stable, so rows stay in ascending (token, slot) order per destination);
 2. gather the token rows of each bucket (moe_gather_rows) with their (local expert, weight);
 3. exchange counts, rows and metadata with all_to_all_single (NCCL over NVLink);
 4. run the rank's experts on the rows it received as a top-1 fused MoE (each received row
    carries exactly one expert): the weighted contribution of each row, rounded to the operand
    type exactly as the single-GPU slot buffer is;
 5. return the contributions with the reverse all_to_all_single;
 6. combine each token's k contributions in slot order in f32 and round once (moe_combine_rows).

The arithmetic per output element is the single-GPU path's (same tile math, same rounding
points, same slot order), so the result equals the single-GPU output.  The compute steps are
injectable (`ops`) so the exchange logic can be tested on CPU ranks with gloo; the default ops
are the CUDA library's, and there is no CPU fallback in them.
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
    def route_prep(dest, w, groups):
        return candle_moe.route_prep_ex(dest, w, groups)

    @staticmethod
    def gather_rows(x, index):
        return candle_moe.gather_rows(x, index)

    @staticmethod
    def local_experts(x, gate, up, down, w, e, num_local, activation, moe_type):
        moe = candle_moe.FusedMoE(num_local, 1, candle_moe.Activation(activation))
        return moe.forward(x, gate, up, down, w, e, moe_type)

    @staticmethod
    def combine_rows(rows, flat, num_tokens, k):
        return candle_moe.combine_rows(rows, flat, num_tokens, k)


class ExpertParallelMoE:
    """Expert-parallel counterpart of candle_moe.FusedMoE for one process group."""

    def __init__(self, num_experts: int, num_selected_experts: int,
                 activation=candle_moe.Activation.Silu, group: Optional[dist.ProcessGroup] = None,
                 ops=None):
        self.num_experts = num_experts
        self.k = num_selected_experts
        self.activation = int(activation)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.start, self.end = expert_range(num_experts, self.world, self.rank)
        self.num_local = self.end - self.start
        self.ops = ops or CudaOps()
        self.last_stats = {}
        self.timing = False          # record CUDA events per stage (benchmark analysis)
        self.stage_ms = {}
        self._events = []

    STAGES = ("bucket", "dispatch", "experts", "return", "combine")

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

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x: torch.Tensor, gate_local: torch.Tensor, up_local: torch.Tensor,
                down_local: Optional[torch.Tensor], routing_weights: torch.Tensor,
                expert_indices: torch.Tensor, moe_type: int) -> torch.Tensor:
        """x [T,H] local tokens; *_local: this rank's experts (gate/up [E/G,H,I], down [E/G,I,H]);
        routing_weights / expert_indices [T,k] with global expert ids.  Returns [T,H]."""
        T, H = x.shape
        k = self.k
        G = self.world
        dev = x.device
        self._mark()
        idx = expert_indices.to(torch.int32)
        dest = torch.div(idx, self.num_local, rounding_mode="floor").to(torch.int32).contiguous()
        # ids >= E land on a destination >= G and are skipped by route preparation
        off, s_tok, s_w, s_flat = self.ops.route_prep(dest, routing_weights.contiguous(), G)
        counts = (off[1:G + 1] - off[:G]).to(torch.int64)
        send_splits = counts.tolist()
        S = int(sum(send_splits))
        s_tok, s_w, s_flat = s_tok[:S], s_w[:S], s_flat[:S]
        send_x = self.ops.gather_rows(x, s_tok)
        local_e = torch.remainder(idx.reshape(-1)[s_flat.long()], self.num_local).to(torch.int32)
        send_meta = torch.stack([local_e, s_w.view(torch.int32)], dim=1).contiguous()
        self._mark()

        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        recv_splits = recv_counts.tolist()
        R = int(sum(recv_splits))
        recv_x = torch.empty((R, H), dtype=x.dtype, device=dev)
        recv_meta = torch.empty((R, 2), dtype=torch.int32, device=dev)
        self._a2a(recv_x, send_x, recv_splits, send_splits)
        self._a2a(recv_meta, send_meta, recv_splits, send_splits)
        self._mark()

        recv_e = recv_meta[:, 0:1].contiguous()
        recv_w = recv_meta[:, 1:2].contiguous().view(torch.float32)
        y = self.ops.local_experts(recv_x, gate_local, up_local, down_local, recv_w, recv_e,
                                   self.num_local, self.activation, moe_type)
        self._mark()
        back = torch.empty((S, H), dtype=x.dtype, device=dev)
        self._a2a(back, y.contiguous(), send_splits, recv_splits)
        self._mark()
        self.last_stats = {"sent_rows": S, "received_rows": R}
        out = self.ops.combine_rows(back, s_flat, T, k)
        self._mark()
        return out
