"""Expert-parallel MoE layer over NCCL (BASELINE config 5 on 2/4/8 GPUs).

The reference crate has no multi-GPU code; this is the expert-parallel layout its north star asks
for.  With G ranks, rank r owns experts [r*E/G, (r+1)*E/G) and its own tokens.  One forward:

 1. plan: a token is sent once to each rank that owns one of its k experts.  moe_ep_dest_groups
    marks the (token, rank) pairs, grouped by (chunk of tokens, rank); route preparation over
    those groups sorts the pairs (stable: token order inside a group); moe_ep_pack gathers each
    pair's token row and its k-slot metadata (local expert id, or E/G for slots owned by other
    ranks, and the routing weight);
 2. one host synchronisation per forward: the [chunk, rank] counts, exchanged with one
    all_to_all_single;
 3. per chunk, dispatch rows and metadata with all_to_all_single (async on the NCCL stream);
 4. per chunk, run the rank's experts on the received rows as a k-slot fused MoE (foreign slots
    are skipped), then return the results with the reverse all_to_all_single:
      "partials" (default): one row per pair, the rank's weighted contributions summed in slot
        order and rounded once -- the fewest bytes back; the origin sums a token's partials in
        rank order (equal to the single-GPU output within the bf16 tolerance);
      "exact": one row per (token, slot) contribution, written straight into the returned
        buffer in pair order (moe_fused_scatter); the origin combines all k in slot order,
        so the output is bit-identical to the single-GPU path;
 5. combine on the origin (moe_combine_rows), f32 accumulation, one rounding.

Dispatch of later chunks and the return of earlier ones run on the NCCL stream while a chunk's
GEMMs run on the compute stream; the GEMMs leave `sm_reserve` SMs to NCCL while the exchange is in
flight (they schedule tiles dynamically, so the reserve costs only those SMs).  The compute steps
are injectable (`ops`) so the exchange logic can be tested on CPU ranks with gloo; the default ops
are the CUDA library's, which have no CPU fallback.
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
    def dest_groups(idx, num_experts, num_ranks, tokens_per_chunk):
        return candle_moe.ep_dest_groups(idx, num_experts, num_ranks, tokens_per_chunk)

    @staticmethod
    def pack(x, pair_token, pair_flat, idx, w, num_experts, num_ranks):
        return candle_moe.ep_pack(x, pair_token, pair_flat, idx, w, num_experts, num_ranks)

    @staticmethod
    def entry_flat(pair_token, pair_flat, pair_start, idx, num_experts, num_ranks, n):
        return candle_moe.ep_entry_flat(pair_token, pair_flat, pair_start, idx, num_experts,
                                        num_ranks, n)

    @staticmethod
    def segment_sum(rows, start):
        return candle_moe.segment_sum_rows(rows, start)

    @staticmethod
    def route_prep(groups_of_rows, w, groups):
        return candle_moe.route_prep_ex(groups_of_rows, w, groups)

    @staticmethod
    def gather_rows(x, index):
        return candle_moe.gather_rows(x, index)

    @staticmethod
    def local_experts_scatter(x, gate, up, down, w, e, out_row, out, num_local, activation,
                              moe_type):
        return candle_moe.fused_moe_scatter(x, gate, up, down, w, e, out_row, out, num_local,
                                            activation, moe_type)

    @staticmethod
    def combine_rows(rows, flat, num_tokens, k):
        return candle_moe.combine_rows(rows, flat, num_tokens, k)

    @staticmethod
    def set_sm_reserve(sms):
        return candle_moe.set_sm_reserve(sms)


class ExpertParallelMoE:
    """Expert-parallel counterpart of candle_moe.FusedMoE for one process group."""

    STAGES = ("plan", "exchange", "combine")

    def __init__(self, num_experts: int, num_selected_experts: int,
                 activation=candle_moe.Activation.Silu, group: Optional[dist.ProcessGroup] = None,
                 ops=None, chunks: int = 4, sm_reserve: int = 24, mode: str = "partials"):
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
        # SMs the expert GEMMs leave to NCCL's kernels while the exchange is in flight: the GEMMs
        # are persistent (one CTA per SM), and without free SMs the collectives would only run
        # between GEMM launches.  The GEMMs take tiles dynamically, so the reserve only costs
        # the SMs themselves.
        self.sm_reserve = sm_reserve
        if mode not in ("partials", "exact"):
            raise ValueError(f"unknown mode {mode!r}")
        self.mode = mode
        self._zeros = {}
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
        k, G, E, El = self.k, self.world, self.num_experts, self.num_local
        C = min(self.chunks, max(T, 1))
        Tc = (T + C - 1) // C
        C = (T + Tc - 1) // Tc if T else 1
        dev = x.device
        exact = self.mode == "exact"
        self._mark()

        # 1. plan: (token, rank) pairs sorted by (chunk, rank, token)
        idx = expert_indices.to(torch.int32).contiguous()
        w = routing_weights.contiguous()
        groups = self.ops.dest_groups(idx, E, G, Tc)
        zw = self._zeros.get(groups.shape)
        if zw is None or zw.device != dev:
            zw = self._zeros[groups.shape] = torch.zeros(groups.shape, dtype=torch.float32,
                                                         device=dev)
        off, p_tok, _, p_flat = self.ops.route_prep(groups, zw, C * G)
        pair_counts = (off[1:C * G + 1] - off[:C * G]).to(torch.int64).view(C, G)
        # (token, slot) entries per (chunk, rank): the expert work each rank will do for us, and in
        # exact mode also the rows that come back
        dst = torch.div(idx, El, rounding_mode="floor").long()
        chunk = torch.div(torch.arange(T, device=dev), Tc, rounding_mode="floor")[:, None]
        g = torch.where(dst < G, chunk * G + dst, torch.full_like(dst, C * G))
        asg = torch.zeros(C * G + 1, dtype=torch.int64, device=dev)
        asg.scatter_add_(0, g.view(-1), torch.ones_like(g.view(-1)))
        asg = asg[:C * G].view(C, G)
        counts = torch.stack([pair_counts, asg if exact else pair_counts, asg], dim=2)
        # 2. the one host synchronisation: counts sent and counts peers send here
        recv_counts = torch.empty((G, C, 3), dtype=torch.int64, device=dev)  # [G_src, C, 3]
        dist.all_to_all_single(recv_counts, counts.permute(1, 0, 2).contiguous(),
                               group=self.group)
        host = torch.cat([counts.reshape(-1), recv_counts.reshape(-1)]).cpu()
        send_rows = host[:3 * C * G].view(C, G, 3)[:, :, 0]
        send_back = host[:3 * C * G].view(C, G, 3)[:, :, 1]
        recv_rows = host[3 * C * G:].view(G, C, 3)[:, :, 0]
        recv_back = host[3 * C * G:].view(G, C, 3)[:, :, 1]
        recv_asg = host[3 * C * G:].view(G, C, 3)[:, :, 2]
        U = int(send_rows.sum())
        n_back = int(send_back.sum())
        p_tok, p_flat = p_tok[:U], p_flat[:U]
        send_x, meta, slot_count = self.ops.pack(x, p_tok, p_flat, idx, w, E, G)
        if exact:
            start = torch.cumsum(slot_count.long(), 0) - slot_count.long()
            back_flat = self.ops.entry_flat(p_tok, p_flat, start.contiguous(), idx, E, G, n_back)
        self._mark()

        # 3-4. per chunk: dispatch, local experts, return (NCCL async, GEMMs on this stream)
        row_off, back_off = [0], [0]
        for c in range(C):
            row_off.append(row_off[-1] + int(send_rows[c].sum()))
            back_off.append(back_off[-1] + int(send_back[c].sum()))
        dispatched = []
        for c in range(C):
            in_splits = send_rows[c].tolist()
            out_splits = recv_rows[:, c].tolist()
            R = int(sum(out_splits))
            rx = torch.empty((R, H), dtype=x.dtype, device=dev)
            rm = torch.empty((R, 2 * k), dtype=torch.int32, device=dev)
            h1 = dist.all_to_all_single(rx, send_x[row_off[c]:row_off[c + 1]], out_splits,
                                        in_splits, group=self.group, async_op=True)
            h2 = dist.all_to_all_single(rm, meta[row_off[c]:row_off[c + 1]], out_splits,
                                        in_splits, group=self.group, async_op=True)
            dispatched.append((rx, rm, h1, h2))
        back = torch.empty((n_back, H), dtype=x.dtype, device=dev)
        prev_reserve = self.ops.set_sm_reserve(self.sm_reserve)
        returned = []
        received = 0
        computed = 0
        for c, (rx, rm, h1, h2) in enumerate(dispatched):
            h1.wait()
            h2.wait()
            R = rx.shape[0]
            received += R
            n_out = int(recv_back[:, c].sum())
            computed += n_out
            e_loc = rm[:, :k].contiguous()
            w_loc = rm[:, k:].contiguous().view(torch.float32)
            # every (row, slot) contribution, written consecutively in row-major order
            n_asg = int(recv_asg[:, c].sum())
            contrib = torch.empty((n_asg, H), dtype=x.dtype, device=dev)
            if n_asg:
                valid = e_loc < El
                out_row = (torch.cumsum(valid.view(-1), 0) - 1).to(torch.int32)
                self.ops.local_experts_scatter(rx, gate_local, up_local, down_local, w_loc,
                                               e_loc, out_row, contrib, El, self.activation,
                                               moe_type)
            if exact:
                y = contrib
            elif R:
                # partial of each received row: its consecutive contributions, in slot order
                start = torch.zeros((R + 1,), dtype=torch.int64, device=dev)
                torch.cumsum(valid.sum(dim=1), 0, out=start[1:])
                y = self.ops.segment_sum(contrib, start)
            else:
                y = torch.empty((0, H), dtype=x.dtype, device=dev)
            h3 = dist.all_to_all_single(back[back_off[c]:back_off[c + 1]], y,
                                        send_back[c].tolist(), recv_back[:, c].tolist(),
                                        group=self.group, async_op=True)
            returned.append((h3, y))
        self.ops.set_sm_reserve(prev_reserve)
        for h3, _ in returned:
            h3.wait()
        self._mark()

        # 5. combine on the origin: slot order (exact) or rank order (partials)
        if exact:
            out = self.ops.combine_rows(back, back_flat, T, k)
        else:
            out = self.ops.combine_rows(back, p_flat.contiguous(), T, G)
        self._mark()
        self.last_stats = {"pairs_sent": U, "rows_returned": n_back, "rows_received": received,
                           "rows_computed": computed, "chunks": C,
                           "assignments_received": int(recv_asg.sum())}
        return out
