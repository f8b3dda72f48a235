"""Expert-parallel MoE layer (BASELINE config 5 on 2/4/8 GPUs).

The reference crate has no multi-GPU code; this is the expert-parallel layout its north star asks
for.  With G ranks, rank r owns experts [r*E/G, (r+1)*E/G) and its own tokens.  One forward:

 1. plan: a token is sent once to each rank that owns one of its k experts.  moe_ep_dest_groups
    marks the (token, rank) pairs, grouped by (chunk of tokens, rank); route preparation over
    those groups sorts the pairs (stable: token order inside a group); moe_ep_pack gathers each
    pair's token row and its k-slot metadata (local expert id, or E/G for slots owned by other
    ranks, and the routing weight) into a send buffer ordered by (chunk, rank);
 2. one host synchronisation per forward: the [chunk, rank] counts of every rank;
 3. per chunk, dispatch rows and metadata to the ranks that own their experts;
 4. per chunk, run the rank's experts on the received rows as a k-slot fused MoE (foreign slots
    are skipped), then return the results:
      "partials" (default): one row per pair, the rank's weighted contributions summed in slot
        order and rounded once -- the fewest bytes back; the origin sums a token's partials in
        rank order (equal to the single-GPU output within the bf16 tolerance);
      "exact": one row per (token, slot) contribution, written by moe_fused_scatter in pair
        order; the origin combines all k in slot order, so the output is bit-identical to the
        single-GPU path;
 5. combine on the origin (moe_combine_rows), f32 accumulation, one rounding.

Three transports move the rows of steps 3-4.  The first two share one landing buffer per rank
(arrival flags, received rows and metadata, returned rows), allocated with moe_peer_alloc and
mapped by every other rank; every offset follows from the all-gathered count matrix
(p2p_layout), so each rank computes the same layout, and buffers grow collectively when a rank's
need exceeds its capacity.  After a chunk's rows are in place the sender release-stores the
chunk's epoch into the destination's flag for this sender (moe_peer_signal); the destination's
compute stream waits for the other senders' flags with a bounded wait (moe_peer_wait) and for its
own rows by stream order (an event of the side stream that wrote them), so no kernel polls a flag
that another kernel of the same GPU writes, before its GEMMs read the rows.

  "push" (default on GPUs): SM stores over NVLink, fused with the kernels that produce the rows:
    moe_ep_push_pairs writes each pair's token row and metadata straight into the destination's
    landing rows (no send buffer; chunks after the first on a side stream with one small block
    per SM, beside the persistent GEMMs), and for the last chunk moe_segment_sum_push writes each
    partial straight into the origin's return rows.  Earlier chunks' partials return by copy
    engine (a slot sum beside the GEMMs would stream its rows through L2 and slow them).
  "copy": a send buffer (moe_ep_pack) and copy-engine copies (moe_copy_async, one stream per
    peer) into the same landing buffers; the copy engines take no SM time but move ~500 GB/s per
    GPU at most in this all-to-all pattern.
  "collective": all_to_all_single on the process group's backend (NCCL; gloo on CPU), async on
    the backend's stream, with `sm_reserve` SMs left free by the persistent GEMMs.

The compute steps are injectable (`ops`) so both transports can be tested on CPU ranks; the
default ops are the CUDA library's, which have no CPU fallback.
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist

import candle_moe


def balanced_placement(expert_load, world: int):
    """Expert placement for load balance: returns slot[e] for each expert e, a permutation of
    range(E) where rank r owns the experts whose slots lie in [r*E/world, (r+1)*E/world) -- still
    E/world experts per rank.  Experts in decreasing load go to the rank with the least load so
    far that still has room (greedy), which evens out the rows each rank computes when the
    router favours some experts (BASELINE config 5's per-expert bias)."""
    loads = [float(v) for v in expert_load]
    E = len(loads)
    if E % world:
        raise ValueError(f"num_experts {E} is not divisible by world size {world}")
    El = E // world
    rank_load, filled = [0.0] * world, [0] * world
    slot = [0] * E
    for e in sorted(range(E), key=lambda e: (-loads[e], e)):
        r = min((r for r in range(world) if filled[r] < El), key=lambda r: (rank_load[r], r))
        slot[e] = r * El + filled[r]
        filled[r] += 1
        rank_load[r] += loads[e]
    return slot


def local_experts(slot, world: int, rank: int):
    """Global ids of the experts `rank` owns under placement `slot`, in local-id order (the order
    in which that rank passes their weights to forward)."""
    E = len(slot)
    El = E // world
    inv = [0] * E
    for e, sl in enumerate(slot):
        inv[sl] = e
    return inv[rank * El:(rank + 1) * El]


def expert_range(num_experts: int, world: int, rank: int):
    """Experts [start, end) owned by `rank` (E must divide evenly)."""
    if num_experts % world:
        raise ValueError(f"num_experts {num_experts} is not divisible by world size {world}")
    n = num_experts // world
    return rank * n, (rank + 1) * n


class CudaOps:
    """The product's compute and transport steps (CUDA library)."""

    @staticmethod
    def dest_groups(idx, num_experts, num_ranks, tokens_per_chunk, num_chunks):
        return candle_moe.ep_dest_groups(idx, num_experts, num_ranks, tokens_per_chunk,
                                         num_chunks)

    @staticmethod
    def pack(x, pair_token, pair_flat, idx, w, num_experts, num_ranks, num_pairs_device=None):
        return candle_moe.ep_pack(x, pair_token, pair_flat, idx, w, num_experts, num_ranks,
                                  num_pairs_device)

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

    # ---- landing-buffer transports ----
    peer_alloc = staticmethod(candle_moe.peer_alloc)
    peer_free = staticmethod(candle_moe.peer_free)
    peer_open = staticmethod(candle_moe.peer_open)
    peer_close = staticmethod(candle_moe.peer_close)
    device_bytes = staticmethod(candle_moe.device_bytes)
    copy_async = staticmethod(candle_moe.copy_async)
    peer_signal = staticmethod(candle_moe.peer_signal)
    peer_wait = staticmethod(candle_moe.peer_wait)

    _count_streams = {}

    @classmethod
    def host_counts(cls, work, gathered):
        """Wait for an async all_gather of counts and copy them to the host, on a side stream:
        the compute stream keeps running what was enqueued after the all_gather."""
        dev = gathered[0].device
        side = cls._count_streams.get(dev)
        if side is None:
            side = cls._count_streams[dev] = torch.cuda.Stream(dev)
        # no wait on the compute stream: the all_gather already ordered itself after the counts,
        # and the host blocks below until the side stream is done with `gathered`
        with torch.cuda.stream(side):
            work.wait()
            host = torch.stack(gathered).cpu()
        return host.numpy()

    @staticmethod
    def push_pairs(x, pair_token, pair_flat, off, chunk, idx, w, num_experts, num_ranks, rows_to,
                   meta_to, stream, blocks):
        candle_moe.ep_push_pairs(x, pair_token, pair_flat, off, chunk, idx, w, num_experts,
                                 num_ranks, rows_to, meta_to, None, stream, blocks)

    @staticmethod
    def segment_sum_push(rows, start, dst, first, stream, blocks):
        candle_moe.segment_sum_push(rows, start, dst, first, stream, blocks)

    @staticmethod
    def num_sms(device):
        return torch.cuda.get_device_properties(device).multi_processor_count

    @staticmethod
    def new_stream(device):
        return torch.cuda.Stream(device)

    @staticmethod
    def current_stream(device):
        return torch.cuda.current_stream(device)

    @staticmethod
    def record(stream):
        ev = torch.cuda.Event()
        ev.record(stream)
        return ev

    @staticmethod
    def wait(stream, event):
        stream.wait_event(event)


def p2p_layout(allc: np.ndarray):
    """Row offsets of the landing-buffer exchange from the all-gathered counts.

    allc[s, c, d] = (pairs, returned rows, assignments) that rank s sends rank d in chunk c.
    Returns exclusive prefix sums (rows):
      send_start[s, c, d]  block (c, d) in s's send buffer, blocks ordered (c, d);
      recv_start[d, c, s]  block from s in chunk c in d's landing rows, ordered (c, s);
      back_start[s, c, d]  rows d returns for chunk c in s's return region, ordered (c, d);
      y_start[d, c, s]     rows d returns to s inside d's chunk-c results, ordered s.
    """
    pairs = allc[..., 0].astype(np.int64)
    back = allc[..., 1].astype(np.int64)

    def excl(a):
        flat = a.reshape(a.shape[0], -1)
        return (np.cumsum(flat, axis=1) - flat).reshape(a.shape)

    bt = back.transpose(2, 1, 0)
    return (excl(pairs), excl(pairs.transpose(2, 1, 0)), excl(back),
            np.cumsum(bt, axis=2) - bt)


def _align(v: int, a: int = 256) -> int:
    return (v + a - 1) // a * a


class _Landing:
    """The landing buffers of all ranks: this rank's own (allocated) and every peer's
    (mapped), with their capacities, and the epoch counters of the arrival flags.

    Buffer of rank r: [flags: 2G u32 | rows: cap_rows x row_bytes | meta: cap_rows x meta_bytes |
    back: cap_back x row_bytes], regions 256-byte aligned.  flags[s] is the dispatch flag written
    by rank s, flags[G + s] its return flag."""

    FLAG_BYTES = 256
    SLACK_ROWS = 256  # rows added to a grown capacity beyond 1.25x the need

    def __init__(self, ops, group, world, rank, device):
        self.ops, self.group, self.world, self.rank, self.device = ops, group, world, rank, device
        self.caps = [(0, 0)] * world
        self.key = None
        self.addr = [0] * world
        self.local = None          # uint8 tensor over this rank's buffer
        self.epoch_dispatch = 0
        self.epoch_return = 0
        self.regrows = 0

    def regions(self, r):
        rows_cap, back_cap = self.caps[r]
        row_b, meta_b = self.key
        rows = self.FLAG_BYTES
        meta = _align(rows + rows_cap * row_b)
        back = _align(meta + rows_cap * meta_b)
        return rows, meta, back, _align(back + back_cap * row_b)

    def ensure(self, need_rows, need_back, key):
        """Collective: every rank calls it with the same arguments (they follow from the
        all-gathered counts).  Grows the buffers that are too small; nothing may be reading or
        writing any landing buffer meanwhile."""
        grow = [key != self.key or need_rows[r] > self.caps[r][0] or
                need_back[r] > self.caps[r][1] for r in range(self.world)]
        if not any(grow):
            return
        self.regrows += 1
        for r in range(self.world):
            if grow[r] and r != self.rank and self.addr[r]:
                self.ops.peer_close(self.addr[r], self.device)
                self.addr[r] = 0
        dist.barrier(group=self.group)  # every mapping of a buffer about to be freed is closed
        self.key = key
        slack = self.SLACK_ROWS
        self.caps = [(max(self.caps[r][0], int(need_rows[r] * 1.25) + slack),
                      max(self.caps[r][1], int(need_back[r] * 1.25) + slack)) if grow[r]
                     else self.caps[r] for r in range(self.world)]
        mine = torch.zeros(candle_moe.PEER_HANDLE_BYTES, dtype=torch.uint8)
        if grow[self.rank]:
            if self.addr[self.rank]:
                self.local = None
                self.ops.peer_free(self.addr[self.rank], self.device)
            total = self.regions(self.rank)[3]
            self.addr[self.rank], handle = self.ops.peer_alloc(total, self.device)
            self.local = self.ops.device_bytes(self.addr[self.rank], total, self.device)
            mine = torch.frombuffer(bytearray(handle), dtype=torch.uint8)
        gathered = [torch.empty_like(mine, device=self.device) for _ in range(self.world)]
        dist.all_gather(gathered, mine.to(self.device), group=self.group)
        for r in range(self.world):
            if grow[r] and r != self.rank:
                self.addr[r] = self.ops.peer_open(bytes(gathered[r].cpu().numpy()), self.device)

    def abandon(self):
        """Local, non-collective release after a failed exchange (peers may be gone): unmap the
        peers' buffers and free this rank's own."""
        for r in range(self.world):
            if r != self.rank and self.addr[r]:
                self.ops.peer_close(self.addr[r], self.device)
                self.addr[r] = 0
        if self.addr[self.rank]:
            self.local = None
            self.ops.peer_free(self.addr[self.rank], self.device)
            self.addr[self.rank] = 0
        self.caps = [(0, 0)] * self.world
        self.key = None

    def release(self):
        for r in range(self.world):
            if self.addr[r] and r != self.rank:
                self.ops.peer_close(self.addr[r], self.device)
                self.addr[r] = 0
        dist.barrier(group=self.group)
        if self.addr[self.rank]:
            self.local = None
            self.ops.peer_free(self.addr[self.rank], self.device)
            self.addr[self.rank] = 0
        self.caps = [(0, 0)] * self.world
        self.key = None


class ExpertParallelMoE:
    """Expert-parallel counterpart of candle_moe.FusedMoE for one process group."""

    STAGES = ("plan", "exchange", "combine")

    def __init__(self, num_experts: int, num_selected_experts: int,
                 activation=candle_moe.Activation.Silu, group: Optional[dist.ProcessGroup] = None,
                 ops=None, chunks: int = 4, sm_reserve: int = 24, mode: str = "partials",
                 transport: str = "auto", wait_timeout_s: float = 5.0,
                 compute_groups: Optional[Sequence[int]] = None):
        self.num_experts = num_experts
        self.k = num_selected_experts
        self.activation = int(activation)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 32:
            raise ValueError("at most 32 ranks")
        self.start, self.end = expert_range(num_experts, self.world, self.rank)
        self.num_local = self.end - self.start
        self.ops = ops or CudaOps()
        self.chunks = max(1, chunks)
        # Landing-buffer transports: consecutive chunks computed as one fused call once the
        # group's last chunk has landed (sizes in chunks, summing to `chunks`; default one chunk
        # per call).  Small first and last groups start the GEMMs early and keep the last
        # return short; larger middle groups pay the per-call costs fewer times.
        groups = list(compute_groups) if compute_groups else [1] * self.chunks
        if sum(groups) != self.chunks or min(groups) < 1:
            raise ValueError(f"compute_groups {groups} must be positive and sum to {self.chunks}")
        self.compute_groups = groups
        # SMs the expert GEMMs leave to NCCL's kernels while the collective exchange is in
        # flight: the GEMMs are persistent (one CTA per SM), and without free SMs the collectives
        # would only run between GEMM launches.  The GEMMs take tiles dynamically, so the reserve
        # only costs the SMs themselves.  The landing-buffer transports need none.
        self.sm_reserve = sm_reserve
        if mode not in ("partials", "exact"):
            raise ValueError(f"unknown mode {mode!r}")
        self.mode = mode
        if transport == "auto":
            transport = "push" if isinstance(self.ops, CudaOps) else "collective"
        if transport not in ("push", "copy", "collective"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.wait_timeout_s = wait_timeout_s
        self._slot = None            # expert placement (set_placement); None: expert_range
        self._slot_dev = {}
        self._landing = None
        self._streams = None
        self._zeros = {}
        self.last_stats = {}
        self.timing = False          # record CUDA events per stage (benchmark analysis)
        self._events = []
        self._timeline = []          # per timed forward: (first stage event, [(point, event)])

    # ---- benchmark instrumentation -----------------------------------------------------------
    def _mark(self):
        if self.timing:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events.append(e)

    def _point(self, name, stream=None):
        """Timeline point of the current timed forward (an event on `stream`, default the
        current one); the landing-buffer transports mark when each chunk's rows landed and were
        used."""
        if self.timing:
            e = torch.cuda.Event(enable_timing=True)
            if stream is None:
                e.record()
            else:
                e.record(stream)
            self._timeline[-1][1].append((name, e))

    def timeline(self):
        """Mean milliseconds from the start of a timed forward to each timeline point."""
        acc = {}
        for origin, pts in self._timeline:
            for name, e in pts:
                e.synchronize()
                acc.setdefault(name, []).append(origin.elapsed_time(e))
        return {k: sum(v) / len(v) for k, v in acc.items()}

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

    def close(self):
        """Collective: unmap and free the landing buffers."""
        if self._landing is not None:
            self._landing.release()
            self._landing = None

    def abandon(self):
        """After a failed forward (a peer stopped signalling): release this rank's landing
        buffers without any collective step."""
        if self._landing is not None:
            self._landing.abandon()
            self._landing = None

    def check_errors(self, device=None):
        """Raise if an arrival wait of this device ran out since the last check (a peer never
        signalled: the rows it should have sent are missing).  Synchronises the device."""
        dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        bits = candle_moe.device_error_bits(dev.index or 0, clear=True)
        if bits & candle_moe.ERR_PEER_WAIT:
            raise TimeoutError(f"expert-parallel exchange: an arrival wait ran out "
                               f"(device error bits {bits:#x})")

    def set_placement(self, slot):
        """Place experts by `slot` (see balanced_placement): expert e lives on rank
        slot[e] // (E/world) as local expert slot[e] % (E/world), so each rank passes forward the
        weights of local_experts(slot, world, rank) in that order.  Every rank must set the same
        placement; None restores the contiguous ranges of expert_range."""
        if slot is not None:
            slot = [int(v) for v in slot]
            if sorted(slot) != list(range(self.num_experts)):
                raise ValueError("placement must be a permutation of range(num_experts)")
        self._slot = slot
        self._slot_dev = {}

    # ---- forward -----------------------------------------------------------------------------
    def _plan(self, x, routing_weights, expert_indices, C, Tc):
        """Pairs sorted by (chunk, rank, token) and the [C, G, 3] counts this rank sends."""
        G, E = self.world, self.num_experts
        dev = x.device
        idx = expert_indices.to(torch.int32).contiguous()
        if self._slot is not None:
            # global expert ids -> placement slots; ids outside [0, E) stay as they are (skipped)
            st = self._slot_dev.get(dev)
            if st is None:
                st = self._slot_dev[dev] = torch.tensor(self._slot, dtype=torch.int32, device=dev)
            valid = (idx >= 0) & (idx < E)
            idx = torch.where(valid, st[idx.clamp(0, E - 1).long()], idx).contiguous()
        w = routing_weights.contiguous()
        groups, asg = self.ops.dest_groups(idx, E, G, Tc, C)
        zw = self._zeros.get(groups.shape)
        if zw is None or zw.device != dev:
            zw = self._zeros[groups.shape] = torch.zeros(groups.shape, dtype=torch.float32,
                                                         device=dev)
        off, p_tok, _, p_flat = self.ops.route_prep(groups, zw, C * G)
        pair_counts = (off[1:C * G + 1] - off[:C * G]).to(torch.int64).view(C, G)
        # asg: (token, slot) entries per (chunk, rank) -- the expert work each rank will do for
        # us, and in exact mode also the rows that come back
        exact = self.mode == "exact"
        counts = torch.stack([pair_counts, asg if exact else pair_counts, asg], dim=2)
        return idx, w, p_tok, p_flat, counts, off

    def _local_experts(self, rx, rm):
        """Slot metadata of received rows: (local expert ids [R,k], weights [R,k], valid slots,
        out_row: each valid slot's row among the chunk's contributions, row-major)."""
        k, El = self.k, self.num_local
        e_loc = rm[:, :k].contiguous()
        w_loc = rm[:, k:].contiguous().view(torch.float32)
        valid = e_loc < El
        out_row = (torch.cumsum(valid.view(-1), 0) - 1).to(torch.int32)
        return e_loc, w_loc, valid, out_row

    def forward(self, x: torch.Tensor, gate_local: torch.Tensor, up_local: torch.Tensor,
                down_local: Optional[torch.Tensor], routing_weights: torch.Tensor,
                expert_indices: torch.Tensor, moe_type: int) -> torch.Tensor:
        """x [T,H] local tokens; *_local: this rank's experts (gate/up [E/G,H,I], down [E/G,I,H]);
        routing_weights / expert_indices [T,k] with global expert ids.  Returns [T,H]."""
        if self.transport in ("push", "copy"):
            return self._forward_landing(x, gate_local, up_local, down_local, routing_weights,
                                         expert_indices, moe_type)
        return self._forward_collective(x, gate_local, up_local, down_local, routing_weights,
                                        expert_indices, moe_type)

    def _wait_others(self, flags, value, stream, ev_own):
        """Stream-ordered arrival wait: a bounded poll of the flags the other ranks write (their
        GPUs run their kernels), and an event for this rank's own contribution, which its own
        side stream produced -- no kernel of this GPU spins on another kernel of the same GPU."""
        ops, G, me = self.ops, self.world, self.rank
        if me > 0:
            ops.peer_wait(flags, me, value, self.wait_timeout_s, stream)
        if me + 1 < G:
            ops.peer_wait(flags + 4 * (me + 1), G - me - 1, value, self.wait_timeout_s, stream)
        ops.wait(stream, ev_own)

    def _chunking(self, T):
        C = self.chunks  # the same on every rank: the counts exchange has shape [C, G, 3]
        Tc = max(1, (T + C - 1) // C)
        return C, Tc

    # ---- landing-buffer transports ("push": SM stores over NVLink, "copy": copy engines) ------
    def _forward_landing(self, x, gate_local, up_local, down_local, routing_weights,
                         expert_indices, moe_type):
        T, H = x.shape
        k, G, E, El, me = self.k, self.world, self.num_experts, self.num_local, self.rank
        C, Tc = self._chunking(T)
        dev = x.device
        ops = self.ops
        exact = self.mode == "exact"
        push = self.transport == "push"
        self._mark()
        if self.timing:
            self._timeline.append((self._events[-1], []))

        # 1-2. plan; the one host synchronisation: every rank's counts
        idx, w, p_tok, p_flat, counts, off = self._plan(x, routing_weights, expert_indices, C, Tc)
        self._point("planned")
        gathered = [torch.empty_like(counts) for _ in range(G)]
        work = dist.all_gather(gathered, counts, group=self.group, async_op=True)
        if not push:
            # pack while the counts travel: the pair count is read on the device, the buffers
            # hold every (token, rank) entry
            send_x, meta, slot_count = ops.pack(x, p_tok, p_flat, idx, w, E, G,
                                                off[C * G:C * G + 1])
            self._point("packed")
        allc = ops.host_counts(work, gathered)               # [G_src, C, G_dst, 3]
        send_start, recv_start, back_start, y_start = p2p_layout(allc)
        pairs, back = allc[..., 0], allc[..., 1]
        U = int(pairs[me].sum())
        n_back = int(back[me].sum())
        es = x.element_size()
        row_b, meta_b = H * es, 2 * k * 4
        if self._landing is None:
            self._landing = _Landing(ops, self.group, G, me, dev)
            self._streams = [ops.new_stream(dev) for _ in range(G + 1)]
        L = self._landing
        L.ensure(pairs.sum(axis=(0, 1)), back.sum(axis=(1, 2)), (row_b, meta_b))
        regions = [L.regions(r) for r in range(G)]
        copy_s, sig_s = self._streams[:G], self._streams[G]
        compute = ops.current_stream(dev)
        sms = ops.num_sms(dev)

        p_tok, p_flat = p_tok[:U], p_flat[:U]
        if exact:
            if push:  # the slots of each pair: its token's experts on the pair's rank
                e = idx.long()[p_tok.long()] & 0xFFFFFFFF
                d = (p_flat.long() % G)[:, None]
                slot_count = ((e < E) & (torch.div(e, El, rounding_mode="floor") == d)).sum(1)
            sc = slot_count[:U].long()
            start = torch.cumsum(sc, 0) - sc
            back_flat = ops.entry_flat(p_tok, p_flat, start.contiguous(), idx, E, G, n_back)
        self._mark()

        # 3. dispatch every chunk, then its arrival flag at every destination
        flag_d = [L.addr[r] + 4 * me for r in range(G)]
        flag_r = [L.addr[r] + 4 * (G + me) for r in range(G)]
        ep_d, ep_r = L.epoch_dispatch, L.epoch_return
        ev_ready = ops.record(compute)
        ev_sent = []  # per chunk: this rank's own rows are in its buffer (stream order)
        if push:
            # fused pack + dispatch: SM stores straight into the destinations' landing rows; the
            # first chunk has the GPU to itself, later ones share it with the GEMMs
            ops.wait(sig_s, ev_ready)
            self._point("copies_start", sig_s)
            for c in range(C):
                rows_to = [L.addr[d] + regions[d][0] + int(recv_start[d, c, me]) * row_b
                           for d in range(G)]
                meta_to = [L.addr[d] + regions[d][1] + int(recv_start[d, c, me]) * meta_b
                           for d in range(G)]
                if int(pairs[me, c].sum()):
                    ops.push_pairs(x, p_tok, p_flat, off, c, idx, w, E, G, rows_to, meta_to,
                                   sig_s, 4 * sms if c == 0 else sms)
                ops.peer_signal(flag_d, ep_d + c + 1, sig_s)
                ev_sent.append(ops.record(sig_s))
                self._point(f"sent{c}", sig_s)
        else:
            # copy engines, one stream per destination
            for s in copy_s:
                ops.wait(s, ev_ready)
            self._point("copies_start", copy_s[(me + 1) % G])
            x_addr, m_addr = send_x.data_ptr(), meta.data_ptr()
            for c in range(C):
                for j in range(G):
                    d = (me + j) % G  # start with the next rank: senders spread over destinations
                    n = int(pairs[me, c, d])
                    if n:
                        r0 = int(recv_start[d, c, me])
                        s0 = int(send_start[me, c, d])
                        ops.copy_async(L.addr[d] + regions[d][0] + r0 * row_b,
                                       x_addr + s0 * row_b, n * row_b, copy_s[d])
                        ops.copy_async(L.addr[d] + regions[d][1] + r0 * meta_b,
                                       m_addr + s0 * meta_b, n * meta_b, copy_s[d])
                for s in copy_s:
                    ops.wait(sig_s, ops.record(s))
                ops.peer_signal(flag_d, ep_d + c + 1, sig_s)
                ev_sent.append(ops.record(sig_s))
                self._point(f"sent{c}", sig_s)

        # 4. per group of chunks: wait for the rows, run the local experts, send the results back
        keep = []
        received = computed = 0
        rows0, meta0, back0, _ = regions[me]
        c_first = 0
        for gsize in self.compute_groups:
            cs = list(range(c_first, c_first + gsize))
            c_first += gsize
            c = cs[-1]
            self._wait_others(L.addr[me], ep_d + c + 1, compute, ev_sent[c])
            self._point(f"landed{c}")
            R = int(pairs[:, cs, me].sum())
            r0 = int(recv_start[me, cs[0], 0])
            received += R
            n_out = int(back[:, cs, me].sum())
            computed += n_out
            if R == 0:
                continue
            rx = L.local[rows0 + r0 * row_b: rows0 + (r0 + R) * row_b].view(x.dtype).view(R, H)
            rm = L.local[meta0 + r0 * meta_b: meta0 + (r0 + R) * meta_b].view(torch.int32) \
                .view(R, 2 * k)
            e_loc, w_loc, valid, out_row = self._local_experts(rx, rm)
            n_asg = int(allc[:, cs, me, 2].sum())
            contrib = torch.empty((n_asg, H), dtype=x.dtype, device=dev)
            if n_asg:
                ops.local_experts_scatter(rx, gate_local, up_local, down_local, w_loc, e_loc,
                                          out_row, contrib, El, self.activation, moe_type)
            # segments of the results: a received row's consecutive contributions (partials),
            # or each contribution alone (exact)
            if exact:
                seg = torch.arange(n_asg + 1, dtype=torch.int64, device=dev)
            else:
                seg = torch.zeros((R + 1,), dtype=torch.int64, device=dev)
                torch.cumsum(valid.sum(dim=1), 0, out=seg[1:])
            if push and gsize == 1 and c == C - 1:
                # the last chunk has the GPU to itself: slot sum fused with the return, the
                # partials stored straight into the origins' buffers.  (Earlier chunks sum on
                # this stream and return by copy engine: a slot sum beside the next chunk's GEMMs
                # streams its rows through L2 and slows them more than it saves.)
                dst = [L.addr[s] + regions[s][2] + int(back_start[s, c, me]) * row_b
                       for s in range(G)]
                first = [int(v) for v in y_start[me, c]] + [n_out]
                keep += [contrib, seg]
                ops.segment_sum_push(contrib, seg, dst, first, compute, 4 * sms)
                self._point(f"computed{c}")
                continue
            y = contrib if exact else ops.segment_sum(contrib, seg).to(x.dtype).contiguous()
            keep.append(y)
            self._point(f"computed{c}")
            ev_y = ops.record(compute)
            y_addr = y.data_ptr()
            base = 0  # the group's results: chunk by chunk, each chunk's rows ordered by origin
            for cc in cs:
                first = [int(v) for v in y_start[me, cc]] + [int(back[:, cc, me].sum())]
                for j in range(G):
                    s = (me + j) % G
                    n = first[s + 1] - first[s]
                    if n:
                        ops.wait(copy_s[s], ev_y)
                        ops.copy_async(L.addr[s] + regions[s][2] + int(back_start[s, cc, me]) * row_b,
                                       y_addr + (base + first[s]) * row_b, n * row_b, copy_s[s])
                base += first[G]
        for s in copy_s + [compute]:
            ops.wait(sig_s, ops.record(s))
        ops.peer_signal(flag_r, ep_r + 1, sig_s)
        ev_back = ops.record(sig_s)
        self._point("returned", sig_s)
        self._wait_others(L.addr[me] + 4 * G, ep_r + 1, compute, ev_back)
        self._point("all_returned")
        L.epoch_dispatch, L.epoch_return = ep_d + C, ep_r + 1
        self._mark()

        # 5. combine on the origin: slot order (exact) or rank order (partials)
        back_rows = L.local[back0: back0 + n_back * row_b].view(x.dtype).view(n_back, H)
        if exact:
            out = ops.combine_rows(back_rows, back_flat, T, k)
        else:
            out = ops.combine_rows(back_rows, p_flat.contiguous(), T, G)
        # the side streams read tensors of this forward (send buffers, results): join them before
        # those tensors can be freed, and before the next forward writes again
        for s in self._streams:
            ops.wait(compute, ops.record(s))
        del keep
        self._mark()
        self.last_stats = {"pairs_sent": U, "rows_returned": n_back, "rows_received": received,
                           "rows_computed": computed, "chunks": C,
                           "assignments_received": int(allc[:, :, me, 2].sum()),
                           "landing_regrows": L.regrows}
        return out

    # ---- collective transport ------------------------------------------------------------------
    def _forward_collective(self, x, gate_local, up_local, down_local, routing_weights,
                            expert_indices, moe_type):
        T, H = x.shape
        k, G, E, El = self.k, self.world, self.num_experts, self.num_local
        C, Tc = self._chunking(T)
        dev = x.device
        exact = self.mode == "exact"
        self._mark()

        # 1. plan
        idx, w, p_tok, p_flat, counts, _ = self._plan(x, routing_weights, expert_indices, C, Tc)
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

        # 3-4. per chunk: dispatch, local experts, return (async on the backend's stream)
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
            e_loc, w_loc, valid, out_row = self._local_experts(rx, rm)
            # every (row, slot) contribution, written consecutively in row-major order
            n_asg = int(recv_asg[:, c].sum())
            contrib = torch.empty((n_asg, H), dtype=x.dtype, device=dev)
            if n_asg:
                self.ops.local_experts_scatter(rx, gate_local, up_local, down_local, w_loc,
                                               e_loc, out_row, contrib, El, self.activation,
                                               moe_type)
            if exact:
                y = contrib
            elif R:
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
