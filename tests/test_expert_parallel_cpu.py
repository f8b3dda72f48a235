"""Expert-parallel exchange logic on two CPU ranks (gloo): bucketing by destination rank, the
counts exchange, dispatch of rows and metadata, the return trip and the slot-ordered combine,
with the oracle standing in for the GPU compute.  All transports run: "collective"
(all_to_all_single), "copy" and "push" (landing buffers written directly by the senders -- a send
buffer and block copies, or rows stored by the fused pack / slot-sum steps -- here host shared
memory in place of peer-mapped HBM, with the same layout, arrival flags, epochs and collective
growth as on GPUs).  Exact mode must equal the single-process oracle bit for bit (every
contribution computed alone, summed in the same slot order); partials mode sums each rank's slots
before the ranks are summed, so it agrees up to f32 reassociation."""
import numpy as np
import pytest
import torch.multiprocessing as mp

import ep_worker
import expert_parallel


def _run(moe_type, mode, transport, sizes=None, T=40, chunks=3, groups=None, placement=None):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = ep_worker.free_port()
    procs = [ctx.Process(target=ep_worker.cpu_rank,
                         args=(r, 2, port, T, 32, 48, 8, 3, moe_type, q, mode, transport, sizes,
                               chunks, groups, placement))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, p.exitcode
    return sorted(q.get() for _ in range(2))


@pytest.mark.parametrize("transport", ["collective", "copy", "push"])
@pytest.mark.parametrize("mode", ["exact", "partials"])
@pytest.mark.parametrize("moe_type", [0, 1])
def test_expert_parallel_matches_single_process_on_gloo(moe_type, mode, transport):
    for rank, maxdiff, stats in _run(moe_type, mode, transport):
        assert maxdiff == 0.0 if mode == "exact" else maxdiff < 1e-6, (rank, maxdiff)
        assert stats["pairs_sent"] > 0 and stats["rows_received"] > 0


@pytest.mark.parametrize("transport", ["collective", "copy", "push"])
@pytest.mark.parametrize("mode", ["exact", "partials"])
def test_expert_placement(mode, transport):
    """Experts placed by a permutation (rank 0 owns experts 7, 2, 4, 1; rank 1 owns 0, 3, 5, 6):
    each rank passes its placed experts' weights, and the outputs equal the single-process
    oracle as with the contiguous ranges."""
    placement = [4, 3, 1, 5, 2, 6, 7, 0]  # slot of expert e; slots 0-3 on rank 0
    assert expert_parallel.local_experts(placement, 2, 0) == [7, 2, 4, 1]
    for rank, maxdiff, stats in _run(0, mode, transport, placement=placement):
        assert maxdiff == 0.0 if mode == "exact" else maxdiff < 1e-6, (rank, maxdiff)


def test_balanced_placement_evens_the_ranks():
    loads = [100, 90, 80, 70, 60, 50, 40, 30]
    slot = expert_parallel.balanced_placement(loads, 2)
    assert sorted(slot) == list(range(8))
    per_rank = [sum(loads[e] for e in range(8) if slot[e] // 4 == r) for r in range(2)]
    assert max(per_rank) - min(per_rank) <= 20, per_rank  # contiguous ranges: 340 vs 180
    loads = [100, 90, 80, 10, 10, 5, 5, 0]  # the best split of four and four is 125 / 175
    slot = expert_parallel.balanced_placement(loads, 2)
    per_rank = [sum(loads[e] for e in range(8) if slot[e] // 4 == r) for r in range(2)]
    assert max(per_rank) == 175, per_rank


@pytest.mark.parametrize("transport", ["copy", "push"])
@pytest.mark.parametrize("mode", ["exact", "partials"])
@pytest.mark.parametrize("groups", [(1, 3, 1), (2, 3), (5,)])
def test_chunks_computed_in_groups(groups, mode, transport):
    """Five dispatch chunks computed as groups of consecutive chunks (one fused call per group,
    results returned chunk by chunk): the same outputs as one call per chunk."""
    for rank, maxdiff, stats in _run(1, mode, transport, sizes=[40, 9], chunks=5, groups=groups):
        assert maxdiff == 0.0 if mode == "exact" else maxdiff < 1e-6, (rank, maxdiff)
        assert stats["chunks"] == 5


@pytest.mark.parametrize("transport", ["copy", "push"])
@pytest.mark.parametrize("mode", ["exact", "partials"])
def test_landing_buffers_grow_and_epochs_continue(mode, transport):
    """Three forwards through one layer: 2 tokens per rank (fewer than the 3 chunks, so some
    chunks are empty), then 40 (the landing buffers must grow on every rank), then 17 (reuse)."""
    for rank, maxdiff, stats in _run(0, mode, transport, sizes=[2, 40, 17]):
        assert maxdiff == 0.0 if mode == "exact" else maxdiff < 1e-6, (rank, maxdiff)
        assert stats["landing_regrows"] == 2, stats


def test_p2p_layout_places_blocks_like_all_to_all():
    """p2p_layout: the landing rows of each rank hold, per chunk, the blocks of every source in
    source order (what all_to_all_single delivers), and the returned rows land in the origin's
    pair order."""
    import expert_parallel
    rng = np.random.default_rng(5)
    G, C = 3, 4
    allc = rng.integers(0, 5, size=(G, C, G, 3))
    allc[..., 1] = allc[..., 0]
    send_start, recv_start, back_start, y_start = expert_parallel.p2p_layout(allc)
    pairs = allc[..., 0]
    # send buffers: row id = (source, chunk, destination, index)
    send = [[(s, c, d, i) for c in range(C) for d in range(G) for i in range(pairs[s, c, d])]
            for s in range(G)]
    land = [[None] * int(pairs[:, :, d].sum()) for d in range(G)]
    for s in range(G):
        for c in range(C):
            for d in range(G):
                n = pairs[s, c, d]
                a, b = send_start[s, c, d], recv_start[d, c, s]
                land[d][b:b + n] = send[s][a:a + n]
    for d in range(G):
        expect = [(s, c, d, i) for c in range(C) for s in range(G) for i in range(pairs[s, c, d])]
        assert land[d] == expect
    # return: rank d's chunk-c results are its chunk-c landing rows in order; they must land in
    # the origin's return region in the origin's pair (send) order
    back = [[None] * int(pairs[s].sum()) for s in range(G)]
    for d in range(G):
        for c in range(C):
            r0 = recv_start[d, c, 0]
            res = land[d][r0:r0 + int(pairs[:, c, d].sum())]
            for s in range(G):
                n = pairs[s, c, d]
                a, b = y_start[d, c, s], back_start[s, c, d]
                back[s][b:b + n] = res[a:a + n]
    for s in range(G):
        assert back[s] == send[s]


@pytest.mark.parametrize("transport", ["copy", "push"])
def test_lost_arrival_signal_ends_in_timeouts_not_a_hang(transport):
    """Failure detection without a GPU fault: rank 1's arrival signals stop after its first
    (lost messages).  Rank 0's wait for the next chunk runs out after its 1 s limit, and rank 1,
    whose returns from rank 0 then never come, runs out too; both release their buffers locally."""
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = ep_worker.free_port()
    procs = [ctx.Process(target=ep_worker.cpu_rank_dropped_signal,
                         args=(r, 2, port, transport, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, p.exitcode
    results = sorted(q.get() for _ in range(2))
    for rank, outcome, seconds in results:
        assert outcome.startswith("timeout"), (rank, outcome)
        assert seconds < 30, (rank, seconds)


def test_p2p_layout_and_landing_regions_properties():
    """For random rank / chunk counts and uneven traffic: every block a sender writes lies inside
    the receiver's landing rows, blocks of different senders never overlap, the returned rows
    fill the origin's return region exactly once, and the landing regions are 256-byte aligned
    and large enough for the capacities."""
    from hypothesis import given, settings
    from hypothesis import strategies as st
    import expert_parallel

    @settings(max_examples=60, deadline=None)
    @given(st.integers(1, 8), st.integers(1, 5), st.integers(0, 2 ** 31 - 1))
    def check(G, C, seed):
        rng = np.random.default_rng(seed)
        allc = rng.integers(0, 7, size=(G, C, G, 3))
        allc[..., 2] = allc[..., 0] + rng.integers(0, 3, size=(G, C, G))  # assignments >= pairs
        for exact in (False, True):
            a = allc.copy()
            a[..., 1] = a[..., 2] if exact else a[..., 0]
            send_start, recv_start, back_start, y_start = expert_parallel.p2p_layout(a)
            pairs, back = a[..., 0], a[..., 1]
            for d in range(G):
                cover = np.zeros(int(pairs[:, :, d].sum()), dtype=int)
                for c in range(C):
                    for s in range(G):
                        r0, n = recv_start[d, c, s], pairs[s, c, d]
                        cover[r0:r0 + n] += 1
                        assert r0 + n <= cover.size
                        assert send_start[s, c, d] + n <= pairs[s].sum()
                assert (cover == 1).all()
            for s in range(G):
                cover = np.zeros(int(back[s].sum()), dtype=int)
                for c in range(C):
                    for d in range(G):
                        b0, n = back_start[s, c, d], back[s, c, d]
                        cover[b0:b0 + n] += 1
                        # the rows d returns for s sit inside d's chunk-c results
                        assert y_start[d, c, s] + n <= back[:, c, d].sum()
                assert (cover == 1).all()

        L = expert_parallel._Landing(None, None, G, 0, "cpu")
        L.key = (int(rng.integers(1, 64)) * 16, 2 * int(rng.integers(1, 9)) * 4)
        L.caps = [(int(rng.integers(0, 500)), int(rng.integers(0, 500))) for _ in range(G)]
        for r in range(G):
            rows, meta, back0, total = L.regions(r)
            row_b, meta_b = L.key
            assert rows >= 4 * 2 * G and all(v % 256 == 0 for v in (rows, meta, back0, total))
            assert meta >= rows + L.caps[r][0] * row_b
            assert back0 >= meta + L.caps[r][0] * meta_b
            assert total >= back0 + L.caps[r][1] * row_b

    check()
