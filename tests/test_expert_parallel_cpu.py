"""Expert-parallel exchange logic on two CPU ranks (gloo): bucketing by destination rank,
all_to_all_single of counts / rows / metadata, the return trip and the slot-ordered combine,
with the oracle standing in for the GPU compute.  Exact mode must equal the single-process oracle
bit for bit (every contribution computed alone, summed in the same slot order); partials mode
sums each rank's slots before the ranks are summed, so it agrees up to f32 reassociation."""
import multiprocessing as pymp

import pytest
import torch.multiprocessing as mp

import ep_worker


@pytest.mark.parametrize("mode", ["exact", "partials"])
@pytest.mark.parametrize("moe_type", [0, 1])
def test_expert_parallel_matches_single_process_on_gloo(moe_type, mode):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = ep_worker.free_port()
    procs = [ctx.Process(target=ep_worker.cpu_rank,
                         args=(r, 2, port, 40, 32, 48, 8, 3, moe_type, q, mode))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, p.exitcode
    results = sorted(q.get() for _ in range(2))
    for rank, maxdiff, stats in results:
        assert maxdiff == 0.0 if mode == "exact" else maxdiff < 1e-6, (rank, maxdiff)
        assert stats["pairs_sent"] > 0 and stats["rows_received"] > 0
