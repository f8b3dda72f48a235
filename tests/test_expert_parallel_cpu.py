"""Expert-parallel exchange logic on two CPU ranks (gloo): bucketing by destination rank,
all_to_all_single of counts / rows / metadata, the return trip and the slot-ordered combine,
with the oracle standing in for the GPU compute.  The result must equal the single-process
oracle up to f32 reassociation (each rank sums its slots before the origin sums the ranks)."""
import multiprocessing as pymp

import pytest
import torch.multiprocessing as mp

import ep_worker


@pytest.mark.parametrize("moe_type", [0, 1])
def test_expert_parallel_matches_single_process_on_gloo(moe_type):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = ep_worker.free_port()
    procs = [ctx.Process(target=ep_worker.cpu_rank,
                         args=(r, 2, port, 40, 32, 48, 8, 3, moe_type, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0, p.exitcode
    results = sorted(q.get() for _ in range(2))
    for rank, maxdiff, stats in results:
        assert maxdiff < 1e-5, (rank, maxdiff)
        assert stats["unique_rows_sent"] > 0 and stats["rows_received"] > 0
