"""Expert-parallel config-5-shaped layer on 2 GPUs vs the single-GPU fused path on the same
tokens, two forwards per layer, all transports (landing buffers filled by the fused push kernels
or by copy engines; NCCL all_to_all): exact mode bit-identical (every contribution computed and rounded as on one GPU,
combined in the same slot order); partials mode within the bf16 tolerance (1e-2 relative); no
device error bits (no arrival wait ran out)."""
import pytest
import torch
import torch.multiprocessing as mp

import ep_worker

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["push", "copy", "collective"])
@pytest.mark.parametrize("mode", ["exact", "partials"])
@pytest.mark.parametrize("moe_type", [0, 1])
def test_expert_parallel_two_gpus(moe_type, mode, transport):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = ep_worker.free_port()
    procs = [ctx.Process(target=ep_worker.gpu_rank,
                         args=(r, 2, port, 3000, 256, 256, 16, 8, moe_type, "bf16", q, mode,
                               transport))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, p.exitcode
    for rank, ok, diff, stats in sorted(q.get() for _ in range(2)):
        assert ok, (rank, diff, stats)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["exact", "partials"])
def test_expert_parallel_two_gpus_balanced_placement(mode):
    """Experts placed by balanced_placement (the biased router's loads evened over the ranks),
    each rank holding its placed experts' weights: same results as without placement."""
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = ep_worker.free_port()
    procs = [ctx.Process(target=ep_worker.gpu_rank,
                         args=(r, 2, port, 3000, 256, 256, 16, 8, 0, "bf16", q, mode, "push",
                               True))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, p.exitcode
    for rank, ok, diff, stats in sorted(q.get() for _ in range(2)):
        assert ok, (rank, diff, stats)
