"""Benchmark of the candle-moe-b200 hot path (router + fused MoE expert FFN).

Default workload (N=1): BASELINE config 5, the Qwen3-30B-A3B-shaped MoE layer -- bf16, 65536
tokens, hidden 2048, moe_intermediate 768, 128 experts, top-8, SwiGLU, renormalised top-k
weights, router logits N(0,1) + a per-expert N(0,0.5) bias.  One step = topk_softmax on the
[65536,128] logits + FusedMoE.forward (route preparation, two tcgen05 grouped GEMMs, combine).
Inputs are seeded synthetic tensors (no datasets exist for this layer); weights ~N(0,0.02),
hidden ~N(0,1).  The weights (1.2 GB) and activations (256 MB) are larger than the 126 MB L2,
so no explicit flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1..c5]

N>1 (torchrun, one rank per GPU), config 5: expert parallel -- every rank holds 65536 tokens and
128/N experts; tokens are dispatched to the ranks owning their experts and the weighted
contributions returned with NCCL all_to_all_single (candle-moe_b200/expert_parallel.py); weak
scaling, value = tokens of all ranks / max-over-ranks step time.  Other configs run one replica
per rank.  --impl reference times the reference's algorithm on the host cores (the CPU oracle port,
all threads) on a bounded token sample per step; the reference crate has no CPU implementation
of its own and its CUDA GEMM kernels cannot launch at these sizes.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "candle-moe_b200")]

CONFIGS = {
    # name: (dtype, moe_type, act, T, H, I, E, k, renormalize, bias_std)
    "c1": ("f32", None, None, 512, None, None, 8, 2, False, 0.0),         # router only
    "c2": ("f32", 1, 1, 512, 768, 3072, 8, 2, False, 0.0),
    "c3": ("bf16", 1, 1, 32768, 768, 3072, 8, 2, False, 0.0),
    "c4": ("bf16", 0, 0, 32768, 4096, 1536, 8, 2, True, 0.0),
    "c4-f16": ("f16", 0, 0, 32768, 4096, 1536, 8, 2, True, 0.0),
    "c5": ("bf16", 0, 0, 65536, 2048, 768, 128, 8, True, 0.5),
}
WORKLOAD_NAMES = {
    "c1": "topk-softmax router, 512 tokens x 8 experts, top-2 (BASELINE config 1)",
    "c2": "Nomic MoE f32, 512 tokens, H768 I3072, 8 experts top-2, GELU (BASELINE config 2)",
    "c3": "Nomic MoE bf16, 32768 tokens, H768 I3072, 8 experts top-2, GELU (BASELINE config 3)",
    "c4": "Qwen3 MoE bf16, 32768 tokens, H4096 I1536, 8 experts top-2, SwiGLU (BASELINE config 4)",
    "c4-f16": "Qwen3 MoE f16, 32768 tokens, H4096 I1536, 8 experts top-2 (BASELINE config 4)",
    "c5": "Qwen3-30B-A3B-shaped MoE layer bf16, 65536 tokens, H2048 I768, 128 experts top-8, "
          "SwiGLU, biased router (BASELINE config 5)",
}

# How each workload meets the "flush L2 or exceed it" timing rule (L2 is 126 MB)
L2_NOTES = {
    "c1": "inputs fit in L2 (16 KB of logits); one launch per step, launch-latency bound",
    "c2": "inputs larger than L2 (f32 weights 151 MB), no flush",
    "c3": "inputs larger than L2 (intermediate 403 MB + weights 75 MB per step), no flush",
    "c4": "inputs larger than L2 (weights 302 MB + activations), no flush",
    "c4-f16": "inputs larger than L2 (weights 302 MB + activations), no flush",
    "c5": "inputs larger than L2 (weights 1.2 GB + activations), no flush",
}
METRIC = "fused-MoE tokens/s"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_profile(kernel_key):
    """ncu figures of a kernel from the committed summaries (profiles/traffic.json): per-launch
    DRAM bytes (`dram_bytes`), tensor-pipe activity (`tensor_pipe_pct`), the kernel's name and
    the summary file they come from; {} when none was captured."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        v = json.load(open(p)).get(kernel_key)
        if isinstance(v, dict):
            return v
    return {}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in csv.reader(io.StringIO(out)):
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                mx = float(row[2])
            except ValueError:
                continue
            for n, v in zip(names, row[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        loaded = [s for s in sm if mx and s > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


_JSON_OUT = None


def reserve_stdout():
    """Keep stdout for the one JSON line: file descriptor 1 is pointed at stderr, so whatever
    native libraries print (NCCL prints its version banner at every debug level from VERSION up)
    lands there, and the JSON line is written to a saved copy of the original stdout."""
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def emit(line):
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, value):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(cfg, seed=0, rank=0, n_local_experts=None):
    """Seeded synthetic inputs on the current GPU: this rank's tokens and, with expert
    parallelism, only its n_local_experts experts."""
    import torch
    dtype, moe_type, act, T, H, I, E, k, renorm, bias_std = cfg
    El = E if n_local_experts is None else n_local_experts
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    bias = torch.randn(E, generator=g, device="cuda") * bias_std  # the router bias is global
    g.manual_seed(seed * 1000 + rank)
    logits = torch.randn(T, E, generator=g, device="cuda")
    if bias_std:
        logits += bias
    inp = {"logits": logits}
    if moe_type is None:
        return inp
    inp["x"] = torch.randn(T, H, generator=g, device="cuda").to(tdt)
    inp["gate"] = (torch.randn(El, H, I, generator=g, device="cuda") * 0.02).to(tdt)
    inp["up"] = (torch.randn(El, H, I, generator=g, device="cuda") * 0.02).to(tdt)
    inp["down"] = ((torch.randn(El, I, H, generator=g, device="cuda") * 0.02).to(tdt)
                   if moe_type == 0 else None)
    return inp


def run_ours(args, world, rank, local):
    import torch
    import candle_moe

    cfg = CONFIGS[args.config]
    dtype, moe_type, act, T, H, I, E, k, renorm, _ = cfg
    router_only = moe_type is None
    ep = world > 1 and not router_only and args.config == "c5"
    layer = None
    if ep:
        import expert_parallel
        layer = expert_parallel.ExpertParallelMoE(E, k, candle_moe.Activation(act),
                                                  mode=args.ep_mode, transport=args.ep_transport,
                                                  chunks=args.ep_chunks,
                                                  compute_groups=args.ep_groups)
        if args.sm_reserve >= 0:
            layer.sm_reserve = args.sm_reserve
        inp = make_inputs(cfg, seed=0, rank=rank, n_local_experts=layer.num_local)
        if args.ep_balance:
            # expert placement from the router's loads over every rank's tokens (16 experts per
            # GPU at 8 GPUs either way); the synthetic weights stand for the placed experts
            import torch.distributed as dist
            _, idx0, _ = candle_moe.topk_softmax(inp["logits"], k, renormalize=renorm)
            loads = torch.bincount(idx0.long().flatten().clamp(max=E), minlength=E + 1)[:E]
            dist.all_reduce(loads)
            loads = loads.tolist()
            slot = expert_parallel.balanced_placement(loads, world)
            layer.set_placement(slot)
            El = E // world
            per_rank = [0] * world
            for e in range(E):
                per_rank[slot[e] // El] += loads[e]
            contiguous = [sum(loads[r * El:(r + 1) * El]) for r in range(world)]
            mean = sum(loads) / world
            ep_placement = {"balanced": True,
                            "rank_assignments_max_over_mean": round(max(per_rank) / mean, 4),
                            "contiguous_max_over_mean": round(max(contiguous) / mean, 4)}
        else:
            ep_placement = {"balanced": False}
    else:
        inp = make_inputs(cfg, seed=0, rank=rank)
    moe = None if router_only else candle_moe.FusedMoE(E, k, candle_moe.Activation(act))
    stream = torch.cuda.current_stream()

    def step(logits, x):
        w, idx, _ = candle_moe.topk_softmax(logits, k, renormalize=renorm)
        if router_only:
            return w
        if ep:
            return layer.forward(x, inp["gate"], inp["up"], inp["down"], w, idx, moe_type)
        return moe.forward(x, inp["gate"], inp["up"], inp["down"], w, idx, moe_type)

    x_dev = None if router_only else inp["x"]
    for _ in range(args.warmup):
        step(inp["logits"], x_dev)
    torch.cuda.synchronize()
    graph = None
    if router_only:
        # one router launch is a few microseconds: replay a captured graph so the timing is the
        # kernel's, not Python's dispatch
        graph = torch.cuda.CUDAGraph()
        l0 = candle_moe.kernel_launches()
        with torch.cuda.graph(graph):
            step(inp["logits"], x_dev)
        launches_per_replay = candle_moe.kernel_launches() - l0
        graph.replay()
        torch.cuda.synchronize()

    # ---- device-resident timed region -------------------------------------------------------
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = candle_moe.kernel_launches()
    candle_moe.phase_timing(True)
    if ep:
        layer.timing = True
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step(inp["logits"], x_dev)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    candle_moe.phase_timing(False)
    if ep:
        layer.timing = False
    clk = clocks.stop()
    ms_total = ev0.elapsed_time(ev1)
    launches = candle_moe.kernel_launches() - launches0
    if graph is not None:
        launches = launches_per_replay * args.steps
    phases, ncalls = (candle_moe.phase_times() if not router_only else ({}, 0))
    ms_step = max_over_ranks(world, ms_total / args.steps)
    value = T * world / (ms_step / 1e3)

    # ---- end to end through the public API: host inputs in, host output out ------------------
    h_logits = inp["logits"].cpu().pin_memory()
    h_x = None if router_only else inp["x"].cpu().pin_memory()
    out_shape = (T, k) if router_only else (T, H)
    out_dtype = torch.float32 if router_only else inp["x"].dtype
    h_out = torch.empty(out_shape, dtype=out_dtype).pin_memory()
    h2d = h_logits.numel() * 4 + (0 if router_only else h_x.numel() * h_x.element_size())
    d2h = h_out.numel() * h_out.element_size()

    # Pipelined like a serving loop: the H2D copy of step i+1 and the D2H copy of step i-1 run
    # on side streams while step i computes; every step still moves its own inputs and output
    # across PCIe inside the timed region.
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    nbuf = 2
    d_lg = [torch.empty_like(inp["logits"]) for _ in range(nbuf)]
    d_x = [None if router_only else torch.empty_like(inp["x"]) for _ in range(nbuf)]
    h_outs = [h_out] + [torch.empty(out_shape, dtype=out_dtype).pin_memory()
                        for _ in range(nbuf - 1)]
    free_ev = [None] * nbuf

    def e2e_step(i):
        b = i % nbuf
        with torch.cuda.stream(s_in):
            if free_ev[b] is not None:
                s_in.wait_event(free_ev[b])
            d_lg[b].copy_(h_logits, non_blocking=True)
            if not router_only:
                d_x[b].copy_(h_x, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(s_in)
        stream.wait_event(ready)
        out = step(d_lg[b], d_x[b])
        fe = torch.cuda.Event()
        fe.record(stream)
        free_ev[b] = fe
        with torch.cuda.stream(s_out):
            s_out.wait_event(fe)
            h_outs[b].copy_(out, non_blocking=True)
            out.record_stream(s_out)

    for i in range(min(args.warmup, 3)):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    e0.record(s_in)
    for i in range(args.steps):
        e2e_step(i)
    s_out.wait_stream(stream)
    e1.record(s_out)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t_wall) * 1e3 / args.steps
    barrier(world)
    e2e_ms = max_over_ranks(world, e0.elapsed_time(e1) / args.steps)

    peaks, peak_kind = load_peaks()
    line = {
        "metric": METRIC if not router_only else "topk-softmax us",
        "value": value if not router_only else ms_step * 1e3,
        "unit": "tokens/s" if not router_only else "us",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": not router_only, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic (seeded torch.randn; weights N(0,0.02), hidden N(0,1))",
        "config": {"workload": WORKLOAD_NAMES[args.config], "tokens": T, "hidden": H,
                   "intermediate": I, "experts": E, "top_k": k,
                   "parallelism": (f"ep{world}" if ep else "replicas") if world > 1 else "single-gpu",
                   "ep_mode": args.ep_mode if ep else None,
                   "ep_transport": layer.transport if ep else None,
                   "tokens_per_rank": T,
                   "l2": L2_NOTES.get(args.config, "no flush") if not args.tokens else
                   "token count overridden (a profiling or decode case): no flush"},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if router_only:
        line["value"] = ms_step * 1e3
        # bytes a call must move: the logits in, the three [T, k] outputs out
        nbytes = T * (4 * E + 12 * k)
        line["roofline"] = {
            "kernel": "router_topk_softmax", "bound": "hbm",
            "achieved": nbytes / (ms_step / 1e3) / 1e9, "peak": peaks.get("hbm_gbs"),
            "unit": "GB/s", "frac": nbytes / (ms_step / 1e3) / 1e9 / peaks.get("hbm_gbs"),
            "peak_kind": f"{peak_kind} HBM copy", "traffic": None, "bytes_per_call": nbytes,
            "note": "launch-latency bound at this size (graph replay of one launch per step)"}
    if ep:
        st, n = layer.stage_times()
        line["ep_stages_ms"] = {s_: v / max(n, 1) for s_, v in st.items()}
        line["ep_rows"] = {k_: int(v) for k_, v in layer.last_stats.items()}
        line["ep_placement"] = ep_placement
        if layer.transport in ("push", "copy"):
            line["ep_timeline_ms"] = {k_: round(v, 3) for k_, v in layer.timeline().items()}
    if not router_only and ncalls:
        rows = layer.last_stats["assignments_received"] if ep else T * k
        n_up = 2 if moe_type == 0 else 1
        elt = 4 if dtype == "f32" else 2
        flops = {"gemm1": 2.0 * rows * H * I * n_up, "gemm2": 2.0 * rows * I * H}
        # algorithmic HBM bytes of one pass: each expert's weights once, each token row once,
        # the intermediate written and read once, the (token, slot) rows written once (k > 1)
        n_exp = layer.num_local if ep else E
        algo_bytes = {
            "gemm1": elt * (n_up * n_exp * H * I + T * H + rows * I),
            "gemm2": elt * (n_exp * I * H + rows * I + (rows * H if k > 1 else T * H)),
        }
        per_call = {p: phases[p] / ncalls for p in phases}
        per_step = {p: phases[p] / args.steps for p in phases}
        dom = max(("gemm1", "gemm2"), key=lambda p: per_call[p])
        # flops[] are per step; with expert parallelism a step makes several fused calls
        tflops = {p: flops[p] / (per_step[p] / 1e3) / 1e12 for p in ("gemm1", "gemm2")}
        step_tflops = (flops["gemm1"] + flops["gemm2"]) / (ms_step / 1e3) / 1e12
        if dtype == "f32" and candle_moe.last_gemm_path() == 2:
            # f32 on the tensor cores: three TF32 products per f32 product, and TF32 runs at
            # half the f16/bf16 dense rate, so the f32-equivalent peak is the measured bf16
            # burst / 6 (no TF32 peak is measured on this pool)
            peak = peaks.get("bf16_tflops") / 6.0
            peak_sus = peaks.get("bf16_tflops_sustained") / 6.0
            kernel, bound = "tf32x3_grouped_gemm", "tensor"
            kind = (f"{peak_kind} bf16 dense burst / 2 (TF32 rate) / 3 (products per f32 "
                    f"product); MEASURED_PEAKS.json")
        elif dtype == "f32":
            # the f32 path runs on the FP32 pipes (SIMT kernel); no measured FP32 peak exists
            # on this pool, so the nominal one: 148 SMs x 128 lanes x 2 FLOP x 1965 MHz
            peak = 148 * 128 * 2 * 1.965e9 / 1e12
            peak_sus = None
            kernel, bound, kind = "simt_grouped_gemm", "fp32", "nominal FP32 FFMA"
        else:
            # the GEMMs run a few ms at a time between lighter kernels, at the SM clock the
            # `clocks` key shows (near the maximum), so the denominator is the burst figure;
            # the fraction of the power-capped sustained figure is given beside it
            peak = peaks.get("bf16_tflops")
            peak_sus = peaks.get("bf16_tflops_sustained")
            kernel, bound = "sm100_grouped_gemm", "tensor"
            kind = (f"{peak_kind} bf16 dense, burst (cuBLAS 8192^3, best of 10); "
                    f"MEASURED_PEAKS.json")
        per_kernel = {}
        for ph in ("gemm1", "gemm2"):
            prof = load_profile(f"{args.config}:{ph}") if not ep else {}
            per_kernel[ph] = {
                "kernel": prof.get("kernel"), "ms_per_step": per_step[ph],
                "tflops": tflops[ph], "frac": tflops[ph] / peak,
                "frac_of_sustained": tflops[ph] / peak_sus if peak_sus else None,
                "algorithmic_bytes": algo_bytes[ph],
                "traffic": prof.get("dram_bytes"),
                "tensor_pipe_active_pct": prof.get("tensor_pipe_pct"),
                "profile": prof.get("source"),
            }
        line["roofline"] = {
            "kernel": per_kernel[dom]["kernel"] or f"{kernel} ({dom})", "phase": dom,
            "bound": bound, "achieved": tflops[dom], "peak": peak, "unit": "TFLOP/s",
            "frac": tflops[dom] / peak, "peak_kind": kind,
            "frac_of_sustained": tflops[dom] / peak_sus if peak_sus else None,
            "sm_mhz_median": clk.get("sm_mhz"),
            "traffic": per_kernel[dom]["traffic"],
            "algorithmic_bytes": algo_bytes[dom],
            "tensor_pipe_active_pct": per_kernel[dom]["tensor_pipe_active_pct"],
            "flops_per_step": flops[dom], "launches_per_step": ncalls // args.steps,
            "kernels": per_kernel,
            "step": {"tflops": step_tflops, "frac": step_tflops / peak,
                     "note": "both GEMMs' FLOPs over the whole step (router, route "
                             "preparation and combine included)"},
        }
        line["phases_ms"] = per_step
        line["tflops_total"] = step_tflops
    line["e2e"] = {"value": T * world / (e2e_ms / 1e3) if not router_only else e2e_ms * 1e3,
                   "unit": line["unit"], "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                   "ms_per_step": e2e_ms, "host_wall_ms_per_step": wall_ms,
                   "pipelining": "H2D of step i+1 and D2H of step i-1 overlap step i's compute"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not router_only:
        line["cpu_baseline"] = cpu_baseline(cfg, inp, target_s=args.cpu_seconds)
    if world == 1 and args.config == "c5" and not args.tokens and not args.no_extra:
        # the metric's other two figures, on their own BASELINE configs: config 1's router
        # microseconds and config 4's decode step (8 tokens)
        line["router_c1"] = measure_router_c1()
        line["decode_c4_t8"] = measure_decode_c4(8)
        line["router_projection_c5"] = measure_router_projection_c5()
    failed = False
    if ep:
        if not args.no_extra:
            line["strong_scaling"] = measure_ep_strong(args, world, inp, layer, renorm, k,
                                                       moe_type, T)
        # non-zero when an arrival wait of the exchange ran out (a rank never signalled): the
        # step's output is incomplete, so the run fails after its line is printed
        bits = int(max_over_ranks(world, candle_moe.device_error_bits(local)))
        line["device_error_bits"] = bits
        failed = bits != 0
        layer.close()
    if rank == 0:
        emit(line)
    if failed:
        raise SystemExit("expert-parallel exchange: an arrival wait ran out "
                         f"(device error bits {bits:#x})")


def measure_ep_strong(args, world, inp, layer, renorm, k, moe_type, T):
    """Strong scaling of the expert-parallel layer: BASELINE config 5's 65536 tokens split
    across the ranks (T / N each; the weak-scaling headline keeps T per rank).  Same timing
    rules: warm-up, barrier + synchronize around the timed steps, max over ranks."""
    import torch
    import candle_moe
    Ts = T // world
    logits = inp["logits"][:Ts].contiguous()
    x = inp["x"][:Ts].contiguous()

    def step():
        w, idx, _ = candle_moe.topk_softmax(logits, k, renormalize=renorm)
        return layer.forward(x, inp["gate"], inp["up"], inp["down"], w, idx, moe_type)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(world, e0.elapsed_time(e1) / args.steps)
    return {"tokens_total": Ts * world, "tokens_per_rank": Ts, "ms_per_step": ms,
            "value": Ts * world / (ms / 1e3), "unit": "tokens/s",
            "note": "BASELINE config 5's 65536 tokens split across the ranks (strong scaling)"}


def _graph_time_us(fn, reps, per_graph):
    """Device time per call of fn (which launches library kernels on the current stream): the
    calls are captured per_graph at a time into a CUDA graph, the graph is replayed `reps`
    times between CUDA events on the launching stream.  Returns (us per call, launches per
    call)."""
    import torch
    import candle_moe
    stream = torch.cuda.current_stream()
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    l0 = candle_moe.kernel_launches()
    with torch.cuda.graph(graph):
        for _ in range(per_graph):
            fn()
    launches = (candle_moe.kernel_launches() - l0) / per_graph
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * per_graph)
    del graph
    return us, launches


def measure_router_c1():
    """BASELINE config 1 (topk-softmax, [512, 8] f32 logits ~ N(0,1), top-2) through the drop-in
    apply_topk_softmax_inplace: device microseconds per call, CUDA-graph replay (the published
    reference figure, README.md:17, is wall-clock per call on an A40)."""
    import torch
    import candle_moe
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    T, E, k = 512, 8, 2
    logits = torch.randn(T, E, generator=g, device="cuda")
    w = torch.empty(T, k, device="cuda")
    idx = torch.empty(T, k, dtype=torch.int32, device="cuda")
    src = torch.empty(T, k, dtype=torch.int32, device="cuda")
    us, launches = _graph_time_us(
        lambda: candle_moe.apply_topk_softmax_inplace(logits, w, idx, src), 50, 20)
    nbytes = T * (4 * E + 12 * k)
    return {"us_per_call": us, "tokens": T, "experts": E, "top_k": k,
            "bytes_per_call": nbytes, "gb_per_s": nbytes / (us * 1e-6) / 1e9,
            "timing": "CUDA-graph replay, 20 calls per graph x 50 replays, CUDA events",
            "gpu_launches_per_call": launches}


def measure_decode_c4(tokens=8, dtype="bf16"):
    """BASELINE config 4 at decode size: Qwen3 SwiGLU, H4096, I1536, 8 experts, top-2,
    renormalised, `tokens` tokens.  One step = router + fused forward, timed as a CUDA-graph
    replay (the per-step host work of a Python loop would otherwise dominate).  Bound by the
    weight read: 3*H*I*elt bytes for every expert the step routes to."""
    import torch
    import candle_moe
    cfg = CONFIGS["c4" if dtype == "bf16" else "c4-f16"]
    cfg = cfg[:3] + (tokens,) + cfg[4:]
    _, moe_type, act, T, H, I, E, k, renorm, _ = cfg
    inp = make_inputs(cfg, seed=0)
    moe = candle_moe.FusedMoE(E, k, candle_moe.Activation(act))

    def step():
        w, idx, _ = candle_moe.topk_softmax(inp["logits"], k, renormalize=renorm)
        return moe.forward(inp["x"], inp["gate"], inp["up"], inp["down"], w, idx, moe_type)

    _, idx, _ = candle_moe.topk_softmax(inp["logits"], k, renormalize=renorm)
    n_exp = int(torch.unique(idx).numel())
    us, launches = _graph_time_us(step, 40, 10)
    nbytes = 3 * H * I * 2 * n_exp + 2 * T * H * 2 + T * E * 4
    peaks, kind = load_peaks()
    del inp
    torch.cuda.empty_cache()
    return {"us_per_step": us, "tokens": T, "dtype": dtype, "experts_routed": n_exp,
            "bytes_per_step": nbytes, "gb_per_s": nbytes / (us * 1e-6) / 1e9,
            "hbm_frac": nbytes / (us * 1e-6) / 1e9 / peaks["hbm_gbs"],
            "peak_kind": f"{kind} HBM copy", "gemm_path": candle_moe.last_gemm_path(),
            "timing": "CUDA-graph replay, 10 steps per graph x 40 replays, CUDA events",
            "gpu_launches_per_step": launches}


def measure_router_projection_c5():
    """The router's gate projection at config 5's shape (65536 tokens, H 2048, 128 experts,
    top-8, renormalised): the fused kernel (moe_router_project_topk) against the two-step path a
    model runs without it -- the Linear (torch, cuBLAS) to bf16 logits, cast to f32, then
    topk_softmax.  Device microseconds per call, CUDA-graph replay.  The fused kernel is bound
    by reading the hidden states once: T*H*2 + E*H*2 + T*k*12 bytes."""
    import torch
    import candle_moe
    T, H, E, k = 65536, 2048, 128, 8
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(E, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    fused_us, fused_launches = _graph_time_us(
        lambda: candle_moe.router_project_topk(x, w, k, renormalize=True), 20, 5)

    def two_step():
        logits = torch.nn.functional.linear(x, w).float()
        return candle_moe.topk_softmax(logits, k, renormalize=True)

    two_us, _ = _graph_time_us(two_step, 20, 5)
    nbytes = T * H * 2 + E * H * 2 + T * k * 12
    peaks, kind = load_peaks()
    del x, w
    torch.cuda.empty_cache()
    return {"fused_us": fused_us, "two_step_us": two_us, "speedup": two_us / fused_us,
            "tokens": T, "hidden": H, "experts": E, "top_k": k, "bytes_per_call": nbytes,
            "fused_gb_per_s": nbytes / (fused_us * 1e-6) / 1e9,
            "fused_hbm_frac": nbytes / (fused_us * 1e-6) / 1e9 / peaks["hbm_gbs"],
            "peak_kind": f"{kind} HBM copy",
            "two_step": "torch linear (cuBLAS) to bf16 logits, .float(), topk_softmax",
            "timing": "CUDA-graph replay, 5 calls per graph x 20 replays, CUDA events",
            "gpu_launches_per_call": fused_launches}


def cpu_baseline(cfg, inp, target_s=10.0):
    """The reference algorithm (CPU oracle port, all host threads) on a token sample."""
    import numpy as np
    import oracle
    oracle.set_num_threads(os.cpu_count() or 1)
    dtype, moe_type, act, T, H, I, E, k, renorm, _ = cfg

    def raw(t):
        import torch
        t = t.contiguous().cpu()
        if t.dtype == torch.float32:
            return t.numpy()
        return t.view(torch.int16).numpy().view(np.uint16)

    G, U = raw(inp["gate"]), raw(inp["up"])
    D = raw(inp["down"]) if inp["down"] is not None else None
    logits = inp["logits"].cpu().numpy()
    x_all = raw(inp["x"])

    def run(n):
        w, idx, _, _ = oracle.topk_softmax(logits[:n], k, renormalize=renorm)
        t0 = time.perf_counter()
        oracle.moe_forward(x_all[:n], G, U, D, w, idx, activation=act, moe_type=moe_type,
                           dtype=dtype)
        return time.perf_counter() - t0

    n = min(T, 256)
    dt = run(n)
    n2 = int(min(T, max(n, n * target_s / max(dt, 1e-3))))
    dt = run(n2)
    return {"value": n2 / dt, "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"first {n2} tokens of the workload, {dt:.1f} s",
            "seconds": dt}


def run_reference(args, world, rank):
    """Reference arm: the reference's algorithm on the host cores (CPU oracle port)."""
    if rank != 0:
        return
    import numpy as np
    import oracle
    # all host threads, whatever OMP_NUM_THREADS the launcher exported (torchrun sets 1)
    oracle.set_num_threads(os.cpu_count() or 1)
    cfg = CONFIGS[args.config]
    dtype, moe_type, act, T, H, I, E, k, renorm, bias_std = cfg
    # the same seeded distributions as our arm, generated on the host
    logits = oracle.randn(11, (T, E))
    if bias_std:
        logits = np.ascontiguousarray(logits + oracle.randn(12, (E,), std=bias_std)[None, :])
    if moe_type is None:
        sample = T
        run = lambda: oracle.topk_softmax(logits, k, renormalize=renorm)  # noqa: E731
    else:
        x = oracle.randn(13, (T, H), dtype=dtype)
        G = oracle.randn(14, (E, H, I), std=0.02, dtype=dtype)
        U = oracle.randn(15, (E, H, I), std=0.02, dtype=dtype)
        D = oracle.randn(16, (E, I, H), std=0.02, dtype=dtype) if moe_type == 0 else None
        sample = min(T, args.ref_sample)

        def run():
            w, idx, _, _ = oracle.topk_softmax(logits[:sample], k, renormalize=renorm)
            oracle.moe_forward(x[:sample], G, U, D, w, idx, activation=act, moe_type=moe_type,
                               dtype=dtype)
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = (time.perf_counter() - t0) / args.steps
    router_only = moe_type is None
    value = dt * 1e6 if router_only else sample / dt
    unit = "us" if router_only else "tokens/s"
    line = {
        "impl": "reference", "metric": METRIC if not router_only else "topk-softmax us",
        "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": not router_only,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD_NAMES[args.config], "tokens": T, "hidden": H,
                   "intermediate": I, "experts": E, "top_k": k},
        "cpu_baseline": {"value": value, "unit": unit, "cores": oracle.num_threads(),
                         "kind": "port",
                         "sample": f"{sample} of {T} tokens per step (router + naive "
                                   "per-expert loop, f32 accumulate, OpenMP)"},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference crate has no CPU implementation; this is its algorithm restated "
                "in C (oracle/) on the host cores",
    }
    emit(line)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c5")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-sample", type=int, default=512)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the config-1 router and config-4 decode figures of the default run")
    ap.add_argument("--ep-mode", choices=["partials", "exact"], default="partials",
                    help="expert-parallel return: per-rank partial sums or per-slot rows")
    ap.add_argument("--ep-transport", choices=["push", "copy", "collective"], default="push",
                    help="expert-parallel row exchange into peer-mapped landing buffers by SM "
                         "stores fused with pack / slot sum (push) or by copy engines (copy), "
                         "or NCCL all_to_all_single (collective)")
    ap.add_argument("--ep-groups", type=lambda v: [int(a) for a in v.split(",")], default=None,
                    help="expert parallelism: chunks computed per fused call, e.g. 1,3,3,1 "
                         "(sums to --ep-chunks; default one chunk per call)")
    ap.add_argument("--ep-balance", action=argparse.BooleanOptionalAction, default=False,
                    help="expert parallelism: place experts by the router's loads "
                         "(balanced_placement) instead of contiguous ranges (off by default: "
                         "the synthetic router's per-rank loads are within 8 %% of even)")
    ap.add_argument("--ep-chunks", type=int, default=4,
                    help="expert-parallel token chunks pipelined through dispatch/compute/return")
    ap.add_argument("--sm-reserve", type=int, default=-1,
                    help="SMs the GEMMs leave to the NCCL exchange (expert parallel; -1 = default)")
    ap.add_argument("--gemm-path", type=int, default=0, choices=[0, 1, 2, 3, 4, 5, 6],
                    help="expert GEMM family: 0 automatic, 1 SIMT, 2 tensor cores, 3 "
                         "automatic without CTA pairs, 4 automatic with GEMM-1 on CTA pairs too "
                         "(experimental), 5 automatic without the decode kernels, 6 decode "
                         "kernels at any size")
    ap.add_argument("--tokens", type=int, default=0,
                    help="override the token count (small profiling cases)")
    args = ap.parse_args()
    if args.tokens:
        CONFIGS[args.config] = CONFIGS[args.config][:3] + (args.tokens,) + CONFIGS[args.config][4:]
        WORKLOAD_NAMES[args.config] += f" [tokens overridden: {args.tokens}]"
    args.warmup = max(args.warmup, 3)
    reserve_stdout()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    if args.gemm_path:
        import candle_moe
        candle_moe.set_gemm_path(args.gemm_path)
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
