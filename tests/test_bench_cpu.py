"""bench.py's output contract, checked through its CPU-only reference arm: exactly one JSON line
on stdout with the keys the round driver reads (metric, value, unit, e2e, cpu_baseline, ...)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_prints_one_contract_line():
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "3", "--ref-sample", "16")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["warmup"] == 3
    assert d["metric"] == "fused-MoE tokens/s" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["tokens"] == 65536 and d["config"]["experts"] == 128


def test_reference_arm_router_config_reports_microseconds():
    d = _run("--impl", "reference", "--config", "c1", "--steps", "2", "--warmup", "3")
    assert d["metric"] == "topk-softmax us" and d["unit"] == "us"
    assert d["higher_is_better"] is False and d["value"] > 0


def test_reference_arm_warmup_is_at_least_three():
    d = _run("--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "1")
    assert d["warmup"] == 3
