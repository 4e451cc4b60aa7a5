"""bench.py's output contract, on the CPU: the reference arm (`--impl reference`, the
oracle timed on the host cores) prints one JSON line with the keys the driver reads, on
the same metric, unit and config as the GPU arm; fewer than 3 warm-up steps are refused.
Runs a 2-layer model so the check takes seconds (a reported number always uses 36)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config"}


def _run(*extra, timeout=300):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *extra], capture_output=True, text=True,
                          timeout=timeout, cwd=ROOT)


def test_reference_arm_line():
    out = _run("--impl", "reference", "--layers", "2", "--steps", "2", "--warmup", "3", "--cpu-seconds", "1")
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert BASE_KEYS <= set(d), BASE_KEYS - set(d)
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["metric"] == "decode tok/s (batch 1, SmolLM3-3B Q4)"
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 2 and d["warmup"] == 3
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cb) and cb["kind"] in ("port", "reference")
    assert cb["value"] == d["value"] and cb["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_warmup_below_three_is_refused():
    out = _run("--impl", "reference", "--layers", "2", "--steps", "2", "--warmup", "2", timeout=120)
    assert out.returncode != 0 and "warmup" in out.stderr


def test_reference_arm_gemv_line():
    """Config 1 (the Q4 GEMV alone, GB/s): the reference arm times the oracle's gemv_q4."""
    out = _run("--impl", "reference", "--workload", "q4-gemv", "--steps", "5", "--warmup", "3", "--cpu-seconds", "1")
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][-1])
    assert BASE_KEYS <= set(d) and d["unit"] == "GB/s" and d["value"] > 0 and d["steps"] >= 5
    assert d["config"]["bytes_per_gemv"] == 2048 * 11008 // 2 + 2048 * 11008 // 32 * 2 + 2048 * 4 + 11008 * 4
    assert d["cpu_baseline"]["unit"] == "GB/s"
