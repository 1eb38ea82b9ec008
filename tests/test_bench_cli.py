"""bench.py's command line and its CPU-only reference arm (the driver runs
both at the end of every round): the options parse, and `--impl reference`
prints one JSON line with the keys the driver reads, timed on a bounded
sample of the CPU reference path."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_bench_options_parse():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                       timeout=120, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--allreduce", "--allreduce-overlap", "--collect",
                "--c4-action", "--profile-minibatch", "--profile-collect", "--fused-minibatch"):
        assert opt in r.stdout, opt


def test_reference_arm_prints_its_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    for k in ("metric", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "dtype", "data", "config"):
        assert k in d, k
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the record describes what ran: one timed sample (--steps 1) after one
    # warm-up sample, each sample's wall time, and the GPU arm's config
    assert d["steps"] == 1 and d["warmup"] == 1 and 1e3 <= d["ms_per_step"] <= 60e3
    sys.path.insert(0, str(ROOT))
    import bench

    assert d["config"] == bench.workload_config(1)
