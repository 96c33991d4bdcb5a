"""bench.py prints one JSON line per run with a fixed set of keys; these tests run it in a
subprocess and check that line (the reference arm on the CPU, our arm on a GPU)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "e2e"}


def run_bench(*args, timeout):
    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=timeout)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, proc.stdout[-2000:]
    return json.loads(lines[0])


def test_default_workload_is_the_largest_single_gpu_config():
    """With no flags the bench measures the 4.59M-entity configuration (uncapped, frontier
    pruned to 0.5% of the entities) on the key-slab engine."""
    sys.path.insert(0, str(ROOT))
    import bench
    from minikg_dev_b200.synth import UNCAPPED, WORKLOADS
    saved = sys.argv
    try:
        sys.argv = ["bench.py"]
        a = bench.parse()
    finally:
        sys.argv = saved
    wl = WORKLOADS[a.workload]
    assert a.workload == "kg_large" and a.gpus == 1 and a.warmup >= 3
    assert (wl.E, wl.R, wl.T, wl.B, wl.L, wl.hops) == (4594485, 822, 20624575, 256, 4, 2)
    assert wl.topk_edges == UNCAPPED and wl.topk_nodes == 22972 and wl.capped_row == 100
    assert a.workload in bench.SLAB_WORKLOADS


def test_reference_arm_line():
    """--impl reference: the oracle port on the host cores, same metric and workload as our arm,
    with its own cpu_baseline and an e2e that moves no bytes (the mid-size workload, to keep the
    test short)."""
    d = run_bench("--impl", "reference", "--workload", "kg_mid", "--steps", "1", "--warmup", "0", timeout=600)
    assert BASE_KEYS <= set(d) and d["impl"] == "reference"
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"] == "kg_mid"
    cb = d["cpu_baseline"]
    assert {"value", "unit", "cores", "kind", "sample"} <= set(cb) and cb["value"] == d["value"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["unit"] == d["unit"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def _check_gpu_line(d, workload):
    assert BASE_KEYS <= set(d) and "impl" not in d
    assert d["steps"] == 2 and d["warmup"] == 3 and d["value"] > 0
    assert d["config"]["workload"] == workload
    rl = d["roofline"]
    assert {"bound", "achieved", "peak", "unit", "frac", "traffic"} <= set(rl)
    assert rl["bound"] == "hbm" and rl["unit"] == "GB/s" and rl["peak"] > 0
    assert rl["frac"] == pytest.approx(rl["achieved"] / rl["peak"])
    e2e = d["e2e"]
    assert e2e["value"] > 0 and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] > 0 and e2e["d2h_bytes_per_step"] > 0
    assert d["gpu_launches"] > 0
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(d["clocks"])


@pytest.mark.gpu
def test_gpu_arm_line():
    """Our arm on the default workload: whole-job value, roofline of the dominant kernel,
    end-to-end figure with its copy sizes, launch count and the clocks seen."""
    d = run_bench("--steps", "2", "--warmup", "3", "--no-cpu-baseline", "--no-extras", timeout=900)
    _check_gpu_line(d, "kg_large")
    assert d["scaling"] == "strong" and d["config"]["messages_per_step"] > 10_000_000


@pytest.mark.gpu
def test_gpu_arm_line_fused_workload():
    """The fused loop's line on the mid-size workload."""
    d = run_bench("--workload", "kg_mid", "--steps", "2", "--warmup", "3", "--no-cpu-baseline", timeout=900)
    _check_gpu_line(d, "kg_mid")
    assert "decode" in d and d["decode"]["roofline"]["frac"] > 0
