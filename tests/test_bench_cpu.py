"""bench.py's contract checked without a GPU: the reference arm's JSON line
(the reference's CPU path on a bounded sample) and the workload table."""

import json
import subprocess
import sys
from pathlib import Path

import bench

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3",
                        "--warmup", "3", "--cpu-seconds", "0.3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["unit"] == "GB/s"
    assert d["config"]["workload"] == bench.DEFAULT_WORKLOAD
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_workload_table():
    for name, wl in bench.WORKLOADS.items():
        assert wl["kind"] in ("w4a16", "fp8", "dense"), name
        assert wl["M"] > 0 and wl["N"] > 0 and wl["K"] > 0, name
        if "ncu_traffic" in wl:  # DRAM bytes of a committed capture, with its file
            nbytes, source = wl["ncu_traffic"]
            assert nbytes > 0 and (ROOT / source).is_file(), (name, source)
    assert bench.DEFAULT_WORKLOAD in bench.WORKLOADS
