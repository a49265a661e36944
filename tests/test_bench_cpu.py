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
    # the same config dict as the GPU arm prints for this workload
    assert d["config"] == bench.workload_config(bench.DEFAULT_WORKLOAD,
                                                bench.WORKLOADS[bench.DEFAULT_WORKLOAD], 1)
    assert d["cpu_baseline"]["kind"] == "port" and "torch" in d["cpu_baseline"]["sample"]
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_workload_table():
    for name, wl in bench.WORKLOADS.items():
        assert wl["kind"] in ("w4a16", "fp8", "dense"), name
        assert wl["M"] > 0 and wl["N"] > 0 and wl["K"] > 0, name
        if "ncu_traffic" in wl:  # DRAM bytes per launch from an ncu capture
            assert wl["ncu_traffic"] > 0, name
        n_sets, set_bytes = bench.input_sets(wl, 1)
        assert n_sets * set_bytes > 2 * bench.L2_BYTES, name
    assert bench.DEFAULT_WORKLOAD in bench.WORKLOADS
    sharded = bench.WORKLOADS[bench.DEFAULT_SHARDED_WORKLOAD]
    assert sharded.get("sharded") and sharded["M"] == 1
    for world in (2, 4, 8):
        cfg = bench.workload_config(bench.DEFAULT_SHARDED_WORKLOAD, sharded, world)
        assert f"sharded over {world} GPUs" in cfg["parallelism"]


def test_cpu_reference_matches_the_oracle():
    """The timed CPU computation is the reference's dequantize-then-matmul:
    its codes and scales are the oracle's, and its product the oracle's."""
    import numpy as np
    import torch

    from oracle import cpu_reference as ref
    from oracle import quant_ref as o
    step = ref.W4A16Step(M=2, K=256, cols=64)
    y = step().numpy()
    codes = step.q.numpy()
    s = step.scales.float().numpy()
    assert np.allclose(y, o.w4a16_reference(step.a.float().numpy(), codes, s, 128),
                       rtol=1e-5, atol=1e-5)
    w = (torch.randn(256, 64, generator=torch.Generator().manual_seed(0)) * 0.02)
    c2, s2 = o.group_quant_codes(w.to(torch.bfloat16).float().numpy(), 128)
    assert np.array_equal(c2, codes)
    assert np.array_equal(o.store_scales(s2, "bf16"), s)
