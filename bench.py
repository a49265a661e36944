#!/usr/bin/env python
"""Benchmark of the B200 quantized-matmul path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Default workload: W4A16 decode GEMM, Llama-7B q_proj shape (M=1, K=N=4096,
int4 weights with group-128 bf16 scales, bf16 activations, fp32 output) --
the configuration BASELINE.json's headline metric is quoted on. A step is
one GEMM over one set of weights; 32 rotating weight sets (277 MB) keep every
step's weights out of the 126 MB L2. Steps are launched from CUDA graphs.

Multi-GPU (torchrun, one process per GPU): the GEMMs are independent, so each
rank runs its own stream of steps (weak scaling, no data-path collective);
time is the max over ranks. The sharded Llama-70B configurations with an
NCCL all-gather of the output are separate workloads (--workload llama70b_*).

--impl reference times the reference's CPU path (the numpy restatement in
oracle/, dequantize-then-matmul in fp32) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "W4A16 GEMM µs & HBM GB/s at M=1/16, TFLOPS at M=4096; fp8 GEMM TFLOPS"
L2_BYTES = 126 * 2 ** 20

WORKLOADS = {
    "w4a16_decode_m1": dict(kind="w4a16", M=1, N=4096, K=4096),
    "w4a16_decode_m4": dict(kind="w4a16", M=4, N=4096, K=4096),
    "w4a16_decode_m16": dict(kind="w4a16", M=16, N=4096, K=4096),
}
DEFAULT_WORKLOAD = "w4a16_decode_m1"


# ---------------------------------------------------------------------------
# peaks and clocks
# ---------------------------------------------------------------------------
def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML on a thread."""

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples: list[tuple[float, int, int]] = []
        self.period = period_s
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = device_index
            if vis:
                ids = [v.strip() for v in vis.split(",") if v.strip()]
                if device_index < len(ids) and ids[device_index].isdigit():
                    idx = int(ids[device_index])
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are best-effort metadata
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def start(self):
        if self._nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()

    def stop(self):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()

    def summary(self, t0: float, t1: float) -> dict:
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win and self.samples:  # timed region shorter than the sampling period
            mid = 0.5 * (t0 + t1)
            win = sorted(self.samples, key=lambda s: abs(s[0] - mid))[:3]
        mhz = [s[1] for s in win]
        bits = 0
        for s in win:
            bits |= s[2]
        reasons = sorted(name for b, name in _REASONS.items() if bits & b and b != 0x1)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(win)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    if world <= 1:
        return None
    import datetime

    import torch.distributed as dist
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist


def max_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


# ---------------------------------------------------------------------------
# W4A16 workload
# ---------------------------------------------------------------------------
def w4a16_bytes(M: int, N: int, K: int) -> int:
    """Algorithmic bytes of one GEMM: packed weights + bf16 scales + bf16 A + fp32 Y."""
    return K * N // 2 + (K // 128) * N * 2 + M * K * 2 + M * N * 4


def make_w4a16_sets(M, N, K, n_sets, device, seed=0):
    import pico_kernels_b200 as pk
    g = torch.Generator(device=device).manual_seed(seed)
    sets = []
    for i in range(n_sets):
        w = (torch.randn(K, N, device=device, generator=g) * 0.02).to(torch.bfloat16)
        packed, scales = pk.quantize_int4_grouped(w, 128)
        a = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
        sets.append((a, packed, scales))
        del w
    torch.cuda.synchronize()
    return sets


def time_graph_steps(step_fn, n_sets: int, steps: int, chunk: int = 1000):
    """Capture `step_fn(i)` for i in a chunk into graphs; return (run(K), n_graph_steps)."""
    chunk = max(1, min(chunk, steps))
    graphs = {}

    def graph_for(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step_fn(0)  # make sure lazily created buffers exist outside capture
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=s):
                    for i in range(n):
                        step_fn(i % n_sets)
            torch.cuda.current_stream().wait_stream(s)
            graphs[n] = g
        return graphs[n]

    def run(k):
        full, rem = divmod(k, chunk)
        gfull = graph_for(chunk) if full else None
        grem = graph_for(rem) if rem else None
        return gfull, full, grem

    return run


def run_ours(args, wl: dict, world: int, rank: int, local: int) -> None:
    import pico_kernels_b200 as pk
    from pico_kernels_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(world, local)
    peaks = load_peaks()
    M, N, K = wl["M"], wl["N"], wl["K"]
    per_step = w4a16_bytes(M, N, K)
    n_sets = max(4, int(2 * L2_BYTES // (K * N // 2 + (K // 128) * N * 2)) + 1)
    sets = make_w4a16_sets(M, N, K, n_sets, device)
    outs = [torch.empty((M, N), dtype=torch.float32, device=device) for _ in range(n_sets)]
    lib = _lib.load()
    split = args.split_k
    ws_bytes = lib.pk_w4a16_workspace_size(M, N, K, split)
    ws = _lib.workspace(device, ws_bytes, tag="bench")
    sms = torch.cuda.get_device_properties(device).multi_processor_count

    def step(i):
        a, packed, scales = sets[i]
        _lib.check(lib.pk_w4a16_gemm(a.data_ptr(), _lib.PK_BF16, K, packed.data_ptr(),
                                     scales.data_ptr(), 1.0, 128, M, N, K, outs[i].data_ptr(),
                                     _lib.PK_F32, N, split, _lib.ptr(ws), ws_bytes,
                                     torch.cuda.current_stream().cuda_stream), "w4a16")

    runner = time_graph_steps(step, n_sets, args.steps)
    # warm-up: W steps through the same graphs
    gw, nw, gwr = runner(args.warmup)
    for _ in range(nw):
        gw.replay()
    if gwr is not None:
        gwr.replay()
    gfull, nfull, grem = runner(args.steps)
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.05)
    barrier(dist)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record()
    for _ in range(nfull):
        gfull.replay()
    if grem is not None:
        grem.replay()
    ev1.record()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier(dist)
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(dist, ms)
    code, where = pk.device_status()
    if code != 0:
        raise RuntimeError(f"device status {code} at site {where}")

    # end-to-end through the public API: pinned host A in, fp32 Y out, every step
    e2e_steps = min(args.steps, args.e2e_steps)
    a_host = [torch.empty((M, K), dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    y_host = [torch.empty((M, N), dtype=torch.float32).pin_memory() for _ in range(4)]
    for h, (a, _, _) in zip(a_host, sets):
        h.copy_(a)
    a_dev = torch.empty((M, K), dtype=torch.bfloat16, device=device)

    def e2e_step(i):
        _, packed, scales = sets[i % n_sets]
        a_dev.copy_(a_host[i % 4], non_blocking=True)
        y = pk.int4_gemm(a_dev, packed, scales)
        y_host[i % 4].copy_(y, non_blocking=True)

    for i in range(max(3, args.warmup // 100)):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(dist, e0.elapsed_time(e1))

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return

    ms_per_step = ms_max / args.steps
    value = world * per_step * args.steps / (ms_max * 1e-3) / 1e9
    achieved = per_step / (ms / args.steps * 1e-3) / 1e9
    e2e_value = world * per_step * e2e_steps / (e2e_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "us_per_gemm": round(ms_per_step * 1e3, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights quantized on device, N(0,1) activations)",
        "config": {
            "workload": args.workload, "M": M, "N": N, "K": K, "group_size": 128,
            "weights": "int4 packed [K, N/2] + bf16 scales [K/128, N]",
            "activations": "bf16", "output": "fp32",
            "split_k": split if split > 0 else "auto",
            "l2": f"{n_sets} rotating weight sets ({n_sets * (K * N // 2 + K // 128 * N * 2) / 2**20:.0f} MiB > 126 MiB L2)",
            "launch": "CUDA graphs of back-to-back GEMMs",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
        },
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
            "peak_source": peaks["source"], "traffic": args.traffic,
            "algorithmic_bytes_per_launch": per_step, "sms": sms,
        },
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 4,
                "steps": e2e_steps, "us_per_step": round(e2e_ms / e2e_steps * 1e3, 3),
                "path": "pico_kernels_b200.int4_gemm (ctypes C ABI) with pinned host buffers"},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(t0, t1),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(M, N, K, budget_s=args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU reference path (oracle restatement of the reference's torch CPU path)
# ---------------------------------------------------------------------------
def _cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def cpu_baseline(M: int, N: int, K: int, budget_s: float = 10.0) -> dict:
    """Time unpack + dequantize + fp32 matmul per step on the host (numpy)."""
    from oracle import quant_ref as o
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((K, N), dtype=np.float32) * 0.02)
    codes, s32 = o.group_quant_codes(w, 128)
    packed = o.pack_int4_n(codes)
    scales = o.store_scales(s32, "bf16")
    a = o.round_to_bf16(rng.standard_normal((M, K), dtype=np.float32))
    per_step = w4a16_bytes(M, N, K)
    n = 0
    t0 = time.perf_counter()
    while True:
        q = o.unpack_int4_n(packed)
        o.w4a16_reference(a, q, scales, 128)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s and n >= 2:
            break
    return {"value": round(per_step * n / el / 1e9, 5), "unit": "GB/s",
            "cores": _cpu_threads(), "kind": "port",
            "sample": f"{n} steps of unpack+dequant+fp32 matmul, M={M} N={N} K={K}, {el:.1f} s",
            "ms_per_step": round(el / n * 1e3, 3)}


def run_reference(args, wl: dict, world: int, rank: int) -> None:
    if rank != 0:
        return
    M, N, K = wl["M"], wl["N"], wl["K"]
    steps = args.steps
    # each step is a bounded sample: the CPU path is ~1e4x slower than the GPU
    budget = args.cpu_seconds
    base = cpu_baseline(M, N, K, budget_s=budget)
    line = {
        "metric": METRIC, "value": base["value"], "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": base["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": args.workload, "M": M, "N": N, "K": K, "group_size": 128},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=2000)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--split-k", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=2000)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per launch from an ncu capture, reported as-is")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_env()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl, world, rank)
    else:
        run_ours(args, wl, world, rank, local)


if __name__ == "__main__":
    main()
