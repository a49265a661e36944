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
    # HBM-bound decode GEMMs: metric GB/s of algorithmic bytes
    "w4a16_decode_m1": dict(kind="w4a16", M=1, N=4096, K=4096,
                            ncu_traffic=(8.69e6, "profiles/w4a16_gemv_m1_4096.md")),
    "w4a16_decode_m4": dict(kind="w4a16", M=4, N=4096, K=4096),
    "w4a16_decode_m16": dict(kind="w4a16", M=16, N=4096, K=4096),
    # tensor-bound prefill GEMM: metric TFLOP/s
    "w4a16_prefill": dict(kind="w4a16", M=4096, N=11008, K=4096,
                          ncu_traffic=(368e6, "profiles/w4a16_prefill_4096x11008x4096.md")),
    # scaled e4m3 GEMMs: metric TFLOP/s, cast excluded as upstream
    "fp8_2048": dict(kind="fp8", M=2048, N=2048, K=2048),
    "fp8_4096": dict(kind="fp8", M=4096, N=4096, K=4096,
                     ncu_traffic=(34.3e6, "profiles/fp8_gemm_4096.md")),
    "fp8_8192": dict(kind="fp8", M=8192, N=8192, K=8192),
    # dense bf16 GEMM, fp32 out (gemm.py:103, the comparison partner of the
    # split-K kernel): metric TFLOP/s
    "dense_bf16_4096": dict(kind="dense", M=4096, N=4096, K=4096),
    "dense_bf16_8192": dict(kind="dense", M=8192, N=8192, K=8192),
    # Llama-70B MLP layers sharded along N over the ranks, output all-gathered
    # with NCCL; strong scaling: the layer is fixed, ranks split it
    "llama70b_up_m1": dict(kind="w4a16", M=1, N=28672, K=8192, sharded=True),
    "llama70b_up_m32": dict(kind="w4a16", M=32, N=28672, K=8192, sharded=True),
    "llama70b_up_m256": dict(kind="w4a16", M=256, N=28672, K=8192, sharded=True,
                             ncu_traffic=(129.6e6, "profiles/w4a16_skinny_m256_llama70b_up.md")),
    "llama70b_down_m1": dict(kind="w4a16", M=1, N=8192, K=28672, sharded=True),
    "llama70b_down_m32": dict(kind="w4a16", M=32, N=8192, K=28672, sharded=True),
    "llama70b_down_m256": dict(kind="w4a16", M=256, N=8192, K=28672, sharded=True),
    "llama70b_up_fp8_m4096": dict(kind="fp8", M=4096, N=28672, K=8192, sharded=True),
}
DEFAULT_WORKLOAD = "w4a16_decode_m1"


def is_hbm_bound(wl: dict) -> bool:
    """Decode-sized W4A16 GEMMs are bound by streaming the weights; the rest by
    the tensor cores (2*M*N*K at the bf16 peak vs the weight bytes at HBM peak)."""
    if wl["kind"] != "w4a16":
        return False
    M, N, K = wl["M"], wl["N"], wl["K"]
    t_flops = 2.0 * M * N * K / 1654e12
    t_bytes = (K * N / 2 + K / 128 * N * 2) / 6553e9
    return t_bytes >= t_flops


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
# workloads: device buffers, one step through the C ABI, algorithmic work
# ---------------------------------------------------------------------------
class Workload:
    """Rotating input sets (so each step's inputs are not L2-resident) and the
    step that runs one GEMM on set i through the C ABI.

    Sharded workloads: every rank builds the same seeded layer and keeps its
    contiguous slice of N columns; a step is one kernel per rank that also
    writes every rank's output (the fused exchange), or, where no kernel with
    the exchange covers the shape or ``exchange`` is False, the local GEMM
    then the NCCL all-gather of the [M, N/p] blocks into [M, N] (reordered for
    M > 1)."""

    def __init__(self, name: str, wl: dict, device: torch.device, split_k: int,
                 world: int = 1, rank: int = 0, dist=None, exchange: bool = True):
        from pico_kernels_b200 import _lib
        self.name, self.wl, self.device = name, wl, device
        self.lib = _lib.load()
        self._lib = _lib
        self.M, self.N, self.K = wl["M"], wl["N"], wl["K"]
        self.kind = wl["kind"]
        self.split_k = split_k
        self.hbm = is_hbm_bound(wl)
        self.sharded = bool(wl.get("sharded"))
        self.world = world if self.sharded else 1
        self.rank = rank if self.sharded else 0
        self.dist = dist
        M, N, K = self.M, self.N, self.K
        if self.sharded and (N % self.world or (N // self.world) % 128):
            raise ValueError(f"N={N} does not shard over {self.world} ranks")
        self.NL = N // self.world                      # local columns
        n0 = self.rank * self.NL
        if self.kind == "w4a16":
            per_set = K * self.NL // 2 + (K // 128) * self.NL * 2 + M * K * 2
        elif self.kind == "dense":
            per_set = (M * K + K * self.NL) * 2
        else:
            per_set = M * K + K * self.NL
        self.n_sets = max(2, int(2 * L2_BYTES // per_set) + 1)
        self.set_bytes = per_set
        g = torch.Generator(device=device).manual_seed(0)
        self.sets = []
        import pico_kernels_b200 as pk
        from pico_kernels_b200 import gemm_fp8
        for _ in range(self.n_sets):
            if self.kind == "w4a16":
                w = (torch.randn(K, N, device=device, generator=g) * 0.02).to(torch.bfloat16)
                packed, scales = pk.quantize_int4_grouped(w, 128)
                del w
                if self.sharded:
                    packed = packed[:, n0 // 2:(n0 + self.NL) // 2].contiguous()
                    scales = scales[:, n0:n0 + self.NL].contiguous()
                a = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
                self.sets.append((a, packed, scales))
            elif self.kind == "dense":
                a = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
                b = torch.randn(K, N, device=device, generator=g).to(torch.bfloat16)
                self.sets.append((a, b))
            else:
                a8, sa = gemm_fp8.quantize(torch.randn(M, K, device=device, generator=g).to(torch.bfloat16))
                b8, sb = gemm_fp8.quantize(torch.randn(K, N, device=device, generator=g).to(torch.bfloat16))
                if self.sharded:
                    b8 = b8[:, n0:n0 + self.NL].contiguous()
                self.sets.append((a8, b8, 1.0 / (sa * sb)))
        torch.cuda.empty_cache()
        # fp8 layers write bf16 (configs[3]: "bf16 output rescaled in the epilogue")
        self.out_dtype = torch.bfloat16 if self.kind == "fp8" else torch.float32
        self.out_code = _lib.PK_BF16 if self.kind == "fp8" else _lib.PK_F32
        # decode outputs are tiny: one per set; large outputs share one buffer
        n_out = self.n_sets if self.hbm else 1
        self.outs = [torch.empty((M, self.NL), dtype=self.out_dtype, device=device)
                     for _ in range(n_out)]
        if self.sharded and self.world > 1:
            self.gather = torch.empty((self.world * M, self.NL), dtype=self.out_dtype, device=device)
            self.full = torch.empty((M, N), dtype=self.out_dtype, device=device)
        self.ws_bytes = (self.lib.pk_w4a16_workspace_size(M, self.NL, K, split_k)
                         if self.kind == "w4a16" else 0)
        self.ws = _lib.workspace(device, self.ws_bytes, tag="bench")
        # sharded W4A16 layers whose local kernel is the GEMV, the decode or
        # the skinny kernel: it writes every rank's output itself
        # (pk_w4a16_gemm_sharded); one probe call per rank decides, and every
        # rank gets the same answer (the kernel choice depends on the shape only)
        self.exchange = None
        if (exchange and self.sharded and self.world > 1 and self.kind == "w4a16"
                and split_k == 0 and M <= 256):
            from pico_kernels_b200 import sharded
            self.exchange = sharded.PeerExchange(max_m=M, n_full=N, dtype=self.out_dtype)
            ex = self.exchange
            self.ex_ws_bytes = max(self.lib.pk_w4a16_workspace_size(M, self.NL, K, 0), 1 << 16)
            self.ex_ws = _lib.workspace(device, self.ex_ws_bytes, tag="exchange")
            import ctypes
            self.ex_outs = [(ctypes.c_uint64 * self.world)(*[b + par * ex.buf_bytes for b in ex.bases])
                            for par in (0, 1)]
            self.ex_flags = (ctypes.c_uint64 * self.world)(*[b + ex.flag_off for b in ex.bases])
            self.ex_calls = 0
            if self.fused_call(0) == _lib.PK_ERR_UNSUPPORTED:
                ex.close()  # collective, like the constructor
                self.exchange = None
        torch.cuda.synchronize()

    def gemm(self, i: int) -> torch.Tensor:
        lib, L, M, K, NL = self.lib, self._lib, self.M, self.K, self.NL
        stream = torch.cuda.current_stream().cuda_stream
        out = self.outs[i % len(self.outs)]
        if self.kind == "w4a16":
            a, packed, scales = self.sets[i]
            st = lib.pk_w4a16_gemm(a.data_ptr(), L.PK_BF16, K, packed.data_ptr(), scales.data_ptr(),
                                   1.0, 128, M, NL, K, out.data_ptr(), self.out_code, NL,
                                   self.split_k, L.ptr(self.ws), self.ws_bytes, stream)
        elif self.kind == "dense":
            a, b = self.sets[i]
            st = lib.pk_gemm_splitk(a.data_ptr(), b.data_ptr(), L.PK_BF16, M, NL, K, 1,
                                    out.data_ptr(), None, 0, stream)
        else:
            a8, b8, out_scale = self.sets[i]
            st = lib.pk_fp8_gemm(a8.data_ptr(), b8.data_ptr(), M, NL, K, out_scale, out.data_ptr(),
                                 self.out_code, stream)
        L.check(st, self.name)
        return out

    def all_gather(self, local: torch.Tensor) -> None:
        self.dist.all_gather_into_tensor(self.gather, local)
        if self.M > 1:
            self.full.copy_(self.gather.view(self.world, self.M, self.NL).permute(1, 0, 2)
                            .reshape(self.M, self.N))

    def fused_call(self, i: int) -> int:
        import ctypes
        lib, L, M, K, NL = self.lib, self._lib, self.M, self.K, self.NL
        a, packed, scales = self.sets[i]
        self.ex_calls += 1
        outs = self.ex_outs[self.ex_calls & 1]
        st = lib.pk_w4a16_gemm_sharded(
            a.data_ptr(), L.PK_BF16, K, packed.data_ptr(), scales.data_ptr(), 1.0, 128, M, NL, K,
            self.out_code, self.N, self.rank * NL, self.world, self.rank, ctypes.addressof(outs),
            ctypes.addressof(self.ex_flags), L.ptr(self.ex_ws), self.ex_ws_bytes,
            torch.cuda.current_stream().cuda_stream)
        if st != L.PK_OK:
            self.ex_calls -= 1
        return st

    def fused_step(self, i: int) -> None:
        self._lib.check(self.fused_call(i), self.name + " (fused exchange)")

    def step(self, i: int) -> None:
        if self.exchange is not None:
            self.fused_step(i)
            return
        out = self.gemm(i)
        if self.sharded and self.world > 1:
            self.all_gather(out)

    def gemm_only(self, i: int) -> None:
        self.gemm(i)

    def gather_only(self, i: int) -> None:
        self.all_gather(self.outs[i % len(self.outs)])

    # algorithmic work of one step (the whole layer, all ranks together)
    def bytes_per_step(self) -> int:
        M, N, K = self.M, self.N, self.K
        if self.kind == "w4a16":
            return K * N // 2 + (K // 128) * N * 2 + M * K * 2 + M * N * 4
        if self.kind == "dense":
            return (M * K + K * N) * 2 + M * N * 4
        return M * K + K * N + M * N * 2

    def flops_per_step(self) -> int:
        return 2 * self.M * self.N * self.K

    def e2e_step_fn(self):
        """Public-API step with host buffers: H2D of the activations, D2H of Y."""
        import pico_kernels_b200 as pk
        from pico_kernels_b200 import gemm_fp8, sharded
        M, N, K, NL = self.M, self.N, self.K, self.NL
        y_host = torch.empty((M, N), dtype=self.out_dtype).pin_memory()
        world = self.world if self.sharded else 1
        if self.kind == "w4a16":
            a_host = torch.empty((M, K), dtype=torch.bfloat16).pin_memory()
            a_host.copy_(self.sets[0][0])
            a_dev = torch.empty((M, K), dtype=torch.bfloat16, device=self.device)

            if world == 1:
                # one public call with host buffers: H2D of A, the GEMM, D2H of
                # Y, all inside pk_w4a16_gemm_host
                def fn(i):
                    _, packed, scales = self.sets[i % self.n_sets]
                    pk.int4_gemm_host(a_host, packed, scales, group_size=128, out=y_host)
                return fn, M * K * 2, M * N * 4

            # sharded: the exchange's or NCCL's output buffer
            def fn(i):
                _, packed, scales = self.sets[i % self.n_sets]
                a_dev.copy_(a_host, non_blocking=True)
                y = sharded.sharded_int4_gemm(a_dev, packed, scales, 128, world,
                                              exchange=self.exchange)
                y_host.copy_(y, non_blocking=True)
            return fn, M * K * 2, M * N * 4
        if self.kind == "dense":
            from pico_kernels_b200 import gemm
            a_host = torch.empty((M, K), dtype=torch.bfloat16).pin_memory()
            a_host.copy_(self.sets[0][0])
            a_dev = torch.empty((M, K), dtype=torch.bfloat16, device=self.device)

            def fn(i):
                _, b = self.sets[i % self.n_sets]
                a_dev.copy_(a_host, non_blocking=True)
                y_host.copy_(gemm.triton_gemm(a_dev, b), non_blocking=True)
            return fn, M * K * 2, M * N * 4
        a8_host = torch.empty((M, K), dtype=torch.uint8).pin_memory()
        a8_host.copy_(self.sets[0][0].view(torch.uint8))
        a8_dev = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=self.device)

        def fn(i):
            _, b8, out_scale = self.sets[i % self.n_sets]
            a8_dev.view(torch.uint8).copy_(a8_host, non_blocking=True)
            y = sharded.sharded_fp8_gemm(a8_dev, 1.0, b8, 1.0 / out_scale, world,
                                         out_dtype=torch.bfloat16)
            y_host.copy_(y, non_blocking=True)
        return fn, M * K, M * N * 2


def capture_runner(step_fn, n_sets: int, steps: int, chunk: int = 1000):
    """CUDA graphs of `chunk` consecutive steps (cycling the input sets); returns
    (graph, replays, remainder_graph) covering exactly `steps` steps."""
    chunk = max(1, min(chunk, steps))
    graphs = {}

    def graph_for(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step_fn(0)  # lazily created state exists before capture
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=s):
                    for i in range(n):
                        step_fn(i % n_sets)
            torch.cuda.current_stream().wait_stream(s)
            graphs[n] = g
        return graphs[n]

    full, rem = divmod(steps, chunk)
    return (graph_for(chunk) if full else None), full, (graph_for(rem) if rem else None)


def _time_graphs(runner_out, dist) -> float:
    """Replay (graph, n, remainder) on the device; return ms (max over ranks)."""
    g, n, grem = runner_out
    barrier(dist)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        g.replay()
    if grem is not None:
        grem.replay()
    e1.record()
    torch.cuda.synchronize()
    return max_over_ranks(dist, e0.elapsed_time(e1))


def run_ours(args, wl: dict, world: int, rank: int, local: int) -> None:
    import pico_kernels_b200 as pk

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = init_dist(world, local)
    peaks = load_peaks()
    work = Workload(args.workload, wl, device, args.split_k, world, rank, dist,
                    exchange=args.exchange == "fused")
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    chunk = 1000 if work.hbm else 20
    gathered = work.sharded and world > 1

    warm = capture_runner(work.step, work.n_sets, args.warmup, chunk)
    for _ in range(warm[1]):
        warm[0].replay()
    if warm[2] is not None:
        warm[2].replay()
    timed = capture_runner(work.step, work.n_sets, args.steps, chunk)
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.05)
    barrier(dist)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record()
    for _ in range(timed[1]):
        timed[0].replay()
    if timed[2] is not None:
        timed[2].replay()
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

    # sharded layers: time the local GEMM and the all-gather on their own too
    breakdown = None
    gemm_ms_local = ms
    if gathered:
        nb = min(args.steps, 1000 if work.hbm else 50)
        g_gemm = capture_runner(work.gemm_only, work.n_sets, nb, chunk)
        g_gath = capture_runner(work.gather_only, work.n_sets, nb, chunk)
        gemm_ms = _time_graphs(g_gemm, dist)
        gath_ms = _time_graphs(g_gath, dist)
        gemm_ms_local = gemm_ms * args.steps / nb
        breakdown = {"gemm_us": round(gemm_ms / nb * 1e3, 3),
                     "allgather_us": round(gath_ms / nb * 1e3, 3), "steps": nb}
        if work.exchange is not None:
            breakdown["step"] = ("one kernel per rank: the local GEMM stores its columns into "
                                 "every rank's output over NVLink and ends with a flag barrier; "
                                 "gemm_us / allgather_us time the unfused local GEMM and an "
                                 "NCCL all-gather of its output for comparison")
        del g_gemm, g_gath

    # end to end through the public API, host buffers in and out every step
    e2e_fn, h2d, d2h = work.e2e_step_fn()
    e2e_steps = min(args.steps, args.e2e_steps if work.hbm else max(3, args.e2e_steps // 100))
    for i in range(3):
        e2e_fn(i)
    torch.cuda.synchronize()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        e2e_fn(i)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(dist, e0.elapsed_time(e1))
    del warm, timed  # graphs holding NCCL calls go before the process group
    if work.exchange is not None:
        work.exchange.close()  # collective: every rank unmaps its peers
    torch.cuda.synchronize()

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return

    sec = ms_max * 1e-3
    # roofline of the dominant kernel: this rank's GEMM launch
    sec_per_launch = gemm_ms_local * 1e-3 / args.steps
    replicas = 1 if work.sharded else world
    if work.hbm:
        per = work.bytes_per_step()
        local_per = per if not work.sharded else (
            work.K * work.NL // 2 + (work.K // 128) * work.NL * 2 + work.M * work.K * 2 + work.M * work.NL * 4)
        unit, scale = "GB/s", 1e9
        peak, bound, punit = peaks["hbm_gbs"], "hbm", "GB/s"
        peak_note = peaks["source"]
    else:
        per = work.flops_per_step()
        local_per = per // (world if work.sharded else 1)
        unit, scale = "TFLOP/s", 1e12
        long_region = sec > 1.0
        bf16 = peaks["bf16_tflops_sustained"] if long_region else peaks["bf16_tflops"]
        if work.kind == "fp8":
            peak = 2.0 * bf16
            peak_note = f"2x {'sustained' if long_region else 'burst'} bf16 ({peaks['source']}); no fp8 peak measured"
        else:
            peak = bf16
            peak_note = f"{'sustained' if long_region else 'burst'} bf16 ({peaks['source']})"
        bound, punit = "tensor", "TFLOP/s"
    # DRAM bytes per launch of the dominant kernel: --traffic, else the figure
    # of the committed ncu capture of this workload's kernel (single GPU only:
    # a shard's kernel reads a different slice)
    traffic, traffic_src = args.traffic, "--traffic" if args.traffic is not None else None
    if traffic is None and "ncu_traffic" in wl and (world == 1 or not work.sharded):
        traffic, traffic_src = wl["ncu_traffic"]
        traffic_src = f"ncu dram__bytes_read.sum + dram__bytes_write.sum, {traffic_src}"
    value = replicas * per * args.steps / sec / scale
    achieved = local_per / sec_per_launch / scale
    e2e_value = replicas * per * e2e_steps / (e2e_ms * 1e-3) / scale
    wl_cfg = {"workload": args.workload, "M": work.M, "N": work.N, "K": work.K}
    if work.kind == "w4a16":
        wl_cfg.update({"group_size": 128, "weights": "int4 packed [K, N/2] + bf16 scales [K/128, N]",
                       "activations": "bf16", "output": "fp32",
                       "split_k": args.split_k if args.split_k > 0 else "auto"})
    elif work.kind == "dense":
        wl_cfg.update({"inputs": "bf16 [M,K] x bf16 [K,N]", "output": "fp32"})
    else:
        wl_cfg.update({"inputs": "e4m3 [M,K] x e4m3 [K,N], per-tensor scales",
                       "output": "bf16 (rescaled in the epilogue)",
                       "cast": "excluded from the timed region (gemm_fp8.py:144)"})
    if work.sharded:
        if world == 1:
            par = "single GPU (unsharded)"
        elif work.exchange is not None:
            par = (f"N sharded over {world} GPUs ({work.NL} columns each), output exchanged inside "
                   "the local GEMM kernel (NVLink peer stores + flag barrier)")
        else:
            par = f"N sharded over {world} GPUs ({work.NL} columns each), NCCL all-gather of the output"
    
    else:
        par = f"replicas x{world}" if world > 1 else "single GPU"
    wl_cfg.update({
        "l2": f"{work.n_sets} rotating input sets per GPU ({work.n_sets * work.set_bytes / 2**20:.0f} MiB > 126 MiB L2)",
        "launch": "CUDA graphs of back-to-back steps",
        "parallelism": par,
    })
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "us_per_gemm": round(ms_max / args.steps * 1e3, 4),
        "higher_is_better": True,
        "scaling": "strong" if work.sharded else "weak",
        "vs_baseline": None,
        "dtype": "e4m3" if work.kind == "fp8" else "bf16",
        "data": "synthetic (seeded N(0,0.02) weights quantized on device, N(0,1) activations)",
        "config": wl_cfg,
        "roofline": {
            "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": punit,
            "frac": round(achieved / peak, 4), "peak_source": peak_note,
            "traffic": traffic, "traffic_source": traffic_src,
            ("algorithmic_bytes_per_launch" if work.hbm else "algorithmic_flops_per_launch"): local_per,
            "sms": sms,
        },
        "e2e": {"value": round(e2e_value, 4), "unit": unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "us_per_step": round(e2e_ms / e2e_steps * 1e3, 3),
                "path": ("pico_kernels_b200.int4_gemm_host -> pk_w4a16_gemm_host (H2D of A, "
                         "the GEMM and D2H of y in one C-ABI call), pinned host buffers"
                         if work.kind == "w4a16" and not (work.sharded and world > 1) else
                         "pico_kernels_b200 public API (ctypes C ABI), pinned host buffers")},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(t0, t1),
    }
    if breakdown is not None:
        line["breakdown"] = breakdown
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl, budget_s=args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU reference path (the oracle's restatement of the reference's torch path)
# ---------------------------------------------------------------------------
def _cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def cpu_baseline(wl: dict, budget_s: float = 10.0) -> dict:
    """Time the reference's CPU path on a bounded sample of the workload.

    W4A16: unpack + dequantize + fp32 matmul (tests/test_gemm_int4.py:26);
    fp8: (a8.float()/sa) @ (b8.float()/sb) (gemm_fp8.py:132); dense: fp32
    matmul of the bf16 inputs (gemm.py:134-142). Large GEMMs are
    sampled by output rows; the rate is scaled to the full step's unit.
    """
    from oracle import quant_ref as o
    M, N, K = wl["M"], wl["N"], wl["K"]
    rng = np.random.default_rng(0)
    rows = M if M <= 16 else max(16, min(M, int(2e9 // (2 * N * K)) or 16))
    if wl["kind"] == "w4a16":
        w = rng.standard_normal((K, N), dtype=np.float32) * 0.02
        codes, s32 = o.group_quant_codes(w, 128)
        packed = o.pack_int4_n(codes)
        scales = o.store_scales(s32, "bf16")
        a = o.round_to_bf16(rng.standard_normal((rows, K), dtype=np.float32))

        def once():  # per step: unpack + dequantize the weights
            return o.dequant_weight(o.unpack_int4_n(packed), scales, 128)

        def per_rows(wd):  # fp32 matmul of `rows` activation rows
            return a @ wd
    elif wl["kind"] == "dense":
        a = o.round_to_bf16(rng.standard_normal((rows, K), dtype=np.float32))
        b = o.round_to_bf16(rng.standard_normal((K, N), dtype=np.float32))

        def once():
            return b

        def per_rows(bd):  # gemm.py:134-142 checks against a.float() @ b.float()
            return a @ bd
    else:
        a8, sa = o.fp8_quantize(rng.standard_normal((rows, K), dtype=np.float32), "bf16")
        b8, sb = o.fp8_quantize(rng.standard_normal((K, N), dtype=np.float32), "bf16")

        def once():
            return o.e4m3_bits_to_f32(b8) / np.float32(sb)

        def per_rows(bd):
            return (o.e4m3_bits_to_f32(a8) / np.float32(sa)) @ bd
    n = 0
    t_once = t_rows = 0.0
    t0 = time.perf_counter()
    while True:
        ta = time.perf_counter()
        wd = once()
        tb = time.perf_counter()
        per_rows(wd)
        tc = time.perf_counter()
        t_once += tb - ta
        t_rows += tc - tb
        n += 1
        el = tc - t0
        if el >= budget_s and n >= 2:
            break
    prep = {"w4a16": "weight dequant", "fp8": "B e4m3 -> f32", "dense": "no weight prep"}[wl["kind"]]
    # one full step = one dequant + the matmul over all M rows
    sec_per_step = t_once / n + (t_rows / n) * (M / rows)
    hbm = is_hbm_bound(wl)
    if hbm:
        per = K * N // 2 + (K // 128) * N * 2 + M * K * 2 + M * N * 4
        value, unit = per / sec_per_step / 1e9, "GB/s"
    else:
        value, unit = 2 * M * N * K / sec_per_step / 1e12, "TFLOP/s"
    return {"value": round(value, 6), "unit": unit, "cores": _cpu_threads(), "kind": "port",
            "sample": f"{n} repetitions of ({prep} + matmul of {rows} of {M} rows), "
                      f"M={M} N={N} K={K}, {el:.1f} s, scaled to all rows; numpy restatement "
                      f"of the reference's torch CPU path",
            "ms_per_step": round(sec_per_step * 1e3, 3)}


def run_reference(args, wl: dict, world: int, rank: int) -> None:
    if rank != 0:
        return
    base = cpu_baseline(wl, budget_s=args.cpu_seconds)
    line = {
        "metric": METRIC, "value": base["value"], "unit": base["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": base["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": args.workload, "M": wl["M"], "N": wl["N"], "K": wl["K"]},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": base["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 100000 for decode, 200 otherwise)")
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--split-k", type=int, default=0)
    ap.add_argument("--exchange", choices=["fused", "nccl"], default="fused",
                    help="sharded W4A16 layers: output exchange inside the kernel where it "
                         "covers the shape, or always the NCCL all-gather")
    ap.add_argument("--e2e-steps", type=int, default=2000)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per launch from an ncu capture, reported as-is")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    hbm = is_hbm_bound(wl)
    if args.steps is None:
        args.steps = 100000 if hbm else 200
    if args.warmup is None:
        args.warmup = 2000 if hbm else 20
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, wl, world, rank)
    else:
        run_ours(args, wl, world, rank, local)


if __name__ == "__main__":
    main()
