#!/usr/bin/env python
"""Benchmark of the B200 quantized-matmul path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Default workload on one GPU: W4A16 decode GEMM, Llama-7B q_proj shape (M=1,
K=N=4096, int4 weights with group-128 bf16 scales, bf16 activations, fp32
output) -- the configuration BASELINE.json's headline metric is quoted on. A
step is one GEMM over one set of weights; rotating weight sets (> 2x the
126 MB L2) keep every step's weights out of L2. Steps are launched from CUDA
graphs; each graph is replayed once before the timed region.

Default workload on N > 1 GPUs (torchrun, one process per GPU): the
Llama-70B up_proj layer at M=1 (K=8192, N=28672) with
its columns sharded over the ranks and the output exchanged inside the
kernel over NVLink (strong scaling). Rank 0 first times the same layer on
its GPU alone (``strong_scaling``), and after the timed region every rank
checks its assembled [M, N] output against the unsharded GEMM on its own GPU
(``parity``). Time is the max over ranks.

--impl reference times the reference's CPU torch computation of the same
workload (oracle/cpu_reference.py) on all host cores, rank 0 only.
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

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "W4A16 GEMM µs & HBM GB/s at M=1/16, TFLOPS at M=4096; fp8 GEMM TFLOPS"
L2_BYTES = 126 * 2 ** 20

WORKLOADS = {
    # HBM-bound decode GEMMs: metric GB/s of algorithmic bytes
    "w4a16_decode_m1": dict(kind="w4a16", M=1, N=4096, K=4096, ncu_traffic=8.71e6),
    "w4a16_decode_m2": dict(kind="w4a16", M=2, N=4096, K=4096),
    "w4a16_decode_m3": dict(kind="w4a16", M=3, N=4096, K=4096),
    "w4a16_decode_m4": dict(kind="w4a16", M=4, N=4096, K=4096),
    "w4a16_decode_m8": dict(kind="w4a16", M=8, N=4096, K=4096),
    "w4a16_decode_m16": dict(kind="w4a16", M=16, N=4096, K=4096),
    # tensor-bound prefill GEMM: metric TFLOP/s
    "w4a16_prefill": dict(kind="w4a16", M=4096, N=11008, K=4096, ncu_traffic=368e6),
    # scaled e4m3 GEMMs: metric TFLOP/s, cast excluded as upstream
    "fp8_2048": dict(kind="fp8", M=2048, N=2048, K=2048),
    "fp8_4096": dict(kind="fp8", M=4096, N=4096, K=4096, ncu_traffic=34.3e6),
    "fp8_8192": dict(kind="fp8", M=8192, N=8192, K=8192),
    # dense bf16 GEMM, fp32 out (gemm.py:103, the comparison partner of the
    # split-K kernel): metric TFLOP/s
    "dense_bf16_4096": dict(kind="dense", M=4096, N=4096, K=4096),
    "dense_bf16_8192": dict(kind="dense", M=8192, N=8192, K=8192),
    # Llama-70B MLP layers sharded along N over the ranks, output all-gathered
    # with NCCL; strong scaling: the layer is fixed, ranks split it
    "llama70b_up_m1": dict(kind="w4a16", M=1, N=28672, K=8192, sharded=True),
    "llama70b_up_m4": dict(kind="w4a16", M=4, N=28672, K=8192, sharded=True),
    "llama70b_up_m8": dict(kind="w4a16", M=8, N=28672, K=8192, sharded=True),
    "llama70b_up_m32": dict(kind="w4a16", M=32, N=28672, K=8192, sharded=True),
    "llama70b_up_m256": dict(kind="w4a16", M=256, N=28672, K=8192, sharded=True,
                             ncu_traffic=129.6e6),
    "llama70b_down_m1": dict(kind="w4a16", M=1, N=8192, K=28672, sharded=True),
    "llama70b_down_m32": dict(kind="w4a16", M=32, N=8192, K=28672, sharded=True),
    "llama70b_down_m256": dict(kind="w4a16", M=256, N=8192, K=28672, sharded=True),
    "llama70b_up_fp8_m4096": dict(kind="fp8", M=4096, N=28672, K=8192, sharded=True),
}
DEFAULT_WORKLOAD = "w4a16_decode_m1"
DEFAULT_SHARDED_WORKLOAD = "llama70b_up_m1"  # the default under torchrun (N > 1)


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
def input_sets(wl: dict, world: int) -> tuple[int, int]:
    """(rotating input sets, bytes per set) so that one pass over the sets
    reads more than twice the L2 on every rank."""
    M, N, K = wl["M"], wl["N"], wl["K"]
    NL = N // world if wl.get("sharded") else N
    if wl["kind"] == "w4a16":
        per_set = K * NL // 2 + (K // 128) * NL * 2 + M * K * 2
    elif wl["kind"] == "dense":
        per_set = (M * K + K * NL) * 2
    else:
        per_set = M * K + K * NL
    return max(2, int(2 * L2_BYTES // per_set) + 1), per_set


def workload_config(name: str, wl: dict, world: int) -> dict:
    """The workload's identity, the same in both arms' lines: shape, data
    types, input rotation and how the GPUs share it."""
    M, N, K = wl["M"], wl["N"], wl["K"]
    cfg = {"workload": name, "M": M, "N": N, "K": K}
    if wl["kind"] == "w4a16":
        cfg.update({"group_size": 128, "weights": "int4 packed [K, N/2] + bf16 scales [K/128, N]",
                    "activations": "bf16", "output": "fp32"})
    elif wl["kind"] == "dense":
        cfg.update({"inputs": "bf16 [M,K] x bf16 [K,N]", "output": "fp32"})
    else:
        cfg.update({"inputs": "e4m3 [M,K] x e4m3 [K,N], per-tensor scales",
                    "output": "bf16 (rescaled in the epilogue)",
                    "cast": "excluded from the timed region (gemm_fp8.py:144)"})
    sharded = bool(wl.get("sharded"))
    n_sets, set_bytes = input_sets(wl, world)
    if sharded and world > 1:
        par = f"N sharded over {world} GPUs ({N // world} columns each), output assembled on every GPU"
    elif sharded:
        par = "single GPU (unsharded)"
    else:
        par = f"replicas x{world}" if world > 1 else "single GPU"
    cfg.update({
        "l2": f"{n_sets} rotating input sets per GPU ({n_sets * set_bytes / 2**20:.0f} MiB > 126 MiB L2)",
        "launch": "CUDA graphs of back-to-back steps",
        "parallelism": par,
    })
    return cfg


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
        self.n_sets, self.set_bytes = input_sets(wl, self.world)
        g = torch.Generator(device=device).manual_seed(0)
        self.sets = []
        import pico_kernels_b200 as pk
        from pico_kernels_b200 import gemm_fp8
        for _ in range(self.n_sets):
            if self.kind == "w4a16":
                w = (torch.randn(K, N, device=device, generator=g) * 0.02).to(torch.bfloat16)
                packed, scales = pk.quantize_int4_grouped(w, 128)
                del w
                if self.sharded and self.world > 1:
                    if not self.sets:  # the whole layer of set 0, for the parity check
                        self.full0 = (packed, scales)
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

    def step_output(self, i: int) -> torch.Tensor:
        """Run one step on set ``i`` and return this rank's assembled [M, N]."""
        if self.exchange is not None:
            self.fused_step(i)
            return self.exchange.output(self.ex_calls & 1, self.M)
        out = self.gemm(i)
        if not (self.sharded and self.world > 1):
            return out
        self.all_gather(out)
        return self.gather.view(1, self.N) if self.M == 1 else self.full

    def parity(self) -> float:
        """Relative Frobenius difference between this rank's assembled output of
        set 0 and the unsharded GEMM of the whole layer on this GPU."""
        import pico_kernels_b200 as pk
        a = self.sets[0][0]
        packed, scales = self.full0
        ref = pk.int4_gemm(a, packed, scales, group_size=128)
        y = self.step_output(0).float()
        torch.cuda.synchronize()
        return float(torch.norm(y - ref) / torch.norm(ref))

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


def capture_timed(step_fn, n_sets: int, steps: int, chunk: int, ev0, ev1) -> list:
    """CUDA graphs covering exactly `steps` steps, replayed in list order, with
    the start event recorded as the first node of the first graph and the stop
    event as the last node of the last (events created with external=True):
    the events then bracket the steps' device time alone, not the launch of
    the first graph."""
    chunk = max(1, min(chunk, steps))
    full, rem = divmod(steps, chunk)
    counts = [chunk] * full + ([rem] if rem else [])
    graphs: dict = {}

    def graph(n, first, last):
        key = (n, first, last)
        if key not in graphs:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step_fn(0)  # lazily created state exists before capture
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=s):
                    if first:
                        ev0.record()
                    for i in range(n):
                        step_fn(i % n_sets)
                    if last:
                        ev1.record()
            torch.cuda.current_stream().wait_stream(s)
            graphs[key] = g
        return graphs[key]

    return [graph(n, i == 0, i == len(counts) - 1) for i, n in enumerate(counts)]


def _replay(runner_out) -> None:
    g, n, grem = runner_out
    for _ in range(n):
        g.replay()
    if grem is not None:
        grem.replay()


def _prime(runner_out) -> None:
    """Replay each graph of a runner once, untimed: a graph's first launch
    uploads it to the device, which must not land in the timed region."""
    g, n, grem = runner_out
    if g is not None and n:
        g.replay()
    if grem is not None:
        grem.replay()
    torch.cuda.synchronize()


def _gate(dist=None) -> None:
    """Hold the stream for ~0.1 ms before the start event, so that the graph
    launches behind it are already queued when timing starts: the timed
    region then holds the steps' device time, not the host's submission.
    With several ranks a one-element NCCL all-reduce follows on the stream:
    it ends on every GPU at about the same time, so the ranks' timed regions
    start together instead of one host's lag each (sharded steps wait for
    each other, and a late rank would count its lag into the others' time)."""
    torch.cuda._sleep(200_000)
    if dist is not None:
        dist.all_reduce(torch.zeros(1, device="cuda"))


def _time_graphs(runner_out, dist) -> float:
    """Replay (graph, n, remainder) on the device; return ms (max over ranks)."""
    _prime(runner_out)
    barrier(dist)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _gate(dist)
    e0.record()
    _replay(runner_out)
    e1.record()
    torch.cuda.synchronize()
    return max_over_ranks(dist, e0.elapsed_time(e1))


def single_gpu_leg(args, wl: dict, device: torch.device) -> dict:
    """The whole sharded layer on this GPU alone (before the process group
    forms), timed like the sharded run: the strong-scaling reference point."""
    work = Workload(args.workload, wl, device, args.split_k, world=1, rank=0)
    steps = max(args.warmup, min(args.steps, 2000 if work.hbm else 50))
    chunk = 1000 if work.hbm else 20
    warm = capture_runner(work.step, work.n_sets, args.warmup, chunk)
    _replay(warm)
    timed = capture_runner(work.step, work.n_sets, steps, chunk)
    ms = _time_graphs(timed, None)
    per = work.bytes_per_step() if work.hbm else work.flops_per_step()
    us = ms / steps * 1e3
    out = {"single_gpu_us": round(us, 3), "steps": steps,
           "single_gpu_value": round(per / (us * 1e-6) / (1e9 if work.hbm else 1e12), 3)}
    del warm, timed, work
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def phase_leg(work, chunk: int) -> dict:
    """Per-CTA phase times of the last launch in a chain of 64 steps, from the
    %globaltimer stamps the decode GEMVs write (pk_debug_phase_stamps):
    microseconds from the launch's first CTA entry, median and max over CTAs."""
    from pico_kernels_b200 import _lib
    lib = _lib.load()
    rows = 4 * torch.cuda.get_device_properties(work.device).multi_processor_count
    buf = torch.zeros((rows, 8), dtype=torch.int64, device=work.device)
    torch.cuda.synchronize()
    _lib.check(lib.pk_debug_phase_stamps(buf.data_ptr(), buf.numel() * 8), "phase stamps")
    try:
        runner = capture_runner(work.step, work.n_sets, 64, chunk)
        _replay(runner)
        torch.cuda.synchronize()
    finally:
        lib.pk_debug_phase_stamps(None, 0)
    # rows [half][cta]: launches alternate between the halves, so they hold
    # the last launch and the one before it (the later entries: the last)
    raw = buf.cpu().view(2, rows // 2, 8)
    ctas = int((raw[0, :, 0] > 0).sum())
    if ctas == 0:
        return {"ctas": 0}
    h0, h1 = raw[0, :ctas].double(), raw[1, :ctas].double()
    prev, st = (h0, h1) if h1[:, 1].min() > h0[:, 1].min() else (h1, h0)
    t0 = st[:, 0].min()

    def stat(x):
        x = x / 1e3
        return {"median": round(float(x.median()), 3), "max": round(float(x.max()), 3)}
    return {
        "ctas": ctas, "sms": int(st[:, 5].unique().numel()),
        "gap_after_previous_launch_us": round(float((st[:, 1].min() - prev[:, 7].max()) / 1e3), 3),
        "entry_us": stat(st[:, 0] - t0),
        "wait_released_us": stat(st[:, 1] - t0),
        "first_weights_after_wait_us": stat(st[:, 2] - st[:, 1]),
        "arithmetic_us": stat(st[:, 3] - st[:, 2]),
        "reduction_and_store_us": stat(st[:, 4] - st[:, 3]),
        "after_store_to_exit_us": stat(st[:, 7] - st[:, 4]),
        "end_us": stat(st[:, 7] - t0),
        "note": ("last launch of a 64-step chain; times from its first CTA's entry "
                 "(%globaltimer); the gap runs from the previous launch's last CTA end to "
                 "this launch's dependency wait returning"),
    }


def run_ours(args, wl: dict, world: int, rank: int, local: int) -> None:
    import pico_kernels_b200 as pk
    from pico_kernels_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.weight_staging is not None:
        _lib.check(_lib.load().pk_set_weight_staging(args.weight_staging), "weight staging")
    sharded_run = bool(wl.get("sharded")) and world > 1
    strong = single_gpu_leg(args, wl, device) if sharded_run and rank == 0 else None
    dist = init_dist(world, local)
    peaks = load_peaks()
    work = Workload(args.workload, wl, device, args.split_k, world, rank, dist,
                    exchange=args.exchange == "fused")
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    chunk = 1000 if work.hbm else 20

    warm = capture_runner(work.step, work.n_sets, args.warmup, chunk)
    _replay(warm)
    ev0 = torch.cuda.Event(enable_timing=True, external=True)
    ev1 = torch.cuda.Event(enable_timing=True, external=True)
    timed = capture_timed(work.step, work.n_sets, args.steps, chunk, ev0, ev1)
    for g in dict.fromkeys(timed):  # each graph's first launch uploads it: untimed
        g.replay()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.05)
    barrier(dist)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _gate(dist)
    for g in timed:  # exactly `steps` GEMMs between the in-graph events
        g.replay()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier(dist)
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(dist, ms)
    code, where = pk.device_status()
    if code != 0:
        raise RuntimeError(f"device status {code} at site {where}")

    # sharded layers: every rank's assembled output against the unsharded GEMM
    # on its own GPU (outside the timed region), and the step's parts timed alone
    parity = breakdown = None
    gemm_ms_local = ms
    if sharded_run:
        rel = work.parity() if work.kind == "w4a16" else 0.0
        code_p, where_p = pk.device_status()
        parity = {"rel_frobenius_max_over_ranks": max_over_ranks(dist, rel),
                  "bar": 1e-5, "device_status": [code_p, where_p],
                  "against": "pk.int4_gemm of the whole layer (set 0) on each rank's GPU"}
        nb = min(args.steps, 1000 if work.hbm else 50)
        g_gemm = capture_runner(work.gemm_only, work.n_sets, nb, chunk)
        g_gath = capture_runner(work.gather_only, work.n_sets, nb, chunk)
        gemm_ms = _time_graphs(g_gemm, dist)
        gath_ms = _time_graphs(g_gath, dist)
        gemm_ms_local = gemm_ms * args.steps / nb
        step_us = ms_max / args.steps * 1e3
        breakdown = {"step_us": round(step_us, 3), "local_gemm_us": round(gemm_ms / nb * 1e3, 3),
                     "nccl_allgather_us": round(gath_ms / nb * 1e3, 3), "steps": nb}
        if work.exchange is not None:
            breakdown["exchange_us"] = round(step_us - gemm_ms / nb * 1e3, 3)
            breakdown["step"] = ("one kernel per rank: the local GEMM stores its columns into "
                                 "every rank's output over NVLink and ends with a flag barrier; "
                                 "exchange_us = step_us - local_gemm_us; nccl_allgather_us times "
                                 "an NCCL all-gather of the same output for comparison")
        else:
            breakdown["step"] = "the local GEMM, then an NCCL all-gather of its output"
        del g_gemm, g_gath

    phases = phase_leg(work, chunk) if args.phases and work.kind == "w4a16" and work.M <= 8 else None

    # end to end through the public API, host buffers in and out every step
    e2e_fn, h2d, d2h = work.e2e_step_fn()
    e2e_steps = args.e2e_steps if work.hbm else max(3, args.e2e_steps // 100)
    for i in range(20 if work.hbm else 3):
        e2e_fn(i)
    torch.cuda.synchronize()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.all_reduce(torch.zeros(1, device="cuda"))  # start the ranks together
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
    # of an ncu capture of this workload's kernel (single GPU only: a shard's
    # kernel reads a different slice)
    traffic, traffic_src = args.traffic, "--traffic" if args.traffic is not None else None
    if traffic is None and "ncu_traffic" in wl and (world == 1 or not work.sharded):
        traffic = wl["ncu_traffic"]
        traffic_src = "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this kernel"
    value = replicas * per * args.steps / sec / scale
    achieved = local_per / sec_per_launch / scale
    e2e_value = replicas * per * e2e_steps / (e2e_ms * 1e-3) / scale
    wl_cfg = workload_config(args.workload, wl, world)
    path = {"split_k": args.split_k if args.split_k > 0 else "auto",
            "weight_staging": args.weight_staging if args.weight_staging is not None else 0}
    if sharded_run:
        path["exchange"] = ("inside the local kernel (NVLink peer stores + flag barrier)"
                            if work.exchange is not None else "NCCL all_gather_into_tensor")
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
        "path": path,
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
                         if work.kind == "w4a16" and not sharded_run else
                         "pico_kernels_b200 public API (ctypes C ABI), pinned host buffers")},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(t0, t1),
    }
    if strong is not None:
        line["strong_scaling"] = strong
    if parity is not None:
        line["parity"] = parity
    if breakdown is not None:
        line["breakdown"] = breakdown
    if phases is not None:
        line["phases"] = phases
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl, budget_s=args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU reference path: the reference's torch computation (oracle/cpu_reference)
# ---------------------------------------------------------------------------
def cpu_baseline(wl: dict, budget_s: float = 10.0) -> dict:
    """Time the reference's CPU torch computation of one step of the workload
    on all host cores: the whole GEMM (weight dequantization + fp32 matmul),
    on a bounded column sample of large layers, scaled to all N columns."""
    from oracle import cpu_reference as ref
    cores = ref.use_all_cores()
    M, N, K = wl["M"], wl["N"], wl["K"]
    # columns whose step is ~1e10 flops / 6.4e7 weights at most (whole N when it fits)
    cap = min(int(1e10 // (2 * M * K)), int(64 * 2**20 // K))
    cols = N if N <= cap else max(128, cap // 128 * 128)
    kind = wl["kind"]
    if kind == "w4a16":
        step = ref.W4A16Step(M, K, cols)
        what = "q.float() * scales (group 128, repeat_interleave along K), then A.float() @ W"
    elif kind == "fp8":
        step = ref.Fp8Step(M, K, cols)
        what = "(a8.float() / sa) @ (b8.float() / sb)"
    else:
        step = ref.DenseStep(M, K, cols)
        what = "a.float() @ b.float()"
    sec, n = ref.time_steps(step, budget_s)
    sec_per_step = sec * N / cols
    if is_hbm_bound(wl):
        per = K * N // 2 + (K // 128) * N * 2 + M * K * 2 + M * N * 4
        value, unit = per / sec_per_step / 1e9, "GB/s"
    else:
        value, unit = 2 * M * N * K / sec_per_step / 1e12, "TFLOP/s"
    sample = (f"{n} calls of {what} on {cols} of {N} columns (M={M}, K={K}), "
              f"{n * sec:.1f} s, scaled to all N; torch {torch.__version__} on {cores} threads")
    return {"value": round(value, 6), "unit": unit, "cores": cores, "kind": "port",
            "sample": sample, "ms_per_step": round(sec_per_step * 1e3, 3)}


def run_reference(args, wl: dict, world: int, rank: int) -> None:
    if rank != 0:
        return
    base = cpu_baseline(wl, budget_s=args.cpu_seconds)
    line = {
        "metric": METRIC, "value": base["value"], "unit": base["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": base["ms_per_step"],
        "higher_is_better": True, "scaling": "strong" if wl.get("sharded") else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": workload_config(args.workload, wl, world),
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
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help=f"default: {DEFAULT_WORKLOAD} on one GPU, {DEFAULT_SHARDED_WORKLOAD} "
                         "sharded over the ranks under torchrun")
    ap.add_argument("--split-k", type=int, default=0)
    ap.add_argument("--exchange", choices=["fused", "nccl"], default="fused",
                    help="sharded W4A16 layers: output exchange inside the kernel where it "
                         "covers the shape, or always the NCCL all-gather")
    ap.add_argument("--weight-staging", type=int, choices=[0, 1], default=None,
                    help="pk_set_weight_staging mode for the M = 1 GEMVs (library default: 0)")
    ap.add_argument("--phases", action="store_true",
                    help="also report per-CTA phase times of the M = 1 GEMV (extra, untimed)")
    ap.add_argument("--e2e-steps", type=int, default=2000)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--traffic", type=float, default=None,
                    help="dram bytes per launch from an ncu capture, reported as-is")
    args = ap.parse_args()
    world, rank, local = dist_env()
    if args.workload is None:
        args.workload = DEFAULT_SHARDED_WORKLOAD if world > 1 else DEFAULT_WORKLOAD
    wl = WORKLOADS[args.workload]
    hbm = is_hbm_bound(wl)
    if args.steps is None:
        args.steps = 100000 if hbm else 200
    if args.warmup is None:
        args.warmup = 2000 if hbm else 20
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args, wl, world, rank)
    else:
        run_ours(args, wl, world, rank, local)


if __name__ == "__main__":
    main()
