"""The reference's CPU torch computation of each bench workload, restated.

TEST AND BENCH INFRASTRUCTURE ONLY: ``bench.py`` times these on the host
cores as the CPU baseline (its ``cpu_baseline`` leg and ``--impl
reference`` arm); nothing in ``pico_kernels_b200`` imports them.

The reference has no CPU implementation of its kernels; its own correctness
checks compute the result with torch, and that expression is what is timed:

* W4A16: ``a.float() @ (w_q.float() * scale)`` (gemm_int4.py:102,
  tests/test_gemm_int4.py:26), with the group scales repeated along K
  (``repeat_interleave(group, 0)``, the per-group form of the same
  dequantize-then-matmul);
* fp8: ``(a8.float() / sa) @ (b8.float() / sb)`` (gemm_fp8.py:132 compares
  the GEMM with the fp32 product; gemm_fp8.py:106 folds 1/(sa*sb) into it);
* dense: ``a.float() @ b.float()`` (gemm.py:134-142).

A step is one whole GEMM: the weight dequantization and the matmul. Large
layers are sampled by output columns (the work per column is the same) and
the time scaled to all N columns.
"""

from __future__ import annotations

import os
import time

import torch

__all__ = ["use_all_cores", "W4A16Step", "Fp8Step", "DenseStep", "time_steps"]


def use_all_cores() -> int:
    """Let torch use every host core (torchrun sets OMP_NUM_THREADS=1)."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


class W4A16Step:
    """``Y = A.float() @ (q.float() * scales.float().repeat_interleave(g, 0))``
    on ``cols`` of the layer's N columns (int8 codes, as the reference's test
    holds them; bf16 group scales)."""

    def __init__(self, M: int, K: int, cols: int, group: int = 128, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(K, cols, generator=g) * 0.02).to(torch.bfloat16).float()
        G = (K + group - 1) // group
        wg = torch.nn.functional.pad(w, (0, 0, 0, G * group - K)).view(G, group, cols)
        s32 = wg.abs().amax(dim=1).clamp_min(1e-12) / 7  # quantize.py:58
        self.q = torch.clamp(torch.round(wg / s32[:, None, :]), -7, 7).view(G * group, cols)[:K]
        self.q = self.q.to(torch.int8)
        self.scales = s32.to(torch.bfloat16)
        self.a = torch.randn(M, K, generator=g).to(torch.bfloat16)
        self.group = group

    def __call__(self) -> torch.Tensor:
        s = self.scales.float().repeat_interleave(self.group, 0)[: self.q.shape[0]]
        return self.a.float() @ (self.q.float() * s)


class Fp8Step:
    """``(a8.float() / sa) @ (b8.float() / sb)`` on ``cols`` columns of B."""

    def __init__(self, M: int, K: int, cols: int, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        a = torch.randn(M, K, generator=g).to(torch.bfloat16)
        b = torch.randn(K, cols, generator=g).to(torch.bfloat16)
        self.sa = 448.0 / a.abs().max().item()  # gemm_fp8.py:94
        self.sb = 448.0 / b.abs().max().item()
        self.a8 = (a * self.sa).to(torch.float8_e4m3fn)
        self.b8 = (b * self.sb).to(torch.float8_e4m3fn)

    def __call__(self) -> torch.Tensor:
        return (self.a8.float() / self.sa) @ (self.b8.float() / self.sb)


class DenseStep:
    """``a.float() @ b.float()`` on ``cols`` columns of B."""

    def __init__(self, M: int, K: int, cols: int, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        self.a = torch.randn(M, K, generator=g).to(torch.bfloat16)
        self.b = torch.randn(K, cols, generator=g).to(torch.bfloat16)

    def __call__(self) -> torch.Tensor:
        return self.a.float() @ self.b.float()


def time_steps(step, budget_s: float, min_steps: int = 2) -> tuple[float, int]:
    """Run ``step`` until ``budget_s`` seconds have passed (at least
    ``min_steps`` times, after one untimed call); return (seconds per call,
    calls)."""
    step()
    n = 0
    t0 = time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s and n >= min_steps:
            return el / n, n
