"""Dense fp16/bf16 GEMM -- drop-in for pico-kernels' ``gemm`` module (gemm.py).

* ``triton_gemm(a, b) -> fp32``  gemm.py:103-131

The reference asserts M and N multiples of 256 and K a multiple of 64 (its
kernel is mask-free, gemm.py:114-116); this kernel accepts any M, and N and K
multiples of 8 (16-byte TMA rows), so every shape the reference accepts runs.
Products of more than one wave of 256 x 256 tiles run on CTA pairs
(cta_group::2), the rest on one-CTA 128 x 256 tiles; both accumulate in fp32
on the tensor cores and write fp32, as the reference does.
"""

from __future__ import annotations

from .gemm_splitk import triton_gemm

__all__ = ["triton_gemm"]
