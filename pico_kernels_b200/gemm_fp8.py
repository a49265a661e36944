"""Scaled e4m3 GEMM -- drop-in for pico-kernels' ``gemm_fp8`` module
(gemm_fp8.py), running hand-written sm_100a kernels.

* ``quantize(x) -> (float8_e4m3fn tensor, float)``   gemm_fp8.py:89-95
* ``fp8_gemm_precast(a8, a_scale, b8, b_scale) -> fp32``  gemm_fp8.py:98-117
* ``fp8_gemm(a, b) -> fp32``                          gemm_fp8.py:120-124

Addition: keyword-only ``out_dtype`` (fp32 default, bf16 optional) on the
two GEMM entry points.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["E4M3_MAX", "quantize", "fp8_gemm_precast", "fp8_gemm"]

# gemm_fp8.py:24 takes the e4m3 maximum from torch.finfo rather than a literal
E4M3_MAX = float(torch.finfo(torch.float8_e4m3fn).max)


def quantize(x: torch.Tensor) -> tuple[torch.Tensor, float]:
    """Cast ``x`` to e4m3, scaled so ``max|x|`` maps to the e4m3 max.

    Returns ``(x_fp8, scale)`` with ``x ~= x_fp8 / scale``. The scale is a
    Python float (this synchronises, as the reference's ``.item()`` does).
    """
    _lib.require_cuda(x)
    lib = _lib.load()
    x = x.contiguous()
    dt = _lib.dtype_code(x.dtype)
    s = _lib.stream_of(x)
    amax = torch.empty((), dtype=torch.float32, device=x.device)
    _lib.check(lib.pk_absmax(x.data_ptr(), dt, x.numel(), amax.data_ptr(), s), "absmax")
    scale = E4M3_MAX / amax.item()
    x8 = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    _lib.check(lib.pk_fp8_quantize(x.data_ptr(), dt, x.numel(), scale, x8.data_ptr(), s),
               "fp8 quantize")
    return x8, scale


def fp8_gemm_precast(a8: torch.Tensor, a_scale: float, b8: torch.Tensor, b_scale: float, *,
                     out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Kernel-only fp8 matmul on already-cast ``a8, b8`` (fp32 output)."""
    _lib.require_cuda(a8, b8)
    if a8.dtype != torch.float8_e4m3fn or b8.dtype != torch.float8_e4m3fn:
        raise _lib.DtypeError("a8 and b8 must be float8_e4m3fn")
    M, K = a8.shape
    K2, N = b8.shape
    if K != K2:
        raise _lib.ShapeError(f"inner dimensions differ ({K} vs {K2})")
    a8 = a8.contiguous()
    b8 = b8.contiguous()
    out_scale = 1.0 / (a_scale * b_scale)
    c = torch.empty((M, N), dtype=out_dtype, device=a8.device)
    _lib.check(_lib.load().pk_fp8_gemm(a8.data_ptr(), b8.data_ptr(), M, N, K, out_scale,
                                       c.data_ptr(), _lib.dtype_code(out_dtype),
                                       _lib.stream_of(a8)), "fp8_gemm")
    return c


def fp8_gemm(a: torch.Tensor, b: torch.Tensor, *,
             out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Convenience: quantize then matmul (the full fp8 path)."""
    a8, a_scale = quantize(a)
    b8, b_scale = quantize(b)
    return fp8_gemm_precast(a8, a_scale, b8, b_scale, out_dtype=out_dtype)
