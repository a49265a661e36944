"""Scaled e4m3 GEMM -- drop-in for pico-kernels' ``gemm_fp8`` module
(gemm_fp8.py), running hand-written sm_100a kernels.

* ``quantize(x) -> (float8_e4m3fn tensor, float)``   gemm_fp8.py:89-95
* ``fp8_gemm_precast(a8, a_scale, b8, b_scale) -> fp32``  gemm_fp8.py:98-117
* ``fp8_gemm(a, b) -> fp32``                          gemm_fp8.py:120-124

Additions: keyword-only ``out_dtype`` (fp32 default, bf16 optional) on the
two GEMM entry points; ``quantize_device(x) -> (x8, scale)``, the same cast
with the scale left on the device as a 0-d fp32 tensor (no host sync);
``fp8_gemm_precast`` accepts such tensors as scales, and ``fp8_gemm`` runs
cast -> cast -> GEMM entirely stream-ordered (graph-capturable), where the
reference synchronises twice on ``.item()`` (gemm_fp8.py:94).
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["E4M3_MAX", "quantize", "quantize_device", "fp8_gemm_precast", "fp8_gemm"]

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


def quantize_device(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``quantize`` with the scale kept on the device: returns ``(x_fp8,
    scale)`` where ``scale`` is a 0-d fp32 CUDA tensor equal to
    ``float32(quantize(x)[1])`` and ``x_fp8`` equals ``quantize(x)[0]``
    bit for bit. An all-zero ``x`` gets scale 1 (``quantize`` raises there,
    as the reference does)."""
    _lib.require_cuda(x)
    lib = _lib.load()
    x = x.contiguous()
    buf = torch.empty(2, dtype=torch.float32, device=x.device)  # [amax, scale]
    x8 = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    _lib.check(lib.pk_fp8_quantize_device(x.data_ptr(), _lib.dtype_code(x.dtype), x.numel(),
                                          x8.data_ptr(), buf.data_ptr(), buf.data_ptr() + 4,
                                          _lib.stream_of(x)), "fp8 quantize (device scale)")
    return x8, buf[1]


def _scale_tensor(s, device: torch.device) -> torch.Tensor:
    if isinstance(s, torch.Tensor):
        _lib.require_cuda(s)
        if s.numel() != 1 or s.dtype != torch.float32:
            raise _lib.DtypeError("a device scale must be a one-element fp32 tensor")
        return s
    return torch.tensor(float(s), dtype=torch.float32, device=device)


def fp8_gemm_precast(a8: torch.Tensor, a_scale, b8: torch.Tensor, b_scale, *,
                     out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Kernel-only fp8 matmul on already-cast ``a8, b8`` (fp32 output).

    ``a_scale`` / ``b_scale``: Python floats (the reference's form), or
    one-element fp32 CUDA tensors from ``quantize_device`` (read on the
    device; no sync)."""
    _lib.require_cuda(a8, b8)
    if a8.dtype != torch.float8_e4m3fn or b8.dtype != torch.float8_e4m3fn:
        raise _lib.DtypeError("a8 and b8 must be float8_e4m3fn")
    M, K = a8.shape
    K2, N = b8.shape
    if K != K2:
        raise _lib.ShapeError(f"inner dimensions differ ({K} vs {K2})")
    a8 = a8.contiguous()
    b8 = b8.contiguous()
    c = torch.empty((M, N), dtype=out_dtype, device=a8.device)
    lib = _lib.load()
    if isinstance(a_scale, torch.Tensor) or isinstance(b_scale, torch.Tensor):
        sa = _scale_tensor(a_scale, a8.device)
        sb = _scale_tensor(b_scale, a8.device)
        _lib.check(lib.pk_fp8_gemm_scaled(a8.data_ptr(), b8.data_ptr(), M, N, K, sa.data_ptr(),
                                          sb.data_ptr(), c.data_ptr(), _lib.dtype_code(out_dtype),
                                          _lib.stream_of(a8)), "fp8_gemm")
        return c
    out_scale = 1.0 / (a_scale * b_scale)
    _lib.check(lib.pk_fp8_gemm(a8.data_ptr(), b8.data_ptr(), M, N, K, out_scale,
                               c.data_ptr(), _lib.dtype_code(out_dtype),
                               _lib.stream_of(a8)), "fp8_gemm")
    return c


def fp8_gemm(a: torch.Tensor, b: torch.Tensor, *,
             out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Convenience: quantize then matmul (the full fp8 path), with the
    scales kept on the device: no host synchronisation."""
    a8, a_scale = quantize_device(a)
    b8, b_scale = quantize_device(b)
    return fp8_gemm_precast(a8, a_scale, b8, b_scale, out_dtype=out_dtype)
