"""Round-to-nearest group quantization -- the hot-path half of pico-kernels'
``quantize`` module (quantize.py:42-68) on CUDA tensors.

``quantize_col`` and ``rtn_layer`` keep the reference's signatures and return
the same fake-quantized values (``clamp(round(w/scale), -qmax, qmax) * scale``
in fp32), computed by the int4 group-quantize kernel. Only ``bits == 4`` runs
here (the width the packed-int4 GEMM consumes); other widths and GPTQ
(quantize.py:71-265) are outside this package.
"""

from __future__ import annotations

import torch

from . import _lib
from .gemm_int4 import quantize_int4_grouped, unpack_int4_n

__all__ = ["quantize_col", "rtn_layer", "fake_quant_grouped"]


def _check_bits(bits: int) -> None:
    if bits != 4:
        raise NotImplementedError("only 4-bit quantization runs on the sm_100a kernels")


def fake_quant_grouped(w: torch.Tensor, group_size: int) -> torch.Tensor:
    """Fake-quant of ``w[K, N]`` with int4 groups along K, in fp32."""
    K, N = w.shape
    pad = N % 2
    if pad:
        w = torch.nn.functional.pad(w, (0, 1))
    packed, scales = quantize_int4_grouped(w, group_size, scale_dtype=torch.float32)
    codes = unpack_int4_n(packed).to(torch.float32)
    rep = scales.repeat_interleave(group_size, dim=0)[:K]
    out = codes * rep
    return out[:, :N] if pad else out


def quantize_col(w: torch.Tensor, bits: int, group_size: int | None = None) -> torch.Tensor:
    """Symmetric round-to-nearest quantization of a column ``[out]``."""
    if bits >= 16:
        return w
    _check_bits(bits)
    _lib.require_cuda(w)
    gs = w.numel() if group_size is None else group_size
    return fake_quant_grouped(w.reshape(-1, 1), gs).reshape(w.shape).to(w.dtype)


def rtn_layer(w: torch.Tensor, bits: int, group_size: int | None = None) -> torch.Tensor:
    """Round-to-nearest over every column of ``w[out, in]`` (groups along out)."""
    if bits >= 16:
        return w.clone()
    _check_bits(bits)
    _lib.require_cuda(w)
    gs = w.shape[0] if group_size is None else group_size
    return fake_quant_grouped(w.float(), gs).to(w.dtype)
