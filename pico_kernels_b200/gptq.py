"""GPTQ producer of packed int4 weights on the GPU.

The reference's ``quantize.gptq_layer`` (quantize.py:71-115) returns
fake-quantized floats; ``gptq_quantize_int4`` runs the same walk over the
input features on the GPU (``pk_gptq_int4``) and returns what the W4A16 GEMM
consumes: ``(packed uint8[in, out // 2], scales[ceil(in / g), out])``, the
layout of ``gemm_int4.quantize_int4_grouped`` and ``int4_gemm``.

Same steps as the reference with ``act_order=False``: the damped Hessian
``H = X^T X / n + damp * mean(diag H) * I`` and its inverse (quantize.py:88-93,
torch on the device, or ``h_inv`` given), then per input feature j in order:
quantize, ``err = w - q``, and ``w[:, j+1:] -= outer(err, Hinv[j, j+1:] /
Hinv[j, j])`` (quantize.py:99-104). The scale is shared by ``group_size``
consecutive input features (the GEMM applies it after its K reduction),
taken when the walk reaches the group from the group's error-updated weights:
``max|w|.clamp_min(1e-12) / 7`` (quantize.py:58). The reference's own
``group_size`` groups output rows instead, which a GEMM cannot apply after the
reduction; its ``act_order`` permutes input features, which the packed layout's
contiguous groups cannot follow without a permutation index the kernels do not
take. Neither is offered here.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["gptq_inverse_hessian", "gptq_quantize_int4"]


def gptq_inverse_hessian(x: torch.Tensor, damp: float = 0.01) -> torch.Tensor:
    """``Hinv`` of quantize.py:88-93 from calibration inputs ``x[n, in]`` (fp32)."""
    xf = x.reshape(-1, x.shape[-1]).float()
    n, d = xf.shape
    h = (xf.t() @ xf) / n
    diag_mean = torch.diag(h).clone().mean()
    h = h + damp * diag_mean * torch.eye(d, device=h.device)
    return torch.linalg.inv(h)


def gptq_quantize_int4(w: torch.Tensor, x: torch.Tensor | None = None, *, group_size: int = 128,
                       damp: float = 0.01, h_inv: torch.Tensor | None = None,
                       scale_dtype: torch.dtype | None = None
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    """GPTQ-quantize ``w[out, in]`` (a linear layer's weight) to packed int4.

    Give calibration inputs ``x[..., in]`` or a precomputed ``h_inv[in, in]``.
    ``scale_dtype`` defaults to ``w.dtype`` for fp16/bf16 weights, else bf16.
    Returns ``(packed uint8[in, out // 2], scales[ceil(in / group_size), out])``.
    """
    _lib.require_cuda(w)
    if w.dim() != 2:
        raise _lib.ShapeError("w must be 2-D [out, in]")
    out_dim, in_dim = w.shape
    if out_dim % 2:
        raise _lib.ShapeError(f"out must be even to pack two codes per byte (got {out_dim})")
    if h_inv is None:
        if x is None:
            raise _lib.ShapeError("give calibration inputs x or h_inv")
        if x.shape[-1] != in_dim:
            raise _lib.ShapeError(f"x has {x.shape[-1]} features, w has {in_dim}")
        h_inv = gptq_inverse_hessian(x.to(w.device), damp)
    if tuple(h_inv.shape) != (in_dim, in_dim):
        raise _lib.ShapeError(f"h_inv must be [{in_dim}, {in_dim}]")
    if scale_dtype is None:
        scale_dtype = w.dtype if w.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
    h = h_inv.to(device=w.device, dtype=torch.float32).contiguous()
    wt = w.detach().float().t().contiguous()               # working copy [in, out]
    G = (in_dim + group_size - 1) // group_size
    packed = torch.empty((in_dim, out_dim // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((G, out_dim), dtype=scale_dtype, device=w.device)
    err = torch.empty((min(group_size, in_dim), out_dim), dtype=torch.float32, device=w.device)
    _lib.check(_lib.load().pk_gptq_int4(wt.data_ptr(), h.data_ptr(), in_dim, out_dim, group_size,
                                        packed.data_ptr(), scales.data_ptr(),
                                        _lib.dtype_code(scale_dtype), err.data_ptr(),
                                        _lib.stream_of(wt)), "gptq_quantize_int4")
    return packed, scales
