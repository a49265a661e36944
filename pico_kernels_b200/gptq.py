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
reduction. ``act_order=True`` (quantize.py:97-101) walks the input features in
order of decreasing activation energy; the packed weights are then stored in
that order and the permutation is returned with them: the layer computes
``x[:, perm] @ dequant(packed)`` (``W4A16Linear`` gathers its inputs).

``gptq_layer`` is the reference's function itself on the GPU
(``pk_gptq_ref``): same signature, same defaults (``act_order=True``), the
same ``quantize_col`` rule per input feature (any width 2-8 bits, groups of
``group_size`` outputs or one scale per feature) and the same fake-quantized
result ``[out, in]`` in ``w.dtype``. Given the reference's inverse Hessian
(and, for ``act_order``, its activation energies) it reproduces the
reference's output bit for bit.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["gptq_inverse_hessian", "gptq_quantize_int4", "gptq_layer"]


def _hessian(x: torch.Tensor, damp: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(``Hinv``, activation energy ``diag(H)`` before damping) of
    quantize.py:86-93 from calibration inputs ``x[..., in]`` (fp32)."""
    xf = x.reshape(-1, x.shape[-1]).float()
    n, d = xf.shape
    h = (xf.t() @ xf) / n
    act_mag = torch.diag(h).clone()
    h = h + damp * act_mag.mean() * torch.eye(d, device=h.device)
    return torch.linalg.inv(h), act_mag


def gptq_inverse_hessian(x: torch.Tensor, damp: float = 0.01) -> torch.Tensor:
    """``Hinv`` of quantize.py:88-93 from calibration inputs ``x[n, in]`` (fp32)."""
    return _hessian(x, damp)[0]


def gptq_layer(w: torch.Tensor, x: torch.Tensor | None, bits: int, damp: float = 0.01,
               act_order: bool = True, group_size: int | None = None, *,
               h_inv: torch.Tensor | None = None, act_mag: torch.Tensor | None = None
               ) -> torch.Tensor:
    """GPTQ-quantize one linear layer ``w[out, in]`` given activations
    ``x[n, in]``: quantize.gptq_layer (quantize.py:71-115) on the GPU.

    Returns the fake-quantized weights ``[out, in]`` in ``w.dtype``. ``h_inv``
    (the inverse damped Hessian) and ``act_mag`` (``diag(X^T X / n)``, the
    order key of ``act_order``) may be given instead of being computed from
    ``x`` on the device."""
    if bits >= 16:
        return w.clone()
    _lib.require_cuda(w)
    if w.dim() != 2:
        raise _lib.ShapeError("w must be 2-D [out, in]")
    if not 2 <= bits <= 8:
        raise _lib.ShapeError(f"bits must be in [2, 8] or >= 16 (got {bits})")
    if group_size is not None and group_size <= 0:
        raise _lib.ShapeError(f"group_size must be positive (got {group_size})")
    out_dim, in_dim = w.shape
    dev = w.device
    if h_inv is None or (act_order and act_mag is None):
        if x is None:
            raise _lib.ShapeError("give calibration inputs x (or h_inv and act_mag)")
        if x.shape[-1] != in_dim:
            raise _lib.ShapeError(f"x has {x.shape[-1]} features, w has {in_dim}")
        hi, mag = _hessian(x.to(dev), damp)
        h_inv = hi if h_inv is None else h_inv
        act_mag = mag if act_mag is None else act_mag
    h = h_inv.to(device=dev, dtype=torch.float32)
    if tuple(h.shape) != (in_dim, in_dim):
        raise _lib.ShapeError(f"h_inv must be [{in_dim}, {in_dim}]")
    wq = w.detach().float()
    order = None
    if act_order:  # quantize.py:97-101
        order = torch.argsort(act_mag.to(dev), descending=True)
        wq = wq[:, order]
        h = h[order][:, order]
    wt = wq.t().contiguous()                     # [in, out]: one row per input feature
    h = h.contiguous()
    err = torch.empty((min(32, in_dim), out_dim), dtype=torch.float32, device=dev)
    _lib.check(_lib.load().pk_gptq_ref(wt.data_ptr(), h.data_ptr(), in_dim, out_dim,
                                       0 if group_size is None else group_size, bits,
                                       err.data_ptr(), _lib.stream_of(wt)), "gptq_layer")
    wq = wt.t()
    if order is not None:
        wq = wq[:, torch.argsort(order)]          # quantize.py:106-107
    return wq.contiguous().to(w.dtype)


def gptq_quantize_int4(w: torch.Tensor, x: torch.Tensor | None = None, *, group_size: int = 128,
                       damp: float = 0.01, h_inv: torch.Tensor | None = None,
                       scale_dtype: torch.dtype | None = None, act_order: bool = False,
                       act_mag: torch.Tensor | None = None):
    """GPTQ-quantize ``w[out, in]`` (a linear layer's weight) to packed int4.

    Give calibration inputs ``x[..., in]`` or a precomputed ``h_inv[in, in]``.
    ``scale_dtype`` defaults to ``w.dtype`` for fp16/bf16 weights, else bf16.
    Returns ``(packed uint8[in, out // 2], scales[ceil(in / group_size), out])``.
    With ``act_order`` the input features are walked (and stored) in order of
    decreasing ``act_mag`` (``diag(X^T X / n)``, from ``x`` unless given) and
    the permutation comes third: ``(packed, scales, perm)``, the layer being
    ``x[:, perm] @ dequant(packed)``.
    """
    _lib.require_cuda(w)
    if w.dim() != 2:
        raise _lib.ShapeError("w must be 2-D [out, in]")
    out_dim, in_dim = w.shape
    if out_dim % 2:
        raise _lib.ShapeError(f"out must be even to pack two codes per byte (got {out_dim})")
    if h_inv is None or (act_order and act_mag is None):
        if x is None:
            raise _lib.ShapeError("give calibration inputs x or h_inv")
        if x.shape[-1] != in_dim:
            raise _lib.ShapeError(f"x has {x.shape[-1]} features, w has {in_dim}")
        hi, mag = _hessian(x.to(w.device), damp)
        h_inv = hi if h_inv is None else h_inv
        act_mag = mag if act_mag is None else act_mag
    if tuple(h_inv.shape) != (in_dim, in_dim):
        raise _lib.ShapeError(f"h_inv must be [{in_dim}, {in_dim}]")
    if scale_dtype is None:
        scale_dtype = w.dtype if w.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
    h = h_inv.to(device=w.device, dtype=torch.float32)
    wf = w.detach().float()
    perm = None
    if act_order:
        perm = torch.argsort(act_mag.to(w.device), descending=True)
        wf = wf[:, perm]
        h = h[perm][:, perm]
    h = h.contiguous()
    wt = wf.t().contiguous()                                # working copy [in, out]
    G = (in_dim + group_size - 1) // group_size
    packed = torch.empty((in_dim, out_dim // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((G, out_dim), dtype=scale_dtype, device=w.device)
    err = torch.empty((min(group_size, in_dim), out_dim), dtype=torch.float32, device=w.device)
    _lib.check(_lib.load().pk_gptq_int4(wt.data_ptr(), h.data_ptr(), in_dim, out_dim, group_size,
                                        packed.data_ptr(), scales.data_ptr(),
                                        _lib.dtype_code(scale_dtype), err.data_ptr(),
                                        _lib.stream_of(wt)), "gptq_quantize_int4")
    if act_order:
        return packed, scales, perm
    return packed, scales
