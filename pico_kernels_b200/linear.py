"""W4A16 ``nn.Linear`` drop-in over the packed-int4 GEMM.

The reference quantizes the transformer's ``nn.Linear`` layers in place
(quantize.py:124-129 selects them, quantize.py:160-184 swaps in fake-quant
weights) and then runs them as dense float layers. ``W4A16Linear`` instead
keeps each layer's weight as packed int4 codes plus group scales and runs
``int4_gemm`` on every call, so the weights stream from HBM at 4 bits:

* ``weight[out, in]`` is stored transposed, as the GEMM's ``B[K = in, N = out]``:
  ``w_packed`` uint8 ``[in, out // 2]`` (``pack_int4_n`` layout) and ``scales``
  ``[ceil(in / group_size), out]`` in the activation dtype; symmetric
  round-to-nearest per group of ``group_size`` input features
  (``quantize_int4_grouped``: ``scale = max|w| / 7``, codes in [-7, 7]).
* ``forward(x)`` flattens the leading dimensions of ``x[..., in]`` into M rows
  and computes ``x @ W^T + bias`` with fp32 accumulation; the result has
  ``x``'s dtype, like ``nn.Linear``. M = 1 runs the CUDA-core GEMV, small M the
  tensor-core decode, large M the tcgen05 prefill path.

``quantize_linear_layers(model)`` swaps every (or every selected) ``nn.Linear``
of a module tree for a ``W4A16Linear`` in place.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.nn as nn

from . import _lib
from .gemm_int4 import int4_gemm, quantize_int4_grouped

__all__ = ["W4A16Linear", "quantize_linear_layers"]


class W4A16Linear(nn.Module):
    """``y = x @ W^T + b`` with W held as packed int4 codes and group scales."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 group_size: int = 128, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | None = None) -> None:
        super().__init__()
        if out_features % 2:
            raise _lib.ShapeError(f"out_features must be even to pack two codes per byte "
                                  f"(got {out_features})")
        if dtype not in (torch.float16, torch.bfloat16):
            raise _lib.DtypeError(f"activation dtype must be fp16 or bf16 (got {dtype})")
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.dtype = dtype
        groups = (in_features + group_size - 1) // group_size
        self.register_buffer("w_packed", torch.zeros((in_features, out_features // 2),
                                                     dtype=torch.uint8, device=device))
        self.register_buffer("scales", torch.zeros((groups, out_features), dtype=dtype,
                                                   device=device))
        if bias:
            self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float32,
                                                     device=device))
        else:
            self.bias = None
        # act_order GPTQ: the packed rows follow this order of the input features
        self.register_buffer("perm", None)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group_size: int = 128,
                    dtype: torch.dtype | None = None, calib: torch.Tensor | None = None,
                    damp: float = 0.01, act_order: bool = False) -> "W4A16Linear":
        """Quantize ``linear.weight`` (on a CUDA device) into a new layer.

        Round-to-nearest per group by default; with calibration inputs
        ``calib[..., in]`` (this layer's inputs) the GPTQ producer
        (``gptq.gptq_quantize_int4``) chooses the codes. ``dtype``
        (activations and stored scales) defaults to the weight's dtype when
        that is fp16/bf16, else bf16. The bias is kept in fp32. With
        ``act_order`` (GPTQ only) the input features are quantized in order of
        decreasing activation energy (quantize.py:97-101) and stored in that
        order; ``forward`` gathers its inputs with the same permutation.
        """
        w = linear.weight.detach()
        _lib.require_cuda(w)
        if dtype is None:
            dtype = w.dtype if w.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
        layer = cls(linear.in_features, linear.out_features, linear.bias is not None,
                    group_size, dtype, w.device)
        # group absmax from the weights as stored (fp32 kept exact), scales rounded
        # to the activation dtype as the GEMM reads them
        if calib is not None:
            from .gptq import gptq_quantize_int4
            res = gptq_quantize_int4(w, calib, group_size=group_size, damp=damp,
                                     scale_dtype=dtype, act_order=act_order)
            packed, scales = res[0], res[1]
            if act_order:
                layer.perm = res[2]
        elif act_order:
            raise _lib.ShapeError("act_order needs calibration inputs (GPTQ)")
        else:
            packed, scales = quantize_int4_grouped(w.t(), group_size, scale_dtype=dtype)
        layer.w_packed.copy_(packed)
        layer.scales.copy_(scales)
        if linear.bias is not None:
            layer.bias.copy_(linear.bias.detach().float())
        return layer

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise _lib.ShapeError(f"expected {self.in_features} input features, got {x.shape[-1]}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        if x2.dtype != self.dtype:
            x2 = x2.to(self.dtype)
        if self.perm is not None:
            x2 = x2.index_select(1, self.perm)
        out_dtype = x.dtype if (self.bias is None and x.dtype == torch.bfloat16) else torch.float32
        y = int4_gemm(x2, self.w_packed, self.scales, group_size=self.group_size,
                      out_dtype=out_dtype)
        if self.bias is not None:
            y = y + self.bias
        return y.to(x.dtype).reshape(*lead, self.out_features)

    def dequantized_weight(self) -> torch.Tensor:
        """fp32 ``W[out, in]`` the layer computes with (codes x group scales)."""
        from .gemm_int4 import unpack_int4_n
        q = unpack_int4_n(self.w_packed).float()
        s = self.scales.float().repeat_interleave(self.group_size, dim=0)[: self.in_features]
        w = (q * s).t()
        if self.perm is not None:
            w = w[:, torch.argsort(self.perm)]
        return w.contiguous()

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, group_size={self.group_size}, int4")


def _capture_inputs(model: nn.Module, module: nn.Module, calib) -> torch.Tensor:
    """Inputs ``module`` sees when ``model`` runs on ``calib`` (a tensor or a
    tuple of positional arguments), flattened to ``[rows, in]``
    (quantize.py:132-157)."""
    seen: list[torch.Tensor] = []

    def hook(_m, args):
        seen.append(args[0].detach())

    handle = module.register_forward_pre_hook(hook)
    try:
        with torch.no_grad():
            model(*calib) if isinstance(calib, tuple) else model(calib)
    finally:
        handle.remove()
    return torch.cat([t.reshape(-1, t.shape[-1]) for t in seen], dim=0)


def quantize_linear_layers(model: nn.Module, group_size: int = 128,
                           select: Callable[[str, nn.Linear], bool] | None = None,
                           dtype: torch.dtype | None = None, calib=None,
                           damp: float = 0.01, act_order: bool = False) -> nn.Module:
    """Replace ``nn.Linear`` children in place with ``W4A16Linear``.

    ``select(name, module)`` picks the layers (default: every ``nn.Linear``
    with an even ``out_features``); quantize.py:124-129 picks those under
    ``transformer.h``, which ``select=lambda n, m: n.startswith("transformer.h")``
    reproduces. With ``calib`` (the model's input: a tensor or a tuple of
    arguments) each layer is GPTQ-quantized from the inputs it sees when the
    model, with the layers before it already quantized, runs on ``calib``
    (the sequential re-capture of quantize.py:160-184); without it, per-group
    round-to-nearest. Returns ``model``.
    """
    targets = [name for name, mod in model.named_modules()
               if isinstance(mod, nn.Linear) and mod.out_features % 2 == 0
               and (select is None or select(name, mod))]
    for name in targets:
        parent = model
        *path, leaf = name.split(".")
        for p in path:
            parent = getattr(parent, p)
        mod = getattr(parent, leaf)
        x = _capture_inputs(model, mod, calib) if calib is not None else None
        setattr(parent, leaf, W4A16Linear.from_linear(mod, group_size, dtype, calib=x, damp=damp,
                                                      act_order=act_order and x is not None))
    return model
