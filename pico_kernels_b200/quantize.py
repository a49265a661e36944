"""Round-to-nearest group quantization -- the hot-path half of pico-kernels'
``quantize`` module (quantize.py:42-68) on CUDA tensors.

``quantize_col`` and ``rtn_layer`` keep the reference's signatures and return
the same fake-quantized values, computed by the sm_100a kernel behind
``pk_fake_quant_groups``:

* ``quantize_col(w, bits, group_size=None)`` (quantize.py:42-60): any width
  from 2 to 8 bits (``qmax = 2**(bits-1) - 1``), groups of ``group_size``
  consecutive elements of the column or one scale for all of it, and the
  arithmetic in ``w``'s own dtype: for fp16/bf16 each step (the clamp at
  1e-12, the division by qmax, ``w / scale``, ``q * scale``) is computed in
  fp32 and rounded to the dtype, as torch evaluates the reference's
  expressions. So an fp16 column keeps the reference's behaviour where 1e-12
  underflows: a group of zeros gets scale 0 and NaN outputs.
* ``rtn_layer(w, bits, group_size=None)`` (quantize.py:63-68): the same rule
  on every input column of ``w[out, in]``, groups along the output rows,
  computed on ``w.float()`` and returned in ``w.dtype``.

``bits >= 16`` returns the input (``quantize_col``) or a copy
(``rtn_layer``), as the reference does. Widths between 9 and 15 bits are not
served (``ValueError``): their ``qmax`` is not exact in fp16/bf16, and no
caller of the reference uses them. GPTQ (quantize.py:71-115) is in
``pico_kernels_b200.gptq``.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["quantize_col", "rtn_layer"]

_FLOATS = (torch.float16, torch.bfloat16, torch.float32)


def _check(w: torch.Tensor, bits: int) -> None:
    _lib.require_cuda(w)
    if w.dtype not in _FLOATS:
        raise _lib.DtypeError(f"quantize runs on fp16, bf16 or fp32 tensors (got {w.dtype})")
    if not 2 <= bits <= 8:
        raise _lib.ShapeError(f"bits must be in [2, 8] or >= 16 (got {bits})")


def _fake_quant(w: torch.Tensor, rows: int, cols: int, group: int, bits: int) -> torch.Tensor:
    """pk_fake_quant_groups on a contiguous ``w`` viewed as ``[rows, cols]``."""
    out = torch.empty_like(w)
    _lib.check(_lib.load().pk_fake_quant_groups(
        w.data_ptr(), _lib.dtype_code(w.dtype), rows, cols, cols, group, bits, out.data_ptr(), cols,
        _lib.stream_of(w)), "quantize")
    return out


def quantize_col(w: torch.Tensor, bits: int, group_size: int | None = None) -> torch.Tensor:
    """Symmetric round-to-nearest quantization of a column ``[out]``.

    ``group_size=None`` uses a single scale for the whole column; otherwise
    consecutive groups of ``group_size`` elements share a scale."""
    if bits >= 16:
        return w
    _check(w, bits)
    if group_size is not None and w.dim() != 1:
        raise _lib.ShapeError("quantize_col with groups takes a 1-D column")
    if group_size is not None and group_size <= 0:
        raise _lib.ShapeError(f"group_size must be positive (got {group_size})")
    if w.numel() == 0:
        return w.clone()
    wc = w.contiguous()
    out = _fake_quant(wc, wc.numel(), 1, 0 if group_size is None else group_size, bits)
    return out.view(w.shape)


def rtn_layer(w: torch.Tensor, bits: int, group_size: int | None = None) -> torch.Tensor:
    """Naive round-to-nearest over every column of ``w[out, in]`` -- the GPTQ
    baseline; groups of ``group_size`` output rows share a scale."""
    if bits >= 16:
        return w.clone()
    _check(w, bits)
    if w.dim() != 2:
        raise _lib.ShapeError("rtn_layer takes a 2-D weight [out, in]")
    if group_size is not None and group_size <= 0:
        raise _lib.ShapeError(f"group_size must be positive (got {group_size})")
    out_dim, in_dim = w.shape
    if w.numel() == 0:
        return w.clone()
    wf = w.float().contiguous()
    out = _fake_quant(wf, out_dim, in_dim, 0 if group_size is None else group_size, bits)
    return out.to(w.dtype)
