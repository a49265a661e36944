"""Packed int4 quantization and the W4A16 GEMM -- drop-in for pico-kernels'
``gemm_int4`` module (gemm_int4.py), running hand-written sm_100a kernels.

Same names, arguments, layouts and return types as the reference:

* ``quantize_int4(w) -> (int8[K, N], float)``           gemm_int4.py:58-62
* ``pack_int4_n(w_q) -> uint8[K, N//2]``                gemm_int4.py:65-72
* ``int4_gemm(a, w_packed, scale, BLOCK_M, BLOCK_N, BLOCK_K) -> fp32[M, N]``
                                                        gemm_int4.py:75-92

Additions: ``quantize_int4_grouped`` (per-group int4 along K, the
``quantize.quantize_col`` arithmetic emitted as packed codes + scales),
``unpack_int4_n``, and keyword-only ``group_size``, ``out_dtype`` and
``split_k`` on ``int4_gemm``. ``scale`` may be the reference's per-tensor
float or a ``[ceil(K/group), N]`` tensor of group scales.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["quantize_int4", "pack_int4_n", "unpack_int4_n", "quantize_int4_grouped",
           "int4_gemm", "int4_gemm_host"]


def quantize_int4(w: torch.Tensor) -> tuple[torch.Tensor, float]:
    """Per-tensor symmetric int4 quantization of ``w`` (fp16/bf16/fp32).

    ``scale = max|w| / 7`` (a Python float; this synchronises, like the
    reference's ``.item()``), codes ``round(w / scale).clamp(-8, 7)`` as int8.
    """
    _lib.require_cuda(w)
    lib = _lib.load()
    w = w.contiguous()
    dt = _lib.dtype_code(w.dtype)
    amax = torch.empty((), dtype=torch.float32, device=w.device)
    s = _lib.stream_of(w)
    _lib.check(lib.pk_absmax(w.data_ptr(), dt, w.numel(), amax.data_ptr(), s), "absmax")
    scale = amax.item() / 7.0
    codes = torch.empty(w.shape, dtype=torch.int8, device=w.device)
    _lib.check(lib.pk_quant_int4_tensor(w.data_ptr(), dt, w.numel(), scale, codes.data_ptr(), s),
               "quantize_int4")
    return codes, scale


def pack_int4_n(w_q: torch.Tensor) -> torch.Tensor:
    """Pack signed int4 codes 2-per-byte along N -> ``(K, N//2)`` uint8.

    Low nibble = even column, high nibble = odd column.
    """
    _lib.require_cuda(w_q)
    K, N = w_q.shape
    if N % 2:
        raise _lib.ShapeError(f"N must be even (got {N})")
    q = w_q if w_q.dtype == torch.int8 else w_q.to(torch.int8)
    q = q.contiguous()
    out = torch.empty((K, N // 2), dtype=torch.uint8, device=q.device)
    _lib.check(_lib.load().pk_pack_int4_n(q.data_ptr(), K, N, out.data_ptr(), _lib.stream_of(q)),
               "pack_int4_n")
    return out


def unpack_int4_n(w_packed: torch.Tensor) -> torch.Tensor:
    """Inverse of ``pack_int4_n``: sign-extended int8 codes ``(K, N)``."""
    _lib.require_cuda(w_packed)
    K, Nh = w_packed.shape
    p = w_packed.contiguous()
    out = torch.empty((K, 2 * Nh), dtype=torch.int8, device=p.device)
    _lib.check(_lib.load().pk_unpack_int4_n(p.data_ptr(), K, 2 * Nh, out.data_ptr(),
                                            _lib.stream_of(p)), "unpack_int4_n")
    return out


def quantize_int4_grouped(w: torch.Tensor, group_size: int = 128,
                          scale_dtype: torch.dtype | None = None
                          ) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-group symmetric int4 quantize + pack of ``w[K, N]``, groups along K.

    Per column ``n`` and group ``g`` this is ``quantize.quantize_col``'s
    arithmetic (quantize.py:42-60): ``scale = max|w|.clamp_min(1e-12) / 7``
    in fp32 and ``q = clamp(round(w / scale), -7, 7)``; the codes are packed
    with ``pack_int4_n``'s byte layout and the scale is stored rounded to
    ``scale_dtype`` (default: ``w.dtype`` for fp16/bf16, fp32 otherwise).
    Returns ``(packed uint8[K, N//2], scales[ceil(K/group_size), N])``.
    """
    _lib.require_cuda(w)
    if w.dim() != 2:
        raise _lib.ShapeError("w must be 2-D [K, N]")
    K, N = w.shape
    if N % 2:
        raise _lib.ShapeError(f"N must be even (got {N})")
    if scale_dtype is None:
        scale_dtype = w.dtype if w.dtype in (torch.float16, torch.bfloat16) else torch.float32
    if w.stride(1) != 1:
        w = w.contiguous()
    G = (K + group_size - 1) // group_size
    packed = torch.empty((K, N // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((G, N), dtype=scale_dtype, device=w.device)
    _lib.check(_lib.load().pk_quant_int4_group(
        w.data_ptr(), _lib.dtype_code(w.dtype), K, N, w.stride(0), group_size, packed.data_ptr(),
        scales.data_ptr(), _lib.dtype_code(scale_dtype), _lib.stream_of(w)), "quantize_int4_grouped")
    return packed, scales


def int4_gemm(a: torch.Tensor, w_packed: torch.Tensor, scale,
              BLOCK_M: int = 64, BLOCK_N: int = 64, BLOCK_K: int = 64, *,
              group_size: int | None = None, out_dtype: torch.dtype = torch.float32,
              split_k: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """``a @ (W_int4 * scale)`` where ``w_packed`` is ``(K, N//2)`` uint8.

    ``scale``: the reference's per-tensor float, or a ``[G, N]`` tensor of
    group scales (``group_size`` defaults to ``K // G``). ``BLOCK_*`` are
    accepted for signature compatibility; the tile shape is fixed by the
    sm_100a kernels. Output fp32 (or ``out_dtype=torch.bfloat16``), written to
    ``out`` when given (a contiguous ``[M, N]`` tensor of ``out_dtype`` on
    ``a``'s device; a decode loop reuses it instead of allocating per call).
    """
    del BLOCK_M, BLOCK_N, BLOCK_K
    tf = _lib.torch_fast()  # the same checks and call in C++, when it serves them
    if tf is not None:
        res = tf.int4_gemm(a, w_packed, scale, group_size, out, out_dtype, split_k)
        if type(res) is not int:
            return res
        if res > 0:
            _lib.check(res, "int4_gemm")
    _lib.require_cuda(a, w_packed)
    if a.dtype not in (torch.float16, torch.bfloat16):
        raise _lib.DtypeError(f"a must be fp16 or bf16 (got {a.dtype})")
    if a.dim() != 2 or w_packed.dim() != 2:
        raise _lib.ShapeError("a and w_packed must be 2-D")
    M, K = a.shape
    K2, N_half = w_packed.shape
    if K2 != K:
        raise _lib.ShapeError(f"inner dimensions differ: a has K={K}, w_packed has K={K2}")
    if w_packed.dtype != torch.uint8:
        raise _lib.DtypeError("w_packed must be uint8")
    N = 2 * N_half
    if a.stride(1) != 1 or a.stride(0) < K:
        a = a.contiguous()
    if not w_packed.is_contiguous():
        w_packed = w_packed.contiguous()

    scales, scalar, group = _scale_args(scale, K, N, a.dtype, group_size)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    elif (out.shape != (M, N) or out.dtype != out_dtype or out.device != a.device
          or not out.is_contiguous()):
        raise _lib.ShapeError(f"out must be a contiguous [{M}, {N}] {out_dtype} tensor on "
                              f"{a.device}")
    lib = _lib.load()
    key = (M, N, K, split_k)
    ws_bytes = _ws_bytes.get(key)
    if ws_bytes is None:
        ws_bytes = _ws_bytes[key] = lib.pk_w4a16_workspace_size(M, N, K, split_k)
    stream = _lib.stream_of(a)
    ws = _lib.workspace(a.device, ws_bytes, stream=stream) if ws_bytes else None
    st = _lib.fast().w4a16_gemm(
        a.data_ptr(), _lib.dtype_code(a.dtype), a.stride(0), w_packed.data_ptr(),
        _lib.ptr(scales), scalar, group, M, N, K, out.data_ptr(), _lib.dtype_code(out_dtype), N,
        split_k, _lib.ptr(ws), ws_bytes, stream)
    if st:
        _lib.check(st, "int4_gemm")
    return out


# pk_w4a16_workspace_size per (M, N, K, split_k): a pure function of the shape
_ws_bytes: dict[tuple[int, int, int, int], int] = {}


def _scale_args(scale, K: int, N: int, dtype: torch.dtype, group_size: int | None):
    """(group scales tensor or None, scalar scale, group size) for the C ABI."""
    if isinstance(scale, torch.Tensor) and scale.numel() > 1:
        _lib.require_cuda(scale)
        if scale.dim() != 2 or scale.shape[1] != N:
            raise _lib.ShapeError(f"group scales must be [G, N={N}] (got {tuple(scale.shape)})")
        G = scale.shape[0]
        if group_size is not None:
            group = group_size
        else:  # several sizes can give G groups when the last one is ragged: prefer 128
            group = next((g for g in (128, K // G) if g > 0 and (K + g - 1) // g == G), K // G)
        if group <= 0 or (K + group - 1) // group != G:
            raise _lib.ShapeError(f"{G} scale rows do not tile K={K} with group_size={group}")
        scales = scale if scale.dtype == dtype else scale.to(dtype)
        if not scales.is_contiguous():
            scales = scales.contiguous()
        return scales, 1.0, group
    return None, float(scale), 0


def int4_gemm_host(a: torch.Tensor, w_packed: torch.Tensor, scale, *,
                   group_size: int | None = None, out_dtype: torch.dtype = torch.float32,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """``int4_gemm`` for a caller whose activations and outputs live in host
    memory: ``a`` is a CPU ``[M, K]`` fp16/bf16 tensor, ``w_packed`` and
    ``scale`` are resident on the GPU. One C-ABI call (``pk_w4a16_gemm_host``)
    copies A into a device staging buffer, runs the same kernels as
    ``int4_gemm`` and copies the output into ``out`` (a CPU ``[M, N]`` tensor
    of ``out_dtype``; allocated page-locked when None). Enqueued on the
    current stream of the weights' device: synchronise it before reading
    ``out``. Page-locked ``a`` and ``out`` make the copies asynchronous.
    """
    if out is not None:  # the same checks and call in C++, when it serves them
        tf = _lib.torch_fast()
        if tf is not None:
            res = tf.int4_gemm_host(a, w_packed, scale, group_size, out, out_dtype)
            if type(res) is not int:
                return res
            if res > 0:
                _lib.check(res, "int4_gemm_host")
    if a.is_cuda or (out is not None and out.is_cuda):
        raise _lib.DtypeError("int4_gemm_host takes host tensors for a and out")
    _lib.require_cuda(w_packed)
    if a.dtype not in (torch.float16, torch.bfloat16):
        raise _lib.DtypeError(f"a must be fp16 or bf16 (got {a.dtype})")
    if a.dim() != 2 or w_packed.dim() != 2:
        raise _lib.ShapeError("a and w_packed must be 2-D")
    if w_packed.dtype != torch.uint8:
        raise _lib.DtypeError("w_packed must be uint8")
    M, K = a.shape
    K2, N_half = w_packed.shape
    if K2 != K:
        raise _lib.ShapeError(f"inner dimensions differ: a has K={K}, w_packed has K={K2}")
    N = 2 * N_half
    if a.stride(1) != 1 or a.stride(0) < K:
        a = a.contiguous()
    if not w_packed.is_contiguous():
        w_packed = w_packed.contiguous()
    scales, scalar, group = _scale_args(scale, K, N, a.dtype, group_size)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, pin_memory=True)
    elif out.shape != (M, N) or out.dtype != out_dtype or not out.is_contiguous():
        raise _lib.ShapeError(f"out must be a contiguous [{M}, {N}] {out_dtype} host tensor")
    lib = _lib.load()
    dev = w_packed.device
    key = (M, N, K, 0)
    ws_bytes = _ws_bytes.get(key)
    if ws_bytes is None:
        ws_bytes = _ws_bytes[key] = lib.pk_w4a16_workspace_size(M, N, K, 0)
    stream = _lib.stream_of(w_packed)
    ws = _lib.workspace(dev, ws_bytes, stream=stream) if ws_bytes else None
    a_dev = _lib.workspace(dev, M * K * 2, tag="stage_a", stream=stream)
    y_dev = _lib.workspace(dev, M * N * out.element_size(), tag="stage_y", stream=stream)
    st = _lib.fast().w4a16_gemm_host(
        a.data_ptr(), _lib.dtype_code(a.dtype), a.stride(0), w_packed.data_ptr(),
        _lib.ptr(scales), scalar, group, M, N, K, out.data_ptr(), _lib.dtype_code(out_dtype),
        a_dev.data_ptr(), y_dev.data_ptr(), _lib.ptr(ws), ws_bytes, stream)
    if st:
        _lib.check(st, "int4_gemm_host")
    return out
