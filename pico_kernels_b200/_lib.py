"""ctypes binding of libpico_b200.so (the C ABI in include/pico_b200.h).

Only plain pointers, sizes and the current CUDA stream cross the boundary.
The library is built in-tree (``python -m pico_kernels_b200.build``); if it is
missing, every call raises instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libpico_b200.so"

# pk_status
PK_OK, PK_ERR_SHAPE, PK_ERR_DTYPE, PK_ERR_ALIGN = 0, 1, 2, 3
PK_ERR_CUDA, PK_ERR_TIMEOUT, PK_ERR_WORKSPACE, PK_ERR_UNSUPPORTED = 4, 5, 6, 7
# pk_dtype
PK_F16, PK_BF16, PK_F32, PK_E4M3, PK_U8, PK_I8 = 0, 1, 2, 3, 4, 5

_DTYPE = {
    torch.float16: PK_F16,
    torch.bfloat16: PK_BF16,
    torch.float32: PK_F32,
    torch.float8_e4m3fn: PK_E4M3,
    torch.uint8: PK_U8,
    torch.int8: PK_I8,
}


class ShapeError(ValueError, AssertionError):
    """Bad shape or size. Also an AssertionError: the reference asserts."""


class DtypeError(TypeError, AssertionError):
    """Unsupported dtype. Also an AssertionError: the reference asserts."""


class KernelError(RuntimeError):
    """A CUDA call failed or a device-side bounded wait expired."""


_c = ctypes
_vp, _i64, _int, _f32, _sz = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_float, _c.c_size_t

# name -> (restype, argtypes); must match include/pico_b200.h
SIGNATURES = {
    "pk_version": (_int, []),
    "pk_last_error_string": (_c.c_char_p, []),
    "pk_device_status": (_int, [_c.POINTER(_int), _c.POINTER(_int), _int]),
    "pk_quant_int4_group": (_int, [_vp, _int, _i64, _i64, _i64, _int, _vp, _vp, _int, _vp]),
    "pk_absmax": (_int, [_vp, _int, _i64, _vp, _vp]),
    "pk_quant_int4_tensor": (_int, [_vp, _int, _i64, _f32, _vp, _vp]),
    "pk_pack_int4_n": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "pk_unpack_int4_n": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "pk_w4a16_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "pk_w4a16_gemm": (_int, [_vp, _int, _i64, _vp, _vp, _f32, _int, _i64, _i64, _i64, _vp,
                             _int, _i64, _int, _vp, _sz, _vp]),
    "pk_w4a16_gemm_noalloc": (_int, [_vp, _int, _i64, _vp, _vp, _f32, _int, _i64, _i64, _i64,
                                     _vp, _int, _i64, _int, _vp]),
    "pk_w4a16_gemm_host": (_int, [_vp, _int, _i64, _vp, _vp, _f32, _int, _i64, _i64, _i64, _vp,
                                  _int, _vp, _vp, _vp, _sz, _vp]),
    "pk_fp8_quantize": (_int, [_vp, _int, _i64, _f32, _vp, _vp]),
    "pk_fp8_gemm": (_int, [_vp, _vp, _i64, _i64, _i64, _f32, _vp, _int, _vp]),
    "pk_fp8_quantize_device": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp]),
    "pk_gptq_int4": (_int, [_vp, _vp, _i64, _i64, _int, _vp, _vp, _int, _vp, _vp]),
    "pk_fp8_gemm_scaled": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _int, _vp]),
    "pk_gemm_splitk_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "pk_gemm_splitk": (_int, [_vp, _vp, _int, _i64, _i64, _i64, _int, _vp, _vp, _sz, _vp]),
    "pk_shared_alloc": (_int, [_sz, _c.POINTER(_vp)]),
    "pk_shared_free": (_int, [_vp]),
    "pk_ipc_get_handle": (_int, [_vp, _vp]),
    "pk_ipc_open": (_int, [_vp, _c.POINTER(_vp)]),
    "pk_ipc_close": (_int, [_vp]),
    "pk_w4a16_gemm_sharded": (_int, [_vp, _int, _i64, _vp, _vp, _f32, _int, _i64, _i64, _i64,
                                     _int, _i64, _i64, _int, _int, _vp, _vp, _vp, _sz, _vp]),
    "pk_fake_quant_groups": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _int, _vp, _i64, _vp]),
    "pk_gptq_ref": (_int, [_vp, _vp, _i64, _i64, _int, _int, _vp, _vp]),
    "pk_set_wait_limit_ns": (_int, [_i64]),
    "pk_set_weight_staging": (_int, [_int]),
    "pk_debug_phase_stamps": (_int, [_vp, _sz]),
}

_lib = None
_lock = threading.Lock()


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the shared library; raise if it is missing."""
    global _lib
    lib = _lib
    if lib is not None:  # every call after the first: no lock on the hot path
        return lib
    with _lock:
        if _lib is None:
            p = Path(path) if path else LIB_PATH
            if not p.exists():
                raise ImportError(
                    f"{p} is missing: build it with `python -m pico_kernels_b200.build`")
            lib = ctypes.CDLL(str(p))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


_fast = None


def fast():
    """The CPython fast-call module (_pkfast) over the same library, or the
    ctypes library when that module was not built: both expose the hot calls
    under their C names' suffix (w4a16_gemm, w4a16_gemm_host)."""
    global _fast
    f = _fast
    if f is not None:
        return f
    lib = load()  # the library first, by path: the module then binds to it
    try:
        from . import _pkfast as mod  # noqa: PLC0415
        f = mod
    except ImportError:
        class _Ctypes:
            w4a16_gemm = lib.pk_w4a16_gemm
            w4a16_gemm_host = lib.pk_w4a16_gemm_host
        f = _Ctypes
    _fast = f
    return f


_tfast = None


def torch_fast():
    """The module _pktorch (tensor checks of int4_gemm / int4_gemm_host in
    C++, over the same library and the same cached workspaces), or None when
    it was not built; its calls return -1 for what they leave to Python."""
    global _tfast
    f = _tfast
    if f is None:
        load()  # the library first, by path: the module then binds to it
        try:
            from . import _pktorch as mod  # noqa: PLC0415
            mod.bind(_workspaces)
            f = mod
        except ImportError:
            f = False
        _tfast = f
    return f or None


def last_error() -> str:
    return load().pk_last_error_string().decode(errors="replace")


def check(status: int, what: str) -> None:
    if status == PK_OK:
        return
    msg = f"{what}: {last_error()}"
    if status in (PK_ERR_SHAPE, PK_ERR_ALIGN, PK_ERR_WORKSPACE):
        raise ShapeError(msg)
    if status == PK_ERR_DTYPE:
        raise DtypeError(msg)
    if status == PK_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise KernelError(msg)


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPE[t]
    except KeyError:
        raise DtypeError(f"unsupported dtype {t}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# torch's raw current-stream query (an int, no Stream object), when present;
# the public call below is the fallback and gives the same handle.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    """Handle of the current CUDA stream of ``t``'s device."""
    if _raw_stream is not None:
        return _raw_stream(t.get_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise DtypeError("pico_kernels_b200 runs on CUDA tensors only (no CPU path)")


def device_status(reset: bool = True) -> tuple[int, int]:
    """(code, site) recorded by a device-side bounded wait; synchronises."""
    code, where = _c.c_int(0), _c.c_int(0)
    check(load().pk_device_status(_c.byref(code), _c.byref(where), int(reset)), "pk_device_status")
    return code.value, where.value


# ---------------------------------------------------------------------------
# workspaces: one zero-filled buffer per (device, stream), grown on demand.
# The kernels leave their arrival counters at zero after every call, so a
# buffer is zeroed only when it is created.
# ---------------------------------------------------------------------------
_workspaces: dict[tuple[int, int, str], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int, tag: str = "splitk",
              stream: int | None = None) -> torch.Tensor | None:
    """The cached workspace of at least ``nbytes`` for (device, stream, tag);
    ``stream`` is the current stream's handle when the caller has it."""
    if nbytes == 0:
        return None
    index = device.index if device.index is not None else torch.cuda.current_device()
    if stream is None:
        stream = torch.cuda.current_stream(device).cuda_stream
    key = (index, stream, tag)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def set_wait_limit(seconds: float | None) -> None:
    """Limit of the kernels' device-side waits on the current device (None:
    the built-in ~2 s); a wait that runs out is reported by device_status()."""
    ns = 0 if seconds is None else max(1, int(seconds * 1e9))
    check(load().pk_set_wait_limit_ns(ns), "pk_set_wait_limit_ns")


def reset_workspaces() -> None:
    """Zero every cached workspace (needed only after a failed kernel)."""
    for buf in _workspaces.values():
        buf.zero_()
