"""The C-ABI library loads without a GPU and exports what the header declares."""

import ctypes
import re
from pathlib import Path

import pytest

from pico_kernels_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "pico_b200.h").read_text()
    return sorted(set(re.findall(r"PK_API\s+[\w\s\*]+?\b(pk_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = header_functions()
    for must in ("pk_quant_int4_group", "pk_pack_int4_n", "pk_w4a16_gemm", "pk_fp8_gemm",
                 "pk_fp8_quantize_device", "pk_fp8_gemm_scaled",
                 "pk_gemm_splitk", "pk_w4a16_workspace_size", "pk_last_error_string"):
        assert must in names


def test_library_exports_every_declared_symbol():
    if not _lib.LIB_PATH.exists():
        pytest.fail(f"{_lib.LIB_PATH} not built (run python -m pico_kernels_b200.build)")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert sorted(_lib.SIGNATURES) == header_functions()


def test_host_only_calls_work_without_gpu():
    lib = _lib.load()
    assert lib.pk_version() >= 100
    # shape validation happens on the host before any CUDA call
    st = lib.pk_pack_int4_n(None, 4, 3, None, None)
    assert st == _lib.PK_ERR_SHAPE
    assert _lib.last_error() != ""
    with pytest.raises(ValueError):
        _lib.check(st, "pack")
    with pytest.raises(AssertionError):  # the reference's error type still catches it
        _lib.check(st, "pack")
    # device-scale fp8 entries validate their pointers on the host too
    assert lib.pk_fp8_quantize_device(None, _lib.PK_BF16, 16, None, None, None, None) == \
        _lib.PK_ERR_SHAPE
    assert lib.pk_fp8_quantize_device(8, _lib.PK_BF16, 16, 8, 64, 64, None) == _lib.PK_ERR_SHAPE
    assert lib.pk_fp8_gemm_scaled(16, 16, 16, 16, 16, None, None, 16, _lib.PK_F32, None) == \
        _lib.PK_ERR_SHAPE
    # GPTQ producer: odd N and oversized groups are rejected on the host
    assert lib.pk_gptq_int4(16, 16, 64, 33, 16, 16, 16, _lib.PK_F32, 16, None) == _lib.PK_ERR_SHAPE
    assert lib.pk_gptq_int4(16, 16, 64, 32, 256, 16, 16, _lib.PK_F32, 16, None) == _lib.PK_ERR_SHAPE
    # host-buffer W4A16: missing staging buffers, a short row stride and a bad
    # output dtype are caught before any copy is enqueued
    args = dict(a_host=64, a_dtype=_lib.PK_BF16, lda=256, wp=64, scales=64, scalar=1.0, group=128,
                M=1, N=256, K=256, y_host=64, out_dtype=_lib.PK_F32, a_dev=64, y_dev=64, ws=None,
                ws_bytes=0, stream=None)

    def host_call(**kw):
        a = dict(args, **kw)
        return lib.pk_w4a16_gemm_host(*a.values())
    assert host_call(a_dev=None) == _lib.PK_ERR_SHAPE
    assert host_call(y_host=None) == _lib.PK_ERR_SHAPE
    assert host_call(lda=128) == _lib.PK_ERR_SHAPE
    assert host_call(M=0) == _lib.PK_ERR_SHAPE
    assert host_call(a_dtype=_lib.PK_F32) == _lib.PK_ERR_DTYPE
    assert host_call(out_dtype=_lib.PK_I8) == _lib.PK_ERR_DTYPE
    # sharded W4A16: bad world / rank / slice are shape errors; shapes no kernel
    # with the fused exchange serves (K not a multiple of 64) report
    # PK_ERR_UNSUPPORTED so the caller falls back to NCCL
    outs = (ctypes.c_uint64 * 2)(4096, 8192)
    flags = (ctypes.c_uint64 * 2)(4096, 8192)
    sh = dict(a=4096, a_dtype=_lib.PK_BF16, lda=1024, wp=4096, scales=4096, scalar=1.0,
              group=128, M=1, N=1024, K=1024, out_dtype=_lib.PK_F32, ldo=2048, n_offset=0,
              world=2, rank=0, outs=ctypes.addressof(outs), flags=ctypes.addressof(flags),
              ws=4096, ws_bytes=1 << 20, stream=None)

    def sharded_call(**kw):
        a = dict(sh, **kw)
        return lib.pk_w4a16_gemm_sharded(*a.values())
    assert sharded_call(world=9) == _lib.PK_ERR_SHAPE
    assert sharded_call(rank=2) == _lib.PK_ERR_SHAPE
    assert sharded_call(n_offset=1536) == _lib.PK_ERR_SHAPE
    assert sharded_call(M=300, K=1000, lda=1000) == _lib.PK_ERR_UNSUPPORTED
    # the fused-or-NCCL choice depends on the shape only: a misaligned A or
    # leading dimension on a covered shape is an error (never UNSUPPORTED,
    # which would send this rank alone to the all-gather), and an uncovered
    # shape is UNSUPPORTED whatever the pointers
    assert sharded_call(a=4098) == _lib.PK_ERR_ALIGN
    assert sharded_call(lda=1025) == _lib.PK_ERR_ALIGN
    assert sharded_call(wp=4100) == _lib.PK_ERR_ALIGN
    assert sharded_call(M=300, K=1000, lda=1000, a=4098) == _lib.PK_ERR_UNSUPPORTED
    # the fused prefill serves the other shapes: misaligned operands are errors there too
    assert sharded_call(M=300, a=4098) == _lib.PK_ERR_ALIGN
    assert sharded_call(M=64, N=256, K=256, ldo=512, a=4098) in (_lib.PK_ERR_UNSUPPORTED,
                                                                 _lib.PK_ERR_ALIGN)
    assert sharded_call(M=64, N=256, K=256, ldo=512, a=4098) == \
        (_lib.PK_ERR_UNSUPPORTED if sharded_call(M=64, N=256, K=256, ldo=512, ws=None)
         == _lib.PK_ERR_UNSUPPORTED else _lib.PK_ERR_ALIGN)


def test_workspace_size_is_host_only():
    lib = _lib.load()
    assert lib.pk_w4a16_workspace_size(1, 4096, 4096, 1) == 0
    assert lib.pk_w4a16_workspace_size(1, 4096, 4096, 8) > 0
    assert lib.pk_w4a16_workspace_size(1, 4096, 4096, 8) < lib.pk_w4a16_workspace_size(16, 4096, 4096, 8)


def test_fast_call_module_shares_the_library():
    # the CPython fast-call module binds to the library ctypes loaded: an
    # error it records is the one pk_last_error_string reports
    from pico_kernels_b200 import _lib
    f = _lib.fast()
    assert f.__name__.endswith("_pkfast"), "the fast-call module is built beside the library"
    st = f.w4a16_gemm(0, _lib.PK_BF16, 256, 0, None, 1.0, 128, 1, 256, 256, 0, _lib.PK_F32, 256,
                      0, None, 0, 0)
    assert st == _lib.PK_ERR_SHAPE
    assert "null pointer" in _lib.last_error()
    st = f.w4a16_gemm_host(0, _lib.PK_BF16, 256, 0, None, 1.0, 128, 1, 256, 256, 0, _lib.PK_F32,
                           0, 0, None, 0, 0)
    assert st != _lib.PK_OK
    import pytest
    with pytest.raises(TypeError):
        f.w4a16_gemm(0, 1)


def test_torch_fast_module_leaves_host_tensors_to_python():
    # _pktorch serves CUDA tensors only: host tensors go back to the Python
    # path (-1), which raises the documented error
    import pytest
    import torch

    import pico_kernels_b200 as pk
    from pico_kernels_b200 import _lib
    tf = _lib.torch_fast()
    assert tf is not None and tf.__name__.endswith("_pktorch")
    a = torch.zeros(1, 256, dtype=torch.bfloat16)
    wp = torch.zeros(256, 128, dtype=torch.uint8)
    out = torch.zeros(1, 256)
    assert tf.int4_gemm(a, wp, 1.0, None, out, torch.float32, 0) == -1
    assert tf.int4_gemm_host(a, wp, 1.0, None, out, torch.float32) == -1
    with pytest.raises(_lib.DtypeError):
        pk.int4_gemm(a, wp, 1.0, out=out)
    with pytest.raises(TypeError):
        tf.int4_gemm(a)
