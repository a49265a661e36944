"""The C++ tensor-check path of int4_gemm / int4_gemm_host (module _pktorch).

The wrappers hand each call to _pktorch first, which checks the tensors in
C++, allocates a device output when none is given, and calls the same C ABI;
what it does not serve it returns to the Python path (-1). Results must
equal the Python path's bit for bit (same kernel routing, same workspaces),
the C++ path must actually serve the common calls, and misuse must raise the
Python path's errors.
"""

import pytest
import torch

import pico_kernels_b200 as pk
from pico_kernels_b200 import _lib

pytestmark = pytest.mark.gpu


def _weights(N, K, seed=0, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(K, N, device="cuda", generator=g) * 0.02).to(dtype)
    return pk.quantize_int4_grouped(w, 128)


def _python_path(fn):
    """Run fn with the C++ path switched off."""
    saved = _lib._tfast
    _lib._tfast = False
    try:
        return fn()
    finally:
        _lib._tfast = saved


def test_module_is_built():
    assert _lib.torch_fast() is not None, "_pktorch is built beside the library"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (4, 2048, 1024), (8, 28672, 512),
                                   (16, 1024, 2048), (64, 1024, 1024), (300, 512, 256)])
def test_device_call_equals_python_path(M, N, K, dtype, out_dtype):
    packed, scales = _weights(N, K, dtype=dtype)
    a = torch.randn(M, K, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    a = a.to(dtype)
    ref = _python_path(lambda: pk.int4_gemm(a, packed, scales, out_dtype=out_dtype,
                                            out=torch.empty(M, N, device="cuda",
                                                            dtype=out_dtype)))
    out = torch.full((M, N), float("nan"), device="cuda", dtype=out_dtype)
    res = _lib.torch_fast().int4_gemm(a, packed, scales, None, out, out_dtype, 0)
    assert res is out, "the C++ path serves a call whose workspace exists"
    torch.cuda.synchronize()
    assert pk.device_status() == (0, 0)
    assert torch.equal(out, ref)
    y = pk.int4_gemm(a, packed, scales, out_dtype=out_dtype, out=out)
    assert y is out and torch.equal(y, ref)
    # no out: allocated by the C++ path on a's device
    y = _lib.torch_fast().int4_gemm(a, packed, scales, None, None, out_dtype, 0)
    assert isinstance(y, torch.Tensor) and y.dtype == out_dtype and y.device == a.device
    assert y.shape == (M, N) and torch.equal(y, ref)
    assert torch.equal(pk.int4_gemm(a, packed, scales, out_dtype=out_dtype), ref)


def test_scalar_scale_and_split_k():
    M, N, K = 4, 1024, 2048
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randint(0, 256, (K, N // 2), device="cuda", generator=g, dtype=torch.uint8)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    for split in (0, 4):
        ref = _python_path(lambda: pk.int4_gemm(a, q, 0.03, split_k=split,
                                                out=torch.empty(M, N, device="cuda")))
        out = torch.empty(M, N, device="cuda")
        assert _lib.torch_fast().int4_gemm(a, q, 0.03, None, out, torch.float32, split) is out
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_unserved_calls_fall_back_with_the_same_errors():
    packed, scales = _weights(1024, 512)
    a = torch.randn(2, 512, device="cuda").to(torch.bfloat16)
    tf = _lib.torch_fast()
    wrong = torch.empty(2, 1000, device="cuda")
    assert tf.int4_gemm(a, packed, scales, None, wrong, torch.float32, 0) == -1
    with pytest.raises(_lib.ShapeError):
        pk.int4_gemm(a, packed, scales, out=wrong)
    out = torch.empty(2, 1024, device="cuda")
    with pytest.raises(_lib.ShapeError):  # out dtype differs from out_dtype
        pk.int4_gemm(a, packed, scales, out_dtype=torch.bfloat16, out=out)
    # a column-strided A and fp32 scales: the Python path copies / casts them
    at = torch.randn(512, 2, device="cuda").to(torch.bfloat16).t()
    assert tf.int4_gemm(at, packed, scales, None, out, torch.float32, 0) == -1
    ref = pk.int4_gemm(at.contiguous(), packed, scales)
    assert torch.equal(pk.int4_gemm(at, packed, scales, out=out), ref)
    assert tf.int4_gemm(a, packed, scales.float(), None, out, torch.float32, 0) == -1
    with pytest.raises(_lib.DtypeError):
        pk.int4_gemm(a.cpu(), packed, scales, out=out)


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (4, 1024, 2048), (32, 1024, 1024),
                                   (300, 512, 256)])
def test_host_call_equals_python_path(M, N, K):
    packed, scales = _weights(N, K, seed=3)
    a = torch.randn(M, K, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    a = a.pin_memory()
    ref = _python_path(lambda: pk.int4_gemm_host(a, packed, scales,
                                                 out=torch.empty(M, N).pin_memory()))
    torch.cuda.synchronize()
    out = torch.full((M, N), float("nan")).pin_memory()
    res = _lib.torch_fast().int4_gemm_host(a, packed, scales, None, out, torch.float32)
    assert res is out, "the C++ path serves a call whose staging buffers exist"
    torch.cuda.synchronize()
    assert pk.device_status() == (0, 0)
    assert torch.equal(out, ref)
    # a device tensor where a host one belongs: the Python path's error
    with pytest.raises(_lib.DtypeError):
        pk.int4_gemm_host(a.cuda(), packed, scales, out=out)
