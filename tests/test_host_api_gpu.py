"""int4_gemm_host / pk_w4a16_gemm_host: activations and outputs in host memory.

One C-ABI call copies A to the device, runs the same kernels as int4_gemm
(split_k = 0, so the same routing and split) and copies y back (decode
kernels store it through the page-locked output's mapping): the result must
equal the device-tensor call bit for bit, for page-locked and pageable
buffers, row-strided activations (the 2-D copy) and a bf16 output.
"""

import pytest
import torch

import pico_kernels_b200 as pk

pytestmark = pytest.mark.gpu


def _weights(N, K, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(K, N, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    return pk.quantize_int4_grouped(w, 128)


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (4, 1024, 2048), (32, 1024, 1024),
                                   (64, 1024, 1024), (300, 512, 256)])
def test_host_call_equals_device_call(M, N, K, pinned):
    packed, scales = _weights(N, K)
    a = torch.randn(M, K, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    if pinned:
        a = a.pin_memory()
    ref = pk.int4_gemm(a.cuda(), packed, scales).cpu()
    y = pk.int4_gemm_host(a, packed, scales)
    torch.cuda.synchronize()
    assert pk.device_status() == (0, 0)
    assert torch.equal(y, ref)


def test_strided_rows_and_bf16_output():
    M, N, K = 16, 1024, 512
    packed, scales = _weights(N, K, seed=2)
    big = torch.randn(M, K + 64, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    a = big.pin_memory()[:, :K]  # row stride K + 64: the 2-D host-to-device copy
    assert a.stride(0) == K + 64
    ref = pk.int4_gemm(a.cuda(), packed, scales, out_dtype=torch.bfloat16).cpu()
    out = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    y = pk.int4_gemm_host(a, packed, scales, out_dtype=torch.bfloat16, out=out)
    torch.cuda.synchronize()
    assert y.data_ptr() == out.data_ptr()
    assert torch.equal(y, ref)


def test_calls_in_flight_stay_ordered():
    """Several calls enqueued before one synchronisation (the staging buffers
    are reused call after call on the stream) each produce their own output."""
    M, N, K = 4, 2048, 1024
    packed, scales = _weights(N, K, seed=4)
    gen = torch.Generator().manual_seed(5)
    acts = [torch.randn(M, K, generator=gen).to(torch.bfloat16).pin_memory() for _ in range(4)]
    outs = [torch.empty((M, N)).pin_memory() for _ in range(4)]
    for a, o in zip(acts, outs):
        pk.int4_gemm_host(a, packed, scales, out=o)
    torch.cuda.synchronize()
    for a, o in zip(acts, outs):
        assert torch.equal(o, pk.int4_gemm(a.cuda(), packed, scales).cpu())


def test_device_tensors_are_rejected():
    packed, scales = _weights(256, 256)
    with pytest.raises(pk.DtypeError):
        pk.int4_gemm_host(torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda"), packed, scales)


@pytest.mark.parametrize("M", [1, 4, 8])
def test_cluster_gemv_from_host_buffers(M):
    """The one-wave cluster GEMV path from page-locked host buffers: row
    strides, several calls in flight, the result bit-equal to the
    device-tensor call."""
    N = K = 4096
    packed, scales = _weights(N, K, seed=6)
    gen = torch.Generator().manual_seed(7)
    bigs = [torch.randn(M, K + 64, generator=gen).to(torch.bfloat16).pin_memory() for _ in range(3)]
    acts = [b[:, :K] for b in bigs]
    outs = [torch.empty((M, N)).pin_memory() for _ in range(3)]
    for a, o in zip(acts, outs):
        pk.int4_gemm_host(a, packed, scales, out=o)
    torch.cuda.synchronize()
    assert pk.device_status() == (0, 0)
    for a, o in zip(acts, outs):
        assert torch.equal(o, pk.int4_gemm(a.contiguous().cuda(), packed, scales).cpu())
