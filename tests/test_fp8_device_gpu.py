"""GPU checks of the fp8 cast with the scale kept on the device
(``gemm_fp8.quantize_device``, ``pk_fp8_quantize_device``) and the GEMM that
reads its scales from device memory (``pk_fp8_gemm_scaled``).

* The cast is the reference's ``quantize`` (gemm_fp8.py:89-95) without the
  host round trip: bytes and scale must equal the host-scale path exactly.
* The GEMM's epilogue multiplier is formed from the device scales in double
  and rounded once, as the host forms it: output equal to the host-scale call
  up to a possible last-bit difference of that multiplier (rel <= 1e-6).
* ``fp8_gemm`` (cast, cast, GEMM) runs with no host synchronisation: it is
  captured in a CUDA graph, which a ``.item()`` would make fail.
"""

import pytest
import torch

import pico_kernels_b200 as pk
from pico_kernels_b200 import gemm_fp8

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(256, 512), (3, 1001), (1, 7)])
def test_quantize_device_matches_host_scale(dt, shape):
    torch.manual_seed(sum(shape))
    x = (torch.randn(*shape, device="cuda") * 3).to(dt)
    x8_host, s_host = gemm_fp8.quantize(x)
    x8_dev, s_dev = gemm_fp8.quantize_device(x)
    assert s_dev.dtype == torch.float32 and s_dev.numel() == 1 and s_dev.is_cuda
    assert s_dev.item() == torch.tensor(s_host, dtype=torch.float32).item()
    assert torch.equal(x8_dev.view(torch.uint8), x8_host.view(torch.uint8))


def test_quantize_device_unaligned_view_and_zero_input():
    base = torch.randn(4097, device="cuda", dtype=torch.bfloat16)
    x = base[1:]  # 2-byte offset: the cast takes its scalar path
    x8_host, s_host = gemm_fp8.quantize(x)
    x8_dev, s_dev = gemm_fp8.quantize_device(x)
    assert torch.equal(x8_dev.view(torch.uint8), x8_host.view(torch.uint8))
    z8, zs = gemm_fp8.quantize_device(torch.zeros(100, device="cuda", dtype=torch.bfloat16))
    assert zs.item() == 1.0 and torch.all(z8.view(torch.uint8) == 0)
    with pytest.raises(ZeroDivisionError):  # the reference's host path raises here
        gemm_fp8.quantize(torch.zeros(100, device="cuda", dtype=torch.bfloat16))


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (4096, 4096, 4096), (100, 272, 96)])
def test_gemm_with_device_scales(M, N, K):
    torch.manual_seed(M + K)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    a8, sa = gemm_fp8.quantize(a)
    b8, sb = gemm_fp8.quantize(b)
    y_host = gemm_fp8.fp8_gemm_precast(a8, sa, b8, sb)
    a8d, sad = gemm_fp8.quantize_device(a)
    b8d, sbd = gemm_fp8.quantize_device(b)
    y_dev = gemm_fp8.fp8_gemm_precast(a8d, sad, b8d, sbd)
    assert (torch.norm(y_dev - y_host) / torch.norm(y_host)).item() <= 1e-6
    # mixed: one float, one device scale
    y_mix = gemm_fp8.fp8_gemm_precast(a8, sa, b8d, sbd, out_dtype=torch.bfloat16)
    assert (torch.norm(y_mix.float() - y_host) / torch.norm(y_host)).item() <= 5e-3
    assert pk.device_status() == (0, 0)


def test_fp8_gemm_is_graph_capturable():
    torch.manual_seed(5)
    a = torch.randn(1024, 1024, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(1024, 1024, device="cuda", dtype=torch.bfloat16)
    eager = gemm_fp8.fp8_gemm(a, b)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        gemm_fp8.fp8_gemm(a, b)  # warm-up on the capture stream
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            y = gemm_fp8.fp8_gemm(a, b)
    torch.cuda.current_stream().wait_stream(s)
    a.mul_(2.0)  # new inputs: the replay recomputes the scales on the device
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, gemm_fp8.fp8_gemm(a, b))
    assert (torch.norm(y - 2 * eager) / torch.norm(eager)).item() < 1e-6
    ref = a.float() @ b.float()
    assert (torch.norm(y - ref) / torch.norm(ref)).item() < 0.10  # tests/test_gemm_fp8.py:28
    del g
