"""The allocation-free decode entry point, pk_w4a16_gemm_noalloc.

It serves callers that cannot call cudaMalloc (a runtime that owns every
byte of device memory, a decode loop that cannot take cudaMalloc's implicit
synchronization): instead of a caller-provided workspace, its split-K partials
go through a static scratch array inside the library. These tests call it
through the C ABI and check it against pk_w4a16_gemm (the existing entry
point, which reduces through thread-block-cluster shared memory) within the
W4A16 tolerance the other tests use, twice in a row, since the second call
runs on scratch the first one left behind. This file is named to be collected
last; it also passes when run on its own in a fresh process.
"""

import pytest
import torch

import pico_kernels_b200 as pk
from pico_kernels_b200 import _lib

pytestmark = pytest.mark.gpu


def _case(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(K, N, generator=g) * 0.02).to(torch.bfloat16).cuda()
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    packed, scales = pk.quantize_int4_grouped(w, 128)
    return a, packed, scales


def _noalloc(a, packed, scales, split_k, out):
    M, K = a.shape
    N = out.shape[1]
    lib = _lib.load()
    return lib.pk_w4a16_gemm_noalloc(a.data_ptr(), _lib.PK_BF16, K, packed.data_ptr(),
                                     scales.data_ptr(), 1.0, 128, M, N, K, out.data_ptr(),
                                     _lib.PK_F32, N, split_k,
                                     torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("M,N,K,split", [(1, 4096, 4096, 8), (16, 4096, 4096, 8),
                                         (4, 2048, 4096, 16), (16, 1024, 8192, 0)])
def test_noalloc_matches_existing_entry_twice(M, N, K, split):
    a, packed, scales = _case(M, N, K, seed=M + split)
    ref = pk.int4_gemm(a, packed, scales, split_k=split)
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        st = _noalloc(a, packed, scales, split, out)
        assert st == _lib.PK_OK, _lib.last_error()
        torch.cuda.synchronize()
        rel = (torch.norm(out - ref) / torch.norm(ref)).item()
        assert rel <= 5e-3, (call, rel)
        assert (out - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    assert pk.device_status() == (0, 0)


def test_noalloc_rejects_requests_beyond_its_scratch():
    # 16 x 32768 outputs split 16 ways needs 256 * 16 * 16 * 512 B = 32 MiB > 4 MiB
    a, packed, scales = _case(16, 32768, 2048, seed=5)
    out = torch.zeros((16, 32768), dtype=torch.float32, device="cuda")
    st = _noalloc(a, packed, scales, 16, out)
    assert st == _lib.PK_ERR_WORKSPACE
    assert "scratch" in _lib.last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0  # nothing was launched


def test_noalloc_rejects_non_decode_shapes():
    a, packed, scales = _case(40, 256, 512, seed=6)    # M > 32: not a decode shape
    out = torch.zeros((40, 256), dtype=torch.float32, device="cuda")
    assert _noalloc(a, packed, scales, 0, out) == _lib.PK_ERR_UNSUPPORTED
