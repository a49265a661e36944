"""The allocation-free decode entry point, pk_w4a16_gemm_noalloc.

It serves callers that cannot call cudaMalloc (a runtime that owns every
byte of device memory, a decode loop that cannot take cudaMalloc's implicit
synchronization): instead of a caller-provided workspace, its split-K partials
go through a static scratch array inside the library. These tests call it
through the C ABI and check it against pk_w4a16_gemm (the existing entry
point) with the same split: the decode kernel sums the K splits in the same
order whether it reduces through cluster shared memory or through memory, so
the two outputs must be equal bit for bit. Each case runs twice in a row,
since the second call starts from the scratch the first one left behind. This
file is named to be collected last; it also passes when run on its own in a
fresh process.
"""

import pytest
import torch

import pico_kernels_b200 as pk
from pico_kernels_b200 import _lib

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 4 << 20  # the entry point's static partials


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


def _split_used(M, N, K, split_k):
    """The split the entry point runs: an explicit one as given, the automatic
    one (two CTAs per SM over the 128-column tiles, at most 8) lowered until
    its partials fit the scratch."""
    if split_k > 0:
        return min(split_k, K // 128)
    tiles = N // 128
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    auto = max(1, min(2 * sms // tiles, 8, K // 128))
    fit = SCRATCH_BYTES // (tiles * M * 128 * 4)
    return max(1, min(auto, fit))


@pytest.mark.parametrize("M,N,K,split", [(1, 4096, 4096, 8), (16, 4096, 4096, 8),
                                         (4, 2048, 4096, 16), (16, 1024, 8192, 0),
                                         (32, 5120, 4096, 0), (30, 6144, 2048, 0)])
def test_noalloc_matches_existing_entry_twice(M, N, K, split):
    a, packed, scales = _case(M, N, K, seed=M + split)
    used = _split_used(M, N, K, split)
    ref = pk.int4_gemm(a, packed, scales, split_k=used)
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        st = _noalloc(a, packed, scales, split, out)
        assert st == _lib.PK_OK, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), (call, (out - ref).abs().max().item())
    assert pk.device_status() == (0, 0)


def test_noalloc_automatic_split_shrinks_to_fit():
    # M = 32 over 40 column tiles: the automatic split (7 on 148 SMs) needs
    # 40 * 7 * 32 * 512 B = 4.4 MiB of partials, more than the scratch holds;
    # the entry point lowers it instead of rejecting the call
    M, N, K = 32, 5120, 4096
    assert 40 * 7 * 32 * 512 > SCRATCH_BYTES
    a, packed, scales = _case(M, N, K, seed=11)
    out = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    assert _noalloc(a, packed, scales, 0, out) == _lib.PK_OK, _lib.last_error()
    ref = pk.int4_gemm(a, packed, scales)
    torch.cuda.synchronize()
    rel = (torch.norm(out - ref) / torch.norm(ref)).item()
    assert rel <= 5e-3, rel


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
