"""Failure detection on the GPU without a GPU fault.

Every device-side wait of the library is bounded; pk_set_wait_limit_ns makes
the bound short enough to test. A sharded layer is called with world = 2 on
one GPU: its "peer" buffers are local memory and nothing ever increments this
rank's arrival flag, so the kernel's last CTA waits for a peer that never
comes. With a 10 ms limit the wait runs out, the kernel records
PK_ERR_TIMEOUT and the site (303 the GEMV, 104 the tensor-core decode kernel,
404 the skinny kernel) in the device status word and returns: the process and
the GPU stay usable, and the next ordinary call gives the exact result.

The split-K reductions never wait for their contributors (the last of a
tile's CTAs to arrive sums the partials, counted by an atomic), so a
contributor that never arrives cannot hang a later call; what it leaves is an
arrival counter off by its missing count. The test plants such a counter in
the cached workspace: the call still completes, and after
reset_workspaces() the result is exact again.
"""

import ctypes

import pytest
import torch

import pico_kernels_b200 as pk
from pico_kernels_b200 import _lib

pytestmark = pytest.mark.gpu


def _layer(M, N, K, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn(K, N, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    packed, scales = pk.quantize_int4_grouped(w, 128)
    return a, packed, scales


@pytest.mark.parametrize("M,site", [(1, 303), (16, 104), (64, 404)])
def test_peer_that_never_arrives_times_out(M, site):
    N, K = 4096, 4096
    a, packed, scales = _layer(M, N, K, seed=M)
    ref = pk.int4_gemm(a, packed, scales)
    assert pk.device_status() == (0, 0)
    lib = _lib.load()
    bufs = [torch.full((M, 2 * N), float("nan"), device="cuda") for _ in range(2)]
    flags = torch.zeros(4, dtype=torch.int64, device="cuda")  # rank 0's and rank 1's words
    ws_bytes = max(lib.pk_w4a16_workspace_size(M, N, K, 0), 1 << 16)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    outs = (ctypes.c_uint64 * 2)(bufs[0].data_ptr(), bufs[1].data_ptr())
    fl = (ctypes.c_uint64 * 2)(flags.data_ptr(), flags.data_ptr() + 16)
    pk.set_wait_limit(0.01)
    try:
        st = lib.pk_w4a16_gemm_sharded(
            a.data_ptr(), _lib.PK_BF16, K, packed.data_ptr(), scales.data_ptr(), 1.0, 128, M, N, K,
            _lib.PK_F32, 2 * N, 0, 2, 0, ctypes.addressof(outs), ctypes.addressof(fl),
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        if st == _lib.PK_ERR_UNSUPPORTED:
            pytest.skip(f"no kernel with the fused exchange serves M={M} here")
        assert st == _lib.PK_OK, _lib.last_error()
        torch.cuda.synchronize()  # returns: the wait is bounded
        assert pk.device_status() == (_lib.PK_ERR_TIMEOUT, site)
    finally:
        pk.set_wait_limit(None)
    # the kernel stored its columns into both buffers before waiting, and it
    # added its arrival to the (local) peer flag: 1 in rank 1's count
    assert int(flags[2]) == 1
    for b in bufs:
        torch.testing.assert_close(b[:, :N], ref, rtol=0, atol=0)
        assert torch.isnan(b[:, N:]).all()
    # the context is intact: the next ordinary call is exact
    pk.reset_workspaces()
    assert torch.equal(pk.int4_gemm(a, packed, scales), ref)
    assert pk.device_status() == (0, 0)


def test_wait_limit_rejects_negative_and_restores_default():
    lib = _lib.load()
    assert lib.pk_set_wait_limit_ns(-1) == _lib.PK_ERR_SHAPE
    pk.set_wait_limit(0.5)
    pk.set_wait_limit(None)
    a, packed, scales = _layer(4, 2048, 2048, seed=9)
    y = pk.int4_gemm(a, packed, scales)  # an ordinary call under the default limit
    torch.cuda.synchronize()
    assert pk.device_status() == (0, 0)
    assert torch.isfinite(y).all()


def test_split_k_with_a_missing_contributor_is_cleared_by_reset():
    M, N, K, split = 4, 2048, 4096, 16  # > 8: the workspace (last-arriver) reduction
    a, packed, scales = _layer(M, N, K, seed=5)
    good = pk.int4_gemm(a, packed, scales, split_k=split)
    stream = torch.cuda.current_stream().cuda_stream
    ws = _lib.workspace(a.device, _lib.load().pk_w4a16_workspace_size(M, N, K, split),
                        stream=stream)
    counters = ws.view(torch.int32)
    assert int(counters[: N // 128].abs().sum()) == 0  # re-armed by every call
    counters[0] = 1  # tile 0: one arrival from a contributor that never finished
    bad = pk.int4_gemm(a, packed, scales, split_k=split)
    torch.cuda.synchronize()  # completes: no reduction waits for a contributor
    assert pk.device_status() == (0, 0)
    assert torch.equal(bad[:, 128:], good[:, 128:])  # the other tiles are untouched
    pk.reset_workspaces()
    assert int(counters[: N // 128].abs().sum()) == 0
    assert torch.equal(pk.int4_gemm(a, packed, scales, split_k=split), good)
