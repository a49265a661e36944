"""Host logic of the N-sharded layers on world_size-2 gloo ranks (no GPU).

The local GEMM is injected (the oracle's dequantize-then-matmul on CPU), so
these tests check the sharding, the all-gather and the reassembly of
rank-major column blocks, against the unsharded oracle result.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import quant_ref as o
from pico_kernels_b200 import sharded


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _cpu_int4_gemm(a, packed, scales, group_size=128):
    codes = o.unpack_int4_n(packed.numpy())
    y = o.w4a16_reference(a.float().numpy(), codes, scales.float().numpy(), group_size)
    return torch.from_numpy(y)


def _cpu_fp8_gemm(a8, sa, b8, sb):
    return torch.from_numpy(o.fp8_gemm_reference(a8.numpy(), sa, b8.numpy(), sb))


def _worker(rank, world, port, M, N, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        w = rng.standard_normal((K, N), dtype=np.float32) * 0.02
        codes, s32 = o.group_quant_codes(w, 128)
        packed = torch.from_numpy(o.pack_int4_n(codes))
        scales = torch.from_numpy(s32)
        a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32))
        p_r, s_r = sharded.shard_int4(packed, scales, world, rank)
        y = sharded.sharded_int4_gemm(a, p_r, s_r, 128, world, local_gemm=_cpu_int4_gemm)
        ref = o.w4a16_reference(a.numpy(), codes, s32, 128)
        ok_int4 = bool(np.allclose(y.numpy(), ref, rtol=1e-5, atol=1e-5))

        a8, sa = o.fp8_quantize(a.numpy(), "f32")
        b8, sb = o.fp8_quantize(rng.standard_normal((K, N), dtype=np.float32), "f32")
        n0, n1 = sharded.shard_columns(N, world, rank)
        yf = sharded.sharded_fp8_gemm(torch.from_numpy(a8), sa,
                                      torch.from_numpy(np.ascontiguousarray(b8[:, n0:n1])), sb,
                                      world, local_gemm=_cpu_fp8_gemm)
        reff = o.fp8_gemm_reference(a8, sa, b8, sb)
        ok_fp8 = bool(np.allclose(yf.numpy(), reff, rtol=1e-6, atol=1e-6))

        # an exchange that declines the shape (as PeerExchange does where no
        # kernel with the fused exchange serves it): the layer still comes out
        # of the local GEMM plus the all-gather; the library GEMM is stood in
        # for by the CPU one
        class Declines:
            calls = 0

            def int4_gemm(self, *args):
                Declines.calls += 1
                return None
        saved = sharded.gemm_int4.int4_gemm
        sharded.gemm_int4.int4_gemm = _cpu_int4_gemm
        try:
            y2 = sharded.sharded_int4_gemm(a, p_r, s_r, 128, world, exchange=Declines())
        finally:
            sharded.gemm_int4.int4_gemm = saved
        ok_fallback = Declines.calls == 1 and bool(np.allclose(y2.numpy(), ref, rtol=1e-5,
                                                               atol=1e-5))
        q.put((rank, ok_int4, ok_fp8 and ok_fallback, tuple(y.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [1, 3])
def test_sharded_layers_two_gloo_ranks(M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, M, 512, 256, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=5) for _ in range(2))
    for rank, ok_int4, ok_fp8, shape in results:
        assert shape == (M, 512)
        assert ok_int4, f"rank {rank} int4"
        assert ok_fp8, f"rank {rank} fp8 or exchange fallback"


def test_shard_columns_rules():
    assert sharded.shard_columns(28672, 8, 7) == (25088, 28672)
    assert sharded.shard_columns(8192, 8, 0) == (0, 1024)
    with pytest.raises(ValueError):
        sharded.shard_columns(1000, 8, 0)


def _decision_worker(rank, world, port, q):
    """Each rank asks the library to run its slice of the same layer; rank 1's
    activations start 2 bytes off a 16-byte boundary (a view with an offset).
    No rank may be told UNSUPPORTED (the signal to fall back to the NCCL
    all-gather) unless every rank is: the aligned rank reaches the workspace
    check (it would launch the fused kernel), the misaligned one gets an
    error. Fake pointers: every call returns before touching a GPU."""
    import ctypes

    from pico_kernels_b200 import _lib
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = _lib.load()
        outs = (ctypes.c_uint64 * world)(*[4096 * (r + 1) for r in range(world)])
        flags = (ctypes.c_uint64 * world)(*[1 << 20 + r for r in range(world)])
        codes = {}
        for M, N, K in ((1, 3584, 8192), (32, 1024, 28672), (300, 1024, 1000)):
            a = 4096 + (2 if rank == 1 else 0)
            codes[M] = lib.pk_w4a16_gemm_sharded(
                a, _lib.PK_BF16, K, 8192, 16384, 1.0, 128, M, N, K, _lib.PK_F32, N * world,
                rank * N, world, rank, ctypes.addressof(outs), ctypes.addressof(flags), None, 0,
                None)
        got = [None] * world
        dist.all_gather_object(got, codes)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_fused_exchange_decision_agrees_across_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decision_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    rank, got = q.get(timeout=5)
    from pico_kernels_b200 import _lib
    for M in (1, 32, 300):
        unsupported = [g[M] == _lib.PK_ERR_UNSUPPORTED for g in got]
        assert all(unsupported) or not any(unsupported), (M, [g[M] for g in got])
    assert got[0][1] == _lib.PK_ERR_WORKSPACE and got[1][1] == _lib.PK_ERR_ALIGN
    assert got[0][32] == _lib.PK_ERR_WORKSPACE and got[1][32] == _lib.PK_ERR_ALIGN
    assert got[0][300] == got[1][300] == _lib.PK_ERR_UNSUPPORTED
