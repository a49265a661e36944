"""N-sharded W4A16 / fp8 layers on GPUs with NCCL (one process per GPU).

With at least two (four, eight) GPUs, as many ranks each compute their column slice with the
sm_100a kernels and all-gather the output over NVLink (NCCL, or the fused
peer-store exchange inside the GEMV, decode and skinny kernels); the result
must equal the unsharded kernel's output (same kernels, same per-column
arithmetic). With one GPU the single-rank paths are checked.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import pico_kernels_b200 as pk
from pico_kernels_b200 import gemm_fp8, sharded

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _layer(M, N, K, device):
    g = torch.Generator(device=device).manual_seed(0)
    w = (torch.randn(K, N, device=device, generator=g) * 0.02).to(torch.bfloat16)
    a = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
    packed, scales = pk.quantize_int4_grouped(w, 128)
    return a, packed, scales


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        ok = []
        for M, N, K in ((1, 2048, 1024), (16, 1024, 2048), (40, 1024, 512)):
            a, packed, scales = _layer(M, N, K, dev)
            full = pk.int4_gemm(a, packed, scales)
            p_r, s_r = sharded.shard_int4(packed, scales, world, rank)
            y = sharded.sharded_int4_gemm(a, p_r, s_r, 128, world)
            # the unsharded and sharded runs may pick different split-K factors
            rel = (torch.norm(y - full) / torch.norm(full)).item()
            ok.append(rel < 1e-5)
        g = torch.Generator(device=dev).manual_seed(1)  # the same inputs on every rank
        a8, sa = gemm_fp8.quantize(torch.randn(256, 512, device=dev, generator=g))
        b8, sb = gemm_fp8.quantize(torch.randn(512, 1024, device=dev, generator=g))
        full = gemm_fp8.fp8_gemm_precast(a8, sa, b8, sb)
        n0, n1 = sharded.shard_columns(1024, world, rank)
        y = sharded.sharded_fp8_gemm(a8, sa, b8[:, n0:n1].contiguous(), sb, world)
        ok.append(bool(torch.equal(y, full)))
        # fused exchange: the local kernel writes every rank's output over
        # NVLink -- the GEMV (M = 1), the decode kernel (M = 16, 32: cluster
        # split-K) and the skinny kernel (M = 64, 200)
        for n_full, max_m, cases in ((8192, 64, ((1, 4096), (1, 2048), (16, 1024), (32, 2048),
                                                  (1, 4096), (64, 1024))),
                                     (40960, 256, ((200, 512), (200, 512)))):
            ex = sharded.PeerExchange(max_m=max_m, n_full=n_full)
            try:
                for it, (M, K) in enumerate(cases):
                    a, packed, scales = _layer(M, n_full, K, dev)
                    a = a + it  # a different input on every call
                    full = pk.int4_gemm(a, packed, scales)
                    p_r, s_r = sharded.shard_int4(packed, scales, world, rank)
                    y = ex.int4_gemm(a, p_r, s_r, 128)
                    if y is None:
                        ok.append(("not fused", M, K))
                        continue
                    rel = (torch.norm(y - full) / torch.norm(full)).item()
                    ok.append(rel < 1e-5 and pk.device_status() == (0, 0))
            finally:
                ex.close()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K", [(1, 1024, 2048), (1, 4096, 4096), (4, 1024, 2048),
                                   (8, 3072, 4096), (8, 4096, 4096), (16, 1024, 2048),
                                   (32, 1024, 1024), (64, 1024, 1024), (200, 20480, 512),
                                   (300, 2048, 1024), (512, 1024, 2048)])
def test_sharded_entry_one_rank(M, N, K):
    """pk_w4a16_gemm_sharded at world = 1 (no flag barrier): each kernel with
    the exchange epilogue (the stream-K and cluster GEMVs, the decode, skinny
    and fused prefill kernels) writes exactly its column slice of the
    full-width buffer, bit-identical to the unsharded call (same kernel, same
    split)."""
    import ctypes
    from pico_kernels_b200 import _lib
    dev = torch.device("cuda")
    a, packed, scales = _layer(M, N, K, dev)
    ref = pk.int4_gemm(a, packed, scales)
    lib = _lib.load()
    n_off, n_full = 256, N + 512
    y = torch.full((M, n_full), 7.0, device=dev)
    flag = torch.zeros(4, dtype=torch.int64, device=dev)
    ws = torch.zeros(max(lib.pk_w4a16_workspace_size(M, N, K, 0), 1 << 16), dtype=torch.uint8,
                     device=dev)
    outs = (ctypes.c_uint64 * 1)(y.data_ptr())
    flags = (ctypes.c_uint64 * 1)(flag.data_ptr())
    rc = lib.pk_w4a16_gemm_sharded(
        a.data_ptr(), _lib.PK_BF16, K, packed.data_ptr(), scales.data_ptr(), 1.0, 128, M, N, K,
        _lib.PK_F32, n_full, n_off, 1, 0, ctypes.addressof(outs), ctypes.addressof(flags),
        ws.data_ptr(), ws.numel(), _lib.stream_of(a))
    _lib.check(rc, "pk_w4a16_gemm_sharded")
    assert pk.device_status() == (0, 0)
    assert torch.equal(y[:, n_off:n_off + N], ref)
    assert bool((y[:, :n_off] == 7.0).all()) and bool((y[:, n_off + N:] == 7.0).all())


def test_single_rank_path():
    a, packed, scales = _layer(4, 1024, 1024, torch.device("cuda"))
    y = sharded.sharded_int4_gemm(a, packed, scales, 128, world=1)
    assert torch.equal(y, pk.int4_gemm(a, packed, scales))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_exchange(world):
    """`world` ranks, one per GPU: the NCCL paths and the fused exchange
    (every rank's flag barrier adds to world - 1 peers' flags)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for rank, ok in sorted(q.get(timeout=5) for _ in range(world)):
        assert all(ok), (rank, ok)
