"""GPU parity of the cluster form of the W4A16 GEMV (M = 1..8 on small layers:
one wave of one CTA per SM, mma.sync tiles of exactly decoded fp16 operands).

Every product is exact (weights as (q + 8) * 2^-24 fp16 subnormals, bf16
activations scaled into fp16 per output row by 2^S_m, fp32 accumulators), the
+8 offsets and group scales are folded per 512-row unit, so the bounds against
the oracle's fp32 dequantize-then-matmul are tight: rel-Frobenius <= 1e-5 and
max-abs <= 1e-4 * max|Y|. The K split is reduced in CTA order inside each
cluster, so results are bitwise reproducible, with and without weight staging
(which changes only when the weights are loaded). The phase stamps the kernel
writes on request show which kernel ran: one row per CTA, strips * split rows.
Shapes: 128-column strips split over at most 4 CTAs in K (a cluster), at most
4 units of 512 rows per CTA, at least 3/4 of the SMs busy.
"""

import ctypes

import pytest
import torch

import pico_kernels_b200 as pk
from pico_kernels_b200 import _lib

from test_gemv_gpu import check_tight, make_case

pytestmark = pytest.mark.gpu


def _sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def _split(N, K):
    return min(4, _sms() // (N // 128), K // 512)


def _cluster_grid(N, K):
    """CTAs of the cluster GEMV for this shape, or 0 when it does not run
    (128-column strips, at most 4 CTAs per strip, at most 4 units of 512
    rows per CTA, at least 3/4 of the SMs busy)."""
    s = _split(N, K)
    if N % 128 or K % 512 or s < 2 or 4 * (N // 128) * s < 3 * _sms():
        return 0
    if (K // 512 + s - 1) // s > 4:
        return 0
    return (N // 128) * s


class Stamps:
    """pk_debug_phase_stamps around a block of one launch: ``rows()`` gives its
    per-CTA stamps (launches alternate between the buffer's two halves)."""

    def __init__(self, rows=1024):
        self.buf = torch.zeros((rows, 8), dtype=torch.int64, device="cuda")

    def rows(self):
        halves = self.buf.cpu().view(2, -1, 8)
        used = [h for h in halves if (h[:, 0] > 0).any()]
        assert len(used) == 1, "one launch recorded"
        return used[0]

    def __enter__(self):
        torch.cuda.synchronize()
        _lib.check(_lib.load().pk_debug_phase_stamps(self.buf.data_ptr(),
                                                     self.buf.numel() * 8), "stamps")
        return self

    def __exit__(self, *exc):
        torch.cuda.synchronize()
        _lib.load().pk_debug_phase_stamps(None, 0)


def _staging(mode):
    _lib.check(_lib.load().pk_set_weight_staging(mode), "weight staging")


CASES = [(1, 4096, 4096), (1, 8192, 2048), (1, 5120, 4096), (1, 4608, 2048), (1, 3584, 8192),
         (2, 4096, 4096), (2, 8192, 2048), (3, 5120, 4096), (3, 4096, 4096), (3, 3584, 8192),
         (4, 4096, 4096), (5, 8192, 2048), (6, 4608, 2048), (7, 3584, 8192), (8, 4096, 4096),
         (8, 5120, 4096)]


@pytest.mark.parametrize("M,N,K", CASES)
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_cluster_gemv_vs_oracle(M, N, K, dt):
    grid = _cluster_grid(N, K)
    assert grid > 0, "shape chosen to run the cluster GEMV"
    a, packed, scales, ref = make_case(M, N, K, dt, seed=M + N // 256 + K // 256)
    with Stamps() as st:
        y = pk.int4_gemm(a, packed, scales)
    check_tight(y, ref, f"M={M} N={N} K={K} {dt}")
    rows = st.rows()
    assert (rows[:grid, 0] > 0).all() and (rows[grid:, 0] == 0).all(), "the cluster GEMV ran"
    units = K // 512
    assert int(rows[:grid, 6].sum()) == units * (N // 128)  # every unit once
    t = rows[:grid, :5]
    assert (t[:, 1:] >= t[:, :-1]).all(), "phases in order"
    assert pk.device_status() == (0, 0)


def test_nine_rows_take_the_tcgen05_decode():
    # M = 9 is past the mma's n8 block: the tcgen05 decode kernel runs (no
    # GEMV stamps) and the result still matches at its bf16 tolerance
    a, packed, scales, ref = make_case(9, 4096, 4096, seed=11)
    with Stamps() as st:
        y = pk.int4_gemm(a, packed, scales)
        torch.cuda.synchronize()
        assert not (st.buf[:, 0] > 0).any().item(), "no GEMV ran"
    r = torch.from_numpy(ref).to(y.device)
    rel = (torch.norm(y.float() - r) / torch.norm(r)).item()
    assert rel <= 1e-2, rel


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_rows_far_apart_in_magnitude(dt):
    # each output row has its own activation scale 2^S_m in the tensor-core
    # form: rows 2^-40 / 2^40 apart (bf16; fp16: 2^-12 / 2^3, within its
    # range), an all-zero row and subnormal activations each keep the tight
    # bound on their own
    M, N, K = 5, 4096, 4096
    a, packed, scales, _ = make_case(M, N, K, dt, seed=21)
    af = a.float()
    lo, hi = (2.0 ** -40, 2.0 ** 40) if dt == torch.bfloat16 else (2.0 ** -12, 2.0 ** 3)
    af[0] *= lo
    af[1] *= hi
    af[2] = 0.0
    af[3] *= 2.0 ** -130 if dt == torch.bfloat16 else 2.0 ** -16
    a = af.to(dt)
    y = pk.int4_gemm(a, packed, scales).float().cpu()
    w = (pk.unpack_int4_n(packed).float() * scales.float().repeat_interleave(128, 0)).cpu()
    ref = a.float().cpu().double() @ w.double()
    for m in range(M):
        r = ref[m]
        if m == 2:
            assert torch.equal(y[m], torch.zeros_like(y[m]))
            continue
        rel = (torch.norm(y[m].double() - r) / torch.norm(r)).item()
        assert rel <= 1e-5, (m, rel)


@pytest.mark.parametrize("mode", [0, 1])
def test_weight_staging_gives_identical_results(mode):
    a, packed, scales, ref = make_case(1, 4096, 4096, seed=3)
    _staging(0)
    y0 = pk.int4_gemm(a, packed, scales)
    _staging(mode)
    try:
        ys = [pk.int4_gemm(a, packed, scales) for _ in range(3)]
    finally:
        _staging(0)
    for y in ys:
        assert torch.equal(y, y0)
    check_tight(y0, ref)


def test_weight_staging_after_the_weights_are_written():
    # the quantizer (launched without early dependents) writes the weights the
    # very next GEMV reads; with staging on, the GEMV must still see them
    _staging(1)
    try:
        for seed in range(4):
            g = torch.Generator(device="cuda").manual_seed(seed)
            w = (torch.randn(4096, 4096, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
            a = torch.randn(1, 4096, device="cuda", generator=g).to(torch.bfloat16)
            packed, scales = pk.quantize_int4_grouped(w, 128)
            y = pk.int4_gemm(a, packed, scales)
            ref = a.float() @ (pk.unpack_int4_n(packed).float()
                               * scales.float().repeat_interleave(128, 0))
            rel = (torch.norm(y - ref) / torch.norm(ref)).item()
            assert rel <= 1e-5, (seed, rel)
    finally:
        _staging(0)


def test_cluster_gemv_variants():
    a, packed, scales, ref = make_case(1, 4096, 4096, seed=9)
    y = pk.int4_gemm(a, packed, scales)
    assert torch.equal(y, pk.int4_gemm(a, packed, scales))  # deterministic
    yb = pk.int4_gemm(a, packed, scales, out_dtype=torch.bfloat16)
    assert torch.equal(yb, y.to(torch.bfloat16))
    # the reference's per-tensor float scale (gemm_int4.py:58-62)
    codes, s = pk.quantize_int4(torch.randn(4096, 4096, device="cuda", dtype=torch.float16) * 0.02)
    p2 = pk.pack_int4_n(codes)
    a2 = torch.randn(1, 4096, device="cuda", dtype=torch.float16)
    y2 = pk.int4_gemm(a2, p2, s)
    ref2 = a2.float() @ (codes.float() * s)
    assert (torch.norm(y2 - ref2) / torch.norm(ref2)).item() <= 1e-5
    # a strided A row and an output with a leading dimension through the C ABI
    big = torch.randn(3, 4104, device="cuda").to(torch.bfloat16)
    a3 = big[1:2, :4096]
    out = torch.full((2, 4100), float("nan"), device="cuda")
    lib = _lib.load()
    st = lib.pk_w4a16_gemm(a3.data_ptr(), _lib.PK_BF16, 4104, packed.data_ptr(),
                           scales.data_ptr(), 1.0, 128, 1, 4096, 4096, out.data_ptr(), _lib.PK_F32,
                           4100, 0, None, 0, torch.cuda.current_stream().cuda_stream)
    assert st == _lib.PK_OK, _lib.last_error()
    ref3 = pk.int4_gemm(a3.contiguous(), packed, scales)
    assert torch.equal(out[0, :4096], ref3[0])
    assert torch.isnan(out[0, 4096:]).all() and torch.isnan(out[1]).all()


def test_cluster_gemv_sharded_entry_world_one():
    # pk_w4a16_gemm_sharded at world = 1: the exchange epilogue of the cluster
    # form writes exactly this rank's columns, bit-identical to the plain call
    a, packed, scales, _ = make_case(1, 4096, 4096, seed=4)
    lib = _lib.load()
    ref = pk.int4_gemm(a, packed, scales)
    buf = torch.full((1, 8192), float("nan"), device="cuda")
    flag = torch.zeros(2, dtype=torch.int64, device="cuda")
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    outs = (ctypes.c_uint64 * 1)(buf.data_ptr())
    flags = (ctypes.c_uint64 * 1)(flag.data_ptr())
    for _ in range(2):
        st = lib.pk_w4a16_gemm_sharded(
            a.data_ptr(), _lib.PK_BF16, 4096, packed.data_ptr(), scales.data_ptr(), 1.0, 128, 1,
            4096, 4096, _lib.PK_F32, 8192, 2048, 1, 0, ctypes.addressof(outs),
            ctypes.addressof(flags), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream().cuda_stream)
        assert st == _lib.PK_OK, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(buf[0, 2048:6144], ref[0])
        assert torch.isnan(buf[0, :2048]).all() and torch.isnan(buf[0, 6144:]).all()
    assert pk.device_status() == (0, 0)
