"""GPU parity of the W4A16 GEMV (CUDA cores; M = 1, and M = 2 on layers of 16 MB
or more) against the oracle.

The GEMV multiplies exact integer codes by the activations in fp32 and applies
each fp32 group scale to the fp32 group sum, so it differs from the oracle's
fp32 dequantize-then-matmul (tests/test_gemm_int4.py:26 with group scales)
only in summation order: relative Frobenius error ~1e-7. Bounds:
rel-Frobenius <= 1e-5 and max-abs <= 1e-4 * max|Y| -- tighter than any path
that rounds q*s to 16 bits, so a pass also shows the GEMV ran.
"""

import numpy as np
import pytest
import torch

import pico_kernels_b200 as pk
from oracle import quant_ref as o

pytestmark = pytest.mark.gpu


def make_case(M, N, K, dt=torch.bfloat16, group=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(K, N, generator=g) * 0.02).to(dt)
    g1 = torch.Generator().manual_seed(seed + 1)
    a = torch.randn(M, K, generator=g1).to(dt)
    codes, s32 = o.group_quant_codes(w.float().numpy(), group)
    s_stored = o.store_scales(s32, "bf16" if dt == torch.bfloat16 else "f16")
    ref = o.w4a16_reference(a.float().numpy(), codes, s_stored, group)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), group)
    return a.cuda(), packed, scales, ref


def check_tight(y, ref, what=""):
    y = y.float().cpu().numpy()
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    mx = np.abs(y - ref).max()
    assert rel <= 1e-5, (what, rel)
    assert mx <= 1e-4 * np.abs(ref).max(), (what, mx)


@pytest.mark.parametrize("M,N", [(1, 4096), (2, 8192)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemv_decode(M, N, dt):
    a, packed, scales, ref = make_case(M, N, 4096, dt, seed=M)
    y = pk.int4_gemm(a, packed, scales)
    assert y.shape == (M, N) and y.dtype == torch.float32
    check_tight(y, ref, f"M={M} {dt}")
    assert pk.device_status() == (0, 0)


@pytest.mark.parametrize("M,N,K,group", [
    (1, 4128, 4096, 128),    # last 128-column slice ragged (32 columns)
    (1, 1024, 4160, 64),     # K not a multiple of 128, group 64 (eight scale rows per unit)
    (2, 8192, 4160, 64),     # M = 2
    (1, 2048, 4100, 128),    # K not a multiple of the 512-row unit
    (1, 512, 8192, 256),     # group 256
    (1, 1024, 4224, 192),    # groups straddle the 512-row units
    (1, 256, 163840, 64),    # stream-K: one slice split over every CTA (fan-in 148; group 64 keeps it off the decode kernel)
    (2, 65536, 512, 128),    # stream-K, M = 2: CTA ranges span several slices
    (1, 8192, 256, 64),      # one partial unit per slice: every segment a whole slice
    (3, 4128, 4096, 128),    # M = 3..8: the n8 block of the tiles
    (4, 28672, 2048, 128),
    (5, 1024, 4224, 192),
    (6, 2048, 4100, 128),
    (7, 65536, 512, 128),
    (8, 8192, 4160, 64),
    (8, 256, 163840, 64),
])
def test_gemv_shapes(M, N, K, group):
    a, packed, scales, ref = make_case(M, N, K, group=group, seed=N + K)
    y = pk.int4_gemm(a, packed, scales, group_size=group)
    check_tight(y, ref, f"M={M} N={N} K={K} g={group}")


def test_gemv_llama70b_shapes():
    for (M, N, K) in ((1, 28672, 8192), (1, 8192, 28672), (8, 28672, 8192)):
        a, packed, scales, ref = make_case(M, N, K, seed=7)
        check_tight(pk.int4_gemm(a, packed, scales), ref, f"M={M} N={N} K={K}")


def test_gemv_deterministic_and_bf16_out():
    a, packed, scales, ref = make_case(1, 4096, 4096, seed=21)
    y1 = pk.int4_gemm(a, packed, scales)
    y2 = pk.int4_gemm(a, packed, scales)
    assert torch.equal(y1, y2)
    yb = pk.int4_gemm(a, packed, scales, out_dtype=torch.bfloat16)
    assert yb.dtype == torch.bfloat16
    assert torch.equal(yb, y1.to(torch.bfloat16))


def test_gemv_per_tensor_scale():
    """tests/test_gemm_int4.py:19-30 form (per-tensor float scale) at M=1."""
    torch.manual_seed(0)
    a = torch.randn(1, 2048, device="cuda", dtype=torch.float16)
    w = torch.randn(2048, 1024, device="cuda", dtype=torch.float16)
    w_q, scale = pk.quantize_int4(w)
    c = pk.int4_gemm(a, pk.pack_int4_n(w_q), scale)
    ref = a.float() @ (w_q.float() * scale)
    assert (torch.norm(c - ref) / torch.norm(ref)).item() < 1e-5


def test_gemv_agrees_with_tensor_core_decode():
    """An explicit split_k selects the tcgen05 decode kernel (q*s rounded to
    bf16 before the MMA); both must agree within that kernel's tolerance."""
    a, packed, scales, ref = make_case(1, 4096, 4096, seed=33)
    y_gemv = pk.int4_gemm(a, packed, scales)
    y_tc = pk.int4_gemm(a, packed, scales, split_k=4)
    rel = (torch.norm(y_gemv - y_tc) / torch.norm(y_gemv)).item()
    assert 0 < rel < 5e-3


def test_gemv_output_strides_and_stream():
    """Through the C-ABI with ldo > N on a side stream."""
    from pico_kernels_b200 import _lib as L
    lib = L.load()
    M, N, K = 1, 1024, 2048
    a, packed, scales, ref = make_case(M, N, K, seed=41)
    ldo = N + 64
    out = torch.full((M, ldo), 7.0, device="cuda")
    s = torch.cuda.Stream()
    ws_bytes = lib.pk_w4a16_workspace_size(M, N, K, 0)
    ws = L.workspace(a.device, ws_bytes, tag="gemv-test")
    with torch.cuda.stream(s):
        rc = lib.pk_w4a16_gemm(L.ptr(a), L.dtype_code(a.dtype), K, L.ptr(packed), L.ptr(scales),
                               1.0, 128, M, N, K, L.ptr(out), L.dtype_code(torch.float32), ldo, 0,
                               L.ptr(ws), ws_bytes, s.cuda_stream)
    s.synchronize()
    assert rc == 0, lib.pk_last_error_string()
    check_tight(out[:, :N], ref)
    assert torch.all(out[:, N:] == 7.0)


def test_workspace_shared_across_kernels():
    """One cached workspace serves the tensor-core decode (split 32, partials in
    the workspace), the GEMV and the dense split-K GEMM in turn: partials of
    one call never land on another call's arrival counters."""
    a1, p1, s1, ref1 = make_case(4, 4096, 4096, seed=51)
    a2, p2, s2, ref2 = make_case(1, 28672, 2048, seed=52)  # stream-K with a workspace
    from pico_kernels_b200 import _lib as L
    assert L.load().pk_w4a16_workspace_size(1, 28672, 2048, 0) > 0
    for _ in range(2):
        y1 = pk.int4_gemm(a1, p1, s1, split_k=32)
        y2 = pk.int4_gemm(a2, p2, s2)
        check_tight(y2, ref2, "GEMV after split-32 decode")
        rel = np.linalg.norm(y1.cpu().numpy() - ref1) / np.linalg.norm(ref1)
        assert rel < 5e-3
        x = torch.randn(64, 512, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(512, 2048, device="cuda", dtype=torch.bfloat16)
        c = pk.triton_gemm_splitk(x, b, split_k=4)
        assert torch.allclose(c, x.float() @ b.float(), atol=1e-2, rtol=1e-3)
        # large-M W4A16: its dequantized weights go after the counter region
        a3, p3, s3, ref3 = make_case(1024, 512, 1024, seed=53)
        y3 = pk.int4_gemm(a3, p3, s3)
        rel3 = np.linalg.norm(y3.cpu().numpy() - ref3) / np.linalg.norm(ref3)
        assert rel3 < 5e-3
    assert pk.device_status() == (0, 0)


def test_out_parameter_reuses_the_buffer():
    """int4_gemm(out=...) writes into the given buffer (no allocation) and
    rejects one of the wrong shape, dtype or layout."""
    a, packed, scales, ref = make_case(1, 4096, 4096, seed=61)
    buf = torch.full((1, 4096), 3.0, device="cuda")
    y = pk.int4_gemm(a, packed, scales, out=buf)
    assert y is buf
    assert torch.equal(buf, pk.int4_gemm(a, packed, scales))
    check_tight(buf, ref)
    for bad in (torch.empty(2, 4096, device="cuda"),
                torch.empty(1, 4096, device="cuda", dtype=torch.bfloat16),
                torch.empty(4096, 2, device="cuda").t()):
        with pytest.raises(AssertionError):
            pk.int4_gemm(a, packed, scales, out=bad)
