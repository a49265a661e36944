"""GPU parity of the W4A16 GEMM against the oracle's dequantize-then-matmul in
fp32 (the reference's own formula, tests/test_gemm_int4.py:26).

Tolerances: the kernel rounds each dequantized weight q*s to the activation
dtype before the MMA (unit roundoff 2^-8 for bf16, 2^-11 for fp16), then
accumulates in fp32. For N(0,1) activations and N(0,0.02) weights that gives
a relative Frobenius error near 2.3e-3 (bf16) / 3e-4 (fp16). Bounds:
rel-Frobenius <= 5e-3 (bf16) / 1e-3 (fp16), max-abs <= 2e-2 * max|Y|.
"""

import numpy as np
import pytest
import torch

import pico_kernels_b200 as pk
from oracle import quant_ref as o

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 5e-3, torch.float16: 1e-3}


def make_case(M, N, K, dt, group=128, seed=0, wstd=0.02):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(K, N, generator=g) * wstd).to(dt)
    g1 = torch.Generator().manual_seed(seed + 1)
    a = torch.randn(M, K, generator=g1).to(dt)
    codes, s32 = o.group_quant_codes(w.float().numpy(), group)
    s_stored = o.store_scales(s32, "bf16" if dt == torch.bfloat16 else "f16")
    ref = o.w4a16_reference(a.float().numpy(), codes, s_stored, group)
    return a, w, ref


def check(y: torch.Tensor, ref: np.ndarray, dt, what=""):
    y = y.float().cpu().numpy()
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    mx = np.abs(y - ref).max()
    assert rel <= TOL[dt], (what, rel)
    assert mx <= 2e-2 * np.abs(ref).max(), (what, mx)
    return rel


@pytest.mark.parametrize("M", [1, 4, 16, 17, 24, 32])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_decode_4096(M, dt):
    a, w, ref = make_case(M, 4096, 4096, dt)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    y = pk.int4_gemm(a.cuda(), packed, scales)
    assert y.dtype == torch.float32 and y.shape == (M, 4096)
    check(y, ref, dt, f"M={M}")
    assert pk.device_status() == (0, 0)


@pytest.mark.parametrize("split", [1, 2, 3, 8, 32])
@pytest.mark.parametrize("M", [4, 32])
def test_decode_split_k_deterministic(split, M):
    a, w, ref = make_case(M, 4096, 4096, torch.bfloat16, seed=3)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    a = a.cuda()
    y1 = pk.int4_gemm(a, packed, scales, split_k=split)
    y2 = pk.int4_gemm(a, packed, scales, split_k=split)
    assert torch.equal(y1, y2), "split-K reduction must be bitwise reproducible"
    check(y1, ref, torch.bfloat16, f"split={split}")


def test_decode_splits_agree():
    a, w, _ = make_case(16, 2048, 4096, torch.bfloat16, seed=5)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    a = a.cuda()
    y1 = pk.int4_gemm(a, packed, scales, split_k=1)
    for s in (2, 4, 16):
        ys = pk.int4_gemm(a, packed, scales, split_k=s)
        assert (ys - y1).abs().max().item() <= 1e-4 * y1.abs().max().item()


def test_decode_llama70b_shapes():
    for (N, K) in ((28672, 8192), (8192, 28672)):
        a, w, ref = make_case(32, N, K, torch.bfloat16, seed=7)
        packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
        y = pk.int4_gemm(a.cuda(), packed, scales)             # M = 32: decode kernel
        rel = check(y, ref, torch.bfloat16, f"N={N} K={K}")
        assert rel < 1e-5, rel  # exact codes, fp32 scale after the MMA
        y4 = pk.int4_gemm(a[:4].cuda(), packed, scales)        # M = 4
        check(y4, ref[:4], torch.bfloat16, f"M=4 N={N} K={K}")


def test_decode_bf16_output():
    a, w, ref = make_case(2, 1024, 2048, torch.bfloat16, seed=9)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    y = pk.int4_gemm(a.cuda(), packed, scales, out_dtype=torch.bfloat16)
    assert y.dtype == torch.bfloat16
    check(y, ref, torch.bfloat16)


def test_per_tensor_scale_reference_api():
    """tests/test_gemm_int4.py:19-30 at a decode shape: per-tensor float scale."""
    torch.manual_seed(0)
    a = torch.randn(16, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(256, 512, device="cuda", dtype=torch.float16)
    w_q, scale = pk.quantize_int4(w)
    c = pk.int4_gemm(a, pk.pack_int4_n(w_q), scale)
    ref = a.float() @ (w_q.float() * scale)
    assert torch.allclose(c, ref, atol=1e-1, rtol=1e-2)
    # codes are exact in fp16, so only fp32 summation order differs
    assert (torch.norm(c - ref) / torch.norm(ref)).item() < 1e-5


@pytest.mark.parametrize("M,N,K,group", [(3, 130, 200, 64), (1, 2, 7, 4), (40, 70, 128, 32)])
def test_ragged_shapes_generic_kernel(M, N, K, group):
    """Shapes no tensor-core path takes run on the CUDA-core kernel, which
    dequantizes in fp32: only summation order differs from the oracle."""
    a, w, ref = make_case(M, N, K, torch.bfloat16, group=group, seed=11)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), group)
    y = pk.int4_gemm(a.cuda(), packed, scales, group_size=group)
    yy = y.cpu().numpy()
    assert np.abs(yy - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("M,N,K", [(40, 256, 384), (33, 96, 192), (20, 192, 320)])
def test_small_m_prefill_path(M, N, K):
    """M > 32, or N / K not multiples of 128, with K % 64 == 0 takes the
    tensor-core prefill kernel (bf16 q*s)."""
    a, w, ref = make_case(M, N, K, torch.bfloat16, seed=12)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    check(pk.int4_gemm(a.cuda(), packed, scales), ref, torch.bfloat16, f"M={M}")


def test_errors_are_reference_compatible():
    a = torch.randn(4, 256, device="cuda", dtype=torch.bfloat16)
    wp = torch.zeros(128, 64, dtype=torch.uint8, device="cuda")
    with pytest.raises(AssertionError):
        pk.int4_gemm(a, wp, 1.0)
    with pytest.raises(TypeError):
        pk.int4_gemm(a.float(), torch.zeros(256, 64, dtype=torch.uint8, device="cuda"), 1.0)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_prefill_dequant_once_matches_fused(dt):
    """M >= 1024 with a workspace: the weights are dequantized once into the
    workspace (q*s rounded to A's dtype, the fused kernel's operand) and the
    dense tcgen05 GEMM runs; without a workspace the fused kernel runs. Same
    operand values and tile order, so the two agree to fp32 summation order."""
    from pico_kernels_b200 import _lib as L
    lib = L.load()
    M, N, K = 1024, 1024, 2048
    a, w, ref = make_case(M, N, K, dt, seed=13)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    a = a.cuda()
    assert lib.pk_w4a16_workspace_size(M, N, K, 0) >= K * N * 2
    y_once = pk.int4_gemm(a, packed, scales)                      # workspace given
    check(y_once, ref, dt, "dequant once")
    y_fused = torch.empty(M, N, device="cuda")
    rc = lib.pk_w4a16_gemm(L.ptr(a), L.dtype_code(dt), K, L.ptr(packed), L.ptr(scales), 1.0, 128,
                           M, N, K, L.ptr(y_fused), L.dtype_code(torch.float32), N, 0, None, 0,
                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.last_error()
    rel = (torch.norm(y_once - y_fused) / torch.norm(y_fused)).item()
    assert rel < 1e-6, rel


def test_prefill_dequant_once_per_tensor_scale():
    torch.manual_seed(1)
    a = torch.randn(1024, 512, device="cuda", dtype=torch.float16)
    w = torch.randn(512, 256, device="cuda", dtype=torch.float16)
    w_q, scale = pk.quantize_int4(w)
    c = pk.int4_gemm(a, pk.pack_int4_n(w_q), scale)
    ref = a.float() @ (w_q.float() * scale)
    assert (torch.norm(c - ref) / torch.norm(ref)).item() < 1e-5


@pytest.mark.parametrize("M,N,K", [(33, 1024, 2048), (64, 1024, 2048), (100, 1024, 2048),
                                   (128, 1024, 2048), (129, 20480, 512), (200, 20480, 512),
                                   (256, 20480, 512)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_skinny_prefill_vs_oracle(M, N, K, dt):
    """32 < M <= 256 on shapes where the swap-AB kernel is chosen (each weight
    dequantized once, q*s rounded to A's dtype as in the prefill kernel):
    activation widths 64, 128 and 256."""
    a, w, ref = make_case(M, N, K, dt, seed=M)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    y = pk.int4_gemm(a.cuda(), packed, scales)
    assert y.shape == (M, N)
    check(y, ref, dt, f"M={M}")
    # same operand values as the fused prefill kernel (split_k=1 skips this
    # path): the two agree to fp32 summation order
    y_pf = pk.int4_gemm(a.cuda(), packed, scales, split_k=1)
    assert (torch.norm(y - y_pf) / torch.norm(y_pf)).item() < 1e-5
    assert pk.device_status() == (0, 0)


def test_skinny_prefill_variants():
    """group 64, per-tensor scale, bf16 output, ldo > N through the C-ABI."""
    a, w, ref = make_case(72, 512, 1024, torch.bfloat16, group=64, seed=77)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 64)
    check(pk.int4_gemm(a.cuda(), packed, scales, group_size=64), ref, torch.bfloat16, "g64")
    yb = pk.int4_gemm(a.cuda(), packed, scales, group_size=64, out_dtype=torch.bfloat16)
    assert yb.dtype == torch.bfloat16
    assert torch.equal(yb, pk.int4_gemm(a.cuda(), packed, scales, group_size=64).to(torch.bfloat16))
    torch.manual_seed(2)
    a2 = torch.randn(96, 512, device="cuda", dtype=torch.float16)
    w2 = torch.randn(512, 256, device="cuda", dtype=torch.float16)
    w_q, scale = pk.quantize_int4(w2)
    c = pk.int4_gemm(a2, pk.pack_int4_n(w_q), scale)
    ref2 = a2.float() @ (w_q.float() * scale)
    assert (torch.norm(c - ref2) / torch.norm(ref2)).item() < 1e-5
    from pico_kernels_b200 import _lib as L
    lib = L.load()
    a3, w3, ref3 = make_case(48, 256, 512, torch.bfloat16, seed=78)
    p3, s3 = pk.quantize_int4_grouped(w3.cuda(), 128)
    a3 = a3.cuda()
    out = torch.full((48, 320), 5.0, device="cuda")
    rc = lib.pk_w4a16_gemm(L.ptr(a3), L.PK_BF16, 512, L.ptr(p3), L.ptr(s3), 1.0, 128, 48, 256, 512,
                           L.ptr(out), L.PK_F32, 320, 0, None, 0,
                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.last_error()
    check(out[:, :256], ref3, torch.bfloat16, "ldo")
    assert torch.all(out[:, 256:] == 5.0)


def test_skinny_prefill_llama70b_m256():
    a, w, ref = make_case(256, 28672, 8192, torch.bfloat16, seed=79)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    check(pk.int4_gemm(a.cuda(), packed, scales), ref, torch.bfloat16, "70B up M=256")
