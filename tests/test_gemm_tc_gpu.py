"""GPU parity of the persistent tcgen05 GEMM: fp8 (gemm_fp8.py), dense split-K
(gemm_splitk.py) and W4A16 prefill (gemm_int4.py at large M).

Tolerances:
* fp8 vs the oracle's exact dequantized product (fp64 sum of the e4m3
  values, times out_scale): only fp32 accumulation order differs ->
  rel-Frobenius <= 1e-5;
* fp8 vs the fp32 product of the unquantized inputs: rel < 0.10
  (tests/test_gemm_fp8.py:19-28);
* dense split-K vs fp32: allclose(atol=1e-2, rtol=1e-2)
  (tests/test_gemm_splitk.py:19-38), bitwise reproducible run to run;
* W4A16 prefill dequantizes q*s to bf16 before the MMA (unit roundoff
  2^-8): rel-Frobenius <= 5e-3, max-abs <= 2e-2 * max|Y|.
"""

import numpy as np
import pytest
import torch

import pico_kernels_b200 as pk
from oracle import quant_ref as o
from pico_kernels_b200 import gemm_fp8, gemm_splitk

pytestmark = pytest.mark.gpu


def _rel(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.linalg.norm(y - ref) / np.linalg.norm(ref)


# ----------------------------------------------------------------------- fp8
def test_fp8_matches_reference_golden(golden):
    for dt in ("float16", "bfloat16"):
        key = f"fp8/{dt}"
        a8 = torch.from_numpy(golden[f"{key}/a8"].copy()).cuda().view(torch.float8_e4m3fn)
        b8 = torch.from_numpy(golden[f"{key}/b8"].copy()).cuda().view(torch.float8_e4m3fn)
        y = gemm_fp8.fp8_gemm_precast(a8, float(golden[f"{key}/sa"]), b8, float(golden[f"{key}/sb"]))
        assert y.dtype == torch.float32
        assert _rel(y.cpu().numpy(), golden[f"{key}/y"]) < 1e-5


@pytest.mark.parametrize("S", [512, 1024, 2048])
def test_fp8_vs_oracle(S):
    g = torch.Generator().manual_seed(S)
    a = torch.randn(S, S, generator=g).to(torch.bfloat16)
    b = torch.randn(S, S, generator=g).to(torch.bfloat16)
    a8, sa = gemm_fp8.quantize(a.cuda())
    b8, sb = gemm_fp8.quantize(b.cuda())
    y = gemm_fp8.fp8_gemm_precast(a8, sa, b8, sb).cpu().numpy()
    a8b = a8.view(torch.uint8).cpu().numpy()
    b8b = b8.view(torch.uint8).cpu().numpy()
    ref = o.fp8_gemm_reference(a8b, sa, b8b, sb)
    assert _rel(y, ref) < 1e-5
    ref32 = a.float().numpy() @ b.float().numpy()
    assert _rel(y, ref32) < 0.10


def test_fp8_reference_tests():
    """tests/test_gemm_fp8.py:19-35 on this implementation."""
    torch.manual_seed(0)
    a = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    b = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    c = gemm_fp8.fp8_gemm(a, b)
    ref = a.float() @ b.float()
    assert (torch.norm(c - ref) / torch.norm(ref)).item() < 0.10
    assert c.dtype == torch.float32
    cb = gemm_fp8.fp8_gemm(a, b, out_dtype=torch.bfloat16)
    assert cb.dtype == torch.bfloat16
    assert (cb.float() - c).abs().max().item() <= 1e-2 * c.abs().max().item()


@pytest.mark.parametrize("M,N,K", [(300, 512, 256), (128, 272, 96), (1, 256, 512), (777, 1040, 1104)])
def test_fp8_ragged(M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    a8, sa = gemm_fp8.quantize(a.cuda())
    b8, sb = gemm_fp8.quantize(b.cuda())
    y = gemm_fp8.fp8_gemm_precast(a8, sa, b8, sb).cpu().numpy()
    ref = o.fp8_gemm_reference(a8.view(torch.uint8).cpu().numpy(), sa,
                               b8.view(torch.uint8).cpu().numpy(), sb)
    assert _rel(y, ref) < 1e-5


# ------------------------------------------------------------- dense split-K
def test_splitk_matches_fp32():
    """tests/test_gemm_splitk.py:19-27."""
    torch.manual_seed(0)
    a = torch.randn(512, 1024, device="cuda", dtype=torch.float16)
    b = torch.randn(1024, 512, device="cuda", dtype=torch.float16)
    c = gemm_splitk.triton_gemm_splitk(a, b, split_k=4)
    ref = a.float() @ b.float()
    assert torch.allclose(c, ref, atol=1e-2, rtol=1e-2)


def test_splitk_matches_non_split():
    """tests/test_gemm_splitk.py:30-38."""
    torch.manual_seed(1)
    a = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    b = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    c_split = gemm_splitk.triton_gemm_splitk(a, b, split_k=4)
    c_plain = gemm_splitk.triton_gemm(a, b)
    assert torch.allclose(c_split, c_plain, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("split", [1, 2, 3, 8])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_splitk_deterministic_and_correct(split, dt):
    g = torch.Generator().manual_seed(split)
    a = torch.randn(384, 2048, generator=g).to(dt).cuda()
    b = torch.randn(2048, 640, generator=g).to(dt).cuda()
    c1 = gemm_splitk.triton_gemm_splitk(a, b, split_k=split)
    c2 = gemm_splitk.triton_gemm_splitk(a, b, split_k=split)
    assert torch.equal(c1, c2)
    ref = a.float() @ b.float()
    assert torch.allclose(c1, ref, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("shape", [(256, 256, 256), (1024, 1024, 1024), (200, 136, 72)])
def test_dense_gemm_matches_torch(shape):
    """tests/test_gemm.py:20-34 (the non-split partner)."""
    m, n, k = shape
    for dt in (torch.float16, torch.bfloat16):
        torch.manual_seed(0)
        a = torch.randn(m, k, device="cuda", dtype=dt)
        b = torch.randn(k, n, device="cuda", dtype=dt)
        c = gemm_splitk.triton_gemm(a, b)
        assert c.dtype == torch.float32
        assert torch.allclose(c, a.float() @ b.float(), atol=1e-2, rtol=1e-2)


# ---------------------------------------------------------- CTA-pair tiles
@pytest.mark.parametrize("M,N,K", [
    (4096, 4096, 4096),   # 256 pair tiles over the resident pairs: 3.5 waves
    (3000, 2000, 1040),   # ragged M and N edges inside pair tiles (96 tiles)
    (2048, 2048, 2048),   # one wave of pair tiles: one-CTA tiles instead
])
def test_fp8_pair_tiles(M, N, K):
    """fp8 on 256 x 256 CTA-pair tiles (cta_group::2) matches the exact
    product (e4m3 products are exact in fp32: only summation order differs)
    and is bitwise reproducible."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a8, sa = gemm_fp8.quantize(torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16))
    b8, sb = gemm_fp8.quantize(torch.randn(K, N, device="cuda", generator=g).to(torch.bfloat16))
    y = gemm_fp8.fp8_gemm_precast(a8, sa, b8, sb)
    assert torch.equal(y, gemm_fp8.fp8_gemm_precast(a8, sa, b8, sb))
    ref = (a8.float() @ b8.float()) / (sa * sb)
    assert (torch.norm(y - ref) / torch.norm(ref)).item() < 1e-5
    yb = gemm_fp8.fp8_gemm_precast(a8, sa, b8, sb, out_dtype=torch.bfloat16)
    assert torch.equal(yb, y.to(torch.bfloat16))
    assert pk.device_status() == (0, 0)


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096), (3000, 2000, 1000), (200, 4104, 264)])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_dense_pair_tiles(M, N, K, dt):
    """Dense 16-bit GEMM on CTA-pair tiles (and, for the last shape, one wave
    of one-CTA tiles) against the fp32 product: bf16/fp16 products are exact
    in fp32, so only summation order differs."""
    torch.manual_seed(M + K)
    a = torch.randn(M, K, device="cuda", dtype=dt)
    b = torch.randn(K, N, device="cuda", dtype=dt)
    c = gemm_splitk.triton_gemm(a, b)
    ref = a.float() @ b.float()
    assert (torch.norm(c - ref) / torch.norm(ref)).item() < 1e-5
    assert torch.equal(c, gemm_splitk.triton_gemm(a, b))


# ------------------------------------------------------------ W4A16 prefill
def _w4a16_case(M, N, K, seed=0, dt=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(K, N, generator=g) * 0.02).to(dt)
    a = torch.randn(M, K, generator=g).to(dt)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    return a.cuda(), packed, scales


def _dequant_torch(packed, scales, group=128):
    q = pk.unpack_int4_n(packed).float()
    return q * scales.float().repeat_interleave(group, dim=0)[: q.shape[0]]


@pytest.mark.parametrize("M,N,K", [(17, 256, 512), (128, 512, 1024), (300, 1024, 2048),
                                   (256, 11008, 4096)])
def test_w4a16_prefill_vs_oracle(M, N, K):
    a, packed, scales = _w4a16_case(M, N, K, seed=M)
    y = pk.int4_gemm(a, packed, scales).cpu().numpy()
    codes = pk.unpack_int4_n(packed).cpu().numpy()
    ref = o.w4a16_reference(a.float().cpu().numpy(), codes, scales.float().cpu().numpy(), 128)
    assert _rel(y, ref) <= 5e-3
    assert np.abs(y - ref).max() <= 2e-2 * np.abs(ref).max()


def test_w4a16_prefill_full_size_vs_torch_fp32():
    """M=4096, K=4096, N=11008 against a torch fp32 GPU reference."""
    a, packed, scales = _w4a16_case(4096, 11008, 4096, seed=42)
    y = pk.int4_gemm(a, packed, scales)
    ref = a.float() @ _dequant_torch(packed, scales)
    rel = (torch.norm(y - ref) / torch.norm(ref)).item()
    assert rel <= 5e-3
    assert (y - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()


def test_w4a16_prefill_per_tensor_reference_api():
    """tests/test_gemm_int4.py:19-30 exactly: M=128, fp16, per-tensor float scale."""
    torch.manual_seed(0)
    a = torch.randn(128, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(256, 512, device="cuda", dtype=torch.float16)
    w_q, scale = pk.quantize_int4(w)
    c = pk.int4_gemm(a, pk.pack_int4_n(w_q), scale)
    ref = a.float() @ (w_q.float() * scale)
    assert torch.allclose(c, ref, atol=1e-1, rtol=1e-2)
    assert (torch.norm(c - ref) / torch.norm(ref)).item() < 1e-5


def test_w4a16_prefill_fp16_and_bf16_out():
    a, packed, scales = _w4a16_case(64, 512, 1024, seed=3, dt=torch.float16)
    y = pk.int4_gemm(a, packed, scales, out_dtype=torch.bfloat16)
    ref = a.float() @ _dequant_torch(packed, scales)
    assert y.dtype == torch.bfloat16
    assert (torch.norm(y.float() - ref) / torch.norm(ref)).item() <= 5e-3
    assert pk.device_status() == (0, 0)
