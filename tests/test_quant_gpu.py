"""GPU parity of the int4 / fp8 quantizers against the golden vectors and the
oracle: bit-exact (packed bytes, codes, scales, e4m3 bytes)."""

import hashlib

import numpy as np
import pytest
import torch

import pico_kernels_b200 as pk
from oracle import quant_ref as o

pytestmark = pytest.mark.gpu

_TORCH = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def _tensor(arr: np.ndarray, dt: str) -> torch.Tensor:
    if dt == "bfloat16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(arr.copy()).cuda()


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _group_names(golden):
    return sorted({k.split("/")[1] for k in golden if k.startswith("group/")})


def test_group_quant_matches_reference_bytes(golden):
    for name in _group_names(golden):
        key = f"group/{name}"
        if f"{key}/packed" not in golden:
            continue
        dt = str(golden[f"{key}/dtype"])
        g = int(golden[f"{key}/group"])
        w = _tensor(golden[f"{key}/w"], dt)
        for sdt, ref in ((torch.float32, golden[f"{key}/scales_f32"]),
                         (torch.float16, golden[f"{key}/scales_f16"]),
                         (torch.bfloat16, golden[f"{key}/scales_bf16"])):
            packed, scales = pk.quantize_int4_grouped(w, g, scale_dtype=sdt)
            assert np.array_equal(packed.cpu().numpy(), golden[f"{key}/packed"]), (name, sdt)
            got = _u16(scales) if sdt == torch.bfloat16 else scales.cpu().numpy()
            assert np.array_equal(got.view(np.uint8), ref.view(np.uint8)), (name, sdt)


def test_group_quant_strided_and_generic_paths(golden):
    """A column slice (ld > N) takes the generic kernel; results stay exact."""
    key = "group/rand_float16_K256_N64_g128"
    w = _tensor(golden[f"{key}/w"], "float16")
    wide = torch.zeros(256, 96, dtype=torch.float16, device="cuda")
    wide[:, 16:80] = w
    packed, scales = pk.quantize_int4_grouped(wide[:, 16:80], 128)
    assert np.array_equal(packed.cpu().numpy(), golden[f"{key}/packed"])
    assert np.array_equal(scales.cpu().numpy(), golden[f"{key}/scales_f16"])


def test_per_tensor_quantize_int4(golden):
    for name in sorted({k.split("/")[1] for k in golden if k.startswith("pt/")}):
        key = f"pt/{name}"
        dt = "bfloat16" if name.startswith("bfloat16") else "float16"
        w = _tensor(golden[f"{key}/w"], dt)
        q, s = pk.quantize_int4(w)
        assert s == float(golden[f"{key}/scale"]), name
        assert np.array_equal(q.cpu().numpy(), golden[f"{key}/codes"]), name
        assert np.array_equal(pk.pack_int4_n(q).cpu().numpy(), golden[f"{key}/packed"]), name


def test_pack_unpack(golden):
    for case in ("roundtrip", "allnibbles"):
        q = torch.from_numpy(golden[f"pack/{case}/codes"].copy()).cuda()
        p = pk.pack_int4_n(q)
        assert np.array_equal(p.cpu().numpy(), golden[f"pack/{case}/packed"])
        assert torch.equal(pk.unpack_int4_n(p), q)
    # odd byte count takes the scalar path
    q = torch.randint(-8, 8, (3, 10), dtype=torch.int8, device="cuda")
    assert np.array_equal(pk.pack_int4_n(q).cpu().numpy(), o.pack_int4_n(q.cpu().numpy()))
    with pytest.raises(ValueError):
        pk.pack_int4_n(torch.zeros(4, 3, dtype=torch.int8, device="cuda"))


def test_fp8_quantize(golden):
    for dt in ("float16", "bfloat16"):
        key = f"fp8/{dt}"
        for src, dst, sc in (("a", "a8", "sa"), ("b", "b8", "sb")):
            x = _tensor(golden[f"{key}/{src}"], dt)
            x8, s = pk.gemm_fp8.quantize(x)
            assert x8.dtype == torch.float8_e4m3fn
            assert s == float(golden[f"{key}/{sc}"])
            assert np.array_equal(x8.view(torch.uint8).cpu().numpy(), golden[f"{key}/{dst}"])


def test_fp8_quantize_roundtrip():
    """tests/test_gemm_fp8.py:38-44: cast round-trip rel err < 0.05."""
    torch.manual_seed(1)
    x = torch.randn(256, 256, device="cuda", dtype=torch.float16)
    x8, scale = pk.gemm_fp8.quantize(x)
    back = x8.to(torch.float32) / scale
    rel = torch.norm(back - x.float()) / torch.norm(x.float())
    assert rel.item() < 0.05


@pytest.mark.parametrize("shape,dt", [((4096, 4096), torch.bfloat16),
                                      ((4096, 11008), torch.bfloat16),
                                      ((1024, 1024), torch.float16)])
def test_group_quant_full_size_vs_oracle(shape, dt):
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(*shape, generator=g) * 0.02).to(dt)
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    codes, s32 = o.group_quant_codes(w.float().numpy(), 128)
    assert np.array_equal(packed.cpu().numpy(), o.pack_int4_n(codes))
    ref_s = (o.f32_to_bf16_bits(s32) if dt == torch.bfloat16
             else s32.astype(np.float16).view(np.uint16))
    assert np.array_equal(_u16(scales), ref_s)


def test_config1_quantize_and_gemm(config1):
    """packed bytes and fp16 scales exact; Y within tolerance."""
    g0 = torch.Generator().manual_seed(0)
    w = (torch.randn(1024, 1024, generator=g0) * 0.02).to(torch.float16)
    g1 = torch.Generator().manual_seed(1)
    a = torch.randn(16, 1024, generator=g1).to(torch.float16)
    assert hashlib.sha256(w.numpy().tobytes()).hexdigest() == str(config1["w_sha256"])
    packed, scales = pk.quantize_int4_grouped(w.cuda(), 128)
    assert np.array_equal(packed.cpu().numpy(), config1["packed"])
    assert np.array_equal(scales.cpu().numpy(), config1["scales_f16"])
    y = pk.int4_gemm(a.cuda(), packed, scales).cpu().numpy()
    ref = config1["y"]
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    # fp16 dequant (unit roundoff 2^-11) before an fp32-accumulated MMA
    assert rel < 1e-3, rel
    assert np.abs(y - ref).max() < 1e-2 * np.abs(ref).max()
