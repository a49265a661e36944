"""Pin the CPU oracle to the reference's own outputs (no GPU needed).

Golden vectors come from running pico-kernels' functions
(``tests/golden/make_golden.py``). Every check here is bit-exact.
"""

import hashlib

import numpy as np
import pytest
import torch

from oracle import quant_ref as o


def _f32(arr: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return o.bf16_bits_to_f32(arr)
    return arr.astype(np.float32)


def _group_keys(golden):
    return sorted({k.split("/")[1] for k in golden if k.startswith("group/")})


def test_kat_quantize_col(golden):
    """tests/test_quantize.py:35-42 known answer, reproduced exactly."""
    w = golden["kat_quantize_col/w"]
    assert np.array_equal(o.quantize_col_fake(w, 4, 16), golden["kat_quantize_col/out"])
    assert np.array_equal(o.quantize_col_fake(w, 4), golden["kat_quantize_col_nogroup/out"])
    assert np.array_equal(o.quantize_col_fake(w, 3, 16), golden["kat_quantize_col_3bit/out"])


def test_group_codes_scales_packed(golden):
    names = _group_keys(golden)
    assert len(names) >= 14
    for name in names:
        key = f"group/{name}"
        dt = str(golden[f"{key}/dtype"])
        g = int(golden[f"{key}/group"])
        w = _f32(golden[f"{key}/w"], dt)
        codes, scales = o.group_quant_codes(w, g)
        assert np.array_equal(scales.view(np.uint32), golden[f"{key}/scales_f32"].view(np.uint32)), name
        assert np.array_equal(codes, golden[f"{key}/codes"]), name
        rep = np.repeat(scales, g, axis=0)[: w.shape[0]]
        # by value: the reference's fake-quant keeps -0.0, int8 codes cannot
        assert np.array_equal(codes.astype(np.float32) * rep, golden[f"{key}/fake"]), name
        assert np.array_equal(o.store_scales(scales, "f16").astype(np.float16),
                              golden[f"{key}/scales_f16"]), name
        assert np.array_equal(o.f32_to_bf16_bits(scales), golden[f"{key}/scales_bf16"]), name
        if f"{key}/packed" in golden:
            assert np.array_equal(o.pack_int4_n(codes), golden[f"{key}/packed"]), name


def test_group_fake_quant_matches_column_walk(golden):
    """quantize_col on each column == codes * fp32 scale (quantize.py:63-68)."""
    key = "group/rand_float32_K200_N32_g128"
    w = golden[f"{key}/w"]
    fake = np.stack([o.quantize_col_fake(w[:, n], 4, 128) for n in range(w.shape[1])], 1)
    assert np.array_equal(fake, golden[f"{key}/fake"])


def test_per_tensor_quantize_int4(golden):
    keys = sorted({k.split("/")[1] for k in golden if k.startswith("pt/")})
    assert len(keys) == 4
    for name in keys:
        key = f"pt/{name}"
        dt = "bf16" if name.startswith("bfloat16") else "f16"
        w = _f32(golden[f"{key}/w"], "bfloat16" if dt == "bf16" else "float16")
        q, s = o.quantize_int4_per_tensor(w, dt)
        assert s == float(golden[f"{key}/scale"]), name
        assert np.array_equal(q, golden[f"{key}/codes"]), name
        assert np.array_equal(o.pack_int4_n(q), golden[f"{key}/packed"]), name


def test_pack_roundtrip(golden):
    for case in ("roundtrip", "allnibbles"):
        q = golden[f"pack/{case}/codes"]
        p = o.pack_int4_n(q)
        assert np.array_equal(p, golden[f"pack/{case}/packed"])
        assert np.array_equal(o.unpack_int4_n(p), q)


def test_fp8_quantize_and_gemm(golden):
    for dt, odt in (("float16", "f16"), ("bfloat16", "bf16")):
        key = f"fp8/{dt}"
        a = _f32(golden[f"{key}/a"], dt)
        b = _f32(golden[f"{key}/b"], dt)
        a8, sa = o.fp8_quantize(a, odt)
        b8, sb = o.fp8_quantize(b, odt)
        assert sa == float(golden[f"{key}/sa"]) and sb == float(golden[f"{key}/sb"])
        assert np.array_equal(a8, golden[f"{key}/a8"])
        assert np.array_equal(b8, golden[f"{key}/b8"])
        y = o.fp8_gemm_reference(a8, sa, b8, sb)
        assert np.array_equal(y.view(np.uint32), golden[f"{key}/y"].view(np.uint32))


def config1_inputs():
    g0 = torch.Generator().manual_seed(0)
    w = (torch.randn(1024, 1024, generator=g0) * 0.02).to(torch.float16)
    g1 = torch.Generator().manual_seed(1)
    a = torch.randn(16, 1024, generator=g1).to(torch.float16)
    return w.numpy(), a.numpy()


def test_config1_cpu_reference_run(config1):
    """the whole CPU reference run (packed bytes, scales, Y)."""
    w, a = config1_inputs()
    assert hashlib.sha256(w.tobytes()).hexdigest() == str(config1["w_sha256"])
    assert hashlib.sha256(a.tobytes()).hexdigest() == str(config1["a_sha256"])
    codes, scales = o.group_quant_codes(w.astype(np.float32), 128)
    s16 = scales.astype(np.float16)
    assert np.array_equal(o.pack_int4_n(codes), config1["packed"])
    assert np.array_equal(s16, config1["scales_f16"])
    y = o.w4a16_reference(a.astype(np.float32), codes, s16.astype(np.float32), 128)
    # fp32 matmul summation order differs between numpy BLAS and torch CPU
    ref = config1["y"]
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 1e-6 and np.abs(y - ref).max() < 1e-4


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_e4m3_encoder_matches_torch(seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1 << 16, generator=g) * (10.0 ** (seed - 1))
    x = x[x.abs() < 464]
    ref = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(o.f32_to_e4m3_bits(x.numpy()), ref)


def _gptq_keys(g):
    return sorted({k.rsplit("/", 1)[0] for k in g if k.startswith("gptq/")})


def test_gptq_loop_matches_reference(gptq_golden):
    """quantize.gptq_layer (act_order=False) reproduced bit for bit from the
    reference's own inverse Hessian: quantize.py:99-104."""
    keys = _gptq_keys(gptq_golden)
    assert len(keys) == 3
    for key in keys:
        gs = int(gptq_golden[f"{key}/group"]) or None
        wq = o.gptq_fake_quant_columns(gptq_golden[f"{key}/w"], gptq_golden[f"{key}/h_inv"], 4, gs)
        assert np.array_equal(wq.view(np.uint32), gptq_golden[f"{key}/wq"].view(np.uint32)), key


def test_gptq_hessian_restatement_is_close(gptq_golden):
    """The damped Hessian (quantize.py:88-92) in numpy matches torch's to fp32
    summation order; the GPU producer and the tests use the inverse as given."""
    for key in _gptq_keys(gptq_golden):
        h = o.gptq_inverse_hessian_inputs(gptq_golden[f"{key}/x"], 0.01)
        hi = np.linalg.inv(h.astype(np.float64))
        ref = gptq_golden[f"{key}/h_inv"].astype(np.float64)
        assert np.abs(hi - ref).max() <= 1e-4 * np.abs(ref).max(), key


def test_gptq_packed_form_reduces_to_rtn_without_feedback():
    """With an identity inverse Hessian the packed GPTQ form is the RTN group
    quantizer (group_quant_codes) exactly; with a real one it lowers the
    calibration error below RTN's (the point of quantize.py:1-17)."""
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((24, 64)) * 0.02).astype(np.float32)
    codes, scales = o.gptq_int4_codes(w, np.eye(64, dtype=np.float32), 16)
    c2, s2 = o.group_quant_codes(w.T, 16)
    assert np.array_equal(codes, c2) and np.array_equal(scales, s2)
    x = (rng.standard_normal((512, 64)) * np.linspace(0.2, 3.0, 64)).astype(np.float32)
    x[:, 1:] += 0.7 * x[:, :-1]  # correlated features
    h_inv = np.linalg.inv(o.gptq_inverse_hessian_inputs(x, 0.01).astype(np.float64)).astype(np.float32)
    codes, scales = o.gptq_int4_codes(w, h_inv, 16)
    wq_gptq = (codes.astype(np.float32) * np.repeat(scales, 16, axis=0)).T
    wq_rtn = (c2.astype(np.float32) * np.repeat(s2, 16, axis=0)).T
    err_g = np.linalg.norm(x @ (wq_gptq - w).T)
    err_r = np.linalg.norm(x @ (wq_rtn - w).T)
    assert err_g < 0.9 * err_r, (err_g, err_r)


def test_group_rtn_properties_random_shapes():
    """Size-independent properties of the oracle's per-group RTN on seeded
    random shapes (ragged last groups, several group sizes): codes stay in
    [-7, 7], each group's largest magnitude maps to +-7, every weight lies
    within half a step of its reconstruction, and packing round-trips."""
    rng = np.random.default_rng(11)
    for K, N, g in ((200, 6, 64), (128, 10, 128), (333, 4, 32), (96, 2, 96)):
        w = (rng.standard_normal((K, N)) * rng.uniform(1e-3, 10)).astype(np.float32)
        codes, s = o.group_quant_codes(w, g)
        assert codes.min() >= -7 and codes.max() <= 7
        rows = np.repeat(np.asarray(s, dtype=np.float32), g, axis=0)[:K]
        err = np.abs(w - codes.astype(np.float32) * rows)
        assert np.all(err <= 0.5 * rows * (1 + 1e-5) + 1e-30)
        for gi in range(0, K, g):
            blk = np.abs(codes[gi:gi + g])
            assert np.all(blk.max(axis=0) == 7)
        assert np.array_equal(o.unpack_int4_n(o.pack_int4_n(codes)), codes)


def _cases(z, prefix):
    keys = sorted({k.rsplit("/", 1)[0] for k in z if k.startswith(prefix)})
    assert keys, prefix
    return keys


def test_oracle_quantize_col_all_dtypes_and_widths(qcol_golden):
    """quantize.quantize_col on fp16 / bf16 / fp32 columns at 2, 3, 4 and 8
    bits (quantize.py:42-60), bit for bit, NaN where the reference gives NaN."""
    from conftest import SHORT, golden_values
    z = qcol_golden
    for key in _cases(z, "qcol/"):
        dt = str(z[f"{key}/dtype"])
        w = golden_values(z[f"{key}/w"], dt)
        want = golden_values(z[f"{key}/out"], dt)
        g = int(z[f"{key}/group"])
        got = o.quantize_col_fake(w, int(z[f"{key}/bits"]), g or None, SHORT[dt])
        assert np.array_equal(np.isnan(got), np.isnan(want)), key
        assert np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)]), key


def test_oracle_fp16_zero_group_is_nan(qcol_golden):
    # the reference's 1e-12 floor underflows in fp16: the zero group is NaN
    from conftest import golden_values
    z = qcol_golden
    hits = [k for k in _cases(z, "qcol/") if str(z[f"{k}/name"]) == "edge"
            and str(z[f"{k}/dtype"]) == "float16" and int(z[f"{k}/group"]) == 16]
    assert hits
    for k in hits:
        out = golden_values(z[f"{k}/out"], "float16")
        assert np.isnan(out[:16]).all() and not np.isnan(out[32:]).any()


def test_oracle_rtn_layer(qcol_golden):
    from conftest import SHORT, golden_values
    z = qcol_golden
    for key in _cases(z, "rtn/"):
        dt = str(z[f"{key}/dtype"])
        w = golden_values(z[f"{key}/w"], dt)
        g = int(z[f"{key}/group"])
        got = o.rtn_layer_fake(w, int(z[f"{key}/bits"]), g or None, SHORT[dt])
        assert np.array_equal(got, golden_values(z[f"{key}/out"], dt)), key


def test_oracle_gptq_act_order(gptq_ao_golden):
    """quantize.gptq_layer with its default act_order=True (quantize.py:97-107),
    and a 3-bit case without it, given the reference's inverse Hessian and
    activation energies: bit for bit."""
    z = gptq_ao_golden
    for key in _cases(z, "gptq/"):
        g = int(z[f"{key}/group"])
        ao = int(z[f"{key}/act_order"])
        got = o.gptq_fake_quant_columns(z[f"{key}/w"], z[f"{key}/h_inv"], int(z[f"{key}/bits"]),
                                        g or None, z[f"{key}/act_mag"] if ao else None)
        assert np.array_equal(got, z[f"{key}/wq"]), key
