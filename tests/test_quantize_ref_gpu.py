"""GPU parity of the reference-rule quantizers against the reference's own
outputs (golden vectors made by importing pico-kernels' quantize module).

* ``quantize.quantize_col`` (quantize.py:42-60) on fp16 / bf16 / fp32 columns
  at 2, 3, 4 and 8 bits, with and without groups: bit-exact, NaN where the
  reference gives NaN (fp16 groups of zeros, whose 1e-12 floor underflows);
* ``quantize.rtn_layer`` (quantize.py:63-68): bit-exact;
* ``gptq.gptq_layer`` (quantize.py:71-115), the reference's GPTQ walk on the
  GPU: given the reference's inverse Hessian (and, for its default
  act_order=True, its activation energies), bit-exact with its output;
* the packed producer with act_order: the permuted walk equals the oracle's
  K-grouped walk on the permuted layer, and the layer computes x @ W^T.
"""

import numpy as np
import pytest
import torch

import pico_kernels_b200 as pk
from conftest import SHORT, golden_values
from oracle import quant_ref as o
from pico_kernels_b200 import gptq, quantize

pytestmark = pytest.mark.gpu

TORCH = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def _cases(z, prefix):
    return sorted({k.rsplit("/", 1)[0] for k in z if k.startswith(prefix)})


def _to_torch(arr, dt):
    if dt == "bfloat16":
        return torch.from_numpy(arr.astype(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(arr).to(TORCH[dt])


def _same(got: torch.Tensor, want: np.ndarray, key):
    g = got.float().cpu().numpy()
    assert np.array_equal(np.isnan(g), np.isnan(want)), key
    assert np.array_equal(g[~np.isnan(g)], want[~np.isnan(want)]), key


def test_quantize_col_matches_reference(qcol_golden):
    z = qcol_golden
    keys = _cases(z, "qcol/")
    assert len(keys) == 48
    for key in keys:
        dt = str(z[f"{key}/dtype"])
        w = _to_torch(z[f"{key}/w"], dt).cuda()
        g = int(z[f"{key}/group"])
        out = quantize.quantize_col(w, int(z[f"{key}/bits"]), g or None)
        assert out.dtype == w.dtype and out.shape == w.shape
        _same(out, golden_values(z[f"{key}/out"], dt), key)


def test_rtn_layer_matches_reference(qcol_golden):
    z = qcol_golden
    for key in _cases(z, "rtn/"):
        dt = str(z[f"{key}/dtype"])
        w = _to_torch(z[f"{key}/w"], dt).cuda()
        g = int(z[f"{key}/group"])
        out = quantize.rtn_layer(w, int(z[f"{key}/bits"]), g or None)
        assert out.dtype == w.dtype
        _same(out, golden_values(z[f"{key}/out"], dt), key)


def test_quantize_col_large_columns_vs_oracle():
    g = torch.Generator().manual_seed(5)
    for dt in ("f16", "bf16", "f32"):
        w = (torch.randn(100003, generator=g) * 0.1).to(TORCH[{"f16": "float16", "bf16": "bfloat16",
                                                                "f32": "float32"}[dt]])
        for bits, gs in ((4, 128), (8, None), (2, 1000)):
            out = quantize.quantize_col(w.cuda(), bits, gs)
            want = o.quantize_col_fake(w.float().numpy(), bits, gs, dt)
            _same(out, want, (dt, bits, gs))


def test_quantize_passthrough_and_errors():
    w = torch.randn(64, device="cuda")
    assert quantize.quantize_col(w, 16) is w
    assert torch.equal(quantize.rtn_layer(w.view(8, 8), 16), w.view(8, 8))
    with pytest.raises(ValueError):
        quantize.quantize_col(w, 12)
    with pytest.raises(TypeError):
        quantize.quantize_col(w.double(), 4)
    with pytest.raises(ValueError):
        quantize.quantize_col(w.view(8, 8), 4, 4)


@pytest.mark.parametrize("name", ["gptq_small", "gptq_act_order"])
def test_gptq_layer_matches_reference(name, gptq_golden, gptq_ao_golden):
    z = gptq_golden if name == "gptq_small" else gptq_ao_golden
    keys = _cases(z, "gptq/")
    assert keys
    for key in keys:
        g = int(z[f"{key}/group"])
        bits = int(z.get(f"{key}/bits", 4))
        ao = bool(int(z.get(f"{key}/act_order", 0)))
        w = torch.from_numpy(z[f"{key}/w"]).cuda()
        h_inv = torch.from_numpy(z[f"{key}/h_inv"]).cuda()
        mag = torch.from_numpy(z[f"{key}/act_mag"]).cuda() if ao else None
        out = gptq.gptq_layer(w, None, bits, act_order=ao, group_size=g or None, h_inv=h_inv,
                              act_mag=mag)
        assert torch.equal(out.cpu(), torch.from_numpy(z[f"{key}/wq"])), key


def test_gptq_layer_from_calibration_inputs(gptq_ao_golden):
    # computed end to end on the device (Hessian, inverse, order): the device's
    # summation order differs from the CPU's, so compare the layer's error, not bits
    z = gptq_ao_golden
    key = "gptq/o32_i64_g0_b4_ao1"
    w = torch.from_numpy(z[f"{key}/w"]).cuda()
    x = torch.from_numpy(z[f"{key}/x"]).cuda()
    out = gptq.gptq_layer(w, x, 4)
    ref = torch.from_numpy(z[f"{key}/wq"]).cuda()
    err = torch.norm(x @ (out - w).t()) / torch.norm(x @ (ref - w).t())
    assert 0.9 < err.item() < 1.1
    rtn = quantize.rtn_layer(w, 4)
    assert torch.norm(x @ (out - w).t()) < torch.norm(x @ (rtn - w).t())


def test_packed_gptq_act_order():
    g = torch.Generator().manual_seed(3)
    out_dim, in_dim, n = 256, 512, 1024
    w = (torch.randn(out_dim, in_dim, generator=g) * 0.02).cuda()
    x = (torch.randn(n, in_dim, generator=g) * torch.linspace(0.1, 4.0, in_dim)[torch.randperm(in_dim, generator=g)]).cuda()
    h_inv = gptq.gptq_inverse_hessian(x)
    mag = (x.t() @ x / n).diag()
    packed, scales, perm = gptq.gptq_quantize_int4(w, h_inv=h_inv, act_mag=mag, act_order=True,
                                                   scale_dtype=torch.float32)
    order = torch.argsort(mag, descending=True)
    assert torch.equal(perm, order)
    codes, s32 = o.gptq_int4_codes(w[:, order].cpu().numpy(), h_inv[order][:, order].cpu().numpy(), 128)
    assert np.array_equal(pk.unpack_int4_n(packed).cpu().numpy(), codes)
    assert np.array_equal(scales.cpu().numpy(), s32)
    # the layer: x[:, perm] @ dequant(packed) == x @ W_fake^T
    lin = torch.nn.Linear(in_dim, out_dim, bias=False).cuda()
    lin.weight.data.copy_(w)
    layer = pk.linear.W4A16Linear.from_linear(lin, calib=x, act_order=True, dtype=torch.bfloat16)
    xb = x[:16].to(torch.bfloat16)
    y = layer(xb).float()
    ref = xb.float() @ layer.dequantized_weight().t()
    assert (torch.norm(y - ref) / torch.norm(ref)).item() < 5e-3
    # act_order is at least as good as the plain walk on its calibration inputs
    plain = pk.linear.W4A16Linear.from_linear(lin, calib=x, dtype=torch.bfloat16)
    e_ao = torch.norm(x @ (layer.dequantized_weight() - w).t())
    e_pl = torch.norm(x @ (plain.dequantized_weight() - w).t())
    assert e_ao < 1.05 * e_pl
