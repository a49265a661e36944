"""GPU checks of the W4A16 ``nn.Linear`` drop-in (``pico_kernels_b200.linear``).

Reference: the same layer computed in fp32 torch from the layer's own
dequantized weight (codes x group scales), the reference's formula
(tests/test_gemm_int4.py:26) applied to an ``nn.Linear``. Bounds follow the
GEMM path M selects: M = 1 (CUDA-core GEMV, exact codes, fp32 scale) and M = 8
(tensor-core decode, exact codes, scale in fp32 after the MMA) rel <= 1e-5;
M >= 17 (prefill: q*s rounded to bf16 before the MMA) rel <= 5e-3.
"""

import pytest
import torch
import torch.nn as nn

import pico_kernels_b200 as pk

pytestmark = pytest.mark.gpu


def _ref(layer, x):
    y = x.float().reshape(-1, layer.in_features) @ layer.dequantized_weight().t()
    if layer.bias is not None:
        y = y + layer.bias
    return y.reshape(*x.shape[:-1], layer.out_features)


@pytest.mark.parametrize("lead,tol", [((1,), 1e-5), ((2, 4), 1e-5), ((3, 40), 5e-3)])
@pytest.mark.parametrize("bias", [True, False])
def test_w4a16_linear_matches_dequantized_layer(lead, tol, bias):
    torch.manual_seed(0)
    lin = nn.Linear(1024, 768, bias=bias).cuda().to(torch.bfloat16)
    q = pk.W4A16Linear.from_linear(lin, group_size=128)
    x = torch.randn(*lead, 1024, device="cuda", dtype=torch.bfloat16)
    # fp32 input: the layer rounds it to bf16 (exact here) and returns fp32
    y32 = q(x.float())
    assert y32.shape == (*lead, 768) and y32.dtype == torch.float32
    ref = _ref(q, x)
    rel = (torch.norm(y32 - ref) / torch.norm(ref)).item()
    assert rel <= tol, rel
    # bf16 input: the same fp32 result, rounded once to bf16
    y = q(x)
    assert y.dtype == torch.bfloat16
    assert torch.equal(y, y32.to(torch.bfloat16))
    # the int4 weight stays within about half a quantization step of the float weight
    w = lin.weight.float()
    step = q.scales.float().repeat_interleave(128, dim=0)[:1024].t()
    # (half a step of the fp32 scale, plus |q| <= 7 times the bf16 rounding of the scale)
    assert torch.all((q.dequantized_weight() - w).abs() <= 0.52 * step + 1e-6)


def test_w4a16_linear_fp32_output_path_is_tight():
    """fp16 activations with a bias: fp32 accumulate, bias in fp32, one rounding."""
    torch.manual_seed(1)
    lin = nn.Linear(512, 256).cuda().half()
    q = pk.W4A16Linear.from_linear(lin, group_size=64)
    x = torch.randn(1, 512, device="cuda", dtype=torch.float16)
    ref = _ref(q, x)
    y = q(x)
    assert y.dtype == torch.float16
    assert torch.allclose(y.float(), ref, rtol=2e-3, atol=2e-3)


def test_quantize_linear_layers_swaps_modules():
    torch.manual_seed(2)
    model = nn.Sequential(nn.Linear(256, 512), nn.GELU(), nn.Linear(512, 256)).cuda()
    x = torch.randn(4, 256, device="cuda")
    y_float = model(x)
    pk.quantize_linear_layers(model, group_size=128, dtype=torch.bfloat16)
    assert isinstance(model[0], pk.W4A16Linear) and isinstance(model[2], pk.W4A16Linear)
    y = model(x)
    assert y.dtype == torch.float32 and y.shape == (4, 256)
    # int4 weights: close to the float model, not equal
    rel = (torch.norm(y - y_float) / torch.norm(y_float)).item()
    assert 0 < rel < 0.15, rel
    # and exactly the dequantized-weight model up to fp32 summation order and
    # the bf16 rounding of the activations
    h = model[1](_ref(model[0], x.to(torch.bfloat16)))
    ref = _ref(model[2], h.to(torch.bfloat16))
    assert (torch.norm(y - ref) / torch.norm(ref)).item() < 1e-3
    assert pk.device_status() == (0, 0)
