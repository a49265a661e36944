"""GPU parity of the GPTQ producer of packed int4 weights (``pk_gptq_int4``).

Oracle: ``oracle.quant_ref.gptq_int4_codes``, the column walk of
quantize.gptq_layer (quantize.py:99-104; pinned bit for bit against the
reference's own output in tests/test_oracle_golden.py) with group scales
along the input features. Given the same inverse Hessian, codes and fp32
scales must be bit-exact: the kernels apply every update in the reference's
order with separately rounded products and differences.
"""

import numpy as np
import pytest
import torch

import pico_kernels_b200 as pk
from oracle import quant_ref as o

pytestmark = pytest.mark.gpu


def _case(out_dim, in_dim, n, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((out_dim, in_dim)) * 0.02).astype(np.float32)
    x = (rng.standard_normal((n, in_dim)) * np.linspace(0.2, 3.0, in_dim)).astype(np.float32)
    x[:, 1:] += 0.7 * x[:, :-1]  # correlated features: real error feedback
    h = o.gptq_inverse_hessian_inputs(x, 0.01)
    h_inv = np.linalg.inv(h.astype(np.float64)).astype(np.float32)
    return w, x, h_inv


@pytest.mark.parametrize("out_dim,in_dim,group", [
    (256, 384, 128),   # three full groups, trailing updates across groups
    (96, 200, 64),     # ragged last group (8 features)
    (130, 72, 16),     # output count not a multiple of the 64-thread blocks
])
def test_gptq_matches_oracle_bit_exact(out_dim, in_dim, group):
    w, _, h_inv = _case(out_dim, in_dim, 1024, out_dim + in_dim)
    codes_ref, scales_ref = o.gptq_int4_codes(w, h_inv, group)
    packed, scales = pk.gptq_quantize_int4(torch.from_numpy(w).cuda(), group_size=group,
                                           h_inv=torch.from_numpy(h_inv).cuda(),
                                           scale_dtype=torch.float32)
    codes = pk.unpack_int4_n(packed).cpu().numpy()
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), scales_ref.view(np.uint32))
    assert np.array_equal(codes, codes_ref)
    assert np.array_equal(packed.cpu().numpy(), o.pack_int4_n(codes_ref))
    assert pk.device_status() == (0, 0)


def test_gptq_identity_hessian_is_rtn():
    """No error feedback (Hinv = I): the producer equals quantize_int4_grouped."""
    torch.manual_seed(0)
    w = torch.randn(512, 256, device="cuda") * 0.02
    packed, scales = pk.gptq_quantize_int4(w, h_inv=torch.eye(256, device="cuda"), group_size=128,
                                           scale_dtype=torch.bfloat16)
    p2, s2 = pk.quantize_int4_grouped(w.t(), 128, scale_dtype=torch.bfloat16)
    assert torch.equal(packed, p2) and torch.equal(scales, s2)


def test_gptq_lowers_layer_error_and_feeds_the_gemm():
    """From calibration inputs (Hessian and inverse on the device): the layer
    output error on those inputs is below round-to-nearest's, and the packed
    result runs through int4_gemm (which must equal x @ dequantized W)."""
    w_np, x_np, _ = _case(1024, 1024, 4096, 7)
    w = torch.from_numpy(w_np).cuda().to(torch.bfloat16)
    x = torch.from_numpy(x_np).cuda()
    packed, scales = pk.gptq_quantize_int4(w, x, group_size=128)
    p_rtn, s_rtn = pk.quantize_int4_grouped(w.t(), 128)
    xb = x.to(torch.bfloat16)
    ref = xb.float() @ w.float().t()
    y_gptq = pk.int4_gemm(xb[:16], packed, scales)
    y_rtn = pk.int4_gemm(xb[:16], p_rtn, s_rtn)

    def deq(p, s):
        return pk.unpack_int4_n(p).float() * s.float().repeat_interleave(128, dim=0)

    e_gptq = torch.norm(xb.float() @ deq(packed, scales) - ref).item()
    e_rtn = torch.norm(xb.float() @ deq(p_rtn, s_rtn) - ref).item()
    # the reference's update uses the fixed inverse (quantize.py:102), weaker than a
    # downdated one; measured 0.81 x RTN's error on this layer
    assert e_gptq < 0.9 * e_rtn, (e_gptq, e_rtn)
    y_ref = xb[:16].float() @ deq(packed, scales)
    assert (torch.norm(y_gptq - y_ref) / torch.norm(y_ref)).item() < 1e-5
    assert (torch.norm(y_rtn - ref[:16]) / torch.norm(ref[:16])).item() < 0.2


def test_quantize_linear_layers_with_calibration():
    """Sequential GPTQ over a small MLP (quantize.py:160-184): closer to the
    float model on the calibration batch than round-to-nearest."""
    torch.manual_seed(3)
    base = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(),
                               torch.nn.Linear(512, 256)).cuda()
    calib = torch.randn(512, 256, device="cuda")
    calib[:, 1:] += 0.8 * calib[:, :-1].clone()
    y_float = base(calib)
    import copy
    m_rtn = pk.quantize_linear_layers(copy.deepcopy(base), group_size=64)
    m_gptq = pk.quantize_linear_layers(copy.deepcopy(base), group_size=64, calib=calib)
    e_rtn = torch.norm(m_rtn(calib) - y_float).item()
    e_gptq = torch.norm(m_gptq(calib) - y_float).item()
    assert e_gptq < e_rtn, (e_gptq, e_rtn)
    assert isinstance(m_gptq[2], pk.W4A16Linear)
