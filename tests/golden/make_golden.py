"""Generate the golden vectors by running pico-kernels' own functions.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference <path-to-pico-kernels>

It imports ``quantize.quantize_col``, ``gemm_int4.quantize_int4``,
``gemm_int4.pack_int4_n`` and ``gemm_fp8.quantize`` from that checkout and
runs them on CPU torch tensors (the Triton kernels are never launched), then
writes ``golden_small.npz``, ``config1.npz`` and ``gptq_small.npz`` beside
this script (``quantize.gptq_layer`` with act_order=False, the inverse Hessian
it builds, and its fake-quant output), ``quantize_col.npz``
(``quantize.quantize_col`` on fp16 / bf16 / fp32 columns at 2-8 bits and
``quantize.rtn_layer``) and ``gptq_act_order.npz`` (``quantize.gptq_layer``
with its default act_order=True; ``--only`` writes a subset). The GPU box
has no reference checkout: the tests only read the committed ``.npz`` files.

Derived quantities:

* the reference's group quantizer returns fake-quant floats
  (``quantize.py:42-60``); the scale of each group is recomputed here with the
  same torch expression (``quantize.py:58``), and the codes are
  ``round(fake / scale)``, exact because |code| <= 7;
* the packed bytes are ``gemm_int4.pack_int4_n(codes)``;
* Y is ``A.float() @ (codes.float() * scale_stored.float())`` in torch fp32
  (the form of ``tests/test_gemm_int4.py:26``).
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _ref_group_quant(quantize, w: torch.Tensor, group: int, bits: int = 4):
    """Column walk of ``rtn_layer`` (quantize.py:63-68) with groups along K."""
    wf = w.float()
    K, N = wf.shape
    qmax = 2 ** (bits - 1) - 1
    fake = torch.empty_like(wf)
    G = (K + group - 1) // group
    scales = torch.empty(G, N, dtype=torch.float32)
    for n in range(N):
        col = wf[:, n].clone()
        fake[:, n] = quantize.quantize_col(col, bits, group)
        for g in range(G):
            sl = slice(g * group, min((g + 1) * group, K))
            scales[g, n] = col[sl].abs().max().clamp_min(1e-12) / qmax
    rep = scales.repeat_interleave(group, dim=0)[:K]
    codes = torch.round(fake / rep).to(torch.int8)
    assert torch.equal(codes.float() * rep, fake), "codes*scale must reproduce the reference"
    return fake, scales, codes


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


def _edge_weights() -> dict[str, torch.Tensor]:
    torch.manual_seed(7)
    cases = {}
    # ties: a group whose absmax is 7 -> scale exactly 1.0; x.5 values round half-even
    ties = torch.randn(128, 8) * 2
    ties[0, :] = 7.0
    vals = torch.tensor([0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.5, -0.5, -1.5, -2.5, -3.5, -6.5])
    ties[1:1 + vals.numel(), :] = vals[:, None]
    cases["ties_f32_K128_N8"] = ties
    # an all-zero group, a negative absmax, tiny values below the 1e-12 clamp, -0.0
    e = torch.randn(256, 16) * 0.02
    e[:128, 0] = 0.0
    e[128:, 1] = -0.0
    e[:, 2] = -e[:, 2].abs()
    e[:128, 3] = torch.randn(128) * 1e-14
    e[:, 4] = torch.randn(256) * 1e4
    cases["edge_f32_K256_N16"] = e
    return cases


def make_small(ref: Path) -> dict[str, np.ndarray]:
    sys.path.insert(0, str(ref))
    import gemm_fp8  # noqa: E402
    import gemm_int4  # noqa: E402
    import quantize  # noqa: E402

    out: dict[str, np.ndarray] = {}

    # --- reference known-answer test: tests/test_quantize.py:35-42 -----------
    torch.manual_seed(1)
    w = torch.randn(64)
    out["kat_quantize_col/w"] = _np(w)
    out["kat_quantize_col/out"] = _np(quantize.quantize_col(w, 4, group_size=16))
    out["kat_quantize_col_nogroup/out"] = _np(quantize.quantize_col(w, 4))
    out["kat_quantize_col_3bit/out"] = _np(quantize.quantize_col(w, 3, group_size=16))

    # --- per-group quantize + pack (the hot-path quantizer) --------------------
    group_cases = []
    torch.manual_seed(11)
    for dt in (torch.float16, torch.bfloat16, torch.float32):
        for (K, N, g) in ((256, 64, 128), (200, 32, 128), (128, 48, 32), (384, 16, 64)):
            group_cases.append((f"rand_{str(dt)[6:]}_K{K}_N{N}_g{g}",
                                (torch.randn(K, N) * 0.02).to(dt), g))
    for name, wt in _edge_weights().items():
        group_cases.append((name, wt, 128))
    for name, wt, g in group_cases:
        fake, scales, codes = _ref_group_quant(quantize, wt, g)
        key = f"group/{name}"
        out[f"{key}/w"] = _np(wt)
        out[f"{key}/dtype"] = np.array(str(wt.dtype)[6:])
        out[f"{key}/group"] = np.array(g)
        out[f"{key}/fake"] = _np(fake)
        out[f"{key}/scales_f32"] = _np(scales)
        out[f"{key}/scales_f16"] = _np(scales.to(torch.float16))
        out[f"{key}/scales_bf16"] = _np(scales.to(torch.bfloat16))
        out[f"{key}/codes"] = _np(codes)
        if wt.shape[1] % 2 == 0:
            out[f"{key}/packed"] = _np(gemm_int4.pack_int4_n(codes))

    # --- per-tensor quantize_int4 + pack (gemm_int4.py:58-72) -----------------
    torch.manual_seed(12)
    for dt in (torch.float16, torch.bfloat16):
        for (K, N, std) in ((128, 256, 1.0), (64, 128, 0.02)):
            wt = (torch.randn(K, N) * std).to(dt)
            w_q, scale = gemm_int4.quantize_int4(wt)
            key = f"pt/{str(dt)[6:]}_K{K}_N{N}"
            out[f"{key}/w"] = _np(wt)
            out[f"{key}/codes"] = _np(w_q)
            out[f"{key}/scale"] = np.array(scale, dtype=np.float64)
            out[f"{key}/packed"] = _np(gemm_int4.pack_int4_n(w_q))

    # --- pack round trip over the reference test's value range ---------------
    torch.manual_seed(1)
    w_q = torch.randint(-8, 7, (256, 256), dtype=torch.int8)   # tests/test_gemm_int4.py:35
    out["pack/roundtrip/codes"] = _np(w_q)
    out["pack/roundtrip/packed"] = _np(gemm_int4.pack_int4_n(w_q))
    full = torch.arange(-8, 8, dtype=torch.int8).repeat(4, 2)  # every nibble value
    out["pack/allnibbles/codes"] = _np(full)
    out["pack/allnibbles/packed"] = _np(gemm_int4.pack_int4_n(full))

    # --- fp8 quantize (gemm_fp8.py:89-95) and the precast GEMM reference ------
    torch.manual_seed(13)
    for dt in (torch.float16, torch.bfloat16):
        a = torch.randn(64, 96).to(dt)
        b = (torch.randn(96, 80) * 3).to(dt)
        a8, sa = gemm_fp8.quantize(a)
        b8, sb = gemm_fp8.quantize(b)
        key = f"fp8/{str(dt)[6:]}"
        out[f"{key}/a"] = _np(a)
        out[f"{key}/b"] = _np(b)
        out[f"{key}/a8"] = _np(a8)
        out[f"{key}/b8"] = _np(b8)
        out[f"{key}/sa"] = np.array(sa, dtype=np.float64)
        out[f"{key}/sb"] = np.array(sb, dtype=np.float64)
        out_scale = 1.0 / (sa * sb)                                 # gemm_fp8.py:106
        y = (a8.double() @ b8.double()).float() * out_scale
        out[f"{key}/y"] = _np(y)
    return out


def config1_inputs():
    """W[1024,1024] fp16 ~ N(0, 0.02) (seed 0), A[16,1024] fp16 ~ N(0,1) (seed 1)."""
    g0 = torch.Generator().manual_seed(0)
    w = (torch.randn(1024, 1024, generator=g0) * 0.02).to(torch.float16)
    g1 = torch.Generator().manual_seed(1)
    a = torch.randn(16, 1024, generator=g1).to(torch.float16)
    return w, a


def make_config1(ref: Path) -> dict[str, np.ndarray]:
    sys.path.insert(0, str(ref))
    import gemm_int4  # noqa: E402
    import quantize  # noqa: E402

    w, a = config1_inputs()
    fake, scales, codes = _ref_group_quant(quantize, w, 128)
    s16 = scales.to(torch.float16)
    packed = gemm_int4.pack_int4_n(codes)
    y = a.float() @ (codes.float() * s16.float().repeat_interleave(128, dim=0))
    return {
        "w_sha256": np.array(hashlib.sha256(_np(w).tobytes()).hexdigest()),
        "a_sha256": np.array(hashlib.sha256(_np(a).tobytes()).hexdigest()),
        "packed": _np(packed),
        "scales_f16": _np(s16),
        "y": _np(y),
    }


def make_gptq(ref: Path) -> dict[str, np.ndarray]:
    """``quantize.gptq_layer`` (quantize.py:71-115) with act_order=False on CPU,
    plus the inverse Hessian built with the reference's own expressions
    (quantize.py:88-93), which the restatement takes as an input."""
    sys.path.insert(0, str(ref))
    import quantize  # noqa: E402

    out: dict[str, np.ndarray] = {}
    torch.manual_seed(21)
    for (o_dim, i_dim, n, gs) in ((32, 64, 256, None), (48, 40, 128, 8), (16, 96, 512, 16)):
        w = torch.randn(o_dim, i_dim) * 0.02
        x = torch.randn(n, i_dim) * torch.linspace(0.2, 3.0, i_dim)  # uneven feature energy
        xf = x.float()
        H = (xf.t() @ xf) / n
        diag_mean = torch.diag(H).clone().mean()
        H = H + 0.01 * diag_mean * torch.eye(i_dim)
        h_inv = torch.linalg.inv(H)
        wq = quantize.gptq_layer(w, x, 4, damp=0.01, act_order=False, group_size=gs)
        key = f"gptq/o{o_dim}_i{i_dim}_g{gs or 0}"
        out[f"{key}/w"] = _np(w)
        out[f"{key}/x"] = _np(x)
        out[f"{key}/h_inv"] = _np(h_inv)
        out[f"{key}/group"] = np.array(gs or 0)
        out[f"{key}/wq"] = _np(wq)
    return out


def make_quantize_col(ref: Path) -> dict[str, np.ndarray]:
    """``quantize.quantize_col`` (quantize.py:42-60) on fp16 / bf16 / fp32
    columns at 2, 3, 4 and 8 bits, with and without groups (a ragged last
    group included), and ``quantize.rtn_layer`` (quantize.py:63-68) on small
    layers; edge columns: a group of zeros, values below the 1e-12 floor (it
    underflows to 0 in fp16), ties at x.5 of the scale, and large magnitudes."""
    sys.path.insert(0, str(ref))
    import quantize  # noqa: E402

    out: dict[str, np.ndarray] = {}
    torch.manual_seed(31)
    base = torch.randn(100) * 0.05
    edge = torch.randn(64) * 0.02
    edge[:16] = 0.0                                       # a group of zeros
    edge[16:32] = torch.randn(16) * 1e-9                  # below fp16's subnormals
    edge[32:48] = torch.tensor([7.0, 0.5, 1.5, 2.5, -3.5, 4.5, -5.5, 6.5] * 2)  # scale 1, ties
    edge[48:64] = torch.randn(16) * 3e3
    cols = {"rand": base, "edge": edge}
    i = 0
    for dt in (torch.float16, torch.bfloat16, torch.float32):
        for cname, col in cols.items():
            w = col.to(dt)
            for bits in (2, 3, 4, 8):
                for gs in (None, 16):
                    key = f"qcol/{i:03d}"
                    i += 1
                    out[f"{key}/w"] = _np(w)
                    out[f"{key}/out"] = _np(quantize.quantize_col(w, bits, gs))
                    out[f"{key}/dtype"] = np.array(str(dt)[6:])
                    out[f"{key}/bits"] = np.array(bits)
                    out[f"{key}/group"] = np.array(gs or 0)
                    out[f"{key}/name"] = np.array(cname)
    torch.manual_seed(32)
    j = 0
    for dt in (torch.float16, torch.bfloat16, torch.float32):
        w = (torch.randn(48, 24) * 0.02).to(dt)
        for bits, gs in ((4, None), (4, 8), (3, 16), (8, None)):
            key = f"rtn/{j:03d}"
            j += 1
            out[f"{key}/w"] = _np(w)
            out[f"{key}/out"] = _np(quantize.rtn_layer(w, bits, gs))
            out[f"{key}/dtype"] = np.array(str(dt)[6:])
            out[f"{key}/bits"] = np.array(bits)
            out[f"{key}/group"] = np.array(gs or 0)
    return out


def make_gptq_act_order(ref: Path) -> dict[str, np.ndarray]:
    """``quantize.gptq_layer`` (quantize.py:71-115) with its default
    act_order=True (and a 3-bit case without it), plus the inverse Hessian and
    the activation energies it computed with the reference's own expressions
    (quantize.py:86-93), which the GPU walk takes as inputs."""
    sys.path.insert(0, str(ref))
    import quantize  # noqa: E402

    out: dict[str, np.ndarray] = {}
    torch.manual_seed(41)
    cases = ((32, 64, 256, None, 4, True), (48, 40, 128, 8, 4, True), (16, 96, 512, 16, 4, True),
             (40, 48, 192, 8, 3, True), (24, 32, 128, None, 3, False))
    for (o_dim, i_dim, n, gs, bits, ao) in cases:
        w = torch.randn(o_dim, i_dim) * 0.02
        x = torch.randn(n, i_dim) * torch.linspace(0.2, 3.0, i_dim)[torch.randperm(i_dim)]
        xf = x.float()
        H = (xf.t() @ xf) / n
        act_mag = torch.diag(H).clone()
        H = H + 0.01 * act_mag.mean() * torch.eye(i_dim)
        h_inv = torch.linalg.inv(H)
        wq = quantize.gptq_layer(w, x, bits, damp=0.01, act_order=ao, group_size=gs)
        key = f"gptq/o{o_dim}_i{i_dim}_g{gs or 0}_b{bits}_ao{int(ao)}"
        out[f"{key}/w"] = _np(w)
        out[f"{key}/x"] = _np(x)
        out[f"{key}/h_inv"] = _np(h_inv)
        out[f"{key}/act_mag"] = _np(act_mag)
        out[f"{key}/group"] = np.array(gs or 0)
        out[f"{key}/bits"] = np.array(bits)
        out[f"{key}/act_order"] = np.array(int(ao))
        out[f"{key}/wq"] = _np(wq)
    return out


FILES = {
    "golden_small.npz": make_small,
    "config1.npz": make_config1,
    "gptq_small.npz": make_gptq,
    "quantize_col.npz": make_quantize_col,
    "gptq_act_order.npz": make_gptq_act_order,
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", nargs="*", choices=sorted(FILES), default=None,
                    help="write only these files (default: all)")
    args = ap.parse_args()
    torch.set_num_threads(8)
    for name in args.only or sorted(FILES):
        arrays = FILES[name](args.reference)
        np.savez_compressed(HERE / name, **arrays)
        print("wrote", HERE / name, len(arrays), "arrays")


if __name__ == "__main__":
    main()
