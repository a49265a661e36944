"""numpy restatement of pico-kernels' quantized-matmul arithmetic.

TEST INFRASTRUCTURE ONLY. Nothing in ``pico_kernels_b200`` imports this file.

Every function cites the reference line it restates (paths relative to the
pico-kernels project root). The reference is PyTorch; the arithmetic facts
that make this restatement bit-exact were established against torch 2.11 CPU
and are pinned by the golden vectors in ``tests/golden``:

* ``fp32_tensor / fp32_0dim_tensor`` is an IEEE correctly-rounded division
  (not a multiply by a reciprocal);
* ``half_or_bf16_tensor / python_float`` and ``... * python_float`` compute
  ``float32(x) op float32(scalar)`` once, then round to the tensor's dtype;
* ``torch.round`` is round-half-to-even;
* ``.to(float8_e4m3fn)`` is round-to-nearest-even with overflow to NaN.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "E4M3_MAX",
    "f32_to_bf16_bits", "bf16_bits_to_f32", "round_to_bf16", "round_to_dtype",
    "f32_to_e4m3_bits", "e4m3_bits_to_f32",
    "group_quant_codes", "store_scales", "quantize_col_fake", "rtn_layer_fake",
    "quantize_int4_per_tensor", "pack_int4_n", "unpack_int4_n",
    "dequant_weight", "w4a16_reference", "int4_gemm_per_tensor_reference",
    "fp8_quantize", "fp8_gemm_reference", "dense_gemm_reference",
    "gptq_inverse_hessian_inputs", "gptq_fake_quant_columns", "gptq_int4_codes",
]

# gemm_fp8.py:24 -- float(torch.finfo(torch.float8_e4m3fn).max)
E4M3_MAX = 448.0


# ---------------------------------------------------------------------------
# Floating-point storage formats (bit-level, round-to-nearest-even)
# ---------------------------------------------------------------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 -> bf16 (RNE), returned as uint16 bit patterns.

    Matches ``tensor.to(torch.bfloat16)`` for finite inputs.
    """
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) & 0xFFFF
    r = r.astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16, returned as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 ``x`` to ``dtype`` ("f16", "bf16" or "f32"); return fp32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return round_to_bf16(x)
    if dtype == "f32":
        return x
    raise ValueError(dtype)


def _e4m3_positive_table() -> np.ndarray:
    """Magnitudes of e4m3fn codes 0x00..0x7E (0x7F is NaN), ascending."""
    c = np.arange(0x7F)
    e = c >> 3
    m = c & 7
    return np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))


_E4M3_TABLE = _e4m3_positive_table()


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn bit patterns: round to nearest, ties to the even
    code, magnitudes >= 464 (the midpoint above 448) and NaN to 0x7F.

    e4m3fn has bias 7, 3 mantissa bits, largest finite 448 (0x7E), no
    infinities and subnormal spacing 2^-9.
    """
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64).ravel()
    t = _E4M3_TABLE
    hi = np.clip(np.searchsorted(t, a, side="left"), 0, len(t) - 1)
    lo = np.clip(hi - 1, 0, len(t) - 1)
    dlo = a - t[lo]
    dhi = t[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(a <= t[0], 0, code)
    code = np.where(np.isnan(a) | (a >= 464.0), 0x7F, code).astype(np.uint8)
    sign = (np.signbit(x).ravel().astype(np.uint8) << 7)
    return (code | sign).reshape(x.shape)


def e4m3_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    v = np.where((b & 0x7F) == 0x7F, np.nan, v)
    return (s * v).astype(np.float32)


# ---------------------------------------------------------------------------
# Per-group int4 quantization (quantize.py)
# ---------------------------------------------------------------------------
def group_quant_codes(w: np.ndarray, group_size: int = 128, bits: int = 4):
    """Codes and fp32 scales of per-group symmetric RTN along K of ``w[K, N]``.

    Restates ``quantize.quantize_col`` (quantize.py:42-60) applied to each
    column ``w[:, n]`` the way ``rtn_layer`` walks columns (quantize.py:63-68),
    with the groups running along K:

    * ``qmax = 2**(bits-1) - 1`` (quantize.py:51);
    * ``scale = max|w[group]|.clamp_min(1e-12) / qmax`` in fp32 (quantize.py:58);
    * ``q = clamp(round_half_even(w / scale), -qmax, qmax)`` (quantize.py:59).

    The last group is ragged when ``K % group_size != 0`` (quantize.py:57).
    Returns ``(codes int8[K, N], scales float32[ceil(K/g), N])``.
    """
    w = np.asarray(w, dtype=np.float32)
    K, N = w.shape
    qmax = np.float32(2 ** (bits - 1) - 1)
    G = (K + group_size - 1) // group_size
    scales = np.empty((G, N), dtype=np.float32)
    codes = np.empty((K, N), dtype=np.int8)
    for g in range(G):
        sl = slice(g * group_size, min((g + 1) * group_size, K))
        blk = w[sl]
        amax = np.abs(blk).max(axis=0)
        s = np.maximum(amax, np.float32(1e-12)) / qmax       # fp32 IEEE division
        scales[g] = s
        q = np.rint(blk / s[None, :])                         # fp32 div, half-even
        codes[sl] = np.clip(q, -qmax, qmax).astype(np.int8)
    return codes, scales


def store_scales(scales_f32: np.ndarray, dtype: str) -> np.ndarray:
    """The stored scale: fp32 scale rounded (RNE) to the scale dtype, as fp32."""
    return round_to_dtype(scales_f32, dtype)


def quantize_col_fake(w_col: np.ndarray, bits: int, group_size: int | None = None,
                      dtype: str = "f32"):
    """``quantize.quantize_col`` (quantize.py:42-60) on a column of ``dtype``
    ("f16", "bf16" or "f32"; values given as fp32): fake-quant output as fp32
    values of that dtype.

    Each step of quantize.py:58-59 (``.clamp_min(1e-12)``, ``/ qmax``,
    ``w / scale``, ``round``, ``clamp``, ``* scale``) is computed in fp32 and
    rounded to the dtype, as torch evaluates it on a half tensor; in fp16 the
    1e-12 floor rounds to 0, so a zero group gets NaN outputs, as upstream."""
    rt = lambda v: round_to_dtype(v, dtype)  # noqa: E731
    w_col = rt(np.asarray(w_col, dtype=np.float32))
    if bits >= 16:
        return w_col.copy()
    qmax = np.float32(2 ** (bits - 1) - 1)
    gs = w_col.size if group_size is None else group_size
    out = np.empty_like(w_col)
    with np.errstate(divide="ignore", invalid="ignore"):
        for g in range(0, w_col.size, gs):
            blk = w_col[g:g + gs]
            s = rt(rt(np.maximum(np.abs(blk).max(), np.float32(1e-12))) / qmax)
            q = np.clip(np.rint(rt(blk / s)), -qmax, qmax)
            out[g:g + gs] = rt(q * s)
    return out


def rtn_layer_fake(w: np.ndarray, bits: int, group_size: int | None = None,
                   dtype: str = "f32") -> np.ndarray:
    """``quantize.rtn_layer`` (quantize.py:63-68): every input column of
    ``w[out, in]`` (values of ``dtype``) quantized in fp32 (``w.float()``),
    the result rounded back to ``dtype``."""
    wf = round_to_dtype(np.asarray(w, dtype=np.float32), dtype)
    if bits >= 16:
        return wf.copy()
    out = np.empty_like(wf)
    for j in range(wf.shape[1]):
        out[:, j] = quantize_col_fake(wf[:, j], bits, group_size, "f32")
    return round_to_dtype(out, dtype)


# ---------------------------------------------------------------------------
# Per-tensor int4 quantization and packing (gemm_int4.py)
# ---------------------------------------------------------------------------
def quantize_int4_per_tensor(w: np.ndarray, dtype: str):
    """``gemm_int4.quantize_int4`` (gemm_int4.py:58-62).

    ``scale = max|w| / 7.0`` is a Python double (gemm_int4.py:60).
    ``w / scale`` runs in the tensor's dtype: fp32 quotient rounded to ``dtype``;
    then ``round`` (half-even) and ``clamp(-8, 7)`` (gemm_int4.py:61).
    ``w`` holds fp32 values exactly representable in ``dtype``.
    """
    w = np.asarray(w, dtype=np.float32)
    scale = float(np.abs(w).max()) / 7.0
    quo = round_to_dtype(w / np.float32(scale), dtype)
    q = np.clip(np.rint(quo), -8, 7).astype(np.int8)
    return q, scale


def pack_int4_n(q: np.ndarray) -> np.ndarray:
    """``gemm_int4.pack_int4_n`` (gemm_int4.py:65-72).

    byte ``[k, j] = (q[k, 2j] & 0xF) | ((q[k, 2j+1] & 0xF) << 4)``.
    """
    q = np.asarray(q).astype(np.int32)
    K, N = q.shape
    if N % 2:
        raise ValueError("N must be even")
    lo = q[:, 0::2] & 0xF
    hi = q[:, 1::2] & 0xF
    return (lo | (hi << 4)).astype(np.uint8)


def unpack_int4_n(p: np.ndarray) -> np.ndarray:
    """Inverse of ``pack_int4_n``: sign-extend each nibble, low nibble = even
    column (gemm_int4.py:44-49, tests/test_gemm_int4.py:37-41)."""
    p = np.asarray(p, dtype=np.uint8).astype(np.int32)
    lo = p & 0xF
    hi = p >> 4
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    K, Nh = p.shape
    out = np.empty((K, 2 * Nh), dtype=np.int8)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out


# ---------------------------------------------------------------------------
# GEMM references
# ---------------------------------------------------------------------------
def dequant_weight(codes: np.ndarray, scales_stored: np.ndarray, group_size: int) -> np.ndarray:
    """``q.float() * s.float()`` with the scale repeated over each K group."""
    K = codes.shape[0]
    s = np.repeat(np.asarray(scales_stored, dtype=np.float32), group_size, axis=0)[:K]
    return codes.astype(np.float32) * s


def w4a16_reference(a: np.ndarray, codes: np.ndarray, scales_stored: np.ndarray,
                    group_size: int = 128) -> np.ndarray:
    """Dequantize-then-matmul in fp32: ``A.float() @ (q.float() * s)``.

    The form of the reference's own oracle (tests/test_gemm_int4.py:26,
    gemm_int4.py:102) with the per-tensor scale replaced by group scales.
    """
    return np.asarray(a, dtype=np.float32) @ dequant_weight(codes, scales_stored, group_size)


def int4_gemm_per_tensor_reference(a: np.ndarray, codes: np.ndarray, scale: float) -> np.ndarray:
    """``a.float() @ (w_q.float() * scale)`` (tests/test_gemm_int4.py:26)."""
    w = codes.astype(np.float32) * np.float32(scale)
    return np.asarray(a, dtype=np.float32) @ w


def fp8_quantize(x: np.ndarray, dtype: str):
    """``gemm_fp8.quantize`` (gemm_fp8.py:89-95).

    ``scale = 448 / max|x|`` (Python double); ``x * scale`` is an fp32 product
    rounded to x's dtype; the cast to e4m3 is RNE. Returns (e4m3 bits, scale).
    """
    x = np.asarray(x, dtype=np.float32)
    scale = E4M3_MAX / float(np.abs(x).max())
    y = round_to_dtype(x * np.float32(scale), dtype)
    return f32_to_e4m3_bits(y), scale


def fp8_gemm_reference(a8_bits: np.ndarray, a_scale: float, b8_bits: np.ndarray,
                       b_scale: float) -> np.ndarray:
    """``fp8_gemm_precast`` (gemm_fp8.py:98-117): fp32 accumulate of the e4m3
    values, then one multiply by ``out_scale = 1/(a_scale*b_scale)``
    (gemm_fp8.py:106, :86)."""
    a = e4m3_bits_to_f32(a8_bits).astype(np.float64)
    b = e4m3_bits_to_f32(b8_bits).astype(np.float64)
    out_scale = np.float32(1.0 / (a_scale * b_scale))
    return (a @ b).astype(np.float32) * out_scale


def dense_gemm_reference(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """``a.float() @ b.float()`` (tests/test_gemm_splitk.py:24)."""
    return np.asarray(a, dtype=np.float32) @ np.asarray(b, dtype=np.float32)


# ---------------------------------------------------------------------------
# GPTQ (quantize.py:71-115) with act_order=False, given the inverse Hessian
# ---------------------------------------------------------------------------
def gptq_inverse_hessian_inputs(x: np.ndarray, damp: float = 0.01):
    """``H = X^T X / n + damp * mean(diag) * I`` (quantize.py:88-92), fp32.

    The reference inverts this with ``torch.linalg.inv`` (quantize.py:93); the
    inverse is taken as an input by the functions below, so that a restatement
    fed the reference's own inverse reproduces its loop bit for bit."""
    xf = np.asarray(x, dtype=np.float32)
    n, d = xf.shape
    h = (xf.T @ xf) / np.float32(n)
    mean = np.float32(np.diag(h).mean())
    return h + np.float32(damp) * mean * np.eye(d, dtype=np.float32)


def gptq_fake_quant_columns(w: np.ndarray, h_inv: np.ndarray, bits: int,
                            group_size: int | None = None,
                            act_mag: np.ndarray | None = None) -> np.ndarray:
    """``gptq_layer(w, x, bits, act_order=False, group_size)`` (quantize.py:71-115).

    Walks the input columns j of ``w[out, in]`` in order (quantize.py:99):
    ``q = quantize_col(w[:, j])`` with its groups along the OUTPUT rows
    (quantize.py:100), ``err = w[:, j] - q``, ratio ``h_inv[j, j+1:] /
    h_inv[j, j]`` and ``w[:, j+1:] -= outer(err, ratio)`` (quantize.py:101-104),
    each product and difference rounded to fp32 on its own. With ``act_mag``
    (act_order=True, quantize.py:97-101) the columns of ``w`` and the rows and
    columns of ``h_inv`` are first put in order of decreasing ``act_mag``
    (distinct values: the order is unique) and the result is put back."""
    wq = np.array(w, dtype=np.float32, copy=True)
    h_inv = np.asarray(h_inv, dtype=np.float32)
    if bits >= 16:
        return wq
    if act_mag is not None:
        order = np.argsort(-np.asarray(act_mag, dtype=np.float32), kind="stable")
        res = gptq_fake_quant_columns(wq[:, order], h_inv[order][:, order], bits, group_size)
        return res[:, np.argsort(order, kind="stable")]
    d = wq.shape[1]
    for j in range(d):
        col = wq[:, j].copy()
        q = quantize_col_fake(col, bits, group_size)
        err = (col - q).astype(np.float32)
        ratio = (h_inv[j, j + 1:] / h_inv[j, j]).astype(np.float32)
        wq[:, j + 1:] = wq[:, j + 1:] - np.outer(err, ratio).astype(np.float32)
        wq[:, j] = q
    return wq


def gptq_int4_codes(w: np.ndarray, h_inv: np.ndarray, group_size: int = 128):
    """The packed-weight form of the same loop: codes and scales in the W4A16
    GEMM's layout ``B[K = in, N = out]`` with groups along K.

    The column walk, error and update are quantize.py:99-104 as in
    ``gptq_fake_quant_columns``; the only change is the scale, which must be
    shared by ``group_size`` consecutive input features to be applied after
    the GEMM's K reduction: at the first input feature of each group, per
    output row ``n``, ``scale = max|w[n, group]|.clamp_min(1e-12) / 7`` over
    that group's CURRENT (error-updated) weights (quantize.py:58 applied along
    K); each column then uses ``q = clamp(round(w / scale), -7, 7)`` and
    ``q * scale`` (quantize.py:59). With ``h_inv = I`` there is no error
    feedback and this is ``group_quant_codes(w.T, group_size)``.
    Returns ``(codes int8[in, out], scales float32[ceil(in/g), out])``."""
    wq = np.array(w, dtype=np.float32, copy=True)       # [out, in]
    h_inv = np.asarray(h_inv, dtype=np.float32)
    out_dim, d = wq.shape
    qmax = np.float32(7)
    G = (d + group_size - 1) // group_size
    scales = np.empty((G, out_dim), dtype=np.float32)
    codes = np.empty((d, out_dim), dtype=np.int8)
    s = None
    for j in range(d):
        if j % group_size == 0:
            blk = wq[:, j:min(j + group_size, d)]
            s = np.maximum(np.abs(blk).max(axis=1), np.float32(1e-12)) / qmax
            scales[j // group_size] = s
        col = wq[:, j].copy()
        qi = np.clip(np.rint(col / s), -qmax, qmax)
        q = (qi * s).astype(np.float32)
        codes[j] = qi.astype(np.int8)
        err = (col - q).astype(np.float32)
        ratio = (h_inv[j, j + 1:] / h_inv[j, j]).astype(np.float32)
        wq[:, j + 1:] = wq[:, j + 1:] - np.outer(err, ratio).astype(np.float32)
        wq[:, j] = q
    return codes, scales
