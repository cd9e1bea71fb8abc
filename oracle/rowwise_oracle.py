"""CPU restatement (numpy) of the reference's row-wise STU-layer operators.

TEST INFRASTRUCTURE ONLY: imported by tests, never by the product path.

* ``weighted_layer_norm``      -- ``weightedLayerNorm``, recir/ops/kjt_split_per_feature.cpp:197-244
* ``layer_norm_mul_quantized`` -- ``layerNormMulQuantized``, :558-600, with
  ``quantizeFp8Rowwise``, :492-501

The reference computes statistics and the normalisation in float32 and materialises some
intermediates in the input dtype (the normalised rows returned by ``weightedLayerNorm``, silu(u),
sigmoid(u), the product); ``dtype`` names that element type ("float32", "bfloat16", "float16") and
the same roundings are applied here.  Inputs and outputs are float32 arrays holding values that
are representable in ``dtype``; the fp8 copy is returned as e4m3 bytes (uint8).

Pinned against golden vectors produced by the reference's compiled operators
(tests/golden/rowwise_golden.npz, generator tests/golden/make_rowwise_golden.py).
"""
from __future__ import annotations

import numpy as np


def round_to(x, dtype: str):
    """float32 -> dtype -> float32 (round to nearest even), i.e. what materialising a tensor does."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        b = x.view(np.uint32).astype(np.uint64)
        rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
        out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
        return np.where(np.isnan(x), x, out)
    raise ValueError(dtype)


def _sigmoid(x):
    x = np.asarray(x, dtype=np.float32)
    return (np.float32(1) / (np.float32(1) + np.exp(-x, dtype=np.float32))).astype(np.float32)


def weighted_layer_norm(x, weight, bias, eps, dtype="float32", mean=None, rstd=None, is_swish=False):
    """Returns (y, mean, rstd); kjt_split_per_feature.cpp:220-243."""
    xf = np.asarray(x, dtype=np.float32)
    if mean is None or rstd is None:
        mean = xf.mean(axis=1, dtype=np.float32)
        centered = xf - mean[:, None]
        rstd = (np.float32(1) / np.sqrt((centered * centered).mean(axis=1, dtype=np.float32) + np.float32(eps))).astype(np.float32)
    else:
        mean = np.asarray(mean, dtype=np.float32).copy()
        rstd = np.asarray(rstd, dtype=np.float32).copy()
    n = (xf - mean[:, None]) * rstd[:, None]
    if weight is not None:
        n = n * np.asarray(weight, dtype=np.float32) + np.asarray(bias, dtype=np.float32)
    if is_swish:
        n = _sigmoid(n) * xf
    return round_to(n, dtype), mean, rstd


def e4m3_encode(v):
    """float32 (|v| <= 448) -> float8 e4m3fn byte, round to nearest even."""
    v = np.asarray(v, dtype=np.float32)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    m = np.abs(v).astype(np.float64)
    out = np.zeros(v.shape, dtype=np.uint8)
    sub = m < 2.0 ** -6
    q_sub = np.rint(m / 2.0 ** -9).astype(np.int64)  # 0..8; 8 is the smallest normal, same encoding
    e = np.floor(np.log2(np.where(m > 0, m, 1.0))).astype(np.int64)
    frac = m / np.exp2(e.astype(np.float64)) - 1.0
    q = np.rint(frac * 8.0).astype(np.int64)
    e = np.where(q == 8, e + 1, e)
    q = np.where(q == 8, 0, q)
    code = ((e + 7) << 3) | q
    code = np.minimum(code, 0x7E)  # 448 is the largest finite value
    out = np.where(sub, q_sub, code).astype(np.uint8)
    return (out | sign).astype(np.uint8)


def quantize_fp8_rowwise(values):
    """(scale [rows], e4m3 bytes); kjt_split_per_feature.cpp:492-501."""
    vf = np.asarray(values, dtype=np.float32)
    amax = np.abs(vf).max(axis=1) if vf.shape[1] else np.zeros(vf.shape[0], np.float32)
    scale = (np.maximum(amax, np.float32(1e-12)) / np.float32(448.0)).astype(np.float32)
    q = np.clip(vf / scale[:, None], np.float32(-448.0), np.float32(448.0)).astype(np.float32)
    return scale, e4m3_encode(q)


def layer_norm_mul_quantized(x, u, weight, bias, eps, dtype="float32", silu_u=False, concat_u=False,
                             concat_x=False, mul_u_activation="none"):
    """Returns (combined, mean, rstd, scale, q8); kjt_split_per_feature.cpp:573-599."""
    normalized, mean, rstd = weighted_layer_norm(x, weight, bias, eps, dtype)
    uf = np.asarray(u, dtype=np.float32)

    def silu_t(t):
        return round_to(t * round_to(_sigmoid(t), dtype), dtype)

    if mul_u_activation == "silu":
        gate = silu_t(uf)
    elif mul_u_activation == "sigmoid":
        gate = round_to(_sigmoid(uf), dtype)
    else:
        gate = uf
    multiplied = round_to(normalized * gate, dtype)
    parts = []
    if concat_u:
        parts.append(silu_t(uf) if silu_u else uf)
    if concat_x:
        parts.append(np.asarray(x, dtype=np.float32))
    parts.append(multiplied)
    combined = np.concatenate(parts, axis=1)
    scale, q8 = quantize_fp8_rowwise(combined)
    return combined, mean, rstd, scale, q8


def layer_norm_mul_bwd(dout, x, u, weight, bias, eps, dtype="float32", silu_u=False, concat_u=False,
                       concat_x=False, mul_u_activation="none"):
    """Gradients of ``layerNormMulQuantized``'s saved output (recir/ops/kjt_split_per_feature.cpp:558-600; the
    fp8 copy and its scale carry no gradient) with respect to x, u, weight and bias, i.e. what autograd gives
    through the composite: with n = weighted layer norm of x, m = act(u) and
    combined = [ (silu(u) or u) | x | n * m ] (the first two parts optional),
      dn = d_mult * m,   du = d_mult * n * act'(u)  (+ d_u * (silu'(u) or 1) with concat_u),
      dx = layer-norm backward of dn                (+ d_x with concat_x),   dw, db as for the layer norm.
    float64 arithmetic, every gradient rounded to ``dtype`` once.  Returns (dx, du, dw, db)."""
    xf = np.asarray(x, dtype=np.float64)
    uf = np.asarray(u, dtype=np.float64)
    g = np.asarray(dout, dtype=np.float64)
    cols = xf.shape[1]
    parts = 1 + int(bool(concat_u)) + int(bool(concat_x))
    assert g.shape == (xf.shape[0], parts * cols)
    at = 0
    d_u = d_x = None
    if concat_u:
        d_u, at = g[:, at:at + cols], at + cols
    if concat_x:
        d_x, at = g[:, at:at + cols], at + cols
    d_mult = g[:, at:at + cols]
    mean = xf.mean(axis=1, keepdims=True)
    c = xf - mean
    rstd = 1.0 / np.sqrt((c * c).mean(axis=1, keepdims=True) + float(eps))
    xh = c * rstd
    w = np.asarray(weight, dtype=np.float64)
    n = xh * w + np.asarray(bias, dtype=np.float64)
    s = 1.0 / (1.0 + np.exp(-uf))
    silu_grad = s * (1.0 + uf * (1.0 - s))
    if mul_u_activation == "silu":
        m, dm = uf * s, silu_grad
    elif mul_u_activation == "sigmoid":
        m, dm = s, s * (1.0 - s)
    else:
        m, dm = uf, np.ones_like(uf)
    dn = d_mult * m
    du = d_mult * n * dm
    if d_u is not None:
        du = du + d_u * (silu_grad if silu_u else 1.0)
    dxh = dn * w
    dx = rstd * (dxh - dxh.mean(axis=1, keepdims=True) - xh * (dxh * xh).mean(axis=1, keepdims=True))
    if d_x is not None:
        dx = dx + d_x
    dw = round_to((dn * xh).sum(axis=0).astype(np.float32), dtype)
    db = round_to(dn.sum(axis=0).astype(np.float32), dtype)
    return round_to(dx.astype(np.float32), dtype), round_to(du.astype(np.float32), dtype), dw, db


def e4m3_decode(code):
    """float8 e4m3fn bytes -> float32 (exact)."""
    c = np.asarray(code, dtype=np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    normal = np.exp2((e - 7).astype(np.float64)) * (1.0 + m / 8.0)
    sub = m * 2.0 ** -9
    v = np.where(e == 0, sub, normal)
    v = np.where((c & 0x7F) == 0x7F, np.nan, v)
    return (sign * v).astype(np.float32)


def fp8_rowwise_addmm(a_code, b_code, a_scale, b_scale, bias=None, dtype="float32"):
    """``(a * a_scale[:, None]) @ (b * b_scale[:, None]).T + bias`` for e4m3 bytes ``a`` [M, K], ``b`` [N, K];
    kjt_split_per_feature.cpp:533-556 (dequantise to float32, at::mm, add the bias in float32, cast).
    The sum is taken in float64 here: the float32 summation order of a GEMM is not part of the contract."""
    a = e4m3_decode(a_code) * np.asarray(a_scale, dtype=np.float32)[:, None]
    b = e4m3_decode(b_code) * np.asarray(b_scale, dtype=np.float32)[:, None]
    out = a.astype(np.float64) @ b.astype(np.float64).T
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float32).astype(np.float64)
    return round_to(out.astype(np.float32), dtype)


def jagged_dense_bmm_add(seq_offsets, jagged, dense, bias, elementwise=False, dtype="float32"):
    """``out[rows of b] = jagged[rows of b] @ dense[b] + bias[b]`` (``bias[row]`` when elementwise);
    kjt_split_per_feature.cpp:262-305 (one addmm per sequence, concatenated).  Sums in float64: the
    float32 summation order of a GEMM is not part of the contract."""
    offs = np.asarray(seq_offsets, dtype=np.int64)
    jag = np.asarray(jagged, dtype=np.float32).astype(np.float64)
    den = np.asarray(dense, dtype=np.float32).astype(np.float64)
    bia = np.asarray(bias, dtype=np.float32).astype(np.float64)
    parts = []
    for b in range(den.shape[0]):
        s, e = int(offs[b]), int(offs[b + 1])
        parts.append(jag[s:e] @ den[b] + (bia[s:e] if elementwise else bia[b]))
    out = np.concatenate(parts, 0) if parts else np.zeros((0, den.shape[2]))
    return round_to(out.astype(np.float32), dtype)


def addmm(x, w, bias, dtype="float32"):
    """``at::addmm(bias, x, w)`` (``tritonAddMm``, recir/ops/kjt_split_per_feature.cpp:246-262) for operands
    whose values are representable in ``dtype``: products and sums in float64 (so that only the final
    rounding matters), bias added before the single rounding to ``dtype``."""
    acc = np.asarray(x, dtype=np.float64) @ np.asarray(w, dtype=np.float64) + np.asarray(bias, dtype=np.float64)
    return round_to(acc.astype(np.float32), dtype)


def layer_norm_addmm(x, ln_weight, ln_bias, eps, w, bias, dtype="bfloat16", is_swish=False):
    """The layer norm in front of a projection followed by that projection, as the reference chains them
    (``weightedLayerNorm`` :197-244 returns rows rounded to ``dtype``; ``tritonAddMm`` :246-262 consumes them).
    Returns (out, mean, rstd)."""
    y, mean, rstd = weighted_layer_norm(x, ln_weight, ln_bias, eps, dtype, is_swish=is_swish)
    return addmm(y, w, bias, dtype), mean, rstd


def weighted_layer_norm_bwd(dy, x, weight, bias, eps, dtype="float32", is_swish=False):
    """Gradients of ``weightedLayerNorm`` (recir/ops/kjt_split_per_feature.cpp:220-243) with respect to x,
    weight and bias, i.e. what autograd gives through the composite (which is how the reference
    differentiates it): with xh = (x - mean) * rstd, n = xh * w + b and y = n (or sigmoid(n) * x),
      dn = dy                      (or dy * x * s * (1 - s) with s = sigmoid(n)),
      dw = sum_rows dn * xh,   db = sum_rows dn,
      dxh = dn * w,
      dx = rstd * (dxh - mean_cols(dxh) - xh * mean_cols(dxh * xh))   (+ dy * s for the gated form).
    The composite runs in float32 and casts each gradient to its input's element type once; here the
    arithmetic is float64 and the results are rounded to ``dtype`` once.  Returns (dx, dw, db); dw and db are
    None without weight."""
    xf = np.asarray(x, dtype=np.float64)
    g = np.asarray(dy, dtype=np.float64)
    mean = xf.mean(axis=1, keepdims=True)
    c = xf - mean
    rstd = 1.0 / np.sqrt((c * c).mean(axis=1, keepdims=True) + float(eps))
    xh = c * rstd
    w = None if weight is None else np.asarray(weight, dtype=np.float64)
    n = xh if w is None else xh * w + np.asarray(bias, dtype=np.float64)
    direct = 0.0
    dn = g
    if is_swish:
        s = 1.0 / (1.0 + np.exp(-n))
        dn = g * xf * s * (1.0 - s)
        direct = g * s
    dxh = dn if w is None else dn * w
    dx = rstd * (dxh - dxh.mean(axis=1, keepdims=True) - xh * (dxh * xh).mean(axis=1, keepdims=True)) + direct
    dw = None if w is None else round_to((dn * xh).sum(axis=0).astype(np.float32), dtype)
    db = None if w is None else round_to(dn.sum(axis=0).astype(np.float32), dtype)
    return round_to(dx.astype(np.float32), dtype), dw, db
