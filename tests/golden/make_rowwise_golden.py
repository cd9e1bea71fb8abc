"""Generate ``tests/golden/rowwise_golden.npz`` from the reference's own compiled operators.

Run where the reference tree exists (it builds ``oracle/_ref`` first):

    python tests/golden/make_rowwise_golden.py

Cases call ``generative_recommenders::triton_weighted_layer_norm_fwd`` and
``generative_recommenders::_triton_layer_norm_mul_dropout_quantization_fwd_impl``
(recir/ops/kjt_split_per_feature.cpp:197-244, :558-600) on seeded inputs in float32, bfloat16
and float16.  Everything is stored as float32 (values representable in the case's dtype);
the fp8 copy as its raw e4m3 bytes.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "rowwise_golden.npz")
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def ln_cases():
    """(name, rows, cols, dtype, affine, swish, stats_in)"""
    return [
        ("ln_f32_plain", 5, 16, "float32", False, False, False),
        ("ln_f32_affine", 7, 40, "float32", True, False, False),
        ("ln_f32_swish", 4, 264, "float32", True, True, False),
        ("ln_f32_stats_in", 3, 24, "float32", True, False, True),
        ("ln_bf16_affine", 9, 512, "bfloat16", True, False, False),
        ("ln_bf16_swish", 6, 256, "bfloat16", True, True, False),
        ("ln_f16_swish", 6, 1032, "float16", True, True, False),
        ("ln_bf16_wide", 3, 2048, "bfloat16", True, False, False),
        ("ln_empty", 0, 16, "float32", True, False, False),
    ]


def mul_cases():
    """(name, rows, cols, dtype, silu_u, concat_u, concat_x, act)"""
    return [
        ("mul_f32_none", 5, 16, "float32", False, False, False, "none"),
        ("mul_f32_silu_cat", 4, 40, "float32", True, True, True, "silu"),
        ("mul_f32_sigmoid_catx", 3, 24, "float32", False, False, True, "sigmoid"),
        ("mul_bf16_silu", 8, 512, "bfloat16", False, False, False, "silu"),
        ("mul_bf16_silu_cat", 6, 256, "bfloat16", True, True, True, "silu"),
        ("mul_f16_catu", 5, 1032, "float16", True, True, False, "none"),
        ("mul_bf16_wide", 2, 2048, "bfloat16", False, True, False, "sigmoid"),
    ]


def main():
    build_ref.load()
    gr = torch.ops.generative_recommenders
    out = {}
    g = torch.Generator().manual_seed(7)
    for name, rows, cols, dt, affine, swish, stats_in in ln_cases():
        x = (torch.randn(rows, cols, generator=g) * 1.5 + 0.3).to(DT[dt])
        w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(DT[dt]) if affine else None
        b = (torch.randn(cols, generator=g) * 0.2).to(DT[dt]) if affine else None
        mean = (torch.randn(rows, generator=g) * 0.1) if stats_in else None
        rstd = (torch.rand(rows, generator=g) + 0.5) if stats_in else None
        y, m, r = gr.triton_weighted_layer_norm_fwd(x, w, b, 1e-5, mean, rstd, swish)
        out[f"{name}/x"] = x.float().numpy()
        if affine:
            out[f"{name}/w"], out[f"{name}/b"] = w.float().numpy(), b.float().numpy()
        if stats_in:
            out[f"{name}/mean_in"], out[f"{name}/rstd_in"] = mean.numpy(), rstd.numpy()
        out[f"{name}/y"], out[f"{name}/mean"], out[f"{name}/rstd"] = y.float().numpy(), m.numpy(), r.numpy()
        out[f"{name}/cfg"] = np.array([dt, str(int(affine)), str(int(swish)), str(int(stats_in))])
    for name, rows, cols, dt in (("lnq_f32", 5, 24, "float32"), ("lnq_bf16", 7, 512, "bfloat16"), ("lnq_f16", 4, 264, "float16")):
        x = (torch.randn(rows, cols, generator=g) * 1.5 + 0.3).to(DT[dt])
        w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(DT[dt])
        b = (torch.randn(cols, generator=g) * 0.2).to(DT[dt])
        empty = torch.empty(0)
        y, m, r, scale, q8 = gr._triton_weighted_layer_norm_quantization_fwd_impl(x, w, b, 1e-5, empty, empty, 0)
        out[f"{name}/x"], out[f"{name}/w"], out[f"{name}/b"] = x.float().numpy(), w.float().numpy(), b.float().numpy()
        out[f"{name}/y"], out[f"{name}/mean"], out[f"{name}/rstd"] = y.float().numpy(), m.numpy(), r.numpy()
        out[f"{name}/scale"], out[f"{name}/q8"] = scale.numpy(), q8.view(torch.uint8).numpy()
        out[f"{name}/cfg"] = np.array([dt])
    for name, rows, cols, dt, silu_u, cat_u, cat_x, act in mul_cases():
        x = (torch.randn(rows, cols, generator=g) * 1.5 + 0.3).to(DT[dt])
        u = (torch.randn(rows, cols, generator=g) * 2.0).to(DT[dt])
        w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(DT[dt])
        b = (torch.randn(cols, generator=g) * 0.2).to(DT[dt])
        y, m, r, scale, q8 = gr._triton_layer_norm_mul_dropout_quantization_fwd_impl(
            x, u, w, b, 1e-5, 0.0, False, silu_u, cat_u, cat_x, act, 0, True, 0)
        out[f"{name}/x"], out[f"{name}/u"] = x.float().numpy(), u.float().numpy()
        out[f"{name}/w"], out[f"{name}/b"] = w.float().numpy(), b.float().numpy()
        out[f"{name}/y"], out[f"{name}/mean"], out[f"{name}/rstd"] = y.float().numpy(), m.numpy(), r.numpy()
        out[f"{name}/scale"] = scale.numpy()
        out[f"{name}/q8"] = q8.view(torch.uint8).numpy()
        out[f"{name}/cfg"] = np.array([dt, str(int(silu_u)), str(int(cat_u)), str(int(cat_x)), act])
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(ln_cases())} layer-norm cases, {len(mul_cases())} mul cases")


if __name__ == "__main__":
    main()
