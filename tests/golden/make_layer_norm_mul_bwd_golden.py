"""Generate ``tests/golden/layer_norm_mul_bwd_golden.npz``: gradients of the reference's gate stage.

Run where the reference tree exists (``oracle/_ref`` must have been built):

    python tests/golden/make_layer_norm_mul_bwd_golden.py

The reference has no backward operator for ``layerNormMulQuantized``
(recir/ops/kjt_split_per_feature.cpp:558-600): the composite is differentiated by autograd, and that is what runs
here -- ``generative_recommenders::_triton_layer_norm_mul_dropout_quantization_fwd_impl`` with ``save_y`` on
seeded inputs that require gradients, ``y.backward(dout)``, the gradients of x, u, weight and bias stored as
float32.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "layer_norm_mul_bwd_golden.npz")
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def cases():
    """(name, rows, cols, dtype, silu_u, concat_u, concat_x, activation)"""
    return [
        ("f32_none", 6, 16, "float32", False, False, False, "none"),
        ("f32_silu", 29, 40, "float32", False, False, False, "silu"),
        ("f32_sigmoid_cat", 11, 72, "float32", True, True, True, "sigmoid"),
        ("bf16_silu", 66, 512, "bfloat16", False, False, False, "silu"),
        ("bf16_silu_cat_u", 36, 256, "bfloat16", True, True, False, "silu"),
        ("f16_none_cat_x", 17, 1024, "float16", False, False, True, "none"),
        ("bf16_sigmoid_cat_ux", 40, 64, "bfloat16", False, True, True, "sigmoid"),
    ]


def main():
    build_ref.load()
    gr = torch.ops.generative_recommenders
    out = {}
    g = torch.Generator().manual_seed(23)
    for name, rows, cols, dt, silu_u, concat_u, concat_x, act in cases():
        t = DT[dt]
        x = (torch.randn(rows, cols, generator=g) * 1.5 + 0.3).to(t).requires_grad_(True)
        u = torch.randn(rows, cols, generator=g).to(t).requires_grad_(True)
        w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(t).requires_grad_(True)
        b = (torch.randn(cols, generator=g) * 0.2).to(t).requires_grad_(True)
        parts = 1 + int(concat_u) + int(concat_x)
        dout = torch.randn(rows, parts * cols, generator=g).to(t)
        y = gr._triton_layer_norm_mul_dropout_quantization_fwd_impl(
            x, u, w, b, 1e-5, 0.0, False, silu_u, concat_u, concat_x, act, 0, True, 64)[0]
        y.backward(dout)
        for key, val in (("x", x.detach()), ("u", u.detach()), ("w", w.detach()), ("b", b.detach()), ("dout", dout),
                         ("dx", x.grad), ("du", u.grad), ("dw", w.grad), ("db", b.grad)):
            out[f"{name}/{key}"] = val.float().numpy()
        out[f"{name}/cfg"] = np.array([dt, str(int(silu_u)), str(int(concat_u)), str(int(concat_x)), act])
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(cases())} cases, {os.path.getsize(OUT) / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
