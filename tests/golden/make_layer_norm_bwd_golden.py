"""Generate ``tests/golden/layer_norm_bwd_golden.npz``: gradients of the reference's layer norm.

Run where the reference tree exists (``oracle/_ref`` must have been built):

    python tests/golden/make_layer_norm_bwd_golden.py

The reference has no backward operator for ``weightedLayerNorm``
(recir/ops/kjt_split_per_feature.cpp:197-244): the composite is differentiated by autograd, and that is what
runs here -- ``generative_recommenders::triton_weighted_layer_norm_fwd`` on seeded inputs that require
gradients, ``y.backward(dy)``, the gradients of x, weight and bias stored as float32.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "layer_norm_bwd_golden.npz")
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def cases():
    """(name, rows, cols, dtype, affine, swish)"""
    return [
        ("f32_plain", 5, 16, "float32", False, False),
        ("f32_affine", 37, 40, "float32", True, False),
        ("f32_swish", 14, 264, "float32", True, True),
        ("bf16_affine", 140, 512, "bfloat16", True, False),
        ("bf16_swish", 130, 256, "bfloat16", True, True),
        ("f16_swish", 33, 1024, "float16", True, True),
        ("bf16_plain", 9, 64, "bfloat16", False, False),
    ]


def main():
    build_ref.load()
    gr = torch.ops.generative_recommenders
    out = {}
    g = torch.Generator().manual_seed(11)
    for name, rows, cols, dt, affine, swish in cases():
        x = (torch.randn(rows, cols, generator=g) * 1.5 + 0.3).to(DT[dt]).requires_grad_(True)
        w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(DT[dt]).requires_grad_(True) if affine else None
        b = (torch.randn(cols, generator=g) * 0.2).to(DT[dt]).requires_grad_(True) if affine else None
        dy = torch.randn(rows, cols, generator=g).to(DT[dt])
        y, _m, _r = gr.triton_weighted_layer_norm_fwd(x, w, b, 1e-5, None, None, swish)
        y.backward(dy)
        out[f"{name}/x"], out[f"{name}/dy"] = x.detach().float().numpy(), dy.float().numpy()
        out[f"{name}/dx"] = x.grad.float().numpy()
        if affine:
            out[f"{name}/w"], out[f"{name}/b"] = w.detach().float().numpy(), b.detach().float().numpy()
            out[f"{name}/dw"], out[f"{name}/db"] = w.grad.float().numpy(), b.grad.float().numpy()
        out[f"{name}/cfg"] = np.array([dt, str(int(affine)), str(int(swish))])
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(cases())} cases, {os.path.getsize(OUT) / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
