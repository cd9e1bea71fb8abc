"""Generate ``tests/golden/fp8_addmm_golden.npz`` from the reference's own compiled operator.

Run where the reference tree exists (it builds ``oracle/_ref`` first):

    python tests/golden/make_fp8_addmm_golden.py

Cases call ``generative_recommenders::_triton_fp8_rowwise_addmm_fwd_impl``
(recir/ops/kjt_split_per_feature.cpp:533-556) on seeded float8 e4m3 operands with one float32 scale per
row.  Operands are stored as raw e4m3 bytes, everything else as float32.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fp8_addmm_golden.npz")
CASES = (  # name, M, N, K, output dtype, bias
    ("f32_bias", 9, 32, 64, torch.float32, True),
    ("f32_plain", 5, 16, 48, torch.float32, False),
    ("bf16_bias", 33, 48, 512, torch.bfloat16, True),
    ("f16_plain", 4, 64, 128, torch.float16, False),
)


def main():
    build_ref.load()
    gr = torch.ops.generative_recommenders
    g = torch.Generator().manual_seed(11)
    out = {"names": np.array([c[0] for c in CASES])}
    for name, M, N, K, dt, has_bias in CASES:
        a = (torch.randn(M, K, generator=g) * 60.0).clamp(-448, 448).to(torch.float8_e4m3fn)
        b = (torch.randn(N, K, generator=g) * 60.0).clamp(-448, 448).to(torch.float8_e4m3fn)
        sa = torch.rand(M, generator=g) * 0.02 + 0.001
        sb = torch.rand(N, generator=g) * 0.02 + 0.001
        bias = (torch.randn(N, generator=g) * 0.5).to(dt) if has_bias else torch.empty(0)
        y = gr._triton_fp8_rowwise_addmm_fwd_impl(a, b, sa, sb, bias, has_bias, False, dt, False, False)
        out[f"{name}/a"], out[f"{name}/b"] = a.view(torch.uint8).numpy(), b.view(torch.uint8).numpy()
        out[f"{name}/a_scale"], out[f"{name}/b_scale"] = sa.numpy(), sb.numpy()
        if has_bias:
            out[f"{name}/bias"] = bias.float().numpy()
        out[f"{name}/y"] = y.float().numpy()
        out[f"{name}/cfg"] = np.array([str(dt).replace("torch.", ""), str(int(has_bias))])
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(CASES)} cases")


if __name__ == "__main__":
    main()
