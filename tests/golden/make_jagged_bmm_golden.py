"""Generate ``tests/golden/jagged_bmm_golden.npz`` from the reference's own compiled operator.

Run where the reference tree exists (it builds ``oracle/_ref`` first):

    python tests/golden/make_jagged_bmm_golden.py

Cases call ``generative_recommenders::triton_jagged_dense_bmm_add_fwd``
(recir/ops/kjt_split_per_feature.cpp:262-305) on seeded inputs, with a bias per sequence and a bias per
row, in float32 and bfloat16, with empty sequences in the batch.  Everything is stored as float32.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "jagged_bmm_golden.npz")
CASES = (  # name, lengths, K, N, dtype, elementwise
    ("f32_seq_bias", [3, 0, 5, 1], 16, 24, torch.float32, False),
    ("f32_row_bias", [2, 4], 8, 8, torch.float32, True),
    ("bf16_seq_bias", [7, 0, 33, 1, 12], 64, 32, torch.bfloat16, False),
    ("bf16_row_bias", [5, 20, 0, 9], 32, 48, torch.bfloat16, True),
)


def main():
    build_ref.load()
    gr = torch.ops.generative_recommenders
    g = torch.Generator().manual_seed(13)
    out = {"names": np.array([c[0] for c in CASES])}
    for name, lengths, K, N, dt, elementwise in CASES:
        offs = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int64)
        T, B = int(offs[-1]), len(lengths)
        jag = torch.randn(T, K, generator=g).to(dt)
        den = (torch.randn(B, K, N, generator=g) * 0.3).to(dt)
        bias = torch.randn((T if elementwise else B), N, generator=g).to(dt)
        y, b_, k_, n_ = gr.triton_jagged_dense_bmm_add_fwd(max(lengths), offs, jag, den, bias, elementwise)
        assert (b_, k_, n_) == (B, K, N)
        out[f"{name}/offsets"] = offs.numpy()
        out[f"{name}/jagged"], out[f"{name}/dense"] = jag.float().numpy(), den.float().numpy()
        out[f"{name}/bias"], out[f"{name}/y"] = bias.float().numpy(), y.float().numpy()
        out[f"{name}/cfg"] = np.array([str(dt).replace("torch.", ""), str(int(elementwise))])
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(CASES)} cases")


if __name__ == "__main__":
    main()
