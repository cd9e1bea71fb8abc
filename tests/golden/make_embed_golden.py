"""Generate ``tests/golden/embed_golden.npz`` from the reference's own compiled operator.

Run where the reference tree exists (it builds ``oracle/_ref`` first):

    python tests/golden/make_embed_golden.py

Cases call ``hammer::add_ts_pos_emb_fwd_op`` (recir/ops/kjt_split_per_feature.cpp:307-428) on
seeded inputs; floating-point tensors are stored as float32 (values representable in the case's
dtype), the unsorted per-token indices are recovered from the sorted ones and their permutations.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "embed_golden.npz")
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def cases():
    """(name, lengths, targets|None, cols, dtype, table dtype, P, C, interleave, fn)"""
    return [
        ("f32_log", [5, 9, 3], [1, 2, 0], 16, "float32", "float32", 12, 0, False, "log"),
        ("f32_sqrt_ctx", [7, 4], [2, 1], 8, "float32", "float32", 6, 2, False, "sqrt"),
        ("f32_interleave", [8, 6, 10], [2, 1, 3], 8, "float32", "float32", 20, 1, True, "sqrt"),
        ("f32_no_targets", [6, 1, 4], None, 24, "float32", "float32", 5, 0, False, "log"),
        ("bf16_log", [33, 17, 64], [4, 0, 8], 64, "bfloat16", "bfloat16", 48, 3, False, "log"),
        ("bf16_f32_tables", [20, 12], [3, 3], 32, "bfloat16", "float32", 16, 0, False, "sqrt"),
        ("f16_sqrt", [15, 9, 2], [1, 1, 1], 40, "float16", "float16", 64, 2, False, "sqrt"),
    ]


def main():
    build_ref.load()
    op = torch.ops.hammer.add_ts_pos_emb_fwd_op
    g = torch.Generator().manual_seed(21)
    out = {}
    for name, lengths, targets, cols, dt, tdt, p_rows, c, inter, fn in cases():
        b, t = len(lengths), sum(lengths)
        off = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int64)
        x = torch.randn(t, cols, generator=g).to(DT[dt])
        pos = torch.randn(p_rows, cols, generator=g).to(DT[tdt])
        ts = torch.randn(2049, cols, generator=g).to(DT[tdt])
        s_cols = max(lengths) + 2
        # increasing timestamps with gaps from seconds to months, so that many buckets occur
        gaps = torch.exp(torch.rand(b, s_cols, generator=g) * 14.0).to(torch.int64)
        stamps = torch.cumsum(gaps, dim=1) + 1_600_000_000
        lens = torch.tensor(lengths, dtype=torch.int64)
        tg = None if targets is None else torch.tensor(targets, dtype=torch.int64)
        y, sp, po, st, to = op(x, off, pos, ts, stamps, lens, tg, max(lengths), c, inter, fn)
        pos_idx = torch.empty(t, dtype=torch.int32)
        pos_idx[po.long()] = sp
        ts_idx = torch.empty(t, dtype=torch.int32)
        ts_idx[to.long()] = st
        out[f"{name}/lengths"] = np.array(lengths)
        out[f"{name}/targets"] = np.array([-1] if targets is None else targets)
        out[f"{name}/x"], out[f"{name}/pos"], out[f"{name}/ts"] = x.float().numpy(), pos.float().numpy(), ts.float().numpy()
        out[f"{name}/stamps"] = stamps.numpy()
        out[f"{name}/y"], out[f"{name}/pos_idx"], out[f"{name}/ts_idx"] = y.float().numpy(), pos_idx.numpy(), ts_idx.numpy()
        out[f"{name}/cfg"] = np.array([dt, tdt, str(c), str(int(inter)), fn])
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(cases())} cases")


if __name__ == "__main__":
    main()
