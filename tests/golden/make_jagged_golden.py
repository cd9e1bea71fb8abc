"""Generate ``tests/golden/jagged_golden.npz`` from the reference's own Python operators.

Run where the reference tree exists:

    python tests/golden/make_jagged_golden.py

The reference file ``recir/ops/jagged_ops.py`` is a leaf module (it imports only torch), so it is
loaded by path; the cases call its ``recir::jagged_to_padded_dense``, ``recir::dense_to_jagged``,
``recir::concat_2d_jagged`` and ``recir::split_2d_jagged`` operators on CPU tensors (float32
payloads holding small integers, so any element type reproduces them exactly).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle import refroot  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "jagged_golden.npz")


def main():
    refroot.load_reference_module("recir/ops/jagged_ops.py", "ref_jagged_ops")
    ops = torch.ops.recir
    g = torch.Generator().manual_seed(5)
    out = {}

    def vals(rows, d):
        return torch.randint(-50, 50, (rows, d), generator=g).float()

    # jagged <-> dense: (lengths, N, D, total_L override)
    jd = {
        "mixed": ([3, 0, 5, 2], 6, 8, None),
        "truncating": ([7, 2, 9], 4, 8, None),      # sequences longer than the padded width
        "single": ([5], 8, 16, None),
        "padded_total": ([2, 3], 4, 8, 9),           # total_L beyond the last offset
        "full": ([4, 4, 4], 4, 8, None),            # fully padded fast path
        "odd_width": ([3, 1, 4], 5, 6, None),       # rows of 12 / 24 bytes: the 2-byte copy path
    }
    for name, (lengths, n, d, total) in jd.items():
        off = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int64)
        v = vals(int(off[-1]), d)
        dense = ops.jagged_to_padded_dense(v, [off], [n], -7.0)
        back, _ = ops.dense_to_jagged(vals(len(lengths) * n, d).reshape(len(lengths), n, d), [off], total)
        out[f"jd_{name}/lengths"], out[f"jd_{name}/n"] = np.array(lengths), np.array(n)
        out[f"jd_{name}/total"] = np.array(-1 if total is None else total)
        out[f"jd_{name}/values"], out[f"jd_{name}/dense_out"] = v.numpy(), dense.numpy()
        g2 = torch.Generator().manual_seed(len(name))
        src = torch.randint(-50, 50, (len(lengths), n, d), generator=g2).float()
        j, _ = ops.dense_to_jagged(src, [off], total)
        out[f"jd_{name}/dense_in"], out[f"jd_{name}/jagged_out"] = src.numpy(), j.numpy()
    # concat / split: (lengths_left, lengths_right, D)
    cs = {
        "mixed": ([3, 0, 5, 2], [1, 4, 0, 2], 8),
        "targets": ([9, 17, 5], [2, 2, 2], 16),
        "empty_right": ([3, 2], [0, 0], 8),
        "empty_left": ([0, 0, 0], [2, 1, 3], 8),
        "odd_width": ([2, 3], [1, 1], 6),
    }
    for name, (ll, lr, d) in cs.items():
        ol = torch.tensor([0] + list(np.cumsum(ll)), dtype=torch.int64)
        orr = torch.tensor([0] + list(np.cumsum(lr)), dtype=torch.int64)
        vl, vr = vals(int(ol[-1]), d), vals(int(orr[-1]), d)
        cat = ops.concat_2d_jagged(vl, ol, vr, orr)
        left, right = ops.split_2d_jagged(cat, ol, orr, int(ol[-1]), int(orr[-1]))
        out[f"cs_{name}/ll"], out[f"cs_{name}/lr"] = np.array(ll), np.array(lr)
        out[f"cs_{name}/vl"], out[f"cs_{name}/vr"] = vl.numpy(), vr.numpy()
        out[f"cs_{name}/cat"], out[f"cs_{name}/left"], out[f"cs_{name}/right"] = cat.numpy(), left.numpy(), right.numpy()
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(jd)} jagged/dense cases, {len(cs)} concat/split cases")


if __name__ == "__main__":
    main()
