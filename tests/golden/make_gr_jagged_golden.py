"""Generate ``tests/golden/gr_jagged_golden.npz`` from the reference's own compiled operators.

Run where the reference tree exists (it builds ``oracle/_ref`` first):

    python tests/golden/make_gr_jagged_golden.py

Cases call ``generative_recommenders::concat_2D_jagged_fwd_op`` and ``split_2D_jagged_fwd_op``
(recir/ops/kjt_split_per_feature.cpp:100-196, :430-489): two jagged sides, a dense side on the left or on
the right, a prefix of the right side moved to the front, and the replace form.  float32 values.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gr_jagged_golden.npz")
CASES = (  # name, lengths_a or dense L (int), lengths_b or dense L, is_replace, prefix
    ("jj", [3, 0, 5, 2], [1, 4, 0, 2], False, 0),
    ("jj_prefix", [3, 0, 5, 2], [2, 4, 3, 2], False, 2),
    ("dense_a", 3, [1, 0, 4], False, 0),
    ("dense_b", [2, 5, 0], 2, False, 0),
    ("replace", [4, 6, 2], [1, 3, 2], True, 0),
    ("replace_dense_a", 5, [1, 0, 5], True, 0),
)


def main():
    build_ref.load()
    gr = torch.ops.generative_recommenders
    g = torch.Generator().manual_seed(17)
    D = 8
    out = {"names": np.array([c[0] for c in CASES])}
    for name, la, lb, replace, p in CASES:
        batch = len(la) if isinstance(la, list) else len(lb)

        def side(l):
            if isinstance(l, list):
                off = torch.tensor([0] + list(np.cumsum(l)), dtype=torch.int64)
                return torch.randn(int(off[-1]), D, generator=g), off
            return torch.randn(batch, l, D, generator=g), None

        va, oa = side(la)
        vb, ob = side(lb)
        cat = gr.concat_2D_jagged_fwd_op(16, va, vb, oa, ob, replace, p)
        out[f"{name}/a"], out[f"{name}/b"], out[f"{name}/cat"] = va.numpy(), vb.numpy(), cat.numpy()
        out[f"{name}/offsets_a"] = oa.numpy() if oa is not None else np.zeros(0, np.int64)
        out[f"{name}/offsets_b"] = ob.numpy() if ob is not None else np.zeros(0, np.int64)
        out[f"{name}/cfg"] = np.array([int(oa is None), int(ob is None), int(replace), p, batch,
                                       la if oa is None else (lb if ob is None else 0)])
        if not replace:
            dummy = torch.zeros(batch + 1, dtype=torch.int64)
            sa, sb = gr.split_2D_jagged_fwd_op(
                cat, 16, oa if oa is not None else dummy, ob if ob is not None else dummy,
                0 if oa is None else int(oa[-1]), 0 if ob is None else int(ob[-1]), oa is None, ob is None,
                la if oa is None else (lb if ob is None else 0), p, batch)
            assert torch.equal(sa, va) and torch.equal(sb, vb)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(CASES)} cases")


if __name__ == "__main__":
    main()
