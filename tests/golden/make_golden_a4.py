"""Generate ``tests/golden/hstu_golden_a4.npz`` from the reference's SECOND implementation.

Run where the reference tree exists:

    python tests/golden/make_golden_a4.py

``reference_jagged_hstu_attention`` / ``reference_jagged_hstu_attention_bwd``
(``recir/ops/helion/jagged_hstu_attention.py:211-280``) is the pad-then-compute pure-torch
reference of the reference's in-house kernels: padded einsum, ``silu * attn_scale``, the keep mask
``(m >= n and n < len - num_targets) or m == n`` (``:185-208``), and autograd through all of it
for the gradients.  It shares no code with the compiled operator that produced
``hstu_golden.npz``, so the gradients stored here are an independent pin of the backward.
It covers the causal mask with targets only and needs ``Dv == Dqk``.  The file is loaded by path
with the ``helion`` package (absent here, unused by these two functions) replaced by a stub.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import refroot  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "hstu_golden_a4.npz")


def case_list():
    """(name, lengths, targets|None, attn_scale|None, H, D)"""
    return [
        ("mixed_no_targets", [7, 3, 9], None, None, 2, 8),
        ("mixed_zero_targets", [7, 3, 9], [0, 0, 0], None, 2, 8),
        ("empty_seqs_targets", [0, 6, 2, 0], [0, 2, 1, 0], None, 2, 8),
        ("block_invariance", [5, 9], [1, 3], None, 2, 8),
        ("length_one_many", [1, 1, 1, 1, 1, 1, 1, 1, 2], [0, 1, 0, 1, 0, 0, 1, 0, 1], None, 1, 8),
        ("targets_ge_length", [4, 6, 3], [4, 9, 1], None, 2, 8),
        ("scalar_attn_scale", [7, 9], [1, 2], 0.37, 2, 8),
        ("multi_tile_plain", [140, 129, 128, 1], [17, 0, 128, 0], None, 2, 16),
        ("multi_tile_targets", [150, 70, 33, 260], [10, 70, 0, 64], 0.011, 3, 16),
    ] + [(f"residue_{r}", [r, 5], [0, 2], None, 2, 8) for r in range(8)]


def main():
    ref = refroot.load_reference_module("recir/ops/helion/jagged_hstu_attention.py", "ref_helion_hstu",
                                        stub_modules=("helion", "helion.language"))
    out, names = {}, []
    for idx, (name, lengths, targets, scale, H, D) in enumerate(case_list()):
        g = torch.Generator().manual_seed(7000 + idx)
        T = int(sum(lengths))
        q, k, v, do = (torch.randn(T, H, D, generator=g) for _ in range(4))
        offs = torch.zeros(len(lengths) + 1, dtype=torch.int64)
        offs[1:] = torch.cumsum(torch.tensor(lengths, dtype=torch.int64), 0)
        nt = None if targets is None else torch.tensor(targets, dtype=torch.int64)
        N = max(max(lengths), 1) + 3
        alpha = 1.0 / (D ** 0.5)
        sc = (1.0 / N) if scale is None else scale
        o = ref.reference_jagged_hstu_attention(N, alpha, sc, q, k, v, offs, nt)
        dq, dk, dv = ref.reference_jagged_hstu_attention_bwd(do, q, k, v, offs, nt, sc, N, alpha)
        names.append(name)
        p = name + "/"
        out[p + "q"], out[p + "k"], out[p + "v"], out[p + "do"] = (x.numpy() for x in (q, k, v, do))
        out[p + "offsets"] = offs.numpy()
        out[p + "num_targets"] = np.array([]) if nt is None else nt.numpy()
        out[p + "has_targets"] = np.array(nt is not None)
        out[p + "attn_scale"] = np.array([]) if scale is None else np.array(scale, dtype=np.float32)
        out[p + "has_scale"] = np.array(scale is not None)
        out[p + "params"] = np.array([N, 1, 0, 0, 0], dtype=np.int64)
        out[p + "alpha"] = np.array(alpha)
        out[p + "o"], out[p + "dq"], out[p + "dk"], out[p + "dv"] = (x.detach().numpy() for x in (o, dq, dk, dv))
    out["names"] = np.array(names)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(names)} cases, {os.path.getsize(OUT) / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
