"""Generate ``tests/golden/hstu_golden.npz`` from the reference's own compiled operator.

Run where the reference tree exists (it builds ``oracle/_ref`` first):

    python tests/golden/make_golden.py

Each case stores its inputs and the outputs ``o, dq, dk, dv`` of
``hammer::triton_ragged_attention_fwd`` (``recir/ops/kjt_split_per_feature.cpp:602-693``)
and of autograd through it, all in float32.  The case list restates the case
lists of the reference's kernel tests
(``recir/ops/pallas/tests/test_jagged_hstu_attention.py:121-272``: mixed lengths,
empty sequences, every start-offset residue mod 8, many length-1 sequences) and
adds one case per mask feature of ``kjt_split_per_feature.cpp:639-685``.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import build_ref, ref_op  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "hstu_golden.npz")


def case_list():
    """(name, lengths, targets|None, kwargs, H, D, tail_rows)"""
    cases = [
        ("mixed_no_targets", [7, 3, 9], None, {}, 2, 8, 0),
        ("mixed_zero_targets", [7, 3, 9], [0, 0, 0], {}, 2, 8, 0),
        ("empty_seqs_targets", [0, 6, 2, 0], [0, 2, 1, 0], {}, 2, 8, 0),
        ("block_invariance", [5, 9], [1, 3], {}, 2, 8, 0),
        ("length_one_many", [1, 1, 1, 1, 1, 1, 1, 1, 2], [0, 1, 0, 1, 0, 0, 1, 0, 1], {}, 1, 8, 0),
        ("dqk_ne_dv", [6, 4], [2, 1], {"dv": 16}, 2, 8, 0),
        ("window", [12, 20], None, {"max_attn_len": 4}, 2, 8, 0),
        ("window_targets", [12, 20], [3, 5], {"max_attn_len": 4}, 2, 8, 0),
        ("window_ctx", [12, 20], [3, 5], {"max_attn_len": 4, "contextual_seq_len": 3}, 2, 8, 0),
        ("ctx_only", [9, 5], [2, 0], {"contextual_seq_len": 2}, 2, 8, 0),
        ("window_full_tail", [16, 24], [3, 4], {"max_attn_len": 3, "full_attn_size": 5}, 2, 8, 0),
        ("window_full_tail_ctx", [16, 24], [3, 4],
         {"max_attn_len": 3, "full_attn_size": 5, "contextual_seq_len": 1}, 2, 8, 0),
        ("noncausal_window", [10, 7], [2, 1], {"causal": False, "max_attn_len": 3}, 2, 8, 0),
        ("noncausal_plain", [10, 7], None, {"causal": False}, 2, 8, 0),
        ("targets_ge_length", [4, 6, 3], [4, 9, 1], {}, 2, 8, 0),
        ("all_targets_ctx", [4, 6], [4, 2], {"contextual_seq_len": 1}, 2, 8, 0),
        ("scalar_attn_scale", [7, 9], [1, 2], {"attn_scale": "scalar"}, 2, 8, 0),
        ("token_attn_scale", [7, 9], [1, 2], {"attn_scale": "token"}, 2, 8, 0),
        ("tail_rows", [5, 6], [1, 1], {}, 2, 8, 3),
        ("multi_tile", [150, 70, 33], [10, 70, 0], {"max_attn_len": 40, "contextual_seq_len": 2}, 2, 16, 0),
        ("multi_tile_plain", [140, 129, 128, 1], [17, 0, 128, 0], {}, 2, 16, 0),
    ]
    for r in range(8):
        cases.append((f"residue_{r}", [r, 5], [0, 2], {}, 2, 8, 0))
    return cases


def make_inputs(idx, lengths, targets, kw, H, D, tail):
    g = torch.Generator().manual_seed(1000 + idx)
    T = int(sum(lengths)) + tail
    dv = kw.get("dv", D)
    q = torch.randn(T, H, D, generator=g)
    k = torch.randn(T, H, D, generator=g)
    v = torch.randn(T, H, dv, generator=g)
    do = torch.randn(T, H, dv, generator=g)
    offs = torch.zeros(len(lengths) + 1, dtype=torch.int64)
    offs[1:] = torch.cumsum(torch.tensor(lengths, dtype=torch.int64), 0)
    nt = None if targets is None else torch.tensor(targets, dtype=torch.int64)
    scale = None
    if kw.get("attn_scale") == "scalar":
        scale = torch.tensor(0.37)
    elif kw.get("attn_scale") == "token":
        scale = torch.rand(T, generator=g) + 0.25
    return q, k, v, do, offs, nt, scale


def main():
    build_ref.build()
    out = {}
    names = []
    for idx, (name, lengths, targets, kw, H, D, tail) in enumerate(case_list()):
        q, k, v, do, offs, nt, scale = make_inputs(idx, lengths, targets, kw, H, D, tail)
        n_valid = int(offs[-1])
        N = max(max(lengths), 1) + 3
        alpha = 1.0 / (D ** 0.5)
        args = dict(causal=kw.get("causal", True), num_targets=nt, attn_scale=scale,
                    max_attn_len=kw.get("max_attn_len", 0),
                    contextual_seq_len=kw.get("contextual_seq_len", 0),
                    full_attn_size=kw.get("full_attn_size", 0))
        # the reference concatenates per-sequence outputs, so feed it the valid rows only
        sc_valid = scale[:n_valid] if (scale is not None and scale.dim() > 0) else scale
        a = dict(args, attn_scale=sc_valid)
        o, dq, dk, dv_ = ref_op.ref_fwd_bwd(do[:n_valid], q[:n_valid], k[:n_valid], v[:n_valid],
                                            offs, N, alpha, **a)
        names.append(name)
        p = name + "/"
        out[p + "q"], out[p + "k"], out[p + "v"], out[p + "do"] = (x.numpy() for x in (q, k, v, do))
        out[p + "offsets"] = offs.numpy()
        out[p + "num_targets"] = np.array([]) if nt is None else nt.numpy()
        out[p + "has_targets"] = np.array(nt is not None)
        out[p + "attn_scale"] = np.array([]) if scale is None else scale.numpy()
        out[p + "has_scale"] = np.array(scale is not None)
        out[p + "params"] = np.array([N, int(args["causal"]), args["max_attn_len"],
                                      args["contextual_seq_len"], args["full_attn_size"]],
                                     dtype=np.int64)
        out[p + "alpha"] = np.array(alpha)
        out[p + "o"], out[p + "dq"], out[p + "dk"], out[p + "dv"] = (
            x.numpy() for x in (o, dq, dk, dv_))
    out["names"] = np.array(names)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(names)} cases, {os.path.getsize(OUT)/1024:.1f} KiB")


if __name__ == "__main__":
    main()
