"""Shared helpers for the test-suite: golden-vector access and error metrics."""
from __future__ import annotations

import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# "main": outputs of the reference's compiled operator (tests/golden/make_golden.py);
# "a4": outputs of the reference's second, pure-torch pad-then-compute implementation and of
# autograd through it (tests/golden/make_golden_a4.py), causal mask with targets only.
GOLDEN_FILES = {"main": "hstu_golden.npz", "a4": "hstu_golden_a4.npz"}
_cache = {}


def golden(which: str = "main"):
    if which not in _cache:
        _cache[which] = np.load(os.path.join(GOLDEN_DIR, GOLDEN_FILES[which]))
    return _cache[which]


def golden_names(which: str = "main"):
    return [str(n) for n in golden(which)["names"]]


def golden_case(name: str, which: str = "main") -> dict:
    z = golden(which)
    p = name + "/"
    N, causal, w, ctx, f = (int(x) for x in z[p + "params"])
    c = dict(
        q=z[p + "q"], k=z[p + "k"], v=z[p + "v"], do=z[p + "do"], offsets=z[p + "offsets"],
        num_targets=z[p + "num_targets"] if bool(z[p + "has_targets"]) else None,
        attn_scale=z[p + "attn_scale"] if bool(z[p + "has_scale"]) else None,
        max_seq_len=N, causal=bool(causal), max_attn_len=w, contextual_seq_len=ctx,
        full_attn_size=f, alpha=float(z[p + "alpha"]),
        o=z[p + "o"], dq=z[p + "dq"], dk=z[p + "dk"], dv=z[p + "dv"],
    )
    return c


def case_kwargs(c: dict) -> dict:
    return dict(max_seq_len=c["max_seq_len"], alpha=c["alpha"], causal=c["causal"],
                num_targets=c["num_targets"], attn_scale=c["attn_scale"],
                max_attn_len=c["max_attn_len"], contextual_seq_len=c["contextual_seq_len"],
                full_attn_size=c["full_attn_size"])


def rel_l2(a, b) -> float:
    a = torch.as_tensor(np.asarray(a)).double() if not torch.is_tensor(a) else a.double().cpu()
    b = torch.as_tensor(np.asarray(b)).double() if not torch.is_tensor(b) else b.double().cpu()
    den = float(b.norm())
    if den == 0.0:
        return float(a.norm())
    return float((a - b).norm()) / den


def max_abs(a, b) -> float:
    a = torch.as_tensor(np.asarray(a)).double() if not torch.is_tensor(a) else a.double().cpu()
    b = torch.as_tensor(np.asarray(b)).double() if not torch.is_tensor(b) else b.double().cpu()
    if a.numel() == 0:
        return 0.0
    return float((a - b).abs().max())
