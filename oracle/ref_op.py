"""Thin wrapper over the reference's own compiled operator (``oracle/_ref``).

TEST INFRASTRUCTURE ONLY.  Calls ``torch.ops.hammer.triton_ragged_attention_fwd``
(schema ``recir/ops/kjt_split_per_feature.cpp:780-783``); the backward is
autograd through that composite, which is how the reference itself
differentiates it (``CompositeImplicitAutograd``, ``:786-793``).
"""
from __future__ import annotations

import torch

from . import build_ref

_loaded = False


def available() -> bool:
    return build_ref.ref_available()


def _ensure():
    global _loaded
    if not _loaded:
        build_ref.load()
        _loaded = True


def ref_fwd(q, k, v, seq_offsets, max_seq_len, alpha, causal=True, num_targets=None,
            attn_scale=None, max_attn_len=0, contextual_seq_len=0, full_attn_size=0):
    _ensure()
    out, _aux = torch.ops.hammer.triton_ragged_attention_fwd(
        int(max_seq_len), float(alpha), q, k, v, seq_offsets,
        "lower_triangular" if causal else "none", num_targets, attn_scale,
        int(max_attn_len), int(contextual_seq_len), int(full_attn_size), 0)
    return out


def ref_fwd_bwd(dout, q, k, v, seq_offsets, max_seq_len, alpha, causal=True, num_targets=None,
                attn_scale=None, max_attn_len=0, contextual_seq_len=0, full_attn_size=0):
    """Returns (o, dq, dk, dv) from the reference operator and autograd through it."""
    q_ = q.detach().clone().requires_grad_(True)
    k_ = k.detach().clone().requires_grad_(True)
    v_ = v.detach().clone().requires_grad_(True)
    o = ref_fwd(q_, k_, v_, seq_offsets, max_seq_len, alpha, causal, num_targets, attn_scale,
                max_attn_len, contextual_seq_len, full_attn_size)
    o.backward(dout)
    return o.detach(), q_.grad, k_.grad, v_.grad


def ref_fwd_bwd_per_sequence(dout, q, k, v, seq_offsets, max_seq_len, alpha, causal=True,
                             num_targets=None, attn_scale=None, max_attn_len=0,
                             contextual_seq_len=0, full_attn_size=0, backward=True,
                             select=None):
    """Same arithmetic, one sequence per call, so temporaries stay ``O(H L^2)`` of one sequence.

    ``select`` optionally restricts the run to a list of sequence indices (used
    by the bounded CPU-baseline sample); rows of other sequences stay zero.
    """
    offs = seq_offsets.tolist()
    # the composite is pure ATen: it runs wherever its inputs live (host, or a GPU for full-size checks)
    o = torch.zeros(q.shape[0], q.shape[1], v.shape[2], dtype=v.dtype, device=v.device)
    dq = torch.zeros_like(q) if backward else None
    dk = torch.zeros_like(k) if backward else None
    dv = torch.zeros_like(v) if backward else None
    idx = range(len(offs) - 1) if select is None else select
    for b in idx:
        s, e = offs[b], offs[b + 1]
        if e == s:
            continue
        local = torch.tensor([0, e - s], dtype=seq_offsets.dtype)
        nt = None if num_targets is None else num_targets[b:b + 1].cpu()
        sc = attn_scale
        if sc is not None and sc.dim() > 0:
            sc = sc[s:e]
        if backward:
            ob, a, b_, c = ref_fwd_bwd(dout[s:e], q[s:e], k[s:e], v[s:e], local, max_seq_len,
                                       alpha, causal, nt, sc, max_attn_len,
                                       contextual_seq_len, full_attn_size)
            dq[s:e], dk[s:e], dv[s:e] = a, b_, c
        else:
            ob = ref_fwd(q[s:e], k[s:e], v[s:e], local, max_seq_len, alpha, causal, nt, sc,
                         max_attn_len, contextual_seq_len, full_attn_size)
        o[s:e] = ob
    return o, dq, dk, dv
