"""Numpy restatement of the reference HSTU jagged attention (forward and backward).

TEST INFRASTRUCTURE ONLY: this module is the checker, never the thing shipped
or measured as the product.

What it restates (paths relative to the reference project root):

* forward  -- ``raggedAttention`` in ``recir/ops/kjt_split_per_feature.cpp:602-693``:
  per sequence and head ``S = alpha * Q K^T``, ``P = S * sigmoid(S)``, scaled by
  ``attn_scale`` (0-d, or one value per query token, ``:677-682``) or divided by
  ``max_seq_len`` (``:684``), multiplied by the boolean keep mask, ``O = P V``.
* mask     -- ``:639-674`` of the same file (``keep_mask`` below follows it
  statement by statement, including its quirks: the contextual flag only makes
  key 0 visible; a non-causal call without a window keeps the diagonal only).
* backward -- the closed forms listed in
  ``recir/ops/helion/jagged_hstu_attention.py:16-27``:
  ``dP = dO V^T``, ``dV = (keep*silu(S)*sc)^T dO``,
  ``dS = dP*keep*sc*silu'(S)``, ``dQ = alpha dS K``, ``dK = alpha dS^T Q``.

Pinning: ``tests/test_oracle.py`` checks this file against the golden vectors in
``tests/golden/`` (produced by running the reference's own compiled operator,
see ``tests/golden/make_golden.py``), against the reference's known-answer test
(``recir/ops/tests/KjtSplitPerFeatureTest.cpp:237-261``) and, when the compiled
reference is present, against it directly on fresh random inputs.
"""
from __future__ import annotations

import numpy as np


def keep_mask(
    length: int,
    num_targets: int | None,
    causal: bool = True,
    max_attn_len: int = 0,
    contextual_seq_len: int = 0,
    full_attn_size: int = 0,
) -> np.ndarray:
    """Boolean ``[L, L]`` keep mask, rows = queries, columns = keys.

    Follows ``kjt_split_per_feature.cpp:639-674`` line by line.
    """
    ids = np.arange(length, dtype=np.int64)
    mask_ids = ids
    target_count = 0
    if num_targets is not None:
        target_count = int(num_targets)
        mask_ids = np.minimum(ids, length - target_count)
    rows = mask_ids[:, None]
    cols = mask_ids[None, :]
    dist = rows - cols
    mask = np.eye(length, dtype=bool)
    if not causal:
        dist = np.abs(dist)
    if max_attn_len > 0:
        if causal:
            mask |= (dist > 0) & (dist <= max_attn_len)
        else:
            mask |= (dist >= -max_attn_len) & (dist <= max_attn_len)
        if full_attn_size > 0:
            boundary = length - target_count - full_attn_size
            g_rows = np.where(rows < boundary, 0, rows)
            g_cols = np.where(cols < boundary, 0, cols)
            mask |= (g_rows - g_cols) > 0
    elif causal:
        mask |= dist > 0
    if contextual_seq_len > 0:
        mask |= np.broadcast_to(cols == 0, mask.shape)
    return mask


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return 1.0 / (1.0 + np.exp(-x))


def _scale_for(attn_scale, max_seq_len, start, end, dtype):
    """Per-query scale ``[L,1]`` (or scalar) as the reference picks it (``:677-685``)."""
    if attn_scale is None:
        return dtype(1.0) / dtype(max_seq_len)
    a = np.asarray(attn_scale, dtype=dtype)
    if a.ndim == 0:
        return a
    return a[start:end].reshape(1, -1, 1)


def hstu_attention_fwd(
    q, k, v, seq_offsets, max_seq_len, alpha, causal=True, num_targets=None,
    attn_scale=None, max_attn_len=0, contextual_seq_len=0, full_attn_size=0,
    dtype=np.float64,
):
    """Forward.  q,k ``[T,H,Dqk]``, v ``[T,H,Dv]`` -> o ``[T,H,Dv]`` (rows past the
    last offset are zero, the unvisited-row contract of
    ``recir/ops/helion/jagged_hstu_attention.py:807-827``)."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    offs = np.asarray(seq_offsets, dtype=np.int64)
    out = np.zeros((q.shape[0], q.shape[1], v.shape[2]), dtype=dtype)
    for b in range(len(offs) - 1):
        s, e = int(offs[b]), int(offs[b + 1])
        if not (0 <= s <= e <= q.shape[0]):
            raise ValueError(f"invalid jagged range [{s}, {e}) for values with size {q.shape[0]}")
        L = e - s
        if L == 0:
            continue
        t = None if num_targets is None else int(np.asarray(num_targets)[b])
        keep = keep_mask(L, t, causal, max_attn_len, contextual_seq_len, full_attn_size)
        sc = _scale_for(attn_scale, max_seq_len, s, e, dtype)
        qb = q[s:e].transpose(1, 0, 2)
        kb = k[s:e].transpose(1, 0, 2)
        vb = v[s:e].transpose(1, 0, 2)
        scores = np.matmul(qb, kb.transpose(0, 2, 1)) * dtype(alpha)
        w = scores * _sigmoid(scores) * sc * keep[None].astype(dtype)
        out[s:e] = np.matmul(w, vb).transpose(1, 0, 2)
    return out


def hstu_attention_bwd(
    dout, q, k, v, seq_offsets, max_seq_len, alpha, causal=True, num_targets=None,
    attn_scale=None, max_attn_len=0, contextual_seq_len=0, full_attn_size=0,
    dtype=np.float64,
):
    """Backward closed forms (``helion/jagged_hstu_attention.py:16-27``) -> dq, dk, dv."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    do = np.asarray(dout, dtype=dtype)
    offs = np.asarray(seq_offsets, dtype=np.int64)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for b in range(len(offs) - 1):
        s, e = int(offs[b]), int(offs[b + 1])
        L = e - s
        if L == 0:
            continue
        t = None if num_targets is None else int(np.asarray(num_targets)[b])
        keep = keep_mask(L, t, causal, max_attn_len, contextual_seq_len, full_attn_size)[None].astype(dtype)
        sc = _scale_for(attn_scale, max_seq_len, s, e, dtype)
        qb = q[s:e].transpose(1, 0, 2)
        kb = k[s:e].transpose(1, 0, 2)
        vb = v[s:e].transpose(1, 0, 2)
        dob = do[s:e].transpose(1, 0, 2)
        x = np.matmul(qb, kb.transpose(0, 2, 1)) * dtype(alpha)
        sig = _sigmoid(x)
        p = x * sig * sc * keep
        dp = np.matmul(dob, vb.transpose(0, 2, 1))
        ds = dp * keep * sc * (sig * (1.0 + x * (1.0 - sig)))
        dv[s:e] = np.matmul(p.transpose(0, 2, 1), dob).transpose(1, 0, 2)
        dq[s:e] = (dtype(alpha) * np.matmul(ds, kb)).transpose(1, 0, 2)
        dk[s:e] = (dtype(alpha) * np.matmul(ds.transpose(0, 2, 1), qb)).transpose(1, 0, 2)
    return dq, dk, dv


def count_kept_pairs(lengths, num_targets=None, causal=True, max_attn_len=0,
                     contextual_seq_len=0, full_attn_size=0) -> int:
    """Brute-force number of (query, key) pairs kept, summed over sequences."""
    total = 0
    for b, L in enumerate(lengths):
        t = None if num_targets is None else int(num_targets[b])
        total += int(keep_mask(int(L), t, causal, max_attn_len, contextual_seq_len,
                               full_attn_size).sum())
    return total
