"""CPU restatement (numpy, explicit loops over rows) of the reference's jagged marshalling ops.

TEST INFRASTRUCTURE ONLY: imported by tests, never by the product path.

Follows recir/ops/jagged_ops.py: ``_jagged_to_padded_dense_impl`` (:29-66),
``_dense_to_jagged_forward_impl`` (:69-109), ``_concat_2d_jagged_cpu`` (:218-250),
``_split_2d_jagged_cpu`` (:253-277), including their fast paths and clamped indices.
Pinned against golden vectors produced by importing that file
(tests/golden/jagged_golden.npz, generator tests/golden/make_jagged_golden.py).
"""
from __future__ import annotations

import numpy as np


def _upper(seq, x):
    """torch.searchsorted(seq, x, right=True)"""
    return int(np.searchsorted(np.asarray(seq), x, side="right"))


def jagged_to_padded_dense(values, offsets, max_len, padding_value=0.0):
    values, offsets = np.asarray(values), np.asarray(offsets, dtype=np.int64)
    b = len(offsets) - 1
    if values.shape[0] == b * max_len:
        return values.reshape(b, max_len, *values.shape[1:])
    out = np.full((b, max_len, *values.shape[1:]), padding_value, dtype=values.dtype)
    for i in range(b):
        for n in range(max_len):
            if n < offsets[i + 1] - offsets[i]:
                out[i, n] = values[min(max(offsets[i] + n, 0), max(values.shape[0] - 1, 0))]
    return out


def dense_to_jagged(dense, offsets, total_l=None):
    dense, offsets = np.asarray(dense), np.asarray(offsets, dtype=np.int64)
    b, n = dense.shape[0], dense.shape[1]
    if total_l is None:
        total_l = int(offsets[-1])
    if total_l == 0:
        return np.zeros((0, *dense.shape[2:]), dtype=dense.dtype)
    if total_l == b * n:
        return dense.reshape(total_l, *dense.shape[2:])
    flat = dense.reshape(b * n, *dense.shape[2:])
    out = np.zeros((total_l, *dense.shape[2:]), dtype=dense.dtype)
    interior = offsets[1:-1]
    for j in range(total_l):
        seg = min(max(int(np.sum((interior <= j) & (interior < total_l))), 0), b - 1)
        intra = j - offsets[seg]
        valid = j < offsets[b] and intra >= 0 and intra < offsets[seg + 1] - offsets[seg]
        if valid:
            out[j] = flat[min(max(seg * n + intra, 0), max(b * n - 1, 0))]
    return out


def concat_2d_jagged(values_left, offsets_left, values_right, offsets_right):
    vl, vr = np.asarray(values_left), np.asarray(values_right)
    ol, orr = np.asarray(offsets_left, dtype=np.int64), np.asarray(offsets_right, dtype=np.int64)
    if vl.shape[0] == 0:
        return vr
    if vr.shape[0] == 0:
        return vl
    n = len(ol) - 1
    comb = ol + orr
    total = vl.shape[0] + vr.shape[0]
    out = np.empty((total, *vl.shape[1:]), dtype=vl.dtype)
    for p in range(total):
        b = min(max(_upper(comb[1:], p), 0), n - 1)
        intra, la = p - comb[b], ol[b + 1] - ol[b]
        if intra < la:
            out[p] = vl[min(max(ol[b] + intra, 0), vl.shape[0] - 1)]
        else:
            out[p] = vr[min(max(orr[b] + intra - la, 0), vr.shape[0] - 1)]
    return out


def split_2d_jagged(values, offsets_left, offsets_right, seq_len_a, seq_len_b):
    v = np.asarray(values)
    ol, orr = np.asarray(offsets_left, dtype=np.int64), np.asarray(offsets_right, dtype=np.int64)
    n = len(ol) - 1
    left = np.empty((seq_len_a, *v.shape[1:]), dtype=v.dtype)
    right = np.empty((seq_len_b, *v.shape[1:]), dtype=v.dtype)
    for pa in range(seq_len_a):
        ba = min(max(_upper(ol[1:], pa), 0), n - 1)
        left[pa] = v[min(max(pa + orr[ba], 0), v.shape[0] - 1)]
    for pb in range(seq_len_b):
        bb = min(max(_upper(orr[1:], pb), 0), n - 1)
        right[pb] = v[min(max(pb + ol[bb + 1], 0), v.shape[0] - 1)]
    return left, right


def _uniform_offsets(batch, length):
    return np.arange(batch + 1, dtype=np.int64) * int(length)


def gr_concat_2d_jagged(values_a, values_b, offsets_a=None, offsets_b=None, is_replace=False,
                        n_prefix_from_right=0):
    """``generative_recommenders::concat_2D_jagged_fwd_op`` (recir/ops/kjt_split_per_feature.cpp:100-196).
    A side without offsets is dense ``[B, L, D]``.  Per sequence the result is ``[b[:p], a, b[p:]]``
    (p = n_prefix_from_right), or with ``is_replace`` the rows of ``a`` with its last ``len(b)`` rows
    replaced by ``b``; a dense ``a`` keeps its shape under ``is_replace``."""
    va, vb = np.asarray(values_a), np.asarray(values_b)
    if offsets_a is None and offsets_b is None:
        raise ValueError("at least one input must be jagged")
    if is_replace and n_prefix_from_right:
        raise ValueError("n_prefix_from_right is not supported when is_replace is true")
    batch = (len(offsets_a) if offsets_a is not None else len(offsets_b)) - 1
    oa = np.asarray(offsets_a, np.int64) if offsets_a is not None else _uniform_offsets(batch, va.shape[1])
    ob = np.asarray(offsets_b, np.int64) if offsets_b is not None else _uniform_offsets(batch, vb.shape[1])
    fa, fb = va.reshape(-1, va.shape[-1]), vb.reshape(-1, vb.shape[-1])
    p = int(n_prefix_from_right)
    parts = []
    for b in range(batch):
        a_rows, b_rows = fa[oa[b]:oa[b + 1]], fb[ob[b]:ob[b + 1]]
        if is_replace:
            if len(b_rows) > len(a_rows):
                raise ValueError("replacement values_b cannot be longer than values_a")
            parts += [a_rows[:len(a_rows) - len(b_rows)], b_rows]
        else:
            if p > len(b_rows):
                raise ValueError("n_prefix_from_right cannot exceed a values_b sequence length")
            parts += [b_rows[:p], a_rows, b_rows[p:]]
    flat = np.concatenate(parts, 0) if parts else np.zeros((0, va.shape[-1]), va.dtype)
    return flat.reshape(va.shape) if is_replace and va.ndim == 3 else flat


def gr_split_2d_jagged(values, offsets_a, offsets_b, is_dense_a=False, is_dense_b=False, dense_size=0,
                       n_prefix_to_right=0, batch=None):
    """``generative_recommenders::split_2D_jagged_fwd_op`` (recir/ops/kjt_split_per_feature.cpp:430-489):
    the inverse of the concatenation; a dense side has ``dense_size`` rows per sequence and comes back
    as ``[B, dense_size, D]``."""
    v = np.asarray(values)
    if batch is None:
        batch = (len(offsets_b) if is_dense_a else len(offsets_a)) - 1
    oa = _uniform_offsets(batch, dense_size) if is_dense_a else np.asarray(offsets_a, np.int64)
    ob = _uniform_offsets(batch, dense_size) if is_dense_b else np.asarray(offsets_b, np.int64)
    p = int(n_prefix_to_right)
    out_a, out_b, pos = [], [], 0
    for b in range(batch):
        la, lb = int(oa[b + 1] - oa[b]), int(ob[b + 1] - ob[b])
        if p > lb:
            raise ValueError("n_prefix_to_right cannot exceed a values_b sequence length")
        rows = v[pos:pos + la + lb]
        out_a.append(rows[p:p + la])
        out_b += [rows[:p], rows[p + la:]]
        pos += la + lb
    if pos != v.shape[0]:
        raise ValueError("split lengths do not match values")
    a = np.concatenate(out_a, 0) if out_a else np.zeros((0, v.shape[1]), v.dtype)
    bb = np.concatenate(out_b, 0) if out_b else np.zeros((0, v.shape[1]), v.dtype)
    if is_dense_a:
        a = a.reshape(batch, dense_size, v.shape[1])
    if is_dense_b:
        bb = bb.reshape(batch, dense_size, v.shape[1])
    return a, bb
