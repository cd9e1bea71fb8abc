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
