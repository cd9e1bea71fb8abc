"""CPU restatement (numpy) of the reference's position + timestamp embedding add.

TEST INFRASTRUCTURE ONLY: imported by tests, never by the product path.

Follows ``addTimestampPositionEmbeddings``, recir/ops/kjt_split_per_feature.cpp:307-428, one
sequence at a time; ``dtype`` / ``table_dtype`` name the element types whose roundings the
reference's tensor ops apply (see oracle/rowwise_oracle.py:round_to).  Pinned against golden
vectors made by the reference's compiled operator (tests/golden/embed_golden.npz, generator
tests/golden/make_embed_golden.py).
"""
from __future__ import annotations

import numpy as np

from .rowwise_oracle import round_to


def add_ts_pos_emb(x, offsets, pos_table, ts_table, timestamps, seq_lengths, num_targets, max_contextual_seq_len,
                   interleave_targets, time_bucket_fn, dtype="float32", table_dtype=None):
    """Returns (out, pos_index, ts_index) per packed token (unsorted indices)."""
    table_dtype = table_dtype or dtype
    x = np.asarray(x, np.float32)
    offsets = np.asarray(offsets, np.int64)
    out = np.zeros_like(x)
    pos_idx = np.zeros(x.shape[0], np.int32)
    ts_idx = np.zeros(x.shape[0], np.int32)
    p_rows, c = pos_table.shape[0], int(max_contextual_seq_len)
    for b in range(len(seq_lengths)):
        s, e = int(offsets[b]), int(offsets[b + 1])
        n, length = e - s, int(seq_lengths[b])
        high = length - (int(num_targets[b]) * (2 if interleave_targets else 1) if num_targets is not None else 0)
        i = np.arange(n, dtype=np.int64)
        pos = high - np.minimum(i, high) + c
        pos = np.minimum(pos, p_rows - 1)
        pos = np.where(i < c, i, pos)
        stamps = np.asarray(timestamps[b], np.int64)
        d = (stamps[length - 1] - stamps[:n]).astype(np.float32)
        d = np.maximum(d, np.float32(1e-6)) / np.float32(60.0)
        d = np.log(d, dtype=np.float32) if time_bucket_fn == "log" else np.sqrt(d, dtype=np.float32)
        tsb = np.clip(np.trunc(d).astype(np.int64), 0, 2048)
        added = round_to(round_to(np.asarray(pos_table, np.float32)[pos] + np.asarray(ts_table, np.float32)[tsb], table_dtype), dtype)
        out[s:e] = round_to(x[s:e] + added, dtype)
        pos_idx[s:e], ts_idx[s:e] = pos, tsb
    return out, pos_idx, ts_idx
