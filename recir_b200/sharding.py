"""Sample sharding of a jagged batch across GPUs: whole sequences per rank, no collective.

Sequences never interact, so the attention path needs no exchange step; the reference
shards the same way (``recir/ops/helion/jagged_hstu_attention.py:923-967``: each device
owns whole sequences, rebuilds local offsets from its own lengths, drops trailing pad
rows, no input replication and no reduction).  Two partitioners:

* ``token_balanced_partition`` -- longest-first greedy assignment into the lightest
  rank (by tokens, or by the quadratic attention cost).
* ``contiguous_partition`` -- the reference's layout contract: rank ``r`` owns the
  ``r``-th block of ``B/W`` consecutive sequences, every block holds exactly ``T/W``
  tokens, and the last ``pad_seqs`` sequences of each block are pad rows that are
  dropped before the kernel runs (``:1089-1141``).
"""
from __future__ import annotations

import numpy as np
import torch


def pad_seqs_per_device(real_bs: int, padded_bs: int, world_size: int) -> int:
    """Trailing pad sequences per rank: ``padded_bs//W - real_bs//W``
    (``set_pad_seqs_per_device``, ``recir/ops/helion/jagged_hstu_attention.py:987-1010``)."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    if real_bs % world_size != 0 or padded_bs % world_size != 0:
        raise ValueError("real and padded batch sizes must be multiples of world_size")
    if padded_bs < real_bs:
        raise ValueError("padded batch smaller than real batch")
    return padded_bs // world_size - real_bs // world_size


def local_offsets(lengths) -> torch.Tensor:
    """``concat([0], cumsum(lengths))`` as int64: offsets restart at 0 on every rank."""
    lengths = torch.as_tensor(np.asarray(lengths), dtype=torch.int64)
    out = torch.zeros(lengths.numel() + 1, dtype=torch.int64)
    out[1:] = torch.cumsum(lengths, 0)
    return out


def token_balanced_partition(lengths, world_size: int, balance: str = "tokens"):
    """Assign whole sequences to ranks, longest first into the lightest rank.

    ``balance="tokens"`` equalises token counts (memory and HBM traffic);
    ``balance="cost"`` equalises ``L*(L+1)/2`` (attention work).  Returns one sorted
    index array per rank; deterministic (ties break on the lower index / lower rank).
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    lengths = np.asarray(lengths, dtype=np.int64)
    if balance == "tokens":
        weight = lengths.astype(np.float64)
    elif balance == "cost":
        weight = lengths.astype(np.float64) * (lengths + 1) / 2.0
    else:
        raise ValueError("balance must be 'tokens' or 'cost'")
    order = np.lexsort((np.arange(len(lengths)), -weight))
    load = np.zeros(world_size, dtype=np.float64)
    parts = [[] for _ in range(world_size)]
    for i in order:
        r = int(np.argmin(load))
        parts[r].append(int(i))
        load[r] += weight[i]
    return [np.array(sorted(p), dtype=np.int64) for p in parts]


def contiguous_partition(lengths, world_size: int, pad_seqs: int = 0):
    """The reference's batch-aligned layout: equal sequence counts and equal token counts per
    rank; raises if a rank boundary is not a sequence boundary of an even token split."""
    lengths = np.asarray(lengths, dtype=np.int64)
    B = len(lengths)
    if B % world_size != 0:
        raise ValueError("number of sequences must be a multiple of world_size")
    b_local = B // world_size
    total = int(lengths.sum())
    if total % world_size != 0:
        raise ValueError("total tokens must be a multiple of world_size")
    l_local = total // world_size
    sums = lengths.reshape(world_size, b_local).sum(axis=1)
    if not np.all(sums == l_local):
        raise ValueError(
            f"per-device token counts {sums.tolist()} are not all equal to l_local={l_local}; "
            "the packing is not batch-aligned")
    keep = b_local - pad_seqs
    if keep <= 0:
        raise ValueError(f"b_local={b_local} leaves no real sequence after dropping {pad_seqs} pad row(s)")
    return [np.arange(r * b_local, r * b_local + keep, dtype=np.int64) for r in range(world_size)]


def gather_rows(t: torch.Tensor, seq_offsets: torch.Tensor, seq_index) -> torch.Tensor:
    """Token rows of the chosen sequences, concatenated in the given order."""
    offs = seq_offsets.tolist()
    if len(seq_index) == 0:
        return t[:0]
    return torch.cat([t[offs[i]:offs[i + 1]] for i in seq_index], 0)


def shard_summary(lengths, parts) -> dict:
    lengths = np.asarray(lengths, dtype=np.int64)
    tokens = [int(lengths[p].sum()) for p in parts]
    cost = [float((lengths[p].astype(np.float64) * (lengths[p] + 1) / 2).sum()) for p in parts]
    mean_t = max(np.mean(tokens), 1e-9)
    mean_c = max(np.mean(cost), 1e-9)
    return {"tokens": tokens, "token_imbalance": float(max(tokens) / mean_t),
            "cost_imbalance": float(max(cost) / mean_c)}
