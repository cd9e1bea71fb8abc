"""Seeded synthetic jagged batches and the algorithmic-work counters.

The reference measures on recommendation datasets that are not available
offline; these generators reproduce the shapes, length distributions and value
distributions of the five benchmark configurations instead.  Every tensor is
drawn on the CPU (``torch.Generator``/``numpy`` with the stated seed), so the
same numbers come out on every machine.

Draw order per configuration: lengths, (num_targets), q, k, v in fp32
``randn * 0.1``, then the cast to the run dtype.  ``dO`` comes from its own
generator (``randn * 0.01``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class HstuBatch:
    """One jagged attention problem (host tensors)."""

    name: str
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    seq_offsets: torch.Tensor  # int64 [B+1]
    num_targets: torch.Tensor | None  # int64 [B]
    max_seq_len: int
    alpha: float
    causal: bool = True
    max_attn_len: int = 0
    contextual_seq_len: int = 0
    full_attn_size: int = 0
    attn_scale: torch.Tensor | None = None
    dout: torch.Tensor | None = None
    meta: dict = field(default_factory=dict)

    @property
    def lengths(self) -> np.ndarray:
        o = self.seq_offsets.numpy()
        return o[1:] - o[:-1]

    @property
    def total_tokens(self) -> int:
        return int(self.seq_offsets[-1])

    def op_kwargs(self) -> dict:
        return dict(max_seq_len=self.max_seq_len, alpha=self.alpha, causal=self.causal,
                    num_targets=self.num_targets, contextual_seq_len=self.contextual_seq_len,
                    max_attn_len=self.max_attn_len, attn_scale=self.attn_scale,
                    full_attn_size=self.full_attn_size)


def _qkv(gen: torch.Generator, T: int, H: int, D: int, dtype: torch.dtype):
    q = (torch.randn(T, H, D, generator=gen) * 0.1).to(dtype)
    k = (torch.randn(T, H, D, generator=gen) * 0.1).to(dtype)
    v = (torch.randn(T, H, D, generator=gen) * 0.1).to(dtype)
    return q, k, v


def _dout(seed: int, shape, dtype):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * 0.01).to(dtype)


def _offsets(lengths) -> torch.Tensor:
    off = torch.zeros(len(lengths) + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(torch.as_tensor(np.asarray(lengths), dtype=torch.int64), 0)
    return off


def config0(dtype=torch.float32) -> HstuBatch:
    """CPU smoke shape: B=4, H=2, D=32, history U[1,16] + 4 targets, N=20."""
    g = torch.Generator(device="cpu").manual_seed(0)
    B, H, D, t = 4, 2, 32, 4
    hist = torch.randint(1, 17, (B,), generator=g)
    lengths = (hist + t).numpy()
    T = int(lengths.sum())
    q, k, v = _qkv(g, T, H, D, dtype)
    return HstuBatch("cfg0_smoke", q, k, v, _offsets(lengths),
                     torch.full((B,), t, dtype=torch.int64), 20, 1.0 / math.sqrt(D),
                     dout=_dout(2, (T, H, D), dtype))


def config1(dtype=torch.bfloat16, batch: int = 64, with_dout: bool = True) -> HstuBatch:
    """Single STU layer shape: B=64, H=4, D=128, history U[256,2048] + 64 targets, N=2112.

    Used forward-only (configuration 1) and forward+backward (configuration 2).
    """
    g = torch.Generator(device="cpu").manual_seed(1)
    H, D, t = 4, 128, 64
    hist = torch.randint(256, 2049, (batch,), generator=g)
    lengths = (hist + t).numpy()
    T = int(lengths.sum())
    q, k, v = _qkv(g, T, H, D, dtype)
    return HstuBatch("cfg1_stu_layer", q, k, v, _offsets(lengths),
                     torch.full((batch,), t, dtype=torch.int64), 2112, 1.0 / math.sqrt(D),
                     dout=_dout(2, (T, H, D), dtype) if with_dout else None)


def config3(dtype=torch.bfloat16, batch: int = 32) -> HstuBatch:
    """Long skewed sequences: B=32, H=8, D=128, lognormal(7.0,0.8) history in [64,8192]
    + 128 targets, contextual_seq_len=3, sliding window 1024, N=8320."""
    g = torch.Generator(device="cpu").manual_seed(3)
    H, D, t = 8, 128, 128
    hist = torch.floor(torch.exp(7.0 + 0.8 * torch.randn(batch, generator=g))).clamp(64, 8192).long()
    lengths = (hist + t).numpy()
    T = int(lengths.sum())
    q, k, v = _qkv(g, T, H, D, dtype)
    return HstuBatch("cfg3_long_window", q, k, v, _offsets(lengths),
                     torch.full((batch,), t, dtype=torch.int64), 8192 + 128, 1.0 / math.sqrt(D),
                     max_attn_len=1024, contextual_seq_len=3,
                     dout=_dout(3 + 1000, (T, H, D), dtype))


def config4_lengths(global_batch: int = 1024):
    """Zipf(1.2) scaled histories clipped to [16,4096] and U[16,128] targets (numpy seed 4)."""
    rng = np.random.default_rng(4)
    hist = np.clip(16 * rng.zipf(1.2, size=global_batch), 16, 4096).astype(np.int64)
    targets = rng.integers(16, 129, size=global_batch).astype(np.int64)
    return hist, targets


def config4_layer(lengths, targets, layer: int, dtype=torch.bfloat16) -> HstuBatch:
    """One of the 8 stacked layers of the batch-sharded stack, for the given (local) sequences."""
    H, D = 4, 128
    g = torch.Generator(device="cpu").manual_seed(4 + layer)
    T = int(np.sum(lengths))
    q, k, v = _qkv(g, T, H, D, dtype)
    return HstuBatch(f"cfg4_stack_l{layer}", q, k, v, _offsets(lengths),
                     torch.as_tensor(np.asarray(targets), dtype=torch.int64), 4096 + 128,
                     1.0 / math.sqrt(D), dout=_dout(1000 + layer, (T, H, D), dtype))


# ---------------------------------------------------------------------------
# Algorithmic work
# ---------------------------------------------------------------------------

def kept_pairs(length: int, num_targets: int | None, causal: bool = True, max_attn_len: int = 0,
               contextual_seq_len: int = 0, full_attn_size: int = 0) -> int:
    """Number of (query, key) pairs the mask keeps for one sequence (closed form).

    Mask rule: ``recir/ops/kjt_split_per_feature.cpp:639-674`` of the reference.
    Closed forms cover the causal cases without a full-attention tail; any other
    combination is counted row by row (still O(L), no L x L matrix).
    """
    L = int(length)
    if L <= 0:
        return 0
    has_t = num_targets is not None
    t = int(num_targets) if has_t else 0
    h = L - t if has_t else L
    w = int(max_attn_len)
    ctx = contextual_seq_len > 0
    if causal and full_attn_size <= 0 and h >= 1:
        tt = L - h  # rows that carry the clamped id h
        if w <= 0:
            hist = h * (h + 1) // 2
            per_target = h + 1
            return hist + tt * per_target
        # row i < h keeps keys with 0 < i-n <= w, itself, and key 0 if contextual and i > w
        i = np.arange(h, dtype=np.int64)
        hist = int((np.minimum(i, w) + 1 + (ctx & (i > w))).sum())
        per_target = min(h, w) + 1 + int(ctx and h > w)
        return hist + tt * per_target
    # generic fallback: evaluate the rule per row with vector ops
    ids = np.arange(L, dtype=np.int64)
    mid = np.minimum(ids, h) if has_t else ids
    total = 0
    boundary = L - t - full_attn_size
    g = np.where(mid < boundary, 0, mid)
    for m in range(L):
        d = mid[m] - mid
        if not causal:
            d = np.abs(d)
        keep = ids == m
        if w > 0:
            keep |= ((d > 0) & (d <= w)) if causal else (d <= w)
            if full_attn_size > 0:
                keep |= (g[m] - g) > 0
        elif causal:
            keep |= d > 0
        if ctx:
            keep |= mid == 0
        total += int(keep.sum())
    return total


def total_kept_pairs(batch: HstuBatch) -> int:
    nt = None if batch.num_targets is None else batch.num_targets.numpy()
    return sum(
        kept_pairs(int(L), None if nt is None else int(nt[b]), batch.causal, batch.max_attn_len,
                   batch.contextual_seq_len, batch.full_attn_size)
        for b, L in enumerate(batch.lengths))


def useful_flops(pairs: int, H: int, dqk: int, dv: int, backward: bool, forward: bool = True) -> float:
    """Useful (masked) floating-point operations.

    Forward: two GEMMs, ``2*(Dqk+Dv)`` flops per kept pair and head.  Backward:
    five useful GEMMs, ``6*Dqk + 4*Dv``.  Scores recomputed by the two-pass
    backward are not counted.
    """
    f = 0.0
    if forward:
        f += 2.0 * (dqk + dv) * H * pairs
    if backward:
        f += (6.0 * dqk + 4.0 * dv) * H * pairs
    return f


def algorithmic_bytes(T: int, H: int, dqk: int, dv: int, itemsize: int, backward: bool,
                      forward: bool = True) -> float:
    """Compulsory HBM traffic: fwd reads q,k,v and writes o; bwd reads q,k,v,dO, writes dq,dk,dv."""
    b = 0.0
    if forward:
        b += (2 * dqk + 2 * dv) * T * H * itemsize
    if backward:
        b += (4 * dqk + 3 * dv) * T * H * itemsize
    return b
