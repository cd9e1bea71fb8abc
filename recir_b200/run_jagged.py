"""Time the jagged marshalling kernels and the embedding add on the current GPU and print their HBM throughput.

    python -m recir_b200.run_jagged --batch 1024

Uses the length distribution of the Zipf batch (one layer, embedding width 512, bf16).  Algorithmic
bytes: every destination row is written once and every kept source row read once
(jagged -> dense: T rows read, B*N rows written; dense -> jagged, concat and split: T read, T written).
"""
from __future__ import annotations

import argparse
import json

import torch

import recir_b200
from recir_b200 import workload


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--cols", type=int, default=512)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    hist, tg = workload.config4_lengths(args.batch)
    lengths = torch.as_tensor(hist + tg)
    dev = "cuda"
    off = torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)]).to(dev)
    hist_off = torch.cat([torch.zeros(1, dtype=torch.int64), torch.as_tensor(hist).cumsum(0)]).to(dev)
    tgt_off = torch.cat([torch.zeros(1, dtype=torch.int64), torch.as_tensor(tg).cumsum(0)]).to(dev)
    T, n, b = int(off[-1]), int(lengths.max()), len(lengths)
    x = torch.randn(T, args.cols, dtype=torch.bfloat16, device=dev)
    row = args.cols * 2
    ops = torch.ops.recir

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.iters

    dense = ops.b200_jagged_to_padded_dense(x, [off], [n], 0.0)
    left, right = ops.b200_split_2d_jagged(x, hist_off, tgt_off, int(hist_off[-1]), int(tgt_off[-1]))
    cases = {
        "jagged_to_padded_dense": (lambda: ops.b200_jagged_to_padded_dense(x, [off], [n], 0.0), (T + b * n) * row),
        "dense_to_jagged": (lambda: ops.b200_dense_to_jagged(dense, [off], T), 2 * T * row),
        "split_2d_jagged": (lambda: ops.b200_split_2d_jagged(x, hist_off, tgt_off, left.shape[0], right.shape[0]), 2 * T * row),
        "concat_2d_jagged": (lambda: ops.b200_concat_2d_jagged(left, hist_off, right, tgt_off), 2 * T * row),
    }
    # position + timestamp embedding add: x read, out written, two table rows per token (L2-resident tables)
    g = torch.Generator().manual_seed(0)
    pos_t = torch.randn(n + 8, args.cols, generator=g).to(torch.bfloat16).to(dev)
    ts_t = torch.randn(2049, args.cols, generator=g).to(torch.bfloat16).to(dev)
    stamps = (torch.cumsum(torch.exp(torch.rand(b, n, generator=g) * 12.0).to(torch.int64), dim=1) + 1_600_000_000).to(dev)
    lens_d, tg_d = lengths.to(dev), torch.as_tensor(tg).to(dev)
    cases["add_ts_pos_emb"] = (
        lambda: ops.b200_add_ts_pos_emb_fwd(x, off, pos_t, ts_t, stamps, lens_d, tg_d, n, 0, False, "sqrt"),
        2 * T * row + 8 * T + 8 * T)
    out = {"B": b, "T": T, "N": n, "cols": args.cols, "dtype": "bf16"}
    for name, (fn, nbytes) in cases.items():
        ms = timed(fn)
        out[name] = {"ms": ms, "algorithmic_bytes": nbytes, "GB/s": nbytes / ms / 1e6}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
