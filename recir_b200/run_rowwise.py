"""Time the row-wise STU kernels on the current GPU and print their HBM throughput.

    python -m recir_b200.run_rowwise --rows 1650165 --cols 512

``rows`` defaults to the token count of the Zipf batch (one layer), ``cols`` to the embedding
width H*D = 512 of the benchmark configurations.  Algorithmic bytes: layer norm reads x and writes y
(2 * rows * cols * 2 B in bf16, plus 8 B of statistics per row); the layer-norm * gate stage reads
x and u and writes the output row (and its fp8 copy).  Inputs are far larger than L2.
"""
from __future__ import annotations

import argparse
import json

import torch

import recir_b200  # noqa: F401


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=1650165)
    ap.add_argument("--cols", type=int, default=512)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    dev = "cuda"
    g = torch.Generator().manual_seed(0)
    cols = args.cols
    x = (torch.randn(args.rows, cols, generator=g)).to(torch.bfloat16).to(dev)
    u = (torch.randn(args.rows, cols, generator=g)).to(torch.bfloat16).to(dev)
    w = torch.ones(cols, dtype=torch.bfloat16, device=dev)
    b = torch.zeros(cols, dtype=torch.bfloat16, device=dev)

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

    el = args.rows * cols
    cases = {
        "layer_norm_affine": (lambda: torch.ops.recir.b200_weighted_layer_norm_fwd(x, w, b, 1e-6, None, None, False),
                              2 * el * 2 + 8 * args.rows),
        "layer_norm_swish": (lambda: torch.ops.recir.b200_weighted_layer_norm_fwd(x, w, b, 1e-6, None, None, True),
                             2 * el * 2 + 8 * args.rows),
        "layer_norm_mul_silu (y only counted)": (
            lambda: torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
                x, u, w, b, 1e-6, 0.0, False, False, False, False, "silu", 0, True, 0),
            3 * el * 2 + el + 12 * args.rows),
        "layer_norm_mul_silu fp8 only": (
            lambda: torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
                x, u, w, b, 1e-6, 0.0, False, False, False, False, "silu", 0, False, 0),
            2 * el * 2 + el + 12 * args.rows),
    }
    out = {"rows": args.rows, "cols": cols, "dtype": "bf16"}
    for name, (fn, nbytes) in cases.items():
        ms = timed(fn)
        out[name] = {"ms": ms, "algorithmic_bytes": nbytes, "GB/s": nbytes / ms / 1e6}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
