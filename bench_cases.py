"""Single-purpose runners behind ``python bench.py --case NAME ...`` (also the commands profilers are
pointed at: after the inputs are on the device they launch nothing but this library's kernels, plus
the two library sorts of the embedding operator).

    python bench.py --case attn --config cfg1 --passes fwd --iters 5
    python bench.py --case attn --config cfg4 --buckets --calls 10
    python bench.py --case rowwise --rows 1650165 --cols 512
    python bench.py --case jagged --batch 1024
    python bench.py --case gemm --rows 1650165 --k 512 --n 2048

``attn``: one benchmark configuration of the HSTU attention -- cfg0 (smoke shape, fp32), cfg1 (B=64, H=4,
D=128 bf16), cfg3 (long skewed sequences, sliding window + contextual flag), cfg4 (one layer of the Zipf
batch, optionally the shard of one rank).  ``--passes`` is ``fwd``, ``bwd`` or ``both``.  ``--buckets`` (cfg4
only) times each sequence-length bucket of the Zipf batch as a batch of its own, repeated to at least 64k
tokens so that its tensors exceed the L2, and reports useful TFLOP/s and algorithmic GB/s per bucket: short
sequences sit on the HBM roofline, long ones on the tensor-core roofline.
``rowwise``: the row-wise STU kernels (layer norm, gate stage, fp8 copy), HBM throughput.
``jagged``: the jagged marshalling kernels and the embedding add, HBM throughput, on the Zipf lengths.
``gemm``: the fused layer-norm + u/v/q/k projection against the two-kernel chain and the vendor GEMM.
``trace``: per-role cycle accounting and event trace inside the attention kernels (instrumented build only).
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from recir_b200 import ops, sharding, workload


def make_batch(name: str, batch: int | None, rank: int, world: int):
    if name == "cfg0":
        return workload.config0()
    if name == "cfg1":
        return workload.config1(batch=batch or 64)
    if name == "cfg3":
        return workload.config3(batch=batch or 32)
    if name == "cfg4":
        hist, tg = workload.config4_lengths(batch or 1024)
        lengths = hist + tg
        mine = sharding.token_balanced_partition(lengths, world)[rank]
        return workload.config4_layer(lengths[mine], tg[mine], layer=0)
    raise SystemExit(f"unknown config {name}")


BUCKETS = ((32, 128), (128, 256), (256, 512), (512, 1024), (1024, 2048), (2048, 4225))


def bucket_batch(lo: int, hi: int, min_tokens: int = 65536):
    """The cfg4 sequences with lo <= length < hi: repeated until the batch holds min_tokens tokens, or cut
    after the first 4 * min_tokens tokens when the bucket holds more."""
    hist, tg = workload.config4_lengths(1024)
    lengths = hist + tg
    sel = np.nonzero((lengths >= lo) & (lengths < hi))[0]
    if sel.size == 0:
        return None, 0
    n = sel.size
    over = np.nonzero(np.cumsum(lengths[sel]) >= 4 * min_tokens)[0]
    if over.size:
        sel = sel[: int(over[0]) + 1]
    reps = max(1, -(-min_tokens // int(lengths[sel].sum())))
    sel_r = np.tile(sel, reps)
    return workload.config4_layer(lengths[sel_r], tg[sel_r], layer=0), int(n)


def measure(bt, passes: str, iters: int, warmup: int, calls: int = 1) -> dict:
    """Times the forward and/or backward operator call on one batch with CUDA events.  With calls > 1
    each sample is that many calls issued back to back, divided by their number, so that the host's
    launch latency hides behind the previous call's kernels."""
    dev = torch.device("cuda")
    q, k, v, do = (x.to(dev) for x in (bt.q, bt.k, bt.v, bt.dout))
    off = bt.seq_offsets.to(dev)
    nt = None if bt.num_targets is None else bt.num_targets.to(dev)
    a = (off, bt.max_seq_len, bt.alpha, bt.causal, nt, bt.contextual_seq_len, bt.max_attn_len, None,
         bt.full_attn_size)
    H, Dq, Dv = q.shape[1], q.shape[2], v.shape[2]
    pairs = workload.total_kept_pairs(bt)

    def fwd():
        return torch.ops.recir.b200_hstu_attention_fwd(q, k, v, *a)

    def bwd():
        return torch.ops.recir.b200_hstu_attention_bwd(do, q, k, v, *a)

    res = {"config": bt.name, "T": bt.total_tokens, "B": len(bt.lengths), "H": H, "D": Dq,
           "kept_pairs_per_head": pairs}
    for name, fn, fl, by in (
            ("fwd", fwd, workload.useful_flops(pairs, H, Dq, Dv, False),
             workload.algorithmic_bytes(bt.total_tokens, H, Dq, Dv, q.element_size(), False)),
            ("bwd", bwd, workload.useful_flops(pairs, H, Dq, Dv, True, forward=False),
             workload.algorithmic_bytes(bt.total_tokens, H, Dq, Dv, q.element_size(), True, forward=False))):
        if passes not in (name, "both"):
            continue
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(calls):
                fn()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / calls)
        med = float(np.median(times))
        res[name] = {"ms_median": med, "ms_min": float(min(times)), "useful_tflops": fl / (med * 1e-3) / 1e12,
                     "algorithmic_gbs": by / (med * 1e-3) / 1e9}
    return res


def main_attn(argv):
    ap = argparse.ArgumentParser(prog="bench.py --case attn")
    ap.add_argument("--config", default="cfg1")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--passes", default="both", choices=["fwd", "bwd", "both"])
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--rank", type=int, default=0)
    ap.add_argument("--world", type=int, default=1)
    ap.add_argument("--simt", action="store_true", help="use the CUDA-core kernels")
    ap.add_argument("--calls", type=int, default=1, help="calls issued back to back per timed sample")
    ap.add_argument("--buckets", action="store_true", help="cfg4: one measurement per sequence-length bucket")
    ap.add_argument("--bucket", default=None, help="cfg4: only the bucket LO:HI (lengths LO <= L < HI)")
    args = ap.parse_args(argv)

    if args.buckets or args.bucket:
        out = []
        only = tuple(int(x) for x in args.bucket.split(":")) if args.bucket else None
        for lo, hi in ((only,) if only else BUCKETS):
            bt, n = bucket_batch(lo, hi)
            if bt is None:
                continue
            r = measure(bt, args.passes, args.iters, args.warmup, args.calls)
            r.update(bucket=[lo, hi], seqs_in_cfg4=n, mean_length=bt.total_tokens / len(bt.lengths))
            out.append(r)
        print(json.dumps({"config": "cfg4 length buckets", "buckets": out}))
        return

    # under torchrun (one process per GPU) every rank takes its token-balanced shard of the
    # configuration; rank 0 then reports the slowest rank (max over ranks) and global tokens/s
    import os
    dist_run = int(os.environ.get("WORLD_SIZE", "1")) > 1
    if dist_run:
        import torch.distributed as dist
        args.rank, args.world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))

    bt = make_batch(args.config, args.batch, args.rank, args.world)
    dev = torch.device("cuda")
    ops.set_force_simt(args.simt)
    res = measure(bt, args.passes, args.iters, args.warmup, args.calls)
    if dist_run:
        keys = [k for k in ("fwd", "bwd") if k in res]
        t = torch.tensor([res[k]["ms_median"] for k in keys] + [float(bt.total_tokens)], dtype=torch.float64, device=dev)
        tmax, tsum = t.clone(), t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        if args.rank == 0:
            step_ms = float(tmax[:-1].sum())
            print(json.dumps({"config": bt.name, "world": args.world, "T_global": int(tsum[-1].item()),
                              "ms_max_over_ranks": {k: float(tmax[i]) for i, k in enumerate(keys)},
                              "tokens_per_s": float(tsum[-1].item()) / (step_ms * 1e-3), "rank0": res}))
        dist.barrier()
        dist.destroy_process_group()
    else:
        print(json.dumps(res))



def _timed(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main_rowwise(argv):
    """Row-wise STU kernels.  ``rows`` defaults to the token count of the Zipf batch (one layer), ``cols`` to
    the embedding width H*D = 512.  Algorithmic bytes: layer norm reads x and writes y (2 * rows * cols * 2 B
    in bf16, plus 8 B of statistics per row); the layer-norm * gate stage reads x and u and writes the output
    row (and its fp8 copy); the backward kernels read x, dy (and u) and write dx (and du) plus the two
    per-column sums.  Inputs are far larger than L2."""
    ap = argparse.ArgumentParser(prog="bench.py --case rowwise")
    ap.add_argument("--rows", type=int, default=1650165)
    ap.add_argument("--cols", type=int, default=512)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    print(json.dumps(rowwise_numbers(args)))


def rowwise_numbers(args):
    """The measurements of ``main_rowwise`` as a dict; ``args`` has rows, cols, iters, warmup."""
    dev = "cuda"
    g = torch.Generator().manual_seed(0)
    cols = args.cols
    x = (torch.randn(args.rows, cols, generator=g)).to(torch.bfloat16).to(dev)
    u = (torch.randn(args.rows, cols, generator=g)).to(torch.bfloat16).to(dev)
    w = torch.ones(cols, dtype=torch.bfloat16, device=dev)
    b = torch.zeros(cols, dtype=torch.bfloat16, device=dev)
    el = args.rows * cols
    R = torch.ops.recir
    cases = {
        "layer_norm_affine": (lambda: R.b200_weighted_layer_norm_fwd(x, w, b, 1e-6, None, None, False),
                              2 * el * 2 + 8 * args.rows),
        "layer_norm_swish": (lambda: R.b200_weighted_layer_norm_fwd(x, w, b, 1e-6, None, None, True),
                             2 * el * 2 + 8 * args.rows),
        "layer_norm_mul_silu (y only counted)": (
            lambda: R.b200_layer_norm_mul_dropout_quantization_fwd(
                x, u, w, b, 1e-6, 0.0, False, False, False, False, "silu", 0, True, 0),
            3 * el * 2 + el + 12 * args.rows),
        "layer_norm_mul_silu fp8 only": (
            lambda: R.b200_layer_norm_mul_dropout_quantization_fwd(
                x, u, w, b, 1e-6, 0.0, False, False, False, False, "silu", 0, False, 0),
            2 * el * 2 + el + 12 * args.rows),
    }
    if hasattr(R, "b200_weighted_layer_norm_bwd"):
        y, mean, rstd = R.b200_weighted_layer_norm_fwd(x, w, b, 1e-6, None, None, False)[:3]
        cases["layer_norm_bwd"] = (lambda: R.b200_weighted_layer_norm_bwd(u, x, w, b, mean, rstd, False),
                                   3 * el * 2 + 8 * args.rows)
        cases["layer_norm_swish_bwd"] = (lambda: R.b200_weighted_layer_norm_bwd(u, x, w, b, mean, rstd, True),
                                         3 * el * 2 + 8 * args.rows)
        # gate stage backward: x, u and the incoming gradient read, dx and du written
        dout = torch.randn_like(x)
        cases["layer_norm_mul_silu_bwd"] = (
            lambda: R.b200_layer_norm_mul_dropout_quantization_bwd(dout, x, u, w, b, mean, rstd, False, False, False, "silu"),
            5 * el * 2 + 8 * args.rows)
    out = {"rows": args.rows, "cols": cols, "dtype": "bf16"}
    for name, (fn, nbytes) in cases.items():
        ms = _timed(fn, args.iters, args.warmup)
        out[name] = {"ms": ms, "algorithmic_bytes": nbytes, "GB/s": nbytes / ms / 1e6}
    return out


def main_jagged(argv):
    """Jagged marshalling kernels and the embedding add on the length distribution of the Zipf batch (one
    layer, embedding width 512, bf16).  Algorithmic bytes: every destination row is written once and every
    kept source row read once (jagged -> dense: T rows read, B*N rows written; dense -> jagged, concat and
    split: T read, T written)."""
    ap = argparse.ArgumentParser(prog="bench.py --case jagged")
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--cols", type=int, default=512)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    hist, tg = workload.config4_lengths(args.batch)
    lengths = torch.as_tensor(hist + tg)
    dev = "cuda"
    off = torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)]).to(dev)
    hist_off = torch.cat([torch.zeros(1, dtype=torch.int64), torch.as_tensor(hist).cumsum(0)]).to(dev)
    tgt_off = torch.cat([torch.zeros(1, dtype=torch.int64), torch.as_tensor(tg).cumsum(0)]).to(dev)
    T, n, b = int(off[-1]), int(lengths.max()), len(lengths)
    x = torch.randn(T, args.cols, dtype=torch.bfloat16, device=dev)
    row = args.cols * 2
    R = torch.ops.recir
    dense = R.b200_jagged_to_padded_dense(x, [off], [n], 0.0)
    left, right = R.b200_split_2d_jagged(x, hist_off, tgt_off, int(hist_off[-1]), int(tgt_off[-1]))
    cases = {
        "jagged_to_padded_dense": (lambda: R.b200_jagged_to_padded_dense(x, [off], [n], 0.0), (T + b * n) * row),
        "dense_to_jagged": (lambda: R.b200_dense_to_jagged(dense, [off], T), 2 * T * row),
        "split_2d_jagged": (lambda: R.b200_split_2d_jagged(x, hist_off, tgt_off, left.shape[0], right.shape[0]), 2 * T * row),
        "concat_2d_jagged": (lambda: R.b200_concat_2d_jagged(left, hist_off, right, tgt_off), 2 * T * row),
    }
    # position + timestamp embedding add: x read, out written, two table rows per token (L2-resident tables)
    g = torch.Generator().manual_seed(0)
    pos_t = torch.randn(n + 8, args.cols, generator=g).to(torch.bfloat16).to(dev)
    ts_t = torch.randn(2049, args.cols, generator=g).to(torch.bfloat16).to(dev)
    stamps = (torch.cumsum(torch.exp(torch.rand(b, n, generator=g) * 12.0).to(torch.int64), dim=1) + 1_600_000_000).to(dev)
    lens_d, tg_d = lengths.to(dev), torch.as_tensor(tg).to(dev)
    cases["add_ts_pos_emb"] = (
        lambda: R.b200_add_ts_pos_emb_fwd(x, off, pos_t, ts_t, stamps, lens_d, tg_d, n, 0, False, "sqrt"),
        2 * T * row + 8 * T + 8 * T)
    out = {"B": b, "T": T, "N": n, "cols": args.cols, "dtype": "bf16"}
    for name, (fn, nbytes) in cases.items():
        ms = _timed(fn, args.iters, args.warmup)
        out[name] = {"ms": ms, "algorithmic_bytes": nbytes, "GB/s": nbytes / ms / 1e6}
    return out


def main_gemm(argv):
    """The u | v | q | k projection of an STU layer (embedding width K into N = 4 * H * D columns) on the token
    count of the Zipf batch: the fused layer-norm + projection kernel against the two-kernel chain (this
    library's layer norm, then the vendor library's GEMM), and the projection alone against the vendor
    library.  Useful work: 2 * rows * K * N flops; algorithmic bytes of the fused form: x read, out written,
    W read once (it stays in L2)."""
    ap = argparse.ArgumentParser(prog="bench.py --case gemm")
    ap.add_argument("--rows", type=int, default=1650165)
    ap.add_argument("--k", type=int, default=512)
    ap.add_argument("--n", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    print(json.dumps(gemm_numbers(args)))


def gemm_numbers(args):
    """The measurements of ``main_gemm`` as a dict; ``args`` has rows, k, n, iters, warmup."""
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    M, K, N = args.rows, args.k, args.n
    x = (torch.randn(M, K, generator=g, device=dev) * 1.5).to(torch.bfloat16)
    w = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
    b = torch.randn(N, generator=g, device=dev).to(torch.bfloat16)
    lw = torch.ones(K, dtype=torch.bfloat16, device=dev)
    lb = torch.zeros(K, dtype=torch.bfloat16, device=dev)
    R = torch.ops.recir
    y = R.b200_weighted_layer_norm_fwd(x, lw, lb, 1e-5, None, None, False)[0]
    flops = 2.0 * M * K * N
    cases = {
        "fused layer_norm + addmm (this library, one kernel)": lambda: R.b200_layer_norm_addmm_fwd(x, lw, lb, 1e-5, False, w, b),
        "layer_norm kernel, then vendor GEMM": lambda: torch.addmm(b, R.b200_weighted_layer_norm_fwd(x, lw, lb, 1e-5, None, None, False)[0], w),
        "addmm (this library)": lambda: R.b200_addmm_fwd(y, w, b),
        "addmm (vendor GEMM)": lambda: torch.addmm(b, y, w),
    }
    out = {"rows": M, "K": K, "N": N, "dtype": "bf16", "useful_flops": flops,
           "algorithmic_bytes_fused": (M * K + M * N + K * N) * 2}
    for name, fn in cases.items():
        ms = _timed(fn, args.iters, args.warmup)
        out[name] = {"ms": ms, "TFLOP/s": flops / ms / 1e9, "GB/s": out["algorithmic_bytes_fused"] / ms / 1e6}
    # the row-wise scaled fp8 projection on the same sizes (a [M, K] and W [N, K] in e4m3, bf16 out):
    # this library's kernel against the vendor library's fp8 GEMM followed by the scaling pass
    if K % 128 == 0 and K <= 1024:
        a8 = (torch.randn(M, K, generator=g, device=dev) * 60.0).clamp(-448, 448).to(torch.float8_e4m3fn)
        w8 = (torch.randn(N, K, generator=g, device=dev) * 40.0).clamp(-448, 448).to(torch.float8_e4m3fn)
        sa = torch.rand(M, generator=g, device=dev) * 0.02 + 0.001
        sb = torch.rand(N, generator=g, device=dev) * 0.01 + 0.001
        one = torch.ones((), dtype=torch.float32, device=dev)

        def vendor_fp8():
            o = torch._scaled_mm(a8, w8.t(), scale_a=one, scale_b=one, out_dtype=torch.float32) * sa[:, None] * sb[None, :]
            return (o + b.float()).to(torch.bfloat16)

        fp8_bytes = M * K + N * K + M * N * 2
        for name, fn in (("fp8 rowwise addmm (this library)",
                          lambda: R.b200_fp8_rowwise_addmm_fwd(a8, w8, sa, sb, b, True, False, torch.bfloat16, False, False)),
                         ("fp8 rowwise addmm (vendor fp8 GEMM, then scales and bias)", vendor_fp8)):
            ms = _timed(fn, args.iters, args.warmup)
            out[name] = {"ms": ms, "TFLOP/s": flops / ms / 1e9, "GB/s": fp8_bytes / ms / 1e6}
    return out


def main_trace(argv):
    """In-kernel cycle accounting and event trace of the three tensor-core attention kernels on cfg1.  Needs
    the instrumented library (`python -m recir_b200.build -DB200_HSTU_PROFILING`, which instantiates the PROF
    variants of the kernels; rebuild with `--force` afterwards) and goes through the C ABI directly, because
    the trace wants a status buffer of 16 + 8192 ints (B200_HSTU_FLAG_TRACE).  Prints, per kernel: the time of
    the traced call, the per-role wait / busy cycles summed over CTAs (workspace ints 2..15), and for CTA 0 the
    median phases of the epilogue per (half) tile from the event trace."""
    import ctypes
    import os

    ap = argparse.ArgumentParser(prog="bench.py --case trace")
    ap.add_argument("--kernel", default="all", choices=["all", "fwd", "dkv", "dq"])
    args = ap.parse_args(argv)
    os.environ["B200_HSTU_PROFILE"] = "1"
    os.environ["B200_HSTU_PROFILE_DQ"] = "1"
    from recir_b200 import _lib

    bt = workload.config1()
    dev = "cuda"
    q, k, v, do = (x.to(dev) for x in (bt.q, bt.k, bt.v, bt.dout))
    off, nt = bt.seq_offsets.to(dev), bt.num_targets.to(dev)
    lib = _lib.load()
    names_f = ["mma_total", "mma_wait_kfull", "mma_wait_pready", "mma_wait_vfull", "mma_wait_item", "epi_total",
               "epi_wait_sfull", "epi_wait_ofull", "epi_partial", "epi_full", "-", "epi_drain", "prod_wait", "prod_total"]
    names_b = ["mma_total", "mma_wait_load", "mma_wait_p", "mma_wait_acc", "mma_wait_item", "epi_total", "epi_wait_s",
               "epi_wait_acc", "epi_tile", "epi_drain", "epi_ld", "epi_st", "-", "-"]
    out = {}
    for which in (("fwd", "dkv", "dq") if args.kernel == "all" else (args.kernel,)):
        p = _lib.B200HstuParams()
        keep = ops._fill(p, q, k, v, off, bt.max_seq_len, bt.alpha, True, nt, 0, 0, None, 0)
        o, dq, dk, dv = (torch.empty_like(x) for x in (v, q, k, v))
        p.o, p.o_row_stride = o.data_ptr(), o.stride(0)
        p.d_o, p.do_row_stride = do.data_ptr(), do.stride(0)
        p.dq, p.dk, p.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
        p.dq_row_stride = p.dk_row_stride = p.dv_row_stride = dq.stride(0)
        pass_id = 0 if which == "fwd" else 1
        # "dq" traces the recomputing dQ kernel (the one from stored dS tiles has no instrumented variant:
        # it has no epilogue phases to speak of); "dkv" runs as in a default call, storing its tiles
        p.flags |= _lib.FLAG_TRACE | {"fwd": 0, "dkv": _lib.FLAG_BWD_SKIP_DQ,
                                      "dq": _lib.FLAG_BWD_SKIP_DKV | _lib.FLAG_BWD_RECOMPUTE_DQ}[which]
        need = lib.b200_hstu_workspace_bytes(ctypes.byref(p), pass_id)
        ws = torch.zeros(need // 4 + 64, dtype=torch.int32, device=dev)
        base = ((-ws.data_ptr()) % 256) // 4
        p.workspace, p.workspace_bytes = ws.data_ptr() + 4 * base, need
        status = torch.zeros(16 + 8192, dtype=torch.int32, device=dev)
        p.status = status.data_ptr()
        fn = lib.b200_hstu_fwd if pass_id == 0 else lib.b200_hstu_bwd
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for _ in range(2):
            assert fn(ctypes.byref(p), st) == 0
        torch.cuda.synchronize()
        status.zero_(); ws.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(); assert fn(ctypes.byref(p), st) == 0; e1.record()
        torch.cuda.synchronize()
        items = int(ws[base]); ncta = min(148, items)
        vals = ws[base + 2: base + 16].tolist()
        if which != "dq" and not any(vals):  # (the dQ kernel records the event trace only)
            raise SystemExit("no counters were written: build the instrumented library first "
                             "(python -m recir_b200.build -DB200_HSTU_PROFILING)")
        roles = {n: round(x * 64 / ncta / (2 if n.startswith("epi") else 1) / 1e3, 1)
                 for n, x in zip(names_f if which == "fwd" else names_b, vals) if n != "-" and x}
        res = {"ms": e0.elapsed_time(e1), "items": items, "kcycles_per_cta": roles}
        tr = status[16:].cpu().numpy().astype(np.int64) & 0xffffffff
        if which == "fwd":
            # epilogue thread 128, six events per key tile: wait_begin, scores ready, first chunk loaded, both
            # chunks converted and P stored (issue), P visible (+ next tile's scores awaited and its first load
            # issued), arrived; MMA warp, four per tile: K landed, S issued, P and V ready, PV issued
            epi = tr[4096:4096 + 4092].reshape(-1, 6)
            n = int((epi[:, 5] != 0).sum())
            d = lambda a, b: (a - b) & 0xffffffff
            E = epi[:n]
            ok = (E != 0).all(1)
            E = E[ok]
            ph = {"wait_scores": d(E[:, 1], E[:, 0]), "first_chunk_ld": d(E[:, 2], E[:, 1]),
                  "math_both_chunks": d(E[:, 3], E[:, 2]), "next_wait_and_st_wait": d(E[:, 4], E[:, 3]),
                  "arrive": d(E[:, 5], E[:, 4]), "tile_period": d(E[1:, 5], E[:-1, 5])}
            res["cta0_tiles"] = int(ok.sum())
            res["cta0_epilogue_cycles_median"] = {k: int(np.median(x[x < 1 << 20])) for k, x in ph.items()}
            res["cta0_epilogue_cycles_mean"] = {k: int(np.mean(x[x < 1 << 20])) for k, x in ph.items()}
            mma = tr[:4096].reshape(-1, 4)[:n]
            M = mma[(mma != 0).all(1)]
            mp = {"k_ok_to_S_issued": d(M[:, 1], M[:, 0]), "pv_wait_to_issued": d(M[:, 3], M[:, 2]),
                  "S_issued_to_pv_ready(prev)": d(M[1:, 2], M[1:, 1]), "tile_period": d(M[1:, 0], M[:-1, 0])}
            res["cta0_mma_cycles_median"] = {k: int(np.median(x[x < 1 << 20])) for k, x in mp.items()}
            res["cta0_span_cycles_per_tile"] = float(d(E[-1, 5], E[0, 0])) / max(len(E), 1)
        if which != "fwd":  # epilogue thread 128, six events per half tile: wait_begin s_ok ld_done st_issued arrived
            epi = tr[4096:4096 + 4092].reshape(-1, 6)
            n = int((epi[:, 1] != 0).sum())
            d = lambda a, b: (a - b) & 0xffffffff
            E = epi[:n]
            ph = {"wait_scores": d(E[:, 1], E[:, 0]), "tmem_ld": d(E[:, 2], E[:, 1]), "math_and_st_issue": d(E[:, 3], E[:, 2]),
                  "st_wait_and_arrive": d(E[:, 4], E[:, 3]), "period": d(E[1:, 0], E[:-1, 0])}
            res["cta0_half_tiles"] = n
            res["cta0_epilogue_cycles_median"] = {k: int(np.median(x[x < 1 << 20])) for k, x in ph.items()}
            mma = tr[:4096].reshape(-1, 4)[:n]
            res["cta0_span_cycles_per_half_tile"] = float(d(E[n - 1, 4], E[0, 0])) / max(n, 1)
        out[which] = res
        del keep
    print(json.dumps(out))


CASES = {"attn": main_attn, "rowwise": main_rowwise, "jagged": main_jagged, "gemm": main_gemm, "trace": main_trace}


def main(argv=None):
    import sys

    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in CASES:
        raise SystemExit(f"usage: bench.py --case {{{'|'.join(CASES)}}} [options]")
    import recir_b200  # noqa: F401  (registers the operators; fails loudly if the library is missing)

    CASES[argv[0]](argv[1:])


if __name__ == "__main__":
    main()
