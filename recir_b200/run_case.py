"""Run one benchmark configuration of the HSTU attention on the current GPU and print timings.

    python -m recir_b200.run_case --config cfg1 --passes fwd --iters 5

Configurations: cfg0 (smoke shape, fp32), cfg1 (B=64, H=4, D=128 bf16), cfg3 (long skewed
sequences, sliding window + contextual prefix), cfg4 (one layer of the Zipf batch, optionally
the shard of one rank).  ``--passes`` is ``fwd``, ``bwd`` or ``both``.  This is also the
command profilers are pointed at: it launches nothing but the library's kernels after the
inputs have been copied to the device.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import ops, sharding, workload


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="cfg1")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--passes", default="both", choices=["fwd", "bwd", "both"])
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--rank", type=int, default=0)
    ap.add_argument("--world", type=int, default=1)
    ap.add_argument("--simt", action="store_true", help="use the CUDA-core kernels")
    args = ap.parse_args()

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
    q, k, v, do = (x.to(dev) for x in (bt.q, bt.k, bt.v, bt.dout))
    off = bt.seq_offsets.to(dev)
    nt = None if bt.num_targets is None else bt.num_targets.to(dev)
    a = (off, bt.max_seq_len, bt.alpha, bt.causal, nt, bt.contextual_seq_len, bt.max_attn_len, None,
         bt.full_attn_size)
    ops.set_force_simt(args.simt)
    H, Dq, Dv = q.shape[1], q.shape[2], v.shape[2]
    pairs = workload.total_kept_pairs(bt)

    def fwd():
        return torch.ops.recir.b200_hstu_attention_fwd(q, k, v, *a)

    def bwd():
        return torch.ops.recir.b200_hstu_attention_bwd(do, q, k, v, *a)

    res = {"config": bt.name, "T": bt.total_tokens, "B": len(bt.lengths), "H": H, "D": Dq,
           "kept_pairs_per_head": pairs}
    for name, fn, fl in (("fwd", fwd, workload.useful_flops(pairs, H, Dq, Dv, False)),
                         ("bwd", bwd, workload.useful_flops(pairs, H, Dq, Dv, True, forward=False))):
        if args.passes not in (name, "both"):
            continue
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(args.iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        med = float(np.median(times))
        res[name] = {"ms_median": med, "ms_min": float(min(times)), "useful_tflops": fl / (med * 1e-3) / 1e12}
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


if __name__ == "__main__":
    main()
