#!/usr/bin/env python
"""Benchmark of the HSTU jagged attention hot path (forward + backward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N ... bench.py --gpus N ...

One step = one forward + one backward of one STU-layer attention over one batch of
synthetic jagged sequences.  At N=1 the batch is the single-layer train-step shape
(B=64, H=4, D=128 bf16, history U[256,2048] + 64 targets: forward + backward with dO).
At N>1 the global batch holds 64*N sequences of the same distribution, split across ranks
by token-balanced sharding of whole sequences (no collective on the attention path), so
the per-GPU work stays fixed ("weak" scaling).

Prints ONE JSON line on rank 0.  ``value`` is the whole-job useful (masked) TFLOP/s with
inputs resident in HBM; ``e2e`` is the same metric with pinned host inputs copied in and
results copied out inside the timed region; ``roofline`` is for the dominant kernel;
``cpu_baseline`` is the reference operator on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import numpy as np
import torch

METRIC = "hstu_attn_fwd_bwd_useful_tflops"
UNIT = "TFLOP/s"
NOMINAL_BF16_TFLOPS = 2250.0
# dram__bytes_read.sum + dram__bytes_write.sum per launch from the committed ncu capture of the same
# B/H/D and length distribution (profiles/tc_kernels_cfg1_ncu_full.md), and that capture's token count.
NCU_CFG1_DRAM_BYTES = {"hstu_fwd_tc": 315.6e6, "hstu_bwd_dkv_tc": 471.1e6, "hstu_bwd_dq_tc": 405.8e6}
NCU_CFG1_TOKENS = 78262
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["_source"] = "measured"
        return d
    d = dict(FALLBACK_PEAKS)
    d["_source"] = "fallback"
    return d


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons for one GPU while a region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc, self.thread = index, [], None, None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 7:
                continue
            try:
                sm.append(float(r[0])); mx.append(float(r[1]))
            except ValueError:
                continue
            for n, val in zip(names, r[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def build_global_batch(n_gpus: int):
    from recir_b200 import workload
    return workload.config1(dtype=torch.bfloat16, batch=64 * n_gpus, with_dout=True)


def local_shard(batch, rank: int, world: int):
    """Token-balanced shard of whole sequences for this rank (host tensors)."""
    from recir_b200 import sharding
    lengths = batch.lengths
    parts = sharding.token_balanced_partition(lengths, world)
    mine = parts[rank]
    take = lambda t: sharding.gather_rows(t, batch.seq_offsets, mine)
    local = dict(q=take(batch.q), k=take(batch.k), v=take(batch.v), do=take(batch.dout),
                 off=sharding.local_offsets(lengths[mine]), nt=batch.num_targets[torch.as_tensor(mine)])
    return local, sharding.shard_summary(lengths, parts)


def run_reference(args, rank: int):
    """Reference arm: the reference's own CPU operator on the host cores, same config and metric."""
    if rank != 0:
        return
    from oracle import ref_op
    from recir_b200 import workload
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    batch = build_global_batch(1)
    kept = workload.total_kept_pairs(batch)
    # bounded sample per step: every 4th sequence by sorted length (16 of 64), bf16, fwd+bwd
    order = np.argsort(batch.lengths, kind="stable")
    sel = [int(i) for i in order[1::4]]
    nt = batch.num_targets.numpy()
    pairs = sum(workload.kept_pairs(int(batch.lengths[i]), int(nt[i])) for i in sel)
    H, D = batch.q.shape[1], batch.q.shape[2]
    flops = workload.useful_flops(pairs, H, D, D, backward=True)
    kw = dict(max_seq_len=batch.max_seq_len, alpha=batch.alpha, causal=True, num_targets=batch.num_targets)

    def step():
        ref_op.ref_fwd_bwd_per_sequence(batch.dout, batch.q, batch.k, batch.v, batch.seq_offsets,
                                        select=sel, **kw)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = flops * args.steps / dt / 1e12
    sample = (f"{len(sel)} of {len(batch.lengths)} sequences (every 4th by sorted length) of the N=1 batch, "
              f"bf16, fwd+bwd via autograd through the reference operator")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "cfg2_stu_layer_fwd_bwd", "B": 64, "H": H, "D": D,
                   "total_kept_pairs_per_head": kept, "device": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(batch, budget_s: float = 20.0):
    """Reference operator on the host cores over a bounded sample of the N=1 workload."""
    from oracle import ref_op
    from recir_b200 import workload
    if not ref_op.available():
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                "sample": "oracle/_ref shared object missing"}
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    order = np.argsort(batch.lengths, kind="stable")
    sel = [int(i) for i in order[1::4]]
    nt = batch.num_targets.numpy()
    pairs = sum(workload.kept_pairs(int(batch.lengths[i]), int(nt[i])) for i in sel)
    H, D = batch.q.shape[1], batch.q.shape[2]
    flops = workload.useful_flops(pairs, H, D, D, backward=True)
    kw = dict(max_seq_len=batch.max_seq_len, alpha=batch.alpha, causal=True, num_targets=batch.num_targets)
    run = lambda: ref_op.ref_fwd_bwd_per_sequence(batch.dout, batch.q, batch.k, batch.v,
                                                  batch.seq_offsets, select=sel, **kw)
    run()  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        run()
        reps += 1
        dt = time.perf_counter() - t0
        if dt > budget_s / 2 or reps >= 40:
            break
    return {"value": flops * reps / dt / 1e12, "unit": UNIT, "cores": cores, "kind": "reference",
            "sample": f"{len(sel)} of {len(batch.lengths)} sequences (every 4th by sorted length), bf16, "
                      f"fwd+bwd, {reps} pass(es) in {dt:.1f} s after one warm-up"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 0)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("launch with torch.distributed.run --nproc-per-node N for --gpus N > 1")
        args.gpus = world
    warm = max(args.warmup, 3)

    import torch.distributed as dist
    import recir_b200
    from recir_b200 import ops, workload, _lib

    _lib.load()  # fail loudly if the CUDA library is missing
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", device_id=dev)

    batch = build_global_batch(world)
    local, shard_info = local_shard(batch, rank, world)
    H, D = batch.q.shape[1], batch.q.shape[2]
    pairs_global = workload.total_kept_pairs(batch)
    flops_step = workload.useful_flops(pairs_global, H, D, D, backward=True)
    flops_fwd = workload.useful_flops(pairs_global, H, D, D, backward=False)
    T_global = batch.total_tokens

    host = {k: local[k].pin_memory() for k in ("q", "k", "v", "do")}
    off, nt = local["off"].to(dev), local["nt"].to(dev)
    d = {k: host[k].to(dev, non_blocking=True) for k in host}
    args_op = (off, batch.max_seq_len, batch.alpha, True, nt, 0, 0, None, 0)

    def step_resident():
        o = torch.ops.recir.b200_hstu_attention_fwd(d["q"], d["k"], d["v"], *args_op)
        g = torch.ops.recir.b200_hstu_attention_bwd(d["do"], d["q"], d["k"], d["v"], *args_op)
        return o, g

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ------------------------------------------------------------ resident (value)
    for _ in range(warm):
        step_resident()
    sampler = ClockSampler(local_rank)
    barrier()
    sampler.start()
    launches0 = ops.launch_counter
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step_resident()
    ev1.record()
    barrier()
    launches = ops.launch_counter - launches0
    ms_total = max_over_ranks(ev0.elapsed_time(ev1))
    # per-kernel device time (same stream), for the roofline of the dominant kernel: each pass is
    # issued `reps` times back to back between two events so that the host's launch latency does not
    # sit inside the measurement; the backward kernels also run one at a time (C-ABI flag).
    def time_pass(fn, reps=10, rounds=5):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        out = []
        for r in range(rounds + 1):
            e[0].record()
            for _ in range(reps):
                fn()
            e[1].record()
            torch.cuda.synchronize()
            if r > 0:
                out.append(e[0].elapsed_time(e[1]) / reps)
        return out

    run_fwd = lambda: torch.ops.recir.b200_hstu_attention_fwd(d["q"], d["k"], d["v"], *args_op)
    run_bwd = lambda: torch.ops.recir.b200_hstu_attention_bwd(d["do"], d["q"], d["k"], d["v"], *args_op)
    fwd_ms, bwd_ms = time_pass(run_fwd), time_pass(run_bwd)
    ops.set_backward_passes(dkv=True, dq=False)
    dkv_ms = time_pass(run_bwd)
    ops.set_backward_passes(dkv=False, dq=True)
    dq_ms = time_pass(run_bwd)
    ops.set_backward_passes(True, True)
    value = flops_step * args.steps / (ms_total * 1e-3) / 1e12

    # ------------------------------------------------------------ end to end (host buffers)
    # Public host-memory API: chunks of whole sequences stream through copy-in / compute / copy-out
    # streams (recir_b200.HostPipeline), so both PCIe directions overlap with the kernels.
    out_host = {k: torch.empty_like(host[k]).pin_memory() for k in ("q", "k", "v", "do")}
    pipe = recir_b200.HostPipeline(local["off"], local["nt"], H, D, D, torch.bfloat16, batch.max_seq_len,
                                   batch.alpha, n_chunks=16, device=dev)

    def step_e2e():
        pipe.run(host["q"], host["k"], host["v"], host["do"], out_host["do"], out_host["q"], out_host["k"],
                 out_host["v"])

    for _ in range(3):
        step_e2e()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step_e2e()
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    clocks = sampler.stop()  # sampled over the resident, per-pass and end-to-end timed regions
    e2e_value = flops_step * args.steps / (e2e_ms * 1e-3) / 1e12
    bytes_local = sum(host[k].numel() * host[k].element_size() for k in host)
    if world > 1:
        tb = torch.tensor([float(bytes_local)], dtype=torch.float64, device=dev)
        dist.all_reduce(tb)
        bytes_global = int(tb.item())
    else:
        bytes_global = bytes_local

    # ------------------------------------------------------------ report
    if rank == 0:
        peaks = measured_peaks()
        uses_tc = {}
        p = _lib.B200HstuParams()
        fwd_med, bwd_med = float(np.median(fwd_ms)), float(np.median(bwd_ms))
        local_pairs = pairs_global / world  # token-balanced shards of one distribution
        # One launch of each main kernel: useful flops (2*D per kept pair per GEMM: forward 2 GEMMs,
        # dK/dV pass 4 -- S, dP, dV, dK -- and the dQ pass 1; its recomputed S and dP count as overhead)
        # over the kernel's own device time.
        gemm = 2.0 * local_pairs * H * D
        kernels = {
            "hstu_fwd_tc": (2 * gemm, fwd_med, NCU_CFG1_DRAM_BYTES["hstu_fwd_tc"]),
            "hstu_bwd_dkv_tc": (4 * gemm, float(np.median(dkv_ms)), NCU_CFG1_DRAM_BYTES["hstu_bwd_dkv_tc"]),
            "hstu_bwd_dq_tc": (1 * gemm, float(np.median(dq_ms)), NCU_CFG1_DRAM_BYTES["hstu_bwd_dq_tc"]),
        }
        dom = max(kernels, key=lambda k: kernels[k][1])
        dom_flops, dom_ms, dom_traffic = kernels[dom]
        achieved = dom_flops / (dom_ms * 1e-3) / 1e12
        peak = peaks["bf16_tflops"]
        local_tokens = T_global / world
        roofline = {
            "bound": "tensor", "kernel": dom,
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{peaks['_source']} burst bf16 GEMM",
            # DRAM bytes of one launch from the ncu capture of the same shapes at T=78262 tokens,
            # scaled by tokens (traffic grows with the token count at a fixed length distribution)
            "traffic": dom_traffic * local_tokens / NCU_CFG1_TOKENS,
            # fwd: q,k,v read + o written; dK/dV pass: q,k,v,dO read + dk,dv written; dQ pass: q,k,v,dO read + dq written
            "algorithmic_bytes": {"hstu_fwd_tc": 4, "hstu_bwd_dkv_tc": 6, "hstu_bwd_dq_tc": 5}[dom]
            * local_tokens * H * D * 2,
            "per_kernel_ms": {k: v[1] for k, v in kernels.items()},
            "per_kernel_tflops": {k: v[0] / (v[1] * 1e-3) / 1e12 for k, v in kernels.items()},
            "fwd_ms": fwd_med, "bwd_ms": bwd_med,
            "fwd_tflops": workload.useful_flops(local_pairs, H, D, D, backward=False) / (fwd_med * 1e-3) / 1e12,
            "bwd_tflops": workload.useful_flops(local_pairs, H, D, D, backward=True, forward=False) / (bwd_med * 1e-3) / 1e12,
        }
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2_stu_layer_fwd_bwd", "B_global": 64 * world, "H": H, "D": D,
                       "T_global": T_global, "kept_pairs_per_head": pairs_global,
                       "sharding": "token-balanced whole sequences, no collective",
                       "shard": shard_info, "l2": "inputs+outputs per step (~640 MB/GPU) exceed the 126 MB L2"},
            "tokens_per_s": T_global * args.steps / (ms_total * 1e-3),
            "pct_of_peak": {"nominal_2250": 100 * value / world / NOMINAL_BF16_TFLOPS,
                            "measured_burst": 100 * value / world / peaks["bf16_tflops"],
                            "measured_sustained": 100 * value / world / peaks["bf16_tflops_sustained"]},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": bytes_global,
                    "d2h_bytes_per_step": bytes_global, "ms_per_step": e2e_ms / args.steps},
            "gpu_launches": launches * world,
            "roofline": roofline,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(batch)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
