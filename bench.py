#!/usr/bin/env python
"""Benchmark of the HSTU jagged attention hot path (forward + backward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N ... bench.py --gpus N ...
    python bench.py --case NAME ...        (single-purpose runners, see bench_cases.py)

Headline (``value``): one step = one forward + one backward of one STU-layer attention over one
batch of synthetic jagged sequences.  At N=1 the batch is the single-layer train-step shape
(B=64, H=4, D=128 bf16, history U[256,2048] + 64 targets: forward + backward with dO).  At N>1
the global batch holds 64*N sequences of the same distribution, split across ranks by
token-balanced sharding of whole sequences (no collective on the attention path), so the per-GPU
work stays fixed ("weak" scaling).

The same JSON line also carries, measured in the same process:

* ``stack8``    the 8-layer stack over the FIXED global batch of 1024 Zipf-length sequences, forward
                through all layers then backward through all layers, token-balanced over the N ranks
                (strong scaling: ``tokens_per_s`` at every N, per-rank times, imbalance);
* ``long_window`` the long skewed sequences with a 1024-token window (N=1 only);
* ``stu_layer`` the projections and row-wise kernels around the attention on the cfg4 token count (N=1 only);
* ``sustained`` the headline step looped for >= 2 s with the SM clock sampled meanwhile;
* ``per_rank_ms`` every rank's own time for the headline region;
* ``grad_check`` (N>1) per-sequence float64 checksums of dq, dk, dv of every rank's shard, exchanged
                over NCCL and compared on rank 0 with the un-sharded run of the same global batch;
* ``e2e``       the headline metric with pinned host inputs copied in and results copied out inside the
                timed region, and the plain-copy floor for the same bytes;
* ``roofline``  for the dominant kernel; ``cpu_baseline``: the reference operator on the host cores.

Prints ONE JSON line on rank 0.
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
WORKLOAD = "cfg2_stu_layer_fwd_bwd"
NOMINAL_BF16_TFLOPS = 2250.0
# dram__bytes_read.sum + dram__bytes_write.sum per launch from the committed ncu capture of the same
# B/H/D and length distribution (profiles/tc_kernels_cfg1_ncu_full.md names the build it was taken
# from), and that capture's token count.
NCU_CFG1_DRAM_BYTES = {"hstu_fwd_tc": 313.8e6, "hstu_bwd_dkv_tc": 1071.1e6, "hstu_bwd_dq_tc": 717.8e6}
NCU_CFG1_TOKENS = 78262
NCU_CAPTURE = "profiles/tc_kernels_cfg1_ncu_full.md"
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

    def __init__(self, index: int, period_ms: int = 20):
        self.index, self.rows, self.proc, self.thread, self.period_ms = index, [], None, None, period_ms

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
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
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 7:
                continue
            try:
                sm.append(float(r[0])); mx.append(float(r[1])); pw.append(float(r[2]))
            except ValueError:
                continue
            for n, val in zip(names, r[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(sm), "reasons": sorted(reasons)}


# --------------------------------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------------------------------

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


def headline_config(world: int, H: int, D: int, T_global: int, pairs_global: int, shard_info) -> dict:
    """The ``config`` object of the headline; both arms print the same keys."""
    return {"workload": WORKLOAD, "B_global": 64 * world, "H": H, "D": D, "T_global": T_global,
            "kept_pairs_per_head": pairs_global, "sharding": "token-balanced whole sequences, no collective",
            "shard": shard_info, "l2": "inputs+outputs per step (~640 MB/GPU) exceed the 126 MB L2"}


# --------------------------------------------------------------------------------------------------
# the reference operator on the host cores (reference arm and cpu_baseline leg: ONE procedure)
# --------------------------------------------------------------------------------------------------

class ReferenceSample:
    """A bounded sample of the N=1 headline batch for the reference's CPU operator: every 4th sequence by
    sorted length (16 of 64), bf16, forward + backward through autograd, all host threads."""

    def __init__(self):
        from oracle import ref_op
        from recir_b200 import workload
        self.ref_op = ref_op
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        self.batch = batch = build_global_batch(1)
        order = np.argsort(batch.lengths, kind="stable")
        self.sel = [int(i) for i in order[1::4]]
        nt = batch.num_targets.numpy()
        pairs = sum(workload.kept_pairs(int(batch.lengths[i]), int(nt[i])) for i in self.sel)
        self.H, self.D = batch.q.shape[1], batch.q.shape[2]
        self.flops = workload.useful_flops(pairs, self.H, self.D, self.D, backward=True)
        self.kw = dict(max_seq_len=batch.max_seq_len, alpha=batch.alpha, causal=True, num_targets=batch.num_targets)
        self.what = (f"{len(self.sel)} of {len(batch.lengths)} sequences (every 4th by sorted length) of the N=1 "
                     f"batch, bf16, fwd+bwd via autograd through the reference operator")

    def step(self):
        b = self.batch
        self.ref_op.ref_fwd_bwd_per_sequence(b.dout, b.q, b.k, b.v, b.seq_offsets, select=self.sel, **self.kw)

    def run(self, steps: int, warmup: int):
        """`warmup` untimed passes (thread pool, allocator, page cache), then `steps` timed ones."""
        for _ in range(warmup):
            self.step()
        per = []
        for _ in range(steps):
            t0 = time.perf_counter()
            self.step()
            per.append(time.perf_counter() - t0)
        total = float(sum(per))
        return {"value": self.flops * steps / total / 1e12, "seconds": total, "steps": steps,
                "step_s_min": float(min(per)), "step_s_median": float(np.median(per))}


def run_reference(args, rank: int):
    """Reference arm: the reference's own CPU operator on the host cores, same config and metric."""
    if rank != 0:
        return
    from oracle import ref_op
    from recir_b200 import workload
    if not ref_op.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref shared object missing"}), flush=True)
        return
    rs = ReferenceSample()
    warm = max(args.warmup, 2)
    r = rs.run(args.steps, warm)
    # same `config` keys and values as the other arm prints at this N (the timed sample is of the N=1 batch)
    from recir_b200 import sharding
    n = max(args.gpus, 1)
    g = rs.batch if n == 1 else build_global_batch(n)
    parts = sharding.token_balanced_partition(g.lengths, n)
    cfg = headline_config(n, rs.H, rs.D, g.total_tokens, workload.total_kept_pairs(g),
                          sharding.shard_summary(g.lengths, parts))
    sample = rs.what + f"; {r['steps']} timed pass(es) in {r['seconds']:.1f} s after {warm} warm-up(s)"
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["seconds"] / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": {"value": r["value"], "unit": UNIT, "cores": rs.cores, "kind": "reference", "sample": sample,
                         "step_s_min": r["step_s_min"], "step_s_median": r["step_s_median"]},
        "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(budget_s: float = 12.0):
    """Reference operator on the host cores over the same bounded sample, timed the same way as the
    reference arm (two warm-up passes, then whole passes until the budget is used)."""
    from oracle import ref_op
    if not ref_op.available():
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                "sample": "oracle/_ref shared object missing"}
    rs = ReferenceSample()
    rs.step()
    t0 = time.perf_counter()
    rs.step()
    one = time.perf_counter() - t0
    steps = int(min(40, max(3, budget_s / max(one, 1e-3))))
    r = rs.run(steps, 0)  # the two passes above were the warm-ups
    return {"value": r["value"], "unit": UNIT, "cores": rs.cores, "kind": "reference",
            "sample": rs.what + f"; {steps} timed pass(es) in {r['seconds']:.1f} s after 2 warm-ups",
            "step_s_min": r["step_s_min"], "step_s_median": r["step_s_median"]}


# --------------------------------------------------------------------------------------------------
# the 8-layer stack over the fixed global Zipf batch (strong scaling) and the gradient check
# --------------------------------------------------------------------------------------------------

class Stack8:
    """global B=1024, H=4, D=128 bf16, 8 independent attention layers run
    forward 0..7 then backward 7..0, sequences token-balanced over the ranks.  Lengths come from the
    seeded host generator (`workload.config4_lengths`); q/k/v/dO values are N(0, 0.1) / N(0, 0.01) drawn
    ON THE DEVICE (1.65 M tokens x 8 layers would take minutes on the host), global tensors first, then
    this rank's rows, so every N sees the same numbers."""

    LAYERS = 8

    def __init__(self, rank: int, world: int, dev):
        from recir_b200 import sharding, workload
        self.dev, self.rank, self.world = dev, rank, world
        hist, tg = workload.config4_lengths(1024)
        self.lengths = lengths = hist + tg
        self.targets = tg
        self.parts = sharding.token_balanced_partition(lengths, world)
        self.mine = mine = self.parts[rank]
        self.summary = sharding.shard_summary(lengths, self.parts)
        self.T_global = int(lengths.sum())
        self.H, self.D, self.N = 4, 128, 4096 + 128
        self.alpha = 1.0 / self.D ** 0.5
        goff = np.concatenate([[0], np.cumsum(lengths)])
        self.global_off = torch.as_tensor(goff, dtype=torch.int64, device=dev)
        self.off = sharding.local_offsets(lengths[mine]).to(dev)
        self.nt = torch.as_tensor(tg[mine], dtype=torch.int64, device=dev)
        self.T_local = int(lengths[mine].sum())
        if world == 1:
            self.rows = None
        else:  # global token rows of this rank's sequences, in local order
            starts = torch.as_tensor(goff[:-1][mine], dtype=torch.int64, device=dev)
            lens = torch.as_tensor(lengths[mine], dtype=torch.int64, device=dev)
            base = torch.repeat_interleave(starts - self.off[:-1], lens)
            self.rows = base + torch.arange(self.T_local, device=dev)
        self.pairs_global = sum(workload.kept_pairs(int(L), int(t)) for L, t in zip(lengths, tg))
        self.layers = [self._draw(layer) for layer in range(self.LAYERS)]
        self.args = (self.off, self.N, self.alpha, True, self.nt, 0, 0, None, 0)

    def _draw_global(self, layer: int):
        g = torch.Generator(device=self.dev).manual_seed(4 + layer)
        shape = (self.T_global, self.H, self.D)
        q, k, v = ((torch.randn(shape, generator=g, device=self.dev) * 0.1).to(torch.bfloat16) for _ in range(3))
        g2 = torch.Generator(device=self.dev).manual_seed(1000 + layer)
        do = (torch.randn(shape, generator=g2, device=self.dev) * 0.01).to(torch.bfloat16)
        return q, k, v, do

    def _draw(self, layer: int):
        t = self._draw_global(layer)
        if self.rows is None:
            return t
        return tuple(x.index_select(0, self.rows) for x in t)

    def step(self):
        fwd, bwd = torch.ops.recir.b200_hstu_attention_fwd, torch.ops.recir.b200_hstu_attention_bwd
        outs = None
        for q, k, v, _do in self.layers:
            outs = fwd(q, k, v, *self.args)
        for q, k, v, do in reversed(self.layers):
            outs = bwd(do, q, k, v, *self.args)
        return outs

    def flops_global(self) -> float:
        from recir_b200 import workload
        return self.LAYERS * workload.useful_flops(self.pairs_global, self.H, self.D, self.D, backward=True)

    # ---- gradient check -----------------------------------------------------------------------
    @staticmethod
    def _per_sequence_checksums(grads, off):
        """int64 [B, 6]: for each of dq, dk, dv the sum and the sum of squares of the raw 16-bit patterns of each
        sequence's rows.  Integer sums are exact and independent of the order of addition, so equal gradients
        give equal checksums bit for bit (a float64 sum would differ in its last bits with the order)."""
        B = off.numel() - 1
        lens = off[1:] - off[:-1]
        seg = torch.repeat_interleave(torch.arange(B, device=off.device), lens)
        out = torch.zeros(B, 6, dtype=torch.int64, device=off.device)
        for i, g in enumerate(grads):
            x = g.contiguous().view(torch.int16).flatten(1).to(torch.int64)
            out[:, 2 * i].index_add_(0, seg, x.sum(1))
            out[:, 2 * i + 1].index_add_(0, seg, (x * x).sum(1))
        return out

    def grad_check(self, dist):
        """Every rank: checksums of its shard's gradients (layer 0), placed at the global sequence indices,
        summed over NCCL; per-rank float64 squared norms gathered over NCCL; rank 0 also runs the un-sharded
        global batch and compares.  Sequences are independent and the kernels deterministic, so the match is
        exact."""
        q, k, v, do = self.layers[0]
        grads = torch.ops.recir.b200_hstu_attention_bwd(do, q, k, v, *self.args)
        local = self._per_sequence_checksums(grads, self.off)
        B = len(self.lengths)
        table = torch.zeros(B, 6, dtype=torch.int64, device=self.dev)
        table[torch.as_tensor(self.mine, device=self.dev)] = local
        norms = torch.stack([g.double().pow(2).sum() for g in grads])
        if self.world > 1:
            dist.all_reduce(table)  # every sequence belongs to exactly one rank
            gathered = [torch.zeros_like(norms) for _ in range(self.world)]
            dist.all_gather(gathered, norms)
        else:
            gathered = [norms]
        if self.rank != 0:
            return None
        gq, gk, gv, gdo = self._draw_global(0)
        gnt = torch.as_tensor(self.targets, dtype=torch.int64, device=self.dev)
        ref = torch.ops.recir.b200_hstu_attention_bwd(gdo, gq, gk, gv, self.global_off, self.N, self.alpha, True, gnt,
                                                      0, 0, None, 0)
        want = self._per_sequence_checksums(ref, self.global_off)
        bad = int((table != want).any(1).sum().item())
        ref_norms = torch.stack([g.double().pow(2).sum() for g in ref])
        sum_ranks = torch.stack(gathered).sum(0)
        return {"what": "per-sequence exact integer checksums (sum and sum of squares of the 16-bit patterns) of dq, dk, dv "
                        "of stack layer 0: every rank's shard against the un-sharded run of the global batch on rank 0",
                "collective": "nccl all_reduce + all_gather" if self.world > 1 else "none (one rank)",
                "sequences": B, "mismatched_sequences": bad,
                "squared_norms_unsharded": [float(x) for x in ref_norms],
                "squared_norms_rel_diff": float(((sum_ranks - ref_norms).abs() / ref_norms.clamp_min(1e-300)).max().item()),
                "ok": bad == 0}


# --------------------------------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="headline, roofline and e2e only")
    ap.add_argument("--grad-check", dest="grad_check", action="store_true", default=None)
    ap.add_argument("--no-grad-check", dest="grad_check", action="store_false")
    ap.add_argument("--case", default=None, help="run one of the single-purpose runners of bench_cases.py instead")
    argv = sys.argv[1:]
    if "--case" in argv:  # everything else on the line belongs to the runner (its options may share names with ours)
        i = argv.index("--case")
        if i + 1 >= len(argv):
            ap.error("--case needs a name")
        import bench_cases
        bench_cases.main([argv[i + 1], *argv[:i], *argv[i + 2:]])
        return
    args = ap.parse_args(argv)
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
    if args.grad_check is None:
        args.grad_check = world > 1

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

    def all_ranks(x: float) -> list:
        if world == 1:
            return [x]
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [float(y.item()) for y in out]

    def timed_region(fn, steps: int):
        """barrier + synchronize, `steps` calls between two events on the launching stream, barrier +
        synchronize; returns this rank's milliseconds."""
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        barrier()
        return e0.elapsed_time(e1)

    # ------------------------------------------------------------ resident (value)
    for _ in range(warm):
        step_resident()
    # only rank 0 reports clocks, so only rank 0 runs a sampler (of its own GPU)
    sampler = ClockSampler(local_rank) if rank == 0 else None
    barrier()
    if sampler is not None:
        sampler.start()
    launches0 = ops.launch_counter
    my_ms = timed_region(step_resident, args.steps)
    launches = ops.launch_counter - launches0
    ms_total = max_over_ranks(my_ms)
    per_rank_ms = [x / args.steps for x in all_ranks(my_ms)]
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

    # One call at a time with the L2 written over in between (a 256 MB fill): the cold-cache variant.
    def time_cold(fn, rounds=7):
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        out = []
        for _ in range(rounds):
            flush.fill_(1)
            e[0].record()
            fn()
            e[1].record()
            torch.cuda.synchronize()
            out.append(e[0].elapsed_time(e[1]))
        del flush
        return float(np.median(out[1:]))

    run_fwd = lambda: torch.ops.recir.b200_hstu_attention_fwd(d["q"], d["k"], d["v"], *args_op)
    run_bwd = lambda: torch.ops.recir.b200_hstu_attention_bwd(d["do"], d["q"], d["k"], d["v"], *args_op)
    fwd_ms, bwd_ms = time_pass(run_fwd), time_pass(run_bwd)
    ops.set_backward_passes(dkv=True, dq=False, timing_only=True)
    dkv_ms = time_pass(run_bwd, rounds=11)  # (the dominant kernel of `roofline`, and the noisiest: more samples)
    ops.set_backward_passes(dkv=False, dq=True, timing_only=True)
    dq_ms = time_pass(run_bwd)
    # the same two kernels in the recomputing form of the backward (no dS tiles written or read)
    ops.set_backward_passes(dkv=True, dq=False)
    dkv_plain_ms = float(np.median(time_pass(run_bwd)))
    ops.set_backward_passes(dkv=False, dq=True)
    dq_plain_ms = float(np.median(time_pass(run_bwd)))
    ops.set_backward_passes(True, True)
    ops.set_recompute_dq(True)
    bwd_plain_ms = float(np.median(time_pass(run_bwd)))
    ops.set_recompute_dq(False)
    cold = None if args.no_extras else {"fwd_ms": time_cold(run_fwd), "bwd_ms": time_cold(run_bwd),
                                        "note": "one call at a time, a 256 MB fill before each (L2 holds 126 MB)"}
    value = flops_step * args.steps / (ms_total * 1e-3) / 1e12
    clocks = sampler.stop() if sampler is not None else None  # over the headline and the per-pass timed regions

    # ------------------------------------------------------------ sustained: the same step for >= 2 s
    sustained = None
    if not args.no_extras:
        n_sus = max(args.steps, int(2200.0 / max(ms_total / args.steps, 1e-3)))
        s2 = ClockSampler(local_rank, period_ms=50) if rank == 0 else None
        barrier()
        if s2 is not None:
            s2.start()
        sus_ms = max_over_ranks(timed_region(step_resident, n_sus))
        c2 = s2.stop() if s2 is not None else None
        sus_value = flops_step * n_sus / (sus_ms * 1e-3) / 1e12
        sustained = {"steps": n_sus, "seconds": sus_ms * 1e-3, "ms_per_step": sus_ms / n_sus, "value": sus_value,
                     "unit": UNIT, "clocks": c2,
                     "note": "same step as `value`, looped back to back; `value` itself is a burst of "
                             f"{args.steps} steps, and the per-pass times of `roofline` are bursts of 10 calls"}

    # ------------------------------------------------------------ end to end (host buffers)
    # Public host-memory API: chunks of whole sequences stream through copy-in / compute / copy-out
    # streams (recir_b200.HostPipeline), so both PCIe directions overlap with the kernels.
    out_host = {k: torch.empty_like(host[k]).pin_memory() for k in ("q", "k", "v", "do")}
    pipe = recir_b200.HostPipeline(local["off"], local["nt"], H, D, D, torch.bfloat16, batch.max_seq_len,
                                   batch.alpha, n_chunks=12, device=dev)

    def step_e2e():
        pipe.run(host["q"], host["k"], host["v"], host["do"], out_host["do"], out_host["q"], out_host["k"],
                 out_host["v"])

    for _ in range(3):
        step_e2e()
    e2e_ms = max_over_ranks(timed_region(step_e2e, args.steps))
    e2e_value = flops_step * args.steps / (e2e_ms * 1e-3) / 1e12
    bytes_local = sum(host[k].numel() * host[k].element_size() for k in host)
    # plain-copy floor: the same bytes in and out on two streams, no kernels, all ranks at once
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def copy_only():
        with torch.cuda.stream(s_in):
            for kname in host:
                d[kname].copy_(host[kname], non_blocking=True)
        with torch.cuda.stream(s_out):
            for kname in host:
                out_host[kname].copy_(d[kname], non_blocking=True)

    def copy_step():
        cur = torch.cuda.current_stream()
        s_in.wait_stream(cur); s_out.wait_stream(cur)
        copy_only()
        cur.wait_stream(s_in); cur.wait_stream(s_out)

    for _ in range(2):
        copy_step()
    n_copy = max(3, min(args.steps, 10))
    copy_ms = max_over_ranks(timed_region(copy_step, n_copy)) / n_copy
    if world > 1:
        tb = torch.tensor([float(bytes_local)], dtype=torch.float64, device=dev)
        dist.all_reduce(tb)
        bytes_global = int(tb.item())
    else:
        bytes_global = bytes_local
    del pipe
    out_host.clear()

    # ------------------------------------------------------------ long skewed sequences (N=1 only)
    long_window = None
    if not args.no_extras and world == 1:
        b3 = workload.config3()
        t3 = {k: getattr(b3, k).to(dev) for k in ("q", "k", "v", "dout")}
        a3 = (b3.seq_offsets.to(dev), b3.max_seq_len, b3.alpha, True, b3.num_targets.to(dev), b3.contextual_seq_len,
              b3.max_attn_len, None, 0)
        f3 = lambda: torch.ops.recir.b200_hstu_attention_fwd(t3["q"], t3["k"], t3["v"], *a3)
        g3 = lambda: torch.ops.recir.b200_hstu_attention_bwd(t3["dout"], t3["q"], t3["k"], t3["v"], *a3)
        for _ in range(3):
            f3(); g3()
        fm, gm = float(np.median(time_pass(f3))), float(np.median(time_pass(g3)))
        p3 = workload.total_kept_pairs(b3)
        H3, D3 = b3.q.shape[1], b3.q.shape[2]
        long_window = {
            "workload": "cfg3_long_window_fwd_bwd", "B": len(b3.lengths), "H": H3, "D": D3, "T": b3.total_tokens,
            "max_len": int(b3.lengths.max()), "max_attn_len": b3.max_attn_len, "contextual_seq_len": b3.contextual_seq_len,
            "kept_pairs_per_head": p3, "fwd_ms": fm, "bwd_ms": gm,
            "fwd_tflops": workload.useful_flops(p3, H3, D3, D3, False) / (fm * 1e-3) / 1e12,
            "bwd_tflops": workload.useful_flops(p3, H3, D3, D3, True, forward=False) / (gm * 1e-3) / 1e12,
            "fwd_bwd_tflops": workload.useful_flops(p3, H3, D3, D3, True) / ((fm + gm) * 1e-3) / 1e12,
            "timing": "median of 5 samples of 10 calls issued back to back"}
        t3.clear()

    # ------------------------------------------------------------ 8-layer stack, fixed global batch
    stack8, grad_check = None, None
    if not args.no_extras:
        d.clear()
        host.clear()
        torch.cuda.empty_cache()
        st = Stack8(rank, world, dev)
        for _ in range(2):
            st.step()
        n8 = 5
        l0 = ops.launch_counter
        my8 = timed_region(st.step, n8) / n8
        launches8 = (ops.launch_counter - l0) // n8
        ranks8 = all_ranks(my8)
        t8 = max(ranks8)
        stack8 = {
            "workload": "cfg4_stack8_fwd_bwd", "scaling": "strong", "layers": st.LAYERS, "B_global": len(st.lengths),
            "H": st.H, "D": st.D, "T_global": st.T_global, "kept_pairs_per_head_per_layer": st.pairs_global,
            "steps": n8, "ms_per_step": t8, "tokens_per_s": st.T_global / (t8 * 1e-3),
            "token_layers_per_s": st.T_global * st.LAYERS / (t8 * 1e-3),
            "useful_tflops": st.flops_global() / (t8 * 1e-3) / 1e12,
            "per_rank_ms": ranks8, "token_imbalance": st.summary["token_imbalance"],
            "cost_imbalance": st.summary["cost_imbalance"], "tokens_per_rank": st.summary["tokens"],
            "launches_per_step_per_rank": launches8,
            "data": "lengths from the seeded host generator; q/k/v/dO drawn on the device per layer (seeds 4+layer, "
                    "1000+layer), global tensors first, then this rank's rows"}
        if args.grad_check:
            grad_check = st.grad_check(dist)
        del st

    # ------------------------------------------------------------ the STU layer around the attention (N=1 only)
    stu_layer = None
    if not args.no_extras and world == 1:
        import argparse as _ap
        import bench_cases
        torch.cuda.empty_cache()
        rows = 1650165  # tokens of the cfg4 batch (one layer)
        stu_layer = {
            "note": "the layer's other operators on the cfg4 token count, bf16, embedding width 512: projections "
                    "(u|v|q|k: K = 512 -> N = 2048; fp8 output projection sizes) against the vendor GEMM, row-wise "
                    "kernels as algorithmic GB/s; same code as `bench.py --case gemm` / `--case rowwise`",
            "projection": bench_cases.gemm_numbers(_ap.Namespace(rows=rows, k=512, n=2048, iters=5, warmup=2)),
            "rowwise": bench_cases.rowwise_numbers(_ap.Namespace(rows=rows, cols=512, iters=5, warmup=2)),
        }
        torch.cuda.empty_cache()

    # ------------------------------------------------------------ report
    if rank == 0:
        peaks = measured_peaks()
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
            "traffic_source": NCU_CAPTURE,
            # tensors of T*H*D 16-bit elements: fwd q,k,v read + o written; dK/dV pass q,k,v,dO read + dk,dv
            # written; dQ pass k read + dq written.  The dS tiles that the dK/dV pass writes and the dQ pass
            # reads (32 KB per kept 128x128 tile) are this design's own traffic on top: see `traffic`.
            "algorithmic_bytes": {"hstu_fwd_tc": 4, "hstu_bwd_dkv_tc": 6, "hstu_bwd_dq_tc": 2}[dom]
            * local_tokens * H * D * 2,
            "kernels": {"hstu_bwd_dq_tc": "hstu_bwd_dq_stored_tc: dQ from the dS tiles the dK/dV pass stored "
                                          "(C-ABI default; B200_HSTU_FLAG_BWD_RECOMPUTE_DQ selects the recomputing kernel)"},
            "per_kernel_ms": {k: v[1] for k, v in kernels.items()},
            "per_kernel_tflops": {k: v[0] / (v[1] * 1e-3) / 1e12 for k, v in kernels.items()},
            "fwd_ms": fwd_med, "bwd_ms": bwd_med,
            "fwd_tflops": workload.useful_flops(local_pairs, H, D, D, backward=False) / (fwd_med * 1e-3) / 1e12,
            "bwd_tflops": workload.useful_flops(local_pairs, H, D, D, backward=True, forward=False) / (bwd_med * 1e-3) / 1e12,
            "timing": "per-pass and per-kernel times: median of 5 samples (dK/dV kernel: 11) of 10 calls issued back to back (a burst, "
                      "each pass with its work-list kernel); they need not add up to ms_per_step, which is "
                      "forward and backward alternating",
            "cold_l2": cold,
            # The dominant kernel also writes the dS tiles (32 KB per kept tile) that spare the dQ pass two of its
            # three GEMMs and its transcendental pass: the same pair of kernels without the tiles, for comparison.
            "recomputing_backward": {
                "hstu_bwd_dkv_tc_ms": dkv_plain_ms, "hstu_bwd_dq_tc_ms": dq_plain_ms, "bwd_ms": bwd_plain_ms,
                "hstu_bwd_dkv_tc_frac": kernels["hstu_bwd_dkv_tc"][0] / (dkv_plain_ms * 1e-3) / 1e12 / peak,
                "note": "B200_HSTU_FLAG_BWD_RECOMPUTE_DQ: dK/dV kernel without the tile stores, dQ kernel "
                        "recomputing S and dP; the default backward is `bwd_ms` above"},
        }
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": headline_config(world, H, D, T_global, pairs_global, shard_info),
            "tokens_per_s": T_global * args.steps / (ms_total * 1e-3),
            "per_rank_ms": {"min": min(per_rank_ms), "median": float(np.median(per_rank_ms)), "max": max(per_rank_ms),
                            "all": per_rank_ms},
            "pct_of_peak": {"nominal_2250": 100 * value / world / NOMINAL_BF16_TFLOPS,
                            "measured_burst": 100 * value / world / peaks["bf16_tflops"],
                            "measured_sustained": 100 * value / world / peaks["bf16_tflops_sustained"]},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": bytes_global,
                    "d2h_bytes_per_step": bytes_global, "ms_per_step": e2e_ms / args.steps,
                    "copy_floor_ms": copy_ms,
                    "copy_floor_note": "the same bytes host->device and device->host on two streams from pinned "
                                       "memory, no kernels, every rank at once (max over ranks)"},
            "gpu_launches": launches * world,
            "roofline": roofline,
        }
        if sustained is not None:
            sustained["pct_of_measured_sustained"] = 100 * sustained["value"] / world / peaks["bf16_tflops_sustained"]
            line["sustained"] = sustained
        if long_window is not None:
            line["long_window"] = long_window
        if stack8 is not None:
            line["stack8"] = stack8
        if grad_check is not None:
            line["grad_check"] = grad_check
        if stu_layer is not None:
            line["stu_layer"] = stu_layer
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
