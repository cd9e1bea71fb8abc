"""World-size-2 gloo test of the multi-GPU host logic: every rank plans the same partition,
owns whole sequences, and the union of the rank-local problems is the global problem; the
cross-rank checksum gather that the benchmark's gradient check uses works over gloo."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    from recir_b200 import sharding, workload
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    hist, tg = workload.config4_lengths(64)
    lengths = hist + tg
    parts = sharding.token_balanced_partition(lengths, world)
    mine = parts[rank]
    off = sharding.local_offsets(lengths[mine])
    local = torch.tensor([float(lengths[mine].sum()), float(len(mine)), float(off[-1])], dtype=torch.float64)
    gathered = [torch.zeros_like(local) for _ in range(world)]
    dist.all_gather(gathered, local)
    dist.barrier()
    if rank == 0:
        q.put([g.tolist() for g in gathered] + [[float(lengths.sum()), float(len(lengths))]])
    dist.destroy_process_group()


def test_two_rank_partition_is_consistent_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 2000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (t0, n0, o0), (t1, n1, o1), (tot, nseq) = res
    assert t0 + t1 == tot and n0 + n1 == nseq
    assert o0 == t0 and o1 == t1
    assert abs(t0 - t1) / tot < 0.02
