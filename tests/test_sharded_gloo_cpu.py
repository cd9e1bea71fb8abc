"""World-size-2 gloo tests of the multi-GPU host logic: every rank plans the same partition, owns whole
sequences, and the union of the rank-local problems is the global problem; and the exchange behind the
benchmark's cross-rank gradient check (per-sequence integer checksums placed at global sequence indices,
summed over the process group, compared with the un-sharded tensors on rank 0) finds equal gradients equal
and a single flipped bit unequal."""
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


def _checksum_worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import bench
    from recir_b200 import sharding, workload
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    hist, tg = workload.config4_lengths(48)
    lengths = np.minimum(hist + tg, 300)
    goff = sharding.local_offsets(lengths)
    g = torch.Generator().manual_seed(3)
    T = int(lengths.sum())
    grads = [torch.randn(T, 2, 8, generator=g).to(torch.bfloat16) for _ in range(3)]  # the "un-sharded" gradients
    mine = sharding.token_balanced_partition(lengths, world)[rank]
    local = [sharding.gather_rows(x, goff, mine).clone() for x in grads]
    if rank == 1:
        local[1].view(torch.int16)[5, 1, 3] ^= 1  # one bit of one element on one rank
    check = bench.Stack8._per_sequence_checksums
    table = torch.zeros(len(lengths), 6, dtype=torch.int64)
    table[torch.as_tensor(mine)] = check(local, sharding.local_offsets(lengths[mine]))
    dist.all_reduce(table)
    if rank == 0:
        want = check(grads, goff)
        bad = (table != want).any(1).nonzero().flatten().tolist()
        q.put((bad, int(mine_of(lengths, world, 1)[_seq_of_row(lengths, mine_of(lengths, world, 1), 5)])))
    dist.barrier()
    dist.destroy_process_group()


def mine_of(lengths, world, rank):
    sys.path.insert(0, ROOT)
    from recir_b200 import sharding
    return sharding.token_balanced_partition(lengths, world)[rank]


def _seq_of_row(lengths, mine, row):
    """Local sequence index that owns local token row `row`."""
    ends = np.cumsum(np.asarray(lengths)[mine])
    return int(np.searchsorted(ends, row, side="right"))


def test_gradient_checksum_exchange_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 31500 + os.getpid() % 2000
    procs = [ctx.Process(target=_checksum_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    bad, flipped_seq = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # exactly the sequence whose gradient had one bit flipped on rank 1 is reported, nothing else
    assert bad == [flipped_seq]
