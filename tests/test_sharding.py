"""Sample-sharding planner: whole sequences per rank, local offsets restart at zero, pad rows
dropped.  Expectations restate recir/tests/xla/test_helion_hstu_sharding.py:97-162 and
recir/tests/xla/test_pallas_jagged_hstu_sharding.py:93-100,151-178 of the reference."""
import numpy as np
import pytest
import torch

from recir_b200 import sharding, workload


def test_pad_seqs_per_device_reference_values():
    assert sharding.pad_seqs_per_device(6, 8, 2) == 1
    assert sharding.pad_seqs_per_device(256, 512, 64) == 4
    assert sharding.pad_seqs_per_device(8, 8, 2) == 0


def test_contiguous_partition_local_offsets_and_pad_rows():
    # two ranks, four sequences each, last one per rank is a pad row absorbing the deficit
    lengths = np.array([4, 3, 5, 4, 2, 5, 4, 5])
    targets = np.array([1, 2, 3, 99, 4, 5, 6, 98])
    parts = sharding.contiguous_partition(lengths, 2, pad_seqs=1)
    assert [p.tolist() for p in parts] == [[0, 1, 2], [4, 5, 6]]
    assert sharding.local_offsets(lengths[parts[0]]).tolist() == [0, 4, 7, 12]
    assert sharding.local_offsets(lengths[parts[1]]).tolist() == [0, 2, 7, 11]
    assert targets[parts[0]].tolist() == [1, 2, 3] and targets[parts[1]].tolist() == [4, 5, 6]
    assert 99 not in targets[np.concatenate(parts)] and 98 not in targets[np.concatenate(parts)]


def test_contiguous_partition_rejects_crossed_boundaries():
    with pytest.raises(ValueError, match="not batch-aligned"):
        sharding.contiguous_partition(np.array([5, 4, 3, 4]), 2)
    with pytest.raises(ValueError, match="no real sequence"):
        sharding.contiguous_partition(np.array([4, 4]), 2, pad_seqs=1)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_token_balanced_partition_covers_everything_once(world):
    hist, tg = workload.config4_lengths(1024)
    lengths = hist + tg
    parts = sharding.token_balanced_partition(lengths, world)
    allidx = np.sort(np.concatenate(parts))
    assert (allidx == np.arange(len(lengths))).all()
    summ = sharding.shard_summary(lengths, parts)
    assert summ["token_imbalance"] < 1.01
    parts_c = sharding.token_balanced_partition(lengths, world, balance="cost")
    assert sharding.shard_summary(lengths, parts_c)["cost_imbalance"] < 1.05


def test_gather_rows_matches_offsets():
    lengths = [3, 0, 2, 4]
    offs = sharding.local_offsets(lengths)
    x = torch.arange(9).view(9, 1, 1)
    got = sharding.gather_rows(x, offs, [3, 0])
    assert got.flatten().tolist() == [5, 6, 7, 8, 0, 1, 2]


def test_length_buckets_of_the_zipf_batch_partition_it():
    """The per-length-bucket runner covers every sequence of the Zipf batch exactly once, keeps each
    batch's lengths inside its bucket and repeats / cuts buckets to the advertised token range."""
    import bench_cases as run_case

    hist, tg = workload.config4_lengths(1024)
    lengths = hist + tg
    seen = 0
    for lo, hi in run_case.BUCKETS:
        bt, n = run_case.bucket_batch(lo, hi, min_tokens=4096)
        assert n == int(((lengths >= lo) & (lengths < hi)).sum())
        seen += n
        got = np.diff(bt.seq_offsets.numpy())
        assert got.min() >= lo and got.max() < hi
        assert 4096 <= bt.total_tokens <= 4 * 4096 + hi
        assert bt.q.shape == (bt.total_tokens, 4, 128)
        assert (bt.num_targets.numpy() < got).all()
    assert seen == 1024
