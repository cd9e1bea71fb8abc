"""Schedule of the host-memory pipeline (no GPU): every row is copied in once and out once, every sequence is
computed once, nothing is computed before its rows are on the device, and nothing leaves before it is computed."""
import numpy as np
import pytest

from recir_b200.host_api import plan_steps


def _check(offs, n_chunks):
    offs = np.asarray(offs, dtype=np.int64)
    total, B = int(offs[-1]), len(offs) - 1
    steps = plan_steps(offs, n_chunks)
    assert len(steps) == n_chunks
    t_prev = b_prev = r_prev = 0
    for st in steps:
        (t0, t1), (b0, b1), (r0, r1) = st["rows_in"], st["seqs"], st["rows_out"]
        assert (t0, b0, r0) == (t_prev, b_prev, r_prev)          # contiguous, in order
        assert t1 >= t0 and b1 >= b0 and r1 >= r0
        assert int(offs[b1]) <= t1                                 # computed sequences are on the device
        assert r1 <= int(offs[b1])                                 # rows that leave are computed
        t_prev, b_prev, r_prev = t1, b1, r1
    assert (t_prev, b_prev, r_prev) == (total, B, total)
    sizes = [st["rows_in"][1] - st["rows_in"][0] for st in steps]
    assert max(sizes) - min(sizes) <= 1                            # copy-in pieces of equal size
    # copy-out pieces: the copy-in pieces shifted back by one constant (at most the longest sequence)
    lags = {st["rows_in"][1] - st["rows_out"][1] for st in steps[:-1] if st["rows_out"][1] > 0}
    assert len(lags) <= 1
    if lags:
        assert 0 <= lags.pop() <= (int(np.diff(offs).max()) if B else 0)
    return steps


@pytest.mark.parametrize("n_chunks", [1, 2, 3, 7, 16])
def test_schedule_covers_everything_once(n_chunks):
    rng = np.random.default_rng(n_chunks)
    lengths = rng.integers(0, 700, size=37)
    lengths[[3, 4, 36]] = 0                                        # empty sequences, one of them last
    _check(np.concatenate([[0], np.cumsum(lengths)]), n_chunks)


def test_sequences_longer_than_a_piece():
    steps = _check([0, 10, 5000, 5003, 9000], 8)
    assert any(st["seqs"][0] == st["seqs"][1] for st in steps)     # steps without a complete sequence compute nothing
    _check([0, 4096], 16)                                          # one sequence: computed at the last step
    assert _check([0, 4096], 16)[-1]["seqs"] == (0, 1)


def test_degenerate_batches():
    _check([0, 0, 0], 1)
    _check([0, 1], 1)
    _check([0, 1, 2, 3], 3)
