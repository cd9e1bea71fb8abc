"""The numpy restatement of the reference's jagged marshalling ops against golden vectors made by
the reference's own Python operators (tests/golden/make_jagged_golden.py).  Bit-exact."""
import os

import numpy as np
import pytest

from oracle import jagged_oracle as jo

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "jagged_golden.npz"))
JD = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("jd_")})
CS = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("cs_")})


def offsets(lengths):
    return np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)


@pytest.mark.parametrize("name", JD)
def test_jagged_dense_round(name):
    off, n = offsets(GOLD[f"{name}/lengths"]), int(GOLD[f"{name}/n"])
    total = int(GOLD[f"{name}/total"])
    assert np.array_equal(jo.jagged_to_padded_dense(GOLD[f"{name}/values"], off, n, -7.0), GOLD[f"{name}/dense_out"])
    got = jo.dense_to_jagged(GOLD[f"{name}/dense_in"], off, None if total < 0 else total)
    assert np.array_equal(got, GOLD[f"{name}/jagged_out"])


@pytest.mark.parametrize("name", CS)
def test_concat_split(name):
    ol, orr = offsets(GOLD[f"{name}/ll"]), offsets(GOLD[f"{name}/lr"])
    cat = jo.concat_2d_jagged(GOLD[f"{name}/vl"], ol, GOLD[f"{name}/vr"], orr)
    assert np.array_equal(cat, GOLD[f"{name}/cat"])
    left, right = jo.split_2d_jagged(GOLD[f"{name}/cat"], ol, orr, int(ol[-1]), int(orr[-1]))
    assert np.array_equal(left, GOLD[f"{name}/left"]) and np.array_equal(right, GOLD[f"{name}/right"])


GRJ = np.load(os.path.join(os.path.dirname(__file__), "golden", "gr_jagged_golden.npz"))


@pytest.mark.parametrize("name", [str(n) for n in GRJ["names"]])
def test_gr_concat_and_split_match_the_reference_operators(name):
    from oracle import jagged_oracle as jo
    dense_a, dense_b, replace, p, batch, dense_size = (int(x) for x in GRJ[f"{name}/cfg"])
    oa = None if dense_a else GRJ[f"{name}/offsets_a"]
    ob = None if dense_b else GRJ[f"{name}/offsets_b"]
    a, b, cat = GRJ[f"{name}/a"], GRJ[f"{name}/b"], GRJ[f"{name}/cat"]
    got = jo.gr_concat_2d_jagged(a, b, oa, ob, bool(replace), p)
    assert got.shape == cat.shape and np.array_equal(got, cat)
    if not replace:
        sa, sb = jo.gr_split_2d_jagged(cat, oa, ob, bool(dense_a), bool(dense_b), dense_size, p, batch)
        assert np.array_equal(sa, a) and np.array_equal(sb, b)
