"""The numpy restatement of the reference's position + timestamp embedding add against golden
vectors made by the reference's compiled operator (tests/golden/make_embed_golden.py)."""
import os

import numpy as np
import pytest

from oracle import embed_oracle as eo

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "embed_golden.npz"))
CASES = sorted({k.split("/")[0] for k in GOLD.files})
ULP = {"float32": 2e-6, "bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}


def run_oracle(name):
    dt, tdt, c, inter, fn = GOLD[f"{name}/cfg"]
    lengths = GOLD[f"{name}/lengths"]
    tg = GOLD[f"{name}/targets"]
    tg = None if tg[0] < 0 else tg
    off = np.concatenate([[0], np.cumsum(lengths)])
    return eo.add_ts_pos_emb(GOLD[f"{name}/x"], off, GOLD[f"{name}/pos"], GOLD[f"{name}/ts"], GOLD[f"{name}/stamps"], lengths, tg,
                             int(c), inter == "1", str(fn), str(dt), str(tdt)), str(dt)


@pytest.mark.parametrize("name", CASES)
def test_matches_reference(name):
    (y, pos_idx, ts_idx), dt = run_oracle(name)
    assert np.array_equal(pos_idx, GOLD[f"{name}/pos_idx"])
    assert np.array_equal(ts_idx, GOLD[f"{name}/ts_idx"])
    want = GOLD[f"{name}/y"].astype(np.float64)
    tol = ULP[dt] * np.maximum(np.abs(want), 1.0 if dt == "float32" else 1e-3)
    assert (np.abs(y - want) <= tol).all()
    assert len(np.unique(GOLD[f"{name}/ts_idx"])) >= 3, "the case should exercise several time buckets"
