"""Pins the numpy oracle: golden vectors from the reference operator, the reference's
known-answer test, and (when the compiled reference is present) direct comparison."""
import numpy as np
import pytest
import torch

from oracle import hstu_oracle, ref_op
from recir_b200 import workload
from tests.helpers import case_kwargs, golden_case, golden_names, max_abs


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_golden(name):
    c = golden_case(name)
    kw = case_kwargs(c)
    o = hstu_oracle.hstu_attention_fwd(c["q"], c["k"], c["v"], c["offsets"], **kw)
    dq, dk, dv = hstu_oracle.hstu_attention_bwd(c["do"], c["q"], c["k"], c["v"], c["offsets"], **kw)
    n = int(c["offsets"][-1])
    # golden outputs cover the valid rows; oracle rows past the last offset are zero
    assert max_abs(o[:n], c["o"]) < 2e-5
    assert max_abs(dq[:n], c["dq"]) < 5e-5
    assert max_abs(dk[:n], c["dk"]) < 5e-5
    assert max_abs(dv[:n], c["dv"]) < 5e-5
    assert not o[n:].any() and not dq[n:].any() and not dk[n:].any() and not dv[n:].any()


def test_known_answer_zero_scores():
    # recir/ops/tests/KjtSplitPerFeatureTest.cpp:237-261: zero q/k => silu(0)=0 => zero output
    q = np.zeros((2, 1, 1)); k = np.zeros((2, 1, 1)); v = np.array([2.0, 3.0]).reshape(2, 1, 1)
    o = hstu_oracle.hstu_attention_fwd(q, k, v, np.array([0, 2]), 2, 1.0)
    assert o.shape == v.shape and not o.any()


def test_invalid_offsets_rejected():
    q = np.zeros((2, 1, 1))
    with pytest.raises(ValueError, match="invalid jagged range"):
        hstu_oracle.hstu_attention_fwd(q, q, q, np.array([0, 3]), 2, 1.0)


@pytest.mark.skipif(not ref_op.available(), reason="compiled reference operator not present")
@pytest.mark.parametrize("seed", range(6))
def test_oracle_matches_compiled_reference_random(seed):
    rng = np.random.default_rng(seed)
    B, H, D = 5, 2, 8
    lengths = rng.integers(0, 40, size=B)
    targets = np.minimum(rng.integers(0, 6, size=B), lengths + 2)
    T = int(lengths.sum())
    q, k, v, do = (rng.standard_normal((T, H, D)).astype(np.float32) for _ in range(4))
    offs = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    kw = dict(max_seq_len=48, alpha=0.4, causal=bool(seed % 5 != 4),
              num_targets=targets if seed % 2 == 0 else None,
              max_attn_len=[0, 5, 9][seed % 3], contextual_seq_len=seed % 2 * 2,
              full_attn_size=4 if seed % 3 == 1 else 0, attn_scale=None)
    o = hstu_oracle.hstu_attention_fwd(q, k, v, offs, **kw)
    dq, dk, dv = hstu_oracle.hstu_attention_bwd(do, q, k, v, offs, **kw)
    tk = dict(kw, num_targets=None if kw["num_targets"] is None else torch.from_numpy(targets))
    ro, rdq, rdk, rdv = ref_op.ref_fwd_bwd(*(torch.from_numpy(x) for x in (do, q, k, v)),
                                           torch.from_numpy(offs), **tk)
    assert max_abs(o, ro) < 2e-5 and max_abs(dq, rdq) < 5e-5
    assert max_abs(dk, rdk) < 5e-5 and max_abs(dv, rdv) < 5e-5


@pytest.mark.parametrize("seed", range(40))
def test_kept_pairs_closed_form_vs_bruteforce(seed):
    rng = np.random.default_rng(100 + seed)
    L = int(rng.integers(0, 70))
    t = [None, int(rng.integers(0, L + 3))][seed % 2]
    w = int(rng.choice([0, 1, 3, 17, 100]))
    ctx = int(rng.integers(0, 2)) * 3
    f = int(rng.choice([0, 0, 4])) if w > 0 else 0
    causal = bool(seed % 7 != 6)
    brute = hstu_oracle.count_kept_pairs([L], None if t is None else [t], causal, w, ctx, f)
    assert workload.kept_pairs(L, t, causal, w, ctx, f) == brute


@pytest.mark.parametrize("name", golden_names("a4"))
def test_oracle_matches_second_reference_golden(name):
    """The reference's pure-torch pad-then-compute implementation and autograd through it
    (recir/ops/helion/jagged_hstu_attention.py:211-280) share no code with the compiled operator:
    an independent pin of the closed-form backward."""
    c = golden_case(name, "a4")
    kw = case_kwargs(c)
    o = hstu_oracle.hstu_attention_fwd(c["q"], c["k"], c["v"], c["offsets"], **kw)
    dq, dk, dv = hstu_oracle.hstu_attention_bwd(c["do"], c["q"], c["k"], c["v"], c["offsets"], **kw)
    assert max_abs(o, c["o"]) < 2e-5
    assert max_abs(dq, c["dq"]) < 5e-5
    assert max_abs(dk, c["dk"]) < 5e-5
    assert max_abs(dv, c["dv"]) < 5e-5


@pytest.mark.skipif(not ref_op.available(), reason="compiled reference operator not present")
@pytest.mark.parametrize("name", golden_names("a4"))
def test_two_references_agree(name):
    """The compiled operator (and autograd through it) reproduces the second reference's stored
    outputs: the two golden sets describe one function."""
    c = golden_case(name, "a4")
    kw = case_kwargs(c)
    t = lambda x: None if x is None else torch.from_numpy(np.asarray(x))
    tk = dict(kw, num_targets=t(kw["num_targets"]), attn_scale=t(kw["attn_scale"]))
    ro, rdq, rdk, rdv = ref_op.ref_fwd_bwd(t(c["do"]), t(c["q"]), t(c["k"]), t(c["v"]), t(c["offsets"]), **tk)
    assert max_abs(ro, c["o"]) < 2e-5 and max_abs(rdq, c["dq"]) < 5e-5
    assert max_abs(rdk, c["dk"]) < 5e-5 and max_abs(rdv, c["dv"]) < 5e-5
