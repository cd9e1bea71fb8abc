"""GPU parity of the jagged marshalling kernels (through the torch operators -> C ABI): bit-exact
against the golden vectors made by the reference's Python operators, against the numpy restatement on
random cases in every element width, round trips at benchmark size, and autograd through the pairs."""
import os

import numpy as np
import pytest
import torch

import recir_b200  # noqa: F401
from oracle import jagged_oracle as jo

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "jagged_golden.npz"))
JD = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("jd_")})
CS = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("cs_")})
ops = torch.ops.recir


def offsets(lengths, dtype=torch.int64):
    return torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=dtype, device="cuda")


def cu(a, dtype=None):
    t = torch.as_tensor(np.asarray(a)).cuda()
    return t.to(dtype) if dtype else t


@pytest.mark.parametrize("name", JD)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_jagged_dense_matches_reference_golden(name, dtype):
    off, n = offsets(GOLD[f"{name}/lengths"]), int(GOLD[f"{name}/n"])
    total = int(GOLD[f"{name}/total"])
    dense = ops.b200_jagged_to_padded_dense(cu(GOLD[f"{name}/values"], dtype), [off], [n], -7.0)
    assert torch.equal(dense.float().cpu(), torch.as_tensor(GOLD[f"{name}/dense_out"]))
    j, off_out = ops.b200_dense_to_jagged(cu(GOLD[f"{name}/dense_in"], dtype), [off], None if total < 0 else total)
    assert torch.equal(j.float().cpu(), torch.as_tensor(GOLD[f"{name}/jagged_out"])) and torch.equal(off_out, off)


@pytest.mark.parametrize("name", CS)
@pytest.mark.parametrize("off_dtype", [torch.int64, torch.int32])
def test_concat_split_match_reference_golden(name, off_dtype):
    ol, orr = offsets(GOLD[f"{name}/ll"], off_dtype), offsets(GOLD[f"{name}/lr"], off_dtype)
    cat = ops.b200_concat_2d_jagged(cu(GOLD[f"{name}/vl"]), ol, cu(GOLD[f"{name}/vr"]), orr)
    assert torch.equal(cat.cpu(), torch.as_tensor(GOLD[f"{name}/cat"]))
    left, right = ops.b200_split_2d_jagged(cu(GOLD[f"{name}/cat"]), ol, orr, int(ol[-1]), int(orr[-1]))
    assert torch.equal(left.cpu(), torch.as_tensor(GOLD[f"{name}/left"]))
    assert torch.equal(right.cpu(), torch.as_tensor(GOLD[f"{name}/right"]))


def test_random_cases_against_the_oracle_every_width():
    rng = np.random.default_rng(0)
    for trial in range(12):
        b = int(rng.integers(1, 9))
        lengths = rng.integers(0, 40, b)
        lr = rng.integers(0, 6, b)
        n = int(rng.integers(1, 48))
        d = int(rng.choice([1, 3, 8, 64, 130]))
        for dtype in (torch.float32, torch.bfloat16, torch.int16, torch.int64):
            if (d * torch.empty((), dtype=dtype).element_size()) % 2:
                continue
            off = np.concatenate([[0], np.cumsum(lengths)])
            v = torch.randint(-100, 100, (int(off[-1]), d)).to(dtype)
            dense_in = torch.randint(-100, 100, (b, n, d)).to(dtype)
            as_np = lambda t: t.float().numpy() if t.dtype == torch.bfloat16 else t.numpy()  # noqa: E731
            got = ops.b200_jagged_to_padded_dense(v.cuda(), [cu(off)], [n], 3.0)
            assert np.array_equal(as_np(got.cpu()), jo.jagged_to_padded_dense(as_np(v), off, n, 3.0)), (trial, dtype, "j2d")
            got, _ = ops.b200_dense_to_jagged(dense_in.cuda(), [cu(off)], None)
            assert np.array_equal(as_np(got.cpu()), jo.dense_to_jagged(as_np(dense_in), off)), (trial, dtype, "d2j")
            offr = np.concatenate([[0], np.cumsum(lr)])
            vr = torch.randint(-100, 100, (int(offr[-1]), d)).to(dtype)
            cat = ops.b200_concat_2d_jagged(v.cuda(), cu(off), vr.cuda(), cu(offr))
            want = jo.concat_2d_jagged(as_np(v), off, as_np(vr), offr)
            assert np.array_equal(as_np(cat.cpu()), want), (trial, dtype, "concat")
            if v.shape[0] and vr.shape[0]:
                left, right = ops.b200_split_2d_jagged(cat, cu(off), cu(offr), v.shape[0], vr.shape[0])
                assert torch.equal(left.cpu(), v) and torch.equal(right.cpu(), vr), (trial, dtype, "split")


def test_round_trips_at_benchmark_size_and_autograd():
    bt = recir_b200.workload.config1()
    off = bt.seq_offsets.cuda()
    lengths = (off[1:] - off[:-1])
    n = int(lengths.max())
    x = torch.randn(bt.total_tokens, 512, dtype=torch.bfloat16, device="cuda")
    dense = ops.b200_jagged_to_padded_dense(x, [off], [n], 0.0)
    assert dense.shape == (64, n, 512)
    back, _ = ops.b200_dense_to_jagged(dense, [off], bt.total_tokens)
    assert torch.equal(back, x)                                  # jagged -> dense -> jagged is the identity
    mask = torch.arange(n, device="cuda")[None, :] < lengths[:, None]
    assert not dense[~mask].any()                                # padding is exact zeros
    # split off the 64 targets of every sequence and put them back
    hist_off = off - 64 * torch.arange(65, device="cuda")
    tgt_off = 64 * torch.arange(65, device="cuda")
    left, right = ops.b200_split_2d_jagged(x, hist_off, tgt_off, int(hist_off[-1]), int(tgt_off[-1]))
    assert torch.equal(left[: int(hist_off[1])], x[: int(hist_off[1])])
    assert torch.equal(ops.b200_concat_2d_jagged(left, hist_off, right, tgt_off), x)
    # autograd: each op of a pair is the other's backward
    xs = torch.randn(int(off[3]), 8, device="cuda", requires_grad=True)
    d3 = ops.b200_jagged_to_padded_dense(xs, [off[:4]], [n], 0.0)
    w = torch.randn_like(d3)
    (d3 * w).sum().backward()
    want, _ = ops.b200_dense_to_jagged(w, [off[:4]], xs.shape[0])
    assert torch.equal(xs.grad, want)
    a = torch.randn(int(hist_off[2]), 8, device="cuda", requires_grad=True)
    b = torch.randn(int(tgt_off[2]), 8, device="cuda", requires_grad=True)
    cat = ops.b200_concat_2d_jagged(a, hist_off[:3], b, tgt_off[:3])
    wc = torch.randn_like(cat)
    (cat * wc).sum().backward()
    gl, gr = ops.b200_split_2d_jagged(wc, hist_off[:3], tgt_off[:3], a.shape[0], b.shape[0])
    assert torch.equal(a.grad, gl) and torch.equal(b.grad, gr)


GRJ = np.load(os.path.join(os.path.dirname(__file__), "golden", "gr_jagged_golden.npz"))


@pytest.mark.parametrize("name", [str(n) for n in GRJ["names"]])
def test_gr_concat_and_split_match_the_reference_golden(name):
    """The concat / split operators with the schemas of generative_recommenders (dense sides, a prefix of
    the right side moved to the front, the replace form), bit-exact against the reference operators."""
    dense_a, dense_b, replace, p, batch, dense_size = (int(x) for x in GRJ[f"{name}/cfg"])
    cu = lambda k: torch.as_tensor(GRJ[f"{name}/{k}"]).cuda()
    oa = None if dense_a else cu("offsets_a")
    ob = None if dense_b else cu("offsets_b")
    a, b, cat = cu("a"), cu("b"), cu("cat")
    got = torch.ops.recir.b200_concat_2D_jagged_fwd_op(16, a, b, oa, ob, bool(replace), p)
    assert got.shape == cat.shape and torch.equal(got, cat)
    if not replace:
        dummy = torch.zeros(batch + 1, dtype=torch.int64, device="cuda")
        sa, sb = torch.ops.recir.b200_split_2D_jagged_fwd_op(
            cat, 16, dummy if dense_a else oa, dummy if dense_b else ob, 0 if dense_a else a.shape[0],
            0 if dense_b else b.shape[0], bool(dense_a), bool(dense_b), dense_size, p, batch)
        assert torch.equal(sa, a) and torch.equal(sb, b)


def test_gr_concat_with_prefix_on_a_zipf_batch_against_the_oracle():
    from oracle import jagged_oracle as jo
    from recir_b200 import workload
    hist, tg = workload.config4_lengths(96)
    g = torch.Generator().manual_seed(9)
    oa = torch.as_tensor(np.concatenate([[0], np.cumsum(hist)]))
    ob = torch.as_tensor(np.concatenate([[0], np.cumsum(tg)]))
    a = torch.randn(int(oa[-1]), 64, generator=g).to(torch.bfloat16)
    b = torch.randn(int(ob[-1]), 64, generator=g).to(torch.bfloat16)
    for replace, p in ((False, 0), (False, 3), (True, 0)):
        if replace:  # the replaced tail must fit: whole sequences (history + targets) on the left
            oa = torch.as_tensor(np.concatenate([[0], np.cumsum(hist + tg)]))
            a = torch.randn(int(oa[-1]), 64, generator=g).to(torch.bfloat16)
        got = torch.ops.recir.b200_concat_2D_jagged_fwd_op(4224, a.cuda(), b.cuda(), oa.cuda(), ob.cuda(), replace, p)
        want = jo.gr_concat_2d_jagged(a.view(torch.int16).numpy(), b.view(torch.int16).numpy(), oa.numpy(), ob.numpy(),
                                      replace, p)
        assert np.array_equal(got.view(torch.int16).cpu().numpy(), want)
        if not replace:
            sa, sb = torch.ops.recir.b200_split_2D_jagged_fwd_op(got, 4224, oa.cuda(), ob.cuda(), a.shape[0], b.shape[0],
                                                                 False, False, 0, p, 96)
            assert torch.equal(sa.cpu(), a) and torch.equal(sb.cpu(), b)
    with pytest.raises(ValueError, match="at least one input must be jagged"):
        torch.ops.recir.b200_concat_2D_jagged_fwd_op(8, a.cuda(), b.cuda(), None, None, False, 0)
