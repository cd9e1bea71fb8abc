"""GPU parity of the row-wise STU kernels (through the torch operators -> C ABI) against the golden
vectors made by the reference's compiled operators and against the numpy restatement.

Tolerances (floating point): float32 results within 2e-6 absolute of O(1) values; 16-bit results
equal to the reference up to one unit in the last place on at most 0.1 % of the elements (the
reference's vectorised exp and this kernel's expf can differ in the last float32 bit before a
rounding); fp8 codes identical except for such boundary cases (at most 0.2 %), never by more than
one code."""
import os

import numpy as np
import pytest
import torch

import recir_b200  # noqa: F401
from oracle import rowwise_oracle as ro

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "rowwise_golden.npz"))
LN = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("ln_")})
MUL = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("mul_")})
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
ULP = {"float32": 2e-6, "bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}


def _t(a, dt=None):
    t = torch.as_tensor(np.asarray(a))
    return (t.to(DT[dt]) if dt else t).cuda()


def _close(got, want, dtype, what):
    got, want = got.float().cpu().numpy().astype(np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape, what
    if got.size == 0:
        return
    tol = ULP[dtype] * np.maximum(np.abs(want), 1.0 if dtype == "float32" else 1e-3)
    bad = np.abs(got - want) > tol
    assert bad.mean() <= 1e-3, f"{what}: {bad.sum()} of {bad.size} beyond one ulp"
    assert np.abs(got - want).max() <= 4 * tol.max(), what


def _codes_close(got, want, what):
    got, want = got.view(torch.uint8).cpu().numpy(), np.asarray(want)
    assert got.shape == want.shape, what
    diff = got != want
    assert diff.mean() <= 2e-3, f"{what}: {diff.sum()} of {diff.size} fp8 codes differ"
    if diff.any():
        assert np.abs((got & 0x7F).astype(np.int16) - (want & 0x7F).astype(np.int16))[diff].max() <= 1, what


@pytest.mark.parametrize("name", LN)
def test_layer_norm_matches_reference_golden(name):
    dt, affine, swish, stats_in = GOLD[f"{name}/cfg"]
    x = _t(GOLD[f"{name}/x"], dt)
    w = _t(GOLD[f"{name}/w"], dt) if affine == "1" else None
    b = _t(GOLD[f"{name}/b"], dt) if affine == "1" else None
    m_in = _t(GOLD[f"{name}/mean_in"]) if stats_in == "1" else None
    r_in = _t(GOLD[f"{name}/rstd_in"]) if stats_in == "1" else None
    y, mean, rstd = torch.ops.recir.b200_weighted_layer_norm_fwd(x, w, b, 1e-5, m_in, r_in, swish == "1")
    torch.cuda.synchronize()
    _close(y, GOLD[f"{name}/y"], dt, "y")
    _close(mean, GOLD[f"{name}/mean"], "float32", "mean")
    _close(rstd, GOLD[f"{name}/rstd"], "float32", "rstd")


@pytest.mark.parametrize("name", MUL)
def test_layer_norm_mul_matches_reference_golden(name):
    dt, silu_u, cat_u, cat_x, act = GOLD[f"{name}/cfg"]
    args = [_t(GOLD[f"{name}/{k}"], dt) for k in ("x", "u", "w", "b")]
    y, mean, rstd, scale, q8 = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
        *args, 1e-5, 0.0, False, silu_u == "1", cat_u == "1", cat_x == "1", str(act), 0, True, 0)
    torch.cuda.synchronize()
    _close(y, GOLD[f"{name}/y"], dt, "y")
    _close(mean, GOLD[f"{name}/mean"], "float32", "mean")
    _close(rstd, GOLD[f"{name}/rstd"], "float32", "rstd")
    _close(scale, GOLD[f"{name}/scale"], "float32", "scale")
    _codes_close(q8, GOLD[f"{name}/q8"], "q8")
    # save_y == False: no y, same fp8 copy
    y2, _, _, scale2, q82 = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
        *args, 1e-5, 0.0, False, silu_u == "1", cat_u == "1", cat_x == "1", str(act), 0, False, 0)
    assert y2.numel() == 0 and torch.equal(q82.view(torch.uint8), q8.view(torch.uint8)) and torch.equal(scale2, scale)


LNQ = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("lnq_")})


@pytest.mark.parametrize("name", LNQ)
def test_quantized_layer_norm_matches_reference_golden(name):
    dt = str(GOLD[f"{name}/cfg"][0])
    x, w, b = (_t(GOLD[f"{name}/{k}"], dt) for k in ("x", "w", "b"))
    empty = torch.empty(0, device="cuda")
    y, mean, rstd, scale, q8 = torch.ops.recir.b200_weighted_layer_norm_quantization_fwd(x, w, b, 1e-5, empty, empty, 0)
    torch.cuda.synchronize()
    _close(y, GOLD[f"{name}/y"], dt, "y")
    _close(mean, GOLD[f"{name}/mean"], "float32", "mean")
    _close(scale, GOLD[f"{name}/scale"], "float32", "scale")
    _codes_close(q8, GOLD[f"{name}/q8"], "q8")
    y2, m2, r2 = torch.ops.recir.b200_weighted_layer_norm_fwd(x, w, b, 1e-5, None, None, False)
    assert torch.equal(y2, y) and torch.equal(m2, mean) and torch.equal(r2, rstd)


def test_full_size_rows_against_the_oracle_and_strided_input():
    """Benchmark-sized rows (embedding 512, bf16): a sample of rows against the numpy restatement,
    every row through row-wise invariants, and a strided (column-sliced) input."""
    g = torch.Generator().manual_seed(3)
    rows, cols = 78262, 512
    big = (torch.randn(rows, 2 * cols, generator=g) * 1.3).to(torch.bfloat16).cuda()
    x, u = big[:, :cols], big[:, cols:]  # row stride 1024: two column slices of one buffer
    w = (torch.randn(cols, generator=g) * 0.5 + 1).to(torch.bfloat16).cuda()
    b = (torch.randn(cols, generator=g) * 0.2).to(torch.bfloat16).cuda()
    y, mean, rstd = torch.ops.recir.b200_weighted_layer_norm_fwd(x, w, b, 1e-6, None, None, True)
    ym, _, _, scale, q8 = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
        x, u, w, b, 1e-6, 0.0, False, True, True, False, "silu", 0, True, 0)
    torch.cuda.synchronize()
    sel = torch.arange(0, rows, 997)
    f = lambda t: t[sel.to(t.device)].float().cpu().numpy()
    ry, rm, rr = ro.weighted_layer_norm(f(x), w.float().cpu().numpy(), b.float().cpu().numpy(), 1e-6, "bfloat16",
                                        is_swish=True)
    _close(y[sel.cuda()], ry, "bfloat16", "y sample")
    _close(mean[sel.cuda()], rm, "float32", "mean sample")
    ryy, _, _, rs, rq = ro.layer_norm_mul_quantized(f(x), f(u), w.float().cpu().numpy(), b.float().cpu().numpy(), 1e-6,
                                                    "bfloat16", silu_u=True, concat_u=True, mul_u_activation="silu")
    _close(ym[sel.cuda()], ryy, "bfloat16", "mul sample")
    _close(scale[sel.cuda()], rs, "float32", "scale sample")
    _codes_close(q8[sel.cuda()], rq, "q8 sample")
    # invariants over every row: statistics against torch, the fp8 copy spans its full range in each row
    xf = x.float()
    assert torch.allclose(mean, xf.mean(1), atol=1e-5)
    assert torch.allclose(rstd, torch.rsqrt(xf.var(1, unbiased=False) + 1e-6), rtol=1e-4)
    assert int((q8.view(torch.uint8) & 0x7F).max(dim=1).values.min()) == 0x7E


def test_validation_and_fake_kernels():
    x = torch.zeros(4, 20, device="cuda")
    with pytest.raises(ValueError, match="multiple of 8"):
        torch.ops.recir.b200_weighted_layer_norm_fwd(x, None, None, 1e-5, None, None, False)
    x = torch.zeros(4, 16, device="cuda")
    with pytest.raises(ValueError, match="is_swish requires"):
        torch.ops.recir.b200_weighted_layer_norm_fwd(x, None, None, 1e-5, None, None, True)
    with pytest.raises(ValueError, match="bias is required"):
        torch.ops.recir.b200_weighted_layer_norm_fwd(x, torch.ones(16, device="cuda"), None, 1e-5, None, None, False)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        xf = torch.empty(6, 32, dtype=torch.bfloat16, device="cuda")
        wf = torch.empty(32, dtype=torch.bfloat16, device="cuda")
        out = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
            xf, xf, wf, wf, 1e-5, 0.0, False, True, True, True, "silu", 0, True, 0)
    assert out[0].shape == (6, 96) and out[4].dtype == torch.float8_e4m3fn and out[3].shape == (6,)


def test_addmm_operator_validation_and_library_path_for_other_shapes():
    """The tensor-core kernel serves the 16-bit STU shapes (tests/test_gemm_gpu.py); float32 and odd sizes
    are plain GEMMs handed to the vendor library, and the reference's argument checks apply to both."""
    g = torch.Generator().manual_seed(1)
    x = torch.randn(30, 24, generator=g).cuda()
    w = torch.randn(24, 20, generator=g).cuda()
    y = torch.randn(20, generator=g).cuda()
    assert torch.allclose(torch.ops.recir.b200_addmm_fwd(x, w, y), y + x @ w, atol=1e-4)
    with pytest.raises(ValueError, match="incompatible"):
        torch.ops.recir.b200_addmm_fwd(x, w[:16], y)


FP8MM = np.load(os.path.join(os.path.dirname(__file__), "golden", "fp8_addmm_golden.npz"))


@pytest.mark.parametrize("name", [str(n) for n in FP8MM["names"]])
def test_fp8_rowwise_addmm_matches_reference_golden(name):
    """The fp8 projection behind the quantised layer-norm stage, through the library's fp8 GEMM with
    row-wise scales, against the reference operator's output on the same e4m3 operands."""
    dt, has_bias = FP8MM[f"{name}/cfg"]
    a = torch.as_tensor(FP8MM[f"{name}/a"]).cuda().view(torch.float8_e4m3fn)
    b = torch.as_tensor(FP8MM[f"{name}/b"]).cuda().view(torch.float8_e4m3fn)
    sa, sb = _t(FP8MM[f"{name}/a_scale"]), _t(FP8MM[f"{name}/b_scale"])
    bias = _t(FP8MM[f"{name}/bias"], dt) if has_bias == "1" else torch.empty(0, device="cuda")
    y = torch.ops.recir.b200_fp8_rowwise_addmm_fwd(a, b, sa, sb, bias, has_bias == "1", False, DT[dt], False, False)
    assert y.dtype == DT[dt] and tuple(y.shape) == FP8MM[f"{name}/y"].shape
    want = FP8MM[f"{name}/y"].astype(np.float64)
    got = y.float().cpu().numpy().astype(np.float64)
    tol = (1e-5 if dt == "float32" else 2 * ULP[dt]) * np.maximum(np.abs(want), float(np.abs(want).max()) * 1e-2)
    assert (np.abs(got - want) <= tol).all(), float(np.abs(got - want).max())


def test_fp8_rowwise_addmm_chained_behind_the_quantised_norm_stage():
    """layer-norm x gate with fp8 copy -> fp8 projection, full STU width, against the oracle chain."""
    g = torch.Generator().manual_seed(5)
    rows, cols, n_out = 1024, 512, 256
    x = (torch.randn(rows, cols, generator=g) * 1.5).to(torch.bfloat16).cuda()
    u = (torch.randn(rows, cols, generator=g) * 2.0).to(torch.bfloat16).cuda()
    w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(torch.bfloat16).cuda()
    b = (torch.randn(cols, generator=g) * 0.2).to(torch.bfloat16).cuda()
    wq = (torch.randn(n_out, cols, generator=g) * 30.0).clamp(-448, 448).to(torch.float8_e4m3fn).cuda()
    ws = (torch.rand(n_out, generator=g) * 0.01 + 0.001).cuda()
    y, mean, rstd, scale, q8 = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
        x, u, w, b, 1e-5, 0.0, False, False, False, False, "silu", 0, True, 0)
    out = torch.ops.recir.b200_fp8_rowwise_addmm_fwd(q8, wq, scale, ws, torch.empty(0, device="cuda"), False, False,
                                                     torch.bfloat16, False, False)
    want = ro.fp8_rowwise_addmm(q8.view(torch.uint8).cpu().numpy(), wq.view(torch.uint8).cpu().numpy(),
                                scale.cpu().numpy(), ws.cpu().numpy(), None, "bfloat16")
    _close(out, want, "bfloat16", "fp8 projection")
    with pytest.raises(ValueError, match="float8"):
        torch.ops.recir.b200_fp8_rowwise_addmm_fwd(y, wq, scale, ws, torch.empty(0, device="cuda"), False, False,
                                                   torch.bfloat16, False, False)


JBMM = np.load(os.path.join(os.path.dirname(__file__), "golden", "jagged_bmm_golden.npz"))


@pytest.mark.parametrize("name", [str(n) for n in JBMM["names"] if str(n).startswith("bf16")])
def test_jagged_dense_bmm_add_matches_reference_golden(name):
    """Per-sequence projection of jagged rows against the reference operator's output (bias per sequence and
    per row, empty sequences in the batch): K = 64 runs on this library's tensor-core kernel, K = 32 on the
    vendor library's grouped GEMM."""
    dt, elementwise = JBMM[f"{name}/cfg"]
    offs = torch.as_tensor(JBMM[f"{name}/offsets"]).cuda()
    jag, den, bias = (_t(JBMM[f"{name}/{k}"], dt) for k in ("jagged", "dense", "bias"))
    y, B, K, N = torch.ops.recir.b200_jagged_dense_bmm_add_fwd(int(np.diff(JBMM[f"{name}/offsets"]).max()), offs, jag,
                                                              den, bias, elementwise == "1")
    assert (B, K, N) == tuple(den.shape) and y.dtype == DT[dt]
    want = JBMM[f"{name}/y"].astype(np.float64)
    got = y.float().cpu().numpy().astype(np.float64)
    assert got.shape == want.shape
    tol = 2 * ULP[dt] * np.maximum(np.abs(want), float(np.abs(want).max()) * 5e-2)
    assert (np.abs(got - want) <= tol).all(), float(np.abs(got - want).max())


def test_jagged_dense_bmm_add_on_a_zipf_batch_and_validation():
    from recir_b200 import workload
    hist, tg = workload.config4_lengths(64)
    lengths = hist + tg
    offs = torch.as_tensor(np.concatenate([[0], np.cumsum(lengths)])).cuda()
    T, B, K, N = int(offs[-1]), 64, 128, 64
    g = torch.Generator().manual_seed(3)
    jag = torch.randn(T, K, generator=g).to(torch.bfloat16).cuda()
    den = (torch.randn(B, K, N, generator=g) * 0.2).to(torch.bfloat16).cuda()
    bias = torch.randn(B, N, generator=g).to(torch.bfloat16).cuda()
    y, *_ = torch.ops.recir.b200_jagged_dense_bmm_add_fwd(int(lengths.max()), offs, jag, den, bias, False)
    # K = 128, N = 64: this library's tensor-core kernel (float32 sums, bias added, ONE rounding, as at::addmm)
    once = ro.jagged_dense_bmm_add(offs.cpu().numpy(), jag.float().cpu().numpy(), den.float().cpu().numpy(),
                                   bias.float().cpu().numpy(), False, "bfloat16")
    got = y.float().cpu().numpy().astype(np.float64)
    rel = np.abs(got - once) / np.maximum(np.abs(once), float(np.abs(once).max()) * 1e-2)
    assert rel.max() <= 2.02 * 2.0 ** -8 and (rel > 1.01 * 2.0 ** -8).mean() <= 0.02
    # K = 32 is not one of its sizes: the vendor library's grouped GEMM, which rounds the product to bfloat16
    # before the bias is added (restated here)
    jag2, den2 = jag[:, :32].contiguous(), den[:, :32].contiguous()
    y2, *_ = torch.ops.recir.b200_jagged_dense_bmm_add_fwd(int(lengths.max()), offs, jag2, den2, bias, False)
    prod = ro.jagged_dense_bmm_add(offs.cpu().numpy(), jag2.float().cpu().numpy(), den2.float().cpu().numpy(),
                                   np.zeros((B, N), np.float32), False, "bfloat16")
    seq = np.repeat(np.arange(B), lengths)
    want = ro.round_to(prod + bias.float().cpu().numpy()[seq], "bfloat16")
    got2 = y2.float().cpu().numpy().astype(np.float64)
    tol = 2.0 ** -7 * np.maximum(np.abs(prod), np.abs(want)) + 1e-6
    bad = np.abs(got2 - want) > tol
    assert bad.mean() <= 1e-3 and np.abs(got2 - want).max() <= 4 * tol.max()
    with pytest.raises(ValueError, match="incompatible"):
        torch.ops.recir.b200_jagged_dense_bmm_add_fwd(8, offs, jag, den[:, :64], bias, False)
    with pytest.raises(ValueError, match="unsupported dtype"):
        torch.ops.recir.b200_jagged_dense_bmm_add_fwd(8, offs, jag.float(), den.float(), bias.float(), False)


BWD = np.load(os.path.join(os.path.dirname(__file__), "golden", "layer_norm_bwd_golden.npz"))


@pytest.mark.parametrize("name", sorted({k.split("/")[0] for k in BWD.files}))
def test_layer_norm_backward_matches_reference_autograd_golden(name):
    """dx, dweight, dbias against autograd through the reference's compiled composite
    (tests/golden/make_layer_norm_bwd_golden.py), through autograd of this library's operator.  float32: 3e-5 of
    the gradient scale; 16-bit: two units in the last place (sums of up to 140 float32 terms in another order
    than the reference's, then one rounding), more than one on at most 1 % of the elements."""
    dt, affine, swish = BWD[f"{name}/cfg"]
    x = _t(BWD[f"{name}/x"], dt).requires_grad_(True)
    w = _t(BWD[f"{name}/w"], dt).requires_grad_(True) if affine == "1" else None
    b = _t(BWD[f"{name}/b"], dt).requires_grad_(True) if affine == "1" else None
    y, _m, _r = torch.ops.recir.b200_weighted_layer_norm_fwd(x, w, b, 1e-5, None, None, swish == "1")
    y.backward(_t(BWD[f"{name}/dy"], dt))
    pairs = [("dx", x.grad, BWD[f"{name}/dx"])]
    if affine == "1":
        pairs += [("dw", w.grad, BWD[f"{name}/dw"]), ("db", b.grad, BWD[f"{name}/db"])]
    for what, got, want in pairs:
        got, want = got.float().cpu().numpy().astype(np.float64), want.astype(np.float64)
        rel = np.abs(got - want) / np.maximum(np.abs(want), np.abs(want).max() * 1e-2)
        if dt == "float32":
            assert rel.max() <= 3e-5, (what, float(rel.max()))
        else:
            assert rel.max() <= 2.02 * ULP[dt], (what, float(rel.max()))
            assert (rel > 1.01 * ULP[dt]).mean() <= 1e-2, what


def test_layer_norm_backward_at_benchmark_size_is_deterministic_and_matches_oracle_sample():
    g = torch.Generator().manual_seed(9)
    rows, cols = 60_000, 512
    x = (torch.randn(rows, cols, generator=g) * 1.5 + 0.3).to(torch.bfloat16).cuda()
    dy = torch.randn(rows, cols, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(torch.bfloat16).cuda()
    b = (torch.randn(cols, generator=g) * 0.2).to(torch.bfloat16).cuda()
    _y, mean, rstd = torch.ops.recir.b200_weighted_layer_norm_fwd(x, w, b, 1e-5, None, None, True)
    a = torch.ops.recir.b200_weighted_layer_norm_bwd(dy, x, w, b, mean, rstd, True)
    c = torch.ops.recir.b200_weighted_layer_norm_bwd(dy, x, w, b, mean, rstd, True)
    assert all(torch.equal(p, q) for p, q in zip(a, c))  # no atomics: bitwise repeatable
    f = lambda t: t.float().cpu().numpy()
    rdx, rdw, rdb = ro.weighted_layer_norm_bwd(f(dy), f(x), f(w), f(b), 1e-5, "bfloat16", is_swish=True)
    _close(a[0][::997], rdx[::997], "bfloat16", "dx sample")
    for got, want, what in ((a[1], rdw, "dw"), (a[2], rdb, "db")):
        rel = np.abs(f(got).astype(np.float64) - want) / np.maximum(np.abs(want), np.abs(want).max() * 1e-2)
        assert rel.max() <= 2.02 * ULP["bfloat16"], (what, float(rel.max()))


MULBWD = np.load(os.path.join(os.path.dirname(__file__), "golden", "layer_norm_mul_bwd_golden.npz"))
MULBWD_NAMES = sorted({k.split("/")[0] for k in MULBWD.files})


def _mul_case(name):
    dt, silu_u, concat_u, concat_x, act = MULBWD[f"{name}/cfg"]
    return dt, silu_u == "1", concat_u == "1", concat_x == "1", str(act)


@pytest.mark.parametrize("name", MULBWD_NAMES)
def test_gate_stage_backward_matches_oracle_and_reference_autograd(name):
    """Gradients of the gate stage through autograd of this library's operator.  Against the float64
    restatement rounded once (which the kernel's float32 arithmetic, rounded once, follows closely): float32 3e-5
    of the gradient scale, 16-bit two units in the last place, more than one on at most 1 % of the elements.
    Against autograd through the reference's compiled composite (which differentiates through 16-bit
    intermediates): the bounds the restatement itself meets (tests/test_rowwise_oracle.py)."""
    dt, silu_u, concat_u, concat_x, act = _mul_case(name)
    x = _t(MULBWD[f"{name}/x"], dt).requires_grad_(True)
    u = _t(MULBWD[f"{name}/u"], dt).requires_grad_(True)
    w = _t(MULBWD[f"{name}/w"], dt).requires_grad_(True)
    b = _t(MULBWD[f"{name}/b"], dt).requires_grad_(True)
    y = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(x, u, w, b, 1e-5, 0.0, False, silu_u, concat_u, concat_x,
                                                                    act, 0, True, 64)[0]
    y.backward(_t(MULBWD[f"{name}/dout"], dt))
    want = ro.layer_norm_mul_bwd(MULBWD[f"{name}/dout"], MULBWD[f"{name}/x"], MULBWD[f"{name}/u"], MULBWD[f"{name}/w"],
                                 MULBWD[f"{name}/b"], 1e-5, dt, silu_u, concat_u, concat_x, act)
    ref_l2, ref_max = {"float32": (1e-6, 2e-6), "bfloat16": (6e-3, 8e-3), "float16": (8e-4, 1.5e-3)}[dt]
    for what, got, o in zip(("dx", "du", "dw", "db"), (x.grad, u.grad, w.grad, b.grad), want):
        got = got.float().cpu().numpy().astype(np.float64)
        o = np.asarray(o, np.float64)
        rel = np.abs(got - o) / np.maximum(np.abs(o), np.abs(o).max() * 1e-2)
        if dt == "float32":
            assert rel.max() <= 3e-5, (what, float(rel.max()))
        else:
            assert rel.max() <= 2.02 * ULP[dt], (what, float(rel.max()))
            assert (rel > 1.01 * ULP[dt]).mean() <= 1e-2, what
        ref = MULBWD[f"{name}/{what}"].astype(np.float64)
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= ref_l2, what
        assert np.abs(got - ref).max() / np.abs(ref).max() <= ref_max, what


def test_gate_stage_backward_at_benchmark_size_is_deterministic_and_validates():
    g = torch.Generator().manual_seed(10)
    rows, cols = 60_000, 512
    x = (torch.randn(rows, cols, generator=g) * 1.5 + 0.3).to(torch.bfloat16).cuda()
    u = torch.randn(rows, cols, generator=g).to(torch.bfloat16).cuda()
    dout = torch.randn(rows, cols, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(cols, generator=g) * 0.5 + 1.0).to(torch.bfloat16).cuda()
    b = (torch.randn(cols, generator=g) * 0.2).to(torch.bfloat16).cuda()
    _y, mean, rstd, _s, _q = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
        x, u, w, b, 1e-5, 0.0, False, False, False, False, "silu", 0, False, 64)
    bwd = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_bwd
    a = bwd(dout, x, u, w, b, mean, rstd, False, False, False, "silu")
    c = bwd(dout, x, u, w, b, mean, rstd, False, False, False, "silu")
    assert all(torch.equal(p, q) for p, q in zip(a, c))  # no atomics: bitwise repeatable
    f = lambda t: t.float().cpu().numpy()
    rdx, rdu, rdw, rdb = ro.layer_norm_mul_bwd(f(dout), f(x), f(u), f(w), f(b), 1e-5, "bfloat16", mul_u_activation="silu")
    _close(a[0][::997], rdx[::997], "bfloat16", "dx sample")
    _close(a[1][::997], rdu[::997], "bfloat16", "du sample")
    for got, want, what in ((a[2], rdw, "dw"), (a[3], rdb, "db")):
        rel = np.abs(f(got).astype(np.float64) - want) / np.maximum(np.abs(want), np.abs(want).max() * 1e-2)
        assert rel.max() <= 2.02 * ULP["bfloat16"], (what, float(rel.max()))
    with pytest.raises(ValueError, match="parts"):
        bwd(dout, x, u, w, b, mean, rstd, False, True, False, "silu")  # dout lacks the concatenated part
    # without the saved output there is nothing to differentiate through
    xr = x[:16].clone().requires_grad_(True)
    out = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_fwd(
        xr, u[:16], w, b, 1e-5, 0.0, False, False, False, False, "silu", 0, False, 64)
    assert out[0].numel() == 0
