"""The numpy restatement of the reference's row-wise STU operators against golden vectors made by
the reference's own compiled operators (tests/golden/make_rowwise_golden.py)."""
import os

import numpy as np
import pytest

from oracle import rowwise_oracle as ro

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "rowwise_golden.npz"))
LN = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("ln_")})
MUL = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("mul_")})
# one unit in the last place of the case's dtype, relative
ULP = {"float32": 2e-6, "bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}


def _close(got, want, dtype, what):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape, what
    if got.size == 0:
        return
    # float32: results are sums of O(1) terms, so the error is absolute; 16-bit: one last-place flip
    tol = ULP[dtype] * np.maximum(np.abs(want), 1.0 if dtype == "float32" else 1e-3)
    bad = np.abs(got - want) > tol
    # the restatement reproduces the reference's roundings: at most a stray last-place flip
    assert bad.mean() <= 1e-3, f"{what}: {bad.sum()} of {bad.size} beyond one ulp"
    assert np.abs(got - want).max() <= 4 * tol.max(), what


@pytest.mark.parametrize("name", LN)
def test_layer_norm_matches_reference(name):
    dt, affine, swish, stats_in = GOLD[f"{name}/cfg"]
    x = GOLD[f"{name}/x"]
    w = GOLD[f"{name}/w"] if affine == "1" else None
    b = GOLD[f"{name}/b"] if affine == "1" else None
    kw = dict(mean=GOLD[f"{name}/mean_in"], rstd=GOLD[f"{name}/rstd_in"]) if stats_in == "1" else {}
    y, mean, rstd = ro.weighted_layer_norm(x, w, b, 1e-5, dt, is_swish=swish == "1", **kw)
    _close(y, GOLD[f"{name}/y"], dt, "y")
    _close(mean, GOLD[f"{name}/mean"], "float32", "mean")
    _close(rstd, GOLD[f"{name}/rstd"], "float32", "rstd")


@pytest.mark.parametrize("name", MUL)
def test_layer_norm_mul_matches_reference(name):
    dt, silu_u, cat_u, cat_x, act = GOLD[f"{name}/cfg"]
    y, mean, rstd, scale, q8 = ro.layer_norm_mul_quantized(
        GOLD[f"{name}/x"], GOLD[f"{name}/u"], GOLD[f"{name}/w"], GOLD[f"{name}/b"], 1e-5, dt,
        silu_u=silu_u == "1", concat_u=cat_u == "1", concat_x=cat_x == "1", mul_u_activation=act)
    _close(y, GOLD[f"{name}/y"], dt, "y")
    _close(mean, GOLD[f"{name}/mean"], "float32", "mean")
    _close(rstd, GOLD[f"{name}/rstd"], "float32", "rstd")
    _close(scale, GOLD[f"{name}/scale"], "float32", "scale")
    want = GOLD[f"{name}/q8"]
    assert q8.shape == want.shape
    # e4m3 codes: identical except where the value sat within rounding noise of a code boundary
    diff = q8.astype(np.int16) != want.astype(np.int16)
    assert diff.mean() <= 2e-3, f"{diff.sum()} of {diff.size} fp8 codes differ"
    mag = np.abs((q8 & 0x7F).astype(np.int16) - (want & 0x7F).astype(np.int16))
    assert mag.max() <= 1 and ((q8 ^ want) & 0x80)[mag > 0].sum() == 0 or diff.sum() == 0


LNQ = sorted({k.split("/")[0] for k in GOLD.files if k.startswith("lnq_")})


@pytest.mark.parametrize("name", LNQ)
def test_quantized_layer_norm_matches_reference(name):
    dt = str(GOLD[f"{name}/cfg"][0])
    y, mean, rstd = ro.weighted_layer_norm(GOLD[f"{name}/x"], GOLD[f"{name}/w"], GOLD[f"{name}/b"], 1e-5, dt)
    scale, q8 = ro.quantize_fp8_rowwise(y)
    _close(y, GOLD[f"{name}/y"], dt, "y")
    _close(scale, GOLD[f"{name}/scale"], "float32", "scale")
    diff = q8 != GOLD[f"{name}/q8"]
    assert diff.mean() <= 2e-3


def test_e4m3_known_codes():
    # float8 e4m3fn: bias 7, 3 mantissa bits, subnormal step 2^-9, largest finite 448 = 0x7E
    vals = np.array([0.0, 2.0 ** -9, 2.0 ** -6, 1.0, 1.5, 448.0, -448.0, -1.0, 0.0625 * 1.125], np.float32)
    want = np.array([0x00, 0x01, 0x08, 0x38, 0x3C, 0x7E, 0xFE, 0xB8, 0x19], np.uint8)
    assert (ro.e4m3_encode(vals) == want).all()
    # ties go to the even code: halfway between 1.0 (0x38) and 1.125 (0x39) -> 0x38
    assert ro.e4m3_encode(np.array([1.0625], np.float32))[0] == 0x38
    assert ro.e4m3_encode(np.array([1.1875], np.float32))[0] == 0x3A


FP8MM = np.load(os.path.join(os.path.dirname(__file__), "golden", "fp8_addmm_golden.npz"))


def test_e4m3_decode_inverts_encode_on_every_finite_code():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    vals = ro.e4m3_decode(codes)
    assert np.isfinite(vals).all() and float(np.abs(vals).max()) == 448.0
    back = ro.e4m3_encode(vals)
    # +0 and -0 keep their sign bit; every other code round-trips exactly
    assert np.array_equal(back, codes)


@pytest.mark.parametrize("name", [str(n) for n in FP8MM["names"]])
def test_fp8_rowwise_addmm_matches_reference(name):
    dt, has_bias = FP8MM[f"{name}/cfg"]
    bias = FP8MM[f"{name}/bias"] if has_bias == "1" else None
    y = ro.fp8_rowwise_addmm(FP8MM[f"{name}/a"], FP8MM[f"{name}/b"], FP8MM[f"{name}/a_scale"],
                             FP8MM[f"{name}/b_scale"], bias, dt)
    want = FP8MM[f"{name}/y"].astype(np.float64)
    # float32: the reference sums K products in float32 in its own order; 16-bit: one last-place flip
    tol = (1e-5 if dt == "float32" else ULP[dt]) * np.maximum(np.abs(want), float(np.abs(want).max()) * 1e-2)
    assert (np.abs(y.astype(np.float64) - want) <= tol).all()


JBMM = np.load(os.path.join(os.path.dirname(__file__), "golden", "jagged_bmm_golden.npz"))


@pytest.mark.parametrize("name", [str(n) for n in JBMM["names"]])
def test_jagged_dense_bmm_add_matches_reference(name):
    dt, elementwise = JBMM[f"{name}/cfg"]
    y = ro.jagged_dense_bmm_add(JBMM[f"{name}/offsets"], JBMM[f"{name}/jagged"], JBMM[f"{name}/dense"],
                                JBMM[f"{name}/bias"], elementwise == "1", dt)
    want = JBMM[f"{name}/y"].astype(np.float64)
    assert y.shape == want.shape
    # float32: summation order; bfloat16: the reference rounds the product before the bias is added
    tol = (1e-5 if dt == "float32" else 2 * ULP[dt]) * np.maximum(np.abs(want), float(np.abs(want).max()) * 5e-2)
    assert (np.abs(y.astype(np.float64) - want) <= tol).all(), float(np.abs(y - want).max())


BWD = np.load(os.path.join(os.path.dirname(__file__), "golden", "layer_norm_bwd_golden.npz"))
BWD_NAMES = sorted({k.split("/")[0] for k in BWD.files})


@pytest.mark.parametrize("name", BWD_NAMES)
def test_layer_norm_backward_matches_reference_autograd(name):
    """The closed-form gradients against autograd through the reference's compiled composite
    (tests/golden/make_layer_norm_bwd_golden.py).  The composite accumulates in float32 and rounds once, the
    restatement in float64: float32 cases agree to 3e-5 of the gradient scale, 16-bit cases to one unit in the
    last place on all but a stray element (the column sums dw, db add up to 140 rounded float32 terms)."""
    dt, affine, swish = BWD[f"{name}/cfg"]
    w = BWD[f"{name}/w"] if affine == "1" else None
    b = BWD[f"{name}/b"] if affine == "1" else None
    dx, dw, db = ro.weighted_layer_norm_bwd(BWD[f"{name}/dy"], BWD[f"{name}/x"], w, b, 1e-5, dt, is_swish=swish == "1")
    pairs = [("dx", dx, BWD[f"{name}/dx"])]
    if affine == "1":
        pairs += [("dw", dw, BWD[f"{name}/dw"]), ("db", db, BWD[f"{name}/db"])]
    for what, got, want in pairs:
        got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
        scale = np.maximum(np.abs(want), np.abs(want).max() * 1e-2)
        rel = np.abs(got - want) / scale
        if dt == "float32":
            assert rel.max() <= 3e-5, (what, float(rel.max()))
        else:
            assert rel.max() <= 2.02 * ULP[dt], (what, float(rel.max()))
            assert (rel > 1.01 * ULP[dt]).mean() <= 5e-3, what


MULBWD = np.load(os.path.join(os.path.dirname(__file__), "golden", "layer_norm_mul_bwd_golden.npz"))
MULBWD_NAMES = sorted({k.split("/")[0] for k in MULBWD.files})
# relative L2 / largest error over largest value: the composite differentiates through 16-bit intermediates
# (normalised rows, gate, product each rounded), the restatement is float64 rounded once
MULBWD_TOL = {"float32": (1e-6, 1e-6), "bfloat16": (6e-3, 8e-3), "float16": (8e-4, 1.5e-3)}


def mul_bwd_case(name):
    dt, silu_u, concat_u, concat_x, act = MULBWD[f"{name}/cfg"]
    return dt, dict(silu_u=silu_u == "1", concat_u=concat_u == "1", concat_x=concat_x == "1", mul_u_activation=str(act))


@pytest.mark.parametrize("name", MULBWD_NAMES)
def test_gate_stage_backward_matches_reference_autograd(name):
    """Closed-form gradients of the gate stage (layer norm times act(u), optional pass-through parts) against
    autograd through the reference's compiled composite (tests/golden/make_layer_norm_mul_bwd_golden.py)."""
    dt, kw = mul_bwd_case(name)
    got = ro.layer_norm_mul_bwd(MULBWD[f"{name}/dout"], MULBWD[f"{name}/x"], MULBWD[f"{name}/u"], MULBWD[f"{name}/w"],
                                MULBWD[f"{name}/b"], 1e-5, dt, **kw)
    for what, g in zip(("dx", "du", "dw", "db"), got):
        want = MULBWD[f"{name}/{what}"].astype(np.float64)
        g = np.asarray(g, np.float64)
        assert g.shape == want.shape
        l2, mx = MULBWD_TOL[dt]
        assert np.linalg.norm(g - want) / np.linalg.norm(want) <= l2, what
        assert np.abs(g - want).max() / np.abs(want).max() <= mx, what
