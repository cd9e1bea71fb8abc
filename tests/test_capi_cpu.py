"""CPU-side checks of the C ABI: the library loads without a GPU, exports every symbol the
header declares, and its mask / tile-skipping logic (the same inline functions the kernels
use) agrees with the oracle's restatement of the reference mask rule."""
import ctypes
import os
import re

import numpy as np
import pytest

from oracle import hstu_oracle
from recir_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    """Every function declared in include/*.h."""
    names = set()
    for header in sorted(f for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")):
        text = open(os.path.join(ROOT, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(b200_(?:hstu|stu)_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = _header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/*.h but not exported"
    assert set(names) == set(_lib.EXPORTS)


def test_version_size_and_strerror():
    lib = _lib.load()
    assert lib.b200_hstu_version() == 1
    assert lib.b200_hstu_params_size() == ctypes.sizeof(_lib.B200HstuParams)
    assert _lib.strerror(0) == "ok"
    for code in range(-6, 0):
        assert "unknown" not in _lib.strerror(code)
    assert "unknown" in _lib.strerror(-99)


def test_argument_errors_detected_on_host():
    lib = _lib.load()
    p = _lib.B200HstuParams()
    assert lib.b200_hstu_fwd(ctypes.byref(p), None) == -6  # struct_size 0
    p.struct_size = ctypes.sizeof(p)
    p.dtype = 7
    assert lib.b200_hstu_fwd(ctypes.byref(p), None) == -2
    p.dtype = _lib.BF16
    p.H, p.Dqk, p.Dv, p.T, p.B, p.max_seq_len = 2, 128, 128, 16, 1, 16
    assert lib.b200_hstu_fwd(ctypes.byref(p), None) == -1  # null seq_offsets
    assert lib.b200_hstu_workspace_bytes(ctypes.byref(p), 0) == 0


def test_backward_workspace_size_is_host_arithmetic():
    """b200_hstu_workspace_bytes needs no GPU: the backward's size follows from T, B, H, max_seq_len, the
    contextual prefix and the recompute flag alone (pointers are only checked for null and alignment)."""
    lib = _lib.load()
    p = _lib.B200HstuParams()
    p.struct_size = ctypes.sizeof(p)
    p.dtype = _lib.BF16
    p.H, p.Dqk, p.Dv, p.T, p.B, p.max_seq_len = 4, 128, 128, 100_000, 64, 2048
    p.flags = _lib.FLAG_CAUSAL | _lib.FLAG_OFFSETS_I64
    fake = 0x7f0000000000  # never dereferenced on the host
    for name in ("q", "k", "v", "o", "d_o", "dq", "dk", "dv", "seq_offsets"):
        setattr(p, name, fake)
    for name in ("q", "k", "v", "o", "do", "dq", "dk", "dv"):
        setattr(p, name + "_row_stride", 4 * 128)
    p.alpha = 0.1
    fwd = lib.b200_hstu_workspace_bytes(ctypes.byref(p), 0)
    bwd = lib.b200_hstu_workspace_bytes(ctypes.byref(p), 1)
    assert 0 < fwd < (1 << 22)
    blocks, nbmax = 100_000 // 128 + 64, 2048 // 128
    tiles = (blocks * (nbmax + 1) + 1) // 2 * 4
    assert fwd + tiles * 32768 <= bwd < fwd + tiles * 32768 + 4096
    p.contextual_seq_len = 2  # all-target sequences keep the whole square: twice the triangle's bound
    assert lib.b200_hstu_workspace_bytes(ctypes.byref(p), 1) >= fwd + blocks * nbmax * 4 * 32768
    p.contextual_seq_len = 0
    p.flags |= _lib.FLAG_BWD_RECOMPUTE_DQ
    assert lib.b200_hstu_workspace_bytes(ctypes.byref(p), 1) == fwd
    p.flags &= ~_lib.FLAG_BWD_RECOMPUTE_DQ
    p.max_seq_len = 1 << 20  # the region would pass the limit of the header: the small workspace again
    assert lib.b200_hstu_workspace_bytes(ctypes.byref(p), 1) == fwd


def _mq(L, t, causal, w, ctx, f):
    q = _lib.B200HstuMaskQuery()
    q.len, q.has_targets, q.num_targets = L, int(t is not None), 0 if t is None else t
    q.causal, q.max_attn_len, q.contextual_seq_len, q.full_attn_size = int(causal), w, ctx, f
    return q


@pytest.mark.parametrize("seed", range(30))
def test_device_keep_rule_matches_oracle_mask(seed):
    lib = _lib.load()
    rng = np.random.default_rng(seed)
    L = int(rng.integers(1, 40))
    t = [None, int(rng.integers(0, L + 3))][seed % 2]
    causal = seed % 5 != 4
    w = int(rng.choice([0, 1, 4, 11]))
    ctx = int(rng.integers(0, 2)) * 2
    f = int(rng.choice([0, 3, 50])) if w > 0 else 0
    ref = hstu_oracle.keep_mask(L, t, causal, w, ctx, f)
    q = _mq(L, t, causal, w, ctx, f)
    got = np.array([[lib.b200_hstu_debug_keep(ctypes.byref(q), m, n) for n in range(L)] for m in range(L)], bool)
    assert (got == ref).all()


@pytest.mark.parametrize("seed", range(60))
def test_tile_classes_and_block_ranges_are_sound(seed):
    """SKIP tiles hold no kept pair, FULL tiles only kept in-range pairs, and the block
    ranges the kernels iterate contain every tile that is not SKIP."""
    lib = _lib.load()
    rng = np.random.default_rng(1000 + seed)
    L = int(rng.integers(1, 700))
    t = [None, int(rng.integers(0, min(L + 3, 300)))][seed % 2]
    if seed % 11 == 0:
        t = L  # all targets
    w = int(rng.choice([0, 0, 5, 100, 130, 300]))
    ctx = int(rng.integers(0, 2))
    f = int(rng.choice([0, 0, 7, 200])) if w > 0 else 0
    keep = hstu_oracle.keep_mask(L, t, True, w, ctx, f)
    q = _mq(L, t, True, w, ctx, f)
    nblk = (L + 127) // 128
    out = (ctypes.c_int32 * 3)()
    for qb in range(nblk):
        lib.b200_hstu_debug_key_blocks(ctypes.byref(q), qb * 128, ctypes.byref(out))
        visited = set(range(out[0], out[1] + 1)) | ({0} if out[2] else set())
        # the kernels rely on the last candidate block of a query block never being skipped
        assert lib.b200_hstu_debug_classify_tile(ctypes.byref(q), qb * 128, out[1] * 128, 1) != 0
        for kb in range(nblk + 1):
            cls = lib.b200_hstu_debug_classify_tile(ctypes.byref(q), qb * 128, kb * 128, 0)
            sub = keep[qb * 128:(qb + 1) * 128, kb * 128:(kb + 1) * 128]
            cls_q = lib.b200_hstu_debug_classify_tile(ctypes.byref(q), qb * 128, kb * 128, 1)
            assert (cls_q == 0) == (cls == 0)
            if cls_q == 2:  # query rows past the end may be anything; keys must all be in range
                assert sub.shape[1] == 128 and sub.all(), (qb, kb)
            if cls == 0:
                assert not sub.any(), (qb, kb)
            else:
                assert kb in visited, (qb, kb, list(out))
            if cls == 2:
                assert sub.shape == (128, 128) and sub.all(), (qb, kb)
            if kb not in visited:
                assert not sub.any(), (qb, kb, list(out))
    for kb in range(nblk):
        lib.b200_hstu_debug_query_blocks(ctypes.byref(q), kb * 128, ctypes.byref(out))
        visited = set(range(out[0], out[1] + 1))
        for qb in range(nblk):
            if qb not in visited:
                assert not keep[qb * 128:(qb + 1) * 128, kb * 128:(kb + 1) * 128].any()


@pytest.mark.parametrize("seed", range(60))
def test_row_and_column_interval_masks_equal_the_keep_rule(seed):
    lib = _lib.load()
    rng = np.random.default_rng(5000 + seed)
    L = int(rng.integers(1, 90))
    t = [None, int(rng.integers(0, L + 3))][seed % 2]
    if seed % 13 == 0:
        t = L
    w = int(rng.choice([0, 0, 1, 5, 20, 200]))
    ctx = int(rng.integers(0, 2))
    f = int(rng.choice([0, 0, 3, 30, 500])) if w > 0 else 0
    keep = hstu_oracle.keep_mask(L, t, True, w, ctx, f)
    q = _mq(L, t, True, w, ctx, f)
    out = (ctypes.c_int32 * 4)()
    ids = np.arange(L)
    for m in range(L + 2):
        lib.b200_hstu_debug_row_mask(ctypes.byref(q), m, ctypes.byref(out))
        lo, hi, diag, extra = list(out)
        got = ((ids >= lo) & (ids < hi)) | (ids == diag) | (ids == extra)
        want = keep[m] if m < L else np.zeros(L, bool)
        assert (got == want).all(), (m, list(out))
    for n in range(L + 2):
        lib.b200_hstu_debug_col_mask(ctypes.byref(q), n, ctypes.byref(out))
        a_lo, a_hi, b_lo, diag = list(out)
        got = (ids == diag) | ((ids >= a_lo) & (ids < a_hi)) | (ids >= b_lo)
        want = keep[:, n] if n < L else np.zeros(L, bool)
        assert (got == want).all(), (n, list(out))


def test_rowwise_params_validation_without_a_gpu():
    """Argument checks of the row-wise entry points run on the host before any launch."""
    lib = _lib.load()
    p = _lib.B200RowwiseParams()
    assert lib.b200_stu_layer_norm_fwd(ctypes.byref(p), None) == -6  # struct_size mismatch
    p.struct_size = ctypes.sizeof(p)
    p.dtype, p.rows, p.cols = _lib.BF16, 4, 20
    assert lib.b200_stu_layer_norm_fwd(ctypes.byref(p), None) == -2  # cols not a multiple of 8
    p.cols = 4096
    assert lib.b200_stu_layer_norm_fwd(ctypes.byref(p), None) == -2  # too wide
    p.cols = 64
    assert lib.b200_stu_layer_norm_fwd(ctypes.byref(p), None) == -1  # null pointers
    assert lib.b200_stu_layer_norm_mul_parts(0) == 1
    assert lib.b200_stu_layer_norm_mul_parts(_lib.ROWWISE_CONCAT_U | _lib.ROWWISE_CONCAT_X) == 3
    p.rows = 0
    assert lib.b200_stu_layer_norm_fwd(ctypes.byref(p), None) == 0  # nothing to do, nothing launched


def test_jagged_params_validation_without_a_gpu():
    lib = _lib.load()
    p = _lib.B200JaggedParams()
    assert lib.b200_stu_jagged_copy(ctypes.byref(p), None) == -6  # struct_size mismatch
    p.struct_size = ctypes.sizeof(p)
    p.mode, p.row_bytes = 7, 16
    assert lib.b200_stu_jagged_copy(ctypes.byref(p), None) == -1  # unknown mode
    p.mode, p.row_bytes = _lib.JAGGED_CONCAT, 3
    assert lib.b200_stu_jagged_copy(ctypes.byref(p), None) == -1  # odd row size
    p.row_bytes, p.dst_rows = 16, 0
    assert lib.b200_stu_jagged_copy(ctypes.byref(p), None) == 0   # nothing to write, nothing launched
    p.dst_rows, p.num_seqs = 4, 2
    assert lib.b200_stu_jagged_copy(ctypes.byref(p), None) == -1  # null pointers
