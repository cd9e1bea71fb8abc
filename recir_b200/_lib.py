"""ctypes binding of the C ABI in ``include/b200_hstu.h`` (the only route to the kernels).

There is no fallback: if the shared library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libb200_hstu.so")

F32, BF16, F16 = 0, 1, 2
FLAG_CAUSAL = 0x1
FLAG_OFFSETS_I64 = 0x2
FLAG_TARGETS_I64 = 0x4
FLAG_SCALE_PER_TOKEN = 0x8
FLAG_FORCE_SIMT = 0x10
FLAG_BWD_SKIP_DQ = 0x20
FLAG_BWD_SKIP_DKV = 0x40
FLAG_TRACE = 0x80
FLAG_BWD_RECOMPUTE_DQ = 0x100

EXPORTS = (
    "b200_hstu_fwd", "b200_hstu_bwd", "b200_hstu_workspace_bytes", "b200_hstu_uses_tensor_cores",
    "b200_hstu_launch_count", "b200_hstu_strerror", "b200_hstu_version", "b200_hstu_params_size",
    "b200_hstu_debug_keep", "b200_hstu_debug_classify_tile", "b200_hstu_debug_key_blocks",
    "b200_hstu_debug_query_blocks", "b200_hstu_fwd_static_scratch", "b200_hstu_debug_row_mask",
    "b200_hstu_debug_col_mask", "b200_hstu_last_cuda_error", "b200_hstu_debug_bounded_wait",
    # include/b200_stu_rowwise.h
    "b200_stu_layer_norm_fwd", "b200_stu_layer_norm_mul_fwd", "b200_stu_layer_norm_mul_parts",
    "b200_stu_layer_norm_bwd", "b200_stu_layer_norm_bwd_workspace_bytes", "b200_stu_layer_norm_mul_bwd",
    # include/b200_stu_gemm.h
    "b200_stu_addmm", "b200_stu_addmm_supported", "b200_stu_jagged_dense_bmm_add", "b200_stu_jagged_bmm_workspace_bytes",
    "b200_stu_fp8_rowwise_addmm", "b200_stu_fp8_rowwise_addmm_supported",
    # include/b200_stu_jagged.h
    "b200_stu_jagged_copy",
    # include/b200_stu_embed.h
    "b200_stu_add_ts_pos_emb",
)
STATIC_SCRATCH_BYTES = 4 << 20


class B200HstuMaskQuery(ctypes.Structure):
    """Mirror of ``struct B200HstuMaskQuery`` (host-only diagnostics)."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "len", "has_targets", "num_targets", "causal", "max_attn_len", "contextual_seq_len",
        "full_attn_size")]


class B200HstuParams(ctypes.Structure):
    """Mirror of ``struct B200HstuParams``; field order and types must match the header."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("flags", ctypes.c_uint32),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p), ("d_o", ctypes.c_void_p),
        ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p),
        ("seq_offsets", ctypes.c_void_p), ("num_targets", ctypes.c_void_p),
        ("attn_scale", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
        ("status", ctypes.c_void_p),
        ("T", ctypes.c_int64),
        ("q_row_stride", ctypes.c_int64), ("k_row_stride", ctypes.c_int64),
        ("v_row_stride", ctypes.c_int64), ("o_row_stride", ctypes.c_int64),
        ("do_row_stride", ctypes.c_int64), ("dq_row_stride", ctypes.c_int64),
        ("dk_row_stride", ctypes.c_int64), ("dv_row_stride", ctypes.c_int64),
        ("B", ctypes.c_int32), ("H", ctypes.c_int32), ("Dqk", ctypes.c_int32), ("Dv", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32), ("max_attn_len", ctypes.c_int32),
        ("contextual_seq_len", ctypes.c_int32), ("full_attn_size", ctypes.c_int32),
        ("alpha", ctypes.c_float),
    ]


# flags of include/b200_stu_rowwise.h
ROWWISE_SWISH, ROWWISE_STATS_IN, ROWWISE_SILU_U, ROWWISE_CONCAT_U = 0x1, 0x2, 0x4, 0x8
ROWWISE_CONCAT_X, ROWWISE_ACT_SILU, ROWWISE_ACT_SIGMOID = 0x10, 0x20, 0x40


class B200RowwiseParams(ctypes.Structure):
    """Mirror of ``struct B200RowwiseParams`` (include/b200_stu_rowwise.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64), ("u_row_stride", ctypes.c_int64),
        ("y_row_stride", ctypes.c_int64), ("q8_row_stride", ctypes.c_int64),
        ("x", ctypes.c_void_p), ("u", ctypes.c_void_p), ("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("mean_in", ctypes.c_void_p), ("rstd_in", ctypes.c_void_p),
        ("y", ctypes.c_void_p), ("mean", ctypes.c_void_p), ("rstd", ctypes.c_void_p),
        ("scale", ctypes.c_void_p), ("q8", ctypes.c_void_p),
    ]


class B200LayerNormBwdParams(ctypes.Structure):
    """Mirror of ``struct B200LayerNormBwdParams`` (include/b200_stu_rowwise.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
        ("dy_row_stride", ctypes.c_int64), ("x_row_stride", ctypes.c_int64), ("dx_row_stride", ctypes.c_int64),
        ("dy", ctypes.c_void_p), ("x", ctypes.c_void_p), ("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("mean", ctypes.c_void_p), ("rstd", ctypes.c_void_p),
        ("dx", ctypes.c_void_p), ("dweight", ctypes.c_void_p), ("dbias", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
    ]


class B200LayerNormMulBwdParams(ctypes.Structure):
    """Mirror of ``struct B200LayerNormMulBwdParams`` (include/b200_stu_rowwise.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
        ("dout_row_stride", ctypes.c_int64), ("x_row_stride", ctypes.c_int64), ("u_row_stride", ctypes.c_int64),
        ("dx_row_stride", ctypes.c_int64), ("du_row_stride", ctypes.c_int64),
        ("dout", ctypes.c_void_p), ("x", ctypes.c_void_p), ("u", ctypes.c_void_p),
        ("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("mean", ctypes.c_void_p), ("rstd", ctypes.c_void_p),
        ("dx", ctypes.c_void_p), ("du", ctypes.c_void_p), ("dweight", ctypes.c_void_p), ("dbias", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
    ]


class B200Fp8GemmParams(ctypes.Structure):
    """Mirror of ``struct B200Fp8GemmParams`` (include/b200_stu_gemm.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("out_dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("M", ctypes.c_int64), ("K", ctypes.c_int64), ("N", ctypes.c_int64),
        ("a_row_stride", ctypes.c_int64), ("b_row_stride", ctypes.c_int64), ("out_row_stride", ctypes.c_int64),
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("a_scale", ctypes.c_void_p), ("b_scale", ctypes.c_void_p),
        ("bias", ctypes.c_void_p), ("out", ctypes.c_void_p), ("status", ctypes.c_void_p),
    ]


# flags of include/b200_stu_gemm.h
GEMM_LAYER_NORM, GEMM_SWISH = 0x1, 0x2


class B200GemmParams(ctypes.Structure):
    """Mirror of ``struct B200GemmParams`` (include/b200_stu_gemm.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
        ("M", ctypes.c_int64), ("K", ctypes.c_int64), ("N", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64), ("w_row_stride", ctypes.c_int64), ("out_row_stride", ctypes.c_int64),
        ("bias_row_stride", ctypes.c_int64),
        ("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("ln_weight", ctypes.c_void_p), ("ln_bias", ctypes.c_void_p),
        ("out", ctypes.c_void_p), ("mean", ctypes.c_void_p), ("rstd", ctypes.c_void_p), ("status", ctypes.c_void_p),
    ]


# modes of include/b200_stu_jagged.h
JAGGED_TO_PADDED_DENSE, DENSE_TO_JAGGED, JAGGED_CONCAT, JAGGED_SPLIT_LEFT, JAGGED_SPLIT_RIGHT = range(5)
JAGGED_OFFSETS_I64 = 0x1


class B200JaggedParams(ctypes.Structure):
    """Mirror of ``struct B200JaggedParams`` (include/b200_stu_jagged.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("mode", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("num_seqs", ctypes.c_int64), ("padded_len", ctypes.c_int64), ("dst_rows", ctypes.c_int64),
        ("src0_rows", ctypes.c_int64), ("src1_rows", ctypes.c_int64), ("row_bytes", ctypes.c_int64),
        ("dst_row_stride", ctypes.c_int64), ("src0_row_stride", ctypes.c_int64), ("src1_row_stride", ctypes.c_int64),
        ("src0", ctypes.c_void_p), ("src1", ctypes.c_void_p), ("dst", ctypes.c_void_p),
        ("offsets0", ctypes.c_void_p), ("offsets1", ctypes.c_void_p),
        ("pad", ctypes.c_ubyte * 16),
    ]


# flags of include/b200_stu_embed.h
EMBED_OFFSETS_I64, EMBED_LENGTHS_I64, EMBED_INTERLEAVE, EMBED_SQRT, EMBED_TABLES_F32 = 0x1, 0x2, 0x4, 0x8, 0x10


class B200EmbedParams(ctypes.Structure):
    """Mirror of ``struct B200EmbedParams`` (include/b200_stu_embed.h)."""

    _fields_ = [
        ("struct_size", ctypes.c_uint32), ("flags", ctypes.c_uint32),
        ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("num_seqs", ctypes.c_int64),
        ("pos_rows", ctypes.c_int64), ("ts_cols", ctypes.c_int64), ("max_contextual_seq_len", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64), ("out_row_stride", ctypes.c_int64),
        ("pos_row_stride", ctypes.c_int64), ("ts_table_row_stride", ctypes.c_int64),
        ("x", ctypes.c_void_p), ("pos_table", ctypes.c_void_p), ("ts_table", ctypes.c_void_p),
        ("timestamps", ctypes.c_void_p), ("seq_offsets", ctypes.c_void_p), ("seq_lengths", ctypes.c_void_p),
        ("num_targets", ctypes.c_void_p), ("out", ctypes.c_void_p),
        ("pos_index", ctypes.c_void_p), ("ts_index", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Load ``libb200_hstu.so`` (built by ``python -m recir_b200.build``); raises if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: the CUDA library has not been built "
            "(run `python -m recir_b200.build`); there is no fallback implementation")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER(B200HstuParams)
    lib.b200_hstu_fwd.argtypes = [P, ctypes.c_void_p]
    lib.b200_hstu_fwd.restype = ctypes.c_int
    lib.b200_hstu_fwd_static_scratch.argtypes = [P, ctypes.c_void_p]
    lib.b200_hstu_fwd_static_scratch.restype = ctypes.c_int
    lib.b200_hstu_bwd.argtypes = [P, ctypes.c_void_p]
    lib.b200_hstu_bwd.restype = ctypes.c_int
    lib.b200_hstu_workspace_bytes.argtypes = [P, ctypes.c_int]
    lib.b200_hstu_workspace_bytes.restype = ctypes.c_size_t
    lib.b200_hstu_uses_tensor_cores.argtypes = [P, ctypes.c_int]
    lib.b200_hstu_uses_tensor_cores.restype = ctypes.c_int
    lib.b200_hstu_launch_count.argtypes = [P, ctypes.c_int]
    lib.b200_hstu_launch_count.restype = ctypes.c_int
    lib.b200_hstu_strerror.argtypes = [ctypes.c_int]
    lib.b200_hstu_strerror.restype = ctypes.c_char_p
    lib.b200_hstu_last_cuda_error.argtypes = []
    lib.b200_hstu_last_cuda_error.restype = ctypes.c_char_p
    lib.b200_hstu_debug_bounded_wait.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_void_p]
    lib.b200_hstu_debug_bounded_wait.restype = ctypes.c_int
    lib.b200_hstu_version.argtypes = []
    lib.b200_hstu_version.restype = ctypes.c_int
    lib.b200_hstu_params_size.argtypes = []
    lib.b200_hstu_params_size.restype = ctypes.c_size_t
    MQ = ctypes.POINTER(B200HstuMaskQuery)
    lib.b200_hstu_debug_keep.argtypes = [MQ, ctypes.c_int, ctypes.c_int]
    lib.b200_hstu_debug_keep.restype = ctypes.c_int
    lib.b200_hstu_debug_classify_tile.argtypes = [MQ, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    for fn in (lib.b200_hstu_debug_row_mask, lib.b200_hstu_debug_col_mask):
        fn.argtypes = [MQ, ctypes.c_int, ctypes.POINTER(ctypes.c_int32 * 4)]
        fn.restype = None
    lib.b200_hstu_debug_classify_tile.restype = ctypes.c_int
    lib.b200_hstu_debug_key_blocks.argtypes = [MQ, ctypes.c_int, ctypes.POINTER(ctypes.c_int32 * 3)]
    lib.b200_hstu_debug_key_blocks.restype = None
    lib.b200_hstu_debug_query_blocks.argtypes = [MQ, ctypes.c_int, ctypes.POINTER(ctypes.c_int32 * 3)]
    lib.b200_hstu_debug_query_blocks.restype = None
    RP = ctypes.POINTER(B200RowwiseParams)
    for fn in (lib.b200_stu_layer_norm_fwd, lib.b200_stu_layer_norm_mul_fwd):
        fn.argtypes = [RP, ctypes.c_void_p]
        fn.restype = ctypes.c_int
    lib.b200_stu_layer_norm_mul_parts.argtypes = [ctypes.c_uint32]
    lib.b200_stu_layer_norm_mul_parts.restype = ctypes.c_int
    lib.b200_stu_layer_norm_bwd.argtypes = [ctypes.POINTER(B200LayerNormBwdParams), ctypes.c_void_p]
    lib.b200_stu_layer_norm_bwd.restype = ctypes.c_int
    lib.b200_stu_layer_norm_mul_bwd.argtypes = [ctypes.POINTER(B200LayerNormMulBwdParams), ctypes.c_void_p]
    lib.b200_stu_layer_norm_mul_bwd.restype = ctypes.c_int
    lib.b200_stu_layer_norm_bwd_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    lib.b200_stu_layer_norm_bwd_workspace_bytes.restype = ctypes.c_size_t
    GP = ctypes.POINTER(B200GemmParams)
    lib.b200_stu_addmm.argtypes = [GP, ctypes.c_void_p]
    lib.b200_stu_addmm.restype = ctypes.c_int
    FP = ctypes.POINTER(B200Fp8GemmParams)
    lib.b200_stu_fp8_rowwise_addmm.argtypes = [FP, ctypes.c_void_p]
    lib.b200_stu_fp8_rowwise_addmm.restype = ctypes.c_int
    lib.b200_stu_fp8_rowwise_addmm_supported.argtypes = [FP]
    lib.b200_stu_fp8_rowwise_addmm_supported.restype = ctypes.c_int
    lib.b200_stu_addmm_supported.argtypes = [GP]
    lib.b200_stu_addmm_supported.restype = ctypes.c_int
    lib.b200_stu_jagged_bmm_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    lib.b200_stu_jagged_bmm_workspace_bytes.restype = ctypes.c_size_t
    lib.b200_stu_jagged_dense_bmm_add.argtypes = [GP, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                                  ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
    lib.b200_stu_jagged_dense_bmm_add.restype = ctypes.c_int
    lib.b200_stu_add_ts_pos_emb.argtypes = [ctypes.POINTER(B200EmbedParams), ctypes.c_void_p]
    lib.b200_stu_add_ts_pos_emb.restype = ctypes.c_int
    lib.b200_stu_jagged_copy.argtypes = [ctypes.POINTER(B200JaggedParams), ctypes.c_void_p]
    lib.b200_stu_jagged_copy.restype = ctypes.c_int
    if lib.b200_hstu_params_size() != ctypes.sizeof(B200HstuParams):
        raise RuntimeError("B200HstuParams layout mismatch between Python binding and library")
    _lib = lib
    return lib


def strerror(code: int) -> str:
    msg = load().b200_hstu_strerror(code).decode()
    if code == -5:
        detail = load().b200_hstu_last_cuda_error().decode()
        if detail:
            msg += f" ({detail})"
    return msg
