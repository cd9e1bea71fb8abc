"""``torch.library`` operators for the row-wise STU-layer kernels either side of the attention.

Positionally identical to the reference's operators, so the same node-retargeting swap applies
(``recir/lowering/op_swap.py:78-97``):

* ``recir::b200_weighted_layer_norm_fwd`` -- schema of
  ``generative_recommenders::triton_weighted_layer_norm_fwd``
  (``recir/ops/kjt_split_per_feature.cpp:724-727``, semantics ``:197-244``);
* ``recir::b200_weighted_layer_norm_quantization_fwd`` -- schema of
  ``generative_recommenders::_triton_weighted_layer_norm_quantization_fwd_impl`` (``:740-743``,
  semantics ``:504-531``): the layer norm plus the row-wise fp8 copy of its output;
* ``recir::b200_layer_norm_mul_dropout_quantization_fwd`` -- schema of
  ``generative_recommenders::_triton_layer_norm_mul_dropout_quantization_fwd_impl``
  (``:744-747``, semantics ``:558-600``).  Like the reference's CPU operator it applies no dropout
  (``dropout_ratio``, ``training`` and ``seed`` are accepted and ignored).

Forward only (the reference differentiates its composites through ATen; a fused backward is not
built).  CUDA tensors only; there is no CPU implementation.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _check, _DTYPES

_LIBDEF = torch.library.Library("recir", "FRAGMENT")
_LIBDEF.define(
    "b200_weighted_layer_norm_fwd(Tensor x, Tensor? weight, Tensor? bias, float eps, Tensor? mean=None, "
    "Tensor? rstd=None, bool is_swish=False) -> (Tensor, Tensor, Tensor)")
_LIBDEF.define(
    "b200_layer_norm_mul_dropout_quantization_fwd(Tensor x, Tensor u, Tensor weight, Tensor bias, float eps, "
    "float dropout_ratio, bool training, bool silu_u, bool concat_u, bool concat_x, str mul_u_activation_type, "
    "int seed, bool save_y, int BLOCK_D) -> (Tensor, Tensor, Tensor, Tensor, Tensor)")

_LIBDEF.define("b200_addmm_fwd(Tensor x, Tensor w, Tensor y) -> Tensor")
_LIBDEF.define(
    "b200_fp8_rowwise_addmm_fwd(Tensor a, Tensor b, Tensor a_scale, Tensor b_scale, Tensor bias, bool has_bias, "
    "bool bias_is_2d, ScalarType dot_out_dtype, bool allow_tf32, bool use_fast_accum) -> Tensor")
_LIBDEF.define(
    "b200_weighted_layer_norm_quantization_fwd(Tensor x, Tensor weight, Tensor bias, float eps, Tensor mean, Tensor rstd, "
    "int BLOCK_D) -> (Tensor, Tensor, Tensor, Tensor, Tensor)")

_LIBDEF.define(
    "b200_jagged_dense_bmm_add_fwd(int max_seq_len, Tensor seq_offsets, Tensor jagged, Tensor dense, Tensor bias, "
    "bool elementwise=False) -> (Tensor, int, int, int)")

# Kernel launches issued through this module since import.
launch_counter = 0


def _rows2d(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0 else t.contiguous()


def _validate(x, weight, bias):
    # messages of recir/ops/kjt_split_per_feature.cpp:205-218
    if x.dim() != 2:
        raise ValueError("x must be two-dimensional")
    if x.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {x.dtype}: expected float32, bfloat16 or float16")
    if weight is not None:
        if bias is None:
            raise ValueError("bias is required when weight is provided")
        if weight.dim() != 1 or weight.numel() != x.shape[1]:
            raise ValueError("weight must match the feature dimension")
        if bias.dim() != 1 or bias.numel() != x.shape[1]:
            raise ValueError("bias must match the feature dimension")
    if x.shape[1] % 8 != 0 or x.shape[1] > 2048:
        raise ValueError("the feature dimension must be a multiple of 8 and at most 2048")


def _params(x, weight, bias, eps):
    p = _lib.B200RowwiseParams()
    p.struct_size = ctypes.sizeof(p)
    p.dtype = _DTYPES[x.dtype]
    p.eps = float(eps)
    p.rows, p.cols = x.shape
    p.x, p.x_row_stride = x.data_ptr(), x.stride(0)
    keep = [x]
    if weight is not None:
        w, b = weight.to(x.dtype).contiguous(), bias.to(x.dtype).contiguous()
        keep += [w, b]
        p.weight, p.bias = w.data_ptr(), b.data_ptr()
    return p, keep


def _layer_norm_cuda(x, weight, bias, eps, mean=None, rstd=None, is_swish=False, _fp8=False):
    global launch_counter
    _validate(x, weight, bias)
    if is_swish and weight is None:
        raise ValueError("is_swish requires learnable layer normalization")
    x = _rows2d(x)
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    mean_out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    rstd_out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    scale = torch.empty(x.shape[0], dtype=torch.float32, device=x.device) if _fp8 else None
    q8 = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device) if _fp8 else None
    if x.shape[0] == 0:
        return (y, mean_out, rstd_out, scale, q8) if _fp8 else (y, mean_out, rstd_out)
    p, keep = _params(x, weight, bias, eps)
    if _fp8:
        p.scale, p.q8, p.q8_row_stride = scale.data_ptr(), q8.data_ptr(), q8.stride(0)
    if mean is not None and rstd is not None:
        if mean.numel() != x.shape[0] or rstd.numel() != x.shape[0]:
            raise ValueError("mean and rstd must match the row count")
        m_in, r_in = mean.to(torch.float32).contiguous(), rstd.to(torch.float32).contiguous()
        keep += [m_in, r_in]
        p.mean_in, p.rstd_in = m_in.data_ptr(), r_in.data_ptr()
        p.flags |= _lib.ROWWISE_STATS_IN
    if is_swish:
        p.flags |= _lib.ROWWISE_SWISH
    p.y, p.y_row_stride = y.data_ptr(), y.stride(0)
    p.mean, p.rstd = mean_out.data_ptr(), rstd_out.data_ptr()
    with torch.cuda.device(x.device):
        rc = _lib.load().b200_stu_layer_norm_fwd(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_layer_norm_fwd")
    launch_counter += 1
    del keep
    return (y, mean_out, rstd_out, scale, q8) if _fp8 else (y, mean_out, rstd_out)


def _layer_norm_quant_cuda(x, weight, bias, eps, mean, rstd, BLOCK_D):
    """``generative_recommenders::_triton_weighted_layer_norm_quantization_fwd_impl``
    (``recir/ops/kjt_split_per_feature.cpp:504-531``): empty ``mean`` / ``rstd`` mean "compute them"."""
    given = mean.numel() != 0 and rstd.numel() != 0
    return _layer_norm_cuda(x, weight, bias, eps, mean if given else None, rstd if given else None, False, _fp8=True)


def _mul_flags(silu_u, concat_u, concat_x, act):
    if act not in ("none", "silu", "sigmoid"):
        raise ValueError(f"unknown mul_u_activation_type {act!r}")
    return ((_lib.ROWWISE_SILU_U if silu_u else 0) | (_lib.ROWWISE_CONCAT_U if concat_u else 0)
            | (_lib.ROWWISE_CONCAT_X if concat_x else 0)
            | (_lib.ROWWISE_ACT_SILU if act == "silu" else (_lib.ROWWISE_ACT_SIGMOID if act == "sigmoid" else 0)))


def _layer_norm_mul_cuda(x, u, weight, bias, eps, dropout_ratio, training, silu_u, concat_u, concat_x,
                         mul_u_activation_type, seed, save_y, BLOCK_D):
    global launch_counter
    _validate(x, weight, bias)
    if u.shape != x.shape or u.dtype != x.dtype:
        raise ValueError("u must have the shape and dtype of x")
    x, u = _rows2d(x), _rows2d(u)
    flags = _mul_flags(silu_u, concat_u, concat_x, mul_u_activation_type)
    parts = 1 + int(bool(concat_u)) + int(bool(concat_x))
    rows, cols = x.shape
    dev = x.device
    y = torch.empty((rows, parts * cols), dtype=x.dtype, device=dev) if save_y else torch.empty((0,), dtype=x.dtype, device=dev)
    mean = torch.empty(rows, dtype=torch.float32, device=dev)
    rstd = torch.empty(rows, dtype=torch.float32, device=dev)
    scale = torch.empty(rows, dtype=torch.float32, device=dev)
    q8 = torch.empty((rows, parts * cols), dtype=torch.float8_e4m3fn, device=dev)
    if rows == 0:
        return y, mean, rstd, scale, q8
    p, keep = _params(x, weight, bias, eps)
    p.flags = flags
    p.u, p.u_row_stride = u.data_ptr(), u.stride(0)
    if save_y:
        p.y, p.y_row_stride = y.data_ptr(), y.stride(0)
    p.mean, p.rstd, p.scale = mean.data_ptr(), rstd.data_ptr(), scale.data_ptr()
    p.q8, p.q8_row_stride = q8.data_ptr(), q8.stride(0)
    with torch.cuda.device(dev):
        rc = _lib.load().b200_stu_layer_norm_mul_fwd(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_layer_norm_mul_fwd")
    launch_counter += 1
    del keep
    return y, mean, rstd, scale, q8


def _layer_norm_fake(x, weight, bias, eps, mean=None, rstd=None, is_swish=False):
    return (torch.empty_like(x, memory_format=torch.contiguous_format),
            x.new_empty((x.shape[0],), dtype=torch.float32), x.new_empty((x.shape[0],), dtype=torch.float32))


def _layer_norm_mul_fake(x, u, weight, bias, eps, dropout_ratio, training, silu_u, concat_u, concat_x,
                         mul_u_activation_type, seed, save_y, BLOCK_D):
    parts = 1 + int(bool(concat_u)) + int(bool(concat_x))
    rows, cols = x.shape
    y = x.new_empty((rows, parts * cols)) if save_y else x.new_empty((0,))
    stat = lambda: x.new_empty((rows,), dtype=torch.float32)  # noqa: E731
    return y, stat(), stat(), stat(), x.new_empty((rows, parts * cols), dtype=torch.float8_e4m3fn)


def _layer_norm_quant_fake(x, weight, bias, eps, mean, rstd, BLOCK_D):
    stat = lambda: x.new_empty((x.shape[0],), dtype=torch.float32)  # noqa: E731
    return (torch.empty_like(x, memory_format=torch.contiguous_format), stat(), stat(), stat(),
            x.new_empty(x.shape, dtype=torch.float8_e4m3fn))


_LIBDEF.impl("b200_weighted_layer_norm_quantization_fwd", _layer_norm_quant_cuda, "CUDA")
torch.library.register_fake("recir::b200_weighted_layer_norm_quantization_fwd", _layer_norm_quant_fake)
_LIBDEF.impl("b200_weighted_layer_norm_fwd", _layer_norm_cuda, "CUDA")
_LIBDEF.impl("b200_layer_norm_mul_dropout_quantization_fwd", _layer_norm_mul_cuda, "CUDA")
torch.library.register_fake("recir::b200_weighted_layer_norm_fwd", _layer_norm_fake)
torch.library.register_fake("recir::b200_layer_norm_mul_dropout_quantization_fwd", _layer_norm_mul_fake)


def _addmm_cuda(x, w, y):
    """The u/v/q/k and output projections of an STU layer: ``y + x @ w``.  A plain GEMM, handed to the
    vendor library (``generative_recommenders::triton_addmm_fwd``,
    ``recir/ops/kjt_split_per_feature.cpp:246-262``, does the same with ``at::addmm``)."""
    if x.dim() != 2 or w.dim() != 2:
        raise ValueError("x and weight must be two-dimensional")
    if x.shape[1] != w.shape[0]:
        raise ValueError("x and weight dimensions are incompatible")
    if not ((y.dim() == 1 and y.shape[0] == w.shape[1]) or (y.dim() == 2 and y.shape[1] == w.shape[1])):
        raise ValueError("bias dimensions are incompatible with the output")
    return torch.addmm(y, x, w)


def _addmm_fake(x, w, y):
    return x.new_empty((x.shape[0], w.shape[1]))


_LIBDEF.impl("b200_addmm_fwd", _addmm_cuda, "CUDA")
torch.library.register_fake("recir::b200_addmm_fwd", _addmm_fake)


def _fp8_rowwise_addmm_cuda(a, b, a_scale, b_scale, bias, has_bias, bias_is_2d, dot_out_dtype, allow_tf32,
                            use_fast_accum):
    """The projection behind the quantised layer-norm stage: ``(a * a_scale[:, None]) @ (b * b_scale[:, None]).T
    + bias`` with ``a`` [M, K] and ``b`` [N, K] in float8 e4m3 and one float32 scale per row of each
    (``generative_recommenders::_triton_fp8_rowwise_addmm_fwd_impl``,
    ``recir/ops/kjt_split_per_feature.cpp:533-556``, which dequantises and calls ``at::mm``; it ignores
    ``bias_is_2d``, ``allow_tf32`` and ``use_fast_accum``, and so does this).  A plain GEMM, handed to the
    vendor library's fp8 path: the float8 products are exact and accumulate in float32, so only the
    summation order differs from the reference."""
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("a and b must be two-dimensional")
    if a.shape[1] != b.shape[1]:
        raise ValueError("a and b dimensions are incompatible")
    if a.dtype != torch.float8_e4m3fn or b.dtype != torch.float8_e4m3fn:
        raise ValueError("a and b must be float8_e4m3fn")
    if a_scale.numel() != a.shape[0] or b_scale.numel() != b.shape[0]:
        raise ValueError("one scale per row of a and of b is required")
    if a.shape[1] % 16 != 0 or b.shape[0] % 16 != 0:
        raise ValueError("the reduction and output dimensions must be multiples of 16")
    sa = a_scale.reshape(-1, 1).to(torch.float32).contiguous()
    sb = b_scale.reshape(1, -1).to(torch.float32).contiguous()
    # the library wants a row-major [M, K] and a column-major [K, N]: b.T of a contiguous [N, K] is that
    a, bt = a.contiguous(), b.contiguous().t()
    # Unscaled float32 sums from the library's fp8 GEMM, then row scale x column scale (+ bias) and the
    # final rounding in one element-wise pass, as the reference rounds once.  (The library's own
    # row-wise scaling writes 16-bit outputs only, and gave different values on small float16 cases.)
    one = torch.ones((), dtype=torch.float32, device=a.device)
    out = torch._scaled_mm(a, bt, scale_a=one, scale_b=one, out_dtype=torch.float32) * sa * sb
    if has_bias:
        out = out + bias.float()
    return out.to(dot_out_dtype)


def _fp8_rowwise_addmm_fake(a, b, a_scale, b_scale, bias, has_bias, bias_is_2d, dot_out_dtype, allow_tf32,
                            use_fast_accum):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=dot_out_dtype)


_LIBDEF.impl("b200_fp8_rowwise_addmm_fwd", _fp8_rowwise_addmm_cuda, "CUDA")
torch.library.register_fake("recir::b200_fp8_rowwise_addmm_fwd", _fp8_rowwise_addmm_fake)


def _jagged_dense_bmm_add_cuda(max_seq_len, seq_offsets, jagged, dense, bias, elementwise=False):
    """Rows of sequence ``b`` times that sequence's own matrix, plus a bias per sequence (or per row):
    ``out[rows of b] = jagged[rows of b] @ dense[b] + bias[b]``
    (``generative_recommenders::triton_jagged_dense_bmm_add_fwd``,
    ``recir/ops/kjt_split_per_feature.cpp:262-305``, which loops over the sequences with ``at::addmm``).
    One grouped GEMM of the vendor library over the jagged rows, no padding and no host read of the
    offsets; bfloat16 only (the library's grouped GEMM: float32 accumulation, bfloat16 product, then the bias
    is added in float32 and the sum rounded).  ``jagged.shape[0]`` must equal ``seq_offsets[-1]`` (not checked: that would need a
    host read); rows past it would be left unspecified by the library and are returned as zeros."""
    if jagged.dim() != 2:
        raise ValueError("jagged must be two-dimensional")
    if dense.dim() != 3:
        raise ValueError("dense must be three-dimensional")
    if seq_offsets.dim() != 1:
        raise ValueError("sequence offsets must be one-dimensional")
    B, K, N = dense.shape
    if K != jagged.shape[1]:
        raise ValueError("jagged and dense input dimensions are incompatible")
    if seq_offsets.numel() != B + 1:
        raise ValueError("sequence offsets size must match the dense batch size")
    if tuple(bias.shape) != ((jagged.shape[0], N) if elementwise else (B, N)):
        raise ValueError("bias dimensions are incompatible with the output")
    if jagged.dtype != torch.bfloat16 or dense.dtype != torch.bfloat16:
        raise ValueError(f"unsupported dtype {jagged.dtype}: the grouped GEMM takes bfloat16")
    T = jagged.shape[0]
    if T == 0 or B == 0:
        return jagged.new_zeros((T, N)), B, K, N
    ends = seq_offsets[1:].to(torch.int32)
    prod = torch.nn.functional.grouped_mm(jagged.contiguous(), dense.contiguous(), offs=ends).float()
    rows = torch.arange(T, device=jagged.device, dtype=ends.dtype)
    seq = torch.searchsorted(ends, rows, right=True)  # sequence of every row; B for rows past the last offset
    owned = (seq < B).unsqueeze(1)
    if elementwise:
        out = prod + bias.float()
    else:
        out = prod + bias.float()[seq.clamp(max=B - 1)]
    return torch.where(owned, out, torch.zeros((), device=out.device)).to(jagged.dtype), B, K, N



def _jagged_dense_bmm_add_fake(max_seq_len, seq_offsets, jagged, dense, bias, elementwise=False):
    return jagged.new_empty((jagged.shape[0], dense.shape[2])), dense.shape[0], dense.shape[1], dense.shape[2]


_LIBDEF.impl("b200_jagged_dense_bmm_add_fwd", _jagged_dense_bmm_add_cuda, "CUDA")
torch.library.register_fake("recir::b200_jagged_dense_bmm_add_fwd", _jagged_dense_bmm_add_fake)
