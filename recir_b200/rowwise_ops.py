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

``recir::b200_weighted_layer_norm_fwd`` is differentiable: ``recir::b200_weighted_layer_norm_bwd`` is the
closed form of what autograd gives through the reference's composite (the reference has no backward
operator of its own).  The gate stage is differentiable through its saved output in the same way
(``recir::b200_layer_norm_mul_dropout_quantization_bwd``), and ``recir::b200_layer_norm_addmm_fwd`` through a
composed backward.  The fp8 variants and the plain projections are forward only.
``recir::b200_layer_norm_addmm_fwd`` fuses the layer norm into the projection behind it (one tcgen05
kernel, ``csrc/stu_gemm.cu``).  CUDA tensors only; there is no CPU implementation.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from . import ops as _ops
from .ops import _check, _DTYPES

_LIBDEF = torch.library.Library("recir", "FRAGMENT")
_LIBDEF.define(
    "b200_weighted_layer_norm_fwd(Tensor x, Tensor? weight, Tensor? bias, float eps, Tensor? mean=None, "
    "Tensor? rstd=None, bool is_swish=False) -> (Tensor, Tensor, Tensor)")
_LIBDEF.define(
    "b200_layer_norm_mul_dropout_quantization_fwd(Tensor x, Tensor u, Tensor weight, Tensor bias, float eps, "
    "float dropout_ratio, bool training, bool silu_u, bool concat_u, bool concat_x, str mul_u_activation_type, "
    "int seed, bool save_y, int BLOCK_D) -> (Tensor, Tensor, Tensor, Tensor, Tensor)")

_LIBDEF.define(
    "b200_weighted_layer_norm_bwd(Tensor dy, Tensor x, Tensor? weight, Tensor? bias, Tensor mean, Tensor rstd, "
    "bool is_swish=False) -> (Tensor, Tensor, Tensor)")
_LIBDEF.define(
    "b200_layer_norm_mul_dropout_quantization_bwd(Tensor dout, Tensor x, Tensor u, Tensor weight, Tensor bias, "
    "Tensor mean, Tensor rstd, bool silu_u, bool concat_u, bool concat_x, str mul_u_activation_type) "
    "-> (Tensor, Tensor, Tensor, Tensor)")
_LIBDEF.define("b200_addmm_fwd(Tensor x, Tensor w, Tensor y) -> Tensor")
_LIBDEF.define(
    "b200_layer_norm_addmm_fwd(Tensor x, Tensor? ln_weight, Tensor? ln_bias, float eps, bool is_swish, Tensor w, "
    "Tensor bias) -> (Tensor, Tensor, Tensor)")
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
def _layer_norm_bwd_cuda(dy, x, weight, bias, mean, rstd, is_swish=False):
    """Gradients of ``b200_weighted_layer_norm_fwd`` (statistics computed from ``x``) with respect to x, weight
    and bias: the closed form of what autograd gives through the reference's composite
    (``recir/ops/kjt_split_per_feature.cpp:197-244``).  Returns ``(dx, dweight, dbias)``; the last two are empty
    tensors when there is no weight.  Feature dimension: a multiple of 8, at most 1024."""
    global launch_counter
    _validate(x, weight, bias)
    if dy.shape != x.shape or dy.dtype != x.dtype:
        raise ValueError("dy must have the shape and dtype of x")
    if is_swish and weight is None:
        raise ValueError("is_swish requires learnable layer normalization")
    if mean.numel() != x.shape[0] or rstd.numel() != x.shape[0]:
        raise ValueError("mean and rstd must match the row count")
    if x.shape[1] > 1024:
        raise ValueError("the layer-norm backward serves feature dimensions up to 1024")
    x, dy = _rows2d(x), _rows2d(dy)
    dx = torch.empty_like(x, memory_format=torch.contiguous_format)
    cols = x.shape[1]
    dw = torch.empty(cols if weight is not None else 0, dtype=x.dtype, device=x.device)
    db = torch.empty_like(dw)
    lib = _lib.load()
    p = _lib.B200LayerNormBwdParams()
    p.struct_size = ctypes.sizeof(p)
    p.flags = _lib.ROWWISE_SWISH if is_swish else 0
    p.dtype = _DTYPES[x.dtype]
    p.rows, p.cols = x.shape
    p.dy, p.x, p.dx = dy.data_ptr(), x.data_ptr(), dx.data_ptr()
    p.dy_row_stride, p.x_row_stride, p.dx_row_stride = dy.stride(0), x.stride(0), dx.stride(0)
    keep = [mean.to(torch.float32).contiguous(), rstd.to(torch.float32).contiguous()]
    p.mean, p.rstd = keep[0].data_ptr(), keep[1].data_ptr()
    if weight is not None:
        w, b = weight.to(x.dtype).contiguous(), bias.to(x.dtype).contiguous()
        keep += [w, b]
        p.weight, p.bias, p.dweight, p.dbias = w.data_ptr(), b.data_ptr(), dw.data_ptr(), db.data_ptr()
        need = lib.b200_stu_layer_norm_bwd_workspace_bytes(x.shape[0], cols)
        if need:
            ws = torch.empty(need // 4, dtype=torch.float32, device=x.device)
            keep.append(ws)
            p.workspace, p.workspace_bytes = ws.data_ptr(), need
    with torch.cuda.device(x.device):
        rc = lib.b200_stu_layer_norm_bwd(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_layer_norm_bwd")
    launch_counter += 2 if (weight is not None and x.shape[0] > 0) else 1
    del keep
    return dx, dw, db


def _layer_norm_bwd_fake(dy, x, weight, bias, mean, rstd, is_swish=False):
    n = x.shape[1] if weight is not None else 0
    return torch.empty_like(x), x.new_empty((n,)), x.new_empty((n,))


def _layer_norm_setup_context(ctx, inputs, output) -> None:
    x, weight, bias, eps, mean_in, rstd_in, is_swish = inputs
    _y, mean, rstd = output
    ctx.save_for_backward(x, weight, bias, mean, rstd)
    ctx.is_swish = is_swish
    ctx.stats_given = mean_in is not None and rstd_in is not None


def _layer_norm_backward(ctx, dy, _dmean, _drstd):
    x, weight, bias, mean, rstd = ctx.saved_tensors
    if ctx.stats_given:
        raise RuntimeError("b200_weighted_layer_norm_fwd: backward with caller-provided statistics is not built")
    dx, dw, db = torch.ops.recir.b200_weighted_layer_norm_bwd(dy.contiguous(), x, weight, bias, mean, rstd, ctx.is_swish)
    has_w = weight is not None
    return dx, (dw if has_w else None), (db if has_w else None), None, None, None, None


def _layer_norm_mul_bwd_cuda(dout, x, u, weight, bias, mean, rstd, silu_u, concat_u, concat_x, mul_u_activation_type):
    """Gradients of the saved output of ``b200_layer_norm_mul_dropout_quantization_fwd`` with respect to x, u,
    weight and bias: the closed form of what autograd gives through the reference's composite
    (``recir/ops/kjt_split_per_feature.cpp:558-600``; the fp8 copy and its scale carry no gradient, and like the
    forward no dropout is applied).  ``dout`` is ``[rows, parts * cols]`` in the forward's part order.  Returns
    ``(dx, du, dweight, dbias)``.  Feature dimension: a multiple of 8, at most 1024."""
    global launch_counter
    _validate(x, weight, bias)
    if u.shape != x.shape or u.dtype != x.dtype:
        raise ValueError("u must have the shape and dtype of x")
    flags = _mul_flags(silu_u, concat_u, concat_x, mul_u_activation_type)
    parts = 1 + int(bool(concat_u)) + int(bool(concat_x))
    x, u, dout = _rows2d(x), _rows2d(u), _rows2d(dout)
    rows, cols = x.shape
    if dout.shape != (rows, parts * cols) or dout.dtype != x.dtype:
        raise ValueError("dout must be [rows, parts * cols] in the dtype of x")
    if mean.numel() != rows or rstd.numel() != rows:
        raise ValueError("mean and rstd must match the row count")
    if cols > 1024:
        raise ValueError("the gate-stage backward serves feature dimensions up to 1024")
    dx = torch.empty_like(x, memory_format=torch.contiguous_format)
    du = torch.empty_like(x, memory_format=torch.contiguous_format)
    dw = torch.empty(cols, dtype=x.dtype, device=x.device)
    db = torch.empty_like(dw)
    lib = _lib.load()
    p = _lib.B200LayerNormMulBwdParams()
    p.struct_size = ctypes.sizeof(p)
    p.flags = flags
    p.dtype = _DTYPES[x.dtype]
    p.rows, p.cols = rows, cols
    p.dout, p.x, p.u, p.dx, p.du = dout.data_ptr(), x.data_ptr(), u.data_ptr(), dx.data_ptr(), du.data_ptr()
    p.dout_row_stride, p.x_row_stride, p.u_row_stride = dout.stride(0), x.stride(0), u.stride(0)
    p.dx_row_stride, p.du_row_stride = dx.stride(0), du.stride(0)
    keep = [mean.to(torch.float32).contiguous(), rstd.to(torch.float32).contiguous(),
            weight.to(x.dtype).contiguous(), bias.to(x.dtype).contiguous()]
    p.mean, p.rstd, p.weight, p.bias = (t.data_ptr() for t in keep)
    p.dweight, p.dbias = dw.data_ptr(), db.data_ptr()
    need = lib.b200_stu_layer_norm_bwd_workspace_bytes(rows, cols)
    if need:
        ws = torch.empty(need // 4, dtype=torch.float32, device=x.device)
        keep.append(ws)
        p.workspace, p.workspace_bytes = ws.data_ptr(), need
    with torch.cuda.device(x.device):
        rc = lib.b200_stu_layer_norm_mul_bwd(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_layer_norm_mul_bwd")
    launch_counter += 2 if rows > 0 else 0
    del keep
    return dx, du, dw, db


def _layer_norm_mul_bwd_fake(dout, x, u, weight, bias, mean, rstd, silu_u, concat_u, concat_x, mul_u_activation_type):
    return torch.empty_like(x), torch.empty_like(x), x.new_empty((x.shape[1],)), x.new_empty((x.shape[1],))


def _layer_norm_mul_setup_context(ctx, inputs, output) -> None:
    (x, u, weight, bias, _eps, _dropout_ratio, _training, silu_u, concat_u, concat_x, act, _seed, save_y, _block) = inputs
    _y, mean, rstd, _scale, _q8 = output
    ctx.save_for_backward(x, u, weight, bias, mean, rstd)
    ctx.cfg = (silu_u, concat_u, concat_x, act)
    ctx.save_y = save_y


def _layer_norm_mul_backward(ctx, dy, _dmean, _drstd, _dscale, _dq8):
    x, u, weight, bias, mean, rstd = ctx.saved_tensors
    if not ctx.save_y:
        raise RuntimeError("b200_layer_norm_mul_dropout_quantization_fwd: only the saved output (save_y=True) is "
                           "differentiable; the fp8 copy carries no gradient")
    silu_u, concat_u, concat_x, act = ctx.cfg
    dx, du, dw, db = torch.ops.recir.b200_layer_norm_mul_dropout_quantization_bwd(
        dy.contiguous(), x, u, weight, bias, mean, rstd, silu_u, concat_u, concat_x, act)
    return (dx, du, dw, db) + (None,) * 10


_LIBDEF.impl("b200_weighted_layer_norm_fwd", _layer_norm_cuda, "CUDA")
_LIBDEF.impl("b200_weighted_layer_norm_bwd", _layer_norm_bwd_cuda, "CUDA")
_LIBDEF.impl("b200_layer_norm_mul_dropout_quantization_bwd", _layer_norm_mul_bwd_cuda, "CUDA")
torch.library.register_fake("recir::b200_layer_norm_mul_dropout_quantization_bwd", _layer_norm_mul_bwd_fake)
torch.library.register_fake("recir::b200_weighted_layer_norm_bwd", _layer_norm_bwd_fake)
torch.library.register_autograd("recir::b200_weighted_layer_norm_fwd", _layer_norm_backward,
                                setup_context=_layer_norm_setup_context)
_LIBDEF.impl("b200_layer_norm_mul_dropout_quantization_fwd", _layer_norm_mul_cuda, "CUDA")
torch.library.register_autograd("recir::b200_layer_norm_mul_dropout_quantization_fwd", _layer_norm_mul_backward,
                                setup_context=_layer_norm_mul_setup_context)
torch.library.register_fake("recir::b200_weighted_layer_norm_fwd", _layer_norm_fake)
torch.library.register_fake("recir::b200_layer_norm_mul_dropout_quantization_fwd", _layer_norm_mul_fake)


def _gemm_params(x, w, bias, out):
    p = _lib.B200GemmParams()
    p.struct_size = ctypes.sizeof(p)
    p.dtype = _DTYPES.get(x.dtype, -1)
    p.M, p.K, p.N = x.shape[0], x.shape[1], w.shape[1]
    p.x, p.w, p.bias, p.out = x.data_ptr(), w.data_ptr(), bias.data_ptr(), out.data_ptr()
    p.x_row_stride, p.w_row_stride, p.out_row_stride = x.stride(0), w.stride(0), out.stride(0)
    p.bias_row_stride = bias.stride(0) if (bias.dim() == 2 and bias.shape[0] != 1) else 0
    return p


def _tc_gemm_serves(x, w) -> bool:
    """bfloat16 / float16, K a multiple of 64 up to 512, N a multiple of 8: the sizes of an STU layer's
    projections (embedding width 512 into u | v | q | k, and back)."""
    return (x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype and x.shape[0] > 0
            and x.shape[1] % 64 == 0 and 0 < x.shape[1] <= 512 and w.shape[1] % 8 == 0 and w.shape[1] > 0)


def _addmm_cuda(x, w, y):
    """The u/v/q/k and output projections of an STU layer: ``y + x @ w``
    (``generative_recommenders::triton_addmm_fwd``, ``recir/ops/kjt_split_per_feature.cpp:246-262``:
    ``at::addmm(bias, x, w)``).  The 16-bit shapes of an STU layer (see ``_tc_gemm_serves``) run on this
    library's tcgen05 kernel (``csrc/stu_gemm.cu``); any other dtype or size is a plain GEMM handed to
    the vendor library."""
    global launch_counter
    if x.dim() != 2 or w.dim() != 2:
        raise ValueError("x and weight must be two-dimensional")
    if x.shape[1] != w.shape[0]:
        raise ValueError("x and weight dimensions are incompatible")
    if not ((y.dim() == 1 and y.shape[0] == w.shape[1]) or (y.dim() == 2 and y.shape[1] == w.shape[1])):
        raise ValueError("bias dimensions are incompatible with the output")
    if not _tc_gemm_serves(x, w) or y.dtype != x.dtype or (y.dim() == 2 and y.shape[0] not in (1, x.shape[0])):
        return torch.addmm(y, x, w)
    x, w, y = _rows2d(x), _rows2d(w), (y if y.dim() == 1 else _rows2d(y))
    if y.data_ptr() % 16 != 0:
        y = y.clone()
    out = torch.empty((x.shape[0], w.shape[1]), dtype=x.dtype, device=x.device)
    p = _gemm_params(x, w, y, out)
    p.status = _ops.status_tensor(x.device).data_ptr()
    with torch.cuda.device(x.device):
        rc = _lib.load().b200_stu_addmm(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_addmm")
    launch_counter += 1
    return out


# The fused layer norm + projection kernel pays off from about this many multiply-adds per row (K * N): at
# K = 512 an output width of 1536 (the u | v | q | k projection of an STU layer is 2048 wide).
FUSED_PROJECTION_MIN_KN = 512 * 1536


def _layer_norm_addmm_cuda(x, ln_weight, ln_bias, eps, is_swish, w, bias):
    """``addmm(bias, weighted_layer_norm(x, ln_weight, ln_bias, eps, is_swish)[0], w)`` in one kernel: the
    layer norm is the prologue of the product's A operand, so the normalised activations never travel
    through HBM (``recir/ops/kjt_split_per_feature.cpp:197-262``).  Returns ``(out, mean, rstd)``; ``out``
    is ``[rows, N]`` and can be consumed as column slices (u | v | q | k) without a copy."""
    global launch_counter
    _validate(x, ln_weight, ln_bias)
    if is_swish and ln_weight is None:
        raise ValueError("is_swish requires learnable layer normalization")
    if w.dim() != 2 or x.shape[1] != w.shape[0]:
        raise ValueError("x and weight dimensions are incompatible")
    if not ((bias.dim() == 1 and bias.shape[0] == w.shape[1]) or (bias.dim() == 2 and bias.shape[1] == w.shape[1])):
        raise ValueError("bias dimensions are incompatible with the output")
    if not _tc_gemm_serves(x, w) or bias.dtype != x.dtype:
        raise ValueError("b200_layer_norm_addmm_fwd serves bfloat16 / float16 with a feature dimension that is a multiple "
                         "of 64 and at most 512, and an output width that is a multiple of 8")
    x, w = _rows2d(x), _rows2d(w)
    if x.shape[1] * w.shape[1] < FUSED_PROJECTION_MIN_KN:
        # Too little product per row for the two layer-norm warps of the fused kernel to keep up with its
        # tensor pipe: the layer-norm kernel (every warp of the GPU on it, at HBM speed) and then the
        # projection kernel are faster, and give the same bits (both round the normalised rows to the
        # input dtype before the product).
        y, mean, rstd = torch.ops.recir.b200_weighted_layer_norm_fwd(x, ln_weight, ln_bias, eps, None, None, is_swish)
        return _addmm_cuda(y, w, bias), mean, rstd
    bias = bias if bias.dim() == 1 else _rows2d(bias)
    if bias.data_ptr() % 16 != 0:
        bias = bias.clone()
    out = torch.empty((x.shape[0], w.shape[1]), dtype=x.dtype, device=x.device)
    mean = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    p = _gemm_params(x, w, bias, out)
    p.flags = _lib.GEMM_LAYER_NORM | (_lib.GEMM_SWISH if is_swish else 0)
    p.eps = float(eps)
    keep = []
    if ln_weight is not None:
        lw, lb = ln_weight.to(x.dtype).contiguous(), ln_bias.to(x.dtype).contiguous()
        keep += [lw, lb]
        p.ln_weight, p.ln_bias = lw.data_ptr(), lb.data_ptr()
    p.mean, p.rstd = mean.data_ptr(), rstd.data_ptr()
    p.status = _ops.status_tensor(x.device).data_ptr()
    with torch.cuda.device(x.device):
        rc = _lib.load().b200_stu_addmm(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_addmm")
    launch_counter += 1
    del keep
    return out, mean, rstd


def _layer_norm_addmm_fake(x, ln_weight, ln_bias, eps, is_swish, w, bias):
    rows = x.shape[0]
    return (x.new_empty((rows, w.shape[1])), x.new_empty((rows,), dtype=torch.float32),
            x.new_empty((rows,), dtype=torch.float32))


def _addmm_fake(x, w, y):
    return x.new_empty((x.shape[0], w.shape[1]))


_LIBDEF.impl("b200_addmm_fwd", _addmm_cuda, "CUDA")
torch.library.register_fake("recir::b200_addmm_fwd", _addmm_fake)
def _layer_norm_addmm_setup_context(ctx, inputs, output) -> None:
    x, ln_weight, ln_bias, eps, is_swish, w, bias = inputs
    _out, mean, rstd = output
    ctx.save_for_backward(x, ln_weight, ln_bias, w, mean, rstd)
    ctx.eps, ctx.is_swish, ctx.bias_shape = eps, is_swish, tuple(bias.shape)


def _layer_norm_addmm_backward(ctx, dout, _dmean, _drstd):
    """Backward of the fused op, composed: the normalised rows are recomputed by the layer-norm kernel from the
    saved statistics (they were never stored), the two products of the projection's backward are plain GEMMs
    (vendor library), and the layer norm's own backward is this library's kernel."""
    x, ln_weight, ln_bias, w, mean, rstd = ctx.saved_tensors
    dout = dout.contiguous()
    a = torch.ops.recir.b200_weighted_layer_norm_fwd(x, ln_weight, ln_bias, ctx.eps, mean, rstd, ctx.is_swish)[0]
    da = dout @ w.t()
    dw = a.t() @ dout
    dbias = dout if len(ctx.bias_shape) == 2 and ctx.bias_shape[0] == x.shape[0] else \
        dout.float().sum(0).to(dout.dtype).reshape(ctx.bias_shape)
    dx, dlw, dlb = torch.ops.recir.b200_weighted_layer_norm_bwd(da, x, ln_weight, ln_bias, mean, rstd, ctx.is_swish)
    has_w = ln_weight is not None
    return dx, (dlw if has_w else None), (dlb if has_w else None), None, None, dw, dbias


_LIBDEF.impl("b200_layer_norm_addmm_fwd", _layer_norm_addmm_cuda, "CUDA")
torch.library.register_fake("recir::b200_layer_norm_addmm_fwd", _layer_norm_addmm_fake)
torch.library.register_autograd("recir::b200_layer_norm_addmm_fwd", _layer_norm_addmm_backward,
                                setup_context=_layer_norm_addmm_setup_context)


def _fp8_rowwise_addmm_tc(a, b, a_scale, b_scale, bias, out_dtype):
    """The tcgen05 route of ``_fp8_rowwise_addmm_cuda``; None when the sizes or types are not the kernel's."""
    global launch_counter
    if out_dtype != torch.bfloat16 or a.shape[0] == 0:
        return None
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != b.shape[0]):
        return None
    a, b = _rows2d(a), _rows2d(b)
    lib = _lib.load()
    p = _lib.B200Fp8GemmParams()
    p.struct_size = ctypes.sizeof(p)
    p.out_dtype = _DTYPES[torch.bfloat16]
    p.M, p.K, p.N = a.shape[0], a.shape[1], b.shape[0]
    p.a_row_stride, p.b_row_stride = a.stride(0), b.stride(0)
    if not lib.b200_stu_fp8_rowwise_addmm_supported(ctypes.byref(p)):
        return None
    if a.data_ptr() % 16 or b.data_ptr() % 16 or a.stride(0) % 16 or b.stride(0) % 16:
        return None
    out = torch.empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16, device=a.device)
    keep = [a_scale.reshape(-1).to(torch.float32).contiguous(), b_scale.reshape(-1).to(torch.float32).contiguous()]
    if bias is not None:
        keep.append(bias.to(torch.bfloat16).contiguous())
        p.bias = keep[-1].data_ptr()
    p.a, p.b, p.out = a.data_ptr(), b.data_ptr(), out.data_ptr()
    p.out_row_stride = out.stride(0)
    p.a_scale, p.b_scale = keep[0].data_ptr(), keep[1].data_ptr()
    p.status = _ops.status_tensor(a.device).data_ptr()
    with torch.cuda.device(a.device):
        rc = lib.b200_stu_fp8_rowwise_addmm(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_fp8_rowwise_addmm")
    launch_counter += 1
    del keep
    return out


def _fp8_rowwise_addmm_cuda(a, b, a_scale, b_scale, bias, has_bias, bias_is_2d, dot_out_dtype, allow_tf32,
                            use_fast_accum):
    """The projection behind the quantised layer-norm stage: ``(a * a_scale[:, None]) @ (b * b_scale[:, None]).T
    + bias`` with ``a`` [M, K] and ``b`` [N, K] in float8 e4m3 and one float32 scale per row of each
    (``generative_recommenders::_triton_fp8_rowwise_addmm_fwd_impl``,
    ``recir/ops/kjt_split_per_feature.cpp:533-556``, which dequantises and calls ``at::mm``; it ignores
    ``bias_is_2d``, ``allow_tf32`` and ``use_fast_accum``, and so does this).  The float8 products are exact and
    accumulate in float32, so only the summation order differs from the reference.  The STU sizes (K a
    multiple of 128 up to 1024, N a multiple of 8, bfloat16 output, a bias vector or none) run on this
    library's tcgen05 kernel (``csrc/stu_gemm.cu``, ``kind::f8f6f4`` on CTA pairs); any other size or output
    type is a plain GEMM handed to the vendor library's fp8 path."""
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("a and b must be two-dimensional")
    if a.shape[1] != b.shape[1]:
        raise ValueError("a and b dimensions are incompatible")
    if a.dtype != torch.float8_e4m3fn or b.dtype != torch.float8_e4m3fn:
        raise ValueError("a and b must be float8_e4m3fn")
    if a_scale.numel() != a.shape[0] or b_scale.numel() != b.shape[0]:
        raise ValueError("one scale per row of a and of b is required")
    out = _fp8_rowwise_addmm_tc(a, b, a_scale, b_scale, bias if has_bias else None, dot_out_dtype)
    if out is not None:
        return out
    if a.shape[1] % 16 != 0 or b.shape[0] % 16 != 0:
        raise ValueError("the reduction and output dimensions must be multiples of 16 (this library's kernel: K a "
                         "multiple of 128 up to 1024, N a multiple of 8, bfloat16 output)")
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
    bfloat16 / float16 with K a multiple of 64 up to 512 and N a multiple of 8 (the STU sizes) run on this
    library's tcgen05 projection kernel over a device-built list of (sequence, 128-row block) items; other
    bfloat16 sizes are one grouped GEMM of the vendor library (which rounds the product to bfloat16 before the
    bias is added).  No padding and no host read of the offsets either way.  Rows at or past
    ``seq_offsets[-1]`` are returned as zeros."""
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
    T = jagged.shape[0]
    if T == 0 or B == 0:
        return jagged.new_zeros((T, N)), B, K, N
    if (jagged.dtype in (torch.bfloat16, torch.float16) and dense.dtype == jagged.dtype and bias.dtype == jagged.dtype
            and K % 64 == 0 and K <= 512 and N % 8 == 0 and seq_offsets.dtype in (torch.int32, torch.int64)
            and B * K < 2 ** 31):
        return _jagged_dense_bmm_add_tc(seq_offsets, jagged, dense, bias, elementwise), B, K, N
    if jagged.dtype != torch.bfloat16 or dense.dtype != torch.bfloat16:
        raise ValueError(f"unsupported dtype {jagged.dtype}: float16 needs K a multiple of 64 up to 512 and N a multiple "
                         "of 8 (tensor-core kernel); other bfloat16 sizes go to the vendor library's grouped GEMM")
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


def _jagged_dense_bmm_add_tc(seq_offsets, jagged, dense, bias, elementwise):
    """This library's tcgen05 projection kernel over (sequence, 128-row block) items built on the device from
    the offsets: float32 sums, the bias added before the single rounding, as ``at::addmm`` does per sequence."""
    global launch_counter
    lib = _lib.load()
    x, w = _rows2d(jagged), dense.contiguous()
    bias = _rows2d(bias)
    off = seq_offsets.contiguous()
    T, K = x.shape
    B, _, N = w.shape
    out = torch.empty((T, N), dtype=x.dtype, device=x.device)
    p = _lib.B200GemmParams()
    p.struct_size = ctypes.sizeof(p)
    p.dtype = _DTYPES[x.dtype]
    p.M, p.K, p.N = T, K, N
    p.x, p.w, p.bias, p.out = x.data_ptr(), w.data_ptr(), bias.data_ptr(), out.data_ptr()
    p.x_row_stride, p.w_row_stride, p.out_row_stride = x.stride(0), w.stride(1), out.stride(0)
    p.bias_row_stride = bias.stride(0)
    p.status = _ops.status_tensor(x.device).data_ptr()
    need = lib.b200_stu_jagged_bmm_workspace_bytes(T, B)
    ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib.b200_stu_jagged_dense_bmm_add(ctypes.byref(p), off.data_ptr(), int(off.dtype == torch.int64), B, w.stride(0),
                                               int(bool(elementwise)), ws.data_ptr(), need,
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_jagged_dense_bmm_add")
    launch_counter += 2
    return out


def _jagged_dense_bmm_add_fake(max_seq_len, seq_offsets, jagged, dense, bias, elementwise=False):
    return jagged.new_empty((jagged.shape[0], dense.shape[2])), dense.shape[0], dense.shape[1], dense.shape[2]


_LIBDEF.impl("b200_jagged_dense_bmm_add_fwd", _jagged_dense_bmm_add_cuda, "CUDA")
torch.library.register_fake("recir::b200_jagged_dense_bmm_add_fwd", _jagged_dense_bmm_add_fake)
