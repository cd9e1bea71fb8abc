"""``torch.library`` operators for jagged <-> dense marshalling and jagged concat / split.

Same schemas as the reference's ``recir::jagged_to_padded_dense``, ``recir::dense_to_jagged``,
``recir::concat_2d_jagged`` and ``recir::split_2d_jagged`` (``recir/ops/jagged_ops.py:115-128``),
registered as ``recir::b200_*`` so that a node can be retargeted positionally
(``recir/lowering/op_swap.py:78-97``).  Like there, the ops of a pair are each other's backward
(``recir/ops/jagged_ops.py:16-18``).  One CUDA row-gather kernel serves all of them; only CUDA
tensors are accepted.  Every index rule of the reference is kept, including the fully-padded
fast paths that merely reshape (``:41-45``, ``:87-90``) and the early returns for an empty side
(``:229-232``).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch

from . import _lib
from .ops import _check

_LIBDEF = torch.library.Library("recir", "FRAGMENT")
_LIBDEF.define("b200_dense_to_jagged(Tensor dense, Tensor[] offsets, int? total_L=None) -> (Tensor, Tensor)")
_LIBDEF.define("b200_jagged_to_padded_dense(Tensor values, Tensor[] offsets, int[] max_lengths, float padding_value=0) -> Tensor")
_LIBDEF.define("b200_concat_2d_jagged(Tensor values_left, Tensor offsets_left, Tensor values_right, Tensor offsets_right) -> Tensor")
_LIBDEF.define("b200_split_2d_jagged(Tensor values, Tensor offsets_left, Tensor offsets_right, SymInt seq_len_a, SymInt seq_len_b) -> (Tensor, Tensor)")

_LIBDEF.define(
    "b200_concat_2D_jagged_fwd_op(int max_seq_len, Tensor values_a, Tensor values_b, Tensor? offsets_a, "
    "Tensor? offsets_b, bool is_replace, int n_prefix_from_right) -> Tensor")
_LIBDEF.define(
    "b200_split_2D_jagged_fwd_op(Tensor values, int max_seq_len, Tensor offsets_a, Tensor offsets_b, int seq_len_a, "
    "int seq_len_b, bool is_dense_a, bool is_dense_b, int dense_size, int n_prefix_to_right, int B) -> (Tensor, Tensor)")

launch_counter = 0


def _rows(t: torch.Tensor) -> torch.Tensor:
    """[rows, ...] with contiguous rows; a row stride larger than the row is passed through."""
    if t.dim() == 1:
        return t.contiguous()
    inner_ok = all(t.stride(i) == (t.stride(i + 1) * t.shape[i + 1]) for i in range(1, t.dim() - 1)) and t.stride(-1) == 1
    return t if inner_ok and t.stride(0) >= max(1, t[0].numel()) else t.contiguous()


def _offsets(*offs):
    dt = torch.int64 if any(o.dtype == torch.int64 for o in offs) else torch.int32
    for o in offs:
        if o.dtype not in (torch.int32, torch.int64) or o.dim() != 1:
            raise ValueError("offsets must be one-dimensional int32 or int64 tensors")
    return [o.to(dt).contiguous() for o in offs], (_lib.JAGGED_OFFSETS_I64 if dt == torch.int64 else 0)


def _launch(mode, dst, src0, src1, off0, off1, num_seqs, padded_len=0, pad=None):
    global launch_counter
    if dst.shape[0] == 0:
        return
    esz = dst.element_size()
    row_elems = dst[0].numel() if dst.dim() > 1 else 1
    if (row_elems * esz) % 2 != 0:
        raise ValueError("rows must hold an even number of bytes")
    offs, flags = _offsets(*(o for o in (off0, off1) if o is not None))
    p = _lib.B200JaggedParams()
    p.struct_size = ctypes.sizeof(p)
    p.flags, p.mode = flags, mode
    p.num_seqs, p.padded_len, p.dst_rows = num_seqs, padded_len, dst.shape[0]
    p.row_bytes = row_elems * esz
    stride = lambda t: (t.stride(0) if t.dim() > 1 else 1) * esz  # noqa: E731
    p.dst, p.dst_row_stride = dst.data_ptr(), stride(dst)
    if src0 is not None:
        p.src0, p.src0_rows, p.src0_row_stride = src0.data_ptr(), src0.shape[0], stride(src0)
    if src1 is not None:
        p.src1, p.src1_rows, p.src1_row_stride = src1.data_ptr(), src1.shape[0], stride(src1)
    p.offsets0 = offs[0].data_ptr()
    if len(offs) > 1:
        p.offsets1 = offs[1].data_ptr()
    if pad is not None:
        raw = pad.view(torch.uint8).cpu().numpy().tobytes()
        raw = (raw * (16 // len(raw)))[:16]
        ctypes.memmove(p.pad, raw, 16)
    with torch.cuda.device(dst.device):
        rc = _lib.load().b200_stu_jagged_copy(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _check(rc, "b200_stu_jagged_copy")
    launch_counter += 1


def _j2d_cuda(values, offsets: List[torch.Tensor], max_lengths: List[int], padding_value: float = 0.0):
    seq_offsets, n = offsets[0], int(max_lengths[0])
    b = seq_offsets.shape[0] - 1
    if values.shape[0] == b * n:  # fully padded: a reshape (recir/ops/jagged_ops.py:41-45)
        return values.reshape(b, n, *values.shape[1:])
    values = _rows(values)
    out = torch.empty((b * n, *values.shape[1:]), dtype=values.dtype, device=values.device)
    pad = torch.full((1,), padding_value, dtype=values.dtype)
    _launch(_lib.JAGGED_TO_PADDED_DENSE, out, values, None, seq_offsets, None, b, n, pad)
    return out.reshape(b, n, *values.shape[1:])


def _d2j_cuda(dense, offsets: List[torch.Tensor], total_L: Optional[int] = None):
    seq_offsets = offsets[0]
    b, n = dense.shape[0], dense.shape[1]
    if total_L is None:
        total_L = int(seq_offsets[-1].item())
    if total_L == 0:
        return torch.zeros((0, *dense.shape[2:]), dtype=dense.dtype, device=dense.device), seq_offsets
    if total_L == b * n:  # fully padded: a reshape (recir/ops/jagged_ops.py:87-90)
        return dense.reshape(total_L, *dense.shape[2:]), seq_offsets
    flat = dense.contiguous().reshape(b * n, *dense.shape[2:])
    out = torch.empty((total_L, *dense.shape[2:]), dtype=dense.dtype, device=dense.device)
    _launch(_lib.DENSE_TO_JAGGED, out, flat, None, seq_offsets, None, b, n)
    return out, seq_offsets


def _concat_cuda(values_left, offsets_left, values_right, offsets_right):
    if values_left.shape[0] == 0:
        return values_right
    if values_right.shape[0] == 0:
        return values_left
    left, right = _rows(values_left), _rows(values_right)
    out = torch.empty((left.shape[0] + right.shape[0], *left.shape[1:]), dtype=left.dtype, device=left.device)
    _launch(_lib.JAGGED_CONCAT, out, left, right, offsets_left, offsets_right, offsets_left.shape[0] - 1)
    return out


def _split_cuda(values, offsets_left, offsets_right, seq_len_a, seq_len_b):
    values = _rows(values)
    n = offsets_left.shape[0] - 1
    left = torch.empty((int(seq_len_a), *values.shape[1:]), dtype=values.dtype, device=values.device)
    right = torch.empty((int(seq_len_b), *values.shape[1:]), dtype=values.dtype, device=values.device)
    _launch(_lib.JAGGED_SPLIT_LEFT, left, values, None, offsets_left, offsets_right, n)
    _launch(_lib.JAGGED_SPLIT_RIGHT, right, values, None, offsets_left, offsets_right, n)
    return left, right


def _uniform(batch: int, length: int, like: torch.Tensor) -> torch.Tensor:
    return torch.arange(batch + 1, device=like.device, dtype=torch.int64) * int(length)


def _gr_concat_cuda(max_seq_len, values_a, values_b, offsets_a, offsets_b, is_replace, n_prefix_from_right):
    """``generative_recommenders::concat_2D_jagged_fwd_op`` (``recir/ops/kjt_split_per_feature.cpp:100-196``):
    per sequence ``[b[:p], a, b[p:]]`` (``p = n_prefix_from_right``), or with ``is_replace`` the rows of
    ``a`` with its last ``len(b)`` rows replaced by ``b``.  A side without offsets is dense ``[B, L, D]``, i.e.
    jagged with uniform offsets.  Composed from the row-gather kernel's concat / split passes (one pass
    for the plain form, two for the replace form, four with a prefix); like every operator here it reads
    no offset on the host, so the per-sequence length checks of the reference (``:170-183``) are not made."""
    if offsets_a is None and offsets_b is None:
        raise ValueError("at least one input must be jagged")
    p = int(n_prefix_from_right)
    if p < 0:
        raise ValueError(f"n_prefix_from_right must be non-negative, got {p}")
    if is_replace and p != 0:
        raise ValueError("n_prefix_from_right is not supported when is_replace is true")
    if p != 0 and (offsets_a is None or offsets_b is None):
        raise ValueError("n_prefix_from_right is only supported for two jagged inputs")
    if values_a.dtype != values_b.dtype:
        raise ValueError("values_a and values_b must have the same dtype")
    if values_a.shape[-1] != values_b.shape[-1]:
        raise ValueError("values_a and values_b must have the same embedding dimension")
    if offsets_a is None:
        if values_a.dim() != 3:
            raise ValueError("dense values_a must be three-dimensional")
        if offsets_b.numel() != values_a.shape[0] + 1:
            raise ValueError("offsets_b size must match the dense batch size")
        offsets_a = _uniform(values_a.shape[0], values_a.shape[1], values_a)
    elif offsets_b is None:
        if values_b.dim() != 3:
            raise ValueError("dense values_b must be three-dimensional")
        if offsets_a.numel() != values_b.shape[0] + 1:
            raise ValueError("offsets_a size must match the dense batch size")
        offsets_b = _uniform(values_b.shape[0], values_b.shape[1], values_b)
    elif offsets_a.numel() != offsets_b.numel():
        raise ValueError("offsets_a and offsets_b must have the same size")
    (oa, ob), _ = _offsets(offsets_a, offsets_b)
    batch = oa.shape[0] - 1
    fa = values_a.reshape(-1, values_a.shape[-1])
    fb = values_b.reshape(-1, values_b.shape[-1])
    if is_replace:
        keep = oa - ob  # rows of a that survive, as offsets
        head, _tail = _split_cuda(fa, keep, ob, fa.shape[0] - fb.shape[0], fb.shape[0])
        flat = _concat_cuda(head, keep, fb, ob)
        return flat.reshape(values_a.shape) if values_a.dim() == 3 else flat
    if p == 0:
        return _concat_cuda(fa, oa, fb, ob)
    op = _uniform(batch, p, fa).to(oa.dtype)
    front, rest = _split_cuda(fb, op, ob - op, batch * p, fb.shape[0] - batch * p)
    return _concat_cuda(_concat_cuda(front, op, fa, oa), op + oa, rest, ob - op)


def _gr_split_cuda(values, max_seq_len, offsets_a, offsets_b, seq_len_a, seq_len_b, is_dense_a, is_dense_b,
                   dense_size, n_prefix_to_right, B):
    """``generative_recommenders::split_2D_jagged_fwd_op`` (``recir/ops/kjt_split_per_feature.cpp:430-489``),
    the inverse of the concatenation above; a dense side has ``dense_size`` rows per sequence and comes
    back as ``[B, dense_size, D]``."""
    if values.dim() != 2:
        raise ValueError("values must be two-dimensional")
    batch, p = int(B), int(n_prefix_to_right)
    oa = _uniform(batch, dense_size, values) if is_dense_a else offsets_a
    ob = _uniform(batch, dense_size, values) if is_dense_b else offsets_b
    (oa, ob), _ = _offsets(oa, ob)
    rows_a = batch * int(dense_size) if is_dense_a else int(seq_len_a)
    rows_b = batch * int(dense_size) if is_dense_b else int(seq_len_b)
    if rows_a + rows_b != values.shape[0]:
        raise ValueError("split lengths do not match values")
    if p == 0:
        a, b = _split_cuda(values, oa, ob, rows_a, rows_b)
    else:
        op = _uniform(batch, p, values).to(oa.dtype)
        front_a, rest = _split_cuda(values, op + oa, ob - op, batch * p + rows_a, rows_b - batch * p)
        front, a = _split_cuda(front_a, op, oa, batch * p, rows_a)
        b = _concat_cuda(front, op, rest, ob - op)
    if is_dense_a:
        a = a.reshape(batch, int(dense_size), values.shape[1])
    if is_dense_b:
        b = b.reshape(batch, int(dense_size), values.shape[1])
    return a, b


_LIBDEF.impl("b200_concat_2D_jagged_fwd_op", _gr_concat_cuda, "CUDA")
_LIBDEF.impl("b200_split_2D_jagged_fwd_op", _gr_split_cuda, "CUDA")


@torch.library.register_fake("recir::b200_concat_2D_jagged_fwd_op")
def _(max_seq_len, values_a, values_b, offsets_a, offsets_b, is_replace, n_prefix_from_right):
    d = values_a.shape[-1]
    if is_replace:
        return values_a.new_empty(values_a.shape)
    rows = values_a.reshape(-1, d).shape[0] + values_b.reshape(-1, d).shape[0]
    return values_a.new_empty((rows, d))


@torch.library.register_fake("recir::b200_split_2D_jagged_fwd_op")
def _(values, max_seq_len, offsets_a, offsets_b, seq_len_a, seq_len_b, is_dense_a, is_dense_b, dense_size,
      n_prefix_to_right, B):
    d = values.shape[1]
    a = values.new_empty((B, dense_size, d) if is_dense_a else (seq_len_a, d))
    b = values.new_empty((B, dense_size, d) if is_dense_b else (seq_len_b, d))
    return a, b


_LIBDEF.impl("b200_jagged_to_padded_dense", _j2d_cuda, "CUDA")
_LIBDEF.impl("b200_dense_to_jagged", _d2j_cuda, "CUDA")
_LIBDEF.impl("b200_concat_2d_jagged", _concat_cuda, "CUDA")
_LIBDEF.impl("b200_split_2d_jagged", _split_cuda, "CUDA")


@torch.library.register_fake("recir::b200_jagged_to_padded_dense")
def _(values, offsets, max_lengths, padding_value=0.0):
    return values.new_empty((offsets[0].shape[0] - 1, max_lengths[0], *values.shape[1:]))


@torch.library.register_fake("recir::b200_dense_to_jagged")
def _(dense, offsets, total_L=None):
    if total_L is None:
        total_L = int(offsets[0][-1].item())
    return dense.new_empty((total_L, *dense.shape[2:])), torch.empty_like(offsets[0])


@torch.library.register_fake("recir::b200_concat_2d_jagged")
def _(values_left, offsets_left, values_right, offsets_right):
    return values_left.new_empty((values_left.shape[0] + values_right.shape[0], *values_left.shape[1:]))


@torch.library.register_fake("recir::b200_split_2d_jagged")
def _(values, offsets_left, offsets_right, seq_len_a, seq_len_b):
    return values.new_empty((seq_len_a, *values.shape[1:])), values.new_empty((seq_len_b, *values.shape[1:]))


# the ops of a pair are each other's backward (recir/ops/jagged_ops.py:16-18, :320-400)
def _j2d_setup(ctx, inputs, output):
    values, offsets, max_lengths, _pad = inputs
    ctx.offsets, ctx.total = offsets, values.shape[0]


def _j2d_backward(ctx, grad):
    g, _ = torch.ops.recir.b200_dense_to_jagged(grad.contiguous(), ctx.offsets, ctx.total)
    # trailing arguments left at their defaults are not passed on by the dispatcher, so the number of
    # non-tensor slots varies with the call
    return (g, [None] * len(ctx.offsets)) + (None,) * (len(ctx.needs_input_grad) - 2)


def _d2j_setup(ctx, inputs, output):
    dense, offsets, _total = inputs
    ctx.offsets, ctx.n = offsets, dense.shape[1]


def _d2j_backward(ctx, grad, _grad_offsets):
    g = torch.ops.recir.b200_jagged_to_padded_dense(grad.contiguous(), ctx.offsets, [ctx.n], 0.0)
    return (g, [None] * len(ctx.offsets)) + (None,) * (len(ctx.needs_input_grad) - 2)


def _concat_setup(ctx, inputs, output):
    vl, ol, vr, orr = inputs
    ctx.save_for_backward(ol, orr)
    ctx.la, ctx.lb = vl.shape[0], vr.shape[0]


def _concat_backward(ctx, grad):
    ol, orr = ctx.saved_tensors
    gl, gr = torch.ops.recir.b200_split_2d_jagged(grad.contiguous(), ol, orr, ctx.la, ctx.lb)
    return gl, None, gr, None


def _split_setup(ctx, inputs, output):
    _v, ol, orr, _a, _b = inputs
    ctx.save_for_backward(ol, orr)


def _split_backward(ctx, grad_left, grad_right):
    ol, orr = ctx.saved_tensors
    return torch.ops.recir.b200_concat_2d_jagged(grad_left.contiguous(), ol, grad_right.contiguous(), orr), None, None, None, None


torch.library.register_autograd("recir::b200_jagged_to_padded_dense", _j2d_backward, setup_context=_j2d_setup)
torch.library.register_autograd("recir::b200_dense_to_jagged", _d2j_backward, setup_context=_d2j_setup)
torch.library.register_autograd("recir::b200_concat_2d_jagged", _concat_backward, setup_context=_concat_setup)
torch.library.register_autograd("recir::b200_split_2d_jagged", _split_backward, setup_context=_split_setup)
