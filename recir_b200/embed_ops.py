"""``torch.library`` operator for the position + timestamp embedding add in front of the STU stack.

``recir::b200_add_ts_pos_emb_fwd`` has the positional schema of the reference's
``hammer::add_ts_pos_emb_fwd_op`` (``recir/ops/kjt_split_per_feature.cpp:776-779``, semantics
``:307-428``) and returns the same five tensors: the embeddings with position and time-bucket rows
added, and the position / time-bucket indices sorted together with their sort permutations (the
indices come out of the CUDA kernel per token; the two sorts are library calls).  The packed rows
must be exactly the sequences (``seq_offsets[-1] == seq_embeddings.shape[0]``), as in the
reference's use.  CUDA tensors only.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _check, _DTYPES

_LIBDEF = torch.library.Library("recir", "FRAGMENT")
_LIBDEF.define(
    "b200_add_ts_pos_emb_fwd(Tensor seq_embeddings, Tensor seq_offsets, Tensor pos_embeddings, Tensor ts_embeddings, "
    "Tensor timestamps, Tensor seq_lengths, Tensor? num_targets, int max_seq_len, int max_contextual_seq_len, "
    "bool interleave_targets, str time_bucket_fn) -> (Tensor, Tensor, Tensor, Tensor, Tensor)")

launch_counter = 0


def _add_ts_pos_emb_cuda(x, seq_offsets, pos, ts, timestamps, seq_lengths, num_targets, max_seq_len,
                         max_contextual_seq_len, interleave_targets, time_bucket_fn):
    global launch_counter
    # messages of recir/ops/kjt_split_per_feature.cpp:320-346
    if x.dim() != 2:
        raise ValueError("sequence embeddings must be two-dimensional")
    if pos.dim() != 2 or ts.dim() != 2:
        raise ValueError("position and timestamp embeddings must be two-dimensional")
    if timestamps.dim() != 2:
        raise ValueError("timestamps must be two-dimensional")
    if seq_lengths.dim() != 1:
        raise ValueError("sequence lengths must be one-dimensional")
    if x.shape[1] != pos.shape[1] or x.shape[1] != ts.shape[1]:
        raise ValueError("all embeddings must have the same dimension")
    if ts.shape[0] < 2049:
        raise ValueError("timestamp embeddings must contain 2049 buckets")
    b = seq_lengths.numel()
    if seq_offsets.numel() != b + 1:
        raise ValueError("sequence offsets size must match the batch size")
    if timestamps.shape[0] != b:
        raise ValueError("timestamps size must match the batch size")
    if num_targets is not None and num_targets.numel() != b:
        raise ValueError("num_targets size must match the batch size")
    if time_bucket_fn not in ("log", "sqrt"):
        raise ValueError(f"unknown time_bucket_fn {time_bucket_fn!r}")
    if x.dtype not in _DTYPES or x.shape[1] % 8 != 0:
        raise ValueError("embeddings must be float32, bfloat16 or float16 with a multiple of 8 columns")
    if pos.dtype != ts.dtype or pos.dtype not in (x.dtype, torch.float32):
        raise ValueError("the embedding tables must share a dtype: that of the sequence embeddings, or float32")
    x, pos, ts = x.contiguous(), pos.contiguous(), ts.contiguous()
    stamps = timestamps.to(torch.int64).contiguous()
    rows = x.shape[0]
    out = torch.empty_like(x)
    pos_idx = torch.empty(rows, dtype=torch.int32, device=x.device)
    ts_idx = torch.empty(rows, dtype=torch.int32, device=x.device)
    if rows > 0:
        lens_dt = torch.int64 if (seq_lengths.dtype == torch.int64 or (num_targets is not None and num_targets.dtype == torch.int64)) \
            else torch.int32
        lens = seq_lengths.to(lens_dt).contiguous()
        tg = None if num_targets is None else num_targets.to(lens_dt).contiguous()
        off = seq_offsets.contiguous() if seq_offsets.dtype in (torch.int32, torch.int64) else seq_offsets.to(torch.int64)
        p = _lib.B200EmbedParams()
        p.struct_size = ctypes.sizeof(p)
        p.flags = ((_lib.EMBED_OFFSETS_I64 if off.dtype == torch.int64 else 0) | (_lib.EMBED_LENGTHS_I64 if lens_dt == torch.int64 else 0)
                   | (_lib.EMBED_INTERLEAVE if interleave_targets else 0) | (_lib.EMBED_SQRT if time_bucket_fn == "sqrt" else 0)
                   | (_lib.EMBED_TABLES_F32 if pos.dtype == torch.float32 and x.dtype != torch.float32 else 0))
        p.dtype = _DTYPES[x.dtype]
        p.rows, p.cols, p.num_seqs = rows, x.shape[1], b
        p.pos_rows, p.ts_cols, p.max_contextual_seq_len = pos.shape[0], stamps.shape[1], int(max_contextual_seq_len)
        p.x_row_stride, p.out_row_stride = x.stride(0), out.stride(0)
        p.pos_row_stride, p.ts_table_row_stride = pos.stride(0), ts.stride(0)
        p.x, p.pos_table, p.ts_table, p.timestamps = x.data_ptr(), pos.data_ptr(), ts.data_ptr(), stamps.data_ptr()
        p.seq_offsets, p.seq_lengths = off.data_ptr(), lens.data_ptr()
        p.num_targets = None if tg is None else tg.data_ptr()
        p.out, p.pos_index, p.ts_index = out.data_ptr(), pos_idx.data_ptr(), ts_idx.data_ptr()
        with torch.cuda.device(x.device):
            rc = _lib.load().b200_stu_add_ts_pos_emb(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        _check(rc, "b200_stu_add_ts_pos_emb")
        launch_counter += 1
    sorted_pos, pos_order = torch.sort(pos_idx)
    sorted_ts, ts_order = torch.sort(ts_idx)
    return out, sorted_pos, pos_order.to(torch.int32), sorted_ts, ts_order.to(torch.int32)


def _add_ts_pos_emb_fake(x, seq_offsets, pos, ts, timestamps, seq_lengths, num_targets, max_seq_len,
                         max_contextual_seq_len, interleave_targets, time_bucket_fn):
    idx = lambda: x.new_empty((x.shape[0],), dtype=torch.int32)  # noqa: E731
    return torch.empty_like(x), idx(), idx(), idx(), idx()


_LIBDEF.impl("b200_add_ts_pos_emb_fwd", _add_ts_pos_emb_cuda, "CUDA")
torch.library.register_fake("recir::b200_add_ts_pos_emb_fwd", _add_ts_pos_emb_fake)
