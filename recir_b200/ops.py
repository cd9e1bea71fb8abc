"""``torch.library`` operators over the C ABI: the drop-in for the reference's attention op.

Registered in the ``recir`` namespace, following the reference's own convention for an
opaque forward op plus an explicit functional backward op with ``register_fake`` and
``register_autograd`` (``recir/ops/linear_cross_entropy_op.py:15-25,116-176``):

* ``recir::b200_hstu_attention_fwd`` / ``_bwd`` -- the operator surface
  (q/k/v jagged ``[T,H,D]``, ``seq_offsets``, ``max_seq_len``, ``alpha``, ``causal``,
  ``num_targets``, ``contextual_seq_len``, ``max_attn_len``, ``attn_scale``, ``full_attn_size``).
* ``recir::b200_ragged_attention_fwd`` -- positionally identical to
  ``hammer::triton_ragged_attention_fwd`` (``recir/ops/kjt_split_per_feature.cpp:780-783``) so
  that ``swap_ops`` (``recir/lowering/op_swap.py:78-97``), which only retargets a node, can
  swap it in; returns ``(out, zeros(1))`` like the reference.
* ``recir::b200_ragged_attention_bwd`` -- the backward argument list of
  ``recir/ops/helion/jagged_hstu_attention.py:875-887``.

Only a CUDA kernel is registered.  There is no CPU implementation and no alternative
backend: calling the ops with CPU tensors raises, as does a missing shared library.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}

_LIBDEF = torch.library.Library("recir", "FRAGMENT")
_COMMON = ("Tensor seq_offsets, int max_seq_len, float alpha, bool causal, Tensor? num_targets, "
           "int contextual_seq_len, int max_attn_len, Tensor? attn_scale, int full_attn_size=0")
_LIBDEF.define(f"b200_hstu_attention_fwd(Tensor q, Tensor k, Tensor v, {_COMMON}) -> Tensor")
_LIBDEF.define(
    f"b200_hstu_attention_bwd(Tensor dout, Tensor q, Tensor k, Tensor v, {_COMMON}) -> (Tensor, Tensor, Tensor)")
_LIBDEF.define(
    "b200_ragged_attention_fwd(int N, float alpha, Tensor q, Tensor k, Tensor v, Tensor seq_offsets, "
    "str invalid_attn_mask_type, Tensor? num_targets, Tensor? attn_scale, int max_attn_len, "
    "int contextual_seq_len, int full_attn_size, int num_softmax_heads=0) -> (Tensor, Tensor)")
_LIBDEF.define(
    "b200_ragged_attention_bwd(Tensor dout, Tensor q, Tensor k, Tensor v, Tensor seq_offsets, "
    "Tensor? num_targets, Tensor? attn_scale, int N, float alpha, int max_attn_len=0, "
    "int full_attn_size=0, int contextual_seq_len=0, str invalid_attn_mask_type='lower_triangular') "
    "-> (Tensor, Tensor, Tensor)")

# Set by tests/benchmarks that want the CUDA-core cross-check kernels instead of the tensor-core ones.
_force_simt = False
# Checked mode: after every call, wait for it and raise if a kernel reported a problem on the device
# (costs a device synchronisation per call; off by default, RECIR_B200_CHECK=1 turns it on).
_checked = os.environ.get("RECIR_B200_CHECK", "0") not in ("", "0")
# One persistent status word (device int32[4]) per device, handed to every call.
_status = {}
_WAIT_NAMES = {101: "WAIT_PRODUCER (TMA producer warp)", 102: "WAIT_MMA (MMA issuer warp)",
               103: "WAIT_EPILOGUE (epilogue warps)", 104: "WAIT_SCHEDULER (work-item scheduler warp)",
               111: "projection kernel: TMA producer or layer-norm warps", 112: "projection kernel: MMA issuer warp",
               113: "projection kernel: epilogue warps",
               114: "projection kernel: shared memory not 1024-byte aligned (nothing ran)"}
# Extra C-ABI flags for the backward (benchmark timing of one pass at a time).
_bwd_extra_flags = 0
# Kernel launches issued through this module since import (launch accounting for the benchmark).
launch_counter = 0
# Forward / backward calls served by the tensor-core kernels since import (the rest ran on the CUDA-core kernels).
tensor_core_calls = 0


def set_force_simt(flag: bool) -> None:
    global _force_simt
    _force_simt = bool(flag)


def set_checked(flag: bool) -> None:
    """Checked mode on/off: every operator call then synchronises and raises ``RuntimeError`` if the
    kernels flagged malformed offsets or a pipeline wait that gave up (see ``check_status``)."""
    global _checked
    _checked = bool(flag)


def status_tensor(device) -> torch.Tensor:
    """The device int32[4] status word every call on ``device`` reports into (created on first use)."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    t = _status.get(device)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=device)
        _status[device] = t
    return t


def check_status(device=None, what: str = "recir_b200") -> None:
    """Waits for the work queued on ``device`` (default: every device used so far), reads the status
    word(s), clears them and raises ``RuntimeError`` naming what the kernels reported:
    malformed ``seq_offsets`` (clamped on the device), or the pipeline wait that gave up
    (``WAIT_PRODUCER`` / ``WAIT_MMA`` / ``WAIT_EPILOGUE`` / ``WAIT_SCHEDULER``).  Unchecked callers can
    call this at a synchronisation point of their own, e.g. once per step."""
    devices = list(_status) if device is None else [status_tensor(device).device]
    problems = []
    for dev in devices:
        t = _status.get(dev)
        if t is None:
            continue
        vals = t.cpu().tolist()  # synchronises with the stream work queued so far
        if any(vals):
            t.zero_()
        if vals[0] & 1:
            problems.append(f"{dev}: seq_offsets were malformed (negative, decreasing, beyond T, overlapping, or a sequence longer than max_seq_len) "
                            "and were clamped on the device; the results are not meaningful")
        if vals[1]:
            problems.append(f"{dev}: a pipeline wait gave up after its time limit: "
                            f"{_WAIT_NAMES.get(vals[1], 'code ' + str(vals[1]))}; outputs are incomplete")
    if problems:
        raise RuntimeError(f"{what}: " + "; ".join(problems))


_recompute_dq = False


def set_backward_passes(dkv: bool = True, dq: bool = True, timing_only: bool = False) -> None:
    """Leave one of the two backward passes out (its outputs stay unwritten).  By default the dQ pass reads the dS
    tiles the dK/dV pass of the SAME call stored in the workspace, so a pass run alone uses the recomputing dQ
    kernel and the gradients are valid.  ``timing_only``: keep the stored-tile kernels (a dQ pass run alone then
    reads whatever the workspace holds: its time is meaningful, its output is not)."""
    global _bwd_extra_flags
    _bwd_extra_flags = (0 if dkv else _lib.FLAG_BWD_SKIP_DKV) | (0 if dq else _lib.FLAG_BWD_SKIP_DQ)
    if not (dkv and dq) and not timing_only:
        _bwd_extra_flags |= _lib.FLAG_BWD_RECOMPUTE_DQ


def set_recompute_dq(flag: bool) -> None:
    """Backward: make the dQ pass recompute S and dP (a workspace of a few hundred KB) instead of reading the dS
    tiles the dK/dV pass stores (32 KB per 128 x 128 tile the mask keeps; see ``b200_hstu_workspace_bytes``)."""
    global _recompute_dq
    _recompute_dq = bool(flag)


# ---------------------------------------------------------------------------
# validation (messages follow recir/ops/pallas/jagged_hstu_attention.py:1486-1515,1373-1376)
# ---------------------------------------------------------------------------

def validate_inputs(q, k, v, seq_offsets, num_targets, max_seq_len, attn_scale=None, dout=None) -> int:
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, and v must have shape [T, H, D]")
    if q.shape[:2] != k.shape[:2] or q.shape[:2] != v.shape[:2]:
        raise ValueError("q, k, and v must share packed-token and head dimensions")
    if q.shape[2] != k.shape[2]:
        raise ValueError("q and k must share their feature dimension")
    if seq_offsets.dim() != 1 or seq_offsets.shape[0] < 2:
        raise ValueError("seq_offsets must have shape [B + 1]")
    num_sequences = seq_offsets.shape[0] - 1
    if num_targets is not None and tuple(num_targets.shape) != (num_sequences,):
        raise ValueError("num_targets must have shape [B]")
    if max_seq_len <= 0:
        raise ValueError("max_seq_len must be positive")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, and v must have the same dtype")
    if q.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {q.dtype}: expected float32, bfloat16 or float16")
    if seq_offsets.dtype not in (torch.int32, torch.int64):
        raise ValueError("seq_offsets must be int32 or int64")
    if num_targets is not None and num_targets.dtype not in (torch.int32, torch.int64):
        raise ValueError("num_targets must be int32 or int64")
    if attn_scale is not None and attn_scale.dim() > 0 and tuple(attn_scale.shape) != (q.shape[0],) \
            and attn_scale.numel() != 1:
        raise ValueError("attn_scale must be a scalar tensor or have shape [T]")
    if dout is not None:
        if dout.shape != v.shape:
            raise ValueError("grad_out must have packed shape [T, H, Dv]")
        if dout.dtype != v.dtype:
            raise ValueError("grad_out and v must have the same dtype")
    return num_sequences


def _rows(t: torch.Tensor) -> torch.Tensor:
    """Dense heads and unit inner stride are required; anything else is copied once."""
    if t.stride(2) == 1 and t.stride(1) == t.shape[2] and (t.shape[0] <= 1 or t.stride(0) >= t.shape[1] * t.shape[2]):
        return t
    return t.contiguous()


def _fill(params, q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets, contextual_seq_len,
          max_attn_len, attn_scale, full_attn_size):
    keep = []
    dev = q.device
    for name, t in (("seq_offsets", seq_offsets), ("num_targets", num_targets), ("attn_scale", attn_scale)):
        if t is not None and t.device != dev:
            raise ValueError(f"{name} must live on the same device as q")
    params.struct_size = ctypes.sizeof(_lib.B200HstuParams)
    flags = _lib.FLAG_CAUSAL if causal else 0
    so = seq_offsets.contiguous()
    keep.append(so)
    if so.dtype == torch.int64:
        flags |= _lib.FLAG_OFFSETS_I64
    params.seq_offsets = so.data_ptr()
    if num_targets is not None:
        nt = num_targets.contiguous()
        keep.append(nt)
        if nt.dtype == torch.int64:
            flags |= _lib.FLAG_TARGETS_I64
        params.num_targets = nt.data_ptr()
    if attn_scale is not None:
        sc = attn_scale.to(torch.float32).contiguous().reshape(-1)
        keep.append(sc)
        # 0-d (or single-value) tensor: one scale; otherwise one value per query token, as the
        # reference slices it (recir/ops/kjt_split_per_feature.cpp:677-682)
        if attn_scale.dim() > 0 and sc.numel() != 1:
            flags |= _lib.FLAG_SCALE_PER_TOKEN
        params.attn_scale = sc.data_ptr()
    if _force_simt:
        flags |= _lib.FLAG_FORCE_SIMT
    params.flags = flags
    params.q, params.k, params.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    params.q_row_stride, params.k_row_stride, params.v_row_stride = q.stride(0), k.stride(0), v.stride(0)
    params.T = q.shape[0]
    params.B = so.shape[0] - 1
    params.H, params.Dqk, params.Dv = q.shape[1], q.shape[2], v.shape[2]
    params.dtype = _DTYPES[q.dtype]
    params.max_seq_len = int(max_seq_len)
    params.max_attn_len = int(max_attn_len)
    params.contextual_seq_len = int(contextual_seq_len)
    params.full_attn_size = int(full_attn_size)
    params.alpha = float(alpha)
    params.status = status_tensor(dev).data_ptr()
    return keep


def _workspace(lib, params, pass_id, device):
    need = lib.b200_hstu_workspace_bytes(ctypes.byref(params), pass_id)
    if need == 0:
        return None
    try:
        ws = torch.empty(need + 256, dtype=torch.uint8, device=device)
    except torch.cuda.OutOfMemoryError:
        # The backward's dS tiles do not fit beside what the caller holds: the recomputing dQ pass needs
        # only the work list (same gradients, bit for bit).
        if pass_id != 1 or (params.flags & _lib.FLAG_BWD_RECOMPUTE_DQ):
            raise
        params.flags |= _lib.FLAG_BWD_RECOMPUTE_DQ
        need = lib.b200_hstu_workspace_bytes(ctypes.byref(params), pass_id)
        ws = torch.empty(need + 256, dtype=torch.uint8, device=device)
    off = (-ws.data_ptr()) % 256
    params.workspace = ws.data_ptr() + off
    params.workspace_bytes = need
    return ws


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = _lib.strerror(rc)
        if rc in (-1, -2, -3, -6):
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what}: {msg}")


TC_HEAD_DIM = 128  # the head dimension of the tensor-core kernels


def _pads_to_tensor_core_width(q, k, v, causal) -> bool:
    """16-bit causal attention with one head dimension below 128 (a multiple of 8) for q, k and v: zero columns
    change neither q kT nor the leading columns of p v, so the tensor-core kernels serve it on inputs padded to
    128 columns (twice the tensor work at D = 64, still far ahead of the CUDA-core kernels, which are what a
    head dimension the tensor-core kernels do not take falls back to)."""
    d = q.shape[2]
    return (not _force_simt and causal and q.dtype in (torch.bfloat16, torch.float16) and k.shape[2] == d
            and v.shape[2] == d and d < TC_HEAD_DIM and d % 8 == 0 and q.shape[0] > 0)


def _pad_head_dim(t: torch.Tensor) -> torch.Tensor:
    out = t.new_zeros((t.shape[0], t.shape[1], TC_HEAD_DIM))
    out[:, :, :t.shape[2]] = t
    return out


def _fwd_cuda(q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets, contextual_seq_len,
              max_attn_len, attn_scale, full_attn_size=0, out=None):
    """``out``: optional result tensor of the caller ([T, H, Dv], rows contiguous); allocated when absent."""
    global launch_counter, tensor_core_calls
    validate_inputs(q, k, v, seq_offsets, num_targets, max_seq_len, attn_scale)
    lib = _lib.load()
    q, k, v = _rows(q), _rows(k), _rows(v)
    if _pads_to_tensor_core_width(q, k, v, causal):
        padded = _fwd_cuda(_pad_head_dim(q), _pad_head_dim(k), _pad_head_dim(v), seq_offsets, max_seq_len, alpha, causal,
                           num_targets, contextual_seq_len, max_attn_len, attn_scale, full_attn_size)
        if out is None:
            return padded[:, :, :v.shape[2]].contiguous()
        out.copy_(padded[:, :, :v.shape[2]])
        return out
    if out is None:
        out = torch.empty((q.shape[0], q.shape[1], v.shape[2]), dtype=v.dtype, device=v.device)
    elif out.shape != (q.shape[0], q.shape[1], v.shape[2]) or out.dtype != v.dtype or out.device != v.device \
            or out.stride(2) != 1 or out.stride(1) != out.shape[2]:
        raise ValueError("out must be a [T, H, Dv] tensor of v's dtype and device with contiguous rows")
    if q.shape[0] == 0:
        return out
    p = _lib.B200HstuParams()
    with torch.cuda.device(q.device):
        keep = _fill(p, q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets,
                     contextual_seq_len, max_attn_len, attn_scale, full_attn_size)
        p.o = out.data_ptr()
        p.o_row_stride = out.stride(0)
        keep.append(_workspace(lib, p, 0, q.device))
        rc = lib.b200_hstu_fwd(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        _check(rc, "b200_hstu_fwd")
        launch_counter += lib.b200_hstu_launch_count(ctypes.byref(p), 0)
        tensor_core_calls += lib.b200_hstu_uses_tensor_cores(ctypes.byref(p), 0) == 1
        if _checked:
            check_status(q.device, "b200_hstu_fwd")
    del keep
    return out


def _bwd_cuda(dout, q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets, contextual_seq_len,
              max_attn_len, attn_scale, full_attn_size=0, grads=None):
    """``grads``: optional (dq, dk, dv) tensors of the caller, shaped like q, k, v with contiguous rows."""
    global launch_counter, tensor_core_calls
    validate_inputs(q, k, v, seq_offsets, num_targets, max_seq_len, attn_scale, dout)
    lib = _lib.load()
    q, k, v, dout = _rows(q), _rows(k), _rows(v), _rows(dout)
    if _pads_to_tensor_core_width(q, k, v, causal):
        d = q.shape[2]
        padded = _bwd_cuda(_pad_head_dim(dout), _pad_head_dim(q), _pad_head_dim(k), _pad_head_dim(v), seq_offsets, max_seq_len,
                           alpha, causal, num_targets, contextual_seq_len, max_attn_len, attn_scale, full_attn_size)
        if grads is None:
            return tuple(g[:, :, :d].contiguous() for g in padded)
        for dst, g in zip(grads, padded):
            dst.copy_(g[:, :, :d])
        return tuple(grads)
    if grads is None:
        dq = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
        dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
    else:
        dq, dk, dv = grads
        for g, like in ((dq, q), (dk, k), (dv, v)):
            if g.shape != like.shape or g.dtype != like.dtype or g.device != like.device or g.stride(2) != 1 \
                    or g.stride(1) != g.shape[2]:
                raise ValueError("grads must be (dq, dk, dv) shaped like q, k, v with contiguous rows")
    if q.shape[0] == 0:
        return dq, dk, dv
    p = _lib.B200HstuParams()
    with torch.cuda.device(q.device):
        keep = _fill(p, q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets,
                     contextual_seq_len, max_attn_len, attn_scale, full_attn_size)
        p.flags |= _bwd_extra_flags | (_lib.FLAG_BWD_RECOMPUTE_DQ if _recompute_dq else 0)
        p.d_o = dout.data_ptr()
        p.do_row_stride = dout.stride(0)
        p.dq, p.dk, p.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
        p.dq_row_stride, p.dk_row_stride, p.dv_row_stride = dq.stride(0), dk.stride(0), dv.stride(0)
        keep.append(_workspace(lib, p, 1, q.device))
        rc = lib.b200_hstu_bwd(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        _check(rc, "b200_hstu_bwd")
        launch_counter += lib.b200_hstu_launch_count(ctypes.byref(p), 1)
        tensor_core_calls += lib.b200_hstu_uses_tensor_cores(ctypes.byref(p), 1) == 1
        if _checked:
            check_status(q.device, "b200_hstu_bwd")
    del keep
    return dq, dk, dv


def _ragged_fwd_cuda(N, alpha, q, k, v, seq_offsets, invalid_attn_mask_type, num_targets, attn_scale,
                     max_attn_len, contextual_seq_len, full_attn_size, num_softmax_heads=0):
    if num_softmax_heads != 0:
        raise ValueError("softmax attention heads are unsupported")
    out = torch.ops.recir.b200_hstu_attention_fwd(
        q, k, v, seq_offsets, N, alpha, invalid_attn_mask_type == "lower_triangular", num_targets,
        contextual_seq_len, max_attn_len, attn_scale, full_attn_size)
    return out, torch.zeros(1, dtype=torch.float32, device=q.device)


def _ragged_bwd_cuda(dout, q, k, v, seq_offsets, num_targets, attn_scale, N, alpha, max_attn_len=0,
                     full_attn_size=0, contextual_seq_len=0, invalid_attn_mask_type="lower_triangular"):
    return torch.ops.recir.b200_hstu_attention_bwd(
        dout, q, k, v, seq_offsets, N, alpha, invalid_attn_mask_type == "lower_triangular", num_targets,
        contextual_seq_len, max_attn_len, attn_scale, full_attn_size)


_LIBDEF.impl("b200_hstu_attention_fwd", _fwd_cuda, "CUDA")
_LIBDEF.impl("b200_hstu_attention_bwd", _bwd_cuda, "CUDA")
_LIBDEF.impl("b200_ragged_attention_fwd", _ragged_fwd_cuda, "CUDA")
_LIBDEF.impl("b200_ragged_attention_bwd", _ragged_bwd_cuda, "CUDA")


# ---------------------------------------------------------------------------
# fake (Meta) kernels: outputs allocated in the ambient fake mode
# ---------------------------------------------------------------------------

@torch.library.register_fake("recir::b200_hstu_attention_fwd")
def _fwd_fake(q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets, contextual_seq_len,
              max_attn_len, attn_scale, full_attn_size=0):
    return v.new_empty((q.shape[0], q.shape[1], v.shape[2]))


@torch.library.register_fake("recir::b200_hstu_attention_bwd")
def _bwd_fake(dout, q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets, contextual_seq_len,
              max_attn_len, attn_scale, full_attn_size=0):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


@torch.library.register_fake("recir::b200_ragged_attention_fwd")
def _ragged_fwd_fake(N, alpha, q, k, v, seq_offsets, invalid_attn_mask_type, num_targets, attn_scale,
                     max_attn_len, contextual_seq_len, full_attn_size, num_softmax_heads=0):
    return v.new_empty((q.shape[0], q.shape[1], v.shape[2])), q.new_empty((1,), dtype=torch.float32)


@torch.library.register_fake("recir::b200_ragged_attention_bwd")
def _ragged_bwd_fake(dout, q, k, v, seq_offsets, num_targets, attn_scale, N, alpha, max_attn_len=0,
                     full_attn_size=0, contextual_seq_len=0, invalid_attn_mask_type="lower_triangular"):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


# ---------------------------------------------------------------------------
# autograd: forward saves q/k/v only (the op keeps no softmax statistics)
# ---------------------------------------------------------------------------

def _fwd_setup_context(ctx, inputs, output) -> None:
    (q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets, contextual_seq_len, max_attn_len,
     attn_scale, full_attn_size) = inputs
    ctx.save_for_backward(q, k, v, seq_offsets, num_targets, attn_scale)
    ctx.cfg = (max_seq_len, alpha, causal, contextual_seq_len, max_attn_len, full_attn_size)


def _fwd_backward(ctx, grad_out):
    q, k, v, seq_offsets, num_targets, attn_scale = ctx.saved_tensors
    max_seq_len, alpha, causal, contextual_seq_len, max_attn_len, full_attn_size = ctx.cfg
    dq, dk, dv = torch.ops.recir.b200_hstu_attention_bwd(
        grad_out, q, k, v, seq_offsets, max_seq_len, alpha, causal, num_targets, contextual_seq_len,
        max_attn_len, attn_scale, full_attn_size)
    return dq, dk, dv, None, None, None, None, None, None, None, None, None


torch.library.register_autograd("recir::b200_hstu_attention_fwd", _fwd_backward,
                                setup_context=_fwd_setup_context)


def _ragged_setup_context(ctx, inputs, output) -> None:
    (N, alpha, q, k, v, seq_offsets, mask_type, num_targets, attn_scale, max_attn_len,
     contextual_seq_len, full_attn_size, _nsh) = inputs
    ctx.save_for_backward(q, k, v, seq_offsets, num_targets, attn_scale)
    ctx.cfg = (N, alpha, mask_type, max_attn_len, contextual_seq_len, full_attn_size)


def _ragged_backward(ctx, grad_out, _grad_aux):
    q, k, v, seq_offsets, num_targets, attn_scale = ctx.saved_tensors
    N, alpha, mask_type, max_attn_len, contextual_seq_len, full_attn_size = ctx.cfg
    dq, dk, dv = torch.ops.recir.b200_ragged_attention_bwd(
        grad_out, q, k, v, seq_offsets, num_targets, attn_scale, N, alpha, max_attn_len, full_attn_size,
        contextual_seq_len, mask_type)
    return None, None, dq, dk, dv, None, None, None, None, None, None, None, None


torch.library.register_autograd("recir::b200_ragged_attention_fwd", _ragged_backward,
                                setup_context=_ragged_setup_context)


# ---------------------------------------------------------------------------
# functional front end
# ---------------------------------------------------------------------------

def hstu_attention(q, k, v, seq_offsets, max_seq_len, alpha=None, causal=True, num_targets=None,
                   contextual_seq_len=0, max_attn_len=0, attn_scale=None, full_attn_size=0):
    """HSTU jagged pointwise attention (differentiable).  ``alpha`` defaults to ``1/sqrt(Dqk)``
    and the scale to ``1/max_seq_len`` (``recir/ops/pallas/jagged_hstu_attention.py:1552-1555``)."""
    validate_inputs(q, k, v, seq_offsets, num_targets, max_seq_len, attn_scale)
    if alpha is None:
        alpha = 1.0 / (q.shape[2] ** 0.5)
    return torch.ops.recir.b200_hstu_attention_fwd(
        q, k, v, seq_offsets, int(max_seq_len), float(alpha), bool(causal), num_targets,
        int(contextual_seq_len), int(max_attn_len), attn_scale, int(full_attn_size))


def hstu_attention_backward(dout, q, k, v, seq_offsets, max_seq_len, alpha=None, causal=True,
                            num_targets=None, contextual_seq_len=0, max_attn_len=0, attn_scale=None,
                            full_attn_size=0):
    """Explicit functional backward: returns ``(dq, dk, dv)``."""
    validate_inputs(q, k, v, seq_offsets, num_targets, max_seq_len, attn_scale, dout)
    if alpha is None:
        alpha = 1.0 / (q.shape[2] ** 0.5)
    return torch.ops.recir.b200_hstu_attention_bwd(
        dout, q, k, v, seq_offsets, int(max_seq_len), float(alpha), bool(causal), num_targets,
        int(contextual_seq_len), int(max_attn_len), attn_scale, int(full_attn_size))
