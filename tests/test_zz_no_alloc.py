"""Forward through ``b200_hstu_fwd_static_scratch``: the entry point for callers that cannot
hand the library any scratch memory (a thread that must not stall on an allocation, a plugin
inside a runtime that owns all device memory, a loop whose memory plan is frozen).  It keeps
the work list in an array built into the library and must produce exactly what the regular
entry point produces, call after call, since every call rebuilds what it reads from that
shared array.  Collected last on purpose, so that a stop-at-first-failure run has already
exercised everything else."""
import ctypes

import pytest
import torch

from recir_b200 import _lib, ops
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


def _problem(seed, lengths, targets, H=2, D=128):
    g = torch.Generator().manual_seed(seed)
    T = sum(lengths)
    q, k, v = ((torch.randn(T, H, D, generator=g) * 0.5).to(torch.bfloat16).cuda() for _ in range(3))
    off = torch.zeros(len(lengths) + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(torch.tensor(lengths), 0)
    return q, k, v, off.cuda(), torch.tensor(targets, dtype=torch.int64).cuda()


def _static_scratch_forward(q, k, v, off, nt, max_seq_len, alpha, **mask):
    """Fills the C struct exactly like the operator does, but passes no workspace."""
    lib = _lib.load()
    out = torch.empty_like(v)
    p = _lib.B200HstuParams()
    keep = ops._fill(p, q, k, v, off, max_seq_len, alpha, True, nt, mask.get("contextual_seq_len", 0),
                     mask.get("max_attn_len", 0), None, 0)
    p.o, p.o_row_stride = out.data_ptr(), out.stride(0)
    assert lib.b200_hstu_uses_tensor_cores(ctypes.byref(p), 0) == 1  # the variant that needs scratch
    assert 0 < lib.b200_hstu_workspace_bytes(ctypes.byref(p), 0) <= _lib.STATIC_SCRATCH_BYTES
    rc = lib.b200_hstu_fwd_static_scratch(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.strerror(rc)
    torch.cuda.synchronize()
    del keep
    return out


def test_static_scratch_forward_matches_regular_entry_point_twice():
    alpha = 1.0 / 128 ** 0.5
    # two different problems back to back: the second call finds the first call's work list
    # in the shared array and must not be affected by it
    first = _problem(1, [300, 129, 64, 700], [20, 129, 0, 64])
    second = _problem(2, [90, 1000], [5, 100])
    for (q, k, v, off, nt), n, mask in ((first, 700, {}), (second, 1000, {"max_attn_len": 200, "contextual_seq_len": 2})):
        ref = torch.ops.recir.b200_hstu_attention_fwd(q, k, v, off, n, alpha, True, nt,
                                                      mask.get("contextual_seq_len", 0), mask.get("max_attn_len", 0),
                                                      None, 0)
        got = _static_scratch_forward(q, k, v, off, nt, n, alpha, **mask)
        assert torch.isfinite(got.float()).all()
        assert rel_l2(got.float(), ref.float()) <= 6e-3  # the bound the other GPU tests use
        assert torch.equal(got, ref)  # same kernels, same order of operations


def test_static_scratch_rejects_oversized_problems_on_the_host():
    lib = _lib.load()
    p = _lib.B200HstuParams()
    q = torch.empty(8, 2, 128, dtype=torch.bfloat16, device="cuda")
    off = torch.tensor([0, 8], device="cuda")
    keep = ops._fill(p, q, q, q, off, 8, 1.0, True, None, 0, 0, None, 0)
    p.o, p.o_row_stride = q.data_ptr(), q.stride(0)
    p.T = 200_000_000  # claims far more tokens than the built-in array can index
    assert lib.b200_hstu_workspace_bytes(ctypes.byref(p), 0) > _lib.STATIC_SCRATCH_BYTES
    assert lib.b200_hstu_fwd_static_scratch(ctypes.byref(p), None) == -7
    assert "scratch" in _lib.strerror(-7)
    del keep


def test_static_scratch_first_use_from_a_fresh_host_thread():
    """The address of the built-in array is looked up per device, with the device that owns the inputs
    made current for the lookup: a host thread whose first CUDA work is this entry point gets the same
    result as the main thread."""
    import threading

    alpha = 1.0 / 128 ** 0.5
    q, k, v, off, nt = _problem(3, [257, 400], [10, 0])
    want = _static_scratch_forward(q, k, v, off, nt, 400, alpha)
    got = {}

    def work():
        got["o"] = _static_scratch_forward(q, k, v, off, nt, 400, alpha)

    t = threading.Thread(target=work)
    t.start()
    t.join()
    assert torch.equal(got["o"], want)
