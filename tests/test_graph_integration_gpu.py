"""Graph integration on the GPU: a small STU-like training step is traced with make_fx
(forward and backward in one graph), the attention nodes are retargeted to this library's
operators exactly the way the reference's pass does it (recir/lowering/op_swap.py:78-97 only
rewrites node.target), and the swapped graph is compiled by Inductor (the reference's
lowering hands segments to torch._inductor.compile_fx, recir/lowering/partial_lower.py:291-390).
The compiled step must keep both attention nodes as opaque calls into the CUDA library and
match the eager run of the un-swapped graph.

The source operators are stand-ins with the reference's schemas
(recir/ops/kjt_split_per_feature.cpp:780-783, recir/ops/helion/jagged_hstu_attention.py:875-887)
and a plain fp32 torch implementation of causal attention with targets."""
import pytest
import torch
from torch.fx.experimental.proxy_tensor import make_fx

import recir_b200  # noqa: F401  (registers the operators)
from recir_b200 import graph, ops
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


def _keep(L, t, device):
    ids = torch.arange(L, device=device).clamp(max=L - t)
    d = ids[:, None] - ids[None, :]
    return (d > 0) | torch.eye(L, dtype=torch.bool, device=device)


def _ref_fwd(N, alpha, q, k, v, off, nt):
    out = torch.zeros_like(v)
    offs, tg = off.tolist(), nt.tolist()
    for b in range(len(offs) - 1):
        s, e = offs[b], offs[b + 1]
        if e == s:
            continue
        qs, ks, vs = (x[s:e].float().transpose(0, 1) for x in (q, k, v))
        p = torch.nn.functional.silu(alpha * qs @ ks.transpose(1, 2)) / N * _keep(e - s, tg[b], q.device)
        out[s:e] = (p @ vs).transpose(0, 1).to(v.dtype)
    return out


@torch.library.custom_op("recir_b200_graph::source_attention_fwd", mutates_args=())
def _src_fwd(N: int, alpha: float, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_offsets: torch.Tensor,
             invalid_attn_mask_type: str, num_targets: torch.Tensor | None, attn_scale: torch.Tensor | None,
             max_attn_len: int, contextual_seq_len: int, full_attn_size: int,
             num_softmax_heads: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    return _ref_fwd(N, alpha, q, k, v, seq_offsets, num_targets), q.new_zeros((1,), dtype=torch.float32)


@_src_fwd.register_fake
def _(N, alpha, q, k, v, seq_offsets, invalid_attn_mask_type, num_targets, attn_scale, max_attn_len,
      contextual_seq_len, full_attn_size, num_softmax_heads=0):
    return torch.empty_like(v), q.new_empty((1,), dtype=torch.float32)


@torch.library.custom_op("recir_b200_graph::source_attention_bwd", mutates_args=())
def _src_bwd(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_offsets: torch.Tensor,
             num_targets: torch.Tensor | None, attn_scale: torch.Tensor | None, N: int, alpha: float,
             max_attn_len: int = 0, full_attn_size: int = 0, contextual_seq_len: int = 0,
             invalid_attn_mask_type: str = "lower_triangular") -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    # recir/ops/helion/jagged_hstu_attention.py:16-27 (autograd is not available below the dispatcher)
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    offs, tg = seq_offsets.tolist(), num_targets.tolist()
    for b in range(len(offs) - 1):
        s, e = offs[b], offs[b + 1]
        if e == s:
            continue
        qs, ks, vs, gs = (x[s:e].float().transpose(0, 1) for x in (q, k, v, dout))
        keep = _keep(e - s, tg[b], q.device) / N
        sc = alpha * qs @ ks.transpose(1, 2)
        sig = torch.sigmoid(sc)
        p = sc * sig * keep
        ds = (gs @ vs.transpose(1, 2)) * keep * sig * (1 + sc * (1 - sig))
        dv[s:e] = (p.transpose(1, 2) @ gs).transpose(0, 1).to(v.dtype)
        dq[s:e] = (alpha * ds @ ks).transpose(0, 1).to(q.dtype)
        dk[s:e] = (alpha * ds.transpose(1, 2) @ qs).transpose(0, 1).to(k.dtype)
    return dq, dk, dv


@_src_bwd.register_fake
def _(dout, q, k, v, seq_offsets, num_targets, attn_scale, N, alpha, max_attn_len=0, full_attn_size=0,
      contextual_seq_len=0, invalid_attn_mask_type="lower_triangular"):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


def _src_setup(ctx, inputs, output):
    N, alpha, q, k, v, off, _mask, nt, sc, *_rest = inputs
    ctx.save_for_backward(q, k, v, off, nt)
    ctx.N, ctx.alpha = N, alpha


def _src_backward(ctx, grad_out, _grad_aux):
    q, k, v, off, nt = ctx.saved_tensors
    dq, dk, dv = torch.ops.recir_b200_graph.source_attention_bwd(grad_out.contiguous(), q, k, v, off, nt, None,
                                                                 ctx.N, ctx.alpha)
    return None, None, dq, dk, dv, None, None, None, None, None, None, None, None


_src_fwd.register_autograd(_src_backward, setup_context=_src_setup)


def test_swapped_training_step_compiles_with_inductor_and_matches():
    from torch._inductor.compile_fx import compile_fx

    dev = "cuda"
    g = torch.Generator(device="cpu").manual_seed(11)
    lengths, targets = [300, 129, 0, 517], [20, 9, 0, 64]
    T, E, H, D, N = sum(lengths), 64, 2, 128, 600
    off = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0)), dtype=torch.int64, device=dev)
    nt = torch.tensor(targets, dtype=torch.int64, device=dev)
    x = (torch.randn(T, E, generator=g) * 0.5).to(dev, torch.bfloat16)
    w_in = (torch.randn(E, 3 * H * D, generator=g) * 0.1).to(dev, torch.bfloat16)
    w_out = (torch.randn(H * D, E, generator=g) * 0.1).to(dev, torch.bfloat16)
    alpha = 1.0 / D ** 0.5

    def step(x, w_in, w_out, off, nt):
        w_in = w_in.detach().requires_grad_(True)
        w_out = w_out.detach().requires_grad_(True)
        qkv = torch.nn.functional.silu(x @ w_in)
        q, k, v = (t.reshape(T, H, D).contiguous() for t in qkv.split(H * D, dim=1))
        o, _aux = torch.ops.recir_b200_graph.source_attention_fwd(N, alpha, q, k, v, off, "lower_triangular", nt, None,
                                                                  0, 0, 0, 0)
        y = o.reshape(T, H * D) @ w_out
        loss = (y.float() ** 2).mean()
        g_in, g_out = torch.autograd.grad(loss, (w_in, w_out))
        return loss, g_in, g_out

    gm = make_fx(step, tracing_mode="fake")(x, w_in, w_out, off, nt)
    src_f = torch.ops.recir_b200_graph.source_attention_fwd.default
    src_b = torch.ops.recir_b200_graph.source_attention_bwd.default
    want = tuple(t.clone() for t in gm(x, w_in, w_out, off, nt))  # eager run of the traced, un-swapped graph

    assert graph.swap_ops(gm, graph.swap_table(source_fwd=src_f, source_bwd=src_b)) == 2
    targets_after = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert src_f not in targets_after and src_b not in targets_after

    before = ops.launch_counter
    compiled = compile_fx(gm, [x, w_in, w_out, off, nt])
    got = compiled(x, w_in, w_out, off, nt)
    torch.cuda.synchronize()
    assert ops.launch_counter > before, "the compiled step must call into the CUDA library"
    assert abs(float(got[0]) - float(want[0])) <= 2e-2 * abs(float(want[0]))
    for a, b in zip(got[1:], want[1:]):
        assert rel_l2(a.float().cpu().numpy(), b.float().cpu().numpy()) <= 2e-2
