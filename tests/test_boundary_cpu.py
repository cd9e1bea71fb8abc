"""Drop-in boundary without a GPU: operator schemas, fake kernels under make_fx, the
positional swap the reference performs (recir/lowering/op_swap.py:78-97), input validation
messages (recir/ops/pallas/tests/test_jagged_hstu_attention.py:679-711) and the absence of
any CPU implementation."""
import operator

import pytest
import torch
from torch.fx.experimental.proxy_tensor import make_fx
from torch._subclasses.fake_tensor import FakeTensorMode

import recir_b200
from recir_b200 import ops


def _fake_inputs(mode, T=12, H=2, D=8, dtype=torch.float32):
    with mode:
        q = torch.empty(T, H, D, dtype=dtype, device="cpu")
        k = torch.empty(T, H, D, dtype=dtype, device="cpu")
        v = torch.empty(T, H, D, dtype=dtype, device="cpu")
        off = torch.empty(3, dtype=torch.int64, device="cpu")
        nt = torch.empty(2, dtype=torch.int64, device="cpu")
    return q, k, v, off, nt


def test_schema_is_positionally_compatible_with_reference_op():
    # hammer::triton_ragged_attention_fwd, recir/ops/kjt_split_per_feature.cpp:780-783
    want = ("N alpha q k v seq_offsets invalid_attn_mask_type num_targets attn_scale max_attn_len "
            "contextual_seq_len full_attn_size num_softmax_heads").split()
    schema = torch.ops.recir.b200_ragged_attention_fwd.default._schema
    assert [a.name for a in schema.arguments] == want
    assert len(schema.returns) == 2
    bwd = torch.ops.recir.b200_ragged_attention_bwd.default._schema
    # recir/ops/helion/jagged_hstu_attention.py:875-887
    assert [a.name for a in bwd.arguments][:11] == (
        "dout q k v seq_offsets num_targets attn_scale N alpha max_attn_len full_attn_size").split()


def test_fake_kernels_trace_forward_and_backward_as_opaque_nodes():
    mode = FakeTensorMode(allow_non_fake_inputs=True)
    q, k, v, off, nt = _fake_inputs(mode)

    def step(q, k, v):
        q = q.detach().requires_grad_(True)
        k = k.detach().requires_grad_(True)
        v = v.detach().requires_grad_(True)
        o = torch.ops.recir.b200_hstu_attention_fwd(q, k, v, off, 8, 0.5, True, nt, 0, 0, None, 0)
        dq, dk, dv = torch.autograd.grad(o.sum(), (q, k, v))
        return o, dq, dk, dv

    with mode:
        gm = make_fx(step, tracing_mode="fake")(q, k, v)
    targets = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert torch.ops.recir.b200_hstu_attention_fwd.default in targets
    assert torch.ops.recir.b200_hstu_attention_bwd.default in targets
    bwd_node = next(n for n in gm.graph.nodes if n.target == torch.ops.recir.b200_hstu_attention_bwd.default)
    assert sum(1 for u in bwd_node.users if u.target is operator.getitem) == 3
    assert bwd_node.meta["val"][0].shape == q.shape


def test_meta_kernel_visible_to_the_lowering_predicate():
    # recir/lowering/lowering_utils.py:19-27 keeps an op inside a compiled segment only if a
    # Meta kernel can be computed for it
    for name in ("b200_hstu_attention_fwd", "b200_hstu_attention_bwd", "b200_ragged_attention_fwd",
                 "b200_ragged_attention_bwd"):
        op = getattr(torch.ops.recir, name).default
        assert torch._C._dispatch_has_computed_kernel_for_dispatch_key(op.name(), "Meta")


@torch.library.custom_op("recir_b200_test::source_ragged_attention", mutates_args=())
def _source_op(N: int, alpha: float, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               seq_offsets: torch.Tensor, invalid_attn_mask_type: str, num_targets: torch.Tensor | None,
               attn_scale: torch.Tensor | None, max_attn_len: int, contextual_seq_len: int,
               full_attn_size: int, num_softmax_heads: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    raise RuntimeError("source op is a stand-in and must be swapped out")


@_source_op.register_fake
def _(N, alpha, q, k, v, seq_offsets, invalid_attn_mask_type, num_targets, attn_scale, max_attn_len,
      contextual_seq_len, full_attn_size, num_softmax_heads=0):
    return torch.empty_like(v), q.new_empty((1,), dtype=torch.float32)


def _swap(gm, mapping):
    """What recir/lowering/op_swap.py:78-97 does: retarget matching call_function nodes."""
    n = 0
    for node in gm.graph.nodes:
        if node.op == "call_function" and node.target in mapping:
            node.target = mapping[node.target]
            n += 1
    gm.recompile()
    return n


def test_positional_swap_of_the_attention_node():
    mode = FakeTensorMode(allow_non_fake_inputs=True)
    q, k, v, off, nt = _fake_inputs(mode)

    def fwd(q, k, v):
        out, _aux = torch.ops.recir_b200_test.source_ragged_attention(
            8, 0.5, q, k, v, off, "lower_triangular", nt, None, 0, 0, 0, 0)
        return out * 2

    with mode:
        gm = make_fx(fwd, tracing_mode="fake")(q, k, v)
    src = torch.ops.recir_b200_test.source_ragged_attention.default
    assert _swap(gm, {src: torch.ops.recir.b200_ragged_attention_fwd.default}) == 1
    tg = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert torch.ops.recir.b200_ragged_attention_fwd.default in tg and src not in tg
    with mode:  # the swapped graph still runs under fake tensors (Meta kernel present)
        out = gm(q, k, v)
    assert out.shape == v.shape


def test_validation_messages():
    q = torch.zeros(5, 2, 4)
    off = torch.tensor([0, 3, 5])
    with pytest.raises(ValueError, match=r"shape \[B\]"):
        recir_b200.validate_inputs(q, q, q, off, torch.zeros(3, dtype=torch.int64), 4)
    with pytest.raises(ValueError, match="packed shape"):
        recir_b200.validate_inputs(q, q, q, off, None, 4, dout=torch.zeros(2, 2, 4, 6))
    with pytest.raises(ValueError, match=r"shape \[T, H, D\]"):
        recir_b200.validate_inputs(q[0], q, q, off, None, 4)
    with pytest.raises(ValueError, match="share packed-token and head"):
        recir_b200.validate_inputs(q, q[:, :1], q, off, None, 4)
    with pytest.raises(ValueError, match="feature dimension"):
        recir_b200.validate_inputs(q, q[:, :, :2], q, off, None, 4)
    with pytest.raises(ValueError, match=r"shape \[B \+ 1\]"):
        recir_b200.validate_inputs(q, q, q, off[:1], None, 4)
    with pytest.raises(ValueError, match="max_seq_len must be positive"):
        recir_b200.validate_inputs(q, q, q, off, None, 0)
    with pytest.raises(ValueError, match="same dtype"):
        recir_b200.validate_inputs(q, q, q, off, None, 4, dout=q.double())


def test_no_cpu_implementation():
    q = torch.zeros(5, 2, 4)
    off = torch.tensor([0, 3, 5])
    with pytest.raises((NotImplementedError, RuntimeError)):
        recir_b200.hstu_attention(q, q, q, off, 4)


def test_batch_dim_rule_and_swap_helper():
    """The token axis stays the batch axis on the forward output and on each gradient taken out of
    the functional backward (recir/compiler/batch_dim.py:309-330)."""
    from recir_b200 import graph

    mode = FakeTensorMode(allow_non_fake_inputs=True)
    q, k, v, off, nt = _fake_inputs(mode)

    def step(q, k, v):
        q = q.detach().requires_grad_(True)
        o, _aux = torch.ops.recir_b200_test.source_ragged_attention(
            8, 0.5, q, k, v, off, "lower_triangular", nt, None, 0, 0, 0, 0)
        o2 = torch.ops.recir.b200_hstu_attention_fwd(q, k, v, off, 8, 0.5, True, nt, 0, 0, None, 0)
        (dq,) = torch.autograd.grad(o2.sum(), (q,))
        return o, dq

    with mode:
        gm = make_fx(step, tracing_mode="fake")(q, k, v)
    src = torch.ops.recir_b200_test.source_ragged_attention.default
    assert graph.swap_ops(gm, graph.swap_table(source_fwd=src)) == 1
    seen = {"fwd": 0, "bwd": 0, "grad": 0, "aux": 0}
    for node in gm.graph.nodes:
        if node.op != "call_function":
            continue
        bd = graph.output_batch_dim(node, 0)
        name = str(node.target)
        if name in graph.FORWARD_OPS:
            assert bd == 0
            seen["fwd"] += 1
        elif name in graph.BACKWARD_OPS:
            assert bd == 0
            seen["bwd"] += 1
        elif node.target is operator.getitem and str(node.args[0].target) in graph.BACKWARD_OPS:
            assert bd == 0
            seen["grad"] += 1
        elif node.target is operator.getitem and str(node.args[0].target) == graph.FORWARD_OPS[1]:
            assert bd == (0 if node.args[1] == 0 else None)
            seen["aux"] += 1
        else:
            assert bd is None
    assert seen["fwd"] == 2 and seen["bwd"] == 1 and seen["grad"] >= 1 and seen["aux"] >= 1


# ---------------------------------------------------------------------------------------------
# The swap as a maintainer of the reference would run it: the reference's OWN registry and pass
# (recir/lowering/op_swap.py:16-97), loaded by file path (the package itself needs jax to import).
# ---------------------------------------------------------------------------------------------

@torch.library.custom_op("recir_b200_test::source_ragged_attention_bwd", mutates_args=())
def _source_bwd_op(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_offsets: torch.Tensor,
                   num_targets: torch.Tensor | None, attn_scale: torch.Tensor | None, N: int, alpha: float,
                   max_attn_len: int = 0, full_attn_size: int = 0) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    raise RuntimeError("source op is a stand-in and must be swapped out")


@_source_bwd_op.register_fake
def _(dout, q, k, v, seq_offsets, num_targets, attn_scale, N, alpha, max_attn_len=0, full_attn_size=0):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


def _reference_op_swap():
    from oracle import refroot

    if not refroot.reference_present():
        pytest.skip("reference source tree not present")
    return refroot.load_reference_module("recir/lowering/op_swap.py", "ref_op_swap")


def test_swap_through_the_reference_registry_forward_and_backward():
    ref = _reference_op_swap()
    mode = FakeTensorMode(allow_non_fake_inputs=True)
    q, k, v, off, nt = _fake_inputs(mode)
    src_f = torch.ops.recir_b200_test.source_ragged_attention.default
    src_b = torch.ops.recir_b200_test.source_ragged_attention_bwd.default

    def step(q, k, v, dout):
        out, _aux = torch.ops.recir_b200_test.source_ragged_attention(
            8, 0.5, q, k, v, off, "lower_triangular", nt, None, 0, 0, 0, 0)
        dq, dk, dv = torch.ops.recir_b200_test.source_ragged_attention_bwd(
            dout, q, k, v, off, nt, None, 8, 0.5, 0, 0)
        return out * 2, dq + dk, dv

    with mode:
        gm = make_fx(step, tracing_mode="fake")(q, k, v, v)
    registry = ref.OpSwapRegistry()
    registry.register(src_f, torch.ops.recir.b200_ragged_attention_fwd.default)
    registry.register(src_b, torch.ops.recir.b200_ragged_attention_bwd.default)
    assert len(registry) == 2 and registry.has(src_f)
    out_gm = ref.swap_ops(gm, registry)
    assert out_gm is gm
    tg = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert tg.count(torch.ops.recir.b200_ragged_attention_fwd.default) == 1
    assert tg.count(torch.ops.recir.b200_ragged_attention_bwd.default) == 1
    assert src_f not in tg and src_b not in tg
    with mode:  # Meta kernels of the replacements: the swapped graph runs under fake tensors
        out, dqk, dv = gm(q, k, v, v)
    assert out.shape == v.shape and dqk.shape == q.shape and dv.shape == v.shape
    # an empty registry leaves the graph alone, as the reference's pass documents
    before = [n.target for n in gm.graph.nodes]
    ref.swap_ops(gm, ref.OpSwapRegistry())
    assert [n.target for n in gm.graph.nodes] == before


def test_swap_table_feeds_the_reference_registry():
    """recir_b200.graph.swap_table is the mapping to hand to the reference's registry."""
    from recir_b200 import graph

    ref = _reference_op_swap()
    src_f = torch.ops.recir_b200_test.source_ragged_attention.default
    src_b = torch.ops.recir_b200_test.source_ragged_attention_bwd.default
    registry = ref.OpSwapRegistry()
    for s, r in graph.swap_table(source_fwd=src_f, source_bwd=src_b).items():
        registry.register(s, r)
    assert registry.get(src_f) is torch.ops.recir.b200_ragged_attention_fwd.default
    assert registry.get(src_b) is torch.ops.recir.b200_ragged_attention_bwd.default


def test_status_reader_names_what_the_device_reported():
    """``check_status`` turns the device status word into an error that names the condition; here the word
    is a host tensor standing in for the per-device one (no GPU needed for the decoding)."""
    cpu = torch.device("cpu")
    try:
        ops._status[cpu] = torch.tensor([1, 102, 0, 0], dtype=torch.int32)
        with pytest.raises(RuntimeError, match=r"malformed.*WAIT_MMA"):
            ops.check_status()
        assert not ops._status[cpu].any()  # reading clears it
        ops.check_status()
        ops._status[cpu] = torch.tensor([0, 777, 0, 0], dtype=torch.int32)
        with pytest.raises(RuntimeError, match="code 777"):
            ops.check_status(what="unit")
    finally:
        ops._status.pop(cpu, None)
