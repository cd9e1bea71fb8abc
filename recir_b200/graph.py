"""Graph-level facts a lowering pipeline needs about the attention operators.

Two things the reference keeps in tables keyed by operator name:

* the swap table: which node targets are replaced by which
  (``recir/lowering/op_swap.py:41-48,78-97`` -- only ``node.target`` is rewritten, so source and
  replacement must agree positionally);
* the batch-dimension rule (``recir/compiler/batch_dim.py:309-330``): the forward output and
  every ``getitem`` of the functional backward keep the token axis (dim 0) of q/k/v as their
  batch axis; an op without a rule is treated as replicated.
"""
from __future__ import annotations

import operator
from typing import Optional

import torch
from torch import fx

from . import ops as _ops  # noqa: F401  (registers the operators)

FORWARD_OPS = ("recir.b200_hstu_attention_fwd.default", "recir.b200_ragged_attention_fwd.default")
BACKWARD_OPS = ("recir.b200_hstu_attention_bwd.default", "recir.b200_ragged_attention_bwd.default")


def swap_table(source_fwd=None, source_bwd=None) -> dict:
    """``{source target: replacement target}`` for a positional swap of the reference's
    ragged-attention nodes (forward schema ``recir/ops/kjt_split_per_feature.cpp:780-783``,
    backward argument list ``recir/ops/helion/jagged_hstu_attention.py:875-887``)."""
    table = {}
    if source_fwd is not None:
        table[source_fwd] = torch.ops.recir.b200_ragged_attention_fwd.default
    if source_bwd is not None:
        table[source_bwd] = torch.ops.recir.b200_ragged_attention_bwd.default
    return table


def swap_ops(gm: fx.GraphModule, table: dict) -> int:
    """Retargets matching ``call_function`` nodes and recompiles; returns how many were changed."""
    changed = 0
    for node in gm.graph.nodes:
        if node.op == "call_function" and node.target in table:
            node.target = table[node.target]
            changed += 1
    if changed:
        gm.recompile()
    return changed


def output_batch_dim(node: fx.Node, input_batch_dim: int) -> Optional[int]:
    """Batch axis of ``node``'s output given the batch axis of its q/k/v inputs, or None if the
    node is not one of this library's attention nodes (same contract as the reference's table)."""
    target = str(node.target)
    if target in FORWARD_OPS or target in BACKWARD_OPS:
        return input_batch_dim
    if node.target is operator.getitem:
        src = node.args[0]
        if isinstance(src, fx.Node) and str(src.target) in BACKWARD_OPS + ("recir.b200_ragged_attention_fwd.default",):
            # (dq, dk, dv) of the backward; element 0 of the ragged forward is the output,
            # element 1 its one-element auxiliary tensor, which has no batch axis
            if str(src.target) == "recir.b200_ragged_attention_fwd.default" and node.args[1] != 0:
                return None
            return input_batch_dim
    return None
