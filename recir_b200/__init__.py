"""B200-native HSTU jagged attention (forward and backward) behind the reference's operator surface.

Importing this package registers the ``recir::b200_*`` operators; the kernels live in
``libb200_hstu.so`` (C ABI in ``include/b200_hstu.h``), built by ``python -m recir_b200.build``.
"""
from .ops import (check_status, hstu_attention, hstu_attention_backward, set_checked,  # noqa: F401
                  validate_inputs)
from . import embed_ops, jagged_ops, rowwise_ops, sharding, workload  # noqa: F401
from .host_api import HostPipeline  # noqa: F401

__all__ = ["hstu_attention", "hstu_attention_backward", "validate_inputs", "check_status", "set_checked", "sharding",
           "workload", "HostPipeline"]
