"""Module-name alias for drop-in use: callers that import the GDN ops from
``torch_mlu_ops.triton_ops`` (``triton_ops.py:9-16``) can import the same
names from ``domesticated_torch_mlu_ops_b200.triton_ops``.  No Triton is
involved; the ops are the CUDA implementations in :mod:`.gdn` and
:mod:`.conv`."""

from .conv import causal_conv1d, causal_conv1d_fn  # noqa: F401
from .gdn import (  # noqa: F401
    chunk_gated_delta_rule,
    fused_recurrent_gated_delta_rule,
    fused_recurrent_gated_delta_rule_fn,
)

__all__ = [
    "chunk_gated_delta_rule",
    "fused_recurrent_gated_delta_rule",
    "fused_recurrent_gated_delta_rule_fn",
    "causal_conv1d",
    "causal_conv1d_fn",
]
