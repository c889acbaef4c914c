"""B200-native gated delta-rule (GDN) ops: drop-in for the GDN entry points
of ``torch_mlu_ops.triton_ops`` (chunked prefill with its autograd backward,
slot-indexed recurrent decode, the plain recurrence) and the causal conv1d
that feeds them (also fused into the prefill), plus a prefill for inputs in
host memory.

The ops run hand-written sm_100a CUDA kernels in ``libgdn_b200.so``, called
through its C ABI (``include/gdn_b200.h``).
"""

from .conv import causal_conv1d, causal_conv1d_fn, causal_conv1d_update  # noqa: F401
from .conv_gdn import causal_conv1d_chunk_gated_delta_rule  # noqa: F401
from .gdn import (  # noqa: F401
    chunk_gated_delta_rule,
    chunk_gated_delta_rule_bwd,
    chunk_gated_delta_rule_from_host,
    chunk_gated_delta_rule_fwd_h,
    fused_recurrent_gated_delta_rule,
    fused_recurrent_gated_delta_rule_fn,
    solve_tril,
)

__all__ = [
    "causal_conv1d",
    "causal_conv1d_chunk_gated_delta_rule",
    "causal_conv1d_fn",
    "causal_conv1d_update",
    "chunk_gated_delta_rule",
    "chunk_gated_delta_rule_bwd",
    "chunk_gated_delta_rule_from_host",
    "chunk_gated_delta_rule_fwd_h",
    "fused_recurrent_gated_delta_rule",
    "fused_recurrent_gated_delta_rule_fn",
    "solve_tril",
]
