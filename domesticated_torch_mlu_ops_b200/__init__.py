"""B200-native gated delta-rule (GDN) forward: drop-in for the GDN entry
points of ``torch_mlu_ops.triton_ops``.

The ops run hand-written sm_100a CUDA kernels in ``libgdn_b200.so``, called
through its C ABI (``include/gdn_b200.h``).
"""

from .gdn import (  # noqa: F401
    chunk_gated_delta_rule,
    fused_recurrent_gated_delta_rule,
    fused_recurrent_gated_delta_rule_fn,
    solve_tril,
)

__all__ = [
    "chunk_gated_delta_rule",
    "fused_recurrent_gated_delta_rule",
    "fused_recurrent_gated_delta_rule_fn",
    "solve_tril",
]
