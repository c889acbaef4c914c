"""CPU oracle for the gated delta-rule (GDN) forward op.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path may import this
package: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and
only as the checker or as the timed CPU restatement of the reference.

Parity pins: ``tests/golden/`` holds input/output vectors produced by the
reference's own recurrent Triton kernels (``triton/fla/fused_recurrent_fn.py``
and ``triton/fla/fused_recurrent.py``) and its chunk-path Triton kernels run
under ``TRITON_INTERPRET=1``; ``tests/test_oracle.py`` checks this oracle
against them.
"""

from .gdn_oracle import (  # noqa: F401
    l2norm,
    recurrent_v_first,
    recurrent_k_first,
    chunk_local_cumsum,
    chunk_scaled_dot_kkt,
    solve_tril,
    recompute_w_u,
    chunk_fwd_h,
    chunk_fwd_h_stage,
    chunk_fwd_o,
    chunk_gated_delta_rule,
    seq_bounds,
)
