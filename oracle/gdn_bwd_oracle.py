"""Gradients of the gated delta rule by float64 autograd through the
token-by-token recurrence.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the
CUDA backward, never the product.

The reference's backward (``triton/fla/chunk.py:76-186``, autograd node
``chunk.py:188-251``) differentiates the chunked forward, which computes the
same function as the recurrence (``triton/fla/fused_recurrent.py:15-131``
with a scalar decay):

    h <- exp(g_t) h;  v'_t = beta_t (v_t - h^T k_t);  h <- h + k_t v'_t^T;
    o_t = scale h^T q_t

so the gradients of that recurrence, taken by torch autograd in float64, are
the reference's gradients up to rounding.  The restatement is pinned to the
reference's own backward kernels run under the Triton CPU interpreter
(``tests/golden/make_golden.py --only bwd``, fixtures ``bwd_*.npz``).
"""

from __future__ import annotations

import numpy as np
import torch


def _bounds(B, T, cu_seqlens):
    if cu_seqlens is None:
        return [(n * T, n * T + T) for n in range(B)]
    cu = [int(c) for c in np.asarray(cu_seqlens)]
    return [(cu[i], cu[i + 1]) for i in range(len(cu) - 1)]


def _forward(q, k, v, g, beta, scale, h0, bounds, l2norm, state_v_first):
    """Token recurrence on flattened [Ttot, heads, dim] float64 tensors."""
    H, HV = q.shape[1], v.shape[1]
    grp = HV // H
    if l2norm:
        q = q / torch.sqrt((q * q).sum(-1, keepdim=True) + 1e-6)
        k = k / torch.sqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    qh = q.repeat_interleave(grp, dim=1)  # v-head hv reads q/k head hv // grp
    kh = k.repeat_interleave(grp, dim=1)
    outs = []
    finals = []
    for n, (bos, eos) in enumerate(bounds):
        if h0 is None:
            h = torch.zeros(HV, q.shape[2], v.shape[2], dtype=q.dtype)
        else:
            h = h0[n].transpose(-1, -2) if state_v_first else h0[n]
        for t in range(bos, eos):
            h = h * torch.exp(g[t])[:, None, None]
            vp = beta[t][:, None] * (v[t] - torch.einsum("hkv,hk->hv", h, kh[t]))
            h = h + torch.einsum("hk,hv->hkv", kh[t], vp)
            outs.append(torch.einsum("hkv,hk->hv", h, qh[t] * scale))
        finals.append(h.transpose(-1, -2) if state_v_first else h)
    o = torch.stack(outs, 0) if outs else v.new_zeros((0,) + v.shape[1:])
    return o, torch.stack(finals, 0)


def chunk_bwd(q, k, v, g, beta, scale, initial_state, do, dht, cu_seqlens=None,
              use_qk_l2norm=False, state_v_first=False):
    """Gradients of ``sum(o * do) + sum(final_state * dht)``.

    Shapes as in ``chunk_gated_delta_rule``: q, k ``[B, T, H, K]``; v, do
    ``[B, T, HV, V]``; g, beta ``[B, T, HV]``; initial_state, dht
    ``[N, HV, K, V]`` (``[N, HV, V, K]`` with ``state_v_first``) or None.
    Returns numpy float64 ``(dq, dk, dv, dbeta, dg, dh0, o, final_state)``
    (dh0 None without an initial state), the order of the reference's
    ``chunk_gated_delta_rule_bwd`` followed by the forward outputs.
    """
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    bounds = _bounds(B, T, cu_seqlens)

    def t64(x, shape=None):
        x = torch.as_tensor(np.asarray(x, np.float64))
        return x if shape is None else x.reshape(shape)

    ins = [t64(q, (B * T, H, K)), t64(k, (B * T, H, K)), t64(v, (B * T, HV, V)),
           t64(g, (B * T, HV)), t64(beta, (B * T, HV))]
    h0 = None if initial_state is None else t64(initial_state)
    leaves = [x.clone().requires_grad_() for x in ins]
    h0l = None if h0 is None else h0.clone().requires_grad_()
    o, ht = _forward(*leaves, scale, h0l, bounds, use_qk_l2norm, state_v_first)
    loss = (o * t64(do, (B * T, HV, V))).sum()
    if dht is not None:
        loss = loss + (ht * t64(dht)).sum()
    loss.backward()
    dq, dk, dv, dg, db = [x.grad if x.grad is not None else torch.zeros_like(x) for x in leaves]
    dh0 = None if h0l is None else (h0l.grad if h0l.grad is not None else torch.zeros_like(h0l))

    def back(x, shape):
        return x.detach().numpy().reshape(shape)

    return (back(dq, (B, T, H, K)), back(dk, (B, T, H, K)), back(dv, (B, T, HV, V)),
            back(db, (B, T, HV)), back(dg, (B, T, HV)),
            None if dh0 is None else dh0.detach().numpy(),
            back(o, (B, T, HV, V)), ht.detach().numpy())
