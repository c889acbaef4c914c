"""numpy restatement of the reference's gated delta-rule forward algorithms.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function takes
numpy arrays, computes in ``dtype`` (float64 by default) and follows one
reference function, cited by file:line inside the ``torch_mlu_ops`` package.

Notation (reference shapes): q, k ``[B, T, H, K]``; v ``[B, T, HV, V]``;
g, beta ``[B, T, HV]`` (beta may also be ``[B, T, HV, V]`` in the recurrent
kernels); states are ``[N, HV, K, V]`` (K-first) or ``[*, HV, V, K]``
(V-first, the decode cache).  With ``cu_seqlens`` the batch dimension is 1
and sequences are packed along T.  The q/k head serving v-head ``hv`` is
``hv // (HV // H)`` (``triton/fla/fused_recurrent_fn.py:52``).
"""

from __future__ import annotations

import numpy as np

BT = 64  # chunk size of the reference chunk path (triton/fla/chunk.py:29)


def seq_bounds(B: int, T: int, cu_seqlens=None):
    """(bos, eos) per sequence: equal-length batch or packed varlen.

    Follows the IS_VARLEN branches, e.g. ``triton/fla/fused_recurrent_fn.py:53-60``.
    """
    if cu_seqlens is None:
        return [(n * T, n * T + T) for n in range(B)]
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    return [(int(cu[i]), int(cu[i + 1])) for i in range(len(cu) - 1)]


def l2norm(x, eps: float = 1e-6):
    """x / sqrt(sum(x^2) + eps) over the last axis (``fused_recurrent_fn.py:110-112``)."""
    return x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + eps)


def _flat(x):
    # [B, T, ...] -> [B*T, ...]: sequences index the flattened token axis by bos.
    return x.reshape((-1,) + x.shape[2:])


# ---------------------------------------------------------------------------
# Recurrent forms
# ---------------------------------------------------------------------------

def recurrent_v_first(q, k, v, g, beta, scale, initial_state, *,
                      inplace_final_state=True, cu_seqlens=None,
                      ssm_state_indices=None, num_accepted_tokens=None,
                      use_qk_l2norm_in_kernel=False, gk=None, dtype=np.float64):
    """Slot-indexed recurrent decode with a V-first state cache.

    Restates ``tmo_fused_recurrent_gated_delta_rule_fwd_kernel`` and its host
    wrapper (``triton/fla/fused_recurrent_fn.py:15-159``, ``:161-233``):

    * initial state: ``initial_state[ssm_state_indices[n, i0]]`` with
      ``i0 = num_accepted_tokens[n] - 1`` under speculative decoding, else 0
      (``:88-99``); a negative index (PAD) skips the sequence entirely.
      Without indices the state row is ``bos`` (``:101-102``).
    * per token (``:105-132``): optional q/k L2 norm, q *= scale,
      S *= exp(g), v' = beta * (v - S k), S += v' k^T, o = S q.
    * ``gk`` ``[B, T, HV, K]``: the kernel's IS_KDA branch (``:77-80``,
      ``:115-120``), S *= exp(gk)[None, :] per token (on the K columns of the
      V-first state); applied after ``g`` when both are given.
    * final state (``:135-148``): in place at ``ssm_state_indices[n, t]``
      (skipped when negative) or, when not in place, at row ``bos + t`` of a
      fresh ``[T, HV, V, K]`` tensor.

    Returns ``(o, final_state, valid)`` where ``valid[n]`` is False for PAD
    sequences (the reference leaves their output rows unwritten).
    """
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    G = HV // H
    qf, kf, vf = (_flat(x).astype(dtype) for x in (q, k, v))
    gf = None if g is None else _flat(g).astype(dtype)
    gkf = None if gk is None else _flat(gk).astype(dtype)
    bf = _flat(beta).astype(dtype)
    beta_per_v = beta.ndim == v.ndim
    bounds = seq_bounds(B, T, cu_seqlens)
    o = np.zeros(vf.shape, dtype=dtype)
    if inplace_final_state:
        ht = initial_state  # mutated in place, like the reference (:185-186)
    else:
        ht = np.zeros((B * T, HV, V, K), dtype=initial_state.dtype)
    idx = None
    if ssm_state_indices is not None:
        idx = np.asarray(ssm_state_indices, dtype=np.int64)
        if idx.ndim == 1:
            idx = idx[:, None]
    h0 = np.array(initial_state, dtype=dtype, copy=True)
    valid = np.ones(len(bounds), dtype=bool)
    for n, (bos, eos) in enumerate(bounds):
        if eos - bos == 0:
            continue
        if idx is not None:
            i0 = int(num_accepted_tokens[n]) - 1 if num_accepted_tokens is not None else 0
            sidx = int(idx[n, i0])
            if sidx < 0:
                valid[n] = False
                continue
            S = h0[sidx].copy()  # [HV, V, K]
        else:
            S = h0[bos].copy()
        for i_t in range(eos - bos):
            t = bos + i_t
            qt = qf[t][np.arange(HV) // G]  # [HV, K]
            kt = kf[t][np.arange(HV) // G]
            if use_qk_l2norm_in_kernel:
                qt, kt = l2norm(qt), l2norm(kt)
            qt = qt * scale
            if gf is not None:
                S = S * np.exp(gf[t])[:, None, None]
            if gkf is not None:
                S = S * np.exp(gkf[t])[:, None, :]
            bt = bf[t] if beta_per_v else bf[t][:, None]  # [HV, V] or [HV, 1]
            vt = bt * (vf[t] - np.einsum('hvk,hk->hv', S, kt))
            S = S + vt[:, :, None] * kt[:, None, :]
            o[t] = np.einsum('hvk,hk->hv', S, qt)
            if inplace_final_state:
                fidx = int(idx[n, i_t])
                if fidx >= 0:
                    ht[fidx] = S.astype(ht.dtype)
            else:
                ht[t] = S.astype(ht.dtype)
    return o.reshape(v.shape), ht, valid


def recurrent_k_first(q, k, v, g=None, beta=None, scale=None, initial_state=None,
                      output_final_state=False, use_qk_l2norm_in_kernel=False,
                      cu_seqlens=None, gk=None, gv=None, dtype=np.float64):
    """Plain recurrence with a K-first ``[N, HV, K, V]`` state.

    Restates ``tmo_fused_recurrent_gated_delta_rule_fwd_kernel`` of
    ``triton/fla/fused_recurrent.py:15-131`` (host side ``:134-187``):
    per token S *= exp(g), S *= exp(gk)[:, None], S *= exp(gv)[None, :],
    v' = beta * (v - S^T k), S += k v'^T, o = S^T q.  ``scale`` defaults to
    K^-0.5 as the public docstring states (``triton_ops.py:204-206``).
    """
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    G = HV // H
    if scale is None:
        scale = K ** -0.5
    qf, kf, vf = (_flat(x).astype(dtype) for x in (q, k, v))
    gf = None if g is None else _flat(g).astype(dtype)
    gkf = None if gk is None else _flat(gk).astype(dtype)
    gvf = None if gv is None else _flat(gv).astype(dtype)
    bf = _flat(beta).astype(dtype)
    beta_per_v = beta.ndim == v.ndim
    bounds = seq_bounds(B, T, cu_seqlens)
    o = np.zeros(vf.shape, dtype=dtype)
    ht = np.zeros((len(bounds), HV, K, V), dtype=dtype) if output_final_state else None
    for n, (bos, eos) in enumerate(bounds):
        S = np.zeros((HV, K, V), dtype=dtype)
        if initial_state is not None:
            S += np.asarray(initial_state[n], dtype=dtype)
        for t in range(bos, eos):
            qt = qf[t][np.arange(HV) // G]
            kt = kf[t][np.arange(HV) // G]
            if use_qk_l2norm_in_kernel:
                qt, kt = l2norm(qt), l2norm(kt)
            qt = qt * scale
            if gf is not None:
                S = S * np.exp(gf[t])[:, None, None]
            if gkf is not None:
                S = S * np.exp(gkf[t])[:, :, None]
            if gvf is not None:
                S = S * np.exp(gvf[t])[:, None, :]
            bt = bf[t] if beta_per_v else bf[t][:, None]
            vt = bt * (vf[t] - np.einsum('hkv,hk->hv', S, kt))
            S = S + kt[:, :, None] * vt[:, None, :]
            o[t] = np.einsum('hkv,hk->hv', S, qt)
        if output_final_state:
            ht[n] = S
    return o.reshape(v.shape), ht


# ---------------------------------------------------------------------------
# Chunked (WY) form, one function per reference stage
# ---------------------------------------------------------------------------

def _chunks(bos, eos, bt=BT):
    return [(s, min(s + bt, eos)) for s in range(bos, eos, bt)]


def chunk_local_cumsum(g, bounds, bt=BT, dtype=np.float64):
    """Chunk-local inclusive prefix sum of g per head.

    ``tmo_chunk_local_cumsum_scalar_kernel`` (``triton/fla/cumsum.py:20-77``),
    forward (non-reverse) mode, fp32 output (``:172``).
    g: ``[Ttot, HV]`` -> ``[Ttot, HV]``.
    """
    out = np.zeros(g.shape, dtype=dtype)
    for bos, eos in bounds:
        for s, e in _chunks(bos, eos, bt):
            out[s:e] = np.cumsum(g[s:e].astype(dtype), axis=0)
    return out


def chunk_scaled_dot_kkt(k, beta, gc, bounds, G, bt=BT, dtype=np.float64):
    """A[t, hv, j] = beta_t * exp(G_t - G_j) * <k_t, k_j> for j < t in the chunk.

    ``tmo_chunk_scaled_dot_kkt_fwd_kernel`` (``triton/fla/chunk_scaled_dot_kkt.py:25-100``),
    restated with the q/k head of v-head hv being ``hv // G`` as in
    ``wy_fast.py:101``.  (The reference kernel offsets k by the v-head index,
    ``chunk_scaled_dot_kkt.py:83``, which only agrees when H == HV.)
    k: ``[Ttot, H, K]``; beta, gc: ``[Ttot, HV]`` -> A ``[Ttot, HV, bt]``.
    """
    Ttot, HV = beta.shape
    A = np.zeros((Ttot, HV, bt), dtype=dtype)
    kh = k[:, np.arange(HV) // G].astype(dtype)  # [Ttot, HV, K]
    for bos, eos in bounds:
        for s, e in _chunks(bos, eos, bt):
            L = e - s
            kc = kh[s:e].transpose(1, 0, 2)  # [HV, L, K]
            kk = kc @ kc.transpose(0, 2, 1)  # [HV, L, L]
            gcc = gc[s:e].T  # [HV, L]
            dec = np.exp(gcc[:, :, None] - gcc[:, None, :])
            a = beta[s:e].T[:, :, None].astype(dtype) * dec * kk
            a = np.tril(a, -1)
            A[s:e, :, :L] = a.transpose(1, 0, 2)
    return A


def solve_tril(A, bounds, bt=BT, dtype=np.float64):
    """(I + A)^-1 for each strictly lower-triangular chunk block.

    Semantics of ``solve_tril`` (``triton/fla/solve_tril.py:491-537``, native
    op declared at ``include/torch_mlu_ops.h:1052-1054``); solved here by
    forward substitution in ``dtype``.
    """
    Ai = np.zeros(A.shape, dtype=dtype)
    for bos, eos in bounds:
        for s, e in _chunks(bos, eos, bt):
            L = e - s
            a = A[s:e, :, :L].transpose(1, 0, 2).astype(dtype)  # [HV, L, L]
            eye = np.broadcast_to(np.eye(L, dtype=dtype), a.shape)
            Ai[s:e, :, :L] = np.linalg.solve(eye + a, eye).transpose(1, 0, 2)
    return Ai


def recompute_w_u(k, v, beta, gc, Ai, bounds, G, bt=BT, dtype=np.float64):
    """u = Ai diag(beta) v and w = Ai diag(beta exp(G)) k per chunk.

    ``tmo_recompute_w_u_fwd_kernel`` (``triton/fla/wy_fast.py:18-119``):
    ``b_Ab = b_A * b_beta`` then ``dot(b_Ab, b_v)`` (``:95-97``) and
    ``b_Abg = b_A * b_beta * exp(g)`` then ``dot(b_Abg, b_k)`` (``:116-119``).
    """
    Ttot, HV = beta.shape
    K = k.shape[-1]
    V = v.shape[-1]
    w = np.zeros((Ttot, HV, K), dtype=dtype)
    u = np.zeros((Ttot, HV, V), dtype=dtype)
    kh = k[:, np.arange(HV) // G].astype(dtype)
    for bos, eos in bounds:
        for s, e in _chunks(bos, eos, bt):
            L = e - s
            a = Ai[s:e, :, :L].transpose(1, 0, 2).astype(dtype)  # [HV, L, L]
            b = beta[s:e].T.astype(dtype)  # [HV, L]
            eg = np.exp(gc[s:e].T)
            u[s:e] = ((a * b[:, None, :]) @ v[s:e].transpose(1, 0, 2).astype(dtype)).transpose(1, 0, 2)
            w[s:e] = ((a * (b * eg)[:, None, :]) @ kh[s:e].transpose(1, 0, 2)).transpose(1, 0, 2)
    return w, u


def chunk_fwd_h(k, w, u, gc, bounds, G, initial_state=None, output_final_state=False,
                bt=BT, dtype=np.float64):
    """Inter-chunk state recurrence (K-first state).

    ``tmo_chunk_gated_delta_rule_fwd_kernel_h_blockdim64``
    (``triton/fla/chunk_delta_h.py:28-197``): for each chunk store h_c
    (``:107-116``), v_new = u - w h_c (``:118-130``), then
    h <- exp(G_last) h + k^T (exp(G_last - G) * v_new) (``:137-190``).
    Returns per-chunk states ``[(n, c) -> [HV, K, V]]`` as a list per
    sequence, v_new ``[Ttot, HV, V]`` and the final states ``[N, HV, K, V]``.
    """
    Ttot, HV, K = w.shape
    V = u.shape[-1]
    kh = k[:, np.arange(HV) // G].astype(dtype)
    v_new = np.zeros((Ttot, HV, V), dtype=dtype)
    hs = []
    ht = np.zeros((len(bounds), HV, K, V), dtype=dtype) if output_final_state else None
    for n, (bos, eos) in enumerate(bounds):
        S = np.zeros((HV, K, V), dtype=dtype)
        if initial_state is not None:
            S += np.asarray(initial_state[n], dtype=dtype)
        hn = []
        for s, e in _chunks(bos, eos, bt):
            hn.append(S.copy())
            wc = w[s:e].transpose(1, 0, 2)  # [HV, L, K]
            vn = u[s:e].transpose(1, 0, 2) - wc @ S  # [HV, L, V]
            v_new[s:e] = vn.transpose(1, 0, 2)
            gcc = gc[s:e].T  # [HV, L]
            glast = gcc[:, -1]
            vd = vn * np.exp(glast[:, None] - gcc)[:, :, None]
            S = S * np.exp(glast)[:, None, None] + kh[s:e].transpose(1, 2, 0) @ vd
        hs.append(hn)
        if output_final_state:
            ht[n] = S
    return hs, v_new, ht


def chunk_fwd_o(q, k, v_new, hs, gc, bounds, G, scale, bt=BT, dtype=np.float64):
    """o = scale * (exp(G) * (q h_c) + tril_incl(exp(G_i - G_j) q k^T) v_new).

    ``tmo_chunk_fwd_kernel_o`` (``triton/fla/chunk_o.py:30-170``), K-first h.
    """
    Ttot, HV, V = v_new.shape
    o = np.zeros((Ttot, HV, V), dtype=dtype)
    qh = q[:, np.arange(HV) // G].astype(dtype)
    kh = k[:, np.arange(HV) // G].astype(dtype)
    for n, (bos, eos) in enumerate(bounds):
        for c, (s, e) in enumerate(_chunks(bos, eos, bt)):
            qc = qh[s:e].transpose(1, 0, 2)  # [HV, L, K]
            kc = kh[s:e].transpose(1, 0, 2)
            gcc = gc[s:e].T  # [HV, L]
            inter = (qc @ hs[n][c]) * np.exp(gcc)[:, :, None]
            att = (qc @ kc.transpose(0, 2, 1)) * np.exp(gcc[:, :, None] - gcc[:, None, :])
            att = np.tril(att)
            o[s:e] = (scale * (inter + att @ v_new[s:e].transpose(1, 0, 2))).transpose(1, 0, 2)
    return o


def chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None,
                           output_final_state=False, cu_seqlens=None,
                           use_qk_l2norm_in_kernel=False, state_v_first=False,
                           bt=BT, dtype=np.float64, return_stages=False):
    """Chunked prefill, the composition in ``chunk_gated_delta_rule_fwd``
    (``triton/fla/chunk.py:10-74``) behind ``triton_ops.chunk_gated_delta_rule``
    (``triton_ops.py:81-165``).  ``scale`` defaults to K^-0.5
    (``chunk_o.py:194-195``).  ``use_qk_l2norm_in_kernel`` normalises q and k
    first with the recurrent kernels' formula.  With ``state_v_first`` the
    initial and final states are ``[N, HV, V, K]`` (``chunk_delta_h.py:235-242``).
    Returns ``(o [B,T,HV,V], final_state or None)``.
    """
    B, T, H, K = k.shape
    HV = v.shape[2]
    G = HV // H
    if scale is None:
        scale = K ** -0.5
    qf, kf, vf = (_flat(x).astype(dtype) for x in (q, k, v))
    if use_qk_l2norm_in_kernel:
        qf, kf = l2norm(qf), l2norm(kf)
    gf, bf = _flat(g).astype(dtype), _flat(beta).astype(dtype)
    bounds = seq_bounds(B, T, cu_seqlens)
    h0 = None
    if initial_state is not None:
        h0 = np.asarray(initial_state, dtype=dtype)
        if state_v_first:
            h0 = h0.transpose(0, 1, 3, 2)
    gc = chunk_local_cumsum(gf, bounds, bt, dtype)
    A = chunk_scaled_dot_kkt(kf, bf, gc, bounds, G, bt, dtype)
    Ai = solve_tril(A, bounds, bt, dtype)
    w, u = recompute_w_u(kf, vf, bf, gc, Ai, bounds, G, bt, dtype)
    hs, v_new, ht = chunk_fwd_h(kf, w, u, gc, bounds, G, h0, output_final_state, bt, dtype)
    o = chunk_fwd_o(qf, kf, v_new, hs, gc, bounds, G, scale, bt, dtype)
    if ht is not None and state_v_first:
        ht = ht.transpose(0, 1, 3, 2).copy()
    o = o.reshape(v.shape)
    if return_stages:
        return o, ht, dict(gc=gc, A=A, Ai=Ai, w=w, u=u, hs=hs, v_new=v_new)
    return o, ht


def chunk_fwd_h_stage(k, w, u, g=None, gk=None, initial_state=None, output_final_state=False,
                      state_v_first=False, cu_seqlens=None, bt=BT, dtype=np.float64):
    """The state-recurrence stage with the reference's own layouts, including
    its per-key decay branch: ``chunk_gated_delta_rule_fwd_h``
    (``triton/fla/chunk_delta_h.py:200-271``, kernel ``:28-197``).

    k ``[B, T, Hg, K]``, w ``[B, T, H, K]``, u ``[B, T, H, V]``; g the
    chunk-local cumsum in head-major ``[H, B*T]`` layout (``:133-134``) or
    None; gk the per-key cumsum ``[B, T, H, K]`` (``:155-171``) or None.
    Per chunk: h = S (``:107-116``), v_new = u - w S (``:118-130``),
    S <- S exp(g_last) exp(gk_last)[:, None] + k^T (v_new exp(g_last - g))
    (``:131-190``; K-first S).  Returns (h ``[B, NT, H, K, V]`` or V-first,
    v_new, final_state or None).
    """
    B, T, Hg, K = k.shape
    H, V = u.shape[2], u.shape[3]
    G = H // Hg
    kf, wf, uf = (_flat(x).astype(dtype) for x in (k, w, u))
    gf = None if g is None else np.asarray(g, dtype=dtype).reshape(H, B * T)
    gkf = None if gk is None else _flat(gk).astype(dtype)
    bounds = seq_bounds(B, T, cu_seqlens)
    nts = [(e - s + bt - 1) // bt for s, e in bounds]
    NT = sum(nts) if cu_seqlens is not None else (T + bt - 1) // bt
    hs = np.zeros((B * NT if cu_seqlens is None else NT, H, K, V), dtype=dtype)
    v_new = np.zeros(uf.shape, dtype=dtype)
    ht = np.zeros((len(bounds), H, K, V), dtype=dtype) if output_final_state else None
    boh = 0
    for n, (bos, eos) in enumerate(bounds):
        S = np.zeros((H, K, V), dtype=dtype)
        if initial_state is not None:
            h0 = np.asarray(initial_state[n], dtype=dtype)
            S += h0.transpose(0, 2, 1) if state_v_first else h0
        base = boh if cu_seqlens is not None else n * NT
        for c, (s, e) in enumerate(_chunks(bos, eos, bt)):
            hs[base + c] = S
            wc = wf[s:e].transpose(1, 0, 2)                       # [H, L, K]
            vn = uf[s:e].transpose(1, 0, 2) - wc @ S              # [H, L, V]
            v_new[s:e] = vn.transpose(1, 0, 2)
            dec = np.ones((H, K, 1), dtype=dtype)
            if gf is not None:
                glast = gf[:, e - 1]
                vn = vn * np.exp(glast[:, None] - gf[:, s:e])[:, :, None]
                dec = dec * np.exp(glast)[:, None, None]
            if gkf is not None:
                dec = dec * np.exp(gkf[e - 1])[:, :, None]          # [H, K, 1]
            kc = kf[s:e][:, np.arange(H) // G].transpose(1, 2, 0)  # [H, K, L]
            S = S * dec + kc @ vn
        boh += nts[n]
        if output_final_state:
            ht[n] = S
    h = hs.reshape((B, NT, H, K, V) if cu_seqlens is None else (1, NT, H, K, V))
    if state_v_first:
        h = h.transpose(0, 1, 2, 4, 3).copy()
        if ht is not None:
            ht = ht.transpose(0, 1, 3, 2).copy()
    return h, v_new.reshape(u.shape), ht
