"""Public gated delta-rule (GDN) ops, drop-in for ``torch_mlu_ops.triton_ops``.

Same names, argument order, keyword names, defaults and return values as the
reference facade (``triton_ops.py:81-285``); the work runs in
``libgdn_b200.so`` (hand-written sm_100a CUDA) through its C ABI.  There is no
CPU or Triton path: the ops raise if the tensors are not on a CUDA device or
the library is not built.

Differences from the reference, all supersets:

* ``chunk_gated_delta_rule`` takes ``use_qk_l2norm_in_kernel`` (q and k are
  divided by ``sqrt(sum(x^2) + 1e-6)``, the formula of
  ``triton/fla/fused_recurrent_fn.py:110-112``).
* ``allow_tf32`` is accepted and ignored: fp32 inputs always take the
  full-precision fp32 path; bf16/fp16 inputs take the tensor-core path with
  fp32 accumulation.
* ``scale=None`` selects ``K ** -0.5`` in every op (the recurrent reference
  kernels would fail on ``None``).
* ``fused_recurrent_gated_delta_rule`` also accepts ``ssm_state_indices``,
  ``inplace_final_state`` and ``num_accepted_tokens``; with
  ``ssm_state_indices`` it runs the slot-indexed decode of
  ``fused_recurrent_gated_delta_rule_fn``.
* Outputs of PAD sequences (negative initial slot index) are zero instead of
  left unwritten.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_DT = {torch.float32: _lib.GDN_F32, torch.bfloat16: _lib.GDN_BF16, torch.float16: _lib.GDN_F16}
_IDT = {torch.int32: _lib.GDN_I32, torch.int64: _lib.GDN_I64}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _cuda(name, *ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{name}: every tensor must be on a CUDA device (got {t.device})")


def _qkv_dtype(q, k, v):
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError(f"q, k, v must share a dtype (got {q.dtype}, {k.dtype}, {v.dtype})")
    if q.dtype not in _DT:
        raise ValueError(f"unsupported dtype {q.dtype}: expected float32, bfloat16 or float16")
    return _DT[q.dtype]


def _f32(t):
    return None if t is None else t.to(torch.float32).contiguous()


def _idx(t):
    if t is None:
        return None, _lib.GDN_I64
    if t.dtype not in _IDT:
        t = t.to(torch.int64)
    return t, _IDT[t.dtype]


def _check_shapes(q, k, v):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k must be [B, T, H, K] and v must be [B, T, HV, V]")
    if q.shape != k.shape:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} must have the same shape")
    if v.shape[:2] != k.shape[:2]:
        raise ValueError(f"v {tuple(v.shape)} must match k {tuple(k.shape)} in [B, T]")
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    if HV % H != 0:
        raise ValueError(f"HV={HV} must be a multiple of H={H}")
    return B, T, H, HV, K, V


# ---------------------------------------------------------------------------
# chunked prefill
# ---------------------------------------------------------------------------

def _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens, state_v_first):
    B, T, H, HV, K, V = _check_shapes(q, k, v)
    if K > 128 or V > 128:
        raise ValueError(f"K={K}, V={V}: both must be <= 128 (triton/fla/chunk.py:27-28)")
    if g.shape != v.shape[:3] or beta.shape != v.shape[:3]:
        raise ValueError(f"g {tuple(g.shape)} and beta {tuple(beta.shape)} must be [B, T, HV]")
    if cu_seqlens is not None and B != 1:
        raise ValueError("cu_seqlens requires batch size 1 (packed sequences)")
    qkv = _qkv_dtype(q, k, v)
    cu, cu_dt = _idx(cu_seqlens)
    N = B if cu is None else cu.numel() - 1
    shape_state = (N, HV, V, K) if state_v_first else (N, HV, K, V)
    if initial_state is not None and tuple(initial_state.shape) != shape_state:
        raise ValueError(f"initial_state must be {shape_state}, got {tuple(initial_state.shape)}")
    return (B, T, N, H, HV, K, V), qkv, cu, cu_dt, shape_state


def _chunk_fwd(q, k, v, g, beta, scale, h0, output_final_state, cu, cu_dt, dims, qkv, shape_state,
               state_v_first, use_qk_l2norm, force_generic):
    B, T, N, H, HV, K, V = dims
    dev = q.device
    o = torch.empty_like(v, dtype=q.dtype)
    ht = torch.empty(shape_state, dtype=torch.float32, device=dev) if output_final_state else None
    args = _lib.ChunkArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), beta=_ptr(beta),
        initial_state=_ptr(h0), o=_ptr(o), final_state=_ptr(ht), cu_seqlens=_ptr(cu),
        workspace=None, workspace_bytes=0, B=B, T=T, N=N, H=H, HV=HV, K=K, V=V,
        qkv_dtype=qkv, cu_dtype=cu_dt, scale=float(scale) if scale is not None else 0.0,
        use_qk_l2norm=int(bool(use_qk_l2norm)), state_v_first=int(bool(state_v_first)),
        force_generic=int(bool(force_generic)))
    lib = _lib.load()
    nbytes = lib.gdn_chunk_workspace_size(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(_lib.GDN_ERR_INVALID)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    args.workspace = ctypes.c_void_p(ws.data_ptr())
    args.workspace_bytes = nbytes
    with torch.cuda.device(dev):
        _lib.check(lib.gdn_chunk_fwd(ctypes.byref(args), _stream(dev)))
    return o, ht


def _chunk_bwd(q, k, v, g, beta, scale, h0, cu, cu_dt, dims, qkv, shape_state, state_v_first,
               use_qk_l2norm, do, dht):
    B, T, N, H, HV, K, V = dims
    dev = q.device
    do = do.to(q.dtype).contiguous()
    dht = None if dht is None else dht.to(torch.float32).contiguous()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(v.shape[:3], dtype=torch.float32, device=dev)
    db = torch.empty(v.shape[:3], dtype=torch.float32, device=dev)
    dh0 = torch.empty(shape_state, dtype=torch.float32, device=dev) if h0 is not None else None
    args = _lib.ChunkBwdArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), beta=_ptr(beta), initial_state=_ptr(h0),
        cu_seqlens=_ptr(cu), dout=_ptr(do), dht=_ptr(dht), dq=_ptr(dq), dk=_ptr(dk), dv=_ptr(dv),
        dg=_ptr(dg), dbeta=_ptr(db), dh0=_ptr(dh0), workspace=None, workspace_bytes=0,
        B=B, T=T, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=qkv, cu_dtype=cu_dt,
        scale=float(scale) if scale is not None else 0.0,
        use_qk_l2norm=int(bool(use_qk_l2norm)), state_v_first=int(bool(state_v_first)))
    lib = _lib.load()
    nbytes = lib.gdn_chunk_bwd_workspace_size(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(_lib.GDN_ERR_INVALID)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    args.workspace = ctypes.c_void_p(ws.data_ptr())
    args.workspace_bytes = nbytes
    with torch.cuda.device(dev):
        _lib.check(lib.gdn_chunk_bwd(ctypes.byref(args), _stream(dev)))
    return dq, dk, dv, dg, db, dh0


class ChunkGatedDeltaRuleFunction(torch.autograd.Function):
    """Autograd node of the chunked forward (``triton/fla/chunk.py:188-251``):
    the forward saves its inputs only and the backward recomputes the
    intermediates (``chunk.py:76-186``) inside ``gdn_chunk_bwd``."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens,
                state_v_first, use_qk_l2norm, force_generic):
        dims, qkv, cu, cu_dt, shape_state = _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens,
                                                           state_v_first)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        g32, b32, h0 = _f32(g), _f32(beta), _f32(initial_state)
        o, ht = _chunk_fwd(q, k, v, g32, b32, scale, h0, output_final_state, cu, cu_dt, dims, qkv,
                           shape_state, state_v_first, use_qk_l2norm, force_generic)
        ctx.save_for_backward(q, k, v, g32, b32, h0, cu)
        ctx.meta = (scale, cu_dt, dims, qkv, shape_state, state_v_first, use_qk_l2norm,
                    g.dtype, beta.dtype, None if initial_state is None else initial_state.dtype)
        return o, ht

    @staticmethod
    def backward(ctx, do, dht):
        q, k, v, g32, b32, h0, cu = ctx.saved_tensors
        scale, cu_dt, dims, qkv, shape_state, svf, l2, g_dt, b_dt, h0_dt = ctx.meta
        if do is None:
            do = torch.zeros_like(v, dtype=q.dtype)
        dq, dk, dv, dg, db, dh0 = _chunk_bwd(q, k, v, g32, b32, scale, h0, cu, cu_dt, dims, qkv,
                                             shape_state, svf, l2, do, dht)
        if dh0 is not None:
            dh0 = dh0.to(h0_dt)
        return (dq, dk, dv, dg.to(g_dt), db.to(b_dt), None, dh0, None, None, None, None, None)


def chunk_gated_delta_rule(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    scale: float | None = None,
    initial_state: torch.Tensor = None,
    output_final_state: bool = False,
    cu_seqlens: torch.LongTensor | None = None,
    chunk_indices: torch.Tensor | None = None,
    chunk_offsets: torch.Tensor | None = None,
    allow_tf32: bool = True,
    state_v_first: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    *,
    force_generic: bool = False,
):
    """Chunked gated delta-rule forward (``triton_ops.py:81-165``).

    q, k ``[B, T, H, K]``; v ``[B, T, HV, V]``; g, beta ``[B, T, HV]``;
    initial_state ``[N, HV, K, V]`` (``[N, HV, V, K]`` with ``state_v_first``).
    Returns ``(o [B, T, HV, V] in q.dtype, final_state fp32 or None)``.
    ``chunk_indices`` / ``chunk_offsets`` are accepted for signature
    compatibility; the chunk table is built on the device from ``cu_seqlens``.

    Differentiable like the reference (``ChunkGatedDeltaRuleFunction``,
    ``triton/fla/chunk.py:188-251``): when grad mode is on and an input
    requires grad, the backward (``gdn_chunk_bwd``) gives dq, dk, dv, dg,
    dbeta and d(initial_state).
    """
    del chunk_indices, chunk_offsets, allow_tf32
    _cuda("chunk_gated_delta_rule", q, k, v, g, beta, initial_state, cu_seqlens)
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (q, k, v, g, beta, initial_state)):
        return ChunkGatedDeltaRuleFunction.apply(
            q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, state_v_first,
            use_qk_l2norm_in_kernel, force_generic)
    dims, qkv, cu, cu_dt, shape_state = _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens,
                                                       state_v_first)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    return _chunk_fwd(q, k, v, _f32(g), _f32(beta), scale, _f32(initial_state), output_final_state, cu,
                      cu_dt, dims, qkv, shape_state, state_v_first, use_qk_l2norm_in_kernel, force_generic)


def chunk_gated_delta_rule_from_host(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    scale: float | None = None,
    initial_state: torch.Tensor = None,
    output_final_state: bool = False,
    cu_seqlens: torch.LongTensor | None = None,
    state_v_first: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    *,
    device=None,
    segment_tokens: int = 2048,
    o_out: torch.Tensor | None = None,
    final_state_out: torch.Tensor | None = None,
    force_generic: bool = False,
):
    """:func:`chunk_gated_delta_rule` for inputs that live in host memory
    (``gdn_chunk_fwd_host``).

    Same arguments and results as the device op, but every tensor is a CPU
    tensor.  The tokens go to the GPU in pieces of about ``segment_tokens``
    tokens (a multiple of 64) while earlier pieces compute and their outputs
    come back, so the host link, not the kernels, sets the time; the results
    are those of the device op.  2048 was the fastest piece size at the
    config-1 shape on a B200 (512: +8 %, 1024: +1.5 %, 4096: +4 %).  Page-locked (pinned) inputs give overlapped
    copies; other host memory is pinned first.

    Returns ``(o, final_state)`` as pinned CPU tensors (``o_out`` /
    ``final_state_out`` when given: contiguous pinned tensors of the output
    shapes, which spares pinning fresh host memory on every call).  They are
    written by asynchronous copies that the current stream of ``device``
    waits for: synchronise that stream (or the device) before reading them,
    and keep the inputs unchanged until then.
    """
    for t in (q, k, v, g, beta, initial_state, cu_seqlens, o_out, final_state_out):
        if t is not None and t.is_cuda:
            raise ValueError("chunk_gated_delta_rule_from_host takes host (CPU) tensors")
    if segment_tokens <= 0 or segment_tokens % 64:
        raise ValueError(f"segment_tokens={segment_tokens} must be a positive multiple of 64")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    dims, qkv, _, _, shape_state = _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens, state_v_first)
    B, T, N, H, HV, K, V = dims
    staged = []  # host temporaries (conversions, pinning) the copies read

    def host_in(t, dtype=None):
        if t is None:
            return None
        x = t if dtype is None else t.to(dtype)
        x = x.contiguous()
        if not x.is_pinned():
            x = x.pin_memory()
        if x is not t:
            staged.append(x)
        return x

    def host_out(t, shape, dtype, name):
        if t is None:
            return torch.empty(shape, dtype=dtype, pin_memory=True)
        if tuple(t.shape) != tuple(shape) or t.dtype != dtype or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous host tensor of shape {tuple(shape)} and dtype {dtype}")
        return t

    qh, kh, vh = host_in(q), host_in(k), host_in(v)
    gh, bh = host_in(g, torch.float32), host_in(beta, torch.float32)
    h0h = host_in(initial_state, torch.float32)
    cuh, cu_dt = _idx(None if cu_seqlens is None else cu_seqlens.contiguous())
    o_h = host_out(o_out, (B, T, HV, V), q.dtype, "o_out")
    ht_h = host_out(final_state_out, shape_state, torch.float32, "final_state_out") if output_final_state else None
    args = _lib.ChunkArgs(
        q=_ptr(qh), k=_ptr(kh), v=_ptr(vh), g=_ptr(gh), beta=_ptr(bh),
        initial_state=_ptr(h0h), o=_ptr(o_h), final_state=_ptr(ht_h), cu_seqlens=_ptr(cuh),
        workspace=None, workspace_bytes=0, B=B, T=T, N=N, H=H, HV=HV, K=K, V=V,
        qkv_dtype=qkv, cu_dtype=cu_dt, scale=float(scale) if scale is not None else 0.0,
        use_qk_l2norm=int(bool(use_qk_l2norm_in_kernel)), state_v_first=int(bool(state_v_first)),
        force_generic=int(bool(force_generic)))
    lib = _lib.load()
    nbytes = lib.gdn_chunk_fwd_host_buffer_size(ctypes.byref(args), segment_tokens)
    if nbytes == 0:
        _lib.check(_lib.GDN_ERR_INVALID)
    with torch.cuda.device(dev):
        buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        args.workspace = ctypes.c_void_p(buf.data_ptr())
        args.workspace_bytes = nbytes
        _lib.check(lib.gdn_chunk_fwd_host(ctypes.byref(args), segment_tokens, _stream(dev)))
        if staged:  # the temporaries must outlive the copies that read them
            torch.cuda.current_stream(dev).synchronize()
    return o_h, ht_h


def chunk_gated_delta_rule_bwd(q, k, v, g, beta, scale, initial_state, dout, dht,
                               cu_seqlens=None, state_v_first=False, use_qk_l2norm_in_kernel=False):
    """Backward of :func:`chunk_gated_delta_rule` as a plain call
    (``triton/fla/chunk.py:76-186``, minus the saved ``A``, which is
    recomputed).  Returns ``(dq, dk, dv, db, dg, dh0)`` in the reference's
    order; dq, dk, dv in q's dtype, db and dg fp32, dh0 fp32 or None."""
    _cuda("chunk_gated_delta_rule_bwd", q, k, v, g, beta, initial_state, dout, dht, cu_seqlens)
    dims, qkv, cu, cu_dt, shape_state = _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens,
                                                       state_v_first)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    dq, dk, dv, dg, db, dh0 = _chunk_bwd(q, k, v, _f32(g), _f32(beta), scale, _f32(initial_state), cu,
                                         cu_dt, dims, qkv, shape_state, state_v_first,
                                         use_qk_l2norm_in_kernel, dout, dht)
    return dq, dk, dv, db, dg, dh0


# ---------------------------------------------------------------------------
# recurrent forms
# ---------------------------------------------------------------------------

def fused_recurrent_gated_delta_rule_fn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor | None = None,
    beta: torch.Tensor | None = None,
    scale: float = None,
    initial_state: torch.Tensor = None,
    inplace_final_state: bool = True,
    cu_seqlens: torch.LongTensor | None = None,
    ssm_state_indices: torch.Tensor = None,
    num_accepted_tokens: torch.Tensor = None,
    use_qk_l2norm_in_kernel: bool = False,
):
    """Slot-indexed recurrent decode (``triton_ops.py:228-285`` ->
    ``triton/fla/fused_recurrent_fn.py:161-233``).

    The state cache is V-first ``[slots, HV, V, K]`` fp32 (the kernel's
    layout, ``fused_recurrent_fn.py:101-104``).  With
    ``inplace_final_state=True`` the cache is updated in place at
    ``ssm_state_indices[n, t]`` and returned; otherwise a fresh
    ``[B*T, HV, V, K]`` tensor receives the state after every token.
    """
    _cuda("fused_recurrent_gated_delta_rule_fn", q, k, v, g, beta, initial_state, cu_seqlens,
          ssm_state_indices, num_accepted_tokens)
    B, T, H, HV, K, V = _check_shapes(q, k, v)
    if K > 128 or V > 128:
        raise ValueError(f"K={K}, V={V}: both must be <= 128 (fused_recurrent_fn.py:181-182)")
    if cu_seqlens is not None and B != 1:
        raise ValueError("cu_seqlens requires batch size 1 (packed sequences)")
    qkv = _qkv_dtype(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if beta is None:
        beta = torch.ones(v.shape[:3], dtype=torch.float32, device=v.device)
    beta_per_v = beta.dim() == v.dim()
    g, beta = _f32(g), _f32(beta)
    cu, cu_dt = _idx(cu_seqlens)
    N = B if cu is None else cu.numel() - 1
    idx, idx_dt = _idx(ssm_state_indices)
    nacc, nacc_dt = _idx(num_accepted_tokens)
    if scale is None:
        scale = K ** -0.5
    if initial_state is not None:
        if initial_state.dtype != torch.float32:
            raise ValueError("initial_state must be float32")
        if initial_state.dim() != 4 or tuple(initial_state.shape[1:]) != (HV, V, K):
            raise ValueError(f"initial_state must be [slots, {HV}, {V}, {K}] (V-first), "
                             f"got {tuple(initial_state.shape)}")
        if initial_state.stride()[1:] != (V * K, K, 1):
            raise ValueError("initial_state rows must be contiguous [HV, V, K] blocks")
    if inplace_final_state:
        if initial_state is None or idx is None:
            raise ValueError("inplace_final_state=True needs initial_state and ssm_state_indices")
        final_state = initial_state
    else:
        final_state = torch.empty(B * T, HV, V, K, dtype=torch.float32, device=q.device)
    if idx is None:
        s_seq, s_tok = 1, 1
    elif idx.dim() == 1:
        s_seq, s_tok = idx.stride(0), 1
    else:
        s_seq, s_tok = idx.stride()
    o = torch.empty_like(v)
    args = _lib.RecurrentArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), beta=_ptr(beta),
        initial_state=_ptr(initial_state), o=_ptr(o), final_state=_ptr(final_state),
        cu_seqlens=_ptr(cu), ssm_state_indices=_ptr(idx), num_accepted_tokens=_ptr(nacc),
        B=B, T=T, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=qkv, cu_dtype=cu_dt,
        idx_dtype=idx_dt, nacc_dtype=nacc_dt,
        stride_init_state_token=initial_state.stride(0) if initial_state is not None else 0,
        stride_final_state_token=final_state.stride(0),
        stride_indices_seq=s_seq, stride_indices_tok=s_tok, scale=float(scale),
        use_qk_l2norm=int(bool(use_qk_l2norm_in_kernel)), beta_per_v=int(beta_per_v),
        inplace_final_state=int(bool(inplace_final_state)))
    dev = q.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().gdn_fused_recurrent_fwd(ctypes.byref(args), _stream(dev)))
    return o, final_state


def fused_recurrent_gated_delta_rule(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor | None = None,
    gk: torch.Tensor | None = None,
    gv: torch.Tensor | None = None,
    beta: torch.Tensor | None = None,
    scale: float = None,
    initial_state: torch.Tensor = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    cu_seqlens: torch.LongTensor | None = None,
    *,
    ssm_state_indices: torch.Tensor | None = None,
    inplace_final_state: bool = True,
    num_accepted_tokens: torch.Tensor | None = None,
):
    """Recurrent gated delta rule (``triton_ops.py:168-226`` ->
    ``triton/fla/fused_recurrent.py:134-187``): K-first state
    ``[N, HV, K, V]``, optional per-channel decays ``gk`` / ``gv``.

    Given ``ssm_state_indices`` it is the slot-indexed decode of
    :func:`fused_recurrent_gated_delta_rule_fn` on a V-first cache instead.
    """
    if ssm_state_indices is not None:
        if gk is not None or gv is not None:
            raise ValueError("gk/gv are not supported with ssm_state_indices")
        return fused_recurrent_gated_delta_rule_fn(
            q, k, v, g, beta, scale, initial_state, inplace_final_state, cu_seqlens,
            ssm_state_indices, num_accepted_tokens, use_qk_l2norm_in_kernel)
    _cuda("fused_recurrent_gated_delta_rule", q, k, v, g, gk, gv, beta, initial_state, cu_seqlens)
    B, T, H, HV, K, V = _check_shapes(q, k, v)
    if K > 128 or V > 128:
        raise ValueError(f"K={K}, V={V}: both must be <= 128 (fused_recurrent.py:155-156)")
    if cu_seqlens is not None and B != 1:
        raise ValueError("cu_seqlens requires batch size 1 (packed sequences)")
    qkv = _qkv_dtype(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if beta is None:
        beta = torch.ones(v.shape[:3], dtype=torch.float32, device=v.device)
    beta_per_v = beta.dim() == v.dim()
    g, gk, gv, beta = _f32(g), _f32(gk), _f32(gv), _f32(beta)
    cu, cu_dt = _idx(cu_seqlens)
    N = B if cu is None else cu.numel() - 1
    h0 = None
    if initial_state is not None:
        if tuple(initial_state.shape) != (N, HV, K, V):
            raise ValueError(f"initial_state must be {(N, HV, K, V)}, got {tuple(initial_state.shape)}")
        h0 = _f32(initial_state)
    o = torch.empty_like(v)
    ht = torch.empty(N, HV, K, V, dtype=torch.float32, device=q.device) if output_final_state else None
    args = _lib.RecurrentPlainArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), gk=_ptr(gk), gv=_ptr(gv), beta=_ptr(beta),
        initial_state=_ptr(h0), o=_ptr(o), final_state=_ptr(ht), cu_seqlens=_ptr(cu),
        B=B, T=T, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=qkv, cu_dtype=cu_dt,
        scale=float(scale) if scale is not None else 0.0,
        use_qk_l2norm=int(bool(use_qk_l2norm_in_kernel)), beta_per_v=int(beta_per_v))
    dev = q.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().gdn_recurrent_plain_fwd(ctypes.byref(args), _stream(dev)))
    return o, ht


def solve_tril(input: torch.Tensor, output: torch.Tensor = None, cu_seqlens: torch.Tensor = None,
               out_dtype: torch.dtype = torch.float):
    """(I + input)^-1 per chunk block (``_ops.py:6232-6257``; native op
    ``include/torch_mlu_ops.h:1052-1054``).  input fp32 ``[B, T, H, BT]``,
    BT in {16, 32, 64}; output bf16/fp16/fp32 of the same shape."""
    _cuda("solve_tril", input, output, cu_seqlens)
    if input.dtype != torch.float32 or input.dim() != 4:
        raise ValueError("input must be a float32 [B, T, H, BT] tensor")
    if output is None:
        output = torch.empty(input.shape, device=input.device, dtype=out_dtype)
    if output.shape != input.shape or output.dtype not in _DT:
        raise ValueError("output must match input's shape with dtype float32/bfloat16/float16")
    B, T, H, BT = input.shape
    x = input.contiguous()
    out = output if output.is_contiguous() else torch.empty_like(output)
    cu, cu_dt = _idx(cu_seqlens)
    N = B if cu is None else cu.numel() - 1
    dev = input.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().gdn_solve_tril(
            _ptr(x), _ptr(out), _DT[out.dtype], _ptr(cu), cu_dt, N, B, T, H, BT, _stream(dev)))
    if out is not output:
        output.copy_(out)
    return output
