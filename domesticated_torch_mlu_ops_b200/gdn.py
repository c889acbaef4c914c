"""Public gated delta-rule (GDN) ops, drop-in for ``torch_mlu_ops.triton_ops``.

Same names, argument order, keyword names, defaults and return values as the
reference facade (``triton_ops.py:81-285``); the work runs in
``libgdn_b200.so`` (hand-written sm_100a CUDA) through its C ABI.  There is no
CPU or Triton path: the ops raise if the tensors are not on a CUDA device or
the library is not built.

Every op is a ``torch.library`` custom op in the ``gdn_b200`` namespace with a
fake (meta) implementation, as the reference registers its native ops with
fakes (``abstract.py:1393-1399``): ``torch.compile`` traces through the public
functions without a graph break and FakeTensor mode gets output shapes and
dtypes without touching the GPU.  The ops are ``gdn_b200::chunk_fwd`` /
``chunk_bwd`` (prefill and its backward), ``recurrent_fn_inplace`` (decode
that updates the slot cache in place; it declares the cache as mutated),
``recurrent_fn`` (decode with per-token states out), ``recurrent_plain`` and
``solve_tril`` (which mutates ``output``, like the reference's native op).

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
* ``fused_recurrent_gated_delta_rule_fn`` accepts a per-key gate ``g`` of
  shape ``[B, T, HV, K]``: the KDA form of the reference kernel
  (``IS_KDA``, ``fused_recurrent_fn.py:77-80,115-120``), which its facade
  never enables.
* Outputs of PAD sequences (negative initial slot index) are zero instead of
  left unwritten.  A slot index at or past the cache's first dimension is
  treated like PAD and reported (the reference would read out of bounds).
* ``check_errors=True`` (keyword) synchronises after the call and raises
  :class:`GdnError` if a kernel recorded a failure (a bounded wait that gave
  up, or a slot index out of range).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DT = {torch.float32: _lib.GDN_F32, torch.bfloat16: _lib.GDN_BF16, torch.float16: _lib.GDN_F16}
_IDT = {torch.int32: _lib.GDN_I32, torch.int64: _lib.GDN_I64}
Tensor = torch.Tensor


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


def _empty_f32(dev):
    return torch.empty(0, dtype=torch.float32, device=dev)


_ERR_WORDS: dict = {}


def _err_word(dev):
    """Per-device int32[4] error word passed to the decode kernels (zeroed
    here once and again after every read)."""
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    w = _ERR_WORDS.get(key)
    if w is None:
        w = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", key))
        _ERR_WORDS[key] = w
    return w


def _raise_err_word(w):
    """Synchronising read of a decode error word; raises GdnError (and clears
    the word) when a kernel recorded a failure."""
    h = w.cpu().tolist()
    if h[0] != 0:
        w.zero_()
        what = {1: "a bounded wait gave up", 2: "state slot index out of range"}.get(h[0], "device error")
        raise _lib.GdnError(_lib.GDN_ERR_DEVICE,
                            f"{what} (code {h[0]}, site {h[1]}, sequence/block {h[2]}, info {h[3]})")


def _real(x):
    return not isinstance(x, torch.Tensor) or type(x) is torch.Tensor or type(x) is torch.nn.Parameter


def _call(op, impl, *args):
    """Run a custom op.  Eager calls on plain tensors go straight to its
    implementation: the custom-op dispatcher costs about 15 us of host time
    per call, which leaves the GPU idle between launches as short as a
    decode step.  Traced calls (torch.compile, FakeTensor and other tensor
    subclasses) go through the registered op, whose fake gives the shapes."""
    if torch.compiler.is_compiling() or not all(_real(x) for x in args):
        return op(*args)
    return impl(*args)


# ---------------------------------------------------------------------------
# torch.library custom ops (CUDA implementations call the C ABI)
# ---------------------------------------------------------------------------

def _rows(t):
    """(tensor, token stride) of a [B, T, heads, d] input for the tensor-core
    prefill: in place when only its token rows are strided (e.g. q, k, v as
    views of one projection) and the stride suits the tensor maps, else a
    packed copy with stride 0."""
    if t.is_contiguous():
        return t, 0
    B, T, nh, d = t.shape
    st = t.stride()
    if (st[3] == 1 and st[2] == d and (B == 1 or st[0] == T * st[1]) and st[1] >= nh * d and st[1] % 8 == 0
            and t.storage_offset() * t.element_size() % 16 == 0):
        return t, st[1]
    return t.contiguous(), 0


def _chunk_fwd_impl(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, scale: float,
                  initial_state: Optional[Tensor], output_final_state: bool,
                  cu_seqlens: Optional[Tensor], state_v_first: bool, use_qk_l2norm: bool,
                  force_generic: bool, check_errors: bool) -> tuple[Tensor, Tensor]:
    """Chunked prefill on prepared inputs (q/k/v in one dtype, packed or, on
    the tensor-core path, with strided token rows; g/beta/initial_state fp32
    contiguous, cu_seqlens int32/int64).  Returns
    ``(o, final_state)``; final_state is an empty tensor when not requested."""
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.numel() - 1
    dev = q.device
    if q.dtype in (torch.bfloat16, torch.float16) and K == 128 and V == 128 and not force_generic:
        (q, sq), (k, sk), (v, sv) = _rows(q), _rows(k), _rows(v)  # the tensor-core path reads strided rows
    else:
        (q, sq), (k, sk), (v, sv) = (q.contiguous(), 0), (k.contiguous(), 0), (v.contiguous(), 0)
    o = torch.empty(v.shape, dtype=q.dtype, device=dev)
    shape_state = (N, HV, V, K) if state_v_first else (N, HV, K, V)
    ht = torch.empty(shape_state, dtype=torch.float32, device=dev) if output_final_state else None
    args = _lib.ChunkArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), beta=_ptr(beta),
        initial_state=_ptr(initial_state), o=_ptr(o), final_state=_ptr(ht), cu_seqlens=_ptr(cu_seqlens),
        workspace=None, workspace_bytes=0, B=B, T=T, N=N, H=H, HV=HV, K=K, V=V,
        qkv_dtype=_DT[q.dtype], cu_dtype=_IDT[cu_seqlens.dtype] if cu_seqlens is not None else _lib.GDN_I64,
        scale=float(scale), use_qk_l2norm=int(use_qk_l2norm), state_v_first=int(state_v_first),
        force_generic=int(force_generic), q_token_stride=sq, k_token_stride=sk, v_token_stride=sv)
    lib = _lib.load()
    nbytes = lib.gdn_chunk_workspace_size(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(_lib.GDN_ERR_INVALID)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    args.workspace = ctypes.c_void_p(ws.data_ptr())
    args.workspace_bytes = nbytes
    with torch.cuda.device(dev):
        _lib.check(lib.gdn_chunk_fwd(ctypes.byref(args), _stream(dev)))
        if check_errors:
            _lib.check(lib.gdn_chunk_check_device_error(args.workspace, _stream(dev)))
    return o, (ht if ht is not None else _empty_f32(dev))


_chunk_fwd_op = torch.library.custom_op("gdn_b200::chunk_fwd", mutates_args=(),
                device_types="cuda")(_chunk_fwd_impl)


@_chunk_fwd_op.register_fake
def _(q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, state_v_first,
      use_qk_l2norm, force_generic, check_errors):
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.shape[0] - 1
    o = v.new_empty(v.shape, dtype=q.dtype)
    if not output_final_state:
        return o, v.new_empty((0,), dtype=torch.float32)
    shape_state = (N, HV, V, K) if state_v_first else (N, HV, K, V)
    return o, v.new_empty(shape_state, dtype=torch.float32)


def _chunk_bwd_impl(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, scale: float,
                  initial_state: Optional[Tensor], cu_seqlens: Optional[Tensor], dout: Tensor,
                  dht: Optional[Tensor], state_v_first: bool,
                  use_qk_l2norm: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Backward on prepared inputs; returns ``(dq, dk, dv, dg, dbeta, dh0)``
    with dh0 an empty tensor when there is no initial state."""
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.numel() - 1
    dev = q.device
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(v.shape[:3], dtype=torch.float32, device=dev)
    db = torch.empty(v.shape[:3], dtype=torch.float32, device=dev)
    shape_state = (N, HV, V, K) if state_v_first else (N, HV, K, V)
    dh0 = torch.empty(shape_state, dtype=torch.float32, device=dev) if initial_state is not None else None
    args = _lib.ChunkBwdArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), beta=_ptr(beta), initial_state=_ptr(initial_state),
        cu_seqlens=_ptr(cu_seqlens), dout=_ptr(dout), dht=_ptr(dht), dq=_ptr(dq), dk=_ptr(dk), dv=_ptr(dv),
        dg=_ptr(dg), dbeta=_ptr(db), dh0=_ptr(dh0), workspace=None, workspace_bytes=0,
        B=B, T=T, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=_DT[q.dtype],
        cu_dtype=_IDT[cu_seqlens.dtype] if cu_seqlens is not None else _lib.GDN_I64,
        scale=float(scale), use_qk_l2norm=int(use_qk_l2norm), state_v_first=int(state_v_first))
    lib = _lib.load()
    nbytes = lib.gdn_chunk_bwd_workspace_size(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(_lib.GDN_ERR_INVALID)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    args.workspace = ctypes.c_void_p(ws.data_ptr())
    args.workspace_bytes = nbytes
    with torch.cuda.device(dev):
        _lib.check(lib.gdn_chunk_bwd(ctypes.byref(args), _stream(dev)))
    return dq, dk, dv, dg, db, (dh0 if dh0 is not None else _empty_f32(dev))


_chunk_bwd_op = torch.library.custom_op("gdn_b200::chunk_bwd", mutates_args=(),
                device_types="cuda")(_chunk_bwd_impl)


@_chunk_bwd_op.register_fake
def _(q, k, v, g, beta, scale, initial_state, cu_seqlens, dout, dht, state_v_first, use_qk_l2norm):
    dg = v.new_empty(v.shape[:3], dtype=torch.float32)
    dh0 = (initial_state.new_empty(initial_state.shape) if initial_state is not None
           else v.new_empty((0,), dtype=torch.float32))
    return (q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape), dg,
            v.new_empty(v.shape[:3], dtype=torch.float32), dh0)


def _recurrent_args(q, k, v, g, gk, beta, scale, initial_state, final_state, o, cu, idx, nacc, l2,
                    inplace, num_slots, err):
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu is None else cu.numel() - 1
    if idx is None:
        s_seq, s_tok = 1, 1
    elif idx.dim() == 1:
        s_seq, s_tok = idx.stride(0), 1
    else:
        s_seq, s_tok = idx.stride()
    return _lib.RecurrentArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), beta=_ptr(beta),
        initial_state=_ptr(initial_state), o=_ptr(o), final_state=_ptr(final_state),
        cu_seqlens=_ptr(cu), ssm_state_indices=_ptr(idx), num_accepted_tokens=_ptr(nacc),
        B=B, T=T, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=_DT[q.dtype],
        cu_dtype=_IDT[cu.dtype] if cu is not None else _lib.GDN_I64,
        idx_dtype=_IDT[idx.dtype] if idx is not None else _lib.GDN_I64,
        nacc_dtype=_IDT[nacc.dtype] if nacc is not None else _lib.GDN_I64,
        stride_init_state_token=initial_state.stride(0) if initial_state is not None else 0,
        stride_final_state_token=final_state.stride(0) if final_state is not None else 0,
        stride_indices_seq=s_seq, stride_indices_tok=s_tok, scale=float(scale),
        use_qk_l2norm=int(l2), beta_per_v=int(beta.dim() == v.dim()), inplace_final_state=int(inplace),
        num_slots=int(num_slots), err=_ptr(err), gk=_ptr(gk))


def _run_recurrent(args, dev, check_errors, err):
    with torch.cuda.device(dev):
        _lib.check(_lib.load().gdn_fused_recurrent_fwd(ctypes.byref(args), _stream(dev)))
        if check_errors:
            _raise_err_word(err)


def _recurrent_fn_inplace_impl(q: Tensor, k: Tensor, v: Tensor, g: Optional[Tensor], gk: Optional[Tensor],
                             beta: Tensor, scale: float, state: Tensor, cu_seqlens: Optional[Tensor],
                             ssm_state_indices: Tensor, num_accepted_tokens: Optional[Tensor],
                             use_qk_l2norm: bool, check_errors: bool) -> Tensor:
    """Slot-indexed decode that updates the V-first cache ``state`` in place
    (rows ``ssm_state_indices[n, t]``); returns o."""
    o = torch.empty_like(v)
    err = _err_word(q.device)
    args = _recurrent_args(q, k, v, g, gk, beta, scale, state, state, o, cu_seqlens, ssm_state_indices,
                           num_accepted_tokens, use_qk_l2norm, True, state.shape[0], err)
    _run_recurrent(args, q.device, check_errors, err)
    return o


_recurrent_fn_inplace_op = torch.library.custom_op("gdn_b200::recurrent_fn_inplace", mutates_args=("state",),
                           device_types="cuda")(_recurrent_fn_inplace_impl)


@_recurrent_fn_inplace_op.register_fake
def _(q, k, v, g, gk, beta, scale, state, cu_seqlens, ssm_state_indices, num_accepted_tokens,
      use_qk_l2norm, check_errors):
    return v.new_empty(v.shape)


def _recurrent_fn_impl(q: Tensor, k: Tensor, v: Tensor, g: Optional[Tensor], gk: Optional[Tensor],
                     beta: Tensor, scale: float, initial_state: Optional[Tensor],
                     cu_seqlens: Optional[Tensor], ssm_state_indices: Optional[Tensor],
                     num_accepted_tokens: Optional[Tensor], use_qk_l2norm: bool,
                     check_errors: bool) -> tuple[Tensor, Tensor]:
    """Decode with the state after every token written to a fresh
    ``[B*T, HV, V, K]`` tensor (``inplace_final_state=False``)."""
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    o = torch.empty_like(v)
    final_state = torch.empty(B * T, HV, V, K, dtype=torch.float32, device=q.device)
    err = _err_word(q.device)
    nslots = initial_state.shape[0] if (initial_state is not None and ssm_state_indices is not None) else 0
    args = _recurrent_args(q, k, v, g, gk, beta, scale, initial_state, final_state, o, cu_seqlens,
                           ssm_state_indices, num_accepted_tokens, use_qk_l2norm, False, nslots, err)
    _run_recurrent(args, q.device, check_errors, err)
    return o, final_state


_recurrent_fn_op = torch.library.custom_op("gdn_b200::recurrent_fn", mutates_args=(),
                   device_types="cuda")(_recurrent_fn_impl)


@_recurrent_fn_op.register_fake
def _(q, k, v, g, gk, beta, scale, initial_state, cu_seqlens, ssm_state_indices, num_accepted_tokens,
      use_qk_l2norm, check_errors):
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    return v.new_empty(v.shape), v.new_empty((B * T, HV, V, K), dtype=torch.float32)


def _recurrent_plain_impl(q: Tensor, k: Tensor, v: Tensor, g: Optional[Tensor], gk: Optional[Tensor],
                        gv: Optional[Tensor], beta: Tensor, scale: float, initial_state: Optional[Tensor],
                        output_final_state: bool, use_qk_l2norm: bool,
                        cu_seqlens: Optional[Tensor]) -> tuple[Tensor, Tensor]:
    """Plain K-first recurrence; final_state is empty when not requested."""
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.numel() - 1
    o = torch.empty_like(v)
    ht = torch.empty(N, HV, K, V, dtype=torch.float32, device=q.device) if output_final_state else None
    args = _lib.RecurrentPlainArgs(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), g=_ptr(g), gk=_ptr(gk), gv=_ptr(gv), beta=_ptr(beta),
        initial_state=_ptr(initial_state), o=_ptr(o), final_state=_ptr(ht), cu_seqlens=_ptr(cu_seqlens),
        B=B, T=T, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=_DT[q.dtype],
        cu_dtype=_IDT[cu_seqlens.dtype] if cu_seqlens is not None else _lib.GDN_I64,
        scale=float(scale), use_qk_l2norm=int(use_qk_l2norm), beta_per_v=int(beta.dim() == v.dim()))
    dev = q.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().gdn_recurrent_plain_fwd(ctypes.byref(args), _stream(dev)))
    return o, (ht if ht is not None else _empty_f32(dev))


_recurrent_plain_op = torch.library.custom_op("gdn_b200::recurrent_plain", mutates_args=(),
                      device_types="cuda")(_recurrent_plain_impl)


@_recurrent_plain_op.register_fake
def _(q, k, v, g, gk, gv, beta, scale, initial_state, output_final_state, use_qk_l2norm, cu_seqlens):
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.shape[0] - 1
    ht = v.new_empty((N, HV, K, V) if output_final_state else (0,), dtype=torch.float32)
    return v.new_empty(v.shape), ht


def _solve_tril_impl(input: Tensor, output: Tensor, cu_seqlens: Optional[Tensor]) -> None:
    """``solve_tril(input, output, cu_seqlens)`` of the native op
    (``include/torch_mlu_ops.h:1052-1054``): input fp32 ``[B, T, H, BT]``
    contiguous, output of the same shape (contiguous) written in place."""
    B, T, H, BT = input.shape
    cu, cu_dt = _idx(cu_seqlens)
    N = B if cu is None else cu.numel() - 1
    dev = input.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().gdn_solve_tril(
            _ptr(input), _ptr(output), _DT[output.dtype], _ptr(cu), cu_dt, N, B, T, H, BT, _stream(dev)))


_solve_tril_op = torch.library.custom_op("gdn_b200::solve_tril", mutates_args=("output",),
                 device_types="cuda")(_solve_tril_impl)


@_solve_tril_op.register_fake
def _(input, output, cu_seqlens):
    return None


def _chunk_fwd_h_impl(k: Tensor, w: Tensor, u: Tensor, g: Optional[Tensor], gk: Optional[Tensor],
                      initial_state: Optional[Tensor], h: Optional[Tensor], v_new: Optional[Tensor],
                      final_state: Optional[Tensor], cu_seqlens: Optional[Tensor], state_v_first: bool) -> None:
    """The state-recurrence stage on prepared inputs (k, w, u contiguous in
    one dtype; g, gk, initial_state fp32 contiguous); writes h, v_new and
    final_state (each optional) in place."""
    B, T, Hg, K = k.shape
    H, V = u.shape[2], u.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.numel() - 1
    args = _lib.ChunkHArgs(
        k=_ptr(k), w=_ptr(w), u=_ptr(u), g=_ptr(g), gk=_ptr(gk), initial_state=_ptr(initial_state),
        h=_ptr(h), v_new=_ptr(v_new), final_state=_ptr(final_state), cu_seqlens=_ptr(cu_seqlens),
        B=B, T=T, N=N, Hg=Hg, H=H, K=K, V=V, dtype=_DT[k.dtype],
        cu_dtype=_IDT[cu_seqlens.dtype] if cu_seqlens is not None else _lib.GDN_I64,
        state_v_first=int(state_v_first))
    dev = k.device
    with torch.cuda.device(dev):
        _lib.check(_lib.load().gdn_chunk_fwd_h(ctypes.byref(args), _stream(dev)))


_chunk_fwd_h_op = torch.library.custom_op("gdn_b200::chunk_fwd_h", mutates_args=("h", "v_new", "final_state"),
                                          device_types="cuda")(_chunk_fwd_h_impl)


@_chunk_fwd_h_op.register_fake
def _(k, w, u, g, gk, initial_state, h, v_new, final_state, cu_seqlens, state_v_first):
    return None


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
    _qkv_dtype(q, k, v)
    cu, _ = _idx(cu_seqlens)
    N = B if cu is None else cu.shape[0] - 1
    shape_state = (N, HV, V, K) if state_v_first else (N, HV, K, V)
    if initial_state is not None and tuple(initial_state.shape) != shape_state:
        raise ValueError(f"initial_state must be {shape_state}, got {tuple(initial_state.shape)}")
    return cu


def _scale(scale):
    return float(scale) if scale is not None else 0.0  # <= 0 selects K ** -0.5 in the library


class ChunkGatedDeltaRuleFunction(torch.autograd.Function):
    """Autograd node of the chunked forward (``triton/fla/chunk.py:188-251``):
    the forward saves its inputs only and the backward recomputes the
    intermediates (``chunk.py:76-186``) inside ``gdn_b200::chunk_bwd``."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens,
                state_v_first, use_qk_l2norm, force_generic, check_errors=False):
        cu = _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens, state_v_first)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        g32, b32, h0 = _f32(g), _f32(beta), _f32(initial_state)
        o, ht = _call(torch.ops.gdn_b200.chunk_fwd, _chunk_fwd_impl, q, k, v, g32, b32, _scale(scale), h0,
                      bool(output_final_state), cu, bool(state_v_first), bool(use_qk_l2norm),
                      bool(force_generic), bool(check_errors))
        ctx.save_for_backward(q, k, v, g32, b32, h0, cu)
        ctx.meta = (_scale(scale), bool(state_v_first), bool(use_qk_l2norm), g.dtype, beta.dtype,
                    None if initial_state is None else initial_state.dtype)
        return o, (ht if output_final_state else None)

    @staticmethod
    def backward(ctx, do, dht):
        q, k, v, g32, b32, h0, cu = ctx.saved_tensors
        scale, svf, l2, g_dt, b_dt, h0_dt = ctx.meta
        if do is None:
            do = torch.zeros_like(v, dtype=q.dtype)
        do = do.to(q.dtype).contiguous()
        dht = None if dht is None else dht.to(torch.float32).contiguous()
        dq, dk, dv, dg, db, dh0 = _call(torch.ops.gdn_b200.chunk_bwd, _chunk_bwd_impl, q, k, v, g32, b32,
                                        scale, h0, cu, do, dht, svf, l2)
        dh0 = dh0.to(h0_dt) if h0 is not None else None
        return (dq, dk, dv, dg.to(g_dt), db.to(b_dt), None, dh0, None, None, None, None, None, None)


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
    check_errors: bool = False,
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
    dbeta and d(initial_state).  ``check_errors=True`` reads the call's device
    error word back (one synchronisation) and raises on a recorded failure.
    """
    del chunk_indices, chunk_offsets, allow_tf32
    _cuda("chunk_gated_delta_rule", q, k, v, g, beta, initial_state, cu_seqlens)
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (q, k, v, g, beta, initial_state)):
        return ChunkGatedDeltaRuleFunction.apply(
            q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, state_v_first,
            use_qk_l2norm_in_kernel, force_generic, check_errors)
    cu = _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens, state_v_first)
    o, ht = _call(
        torch.ops.gdn_b200.chunk_fwd, _chunk_fwd_impl, q, k, v,
        _f32(g), _f32(beta), _scale(scale), _f32(initial_state), bool(output_final_state), cu, bool(state_v_first),
        bool(use_qk_l2norm_in_kernel), bool(force_generic), bool(check_errors))
    return o, (ht if output_final_state else None)


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
    segment_tokens: int = 4096,
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
    are those of the device op.  A single sequence's last ``segment_tokens``
    tokens go in halving pieces (down to 512 tokens), which shortens the
    compute and copy-out of the last piece that nothing overlaps.  4096 was
    the fastest piece size at the config-1 shape on a B200 (3.12 ms; 2048:
    3.20 ms, 3072: 3.18 ms): every piece costs about 50 us of copy set-up.
    Page-locked (pinned) inputs give overlapped copies; other host memory is
    pinned first.

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
    _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens, state_v_first)
    B, T, H, HV, K, V = _check_shapes(q, k, v)
    N = B if cu_seqlens is None else cu_seqlens.numel() - 1
    shape_state = (N, HV, V, K) if state_v_first else (N, HV, K, V)
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
        qkv_dtype=_qkv_dtype(q, k, v), cu_dtype=cu_dt, scale=_scale(scale),
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
    cu = _chunk_prepare(q, k, v, g, beta, initial_state, cu_seqlens, state_v_first)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    h0 = _f32(initial_state)
    dq, dk, dv, dg, db, dh0 = _call(
        torch.ops.gdn_b200.chunk_bwd, _chunk_bwd_impl, q, k, v, _f32(g), _f32(beta), _scale(scale), h0, cu,
        dout.to(q.dtype).contiguous(), None if dht is None else _f32(dht), bool(state_v_first), bool(use_qk_l2norm_in_kernel))
    return dq, dk, dv, db, dg, (dh0 if h0 is not None else None)


def chunk_gated_delta_rule_fwd_h(
    k: torch.Tensor,
    w: torch.Tensor,
    u: torch.Tensor,
    g: torch.Tensor | None = None,
    gk: torch.Tensor | None = None,
    initial_state: torch.Tensor | None = None,
    output_final_state: bool = False,
    chunk_size: int = 64,
    save_new_value: bool = True,
    state_v_first: bool = False,
    cu_seqlens: torch.LongTensor | None = None,
    chunk_indices: torch.Tensor | None = None,
    chunk_offsets: torch.Tensor | None = None,
    allow_tf32: bool = True,
):
    """The inter-chunk state recurrence stage (``triton/fla/chunk_delta_h.py:200-271``),
    with the per-key decay ``gk`` of its KDA branch (``USE_GK``, ``:155-171``).

    k ``[B, T, Hg, K]``; w ``[B, T, H, K]``; u ``[B, T, H, V]`` (one dtype);
    g the chunk-local cumsum of the log decay in the reference's head-major
    layout ``[H, B, T]`` (``chunk.py:32``) or None; gk the per-key cumsum
    ``[B, T, H, K]`` or None.  Returns ``(h, v_new, final_state)``: the state
    before each chunk ``[B, NT, H, K, V]`` (``[.., V, K]`` with
    ``state_v_first``) in k's dtype, ``v_new = u - w h`` like u (or None
    without ``save_new_value``) and the fp32 final state (or None).  Chunks
    are 64 tokens; ``chunk_indices`` / ``chunk_offsets`` / ``allow_tf32`` are
    accepted for signature compatibility (products are full fp32).  With
    ``cu_seqlens`` the chunk count is read on the host, as the reference's
    ``prepare_chunk_indices`` does.
    """
    del chunk_offsets, allow_tf32
    if chunk_size != 64:
        raise ValueError(f"chunk_size={chunk_size}: the kernels use 64-token chunks")
    _cuda("chunk_gated_delta_rule_fwd_h", k, w, u, g, gk, initial_state, cu_seqlens)
    if k.dim() != 4 or w.dim() != 4 or u.dim() != 4 or w.shape[:3] != u.shape[:3] or k.shape[:2] != w.shape[:2]:
        raise ValueError("k must be [B, T, Hg, K], w [B, T, H, K] and u [B, T, H, V]")
    B, T, Hg, K = k.shape
    H, V = u.shape[2], u.shape[3]
    if w.shape[3] != K or H % Hg or K > 128 or V > 128:
        raise ValueError(f"bad head layout or sizes (Hg={Hg}, H={H}, K={K}, V={V}; K, V <= 128)")
    if not (k.dtype == w.dtype == u.dtype) or k.dtype not in _DT:
        raise ValueError("k, w and u must share one dtype (float32, bfloat16 or float16)")
    if cu_seqlens is not None and B != 1:
        raise ValueError("cu_seqlens requires batch size 1 (packed sequences)")
    if g is not None and g.numel() != H * B * T:
        raise ValueError(f"g must hold [H, B, T] = {(H, B, T)} values (head-major)")
    if gk is not None and tuple(gk.shape) != (B, T, H, K):
        raise ValueError(f"gk must be [B, T, H, K] = {(B, T, H, K)}")
    cu, _ = _idx(cu_seqlens)
    if cu is None:
        N, NT = B, (T + 63) // 64
    else:
        N = cu.numel() - 1
        if chunk_indices is not None:
            NT = int(chunk_indices.shape[0])
        else:
            lens = (cu[1:] - cu[:-1]).tolist()
            NT = sum((x + 63) // 64 for x in lens)
    shape_state = (N, H, V, K) if state_v_first else (N, H, K, V)
    if initial_state is not None and tuple(initial_state.shape) != shape_state:
        raise ValueError(f"initial_state must be {shape_state}, got {tuple(initial_state.shape)}")
    h = k.new_empty((B, NT, H, V, K) if state_v_first else (B, NT, H, K, V))
    v_new = torch.empty_like(u) if save_new_value else None
    ht = torch.empty(shape_state, dtype=torch.float32, device=k.device) if output_final_state else None
    _call(torch.ops.gdn_b200.chunk_fwd_h, _chunk_fwd_h_impl, k.contiguous(), w.contiguous(), u.contiguous(),
          None if g is None else g.to(torch.float32).contiguous(), _f32(gk), _f32(initial_state), h, v_new, ht,
          cu, bool(state_v_first))
    return h, v_new, ht


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
    *,
    check_errors: bool = False,
):
    """Slot-indexed recurrent decode (``triton_ops.py:228-285`` ->
    ``triton/fla/fused_recurrent_fn.py:161-233``).

    The state cache is V-first ``[slots, HV, V, K]`` fp32 (the kernel's
    layout, ``fused_recurrent_fn.py:101-104``).  With
    ``inplace_final_state=True`` the cache is updated in place at
    ``ssm_state_indices[n, t]`` and returned; otherwise a fresh
    ``[B*T, HV, V, K]`` tensor receives the state after every token.
    ``g`` is the per-head log decay ``[B, T, HV]``, or ``[B, T, HV, K]`` for
    per-key decays (the kernel's KDA form).  A slot index at or past
    ``initial_state.shape[0]`` skips its sequence like PAD and is recorded in
    the device error word (``check_errors=True`` raises on it).
    """
    _cuda("fused_recurrent_gated_delta_rule_fn", q, k, v, g, beta, initial_state, cu_seqlens,
          ssm_state_indices, num_accepted_tokens)
    B, T, H, HV, K, V = _check_shapes(q, k, v)
    if K > 128 or V > 128:
        raise ValueError(f"K={K}, V={V}: both must be <= 128 (fused_recurrent_fn.py:181-182)")
    if cu_seqlens is not None and B != 1:
        raise ValueError("cu_seqlens requires batch size 1 (packed sequences)")
    _qkv_dtype(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if beta is None:
        beta = torch.ones(v.shape[:3], dtype=torch.float32, device=v.device)
    gk = None
    if g is not None and g.dim() == 4:
        if tuple(g.shape) != (B, T, HV, K):
            raise ValueError(f"per-key g must be [B, T, HV, K] = {(B, T, HV, K)}, got {tuple(g.shape)}")
        g, gk = None, g
    g, gk, beta = _f32(g), _f32(gk), _f32(beta)
    cu, _ = _idx(cu_seqlens)
    idx, _ = _idx(ssm_state_indices)
    nacc, _ = _idx(num_accepted_tokens)
    if nacc is not None:
        nacc = nacc.contiguous()
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
        o = _call(torch.ops.gdn_b200.recurrent_fn_inplace, _recurrent_fn_inplace_impl, q, k, v, g, gk, beta,
                  float(scale), initial_state, cu, idx, nacc, bool(use_qk_l2norm_in_kernel), bool(check_errors))
        return o, initial_state
    return _call(torch.ops.gdn_b200.recurrent_fn, _recurrent_fn_impl, q, k, v, g, gk, beta, float(scale),
                 initial_state, cu, idx, nacc, bool(use_qk_l2norm_in_kernel), bool(check_errors))


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
        if gv is not None:
            raise ValueError("gv is not supported with ssm_state_indices")
        if gk is not None:
            if g is not None:
                raise ValueError("give either g or the per-key gk with ssm_state_indices")
            g = gk
        return fused_recurrent_gated_delta_rule_fn(
            q, k, v, g, beta, scale, initial_state, inplace_final_state, cu_seqlens,
            ssm_state_indices, num_accepted_tokens, use_qk_l2norm_in_kernel)
    _cuda("fused_recurrent_gated_delta_rule", q, k, v, g, gk, gv, beta, initial_state, cu_seqlens)
    B, T, H, HV, K, V = _check_shapes(q, k, v)
    if K > 128 or V > 128:
        raise ValueError(f"K={K}, V={V}: both must be <= 128 (fused_recurrent.py:155-156)")
    if cu_seqlens is not None and B != 1:
        raise ValueError("cu_seqlens requires batch size 1 (packed sequences)")
    _qkv_dtype(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if beta is None:
        beta = torch.ones(v.shape[:3], dtype=torch.float32, device=v.device)
    g, gk, gv, beta = _f32(g), _f32(gk), _f32(gv), _f32(beta)
    cu, _ = _idx(cu_seqlens)
    N = B if cu is None else cu.shape[0] - 1
    h0 = None
    if initial_state is not None:
        if tuple(initial_state.shape) != (N, HV, K, V):
            raise ValueError(f"initial_state must be {(N, HV, K, V)}, got {tuple(initial_state.shape)}")
        h0 = _f32(initial_state)
    o, ht = _call(torch.ops.gdn_b200.recurrent_plain, _recurrent_plain_impl, q, k, v, g, gk, gv, beta,
                  _scale(scale), h0, bool(output_final_state), bool(use_qk_l2norm_in_kernel), cu)
    return o, (ht if output_final_state else None)


def solve_tril(input: torch.Tensor, output: torch.Tensor = None, cu_seqlens: torch.Tensor = None,
               out_dtype: torch.dtype = torch.float):
    """(I + input)^-1 per chunk block (``_ops.py:6232-6257``; native op
    ``include/torch_mlu_ops.h:1052-1054``).  input fp32 ``[B, T, H, BT]`` or
    packed ``[total_tokens, H, BT]``, BT in {16, 32, 64}; output
    bf16/fp16/fp32 of the same shape."""
    _cuda("solve_tril", input, output, cu_seqlens)
    if input.dtype != torch.float32 or input.dim() not in (3, 4):
        raise ValueError("input must be a float32 [B, T, H, BT] or [total_tokens, H, BT] tensor")
    if output is None:
        output = torch.empty(input.shape, device=input.device, dtype=out_dtype)
    if output.shape != input.shape or output.dtype not in _DT:
        raise ValueError("output must match input's shape with dtype float32/bfloat16/float16")
    x = input.contiguous()
    if x.dim() == 3:
        x = x.unsqueeze(0)
    out = output if output.is_contiguous() else torch.empty_like(output)
    out4 = out.unsqueeze(0) if out.dim() == 3 else out
    cu, _ = _idx(cu_seqlens)
    _call(torch.ops.gdn_b200.solve_tril, _solve_tril_impl, x, out4, cu)
    if out is not output:
        output.copy_(out)
    return output
