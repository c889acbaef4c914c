"""Causal depthwise conv1d ops, drop-in for ``torch_mlu_ops.triton_ops``
(``causal_conv1d``, ``causal_conv1d_fn``) and ``triton.conv``
(``causal_conv1d_update``): the short convolution over the q/k/v channels in
front of the GDN layer of Qwen3-Next.

Same names, argument order, keyword names, defaults and return values as the
reference (``triton_ops.py:287-459``, ``triton/conv/ops.py:584-644``); the
work runs in ``libgdn_b200.so`` (``gdn_conv.cu``) through its C ABI.  There is
no CPU or Triton path.

Differences from the reference, all supersets or stricter checks:

* ``causal_conv1d_fn`` skips a sequence whose cache line is ``pad_slot_id``
  as well as ``null_block_id`` (the reference indexes line -1), and writes
  zeros for the tokens of skipped sequences (the reference leaves them
  unwritten); ``has_initial_state=None`` means no initial state and
  ``cache_indices=None`` maps sequence i to line i.
* Products are accumulated in fp32 from the inputs as given (the reference
  first casts x to the ``conv_states`` dtype and multiplies in that dtype).
* Prefix caching (``block_idx_*``, ``initial_state_idx``,
  ``num_computed_tokens``, ``block_size_to_align``) follows the reference
  kernel; ``block_size_to_align`` must be a positive multiple of 64 (the
  reference checks that only with ``validate_data``).
* An unknown ``activation`` string raises ``ValueError`` (the reference
  kernels silently apply none).
"""

from __future__ import annotations

import torch

from . import _lib
from .gdn import _DT, _IDT, _cuda, _ptr, _stream


def _act(activation):
    if activation in (None, False):
        return _lib.GDN_ACT_NONE
    if activation is True or activation in ("silu", "swish"):
        return _lib.GDN_ACT_SILU
    raise ValueError(f"[CausalConv1d] unsupported activation {activation!r} (None, 'silu' or 'swish')")


def _fdt(t, name):
    if t.dtype not in _DT:
        raise ValueError(f"[CausalConv1d] {name} dtype {t.dtype} must be float32, bfloat16 or float16")
    return _DT[t.dtype]


def _fn_args(x, weight, bias, conv_states, query_start_loc, cache_indices, has_initial_state, activation,
             pad_slot_id, null_block_id, block_idx_first_scheduled_token, block_idx_last_scheduled_token,
             initial_state_idx, num_computed_tokens, block_size_to_align, out):
    """``gdn_conv1d_fn_args`` for channel-last x ``(dim, tokens)`` (and ``out``
    of the same layout, or None for the fused prefill); returns the struct and
    the converted tensors it points into (keep them alive until the launch)."""
    dim, total = x.shape
    W = weight.shape[1]
    if W < 2:
        raise ValueError("[CausalConv1d] weight.shape[-1] must be at least 2")
    if conv_states.dim() != 3 or conv_states.shape[1] != dim or conv_states.shape[2] < W - 1:
        raise ValueError(f"[CausalConv1d] conv_states {tuple(conv_states.shape)} must be (lines, {dim}, >= {W - 1})")
    if conv_states.stride(1) != 1:
        raise ValueError("[CausalConv1d] conv_states must have unit stride along dim")
    w = weight.contiguous()
    b = None if bias is None else bias.to(w.dtype).contiguous()
    qsl = (query_start_loc if query_start_loc.dtype in _IDT else query_start_loc.to(torch.int32)).contiguous()
    batch = qsl.numel() - 1
    apc = block_idx_last_scheduled_token is not None
    ci = None
    idx_dt = _lib.GDN_I32
    if cache_indices is not None:
        ci = (cache_indices if cache_indices.dtype in _IDT else cache_indices.to(torch.int32)).contiguous()
        idx_dt = _IDT[ci.dtype]
        if ci.dim() not in (1, 2) or ci.shape[0] != batch or (ci.dim() == 2 and not apc):
            raise ValueError(f"[CausalConv1d] cache_indices must be ({batch},) (or ({batch}, blocks) "
                             "with prefix caching)")
    blocks = [None] * 4
    if apc:
        if cache_indices is None:
            raise ValueError("[CausalConv1d] prefix caching needs cache_indices")
        if ci.dim() == 1:
            ci = ci[:, None]
        blocks = [t if t is None else t.to(torch.int32).contiguous()
                  for t in (block_idx_first_scheduled_token, block_idx_last_scheduled_token,
                            initial_state_idx, num_computed_tokens)]
        if any(t is None for t in blocks):
            raise ValueError("[CausalConv1d] prefix caching needs block_idx_first_scheduled_token, "
                             "block_idx_last_scheduled_token, initial_state_idx and num_computed_tokens")
    hi = None
    if has_initial_state is not None:
        hi = has_initial_state.to(torch.bool).contiguous()
        if hi.numel() != batch:
            raise ValueError(f"[CausalConv1d] has_initial_state must be ({batch},)")
    args = _lib.Conv1dFnArgs(
        x=_ptr(x), out=_ptr(out), weight=_ptr(w), bias=_ptr(b), conv_states=_ptr(conv_states),
        query_start_loc=_ptr(qsl), cache_indices=_ptr(ci), has_initial_state=_ptr(hi),
        stride_x_token=x.stride(1) if total > 1 else dim,
        stride_o_token=(out.stride(1) if total > 1 else dim) if out is not None else 0,
        stride_state_seq=conv_states.stride(0), stride_state_tok=conv_states.stride(2),
        num_cache_lines=conv_states.shape[0], batch=batch, dim=dim, total_tokens=total,
        pad_slot_id=int(pad_slot_id), null_block_id=0 if null_block_id is None else int(null_block_id),
        has_null_block=0 if null_block_id is None else 1, W=W,
        x_dtype=_fdt(x, "x"), w_dtype=_fdt(w, "weight"), state_dtype=_fdt(conv_states, "conv_states"),
        qsl_dtype=_IDT[qsl.dtype], idx_dtype=idx_dt, activation=_act(activation),
        block_idx_first=_ptr(blocks[0]), block_idx_last=_ptr(blocks[1]), initial_state_idx=_ptr(blocks[2]),
        num_computed_tokens=_ptr(blocks[3]), stride_cache_indices=ci.stride(0) if ci is not None else 0,
        block_size_to_align=int(block_size_to_align or 0), apc_dtype=_lib.GDN_I32)
    return args, (w, b, qsl, ci, hi, blocks)


def causal_conv1d(
    x: torch.Tensor,
    weight: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    initial_state: torch.Tensor | None = None,
    output_final_state: bool | None = False,
    activation: str | None = None,
    backend: str | None = "triton",
    cu_seqlens: torch.Tensor | None = None,
    cu_seqlens_cpu: torch.LongTensor | None = None,
    chunk_indices: torch.LongTensor | None = None,
    cp_context=None,
    **kwargs,
):
    """y = act(conv(x) + bias) + residual over x ``[B, T, D]`` with weight
    ``[D, W]``; ``initial_state [N, D, W]`` supplies the tokens before each
    sequence (column j = token j - W).  Returns ``(y, None)``
    (``triton_ops.py:287-363``).  ``backend`` is accepted for signature
    compatibility ('triton' is the reference's only value; the work runs in
    CUDA here)."""
    if cp_context is not None:
        raise ValueError("[CausalConv1d] CP Context not supported.")
    if output_final_state is True:
        raise ValueError("[CausalConv1d] output_final_state true not supported.")
    if backend != "triton":
        raise ValueError(f"[CausalConv1d] Unsupported backend: {backend}")
    if weight is None:
        raise ValueError("[CausalConv1d] weight is required")
    if x.dim() != 3:
        raise ValueError(f"[CausalConv1d] x must be [B, T, D] (got {tuple(x.shape)})")
    if x.shape[-1] != weight.shape[0]:
        raise ValueError("[CausalConv1d] x.shape[-1] must be equal to weight.shape[0].")
    _cuda("causal_conv1d", x, weight, bias, residual, initial_state, cu_seqlens)
    B, T, D = x.shape
    W = weight.shape[1]
    x = x.contiguous()
    w = weight.contiguous()
    b = None if bias is None else bias.to(w.dtype).contiguous()
    r = None if residual is None else residual.to(x.dtype).contiguous()
    if r is not None and r.shape != x.shape:
        raise ValueError(f"[CausalConv1d] residual {tuple(r.shape)} must match x {tuple(x.shape)}")
    cu, cu_dt = None, _lib.GDN_I64
    N = B
    if cu_seqlens is not None:
        cu = cu_seqlens if cu_seqlens.dtype in _IDT else cu_seqlens.to(torch.int64)
        cu_dt = _IDT[cu.dtype]
        N = cu.numel() - 1
    h0 = None if initial_state is None else initial_state.contiguous()
    if h0 is not None and tuple(h0.shape) != (N, D, W):
        raise ValueError(f"[CausalConv1d] initial_state {tuple(h0.shape)} must be [N, D, W] = {(N, D, W)}")
    y = torch.empty_like(x)
    args = _lib.Conv1dArgs(
        x=_ptr(x), weight=_ptr(w), bias=_ptr(b), residual=_ptr(r), initial_state=_ptr(h0), y=_ptr(y),
        cu_seqlens=_ptr(cu), B=B, T=T, N=N, D=D, W=W, x_dtype=_fdt(x, "x"), w_dtype=_fdt(w, "weight"),
        state_dtype=_fdt(h0, "initial_state") if h0 is not None else _lib.GDN_F32, cu_dtype=cu_dt,
        activation=_act(activation))
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().gdn_causal_conv1d_fwd(args, _stream(x.device)))
    return y, None


def causal_conv1d_fn(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    conv_states: torch.Tensor,
    query_start_loc: torch.Tensor,
    cache_indices: torch.Tensor | None = None,
    has_initial_state: torch.Tensor | None = None,
    activation: str | None = "silu",
    pad_slot_id: int = -1,
    null_block_id: int = 0,
    block_idx_first_scheduled_token: torch.Tensor | None = None,
    block_idx_last_scheduled_token: torch.Tensor | None = None,
    initial_state_idx: torch.Tensor | None = None,
    num_computed_tokens: torch.Tensor | None = None,
    block_size_to_align=0,
    metadata=None,
    validate_data=False,
):
    """Continuous-batching causal conv1d (``triton_ops.py:366-459``).

    x ``(dim, total_tokens)`` channel-last (``x.stride(0) == 1``; other
    layouts are copied), weight ``(dim, W)`` with W <= 4, conv_states
    ``(lines, dim, >= W-1)`` with unit channel stride, updated in place to
    each processed sequence's last W-1 inputs.  Returns ``out`` shaped and
    strided like x."""
    if weight is not None and x.shape[0] != weight.shape[0]:
        raise ValueError("[CausalConv1d] x.shape[0] must be equal to weight.shape[0].")
    if weight is not None and weight.shape[-1] > 4:
        raise ValueError("[CausalConv1d] weight.shape[-1] must be less than or equal to 4.")
    if weight is None or x.dim() != 2:
        raise ValueError("[CausalConv1d] x must be (dim, tokens) and weight (dim, width)")
    _cuda("causal_conv1d_fn", x, weight, bias, conv_states, query_start_loc, cache_indices, has_initial_state)
    dim, total = x.shape
    if x.stride(0) != 1 and total > 1:
        x = x.t().contiguous().t()  # channel-last storage [tokens, dim]
    out = torch.empty_like(x)
    if out.stride(0) != 1 and total > 1:
        out = torch.empty(total, dim, dtype=x.dtype, device=x.device).t()
    args, _keep = _fn_args(x, weight, bias, conv_states, query_start_loc, cache_indices, has_initial_state,
                           activation, pad_slot_id, null_block_id, block_idx_first_scheduled_token,
                           block_idx_last_scheduled_token, initial_state_idx, num_computed_tokens,
                           block_size_to_align, out)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().gdn_causal_conv1d_fn(args, _stream(x.device)))
    return out


def causal_conv1d_update(
    x: torch.Tensor,
    cache: torch.Tensor,
    residual: torch.Tensor | None = None,
    weight: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    activation: str | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """One decode token per sequence (``triton/conv/ops.py:584-644``).

    x ``(N, D)``, ``(N, 1, D)`` or ``(1, N, D)``; cache ``[N, D, W]``
    (contiguous) holds the last W inputs and is shifted in place.  Returns
    ``(y, cache)`` with y shaped like x."""
    if x.dim() == 2:
        N, D = x.shape
        sxn = x.stride(0)
    elif x.dim() == 3 and x.shape[0] == 1:
        N, D = x.shape[1], x.shape[2]
        sxn = x.stride(1)
    elif x.dim() == 3:
        N, D = x.shape[0], x.shape[2]
        sxn = x.stride(0)
    else:
        raise ValueError(f"Unsupported input shape: {x.shape}")
    _cuda("causal_conv1d_update", x, cache, residual, weight, bias)
    if x.stride(-1) != 1 or (N > 1 and sxn < D):
        x = x.contiguous()
        sxn = D
    W = weight.shape[1] if weight is not None else (cache.shape[-1] if cache is not None else None)
    if W is None:
        raise ValueError("[CausalConv1d] weight or cache is required")
    if cache is not None:
        if tuple(cache.shape) != (N, D, W) or not cache.is_contiguous():
            raise ValueError(f"[CausalConv1d] cache must be a contiguous [N, D, W] = {(N, D, W)} tensor")
    w = None if weight is None else weight.contiguous()
    b = None if bias is None else bias.to(w.dtype if w is not None else bias.dtype).contiguous()
    r = None if residual is None else residual.to(x.dtype).reshape(N, D).contiguous()
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    args = _lib.Conv1dUpdateArgs(
        x=_ptr(x), cache=_ptr(cache), residual=_ptr(r), weight=_ptr(w), bias=_ptr(b), y=_ptr(y),
        stride_x_n=sxn if N > 1 else D, N=N, D=D, W=W, x_dtype=_fdt(x, "x"),
        cache_dtype=_fdt(cache, "cache") if cache is not None else _lib.GDN_F32,
        w_dtype=_fdt(w if w is not None else (b if b is not None else x), "weight"), activation=_act(activation))
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().gdn_causal_conv1d_update(args, _stream(x.device)))
    return y, cache
