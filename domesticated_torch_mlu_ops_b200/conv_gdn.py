"""Causal conv1d fused into the chunked GDN prefill.

The Qwen3-Next GDN layer runs two ops back to back on a prefill batch: the
short convolution over the projected ``[q | k | v]`` channels
(``causal_conv1d_fn``, ``triton_ops.py:366-459``), then the chunked delta
rule on the q/k/v split of its output (``chunk_gated_delta_rule``,
``triton_ops.py:81-165``).  :func:`causal_conv1d_chunk_gated_delta_rule`
computes both in one pass (``gdn_conv_chunk_fwd``): the prefill's WY kernel
applies the conv (and SiLU) to ``mixed_qkv`` as it loads its q/k/v tiles, so
the conv output does not go through HBM (v not at all; q and k are written
once, for the state kernel).  The results are bit-identical to the two
separate calls, and ``conv_states`` is updated the same way.  The reference
has no single op for the pair.

The fused kernels cover the shapes of that layer: bf16/fp16 data, head
dims 128, width-4 taps, ``conv_states`` in the data dtype.  Other cases run
the two device ops one after the other (same results, no fusion).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .conv import _act, _fn_args, causal_conv1d_fn
from .gdn import (_DT, _IDT, _call, _cuda, _empty_f32, _f32, _ptr, _scale, _stream,
                  chunk_gated_delta_rule)

__all__ = ["causal_conv1d_chunk_gated_delta_rule"]


def _conv_chunk_fwd_impl(x: Tensor, weight: Tensor, bias: Optional[Tensor], conv_states: Tensor,
                         query_start_loc: Tensor, cache_indices: Optional[Tensor],
                         has_initial_state: Optional[Tensor], g: Tensor, beta: Tensor, scale: float,
                         initial_state: Optional[Tensor], output_final_state: bool, num_k_heads: int,
                         num_v_heads: int, head_k_dim: int, head_v_dim: int, activation: int,
                         pad_slot_id: int, null_block_id: int, has_null_block: bool,
                         block_idx_first: Optional[Tensor], block_idx_last: Optional[Tensor],
                         initial_state_idx: Optional[Tensor], num_computed_tokens: Optional[Tensor],
                         block_size_to_align: int, use_qk_l2norm: bool,
                         check_errors: bool) -> tuple[Tensor, Tensor]:
    """Fused prefill on prepared inputs: x ``(dim, tokens)`` channel-last,
    g/beta fp32 ``[1, T, HV]``, initial_state fp32 ``[N, HV, K, V]`` or None.
    Returns ``(o [1, T, HV, V], final_state)`` (an empty tensor when not
    requested) and updates conv_states in place."""
    dim, total = x.shape
    H, HV, K, V = num_k_heads, num_v_heads, head_k_dim, head_v_dim
    dev = x.device
    act = "silu" if activation == _lib.GDN_ACT_SILU else None
    cargs, keep = _fn_args(x, weight, bias, conv_states, query_start_loc, cache_indices, has_initial_state,
                           act, pad_slot_id, null_block_id if has_null_block else None, block_idx_first,
                           block_idx_last, initial_state_idx, num_computed_tokens, block_size_to_align, None)
    qsl = keep[2]
    N = qsl.numel() - 1
    o = torch.empty(1, total, HV, V, dtype=x.dtype, device=dev)
    ht = torch.empty(N, HV, K, V, dtype=torch.float32, device=dev) if output_final_state else None
    args = _lib.ChunkArgs(
        q=None, k=None, v=None, g=_ptr(g), beta=_ptr(beta), initial_state=_ptr(initial_state), o=_ptr(o),
        final_state=_ptr(ht), cu_seqlens=_ptr(qsl), workspace=None, workspace_bytes=0,
        B=1, T=total, N=N, H=H, HV=HV, K=K, V=V, qkv_dtype=_DT[x.dtype], cu_dtype=_IDT[qsl.dtype],
        scale=float(scale), use_qk_l2norm=int(use_qk_l2norm), state_v_first=0, force_generic=0)
    lib = _lib.load()
    nbytes = lib.gdn_conv_chunk_workspace_size(ctypes.byref(args))
    if nbytes == 0:
        _lib.check(_lib.GDN_ERR_INVALID)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    args.workspace = ctypes.c_void_p(ws.data_ptr())
    args.workspace_bytes = nbytes
    with torch.cuda.device(dev):
        _lib.check(lib.gdn_conv_chunk_fwd(ctypes.byref(args), ctypes.byref(cargs), _stream(dev)))
        if check_errors:
            _lib.check(lib.gdn_chunk_check_device_error(args.workspace, _stream(dev)))
    return o, (ht if ht is not None else _empty_f32(dev))


_conv_chunk_fwd_op = torch.library.custom_op("gdn_b200::conv_chunk_fwd", mutates_args=("conv_states",),
                                             device_types="cuda")(_conv_chunk_fwd_impl)


@_conv_chunk_fwd_op.register_fake
def _(x, weight, bias, conv_states, query_start_loc, cache_indices, has_initial_state, g, beta, scale,
      initial_state, output_final_state, num_k_heads, num_v_heads, head_k_dim, head_v_dim, activation,
      pad_slot_id, null_block_id, has_null_block, block_idx_first, block_idx_last, initial_state_idx,
      num_computed_tokens, block_size_to_align, use_qk_l2norm, check_errors):
    total = x.shape[1]
    o = x.new_empty((1, total, num_v_heads, head_v_dim))
    if not output_final_state:
        return o, x.new_empty((0,), dtype=torch.float32)
    N = query_start_loc.shape[0] - 1
    return o, x.new_empty((N, num_v_heads, head_k_dim, head_v_dim), dtype=torch.float32)


def _fusable(x, weight, bias, conv_states, H, HV, K, V):
    # (allocations start 256-byte aligned, so the storage offset decides x's alignment)
    f16 = (torch.bfloat16, torch.float16)
    return (x.dtype in f16 and weight.dtype == x.dtype and conv_states.dtype == x.dtype
            and (bias is None or bias.dtype == x.dtype) and weight.shape[1] == 4 and K == 128 and V == 128
            and x.storage_offset() * x.element_size() % 16 == 0 and (x.shape[1] <= 1 or x.stride(1) % 8 == 0))


def causal_conv1d_chunk_gated_delta_rule(
    mixed_qkv: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    conv_states: torch.Tensor,
    query_start_loc: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    num_k_heads: int,
    num_v_heads: int,
    head_k_dim: int = 128,
    head_v_dim: int = 128,
    scale: float | None = None,
    initial_state: torch.Tensor | None = None,
    output_final_state: bool = False,
    cache_indices: torch.Tensor | None = None,
    has_initial_state: torch.Tensor | None = None,
    activation: str | None = "silu",
    pad_slot_id: int = -1,
    null_block_id: int | None = 0,
    block_idx_first_scheduled_token: torch.Tensor | None = None,
    block_idx_last_scheduled_token: torch.Tensor | None = None,
    initial_state_idx: torch.Tensor | None = None,
    num_computed_tokens: torch.Tensor | None = None,
    block_size_to_align: int = 0,
    use_qk_l2norm_in_kernel: bool = False,
    *,
    check_errors: bool = False,
):
    """``causal_conv1d_fn`` followed by ``chunk_gated_delta_rule`` in one pass.

    mixed_qkv ``(dim, tokens)`` channel-last as ``causal_conv1d_fn`` takes it
    (``x.stride(0) == 1``), dim = ``2 * num_k_heads * head_k_dim +
    num_v_heads * head_v_dim`` channels ``[q heads | k heads | v heads]``;
    weight ``(dim, W)``, bias, conv_states, query_start_loc, cache_indices,
    has_initial_state, activation, pad_slot_id, null_block_id and the prefix
    caching arguments as for ``causal_conv1d_fn``; g, beta ``[1, tokens, HV]``,
    scale, initial_state ``[N, HV, K, V]``, output_final_state and
    use_qk_l2norm_in_kernel as for ``chunk_gated_delta_rule`` with
    ``cu_seqlens = query_start_loc``.

    Returns ``(o [1, tokens, HV, V], final_state or None)``; conv_states is
    updated in place.  Equal, bit for bit, to::

        y = causal_conv1d_fn(mixed_qkv, weight, bias, conv_states, query_start_loc, ...)
        q, k, v = (y.t()[:, a:b].reshape(1, tokens, heads, d) for each part)
        chunk_gated_delta_rule(q, k, v, g, beta, scale, initial_state, output_final_state,
                               cu_seqlens=query_start_loc, use_qk_l2norm_in_kernel=...)
    """
    H, HV, K, V = int(num_k_heads), int(num_v_heads), int(head_k_dim), int(head_v_dim)
    if mixed_qkv.dim() != 2 or weight.dim() != 2 or mixed_qkv.shape[0] != weight.shape[0]:
        raise ValueError("mixed_qkv must be (dim, tokens) and weight (dim, width)")
    dim, total = mixed_qkv.shape
    if dim != 2 * H * K + HV * V:
        raise ValueError(f"mixed_qkv has {dim} channels; 2*H*K + HV*V = {2 * H * K + HV * V}")
    if HV % H != 0:
        raise ValueError(f"num_v_heads={HV} must be a multiple of num_k_heads={H}")
    if weight.shape[1] > 4:
        raise ValueError("[CausalConv1d] weight.shape[-1] must be less than or equal to 4.")
    if g.shape != (1, total, HV) or beta.shape != (1, total, HV):
        raise ValueError(f"g {tuple(g.shape)} and beta {tuple(beta.shape)} must be (1, {total}, {HV})")
    _cuda("causal_conv1d_chunk_gated_delta_rule", mixed_qkv, weight, bias, conv_states, query_start_loc, g,
          beta, initial_state, cache_indices, has_initial_state)
    N = query_start_loc.numel() - 1
    if initial_state is not None and tuple(initial_state.shape) != (N, HV, K, V):
        raise ValueError(f"initial_state must be {(N, HV, K, V)}, got {tuple(initial_state.shape)}")
    x = mixed_qkv
    if x.stride(0) != 1 and total > 1:
        x = x.t().contiguous().t()  # channel-last storage [tokens, dim]
    if not _fusable(x, weight, bias, conv_states, H, HV, K, V):
        y = causal_conv1d_fn(x, weight, bias, conv_states, query_start_loc, cache_indices, has_initial_state,
                             activation, pad_slot_id, null_block_id, block_idx_first_scheduled_token,
                             block_idx_last_scheduled_token, initial_state_idx, num_computed_tokens,
                             block_size_to_align)
        yt = y.t()
        q = yt[:, :H * K].reshape(1, total, H, K)
        k = yt[:, H * K:2 * H * K].reshape(1, total, H, K)
        v = yt[:, 2 * H * K:].reshape(1, total, HV, V)
        return chunk_gated_delta_rule(q, k, v, g, beta, scale, initial_state, output_final_state,
                                      cu_seqlens=query_start_loc, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
                                      check_errors=check_errors)
    qsl = query_start_loc if query_start_loc.dtype in _IDT else query_start_loc.to(torch.int32)
    o, ht = _call(
        torch.ops.gdn_b200.conv_chunk_fwd, _conv_chunk_fwd_impl, x, weight, bias, conv_states, qsl,
        cache_indices, has_initial_state, _f32(g), _f32(beta), _scale(scale), _f32(initial_state),
        bool(output_final_state), H, HV, K, V, _act(activation), int(pad_slot_id),
        0 if null_block_id is None else int(null_block_id), null_block_id is not None,
        block_idx_first_scheduled_token, block_idx_last_scheduled_token, initial_state_idx,
        num_computed_tokens, int(block_size_to_align or 0), bool(use_qk_l2norm_in_kernel), bool(check_errors))
    return o, (ht if output_final_state else None)
