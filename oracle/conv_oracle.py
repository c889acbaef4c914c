"""CPU restatement of the reference's causal depthwise conv1d ops (test
infrastructure only: the checker for the CUDA kernels, never the product).

Three public ops of ``torch_mlu_ops.triton_ops`` feed the GDN layer of
Qwen3-Next (the short convolution over the concatenated q/k/v channels):

* ``causal_conv1d`` (``triton_ops.py:287-363``) -> ``CausalConv1dFunctionFla``
  -> ``causal_conv1d_fwd_fla`` (``triton/conv/ops.py:35-99``), kernel
  ``tmo_causal_conv1d_fwd_fla_kernel`` (``triton/conv/kernels.py:24-153``);
* ``causal_conv1d_fn`` (``triton_ops.py:366-459``) ->
  ``causal_conv1d_fwd_vllm`` (``triton/conv/ops.py:101-349``), kernel
  ``tmo_causal_conv1d_fwd_vllm_kernel`` (``triton/conv/kernels.py:157-609``);
* ``causal_conv1d_update`` (``triton/conv/ops.py:584-644``), kernel
  ``tmo_causal_conv1d_update_kernel`` (``triton/conv/kernels.py:850-934``).

Everything is computed in float64 with numpy; callers round to the dtype
they compare against.  Each function cites the reference lines it follows.
Pinned against the reference's own kernels run under the Triton CPU
interpreter (``tests/golden/make_golden.py``, fixtures ``conv_*.npz``).
"""

from __future__ import annotations

import numpy as np


def _silu(y):
    return y / (1.0 + np.exp(-y))


def _act(y, activation):
    # ``ACTIVATION == 'swish' or 'silu'`` (kernels.py:131-132, :915-916);
    # causal_conv1d_fn also accepts True (ops.py:170-171)
    if activation in ("silu", "swish", True):
        return _silu(y)
    if activation in (None, False):
        return y
    raise ValueError(f"unsupported activation {activation!r}")


def causal_conv1d(x, weight, bias=None, residual=None, initial_state=None, activation=None,
                  cu_seqlens=None):
    """FLA-layout forward (``kernels.py:24-153``).

    x ``[B, T, D]``; weight ``[D, W]``; bias ``[D]``; residual ``[B, T, D]``;
    initial_state ``[N, D, W]`` whose column j holds token j - W of sequence
    n (column 0 is never read, ``kernels.py:123``); with ``cu_seqlens`` the
    B == 1 row holds N packed sequences.  y_t = sum_i x_{t-W+1+i} w_i (tokens
    before the sequence start come from the initial state or are zero), then
    bias, activation, residual, in that order (``kernels.py:128-141``).
    """
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    B, T, D = x.shape
    W = w.shape[1]
    if cu_seqlens is None:
        spans = [(b, 0, T) for b in range(B)]
    else:
        cu = [int(c) for c in cu_seqlens]
        spans = [(0, cu[i], cu[i + 1]) for i in range(len(cu) - 1)]
    y = np.zeros_like(x)
    for n, (b, bos, eos) in enumerate(spans):
        L = eos - bos
        hist = np.zeros((W - 1, D))
        if initial_state is not None:
            hist = np.asarray(initial_state, np.float64)[n][:, 1:W].T
        ext = np.concatenate([hist, x[b, bos:eos]], axis=0)  # [W-1+L, D]
        acc = np.zeros((L, D))
        for i in range(W):
            acc += ext[i:i + L] * w[:, i]
        if bias is not None:
            acc += np.asarray(bias, np.float64)
        acc = _act(acc, activation)
        if residual is not None:
            acc += np.asarray(residual, np.float64)[b, bos:eos]
        y[b, bos:eos] = acc
    return y


def _cmod(a, b):
    """Integer remainder with the sign of the dividend (the device semantics
    of ``%`` on signed integers in the reference kernel)."""
    return a - b * int(a / b)


def causal_conv1d_fn(x, weight, bias, conv_states, query_start_loc, cache_indices=None,
                     has_initial_state=None, activation="silu", pad_slot_id=-1, null_block_id=0,
                     block_idx_first_scheduled_token=None, block_idx_last_scheduled_token=None,
                     initial_state_idx=None, num_computed_tokens=None, block_size_to_align=0):
    """vLLM-layout forward with a slot-indexed state cache
    (``ops.py:101-349``, ``kernels.py:157-609``).

    x ``(dim, total_tokens)``; weight ``(dim, W)``; conv_states
    ``(lines, dim, >= W-1)`` holding the last W-1 tokens of a sequence
    (column j = token j - (W-1)).  Sequence s uses line ``cache_indices[s]``
    (s when None); a sequence whose line equals ``null_block_id`` is skipped
    (``kernels.py:321``), and so, here, is one whose line equals
    ``pad_slot_id``; an empty sequence gets no program (``ops.py:262-266``)
    and leaves its line alone.  The initial window comes from the line when
    ``has_initial_state[s]`` (``kernels.py:336-366``), else zeros; afterwards
    the line holds the sequence's last W-1 tokens, earlier state shifted in
    when the sequence is shorter (``kernels.py:381-484``).  Output token t is
    sum_i ext_{t+i} w_i + bias, then SiLU (``kernels.py:562-608``).

    Prefix caching (``block_idx_last_scheduled_token`` given,
    ``kernels.py:254-289, 389-417, 519-554``): ``cache_indices`` is
    ``(batch, blocks)``; the initial window comes from line
    ``cache_indices[s, initial_state_idx[s]]``, the final state goes to
    ``cache_indices[s, last[s]]`` (to the initial line when the sequence is
    shorter than W-1), and block j < last[s] - first[s] (when the sequence
    has more than j+1 64-token chunks) stores the W-1 inputs before its
    block-aligned end into ``cache_indices[s, first[s] + j]``; token indices
    there are absolute and negative ones read zero.

    Returns ``(out, new_conv_states, processed)``: out ``(dim, total)`` with
    zeros for skipped sequences, a copy of the updated cache, and a boolean
    mask of processed sequences.
    """
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    dim, total = x.shape
    W = w.shape[1]
    sl = W - 1
    cs = np.array(conv_states, np.float64, copy=True)
    qsl = [int(c) for c in query_start_loc]
    out = np.zeros_like(x)
    processed = []
    apc = block_idx_last_scheduled_token is not None
    for s in range(len(qsl) - 1):
        if apc:
            row = [int(c) for c in np.asarray(cache_indices)[s]]
            line = row[int(initial_state_idx[s])]
            out_line = row[int(block_idx_last_scheduled_token[s])]
        else:
            line = s if cache_indices is None else int(cache_indices[s])
            out_line = line
        if (null_block_id is not None and line == null_block_id) or line == pad_slot_id:
            processed.append(False)
            continue
        a, e = qsl[s], qsl[s + 1]
        L = e - a
        if L == 0:  # no program runs for an empty sequence: its line is left alone
            processed.append(False)
            continue
        processed.append(True)
        init = np.zeros((dim, sl))
        if has_initial_state is not None and bool(has_initial_state[s]):
            init = cs[line][:, :sl].copy()
        ext = np.concatenate([init, x[:, a:e]], axis=1)  # (dim, W-1+L)
        acc = np.zeros((dim, L))
        for i in range(W):
            acc += ext[:, i:i + L] * w[:, i:i + 1]
        if bias is not None:
            acc += np.asarray(bias, np.float64)[:, None]
        out[:, a:e] = _act(acc, activation)
        if L >= sl:
            cs[out_line][:, :sl] = ext[:, L:L + sl]
        else:
            cs[line][:, :sl] = ext[:, L:L + sl]
        if apc:
            first = int(block_idx_first_scheduled_token[s])
            nb = int(block_idx_last_scheduled_token[s]) - first
            B = int(block_size_to_align)
            comp_off = B - _cmod(int(num_computed_tokens[s]), B)
            end_off = _cmod(L - comp_off, B)
            last_full = e - end_off - (B if end_off == 0 else 0)
            nchunks = -(-L // 64)
            for j in range(nb):
                if j + 1 >= nchunks:
                    break
                start = last_full - (nb - j - 1) * B - sl
                blk = np.zeros((dim, sl))
                for u in range(sl):
                    if start + u >= 0:
                        blk[:, u] = x[:, start + u]
                cs[row[first + j]][:, :sl] = blk
    return out, cs, np.array(processed, bool)


def causal_conv1d_update(x, cache, residual=None, weight=None, bias=None, activation=None):
    """One decode step per sequence (``ops.py:584-644``, ``kernels.py:850-934``).

    x ``[N, D]`` (the reference also takes ``[N, 1, D]`` and ``[1, N, D]``);
    cache ``[N, D, W]`` holds the last W inputs.  The cache shifts left by
    one and takes x in its last column (``kernels.py:890-904``); y = sum_j
    cache_j w_j (+ bias), activation, + residual (``kernels.py:906-919``).
    Returns ``(y [N, D], new_cache)``; with ``cache=None`` the window is all
    zeros and no cache is returned (``USE_INITIAL_STATE`` false).
    """
    x = np.asarray(x, np.float64)
    N, D = x.shape
    if cache is None:
        W = np.asarray(weight).shape[1]
        win = np.zeros((N, D, W))
        new = None
    else:
        c = np.asarray(cache, np.float64)
        win = np.concatenate([c[:, :, 1:], x[:, :, None]], axis=2)
        new = win
    if weight is not None:
        y = (win * np.asarray(weight, np.float64)[None]).sum(-1)
    else:
        y = win.sum(-1)
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    y = _act(y, activation)
    if residual is not None:
        y = y + np.asarray(residual, np.float64).reshape(N, D)
    return y, new
