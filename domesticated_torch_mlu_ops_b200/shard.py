"""Multi-GPU partitioning of the GDN forward: one process per GPU.

The recurrence of every (sequence, v-head) pair is independent
(``triton/fla/fused_recurrent_fn.py:51-52``, ``triton/fla/chunk_delta_h.py:58-59``),
so work splits across ranks with no collective on the data path:

* many sequences -> whole sequences per rank, longest-first greedy bin
  packing by token count (:func:`partition_sequences`);
* one long sequence -> groups of v-heads that share a q/k head, so no rank
  needs a q/k head another rank also reads (:func:`partition_heads`).

:func:`gather_outputs` is the optional final gather (``torch.distributed``;
NCCL on GPUs, gloo on CPU) when one rank needs every output.
"""

from __future__ import annotations

import heapq

import torch


def partition_sequences(lengths, world_size: int) -> list[list[int]]:
    """Sequence indices per rank, balancing total tokens (LPT greedy).

    Ties break on the lower rank, so every rank computes the same answer
    from the same lengths."""
    lengths = [int(x) for x in lengths]
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    heap = [(0, r) for r in range(world_size)]
    parts: list[list[int]] = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + lengths[i], r))
    return [sorted(p) for p in parts]


def partition_heads(H: int, HV: int, world_size: int) -> list[tuple[int, int]]:
    """[start, stop) q/k-head ranges per rank; rank r owns v-heads
    [start * G, stop * G) with G = HV // H.  Ranks beyond H get empty ranges."""
    if HV % H:
        raise ValueError(f"HV={HV} must be a multiple of H={H}")
    base, extra = divmod(H, world_size)
    out, s = [], 0
    for r in range(world_size):
        n = base + (1 if r < extra else 0)
        out.append((s, s + n))
        s += n
    return out


def pack_sequences(xs, seq_ids, cu_seqlens):
    """Concatenate the tokens of ``seq_ids`` (packed along dim 1 of each
    tensor in ``xs``, B == 1) and return (tensors, local cu_seqlens)."""
    cu = [int(c) for c in cu_seqlens]
    spans = [(cu[i], cu[i + 1]) for i in seq_ids]
    out = [torch.cat([x[:, s:e] for s, e in spans], dim=1) if spans else x[:, :0] for x in xs]
    local = [0]
    for s, e in spans:
        local.append(local[-1] + (e - s))
    return out, torch.tensor(local, dtype=torch.int64, device=xs[0].device)


def sharded_chunk_gated_delta_rule(op, q, k, v, g, beta, cu_seqlens, initial_state, rank: int,
                                   world_size: int, **kw):
    """Run ``op`` (a ``chunk_gated_delta_rule``-compatible callable) on this
    rank's share of the packed sequences.  Returns (seq_ids, o, final_state)
    for the local sequences."""
    lengths = [int(cu_seqlens[i + 1] - cu_seqlens[i]) for i in range(len(cu_seqlens) - 1)]
    ids = partition_sequences(lengths, world_size)[rank]
    (ql, kl, vl, gl, bl), cul = pack_sequences([q, k, v, g, beta], ids, cu_seqlens)
    h0 = initial_state[ids] if initial_state is not None else None
    if not ids:
        return ids, vl, None
    o, ht = op(ql, kl, vl, gl, bl, initial_state=h0, cu_seqlens=cul.to(q.device), **kw)
    return ids, o, ht


def gather_outputs(ids, o, ht, cu_seqlens, world_size: int):
    """All-gather every rank's (ids, o, final_state) and reassemble the full
    packed output ``[1, T, HV, V]`` and states ``[N, ...]`` on every rank."""
    import torch.distributed as dist

    pieces = [None] * world_size
    dist.all_gather_object(pieces, (ids, o.cpu(), None if ht is None else ht.cpu()))
    cu = [int(c) for c in cu_seqlens]
    N = len(cu) - 1
    shape = list(o.shape)
    shape[1] = cu[-1]
    full_o = torch.empty(shape, dtype=o.dtype)
    full_h = None
    for rid, ro, rh in pieces:
        off = 0
        for j, i in enumerate(rid):
            n = cu[i + 1] - cu[i]
            full_o[:, cu[i]:cu[i + 1]] = ro[:, off:off + n]
            off += n
            if rh is not None:
                if full_h is None:
                    full_h = torch.empty((N,) + tuple(rh.shape[1:]), dtype=rh.dtype)
                full_h[i] = rh[j]
    return full_o, full_h
