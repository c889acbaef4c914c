"""Multi-GPU partitioning of the GDN forward: one process per GPU.

The recurrence of every (sequence, v-head) pair is independent
(``triton/fla/fused_recurrent_fn.py:51-52``, ``triton/fla/chunk_delta_h.py:58-59``),
so work splits across ranks with no collective on the data path:

* many sequences -> whole sequences per rank, longest-first greedy bin
  packing by token count (:func:`partition_sequences`);
* one long sequence -> groups of v-heads that share a q/k head, so no rank
  needs a q/k head another rank also reads (:func:`partition_heads`).

:func:`gather_outputs` is the optional final gather through host memory
(``all_gather_object``), and :class:`OutputGather` the same gather kept on the
device: one ``gather`` to a chosen rank (or ``all_gather_into_tensor`` onto
every rank) of the packed outputs and one of the final states (NCCL over
NVLink on GPUs, gloo on CPU), then a row permutation back into sequence
order.  :class:`HeadGather` reassembles a sequence split by v-head groups.
"""

from __future__ import annotations

import heapq
import math

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


def head_slices(q, k, v, g, beta, initial_state, head_range, G: int):
    """This rank's tensors for q/k heads ``[h0, h1)`` and their v-heads
    ``[h0 * G, h1 * G)`` (states ``[N, HV, ...]`` sliced on dim 1)."""
    h0, h1 = head_range
    sl = slice(h0 * G, h1 * G)
    return (q[:, :, h0:h1].contiguous(), k[:, :, h0:h1].contiguous(), v[:, :, sl].contiguous(),
            g[:, :, sl].contiguous(), beta[:, :, sl].contiguous(),
            None if initial_state is None else initial_state[:, sl].contiguous())


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


def _gather_rows(send, world: int, dst: int, rank: int, group=None):
    """``[world * rows, ...]`` on rank ``dst`` (None elsewhere) from every
    rank's ``[rows, ...]`` tensor."""
    import torch.distributed as dist

    if rank != dst:
        dist.gather(send, None, dst=dst, group=group)
        return None
    out = send.new_empty((world * send.shape[0],) + tuple(send.shape[1:]))
    dist.gather(send, list(out.chunk(world)), dst=dst, group=group)
    return out


def _all_gather_rows(send, world: int, group=None):
    """``[world * rows, ...]`` from every rank's ``[rows, ...]`` tensor."""
    import torch.distributed as dist

    out = send.new_empty((world * send.shape[0],) + tuple(send.shape[1:]))
    try:
        dist.all_gather_into_tensor(out, send, group=group)
    except (RuntimeError, NotImplementedError):  # backends without the fused form
        dist.all_gather(list(out.chunk(world)), send, group=group)
    return out


class OutputGather:
    """Device-side gather of sharded prefill outputs onto one rank or every rank.

    ``parts[r]`` lists the sequences rank ``r`` computed, in the order its
    packed output holds them (:func:`partition_sequences` or a contiguous
    split; every rank builds the same plan, so shard sizes need no message),
    and ``lengths[i]`` the token count of sequence ``i``.  Each call pads this
    rank's rows to the longest shard, all-gathers outputs and (when
    ``state_shape``, the per-sequence state dims, is given) final states, and
    returns ``o [1, sum(lengths), HV, V]`` in sequence order (packed, as with
    ``cu_seqlens``) and ``final_state [N, *state_shape]`` (or None).  Every
    rank takes the same collectives: a rank without sequences passes an empty
    output and ``ht=None``.  When the shards are already contiguous and
    equal, the permutation is skipped.  With ``dst`` set, only that rank
    receives (``gather`` instead of ``all_gather``: the other ranks only send
    their shard and get ``(None, None)``); ``dst=None`` gives every rank the
    whole output.
    """

    def __init__(self, parts, lengths, device, rank: int, state_shape=None, group=None, dst=None):
        self.dst = dst
        self.parts = [list(p) for p in parts]
        self.lengths = [int(x) for x in lengths]
        self.world = len(self.parts)
        self.rank = rank
        self.group = group
        self.state_shape = None if state_shape is None else tuple(int(x) for x in state_shape)
        N = len(self.lengths)
        self.tok = [sum(self.lengths[i] for i in p) for p in self.parts]
        self.rows = max(self.tok) if self.tok else 0
        self.nseq = max((len(p) for p in self.parts), default=0)
        cu = [0]
        for n in self.lengths:
            cu.append(cu[-1] + n)
        row_src = [0] * cu[-1]  # packed row -> row of the gathered buffer
        seq_src = [0] * N  # sequence -> slot of the gathered state buffer
        for r, p in enumerate(self.parts):
            off = r * self.rows
            for j, i in enumerate(p):
                row_src[cu[i]:cu[i + 1]] = range(off, off + self.lengths[i])
                off += self.lengths[i]
                seq_src[i] = r * self.nseq + j
        ident = row_src == list(range(cu[-1])) and seq_src == list(range(N))
        self.total = cu[-1]
        self.row_perm = None if ident else torch.tensor(row_src, dtype=torch.int64, device=device)
        self.seq_perm = None if ident else torch.tensor(seq_src, dtype=torch.int64, device=device)

    def gathered_bytes(self, o) -> int:
        """Bytes the receiving rank (each rank, without ``dst``) gets per call
        (padding included) for outputs shaped like ``o``."""
        n = self.world * self.rows * math.prod(o.shape[2:]) * o.element_size()
        if self.state_shape is not None:
            n += self.world * self.nseq * math.prod(self.state_shape) * 4
        return n

    def _collect(self, send):
        if self.dst is None:
            return _all_gather_rows(send, self.world, self.group)
        return _gather_rows(send, self.world, self.dst, self.rank, self.group)

    def __call__(self, o, ht=None):
        rows = o.reshape((o.shape[0] * o.shape[1],) + tuple(o.shape[2:]))
        if rows.shape[0] != self.tok[self.rank]:
            raise ValueError(f"rank {self.rank} holds {rows.shape[0]} rows, the plan says "
                             f"{self.tok[self.rank]}")
        if rows.shape[0] < self.rows:
            pad = rows.new_zeros((self.rows - rows.shape[0],) + tuple(rows.shape[1:]))
            rows = torch.cat([rows, pad])
        full = self._collect(rows.contiguous())
        st = None
        if self.state_shape is not None:
            st = ht if ht is not None else o.new_zeros((0,) + self.state_shape, dtype=torch.float32)
            if tuple(st.shape[1:]) != self.state_shape:
                raise ValueError(f"final states {tuple(st.shape)} do not match the plan's {self.state_shape}")
            if st.shape[0] < self.nseq:
                st = torch.cat([st, st.new_zeros((self.nseq - st.shape[0],) + tuple(st.shape[1:]))])
            st = self._collect(st.contiguous())
        if full is None:  # not the receiving rank
            return None, None
        if self.row_perm is not None:
            full = full.index_select(0, self.row_perm)
        else:
            full = full[:self.total]
        full_o = full.unsqueeze(0)
        if st is None:
            return full_o, None
        fh = st.index_select(0, self.seq_perm) if self.seq_perm is not None else st[:len(self.lengths)]
        return full_o, fh


class HeadGather:
    """Gather of a single-sequence prefill split by v-head groups
    (:func:`partition_heads` with equal groups): every rank holds
    ``o [B, T, HV / world, V]`` and ``final_state [N, HV / world, ...]``;
    rank ``dst`` receives ``o [B, T, HV, V]`` and ``final_state [N, HV, ...]``
    (one ``gather`` of each, then a transpose of the rank axis into the head
    axis on the device); ``dst=None`` gives every rank the result."""

    def __init__(self, world: int, rank: int, group=None, dst=0):
        self.world, self.rank, self.group, self.dst = world, rank, group, dst

    def _collect(self, x):
        x = x.contiguous()
        rows = x.reshape((1,) + tuple(x.shape))
        if self.dst is None:
            full = _all_gather_rows(rows, self.world, self.group)
        else:
            full = _gather_rows(rows, self.world, self.dst, self.rank, self.group)
        return full

    def __call__(self, o, ht=None):
        fo = self._collect(o)              # [world, B, T, HVr, V]
        fh = None if ht is None else self._collect(ht)  # [world, N, HVr, ...]
        if fo is None:
            return None, None
        w, B, T, HVr, V = fo.shape
        full_o = fo.permute(1, 2, 0, 3, 4).reshape(B, T, w * HVr, V)
        full_h = None
        if fh is not None:
            N = fh.shape[1]
            full_h = fh.transpose(0, 1).reshape((N, w * fh.shape[2]) + tuple(fh.shape[3:]))
        return full_o, full_h

    def gathered_bytes(self, o, ht=None) -> int:
        n = self.world * o.numel() * o.element_size()
        if ht is not None:
            n += self.world * ht.numel() * ht.element_size()
        return n
