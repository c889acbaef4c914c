"""Host-side multi-GPU logic on CPU: the (sequence, v-head) partitioners and
the final gather, run as two gloo ranks with the CPU oracle standing in for
the CUDA op (no GPU involved)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from domesticated_torch_mlu_ops_b200 import shard


def test_partition_sequences_balances_tokens():
    lens = [512, 8000, 3000, 3000, 100, 7000, 2500]
    parts = shard.partition_sequences(lens, 3)
    assert sorted(i for p in parts for i in p) == list(range(len(lens)))
    loads = [sum(lens[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(lens)
    assert shard.partition_sequences(lens, 3) == parts  # deterministic on every rank


def test_partition_heads_keeps_qk_groups():
    assert shard.partition_heads(16, 32, 4) == [(0, 4), (4, 8), (8, 12), (12, 16)]
    assert shard.partition_heads(3, 6, 2) == [(0, 2), (2, 3)]
    assert shard.partition_heads(2, 4, 4)[3] == (2, 2)
    with pytest.raises(ValueError):
        shard.partition_heads(3, 4, 2)


def _oracle_op(q, k, v, g, beta, initial_state=None, cu_seqlens=None, **kw):
    f = lambda t: None if t is None else t.double().numpy()
    o, ht = oracle.chunk_gated_delta_rule(f(q), f(k), f(v), f(g), f(beta), None, f(initial_state),
                                          True, None if cu_seqlens is None else cu_seqlens.numpy(),
                                          True)
    return torch.from_numpy(o), torch.from_numpy(ht)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, inputs, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k, v, g, beta, h0, cu = inputs
    ids, o, ht = shard.sharded_chunk_gated_delta_rule(_oracle_op, q, k, v, g, beta, cu, h0, rank, world)
    full_o, full_h = shard.gather_outputs(ids, o, ht, cu, world)
    if rank == 0:
        torch.save({"o": full_o, "h": full_h}, out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_prefill_two_gloo_ranks(tmp_path):
    rng = np.random.default_rng(6)
    lens = [70, 5, 130, 64, 40]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]))
    T, H, HV, K, V = int(cu[-1]), 2, 4, 16, 8
    t = lambda *s: torch.from_numpy(rng.standard_normal(s))
    q, k, v = t(1, T, H, K), t(1, T, H, K), t(1, T, HV, V)
    g = torch.nn.functional.logsigmoid(t(1, T, HV))
    beta = torch.sigmoid(t(1, T, HV))
    h0 = t(len(lens), HV, K, V) * 0.1
    out = tmp_path / "gathered.pt"
    mp.start_processes(_worker, args=(2, _free_port(), (q, k, v, g, beta, h0, cu), str(out)),
                       nprocs=2, join=True, start_method="spawn")
    got = torch.load(out)
    ref_o, ref_h = _oracle_op(q, k, v, g, beta, initial_state=h0, cu_seqlens=cu)
    assert torch.allclose(got["o"], ref_o, atol=1e-10)
    assert torch.allclose(got["h"], ref_h, atol=1e-10)



_GATHER_PARTS = [[[2, 0], [1, 3]], [[0, 1], [2, 3]], [[0, 1, 2, 3], []]]
_GATHER_LENS = [5, 9, 1, 6]


def _gather_worker(rank, world, port, full_o, full_h, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lens = _GATHER_LENS
    cu = np.concatenate([[0], np.cumsum(lens)])
    got = []
    for parts in _GATHER_PARTS:
        p = parts[rank]
        o = torch.cat([full_o[:, cu[i]:cu[i + 1]] for i in p], 1) if p else full_o[:, :0]
        plan = shard.OutputGather(parts, lens, "cpu", rank, state_shape=(3, 4, 5))
        got.append(plan(o, full_h[p] if p else None))
        rows = max(sum(lens[i] for i in q) for q in parts)
        assert plan.gathered_bytes(o) == world * rows * 3 * 7 * 8 + world * max(map(len, parts)) * 60 * 4
        to1 = shard.OutputGather(parts, lens, "cpu", rank, state_shape=(3, 4, 5), dst=1)
        r1 = to1(o, full_h[p] if p else None)
        got.append(r1 if rank == 1 else (full_o, full_h))  # rank 0 receives nothing
        assert rank == 1 or r1 == (None, None)
    torch.save(got, f"{out_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


def test_device_gather_two_gloo_ranks(tmp_path):
    """OutputGather on two gloo ranks: padded all-gather (and gather to rank
    1), then the row and state permutation back into sequence order,
    identical on both ranks, for uneven shards, contiguous shards and a rank
    with no sequences."""
    rng = np.random.default_rng(11)
    full_o = torch.from_numpy(rng.standard_normal((1, sum(_GATHER_LENS), 3, 7)))
    full_h = torch.from_numpy(rng.standard_normal((len(_GATHER_LENS), 3, 4, 5))).float()
    out = tmp_path / "g"
    mp.start_processes(_gather_worker, args=(2, _free_port(), full_o, full_h, str(out)),
                       nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        for o, h in torch.load(f"{out}.{r}"):
            assert torch.equal(o, full_o)
            assert torch.equal(h, full_h)


def _head_worker(rank, world, port, inputs, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k, v, g, beta, h0 = inputs
    H, HV = q.shape[2], v.shape[2]
    rng_ = shard.partition_heads(H, HV, world)[rank]
    ql, kl, vl, gl, bl, hl = shard.head_slices(q, k, v, g, beta, h0, rng_, HV // H)
    o, ht = _oracle_op(ql, kl, vl, gl, bl, initial_state=hl)
    full_o, full_h = shard.HeadGather(world, rank, dst=0)(o, ht)
    if rank == 0:
        torch.save({"o": full_o, "h": full_h}, out_path)
    else:
        assert full_o is None and full_h is None
    dist.barrier()
    dist.destroy_process_group()


def test_head_split_prefill_two_gloo_ranks(tmp_path):
    """One sequence split by v-head groups (each rank owns whole q/k heads),
    run by the oracle on two gloo ranks and gathered on rank 0, equals the
    unsplit sequence."""
    rng = np.random.default_rng(12)
    T, H, HV, K, V = 150, 4, 8, 16, 8
    t = lambda *s: torch.from_numpy(rng.standard_normal(s))
    q, k, v = t(1, T, H, K), t(1, T, H, K), t(1, T, HV, V)
    g = torch.nn.functional.logsigmoid(t(1, T, HV))
    beta = torch.sigmoid(t(1, T, HV))
    h0 = t(1, HV, K, V) * 0.1
    out = tmp_path / "heads.pt"
    mp.start_processes(_head_worker, args=(2, _free_port(), (q, k, v, g, beta, h0), str(out)),
                       nprocs=2, join=True, start_method="spawn")
    got = torch.load(out)
    ref_o, ref_h = _oracle_op(q, k, v, g, beta, initial_state=h0)
    assert torch.allclose(got["o"], ref_o, atol=1e-10)
    assert torch.allclose(got["h"], ref_h, atol=1e-10)
