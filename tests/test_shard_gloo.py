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
