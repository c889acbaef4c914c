"""Parity of the CUDA backward (``gdn_chunk_bwd``) with the reference's
backward fixtures and with the float64 autograd oracle."""

import glob
import os

import numpy as np
import pytest
import torch

from oracle import gdn_bwd_oracle
from gdn_testutil import make_inputs, np64, rel_rms

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FP32_TOL = 1e-4   # rel RMS, fp32 kernels vs fp32 reference / fp64 oracle
BF16_TOL = 1.5e-2  # rel RMS of bf16-rounded dq, dk, dv (fp32 dg, db, dh0 tighter)


def _ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import domesticated_torch_mlu_ops_b200 as ops
    return ops


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "bwd_*.npz"))), ids=os.path.basename)
def test_bwd_matches_reference_fixture(path):
    ops = _ops()
    d = dict(np.load(path))
    dev = "cuda"
    t = {k: torch.from_numpy(d[k]).to(dev) for k in ("q", "k", "v", "g", "beta", "do")}
    h0 = torch.from_numpy(d["h0"]).to(dev) if d["h0"].size else None
    dht = torch.from_numpy(d["dht"]).to(dev) if d["dht"].size else None
    cu = torch.from_numpy(d["cu_seqlens"]).to(dev) if d["cu_seqlens"].size else None
    dq, dk, dv, db, dg, dh0 = ops.chunk_gated_delta_rule_bwd(
        t["q"], t["k"], t["v"], t["g"], t["beta"], float(d["scale"]), h0, t["do"], dht, cu_seqlens=cu)
    torch.cuda.synchronize()
    for name, mine in (("dq", dq), ("dk", dk), ("dv", dv), ("db", db), ("dg", dg)):
        assert rel_rms(np64(mine), d[name]) < FP32_TOL, name
    if h0 is not None:
        assert rel_rms(np64(dh0), d["dh0"]) < FP32_TOL
    else:
        assert dh0 is None


CASES = [
    # (name, dtype, B, T, H, HV, K, V, cu, h0, dht, l2norm, v_first)
    ("gva_varlen_empty", torch.float32, 1, 200, 2, 4, 64, 32, [0, 0, 64, 130, 130, 200], True, True, True, False),
    ("k128_vfirst", torch.float32, 2, 150, 1, 2, 128, 128, None, True, True, False, True),
    ("odd_dims", torch.float32, 1, 97, 3, 3, 40, 24, None, False, True, False, False),
    ("bf16_qwen_like", torch.bfloat16, 1, 256, 2, 4, 128, 128, [0, 100, 256], True, True, True, False),
    ("fp16_no_state", torch.float16, 2, 80, 2, 2, 64, 64, None, False, False, True, False),
    # the tcgen05 backward (16-bit, K = V = 128): V-first states, empty and short sequences, no L2 norm
    ("bf16_tc_vfirst_varlen", torch.bfloat16, 1, 300, 2, 4, 128, 128, [0, 0, 1, 65, 65, 300], True, True, True,
     True),
    ("fp16_tc_gva_nonorm", torch.float16, 2, 130, 1, 2, 128, 128, None, False, True, False, False),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_bwd_matches_oracle(case):
    ops = _ops()
    name, dt, B, T, H, HV, K, V, cu_l, use_h0, use_dht, l2, vfirst = case
    cu = torch.tensor(cu_l, dtype=torch.int32, device="cuda") if cu_l is not None else None
    N = B if cu is None else len(cu_l) - 1
    q, k, v, g, beta, h0 = make_inputs(7 + len(name), B, T, H, HV, K, V, dtype=dt,
                                       nseq_state=N if use_h0 else None, state_std=0.3)
    if not l2:
        q = torch.nn.functional.normalize(q.float(), dim=-1).to(dt)
        k = torch.nn.functional.normalize(k.float(), dim=-1).to(dt)
    if h0 is not None and vfirst:
        h0 = h0.transpose(-1, -2).contiguous()
    gen = torch.Generator().manual_seed(99)
    do = torch.randn(B, T, HV, V, generator=gen).to(dt).cuda()
    shape = (N, HV, V, K) if vfirst else (N, HV, K, V)
    dht = torch.randn(shape, generator=gen).cuda() if use_dht else None
    scale = K ** -0.5
    res = ops.chunk_gated_delta_rule_bwd(q, k, v, g, beta, scale, h0, do, dht, cu_seqlens=cu,
                                         state_v_first=vfirst, use_qk_l2norm_in_kernel=l2)
    torch.cuda.synchronize()
    ref = gdn_bwd_oracle.chunk_bwd(np64(q), np64(k), np64(v), np64(g), np64(beta), scale, np64(h0),
                                   np64(do), np64(dht), cu_seqlens=cu_l, use_qk_l2norm=l2,
                                   state_v_first=vfirst)
    tol = FP32_TOL if dt == torch.float32 else BF16_TOL
    for nm, mine, want in zip(("dq", "dk", "dv", "db", "dg"), res[:5], ref[:5]):
        assert mine.dtype == (dt if nm in ("dq", "dk", "dv") else torch.float32)
        err = rel_rms(np64(mine), want)
        assert err < (tol if nm in ("dq", "dk", "dv") else max(FP32_TOL, tol / 3)), (nm, err)
    if use_h0:
        assert rel_rms(np64(res[5]), ref[5]) < max(FP32_TOL, tol / 3)
    else:
        assert res[5] is None


def test_autograd_through_chunk_gated_delta_rule():
    """chunk_gated_delta_rule is differentiable like the reference's
    ChunkGatedDeltaRuleFunction: .backward() fills every input's grad."""
    ops = _ops()
    B, T, H, HV, K, V = 1, 130, 2, 4, 64, 64
    q, k, v, g, beta, h0 = make_inputs(5, B, T, H, HV, K, V, dtype=torch.float32, nseq_state=B,
                                       state_std=0.3)
    q = torch.nn.functional.normalize(q, dim=-1)
    k = torch.nn.functional.normalize(k, dim=-1)
    leaves = [x.clone().requires_grad_() for x in (q, k, v, g, beta, h0)]
    o, ht = ops.chunk_gated_delta_rule(*leaves[:5], initial_state=leaves[5], output_final_state=True)
    gen = torch.Generator().manual_seed(1)
    do = torch.randn(o.shape, generator=gen).cuda()
    dht = torch.randn(ht.shape, generator=gen).cuda()
    ((o * do).sum() + (ht * dht).sum()).backward()
    ref = gdn_bwd_oracle.chunk_bwd(np64(q), np64(k), np64(v), np64(g), np64(beta), K ** -0.5, np64(h0),
                                   np64(do), np64(dht))
    grads = [leaves[0].grad, leaves[1].grad, leaves[2].grad, leaves[4].grad, leaves[3].grad, leaves[5].grad]
    for nm, mine, want in zip(("dq", "dk", "dv", "db", "dg", "dh0"), grads, ref[:6]):
        assert mine is not None, nm
        assert rel_rms(np64(mine), want) < FP32_TOL, nm


def test_autograd_without_final_state():
    """output_final_state=False: the backward runs with no dht (zero)."""
    ops = _ops()
    q, k, v, g, beta, _ = make_inputs(8, 1, 70, 1, 1, 32, 32, dtype=torch.float32)
    q = torch.nn.functional.normalize(q, dim=-1)
    k = torch.nn.functional.normalize(k, dim=-1)
    vl = v.clone().requires_grad_()
    o, ht = ops.chunk_gated_delta_rule(q, k, vl, g, beta)
    assert ht is None
    o.sum().backward()
    ref = gdn_bwd_oracle.chunk_bwd(np64(q), np64(k), np64(v), np64(g), np64(beta), 32 ** -0.5, None,
                                   np.ones(o.shape), None)
    assert rel_rms(np64(vl.grad), ref[2]) < FP32_TOL


def test_bwd_is_deterministic():
    ops = _ops()
    q, k, v, g, beta, h0 = make_inputs(9, 1, 300, 2, 4, 128, 128, dtype=torch.bfloat16, nseq_state=1,
                                       state_std=0.3)
    do = torch.randn_like(v)
    a = ops.chunk_gated_delta_rule_bwd(q, k, v, g, beta, None, h0, do, None, use_qk_l2norm_in_kernel=True)
    b = ops.chunk_gated_delta_rule_bwd(q, k, v, g, beta, None, h0, do, None, use_qk_l2norm_in_kernel=True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
