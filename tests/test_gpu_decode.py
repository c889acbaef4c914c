"""GPU parity of the recurrent kernels against the oracle and the reference's
own golden vectors (tests/golden/rfn_*.npz, rec_*.npz)."""

import glob
import os

import numpy as np
import pytest
import torch

import oracle
from gdn_testutil import (BF16_MAX_ABS, BF16_REL_RMS, FP32_REL_RMS, make_inputs, max_abs, np64,
                          rel_rms)

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import domesticated_torch_mlu_ops_b200 as m
    return m


def _t(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "rfn_*.npz"))),
                         ids=os.path.basename)
def test_decode_matches_reference_golden(ops, path):
    d = dict(np.load(path))
    nacc = d["num_accepted_tokens"]
    cache = _t(d["cache_in"].astype(np.float32))
    idx = _t(d["ssm_state_indices"])
    o, ht = ops.fused_recurrent_gated_delta_rule_fn(
        _t(d["q"]), _t(d["k"]), _t(d["v"]), _t(d["g"]), _t(d["beta"]), float(d["scale"]),
        cache, inplace_final_state=bool(d["inplace"]), cu_seqlens=_t(d["cu_seqlens"]),
        ssm_state_indices=idx, num_accepted_tokens=_t(nacc) if nacc.size else None,
        use_qk_l2norm_in_kernel=bool(d["l2norm"]))
    torch.cuda.synchronize()
    cu = d["cu_seqlens"]
    idx0 = d["ssm_state_indices"].reshape(len(cu) - 1, -1)
    for n in range(len(cu) - 1):
        i0 = int(nacc[n]) - 1 if nacc.size else 0
        s, e = cu[n], cu[n + 1]
        if idx0[n, i0] < 0:
            assert torch.all(o[0, s:e] == 0)
            continue
        np.testing.assert_allclose(o[0, s:e].cpu().numpy(), d["o"][0, s:e], rtol=1e-5, atol=2e-6)
    n_rows = d["final_state"].shape[0]
    np.testing.assert_allclose(ht[:n_rows].cpu().numpy(), d["final_state"], rtol=1e-5, atol=2e-6)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "rec_*.npz"))),
                         ids=os.path.basename)
def test_plain_recurrent_matches_reference_golden(ops, path):
    d = dict(np.load(path))
    h0 = _t(d["h0"]) if d["h0"].size else None
    cu = _t(d["cu_seqlens"]) if d["cu_seqlens"].size else None
    o, ht = ops.fused_recurrent_gated_delta_rule(
        _t(d["q"]), _t(d["k"]), _t(d["v"]), g=_t(d["g"]), beta=_t(d["beta"]),
        scale=float(d["scale"]), initial_state=h0, output_final_state=True,
        use_qk_l2norm_in_kernel=bool(d["l2norm"]), cu_seqlens=cu)
    assert rel_rms(o.cpu().numpy(), d["o"]) < 1e-5
    assert rel_rms(ht.cpu().numpy(), d["final_state"]) < 1e-5


def _decode_case(ops, seed, N, slots, H, HV, K, V, dtype, idx_dtype=torch.int64, l2=True,
                 beta_per_v=False, inplace=True, pad=()):
    q, k, v, g, beta, _ = make_inputs(seed, 1, N, H, HV, K, V, dtype=dtype)
    gen = torch.Generator().manual_seed(seed + 100)
    if beta_per_v:
        beta = torch.sigmoid(torch.randn(1, N, HV, V, generator=gen)).cuda()
    cache = (torch.randn(slots, HV, V, K, generator=gen) * 0.02).cuda()
    idx = torch.randperm(slots, generator=gen)[:N].to(idx_dtype).cuda()
    for p in pad:
        idx[p] = -1
    cu = torch.arange(N + 1, dtype=torch.int32).cuda()
    cache_np = np64(cache).copy()
    o, ht = ops.fused_recurrent_gated_delta_rule_fn(
        q, k, v, g, beta, K ** -0.5, cache, inplace_final_state=inplace, cu_seqlens=cu,
        ssm_state_indices=idx, use_qk_l2norm_in_kernel=l2)
    ro, rht, valid = oracle.recurrent_v_first(
        np64(q), np64(k), np64(v), np64(g), np64(beta), K ** -0.5, cache_np,
        inplace_final_state=inplace, cu_seqlens=np.arange(N + 1),
        ssm_state_indices=idx.cpu().numpy(), use_qk_l2norm_in_kernel=l2)
    o = np64(o)
    tol = FP32_REL_RMS if dtype == torch.float32 else BF16_REL_RMS
    # the kernel computes in fp32 from the same inputs; outputs are rounded to `dtype`
    assert rel_rms(o[0, valid], ro[0, valid]) < tol
    if dtype != torch.float32:
        assert max_abs(o[0, valid], ro[0, valid]) < BF16_MAX_ABS
    assert rel_rms(np64(ht), rht) < FP32_REL_RMS
    if pad:
        assert np.all(o[0, ~valid] == 0)
    return o, ro


def test_decode_config3_full_size(ops):
    """256 sequences, 16/32 heads, d=128, cache [1024,32,128,128]."""
    _decode_case(ops, 3, 256, 1024, 16, 32, 128, 128, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("K,V", [(128, 128), (128, 96), (128, 32), (64, 64), (32, 16)])
def test_decode_shapes_dtypes(ops, dtype, K, V):
    """K = 128 takes the streaming kernel, which splits each state into
    64-row blocks (V = 96: a full and a half block; V = 32: one short block)."""
    _decode_case(ops, 11, 37, 80, 2, 4, K, V, dtype)


def test_decode_pad_int32_betav_no_l2(ops):
    _decode_case(ops, 12, 20, 50, 4, 8, 128, 128, torch.bfloat16, idx_dtype=torch.int32,
                 l2=False, beta_per_v=True, pad=(0, 7, 19))


@pytest.mark.parametrize("K,V", [(64, 32), (128, 96)])
def test_decode_not_inplace(ops, K, V):
    _decode_case(ops, 13, 9, 30, 2, 2, K, V, torch.bfloat16, inplace=False)


@pytest.mark.parametrize("K,V", [(64, 64), (128, 128)])
def test_decode_spec_tokens(ops, K, V):
    """Speculative decoding: T=3 tokens per sequence, per-token states written
    to ssm_state_indices[n, t], initial state from column num_accepted-1
    (K = 128: the streaming kernel, one bulk store per 64-row block and token)."""
    N, T, H, HV, slots = 5, 3, 2, 4, 40
    q, k, v, g, beta, _ = make_inputs(21, 1, N * T, H, HV, K, V, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(22)
    cache = (torch.randn(slots, HV, V, K, generator=gen) * 0.1).cuda()
    idx = torch.randperm(slots, generator=gen)[:N * T].reshape(N, T).cuda()
    idx[2, 1] = -1
    nacc = torch.tensor([1, 3, 2, 1, 3]).cuda()
    cu = torch.arange(0, N * T + 1, T).cuda()
    cache_np = np64(cache).copy()
    o, ht = ops.fused_recurrent_gated_delta_rule_fn(
        q, k, v, g, beta, 0.2, cache, True, cu, idx, nacc, True)
    ro, rht, valid = oracle.recurrent_v_first(
        np64(q), np64(k), np64(v), np64(g), np64(beta), 0.2, cache_np, cu_seqlens=cu.cpu().numpy(),
        ssm_state_indices=idx.cpu().numpy(), num_accepted_tokens=nacc.cpu().numpy(),
        use_qk_l2norm_in_kernel=True)
    assert rel_rms(np64(o), ro) < BF16_REL_RMS
    assert rel_rms(np64(ht), rht) < FP32_REL_RMS


def test_plain_recurrent_gk_gv_varlen(ops):
    B, T, H, HV, K, V = 1, 70, 2, 4, 32, 64
    q, k, v, g, beta, _ = make_inputs(31, B, T, H, HV, K, V, dtype=torch.float32)
    gen = torch.Generator().manual_seed(32)
    gk = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, K, generator=gen)).cuda() * 0.1
    gv = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, V, generator=gen)).cuda() * 0.1
    cu = torch.tensor([0, 5, 5, 40, 70]).cuda()
    h0 = (torch.randn(4, HV, K, V, generator=gen) * 0.1).cuda()
    o, ht = ops.fused_recurrent_gated_delta_rule(q, k, v, g, gk, gv, beta, None, h0, True, True, cu)
    ro, rht = oracle.recurrent_k_first(np64(q), np64(k), np64(v), g=np64(g), beta=np64(beta),
                                       initial_state=np64(h0), output_final_state=True,
                                       use_qk_l2norm_in_kernel=True, cu_seqlens=cu.cpu().numpy(),
                                       gk=np64(gk), gv=np64(gv))
    assert rel_rms(np64(o), ro) < FP32_REL_RMS
    assert rel_rms(np64(ht), rht) < FP32_REL_RMS


def test_decode_rejects_cpu_tensors(ops):
    q = torch.zeros(1, 1, 1, 8)
    with pytest.raises(ValueError):
        ops.fused_recurrent_gated_delta_rule_fn(q, q, q, None, None)
