"""Pin the numpy oracle to golden vectors produced by the reference's own
Triton kernels (``tests/golden/make_golden.py``), and check the oracle's
chunked form against its recurrent form."""

import glob
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return dict(np.load(os.path.join(GOLD, name)))


def _rel_rms(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2)) / (np.sqrt(np.mean(b ** 2)) + 1e-30))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "rfn_*.npz"))),
                         ids=os.path.basename)
def test_oracle_matches_reference_decode(path):
    d = _load(os.path.basename(path))
    nacc = d["num_accepted_tokens"]
    cache = d["cache_in"].astype(np.float64).copy()
    N = len(d["cu_seqlens"]) - 1
    kda = d["g"].ndim == 4  # per-key decays (the kernel's IS_KDA branch)
    o, ht, valid = oracle.recurrent_v_first(
        d["q"], d["k"], d["v"], None if kda else d["g"], d["beta"], float(d["scale"]), cache,
        inplace_final_state=bool(d["inplace"]), cu_seqlens=d["cu_seqlens"],
        ssm_state_indices=d["ssm_state_indices"],
        num_accepted_tokens=nacc if nacc.size else None,
        use_qk_l2norm_in_kernel=bool(d["l2norm"]), gk=d["g"] if kda else None)
    cu = d["cu_seqlens"]
    for n in range(N):
        if not valid[n]:
            continue
        s, e = cu[n], cu[n + 1]
        np.testing.assert_allclose(o[0, s:e], d["o"][0, s:e], rtol=1e-5, atol=1e-5)
    if bool(d["inplace"]):
        np.testing.assert_allclose(ht, d["final_state"], rtol=1e-5, atol=1e-5)
    else:
        np.testing.assert_allclose(ht[: d["final_state"].shape[0]], d["final_state"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "rec_*.npz"))),
                         ids=os.path.basename)
def test_oracle_matches_reference_recurrent(path):
    d = _load(os.path.basename(path))
    h0 = d["h0"] if d["h0"].size else None
    cu = d["cu_seqlens"] if d["cu_seqlens"].size else None
    o, ht = oracle.recurrent_k_first(
        d["q"], d["k"], d["v"], g=d["g"], beta=d["beta"], scale=float(d["scale"]),
        initial_state=h0, output_final_state=True,
        use_qk_l2norm_in_kernel=bool(d["l2norm"]), cu_seqlens=cu)
    assert _rel_rms(o, d["o"]) < 1e-5
    assert _rel_rms(ht, d["final_state"]) < 1e-5


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "chk_*.npz"))),
                         ids=os.path.basename)
def test_oracle_matches_reference_chunk(path):
    d = _load(os.path.basename(path))
    h0 = d["h0"] if d["h0"].size else None
    cu = d["cu_seqlens"] if d["cu_seqlens"].size else None
    o, ht = oracle.chunk_gated_delta_rule(
        d["q"], d["k"], d["v"], d["g"], d["beta"], scale=float(d["scale"]),
        initial_state=h0, output_final_state=True, cu_seqlens=cu)
    assert _rel_rms(o, d["o"]) < 1e-5
    assert _rel_rms(ht, d["final_state"]) < 1e-5


@pytest.mark.parametrize("varlen", [False, True])
def test_chunk_form_equals_recurrence(varlen):
    rng = np.random.default_rng(5)
    B, T, H, HV, K, V = 1, 150, 2, 4, 32, 16
    q = rng.standard_normal((B, T, H, K))
    k = rng.standard_normal((B, T, H, K))
    v = rng.standard_normal((B, T, HV, V))
    g = -np.log1p(np.exp(-rng.standard_normal((B, T, HV))))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))
    cu = np.array([0, 37, 64, 65, 150]) if varlen else None
    N = 4 if varlen else 1
    h0 = rng.standard_normal((N, HV, K, V)) * 0.1
    o1, h1 = oracle.recurrent_k_first(q, k, v, g=g, beta=beta, scale=0.3, initial_state=h0,
                                      output_final_state=True, use_qk_l2norm_in_kernel=True,
                                      cu_seqlens=cu)
    o2, h2 = oracle.chunk_gated_delta_rule(q, k, v, g, beta, scale=0.3, initial_state=h0,
                                           output_final_state=True, cu_seqlens=cu,
                                           use_qk_l2norm_in_kernel=True)
    assert np.abs(o1 - o2).max() < 1e-10
    assert np.abs(h1 - h2).max() < 1e-10


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "chh_*.npz"))),
                         ids=os.path.basename)
def test_oracle_matches_reference_state_stage(path):
    """chunk_gated_delta_rule_fwd_h with per-key decays (USE_GK), from the
    reference's own kernel: states before every chunk, v_new, final state."""
    d = dict(np.load(path))
    cu = d["cu_seqlens"] if d["cu_seqlens"].size else None
    h, v_new, ht = oracle.chunk_fwd_h_stage(
        d["k"], d["w"], d["u"], d["g"] if d["g"].size else None, d["gk"], d["h0"], True,
        bool(d["state_v_first"]), cu)
    for got, ref in ((h, d["h"]), (v_new, d["v_new"]), (ht, d["final_state"])):
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
