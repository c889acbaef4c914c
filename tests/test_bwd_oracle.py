"""Pin the backward oracle (float64 autograd through the recurrence) to the
reference's own backward kernels (``tests/golden/bwd_*.npz``, made by
``make_golden.py --only bwd`` from ``chunk_gated_delta_rule_bwd``)."""

import glob
import os

import numpy as np
import pytest

from oracle import gdn_bwd_oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _rel_rms(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2)) / (np.sqrt(np.mean(b ** 2)) + 1e-30))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "bwd_*.npz"))), ids=os.path.basename)
def test_bwd_oracle_matches_reference(path):
    d = dict(np.load(path))
    h0 = d["h0"] if d["h0"].size else None
    dht = d["dht"] if d["dht"].size else None
    cu = d["cu_seqlens"] if d["cu_seqlens"].size else None
    dq, dk, dv, db, dg, dh0, _, _ = gdn_bwd_oracle.chunk_bwd(
        d["q"], d["k"], d["v"], d["g"], d["beta"], float(d["scale"]), h0, d["do"], dht, cu_seqlens=cu)
    # the reference computes in fp32 (allow_tf32=False): agreement to ~1e-6
    for name, mine in (("dq", dq), ("dk", dk), ("dv", dv), ("db", db), ("dg", dg)):
        assert _rel_rms(mine, d[name]) < 1e-5, name
        np.testing.assert_allclose(mine, d[name], rtol=1e-4, atol=1e-4, err_msg=name)
    if h0 is not None:
        assert _rel_rms(dh0, d["dh0"]) < 1e-5
        np.testing.assert_allclose(dh0, d["dh0"], rtol=1e-4, atol=1e-4)


def test_bwd_oracle_l2norm_and_vfirst_consistency():
    """The l2-norm and V-first options are compositions: normalising the
    inputs outside and transposing the state give the same gradients."""
    import torch
    rng = np.random.default_rng(3)
    B, T, H, HV, K, V = 1, 20, 1, 2, 8, 4
    q, k = rng.standard_normal((2, B, T, H, K))
    v = rng.standard_normal((B, T, HV, V))
    g = np.log(1 / (1 + np.exp(-rng.standard_normal((B, T, HV)))))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))
    h0 = rng.standard_normal((1, HV, K, V)) * 0.3
    do = rng.standard_normal((B, T, HV, V))
    dht = rng.standard_normal((1, HV, K, V))
    a = gdn_bwd_oracle.chunk_bwd(q, k, v, g, beta, 0.3, h0, do, dht)
    b = gdn_bwd_oracle.chunk_bwd(q, k, v, g, beta, 0.3, h0.transpose(0, 1, 3, 2), do,
                                 dht.transpose(0, 1, 3, 2), state_v_first=True)
    for x, y in zip(a[:5], b[:5]):
        np.testing.assert_allclose(x, y, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(a[5], b[5].transpose(0, 1, 3, 2), rtol=1e-12, atol=1e-12)
    # l2norm: chain rule through x / sqrt(|x|^2 + eps) checked by autograd on the composition
    qt = torch.tensor(q, requires_grad=True)
    qn = qt / torch.sqrt((qt * qt).sum(-1, keepdim=True) + 1e-6)
    kt = torch.tensor(k, requires_grad=True)
    kn = kt / torch.sqrt((kt * kt).sum(-1, keepdim=True) + 1e-6)
    c = gdn_bwd_oracle.chunk_bwd(qn.detach().numpy(), kn.detach().numpy(), v, g, beta, 0.3, h0, do, dht)
    qn.backward(torch.tensor(c[0]))
    kn.backward(torch.tensor(c[1]))
    d = gdn_bwd_oracle.chunk_bwd(q, k, v, g, beta, 0.3, h0, do, dht, use_qk_l2norm=True)
    np.testing.assert_allclose(d[0], qt.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(d[1], kt.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(d[2], c[2], rtol=1e-10, atol=1e-12)
