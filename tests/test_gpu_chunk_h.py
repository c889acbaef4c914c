"""GPU parity of the state-recurrence stage op (chunk_gated_delta_rule_fwd_h,
triton/fla/chunk_delta_h.py:200-271) with per-key decays (its USE_GK branch):
the reference's own kernel outputs (tests/golden/chh_*.npz, fp32) and the
fp64 oracle at the Qwen3-Next head layout in bf16."""

import glob
import os

import numpy as np
import pytest
import torch

import oracle
from gdn_testutil import BF16_REL_RMS, FP32_REL_RMS, np64, rel_rms

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import domesticated_torch_mlu_ops_b200 as m
    return m


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "chh_*.npz"))),
                         ids=os.path.basename)
def test_state_stage_matches_reference_golden(ops, path):
    d = dict(np.load(path))
    cu = _t(d["cu_seqlens"]) if d["cu_seqlens"].size else None
    h, v_new, ht = ops.chunk_gated_delta_rule_fwd_h(
        _t(d["k"]), _t(d["w"]), _t(d["u"]), _t(d["g"]) if d["g"].size else None, _t(d["gk"]), _t(d["h0"]),
        True, state_v_first=bool(d["state_v_first"]), cu_seqlens=cu)
    for got, ref in ((h, d["h"]), (v_new, d["v_new"]), (ht, d["final_state"])):
        assert got.shape == ref.shape
        assert rel_rms(np64(got), ref) < FP32_REL_RMS


@pytest.mark.parametrize("vfirst,varlen", [(False, False), (True, True)])
def test_state_stage_bf16_qwen_layout(ops, vfirst, varlen):
    """K = V = 128, 16 k heads, 32 heads, bf16 k/w/u, g and gk, against the
    fp64 oracle on the same bf16 inputs."""
    gen = torch.Generator().manual_seed(70 + int(vfirst))
    T, Hg, H, K, V = 700, 16, 32, 128, 128
    cu_l = [0, 64, 65, 300, 700] if varlen else None
    bounds = [(0, T)] if cu_l is None else list(zip(cu_l[:-1], cu_l[1:]))

    def chunk_cumsum(x):
        out = torch.zeros_like(x)
        for bos, eos in bounds:
            for s0 in range(bos, eos, 64):
                out[:, s0:min(s0 + 64, eos)] = torch.cumsum(x[:, s0:min(s0 + 64, eos)], dim=1)
        return out

    k = torch.nn.functional.normalize(torch.randn(1, T, Hg, K, generator=gen), dim=-1).bfloat16()
    w = (torch.randn(1, T, H, K, generator=gen) * 0.1).bfloat16()
    u = torch.randn(1, T, H, V, generator=gen).bfloat16()
    g = chunk_cumsum(torch.nn.functional.logsigmoid(torch.randn(1, T, H, generator=gen)))
    gk = chunk_cumsum(torch.nn.functional.logsigmoid(torch.randn(1, T, H, K, generator=gen)) * 0.1)
    N = len(bounds)
    h0 = torch.randn((N, H, V, K) if vfirst else (N, H, K, V), generator=gen) * 0.02
    g_hm = g.permute(2, 0, 1).contiguous()
    cu = None if cu_l is None else torch.tensor(cu_l).cuda()
    h, v_new, ht = ops.chunk_gated_delta_rule_fwd_h(k.cuda(), w.cuda(), u.cuda(), g_hm.cuda(), gk.cuda(),
                                                    h0.cuda(), True, state_v_first=vfirst, cu_seqlens=cu)
    rh, rv, rht = oracle.chunk_fwd_h_stage(np64(k), np64(w), np64(u), np64(g_hm), np64(gk), np64(h0), True,
                                           vfirst, cu_l)
    assert rel_rms(np64(h), rh) < BF16_REL_RMS
    assert rel_rms(np64(v_new), rv) < BF16_REL_RMS
    assert rel_rms(np64(ht), rht) < BF16_REL_RMS
