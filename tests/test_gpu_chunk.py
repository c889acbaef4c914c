"""GPU parity of the chunked prefill against the fp64 oracle and the
reference's golden vectors (tests/golden/chk_*.npz)."""

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


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "chk_*.npz"))),
                         ids=os.path.basename)
def test_chunk_matches_reference_golden(ops, path):
    d = dict(np.load(path))
    h0 = _t(d["h0"]) if d["h0"].size else None
    cu = _t(d["cu_seqlens"]) if d["cu_seqlens"].size else None
    o, ht = ops.chunk_gated_delta_rule(_t(d["q"]), _t(d["k"]), _t(d["v"]), _t(d["g"]),
                                       _t(d["beta"]), float(d["scale"]), h0, True, cu)
    assert rel_rms(np64(o), d["o"]) < FP32_REL_RMS
    assert rel_rms(np64(ht), d["final_state"]) < FP32_REL_RMS


def _check(ops, seed, B, T, H, HV, K, V, dtype, cu=None, h0_std=0.0, l2=True, state_v_first=False,
           force_generic=False, scale=None):
    N = B if cu is None else len(cu) - 1
    q, k, v, g, beta, h0 = make_inputs(seed, B, T, H, HV, K, V, dtype=dtype,
                                       nseq_state=N if h0_std else None, state_std=h0_std)
    if h0 is not None and state_v_first:
        h0 = h0.transpose(-1, -2).contiguous()
    cut = None if cu is None else torch.tensor(cu, dtype=torch.int32).cuda()
    o, ht = ops.chunk_gated_delta_rule(q, k, v, g, beta, scale, h0, True, cut, None, None, True,
                                       state_v_first, l2, force_generic=force_generic)
    ro, rht = oracle.chunk_gated_delta_rule(np64(q), np64(k), np64(v), np64(g), np64(beta), scale,
                                            np64(h0), True, cu, l2, state_v_first)
    e_o, e_h = rel_rms(np64(o), ro), rel_rms(np64(ht), rht)
    if dtype == torch.float32:
        assert e_o < FP32_REL_RMS and e_h < FP32_REL_RMS, (e_o, e_h)
    else:
        m_o = max_abs(np64(o), ro)
        assert e_o < BF16_REL_RMS and m_o < BF16_MAX_ABS, (e_o, m_o)
        assert e_h < BF16_REL_RMS, e_h
    return o, ht


def test_config0_fp32(ops):
    """fp32, B=1 T=256 H=4 d=64, zero initial state."""
    _check(ops, 0, 1, 256, 4, 4, 64, 64, torch.float32)


@pytest.mark.parametrize("T", [1, 17, 64, 65, 200])
def test_fp32_lengths(ops, T):
    _check(ops, 40 + T, 2, T, 2, 4, 32, 48, torch.float32, h0_std=0.1)


def test_fp32_state_v_first_varlen(ops):
    _check(ops, 5, 1, 300, 2, 4, 64, 32, torch.float32, cu=[0, 1, 64, 64, 150, 300], h0_std=0.05,
           state_v_first=True)


@pytest.mark.parametrize("force_generic", [False, True])
def test_bf16_qwen_shape(ops, force_generic):
    _check(ops, 1, 1, 1024, 16, 32, 128, 128, torch.bfloat16, force_generic=force_generic)


@pytest.mark.parametrize("force_generic", [False, True])
def test_bf16_varlen_with_states(ops, force_generic):
    cu = [0, 100, 164, 700, 701, 1500]
    _check(ops, 2, 1, 1500, 16, 32, 128, 128, torch.bfloat16, cu=cu, h0_std=0.02,
           force_generic=force_generic)


def test_fp16_small(ops):
    _check(ops, 3, 2, 130, 2, 2, 128, 128, torch.float16, h0_std=0.02, scale=0.1)


def test_bf16_config1_full_size(ops):
    """B=1, T=8192, 16 q/k heads, 32 v heads, d=128, bf16."""
    _check(ops, 1, 1, 8192, 16, 32, 128, 128, torch.bfloat16)


def test_config2_full_size_packing_equivalence(ops):
    """BASELINE config 2 (16 sequences, lengths U[512, 8192], states N(0, 0.02)):
    the packed varlen call must equal running every sequence alone (a
    size-independent property), and stay finite."""
    rng = np.random.default_rng(2)
    lens = rng.integers(512, 8193, size=16)
    cu = np.concatenate([[0], np.cumsum(lens)])
    T = int(cu[-1])
    q, k, v, g, beta, h0 = make_inputs(2, 1, T, 16, 32, 128, 128, nseq_state=16, state_std=0.02)
    cut = torch.from_numpy(cu).cuda()
    o, ht = ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cut,
                                       use_qk_l2norm_in_kernel=True)
    assert torch.isfinite(o.float()).all() and torch.isfinite(ht).all()
    for n in (0, 7, 15):
        s, e = int(cu[n]), int(cu[n + 1])
        o1, h1 = ops.chunk_gated_delta_rule(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e],
                                            beta[:, s:e], None, h0[n:n + 1], True,
                                            use_qk_l2norm_in_kernel=True)
        assert torch.equal(o1, o[:, s:e])
        assert torch.equal(h1[0], ht[n])


def _oracle_seq(q, k, v, g, beta, h0, s, e):
    """fp64 oracle of one packed sequence [s, e) (bf16-rounded inputs)."""
    sl = lambda t: np64(t[:, s:e])
    return oracle.chunk_gated_delta_rule(sl(q), sl(k), sl(v), sl(g), sl(beta), None,
                                         None if h0 is None else np64(h0), True, None, True)


def _check_bf16(o, ht, ro, rht):
    e_o, m_o, e_h = rel_rms(np64(o), ro), max_abs(np64(o), ro), rel_rms(np64(ht), rht)
    assert e_o < BF16_REL_RMS and m_o < BF16_MAX_ABS and e_h < BF16_REL_RMS, (e_o, m_o, e_h)


def test_config2_full_size_against_oracle(ops):
    """BASELINE config 2 at full size (seed 2: 16 sequences, lengths
    U[512, 8192], packed via cu_seqlens, states N(0, 0.02)): the shortest,
    the median and the longest sequence, all 32 v-heads, outputs and final
    states against the fp64 oracle (cu_seqlens semantics of
    triton/fla/index.py:13-32)."""
    rng = np.random.default_rng(2)
    lens = rng.integers(512, 8193, size=16)
    cu = np.concatenate([[0], np.cumsum(lens)])
    q, k, v, g, beta, h0 = make_inputs(2, 1, int(cu[-1]), 16, 32, 128, 128, nseq_state=16, state_std=0.02)
    o, ht = ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, torch.from_numpy(cu).cuda(),
                                       use_qk_l2norm_in_kernel=True)
    order = np.argsort(lens, kind="stable")
    for n in (int(order[0]), int(order[len(order) // 2]), int(order[-1])):
        s, e = int(cu[n]), int(cu[n + 1])
        ro, rht = _oracle_seq(q, k, v, g, beta, h0[n:n + 1], s, e)
        _check_bf16(o[:, s:e], ht[n:n + 1], ro, rht)


def test_config4_full_size_against_oracle(ops):
    """BASELINE config 4 at full size (seed 4: 64 sequences x 4096 tokens):
    sequences 0, 31 and 63 against the fp64 oracle."""
    B, T = 64, 4096
    q, k, v, g, beta, _ = make_inputs(4, B, T, 16, 32, 128, 128)
    o, ht = ops.chunk_gated_delta_rule(q, k, v, g, beta, None, None, True, use_qk_l2norm_in_kernel=True)
    for n in (0, 31, 63):
        sl = lambda t: t[n:n + 1]
        ro, rht = oracle.chunk_gated_delta_rule(np64(sl(q)), np64(sl(k)), np64(sl(v)), np64(sl(g)),
                                                np64(sl(beta)), None, None, True, None, True)
        _check_bf16(o[n:n + 1], ht[n:n + 1], ro, rht)


def test_chunk_equals_recurrent_on_gpu(ops):
    """The chunked op and the token-by-token op agree (fp32)."""
    q, k, v, g, beta, h0 = make_inputs(9, 1, 333, 2, 4, 64, 64, dtype=torch.float32,
                                       nseq_state=1, state_std=0.1)
    o1, h1 = ops.chunk_gated_delta_rule(q, k, v, g, beta, 0.125, h0, True,
                                        use_qk_l2norm_in_kernel=True)
    o2, h2 = ops.fused_recurrent_gated_delta_rule(q, k, v, g, None, None, beta, 0.125, h0, True, True)
    assert rel_rms(np64(o1), np64(o2)) < FP32_REL_RMS
    assert rel_rms(np64(h1), np64(h2)) < FP32_REL_RMS


def test_solve_tril(ops):
    rng = np.random.default_rng(4)
    for BT, cu in ((64, None), (32, np.array([0, 10, 80, 100])), (16, None)):
        B = 2 if cu is None else 1
        T = 100
        H = 3
        A = np.zeros((B, T, H, BT), np.float32)
        bounds = oracle.seq_bounds(B, T, cu)
        flatA = A.reshape(B * T, H, BT)
        for bos, eos in bounds:
            for s in range(bos, eos, BT):
                L = min(BT, eos - s)
                blk = np.tril(rng.standard_normal((H, L, L)) * 0.2, -1)
                flatA[s:s + L, :, :L] = blk.transpose(1, 0, 2)
        ref = oracle.solve_tril(flatA.astype(np.float64), bounds, BT).reshape(B, T, H, BT)
        for dt, tol in ((torch.float32, 1e-6), (torch.bfloat16, 1e-2)):
            out = ops.solve_tril(_t(A), None, None if cu is None else _t(cu), dt)
            assert rel_rms(np64(out), ref) < tol


TC_CASES = [
    # (name, B, T, H, HV, cu, h0_std, state_v_first)
    ("heads_equal", 2, 300, 16, 16, None, 0.02, False),
    ("gva4_vfirst", 1, 500, 8, 32, None, 0.02, True),
    ("many_sequences", 48, 128, 16, 32, None, 0.02, False),  # 1536 chains: widest state kernel
    ("varlen_empty", 1, 400, 4, 8, [0, 0, 64, 64, 129, 400, 400], 0.02, False),
]


@pytest.mark.parametrize("case", TC_CASES, ids=[c[0] for c in TC_CASES])
def test_bf16_tensor_core_path_variants(ops, case):
    """The tcgen05 path (bf16, K = V = 128) across head ratios, state
    layouts, the state-kernel variants picked by the number of chains, and
    zero-length sequences."""
    name, B, T, H, HV, cu, h0_std, vfirst = case
    _check(ops, 17 + len(name), B, T, H, HV, 128, 128, torch.bfloat16, cu=cu, h0_std=h0_std,
           state_v_first=vfirst)


FUSED_CASES = [
    # (name, B, T, H, HV, cu, h0_std, state_v_first): chunk counts not a
    # multiple of the cluster size, partial chunks, empty and one-chunk
    # sequences, more clusters than fit at once
    ("one_seq", 1, 1000, 16, 32, None, 0.02, False),
    ("varlen", 1, 900, 4, 8, [0, 0, 1, 63, 64, 65, 300, 900], 0.02, True),
    ("many", 40, 200, 8, 16, None, 0.02, False),
]


@pytest.mark.parametrize("case", FUSED_CASES, ids=[c[0] for c in FUSED_CASES])
def test_fused_kernel_matches_split_kernels(ops, case, monkeypatch):
    """The fused cluster kernel (WY tiles delivered through distributed shared
    memory) against the separate WY + state kernels on the same inputs: the
    same arithmetic, so the outputs agree to the last bit when the split path
    uses 32-column slices too, and both meet the oracle tolerance."""
    name, B, T, H, HV, cu, h0_std, vfirst = case
    N = B if cu is None else len(cu) - 1
    q, k, v, g, beta, h0 = make_inputs(60 + len(name), B, T, H, HV, 128, 128, nseq_state=N, state_std=h0_std)
    if vfirst:
        h0 = h0.transpose(-1, -2).contiguous()
    cut = None if cu is None else torch.tensor(cu, dtype=torch.int64).cuda()
    res = {}
    for path in ("1", "0"):
        monkeypatch.setenv("GDN_TC_FUSED", path)
        res[path] = ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cut, state_v_first=vfirst,
                                               use_qk_l2norm_in_kernel=True, check_errors=True)
    (of, hf), (os_, hs) = res["1"], res["0"]
    if N * HV <= 148:  # the split path's state kernel also uses 32-column slices
        assert torch.equal(of, os_) and torch.equal(hf, hs)
    ro, rht = oracle.chunk_gated_delta_rule(np64(q), np64(k), np64(v), np64(g), np64(beta), None, np64(h0),
                                            True, cu, True, vfirst)
    for o_, h_ in ((of, hf), (os_, hs)):
        assert rel_rms(np64(o_), ro) < BF16_REL_RMS and max_abs(np64(o_), ro) < BF16_MAX_ABS
        assert rel_rms(np64(h_), rht) < BF16_REL_RMS


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("width", ["64", "128"])
def test_slice_width_does_not_change_results(ops, monkeypatch, width, dtype):
    """The state kernel's V-slice width (32, 64 or 128 state columns per CTA,
    picked from the number of chains; GDN_TC_VS overrides it) only regroups
    the columns: outputs and final states equal the 32-column kernel's bit for
    bit, here with packed sequences of uneven length and a V-first state."""
    cu = [0, 130, 200, 500]
    q, k, v, g, beta, h0 = make_inputs(91, 1, 500, 4, 8, 128, 128, dtype=dtype, nseq_state=3, state_std=0.05)
    h0 = h0.transpose(-1, -2).contiguous()
    cut = torch.tensor(cu, dtype=torch.int64).cuda()
    res = {}
    for w in ("32", width):
        monkeypatch.setenv("GDN_TC_VS", w)
        res[w] = ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cut, state_v_first=True,
                                            use_qk_l2norm_in_kernel=True, check_errors=True)
    assert torch.equal(res["32"][0], res[width][0]) and torch.equal(res["32"][1], res[width][1])


def test_strided_rows_are_read_in_place(ops):
    """q, k, v as views of one [T, 2*H*K + HV*V] projection (token rows
    strided, heads packed): the tensor-core path reads them through its
    tensor maps without copies, with the results of packed inputs."""
    from domesticated_torch_mlu_ops_b200 import _lib
    lib = _lib.load()
    H, HV, T = 4, 8, 300
    q0, k0, v0, g, beta, h0 = make_inputs(31, 1, T, H, HV, 128, 128, nseq_state=2, state_std=0.05)
    mixed = torch.cat([q0.reshape(T, -1), k0.reshape(T, -1), v0.reshape(T, -1)], dim=1)
    q = mixed[:, :H * 128].view(1, T, H, 128)
    k = mixed[:, H * 128:2 * H * 128].view(1, T, H, 128)
    v = mixed[:, 2 * H * 128:].view(1, T, HV, 128)
    assert not q.is_contiguous() and not v.is_contiguous()
    cu = torch.tensor([0, 100, T], device="cuda")
    ref = ops.chunk_gated_delta_rule(q0, k0, v0, g, beta, None, h0, True, cu, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    n0 = lib.gdn_kernel_launch_count()
    out = ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cu, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert lib.gdn_kernel_launch_count() - n0 == 3  # plan, WY, state: no copy kernels of this library either
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])
