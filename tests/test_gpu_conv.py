"""GPU parity of the causal conv1d kernels (``gdn_conv.cu``) against the
oracle (``oracle/conv_oracle.py``) and the reference's golden vectors.

Tolerances: fp32 inputs, max-abs <= 1e-5 relative to the output scale;
bf16/fp16 inputs, the oracle runs on the rounded inputs and the output must
agree to half a unit of the output dtype plus 2e-3 relative (one output
rounding and fp32 accumulation order)."""

import glob
import os

import numpy as np
import pytest
import torch

from oracle import conv_oracle as C

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _t(a, dtype=torch.float32):
    return None if a is None else torch.as_tensor(np.asarray(a, np.float32)).to("cuda", dtype)


def _opt(a):
    return None if a.size == 0 else a


def _tol(ref, dtype):
    scale = max(1.0, float(np.abs(ref).max()))
    return {torch.float32: 1e-5, torch.bfloat16: 1.6e-2, torch.float16: 2e-3}[dtype] * scale


@pytest.fixture(scope="module")
def ops():
    import domesticated_torch_mlu_ops_b200 as m
    return m


# ---------------------------------------------------------------- goldens

@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(HERE, "golden", "conv_*.npz"))),
                         ids=lambda p: os.path.basename(p)[5:-4])
def test_matches_reference_golden(ops, path):
    d = np.load(path)
    name = os.path.basename(path)[5:-4]
    act = str(d["activation"]) or None
    if name.startswith("fla"):
        cu = _opt(d["cu_seqlens"])
        y, fs = ops.causal_conv1d(_t(d["x"]), _t(d["weight"]), _t(_opt(d["bias"])), _t(_opt(d["residual"])),
                                  _t(_opt(d["initial_state"])), False, act,
                                  cu_seqlens=None if cu is None else torch.tensor(cu, device="cuda"))
        assert fs is None
        np.testing.assert_allclose(y.cpu().numpy(), d["y"], atol=2e-5, rtol=0)
    elif name.startswith("fn"):
        x = _t(d["x"].T.copy()).t()  # channel-last (dim, tokens)
        cs = _t(np.ascontiguousarray(d["conv_states_in"].transpose(0, 2, 1))).transpose(1, 2)
        qsl = torch.tensor(d["query_start_loc"], device="cuda")
        apc = {}
        if "block_idx_last" in d:
            apc = dict(block_idx_first_scheduled_token=torch.tensor(d["block_idx_first"], device="cuda"),
                       block_idx_last_scheduled_token=torch.tensor(d["block_idx_last"], device="cuda"),
                       initial_state_idx=torch.tensor(d["initial_state_idx"], device="cuda"),
                       num_computed_tokens=torch.tensor(d["num_computed_tokens"], device="cuda"),
                       block_size_to_align=int(d["block_size"]))
        out = ops.causal_conv1d_fn(x, _t(d["weight"]), _t(_opt(d["bias"])), cs, qsl,
                                   torch.tensor(d["cache_indices"], device="cuda"),
                                   torch.tensor(d["has_initial_state"], device="cuda"), act, **apc)
        assert out.stride(0) == 1
        o = out.cpu().numpy()
        q = d["query_start_loc"]
        for s in range(len(q) - 1):
            if np.ndim(d["cache_indices"]) == 1 and d["cache_indices"][s] == 0:  # null block: skipped
                assert not o[:, q[s]:q[s + 1]].any()
                continue
            np.testing.assert_allclose(o[:, q[s]:q[s + 1]], d["out"][:, q[s]:q[s + 1]], atol=2e-5, rtol=0)
        assert np.array_equal(cs.cpu().numpy(), d["conv_states_out"])
    else:
        lay = str(d["layout"])
        x = _t(d["x"])
        x = {"nd": x, "n1d": x[:, None], "1nd": x[None]}[lay]
        cache = _t(d["cache_in"])
        y, c2 = ops.causal_conv1d_update(x, cache, _t(_opt(d["residual"])), _t(d["weight"]),
                                         _t(_opt(d["bias"])), act)
        assert c2 is cache and y.shape == x.shape
        np.testing.assert_allclose(y.reshape(d["y"].shape).cpu().numpy(), d["y"], atol=2e-5, rtol=0)
        assert np.array_equal(cache.cpu().numpy(), d["cache_out"])


# ------------------------------------------------------- random fla cases

@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("W", [2, 3, 4, 6])
@pytest.mark.parametrize("varlen", [False, True])
def test_fla_forward(ops, dtype, W, varlen):
    rng = np.random.default_rng(100 + W)
    D = 200 if W == 6 else 264  # 264: vector path; 200 with W=6 hits the generic-width kernel
    if varlen:
        lens = [0, 1, 2, 70, 3, 130, 64]
        B, T, cu = 1, sum(lens), np.concatenate([[0], np.cumsum(lens)])
    else:
        B, T, cu = 2, 150, None
    N = B if cu is None else len(cu) - 1
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    w = (rng.standard_normal((D, W)) * 0.5).astype(np.float32)
    b = rng.standard_normal(D).astype(np.float32)
    r = rng.standard_normal((B, T, D)).astype(np.float32)
    h0 = rng.standard_normal((N, D, W)).astype(np.float32)
    xt, wt, bt, rt, ht = (_t(a, dtype if a is x or a is r else torch.float32) for a in (x, w, b, r, h0))
    for use_init in (False, True):
        for act in (None, "silu"):
            y, _ = ops.causal_conv1d(xt, wt, bt, rt, ht if use_init else None, False, act,
                                     cu_seqlens=None if cu is None else torch.tensor(cu, device="cuda"))
            ref = C.causal_conv1d(xt.float().cpu().numpy(), w, b, rt.float().cpu().numpy(),
                                  h0 if use_init else None, act, cu)
            err = np.abs(y.float().cpu().numpy() - ref).max()
            assert err <= _tol(ref, dtype), (use_init, act, err)


# ------------------------------------------------------- random fn cases

def _fn_case(ops, rng, dtype, W, lens, has, idx, lines, dim, x_stride_pad=0, state_dtype=torch.float32,
             act="silu"):
    total = sum(lens)
    qsl = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    x = rng.standard_normal((total, dim)).astype(np.float32)
    w = (rng.standard_normal((dim, W)) * 0.5).astype(np.float32)
    b = rng.standard_normal(dim).astype(np.float32)
    st = rng.standard_normal((lines, W - 1, dim)).astype(np.float32)
    # x as a channel-last view, optionally inside a wider [tokens, dim + pad] buffer
    big = torch.zeros(total, dim + x_stride_pad, device="cuda", dtype=dtype)
    big[:, :dim] = _t(x, dtype)
    xv = big[:, :dim].t()
    cs = _t(st, state_dtype).transpose(1, 2)  # (lines, dim, W-1), unit dim stride
    cs_in = cs.float().cpu().numpy()
    out = ops.causal_conv1d_fn(xv, _t(w), _t(b), cs, torch.tensor(qsl, device="cuda"),
                               torch.tensor(idx, dtype=torch.int32, device="cuda"),
                               torch.tensor(has, dtype=torch.bool, device="cuda"), act)
    ref, cs_ref, proc = C.causal_conv1d_fn(xv.float().cpu().numpy(), w, b, cs_in, qsl, idx, has, act)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= _tol(ref, dtype), err
    np.testing.assert_allclose(cs.float().cpu().numpy(), cs_ref, atol=_tol(cs_ref, state_dtype), rtol=0)
    return out, cs


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("W", [2, 3, 4])
def test_fn_forward(ops, dtype, W):
    rng = np.random.default_rng(200 + W)
    lens = [5, 1, 0, 3, 70, 2, 129, 64]
    has = [1, 0, 1, 1, 0, 1, 1, 0]
    idx = [3, 7, 9, 1, 5, 0, 4, -1]  # 0: null block, -1: pad slot
    _fn_case(ops, rng, dtype, W, lens, has, idx, lines=10, dim=136, x_stride_pad=24)


def test_fn_scalar_path_and_state_dtype(ops):
    rng = np.random.default_rng(7)
    # dim not a multiple of 8: the one-channel-per-thread variant; bf16 states
    _fn_case(ops, rng, torch.bfloat16, 4, [9, 1, 2], [1, 1, 0], [2, 1, 3], lines=4, dim=52,
             state_dtype=torch.bfloat16, act=None)


def test_fn_split_sequence_is_bit_identical(ops):
    """One sequence run as two continuous-batching calls (the line carrying
    the state) gives the same bits as one call."""
    rng = np.random.default_rng(9)
    dim, W, L, cut = 128, 4, 300, 97
    x = torch.randn(L, dim, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(dim, W, device="cuda") * 0.5
    cs0 = torch.randn(2, W - 1, dim, device="cuda").transpose(1, 2)
    one = lambda xs, cs, h: ops.causal_conv1d_fn(xs.t(), w, None, cs, torch.tensor([0, xs.shape[0]], device="cuda",
                                                  dtype=torch.int32), torch.tensor([1], device="cuda", dtype=torch.int32),
                                                  torch.tensor([h], device="cuda"))
    cs_a = cs0.clone()
    whole = one(x, cs_a, True)
    cs_b = cs0.clone()
    p1 = one(x[:cut], cs_b, True)
    p2 = one(x[cut:], cs_b, True)
    assert torch.equal(torch.cat([p1, p2], 1), whole)
    assert torch.equal(cs_a, cs_b)


# ------------------------------------------------------- update

@pytest.mark.parametrize("dtype,cdtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.float32),
                                          (torch.bfloat16, torch.bfloat16)])
@pytest.mark.parametrize("W", [2, 3, 4])
def test_update(ops, dtype, cdtype, W):
    rng = np.random.default_rng(300 + W)
    N, D = 37, 1000
    x = rng.standard_normal((N, D)).astype(np.float32)
    cache = rng.standard_normal((N, D, W)).astype(np.float32)
    w = (rng.standard_normal((D, W)) * 0.5).astype(np.float32)
    b = rng.standard_normal(D).astype(np.float32)
    r = rng.standard_normal((N, D)).astype(np.float32)
    xt, rt = _t(x, dtype), _t(r, dtype)
    ct = _t(cache, cdtype)
    y, _ = ops.causal_conv1d_update(xt, ct, rt, _t(w), _t(b), "silu")
    ref, nc = C.causal_conv1d_update(xt.float().cpu().numpy(), _t(cache, cdtype).float().cpu().numpy(),
                                     rt.float().cpu().numpy(), w, b, "silu")
    assert np.abs(y.float().cpu().numpy() - ref).max() <= _tol(ref, dtype)
    np.testing.assert_allclose(ct.float().cpu().numpy(), nc, atol=_tol(nc, cdtype), rtol=0)


def test_update_without_cache_or_weight(ops):
    x = torch.randn(4, 16, device="cuda")
    b = torch.randn(16, device="cuda")
    w = torch.randn(16, 3, device="cuda")
    y, c = ops.causal_conv1d_update(x, None, None, w, b, None)  # all-zero window: y = bias
    assert c is None
    torch.testing.assert_close(y, b.expand(4, 16), rtol=0, atol=0)
    cache = torch.randn(4, 16, 3, device="cuda")
    ref, nc = C.causal_conv1d_update(x.cpu().numpy(), cache.cpu().numpy(), None, None, None, None)
    y, _ = ops.causal_conv1d_update(x, cache, None, None, None, None)  # taps of one
    np.testing.assert_allclose(y.cpu().numpy(), ref, atol=1e-5)


# ------------------------------------------------------- full size (Qwen3-Next conv)

def test_qwen3_next_shape_against_torch_conv(ops):
    """Config-1 token count over the Qwen3-Next q/k/v conv channels
    (2*16*128 + 32*128 = 8192, width 4, SiLU): the fla forward equals a
    depthwise torch conv1d in fp32, and the vLLM-layout op equals the fla
    one on the same data (a layout-independent property)."""
    T, D, W = 8192, 8192, 4
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(1, T, D, device="cuda", generator=g).bfloat16()
    w = (torch.randn(D, W, device="cuda", generator=g) * 0.3).bfloat16()
    y, _ = ops.causal_conv1d(x, w, None, None, None, False, "silu")
    ref = torch.nn.functional.conv1d(torch.nn.functional.pad(x.float().transpose(1, 2), (W - 1, 0)),
                                     w.float()[:, None, :], groups=D)
    ref = torch.nn.functional.silu(ref).transpose(1, 2)
    assert (y.float() - ref).abs().max().item() <= 1.6e-2 * max(1.0, ref.abs().max().item())
    cs = torch.zeros(2, W - 1, D, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    out = ops.causal_conv1d_fn(x[0].t(), w, None, cs, torch.tensor([0, T], device="cuda", dtype=torch.int32),
                               torch.tensor([1], device="cuda", dtype=torch.int32),
                               torch.tensor([False], device="cuda"), "silu")
    assert torch.equal(out.t(), y[0])
    assert torch.equal(cs[1].t(), x[0, T - 3:])


@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("W", [2, 3, 4])
def test_16bit_taps_match_fp32_taps(ops, wdtype, W):
    """16-bit taps and bias (read as 16-byte vectors) give the same bits as
    the same values passed in fp32 (read one by one)."""
    g = torch.Generator(device="cuda").manual_seed(30 + W)
    T, D = 300, 2048
    x = torch.randn(1, T, D, device="cuda", generator=g).to(wdtype)
    w = (torch.randn(D, W, device="cuda", generator=g) * 0.3).to(wdtype)
    b = torch.randn(D, device="cuda", generator=g).to(wdtype)
    y16, _ = ops.causal_conv1d(x, w, b, None, None, False, "silu")
    y32, _ = ops.causal_conv1d(x, w.float(), b.float(), None, None, False, "silu")
    assert torch.equal(y16, y32)


def test_errors_match_reference(ops):
    x = torch.randn(1, 8, 16, device="cuda")
    w = torch.randn(16, 4, device="cuda")
    with pytest.raises(ValueError, match="output_final_state"):
        ops.causal_conv1d(x, w, output_final_state=True)
    with pytest.raises(ValueError, match="Unsupported backend"):
        ops.causal_conv1d(x, w, backend="cuda")
    with pytest.raises(ValueError, match="weight.shape"):
        ops.causal_conv1d(x, torch.randn(15, 4, device="cuda"))
    with pytest.raises(ValueError, match="less than or equal to 4"):
        ops.causal_conv1d_fn(x[0].t(), torch.randn(16, 5, device="cuda"), None,
                             torch.zeros(1, 16, 4, device="cuda"), torch.tensor([0, 8], device="cuda"))


def test_fn_prefix_caching_random(ops):
    """Prefix-caching block states against the oracle on random metadata
    whose block arithmetic stays non-negative (as vLLM schedules it)."""
    rng = np.random.default_rng(11)
    dim, W, B = 96, 4, 128
    lens = [300, 64, 129, 5, 257]
    total = sum(lens)
    qsl = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    x = rng.standard_normal((total, dim)).astype(np.float32)
    w = (rng.standard_normal((dim, W)) * 0.5).astype(np.float32)
    lines = 40
    st = rng.standard_normal((lines, W - 1, dim)).astype(np.float32)
    ci = rng.permutation(np.arange(1, lines)).astype(np.int32)[: len(lens) * 6].reshape(len(lens), 6)
    first = np.array([0, 1, 2, 0, 1], np.int32)
    last = np.array([2, 1, 3, 0, 3], np.int32)
    init = np.array([5, 0, 4, 3, 0], np.int32)
    ncomp = np.array([100, 64, 70, 0, 120], np.int32)
    has = np.array([1, 1, 0, 1, 1], bool)
    cs = _t(st).transpose(1, 2)
    cs_in = cs.cpu().numpy()
    out = ops.causal_conv1d_fn(_t(x).t(), _t(w), None, cs, torch.tensor(qsl, device="cuda"),
                               torch.tensor(ci, device="cuda"), torch.tensor(has, device="cuda"), "silu",
                               block_idx_first_scheduled_token=torch.tensor(first, device="cuda"),
                               block_idx_last_scheduled_token=torch.tensor(last, device="cuda"),
                               initial_state_idx=torch.tensor(init, device="cuda"),
                               num_computed_tokens=torch.tensor(ncomp, device="cuda"), block_size_to_align=B)
    ref, cs_ref, _ = C.causal_conv1d_fn(x.T, w, None, cs_in, qsl, ci, has, "silu",
                                        block_idx_first_scheduled_token=first, block_idx_last_scheduled_token=last,
                                        initial_state_idx=init, num_computed_tokens=ncomp, block_size_to_align=B)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=2e-5, rtol=0)
    np.testing.assert_allclose(cs.cpu().numpy(), cs_ref, atol=0, rtol=0)
