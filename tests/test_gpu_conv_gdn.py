"""The causal conv1d fused into the chunked prefill (gdn_conv_chunk_fwd)
against the two separate device ops it replaces: causal_conv1d_fn, then
chunk_gated_delta_rule on the q/k/v split of its output.  Both run the same
arithmetic, so the outputs, final states and updated conv cache lines must be
bit-identical.  The separate ops are themselves pinned to the reference
(conv fixtures and the GDN oracle), which makes the fused path pinned too."""

import numpy as np
import pytest
import torch

from gdn_testutil import BF16_MAX_ABS, BF16_REL_RMS, max_abs, np64, rel_rms

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import domesticated_torch_mlu_ops_b200 as m
    from domesticated_torch_mlu_ops_b200 import _lib
    return m, _lib.load()


def _case(seed, lens, H, HV, dtype=torch.bfloat16, lines=None, bias=True, has=None, idx=None, h0=True,
          state_dtype=None, xs=1.5):
    gen = torch.Generator().manual_seed(seed)
    K = V = 128
    dim = 2 * H * K + HV * V
    total = sum(lens)
    N = len(lens)
    lines = lines or N + 3
    x = (torch.randn(total, dim, generator=gen) * xs).to(dtype).cuda()  # token-major storage
    w = (torch.randn(dim, 4, generator=gen) * 0.5).to(dtype).cuda()
    b = (torch.randn(dim, generator=gen) * 0.2).to(dtype).cuda() if bias else None
    st = (torch.randn(lines, 3, dim, generator=gen)).to(state_dtype or dtype).cuda().transpose(1, 2)
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device="cuda")
    if idx is None:
        idx = torch.randperm(lines, generator=gen)[:N].to(torch.int32)
    if has is None:
        has = torch.rand(N, generator=gen) < 0.6
    g = torch.nn.functional.logsigmoid(torch.randn(1, total, HV, generator=gen)).cuda()
    beta = torch.sigmoid(torch.randn(1, total, HV, generator=gen)).cuda()
    init = (torch.randn(N, HV, K, V, generator=gen) * 0.05).cuda() if h0 else None
    return dict(x=x.t(), w=w, b=b, st=st, qsl=qsl, idx=torch.as_tensor(idx).cuda(),
                has=torch.as_tensor(has).cuda(), g=g, beta=beta, h0=init, H=H, HV=HV)


def _composed(m, c, st, act="silu", l2=True, **apc):
    H, HV, K = c["H"], c["HV"], 128
    y = m.causal_conv1d_fn(c["x"], c["w"], c["b"], st, c["qsl"], c["idx"], c["has"], act, **apc)
    yt = y.t()
    total = yt.shape[0]
    q = yt[:, :H * K].reshape(1, total, H, K)
    k = yt[:, H * K:2 * H * K].reshape(1, total, H, K)
    v = yt[:, 2 * H * K:].reshape(1, total, HV, K)
    o, ht = m.chunk_gated_delta_rule(q, k, v, c["g"], c["beta"], None, c["h0"], True, cu_seqlens=c["qsl"],
                                     use_qk_l2norm_in_kernel=l2)
    return o, ht, (q, k, v)


def _fused(m, c, st, act="silu", l2=True, **apc):
    return m.causal_conv1d_chunk_gated_delta_rule(
        c["x"], c["w"], c["b"], st, c["qsl"], c["g"], c["beta"], c["H"], c["HV"], initial_state=c["h0"],
        output_final_state=True, cache_indices=c["idx"], has_initial_state=c["has"], activation=act,
        use_qk_l2norm_in_kernel=l2, check_errors=True, **apc)


def _check_identical(m, c, act="silu", l2=True, **apc):
    st_a, st_b = c["st"].clone(), c["st"].clone()
    o_a, ht_a, _ = _composed(m, c, st_a, act, l2, **apc)
    o_b, ht_b = _fused(m, c, st_b, act, l2, **apc)
    torch.cuda.synchronize()
    assert torch.equal(o_a, o_b)
    assert torch.equal(ht_a, ht_b)
    assert torch.equal(st_a, st_b)
    return o_b, ht_b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,HV", [(2, 4), (3, 3)])
def test_fused_matches_conv_then_prefill(ops, dtype, H, HV):
    """Ragged lengths: shorter than the conv window, chunk-aligned, one token
    past a chunk, and a long sequence; initial cache lines on some sequences."""
    m, _ = ops
    c = _case(1, [1, 2, 3, 64, 65, 200, 7], H, HV, dtype)
    _check_identical(m, c)


@pytest.mark.parametrize("act", ["silu", None])
def test_fused_activation_bias_l2norm_variants(ops, act):
    m, _ = ops
    # without the L2 norm the keys must be short for a stable recurrence
    c = _case(2, [130, 17, 64], 2, 4, bias=False, h0=False, xs=0.05)
    o, _ = _check_identical(m, c, act=act, l2=False)
    assert torch.isfinite(o.float()).all()
    c = _case(3, [130, 17, 64], 2, 4, bias=True, h0=True)
    _check_identical(m, c, act=act, l2=True)


def test_fused_pad_slot_and_all_initial_states(ops):
    """A PAD cache line: the conv outputs of that sequence are zeros in both
    forms and its line is left alone; every other sequence starts from its
    cached window."""
    m, _ = ops
    c = _case(4, [70, 40, 129], 2, 4, lines=6, idx=[3, -1, 0], has=[True, True, True])
    before = c["st"][[3, 0, 1, 2, 4, 5]].clone()
    _check_identical(m, c)
    st = c["st"].clone()
    _fused(m, c, st)
    torch.cuda.synchronize()
    for ln in (1, 2, 4, 5):  # lines no sequence owns
        assert torch.equal(st[ln], c["st"][ln])
    assert not torch.equal(st[3], before[0])  # an owned line was rewritten


def test_fused_prefix_caching(ops):
    m, _ = ops
    lens = [300, 64, 129]
    c = _case(5, lens, 2, 4, lines=24, has=[True, False, True], idx=torch.arange(1, 19).reshape(3, 6))
    dev = "cuda"
    apc = dict(block_idx_first_scheduled_token=torch.tensor([0, 1, 2], dtype=torch.int32, device=dev),
               block_idx_last_scheduled_token=torch.tensor([2, 1, 3], dtype=torch.int32, device=dev),
               initial_state_idx=torch.tensor([5, 0, 4], dtype=torch.int32, device=dev),
               num_computed_tokens=torch.tensor([100, 64, 70], dtype=torch.int32, device=dev),
               block_size_to_align=128)
    _check_identical(m, c, **apc)


def test_fused_qwen3_next_layer_shape_against_oracle(ops):
    """Config-1 layer shape (one 8192-token sequence, 16 q/k heads, 32 v
    heads): bit-identical to the two ops, and the GDN part within the bf16
    tolerances of the fp64 oracle evaluated on the conv output."""
    import oracle
    m, _ = ops
    c = _case(6, [8192], 16, 32, lines=2, idx=[1], has=[True])
    o, ht = _check_identical(m, c)
    st = c["st"].clone()
    _, _, (q, k, v) = _composed(m, c, st)
    sel = slice(0, 4)  # four v-heads (two q/k heads) of the oracle, to keep the CPU time short
    ref_o, ref_h = oracle.chunk_gated_delta_rule(np64(q)[:, :, :2], np64(k)[:, :, :2], np64(v)[:, :, sel],
                                            np64(c["g"])[:, :, sel], np64(c["beta"])[:, :, sel],
                                            initial_state=np64(c["h0"])[:, sel], output_final_state=True,
                                            use_qk_l2norm_in_kernel=True)
    assert rel_rms(np64(o)[:, :, sel], ref_o) <= BF16_REL_RMS
    assert max_abs(np64(o)[:, :, sel], ref_o) <= BF16_MAX_ABS
    assert rel_rms(np64(ht)[:, sel], ref_h) <= BF16_REL_RMS


def test_fused_launches_its_own_kernels(ops):
    """The fused call runs the plan, WY (with the conv), state and cache-line
    kernels: four launches of this library, against five for the two ops."""
    m, lib = ops
    c = _case(7, [100, 50], 2, 4)
    st = c["st"].clone()
    n0 = lib.gdn_kernel_launch_count()
    _fused(m, c, st)
    n1 = lib.gdn_kernel_launch_count()
    _composed(m, c, st)
    n2 = lib.gdn_kernel_launch_count()
    assert n1 - n0 == 4
    assert n2 - n1 == 5


def test_unfusable_inputs_run_the_two_ops(ops):
    """fp32 cache lines are outside the fused kernels: the call runs the two
    device ops and gives their results."""
    m, _ = ops
    c = _case(8, [90, 33], 2, 4, state_dtype=torch.float32)
    _check_identical(m, c)


def test_fused_argument_errors(ops):
    m, _ = ops
    c = _case(9, [10], 2, 4)
    with pytest.raises(ValueError):
        m.causal_conv1d_chunk_gated_delta_rule(c["x"], c["w"], c["b"], c["st"], c["qsl"], c["g"], c["beta"],
                                               2, 3)  # channel count does not match the heads
    with pytest.raises(ValueError):
        m.causal_conv1d_chunk_gated_delta_rule(c["x"], c["w"], c["b"], c["st"], c["qsl"], c["g"][:, :5],
                                               c["beta"], 2, 4)
