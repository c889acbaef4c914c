"""torch.compile(fullgraph=True) traces the public ops as torch.library custom
ops (no graph break) and the compiled call matches eager bit for bit:
prefill, and the in-place slot-cache decode (whose cache mutation the op
declares)."""

import pytest
import torch

from gdn_testutil import make_inputs

pytestmark = pytest.mark.gpu

BACKENDS = ["aot_eager", "inductor"]


@pytest.fixture(scope="module")
def ops():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import domesticated_torch_mlu_ops_b200 as m
    return m


@pytest.mark.parametrize("backend", BACKENDS)
def test_compile_prefill_matches_eager(ops, backend):
    torch._dynamo.reset()
    q, k, v, g, beta, h0 = make_inputs(40, 1, 300, 2, 4, 128, 128, nseq_state=2, state_std=0.02)
    cu = torch.tensor([0, 120, 300], device="cuda")

    def f(q, k, v, g, beta, h0, cu):
        return ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cu, use_qk_l2norm_in_kernel=True)

    o1, h1 = f(q, k, v, g, beta, h0, cu)
    o2, h2 = torch.compile(f, fullgraph=True, backend=backend)(q, k, v, g, beta, h0, cu)
    assert torch.equal(o1, o2) and torch.equal(h1, h2)


@pytest.mark.parametrize("backend", BACKENDS)
def test_compile_inplace_decode_matches_eager(ops, backend):
    torch._dynamo.reset()
    N, HV, K = 6, 4, 128
    q, k, v, g, beta, _ = make_inputs(41, 1, N, 2, HV, K, K)
    gen = torch.Generator().manual_seed(42)
    cache = (torch.randn(16, HV, K, K, generator=gen) * 0.02).cuda()
    idx = torch.randperm(16, generator=gen)[:N].cuda()
    cu = torch.arange(N + 1, device="cuda")

    def f(q, k, v, g, beta, cache, cu, idx):
        o, c = ops.fused_recurrent_gated_delta_rule_fn(q, k, v, g, beta, K ** -0.5, cache, True, cu, idx,
                                                       None, True)
        return o

    c1, c2 = cache.clone(), cache.clone()
    o1 = f(q, k, v, g, beta, c1, cu, idx)
    o2 = torch.compile(f, fullgraph=True, backend=backend)(q, k, v, g, beta, c2, cu, idx)
    assert torch.equal(o1, o2)
    assert torch.equal(c1, c2) and not torch.equal(c1, cache)
