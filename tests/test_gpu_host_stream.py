"""chunk_gated_delta_rule_from_host (host-resident inputs streamed in pieces)
against one device call of chunk_gated_delta_rule on the same inputs."""

import pytest
import torch

from gdn_testutil import make_inputs, np64, rel_rms

pytestmark = pytest.mark.gpu


def _ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import domesticated_torch_mlu_ops_b200 as ops
    return ops


def _run_both(ops, q, k, v, g, beta, h0, cu, seg, l2=True, vfirst=False):
    o_d, ht_d = ops.chunk_gated_delta_rule(q, k, v, g, beta, None, h0, True, cu, state_v_first=vfirst,
                                           use_qk_l2norm_in_kernel=l2)
    host = [None if x is None else x.cpu() for x in (q, k, v, g, beta, h0, cu)]
    o_h, ht_h = ops.chunk_gated_delta_rule_from_host(*host[:5], None, host[5], True, host[6],
                                                     state_v_first=vfirst, use_qk_l2norm_in_kernel=l2,
                                                     device=q.device, segment_tokens=seg)
    torch.cuda.synchronize()
    assert not o_h.is_cuda and o_h.is_pinned()
    return o_d.cpu(), ht_d.cpu(), o_h, ht_h


@pytest.mark.parametrize("dtype,T,seg", [(torch.bfloat16, 1000, 256), (torch.float32, 300, 128),
                                         (torch.bfloat16, 4096, 1024), (torch.bfloat16, 2100, 2048)])
def test_time_pieces_equal_one_call(dtype, T, seg):
    """One sequence cut along time at 64-token chunk boundaries (the last
    segment in halving pieces), the fp32 state handed over on the device:
    bit-identical to one call."""
    ops = _ops()
    q, k, v, g, beta, h0 = make_inputs(3, 1, T, 2, 4, 128, 128, dtype=dtype, nseq_state=1, state_std=0.1)
    o_d, ht_d, o_h, ht_h = _run_both(ops, q, k, v, g, beta, h0, None, seg)
    assert torch.equal(o_d, o_h)
    assert torch.equal(ht_d, ht_h)


def test_time_pieces_without_initial_state_vfirst():
    ops = _ops()
    q, k, v, g, beta, _ = make_inputs(4, 1, 520, 1, 2, 64, 64, dtype=torch.bfloat16)
    q = torch.nn.functional.normalize(q.float(), dim=-1).bfloat16()  # no in-kernel norm: unit keys
    k = torch.nn.functional.normalize(k.float(), dim=-1).bfloat16()
    o_d, ht_d, o_h, ht_h = _run_both(ops, q, k, v, g, beta, None, None, 192, l2=False, vfirst=True)
    assert torch.equal(o_d, o_h)
    assert torch.equal(ht_d, ht_h)


def test_batch_groups():
    ops = _ops()
    q, k, v, g, beta, h0 = make_inputs(5, 5, 200, 2, 4, 128, 128, nseq_state=5, state_std=0.1)
    o_d, ht_d, o_h, ht_h = _run_both(ops, q, k, v, g, beta, h0, None, 448)
    assert rel_rms(np64(o_h), np64(o_d)) < 1e-3
    assert rel_rms(np64(ht_h), np64(ht_d)) < 1e-4


def test_varlen_groups_with_empty_sequences():
    ops = _ops()
    cu = torch.tensor([0, 100, 100, 300, 1000, 1064], dtype=torch.int64, device="cuda")
    q, k, v, g, beta, h0 = make_inputs(6, 1, 1064, 2, 4, 128, 128, nseq_state=5, state_std=0.1)
    o_d, ht_d, o_h, ht_h = _run_both(ops, q, k, v, g, beta, h0, cu, 256)
    assert rel_rms(np64(o_h), np64(o_d)) < 1e-3
    assert rel_rms(np64(ht_h), np64(ht_d)) < 1e-4
    assert torch.equal(ht_h[1], h0[1].cpu())  # the empty sequence keeps its state


def test_rejects_device_tensors_and_bad_segments():
    ops = _ops()
    q, k, v, g, beta, _ = make_inputs(7, 1, 64, 1, 1, 32, 32)
    with pytest.raises(ValueError):
        ops.chunk_gated_delta_rule_from_host(q, k, v, g, beta)
    with pytest.raises(ValueError):
        ops.chunk_gated_delta_rule_from_host(q.cpu(), k.cpu(), v.cpu(), g.cpu(), beta.cpu(), segment_tokens=100)
