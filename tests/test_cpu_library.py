"""The ops are torch.library custom ops with fake implementations (CPU, no
GPU needed): schemas, mutation declarations, and output shapes / dtypes
under FakeTensorMode for every op, as torch.compile sees them."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import domesticated_torch_mlu_ops_b200 as ops


def test_schemas_declare_mutation():
    s = {n: str(getattr(torch.ops.gdn_b200, n).default._schema)
         for n in ("chunk_fwd", "chunk_bwd", "recurrent_fn_inplace", "recurrent_fn", "recurrent_plain",
                   "solve_tril")}
    assert "!" not in s["chunk_fwd"] and "!" not in s["chunk_bwd"] and "!" not in s["recurrent_fn"]
    assert "Tensor(a7!) state" in s["recurrent_fn_inplace"]
    assert "Tensor(a1!) output" in s["solve_tril"] and s["solve_tril"].endswith("-> ()")


@pytest.mark.parametrize("svf", [False, True])
def test_chunk_fake_shapes(svf):
    with FakeTensorMode():
        q = torch.empty(1, 300, 4, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty_like(q)
        v = torch.empty(1, 300, 8, 64, dtype=torch.bfloat16, device="cuda")
        g = torch.empty(1, 300, 8, device="cuda")
        b = torch.empty(1, 300, 8, device="cuda")
        cu = torch.tensor([0, 100, 250, 300], device="cuda")
        h0 = torch.empty((3, 8, 64, 128) if svf else (3, 8, 128, 64), device="cuda")
        o, ht = ops.chunk_gated_delta_rule(q, k, v, g, b, None, h0, True, cu, state_v_first=svf,
                                           use_qk_l2norm_in_kernel=True)
        assert o.shape == v.shape and o.dtype == torch.bfloat16 and o.device.type == "cuda"
        assert ht.shape == h0.shape and ht.dtype == torch.float32
        o, ht = ops.chunk_gated_delta_rule(q, k, v, g, b)
        assert ht is None and o.shape == v.shape
        dq, dk, dv, db, dg, dh0 = ops.chunk_gated_delta_rule_bwd(q, k, v, g, b, None, h0, o, None, cu,
                                                                  state_v_first=svf)
        assert (dq.shape, dk.shape, dv.shape) == (q.shape, k.shape, v.shape)
        assert dg.shape == g.shape and db.dtype == torch.float32 and dh0.shape == h0.shape


def test_decode_and_misc_fake_shapes():
    with FakeTensorMode():
        N, HV, K = 5, 8, 128
        q = torch.empty(1, N, 4, K, dtype=torch.bfloat16, device="cuda")
        v = torch.empty(1, N, HV, K, dtype=torch.bfloat16, device="cuda")
        g = torch.empty(1, N, HV, device="cuda")
        gk = torch.empty(1, N, HV, K, device="cuda")
        cache = torch.empty(20, HV, K, K, device="cuda")
        idx = torch.empty(N, dtype=torch.int32, device="cuda")
        cu = torch.arange(N + 1, device="cuda")
        o, c = ops.fused_recurrent_gated_delta_rule_fn(q, q, v, g, g, None, cache, True, cu, idx, None, True)
        assert o.shape == v.shape and c is cache
        o, c = ops.fused_recurrent_gated_delta_rule_fn(q, q, v, gk, g, None, cache, False, cu, idx)
        assert c.shape == (N, HV, K, K) and c.dtype == torch.float32
        o, ht = ops.fused_recurrent_gated_delta_rule(q, q, v, g, None, None, g, None, None, True)
        assert o.shape == v.shape and ht.shape == (1, HV, K, K)
        A = torch.empty(300, 8, 64, device="cuda")  # packed [total_tokens, H, BT]
        out = ops.solve_tril(A, None, torch.tensor([0, 300], device="cuda"), torch.bfloat16)
        assert out.shape == A.shape and out.dtype == torch.bfloat16


def test_state_stage_fake_shapes():
    assert "Tensor(a6!)? h" in str(torch.ops.gdn_b200.chunk_fwd_h.default._schema)
    with FakeTensorMode():
        k = torch.empty(1, 130, 2, 64, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(1, 130, 4, 64, dtype=torch.bfloat16, device="cuda")
        u = torch.empty(1, 130, 4, 32, dtype=torch.bfloat16, device="cuda")
        gk = torch.empty(1, 130, 4, 64, device="cuda")
        h, v_new, ht = ops.chunk_gated_delta_rule_fwd_h(k, w, u, None, gk, None, True, state_v_first=True)
        assert h.shape == (1, 3, 4, 32, 64) and h.dtype == torch.bfloat16
        assert v_new.shape == u.shape and ht.shape == (1, 4, 32, 64) and ht.dtype == torch.float32


def test_ops_reject_cpu_tensors():
    q = torch.zeros(1, 4, 2, 16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.chunk_gated_delta_rule(q, q, q, q[..., 0], q[..., 0])


def test_conv_prefill_fake_shapes():
    assert "Tensor(a3!) conv_states" in str(torch.ops.gdn_b200.conv_chunk_fwd.default._schema)
    with FakeTensorMode():
        H, HV, T = 2, 4, 300
        dim = 2 * H * 128 + HV * 128
        x = torch.empty(T, dim, dtype=torch.bfloat16, device="cuda").t()
        w = torch.empty(dim, 4, dtype=torch.bfloat16, device="cuda")
        st = torch.empty(5, 3, dim, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
        qsl = torch.tensor([0, 100, 300], dtype=torch.int32, device="cuda")
        g = torch.empty(1, T, HV, device="cuda")
        o, ht = ops.causal_conv1d_chunk_gated_delta_rule(x, w, None, st, qsl, g, g, H, HV,
                                                         output_final_state=True)
        assert o.shape == (1, T, HV, 128) and o.dtype == torch.bfloat16
        assert ht.shape == (2, HV, 128, 128) and ht.dtype == torch.float32
