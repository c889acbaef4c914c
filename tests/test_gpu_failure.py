"""Failure detection on the GPU without a GPU fault.

* The prefill's device error word starts clear on every call, even in a
  workspace full of stale bytes.
* A bounded wait that runs out: ``gdn_chunk_fwd_test_stall`` makes the first
  block of the state recurrence skip one chunk's operand copies (so nothing
  is in flight on that barrier) and bounds its waits by a few million cycles.
  The call must report ``GDN_ERR_DEVICE`` through
  ``gdn_chunk_check_device_error``, leave the other v-heads' outputs equal to
  a clean run, and the next normal call on the same workspace must be bit
  identical to a clean run (the context stays usable).  Both prefill paths:
  the fused cluster kernel and the separate WY + state kernels.
* The decode slot guard: a declared slot count smaller than the allocated
  cache, so the "bad" index still points inside the allocation; the sequence
  is skipped like PAD and code 2 is recorded.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from domesticated_torch_mlu_ops_b200 import _lib
from gdn_testutil import make_inputs, np64, rel_rms

pytestmark = pytest.mark.gpu

SITE_STATE_LOAD = 4
SITE_SLOT_INITIAL, SITE_SLOT_FINAL = 9, 10


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _chunk_args(q, k, v, g, beta, o, ht):
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    return _lib.ChunkArgs(q=p(q), k=p(k), v=p(v), g=p(g), beta=p(beta), o=p(o), final_state=p(ht),
                          B=B, T=T, N=B, H=H, HV=HV, K=K, V=V, qkv_dtype=_lib.GDN_BF16,
                          cu_dtype=_lib.GDN_I64, scale=0.0, use_qk_l2norm=1)


def _run(lib, fn, a, ws, *extra):
    a.workspace, a.workspace_bytes = ctypes.c_void_p(ws.data_ptr()), ws.numel()
    rc = fn(ctypes.byref(a), *extra, _stream())
    assert rc == _lib.GDN_OK, lib.gdn_last_error()


def test_error_word_starts_clear_in_a_stale_workspace():
    lib = _lib.load()
    q, k, v, g, beta, _ = make_inputs(30, 1, 200, 2, 4, 128, 128)
    o = torch.empty_like(v)
    a = _chunk_args(q, k, v, g, beta, o, None)
    ws = torch.full((lib.gdn_chunk_workspace_size(ctypes.byref(a)),), 0xFF, dtype=torch.uint8,
                    device="cuda")
    _run(lib, lib.gdn_chunk_fwd, a, ws)
    assert lib.gdn_chunk_check_device_error(ctypes.c_void_p(ws.data_ptr()), _stream()) == _lib.GDN_OK


@pytest.fixture(params=["fused", "split"])
def prefill_path(request, monkeypatch):
    """The fused cluster kernel (default) or the separate WY + state kernels."""
    monkeypatch.setenv("GDN_TC_FUSED", "1" if request.param == "fused" else "0")
    return request.param


@pytest.mark.parametrize("stall_chunk", [0, 4])
def test_state_kernel_wait_timeout_is_reported_and_recovers(stall_chunk, prefill_path):
    lib = _lib.load()
    T, HV = 640, 4  # 10 chunks; the state kernel uses 32-column V-slices here
    q, k, v, g, beta, _ = make_inputs(31, 1, T, 2, HV, 128, 128)
    o_ref, ht_ref = torch.empty_like(v), torch.empty(1, HV, 128, 128, device="cuda")
    a = _chunk_args(q, k, v, g, beta, o_ref, ht_ref)
    ws = torch.empty(lib.gdn_chunk_workspace_size(ctypes.byref(a)), dtype=torch.uint8, device="cuda")
    _run(lib, lib.gdn_chunk_fwd, a, ws)
    wsp = ctypes.c_void_p(ws.data_ptr())
    assert lib.gdn_chunk_check_device_error(wsp, _stream()) == _lib.GDN_OK

    o, ht = torch.zeros_like(v), torch.zeros(1, HV, 128, 128, device="cuda")
    b = _chunk_args(q, k, v, g, beta, o, ht)
    _run(lib, lib.gdn_chunk_fwd_test_stall, b, ws, stall_chunk, 4_000_000)
    rc = lib.gdn_chunk_check_device_error(wsp, _stream())
    assert rc == _lib.GDN_ERR_DEVICE
    msg = lib.gdn_last_error().decode()
    assert "code 1" in msg and f"site {SITE_STATE_LOAD}" in msg and "block 0" in msg, msg
    torch.cuda.synchronize()
    # every block but the stalled one (v-head 0, columns 0..31) finished normally
    assert torch.equal(o[:, :, 1:], o_ref[:, :, 1:])
    assert torch.equal(o[:, :, 0, 32:], o_ref[:, :, 0, 32:])
    assert torch.equal(ht[:, 1:], ht_ref[:, 1:])
    # the stalled block emitted the chunks before the one before the stall
    done = 64 * max(stall_chunk - 1, 0)
    assert torch.equal(o[:, :done, 0, :32], o_ref[:, :done, 0, :32])

    # the context and the workspace stay usable: a normal call is bit identical
    o2, ht2 = torch.empty_like(v), torch.empty_like(ht_ref)
    c = _chunk_args(q, k, v, g, beta, o2, ht2)
    _run(lib, lib.gdn_chunk_fwd, c, ws)
    assert lib.gdn_chunk_check_device_error(wsp, _stream()) == _lib.GDN_OK
    assert torch.equal(o2, o_ref) and torch.equal(ht2, ht_ref)


def _decode_args(q, k, v, g, beta, cache, o, cu, idx, num_slots, err):
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    return _lib.RecurrentArgs(
        q=p(q), k=p(k), v=p(v), g=p(g), beta=p(beta), initial_state=p(cache), o=p(o), final_state=p(cache),
        cu_seqlens=p(cu), ssm_state_indices=p(idx), B=B, T=T, N=cu.numel() - 1, H=H, HV=HV, K=K, V=V,
        qkv_dtype=_lib.GDN_BF16, cu_dtype=_lib.GDN_I64, idx_dtype=_lib.GDN_I64, nacc_dtype=_lib.GDN_I64,
        stride_init_state_token=cache.stride(0), stride_final_state_token=cache.stride(0),
        stride_indices_seq=1, stride_indices_tok=1, scale=K ** -0.5, use_qk_l2norm=1,
        beta_per_v=0, inplace_final_state=1, num_slots=num_slots, err=p(err))


@pytest.mark.parametrize("K", [128, 64])  # streaming kernel and the general kernel
def test_decode_slot_guard(K):
    lib = _lib.load()
    N, slots, declared, HV = 6, 40, 30, 4
    q, k, v, g, beta, _ = make_inputs(32, 1, N, 2, HV, K, K)
    gen = torch.Generator().manual_seed(33)
    cache = (torch.randn(slots, HV, K, K, generator=gen) * 0.05).cuda()
    idx = torch.tensor([3, 35, 7, 12, 29, 0], dtype=torch.int64, device="cuda")  # 35 >= declared
    cu = torch.arange(N + 1, device="cuda")
    before = cache.clone()
    o = torch.full_like(v, 7.0)
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    a = _decode_args(q, k, v, g, beta, cache, o, cu, idx, declared, err)
    assert lib.gdn_fused_recurrent_fwd(ctypes.byref(a), _stream()) == _lib.GDN_OK, lib.gdn_last_error()
    torch.cuda.synchronize()
    code, site, seq, info = err.tolist()
    assert (code, site, seq, info) == (2, SITE_SLOT_INITIAL, 1, 35)
    assert torch.all(o[0, 1] == 0)                 # skipped like PAD
    assert torch.equal(cache[35], before[35])      # untouched
    ro, rcache, _ = oracle.recurrent_v_first(
        np64(q), np64(k), np64(v), np64(g), np64(beta), K ** -0.5, np64(before).copy(),
        cu_seqlens=cu.cpu().numpy(), ssm_state_indices=np.array([3, -1, 7, 12, 29, 0]),
        use_qk_l2norm_in_kernel=True)
    ok = [0, 2, 3, 4, 5]
    assert rel_rms(np64(o)[0, ok], ro[0, ok]) < 1e-2
    assert rel_rms(np64(cache), rcache) < 1e-4


def test_decode_check_errors_raises_from_python():
    import domesticated_torch_mlu_ops_b200 as ops
    N, HV, K = 4, 4, 128
    q, k, v, g, beta, _ = make_inputs(34, 1, N, 2, HV, K, K)
    cache = torch.zeros(8, HV, K, K, device="cuda")
    cu = torch.arange(N + 1, device="cuda")
    idx = torch.tensor([0, 1, 2, 9], device="cuda")  # 9 is past the 8-slot cache
    with pytest.raises(_lib.GdnError, match="slot index out of range"):
        ops.fused_recurrent_gated_delta_rule_fn(q, k, v, g, beta, None, cache, True, cu, idx, None, True,
                                                check_errors=True)
    # the word was cleared by the raise: a valid call passes the check
    idx = torch.tensor([0, 1, 2, 3], device="cuda")
    ops.fused_recurrent_gated_delta_rule_fn(q, k, v, g, beta, None, cache, True, cu, idx, None, True,
                                            check_errors=True)
