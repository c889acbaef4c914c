"""GPU test of gdn_chunk_fwd_noalloc, the chunked prefill entry point for
callers that cannot allocate device memory (C hosts without a device
allocator of their own, serving engines that give the whole GPU to their own
memory pool at start-up, where cudaMalloc fails).

It is called through the C ABI twice in a row, and once captured in a CUDA graph
that is replayed twice; each result is compared with
gdn_chunk_fwd run on a caller-allocated workspace.  Both entry points run the
same deterministic kernels on the same inputs, so the outputs must be equal bit
for bit (a stricter check than the parity tolerances of the other tests).  The
error word of the built-in scratch is read back after each call.  The file
sorts last so that a run stopping at the first failure has run every other
test already.
"""

import ctypes

import numpy as np
import pytest
import torch

from domesticated_torch_mlu_ops_b200 import _lib
from gdn_testutil import make_inputs

pytestmark = pytest.mark.gpu

_DT = {torch.float32: _lib.GDN_F32, torch.bfloat16: _lib.GDN_BF16, torch.float16: _lib.GDN_F16}


def _args(q, k, v, g, beta, o, ht, h0=None, cu=None):
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = B if cu is None else cu.numel() - 1
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    return _lib.ChunkArgs(q=p(q), k=p(k), v=p(v), g=p(g), beta=p(beta), initial_state=p(h0),
                          o=p(o), final_state=p(ht), cu_seqlens=p(cu), B=B, T=T, N=N, H=H, HV=HV,
                          K=K, V=V, qkv_dtype=_DT[q.dtype], cu_dtype=_lib.GDN_I64, scale=0.0,
                          use_qk_l2norm=1)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype,K,T,cu", [
    (torch.bfloat16, 128, 300, None),              # tensor-core path
    (torch.bfloat16, 128, 260, [0, 70, 200, 260]),  # tensor-core path, packed sequences
    (torch.float32, 64, 150, None),                 # generic fp32 path
])
def test_noalloc_matches_allocating_entry(dtype, K, T, cu):
    assert torch.cuda.is_available()
    lib = _lib.load()
    N = 1 if cu is None else len(cu) - 1
    q, k, v, g, beta, h0 = make_inputs(7, 1, T, 2, 4, K, K, dtype=dtype, nseq_state=N, state_std=0.05)
    cut = None if cu is None else torch.tensor(cu, dtype=torch.int64, device="cuda")

    o_ref = torch.empty_like(v)
    ht_ref = torch.empty(N, 4, K, K, dtype=torch.float32, device="cuda")
    a = _args(q, k, v, g, beta, o_ref, ht_ref, h0, cut)
    nbytes = lib.gdn_chunk_workspace_size(ctypes.byref(a))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ctypes.c_void_p(ws.data_ptr()), nbytes
    assert lib.gdn_chunk_fwd(ctypes.byref(a), _stream()) == _lib.GDN_OK

    for _ in range(2):  # two calls in a row share (and reuse) the built-in scratch
        o = torch.full_like(v, float("nan"))
        ht = torch.full((N, 4, K, K), float("nan"), dtype=torch.float32, device="cuda")
        b = _args(q, k, v, g, beta, o, ht, h0, cut)
        rc = lib.gdn_chunk_fwd_noalloc(ctypes.byref(b), _stream())
        assert rc == _lib.GDN_OK, lib.gdn_last_error()
        assert lib.gdn_chunk_noalloc_check_device_error(_stream()) == _lib.GDN_OK, lib.gdn_last_error()
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref)
        assert torch.equal(ht, ht_ref)


def test_noalloc_rejects_oversized_requests():
    lib = _lib.load()
    q, k, v, g, beta, _ = make_inputs(8, 1, 8192, 16, 32, 128, 128)
    o = torch.empty_like(v)
    a = _args(q, k, v, g, beta, o, None)
    assert lib.gdn_chunk_workspace_size(ctypes.byref(a)) > (32 << 20)
    assert lib.gdn_chunk_fwd_noalloc(ctypes.byref(a), _stream()) == _lib.GDN_ERR_WORKSPACE
    assert b"32" in lib.gdn_last_error() or b"scratch" in lib.gdn_last_error()


def test_noalloc_replays_in_a_cuda_graph():
    """Callers that cannot allocate often capture their step in a CUDA graph:
    after one eager call, a call captured in a graph and replayed twice gives
    gdn_chunk_fwd's result bit for bit, and the scratch error word stays clear."""
    lib = _lib.load()
    q, k, v, g, beta, h0 = make_inputs(9, 1, 300, 2, 4, 128, 128, dtype=torch.bfloat16, nseq_state=1,
                                       state_std=0.05)
    o_ref = torch.empty_like(v)
    ht_ref = torch.empty(1, 4, 128, 128, dtype=torch.float32, device="cuda")
    a = _args(q, k, v, g, beta, o_ref, ht_ref, h0)
    nbytes = lib.gdn_chunk_workspace_size(ctypes.byref(a))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ctypes.c_void_p(ws.data_ptr()), nbytes
    assert lib.gdn_chunk_fwd(ctypes.byref(a), _stream()) == _lib.GDN_OK

    o = torch.empty_like(v)
    ht = torch.empty_like(ht_ref)
    b = _args(q, k, v, g, beta, o, ht, h0)
    assert lib.gdn_chunk_fwd_noalloc(ctypes.byref(b), _stream()) == _lib.GDN_OK, lib.gdn_last_error()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rc = lib.gdn_chunk_fwd_noalloc(ctypes.byref(b), _stream())
    assert rc == _lib.GDN_OK, lib.gdn_last_error()
    for _ in range(2):
        o.fill_(float("nan"))
        ht.fill_(float("nan"))
        graph.replay()
        assert lib.gdn_chunk_noalloc_check_device_error(_stream()) == _lib.GDN_OK, lib.gdn_last_error()
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref)
        assert torch.equal(ht, ht_ref)
    del graph
