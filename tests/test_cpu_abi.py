"""CPU checks of the C ABI: the library loads, exports every function that
include/gdn_b200.h declares, its struct layouts match the ctypes mirrors, and
argument validation returns status codes (no GPU needed for any of this)."""

import ctypes
import os
import re
import subprocess

import pytest

from domesticated_torch_mlu_ops_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


def _declared():
    txt = open(HEADER).read()
    return re.findall(r"GDN_API\s+[\w\s\*]*?\b(gdn_\w+)\s*\(", txt)


def test_header_declares_expected_api():
    assert sorted(_declared()) == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.gdn_abi_version() == 3
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert set(_declared()) <= exported
    # nothing but the C ABI is exported
    assert {s for s in exported if not s.startswith("gdn_")} <= {"_init", "_fini"}


@pytest.mark.parametrize("struct,cname", [(_lib.ChunkArgs, "gdn_chunk_args"),
                                          (_lib.ChunkBwdArgs, "gdn_chunk_bwd_args"),
                                          (_lib.RecurrentArgs, "gdn_recurrent_args"),
                                          (_lib.ChunkHArgs, "gdn_chunk_h_args"),
                                          (_lib.RecurrentPlainArgs, "gdn_recurrent_plain_args"),
                                          (_lib.Conv1dArgs, "gdn_conv1d_args"),
                                          (_lib.Conv1dFnArgs, "gdn_conv1d_fn_args"),
                                          (_lib.Conv1dUpdateArgs, "gdn_conv1d_update_args")])
def test_struct_layout_matches_c(tmp_path, struct, cname):
    fields = [f[0] for f in struct._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', 'int main(void){',
           f'printf("%zu\\n", sizeof({cname}));']
    src += [f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields]
    src += ['return 0;}']
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(c)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(struct)
    assert vals[1:] == [getattr(struct, f).offset for f in fields]


def _chunk_args(**kw):
    base = dict(B=1, T=8192, N=1, H=16, HV=32, K=128, V=128, qkv_dtype=_lib.GDN_BF16,
                cu_dtype=_lib.GDN_I64)
    base.update(kw)
    return _lib.ChunkArgs(**base)


def test_workspace_size_and_validation():
    lib = _lib.load()
    ok = lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args()))
    assert ok > 0
    # HV not a multiple of H
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(HV=24, H=16))) == 0
    assert b"multiple" in lib.gdn_last_error()
    # K > 128 (reference asserts K <= 128, triton/fla/chunk.py:27)
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(K=256))) == 0
    # bad dtype
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(qkv_dtype=7))) == 0
    # varlen needs B == 1
    a = _chunk_args(B=2, N=3)
    a.cu_seqlens = ctypes.c_void_p(16)
    assert lib.gdn_chunk_workspace_size(ctypes.byref(a)) == 0


def test_token_stride_validation():
    lib = _lib.load()
    # strided rows on the tensor-core path: multiples of 8 at least the packed width
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(q_token_stride=8192, k_token_stride=8192,
                                                                 v_token_stride=8192))) > 0
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(q_token_stride=2047))) == 0
    assert b"token strides" in lib.gdn_last_error()
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(v_token_stride=2048))) == 0  # < HV*V
    # other paths read packed rows only
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(q_token_stride=4096, force_generic=1))) == 0
    assert lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(qkv_dtype=_lib.GDN_F32,
                                                                 q_token_stride=4096))) == 0
    assert b"tensor-core path only" in lib.gdn_last_error()
    assert lib.gdn_chunk_fwd_host_buffer_size(ctypes.byref(_chunk_args(q_token_stride=4096)), 2048) == 0
    # the fused conv prefill: width 4 only, no conv output tensor
    f = _lib.Conv1dFnArgs(x=ctypes.c_void_p(256), weight=ctypes.c_void_p(256), conv_states=ctypes.c_void_p(256),
                          query_start_loc=ctypes.c_void_p(256), stride_x_token=8192, stride_state_seq=3 * 8192,
                          stride_state_tok=8192, num_cache_lines=4, batch=1, dim=8192, total_tokens=8192, W=3,
                          x_dtype=_lib.GDN_BF16, w_dtype=_lib.GDN_BF16, state_dtype=_lib.GDN_BF16,
                          qsl_dtype=_lib.GDN_I32, activation=_lib.GDN_ACT_SILU)
    a = _chunk_args(g=ctypes.c_void_p(256), beta=ctypes.c_void_p(256), o=ctypes.c_void_p(256),
                    cu_seqlens=ctypes.c_void_p(256), cu_dtype=_lib.GDN_I32)
    assert lib.gdn_conv_chunk_workspace_size(ctypes.byref(a)) > lib.gdn_chunk_workspace_size(ctypes.byref(a))
    assert lib.gdn_conv_chunk_fwd(ctypes.byref(a), ctypes.byref(f), None) == _lib.GDN_ERR_UNSUPPORTED
    f.W = 4
    f.out = ctypes.c_void_p(256)
    assert lib.gdn_conv_chunk_fwd(ctypes.byref(a), ctypes.byref(f), None) == _lib.GDN_ERR_INVALID
    f.out = None
    f.dim = 8192 - 128
    assert lib.gdn_conv_chunk_fwd(ctypes.byref(a), ctypes.byref(f), None) == _lib.GDN_ERR_INVALID
    assert b"2*H*K + HV*V" in lib.gdn_last_error()


def test_invalid_calls_return_codes_without_touching_the_gpu():
    lib = _lib.load()
    a = _chunk_args()
    # null input pointers
    assert lib.gdn_chunk_fwd(ctypes.byref(a), None) == _lib.GDN_ERR_INVALID
    # workspace too small
    for name in ("q", "k", "v", "g", "beta", "o"):
        setattr(a, name, ctypes.c_void_p(256))
    a.workspace = ctypes.c_void_p(256)
    a.workspace_bytes = 16
    assert lib.gdn_chunk_fwd(ctypes.byref(a), None) == _lib.GDN_ERR_WORKSPACE
    r = _lib.RecurrentArgs(B=1, T=1, N=1, H=2, HV=4, K=6, V=8, qkv_dtype=_lib.GDN_BF16)
    assert lib.gdn_fused_recurrent_fwd(ctypes.byref(r), None) == _lib.GDN_ERR_UNSUPPORTED
    r = _lib.RecurrentArgs(B=1, T=1, N=1, H=2, HV=4, K=8, V=8, qkv_dtype=_lib.GDN_BF16)
    for name in ("q", "k", "v", "beta", "o", "initial_state", "final_state"):
        setattr(r, name, ctypes.c_void_p(256))
    r.inplace_final_state = 1
    assert lib.gdn_fused_recurrent_fwd(ctypes.byref(r), None) == _lib.GDN_ERR_INVALID
    assert b"ssm_state_indices" in lib.gdn_last_error()
    assert lib.gdn_solve_tril(None, None, 0, None, 0, 1, 1, 64, 2, 48, None) == _lib.GDN_ERR_INVALID


def test_bwd_validation_returns_codes_without_touching_the_gpu():
    lib = _lib.load()
    b = _lib.ChunkBwdArgs(B=1, T=130, N=1, H=2, HV=4, K=64, V=64, qkv_dtype=_lib.GDN_F32)
    need = lib.gdn_chunk_bwd_workspace_size(ctypes.byref(b))
    # forward intermediates (generic layout) plus the backward's own buffers
    fwd = lib.gdn_chunk_workspace_size(ctypes.byref(_chunk_args(T=130, H=2, HV=4, K=64, V=64,
                                                                  qkv_dtype=_lib.GDN_F32, force_generic=1)))
    assert need > fwd > 0
    assert lib.gdn_chunk_bwd(ctypes.byref(b), None) == _lib.GDN_ERR_INVALID  # null pointers
    assert b"dout" in lib.gdn_last_error()
    for name in ("q", "k", "v", "g", "beta", "dout", "dq", "dk", "dv", "dg", "dbeta"):
        setattr(b, name, ctypes.c_void_p(256))
    b.workspace, b.workspace_bytes = ctypes.c_void_p(256), need - 1
    assert lib.gdn_chunk_bwd(ctypes.byref(b), None) == _lib.GDN_ERR_WORKSPACE
    b.HV = 3
    assert lib.gdn_chunk_bwd_workspace_size(ctypes.byref(b)) == 0
    assert b"multiple" in lib.gdn_last_error()


def test_host_stream_sizing_and_validation():
    import numpy as np
    lib = _lib.load()
    a = _chunk_args(T=1000, H=2, HV=4)
    assert lib.gdn_chunk_fwd_host_buffer_size(ctypes.byref(a), 100) == 0  # not a multiple of 64
    assert b"multiple of 64" in lib.gdn_last_error()
    one = lib.gdn_chunk_fwd_host_buffer_size(ctypes.byref(a), 1024)
    four = lib.gdn_chunk_fwd_host_buffer_size(ctypes.byref(a), 256)
    assert one > four > 0  # slots hold one piece each
    cu = np.array([0, 10, 5, 1000], dtype=np.int64)  # cu_seqlens live on the host here
    b = _chunk_args(T=1000, H=2, HV=4, N=3)
    b.cu_seqlens = ctypes.c_void_p(cu.ctypes.data)
    assert lib.gdn_chunk_fwd_host_buffer_size(ctypes.byref(b), 256) == 0
    assert b"decrease" in lib.gdn_last_error()
    cu[2] = 500
    assert lib.gdn_chunk_fwd_host_buffer_size(ctypes.byref(b), 256) > 0
    assert lib.gdn_chunk_fwd_host(ctypes.byref(a), 1024, None) == _lib.GDN_ERR_INVALID  # null pointers


def test_conv_validation_returns_codes_without_touching_the_gpu():
    lib = _lib.load()
    a = _lib.Conv1dArgs(B=1, T=8, N=1, D=16, W=4)
    assert lib.gdn_causal_conv1d_fwd(ctypes.byref(a), None) == _lib.GDN_ERR_INVALID  # null pointers
    for name in ("x", "weight", "y"):
        setattr(a, name, ctypes.c_void_p(256))
    a.W = 17
    assert lib.gdn_causal_conv1d_fwd(ctypes.byref(a), None) == _lib.GDN_ERR_UNSUPPORTED
    a.W, a.B = 4, 2
    a.cu_seqlens = ctypes.c_void_p(256)
    a.cu_dtype = _lib.GDN_I64
    assert lib.gdn_causal_conv1d_fwd(ctypes.byref(a), None) == _lib.GDN_ERR_INVALID
    assert b"B == 1" in lib.gdn_last_error()
    f = _lib.Conv1dFnArgs(batch=2, dim=16, total_tokens=8, W=5)
    for name in ("x", "out", "weight", "conv_states", "query_start_loc"):
        setattr(f, name, ctypes.c_void_p(256))
    f.stride_x_token = f.stride_o_token = 16
    assert lib.gdn_causal_conv1d_fn(ctypes.byref(f), None) == _lib.GDN_ERR_UNSUPPORTED
    f.W, f.stride_x_token = 4, 8  # token stride below dim
    f.qsl_dtype = f.idx_dtype = _lib.GDN_I32
    assert lib.gdn_causal_conv1d_fn(ctypes.byref(f), None) == _lib.GDN_ERR_INVALID
    u = _lib.Conv1dUpdateArgs(N=2, D=16, W=4, stride_x_n=16, activation=3)
    u.x = u.y = ctypes.c_void_p(256)
    assert lib.gdn_causal_conv1d_update(ctypes.byref(u), None) == _lib.GDN_ERR_INVALID
    assert b"activation" in lib.gdn_last_error()


def test_python_errors_are_value_errors():
    with pytest.raises(ValueError):
        _lib.check(_lib.GDN_ERR_INVALID)
    with pytest.raises(_lib.GdnError):
        _lib.check(_lib.GDN_ERR_CUDA)
