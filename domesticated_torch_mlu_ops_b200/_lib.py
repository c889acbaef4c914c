"""ctypes binding of ``libgdn_b200.so`` (C ABI: ``include/gdn_b200.h``).

The struct layouts below mirror the header field by field.  Loading fails
loudly when the library is missing: there is no CPU or Python fallback.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgdn_b200.so")

GDN_OK = 0
GDN_ERR_INVALID = -1
GDN_ERR_UNSUPPORTED = -2
GDN_ERR_CUDA = -3
GDN_ERR_WORKSPACE = -4
GDN_ERR_DEVICE = -5

GDN_F32, GDN_BF16, GDN_F16, GDN_I32, GDN_I64 = 0, 1, 2, 3, 4
GDN_ACT_NONE, GDN_ACT_SILU = 0, 1

EXPORTED = (
    "gdn_chunk_workspace_size",
    "gdn_chunk_fwd",
    "gdn_chunk_fwd_noalloc",
    "gdn_chunk_noalloc_check_device_error",
    "gdn_chunk_check_device_error",
    "gdn_chunk_fwd_test_stall",
    "gdn_chunk_bwd_workspace_size",
    "gdn_chunk_bwd",
    "gdn_chunk_fwd_host_buffer_size",
    "gdn_chunk_fwd_host",
    "gdn_chunk_fwd_h",
    "gdn_fused_recurrent_fwd",
    "gdn_recurrent_plain_fwd",
    "gdn_solve_tril",
    "gdn_causal_conv1d_fwd",
    "gdn_causal_conv1d_fn",
    "gdn_causal_conv1d_update",
    "gdn_conv_chunk_workspace_size",
    "gdn_conv_chunk_fwd",
    "gdn_last_error",
    "gdn_abi_version",
    "gdn_kernel_launch_count",
)

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


class ChunkArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("beta", _vp),
        ("initial_state", _vp), ("o", _vp), ("final_state", _vp), ("cu_seqlens", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("B", _i64), ("T", _i64), ("N", _i64),
        ("H", _i32), ("HV", _i32), ("K", _i32), ("V", _i32),
        ("qkv_dtype", _i32), ("cu_dtype", _i32),
        ("scale", ctypes.c_float),
        ("use_qk_l2norm", _i32), ("state_v_first", _i32), ("force_generic", _i32),
        ("stage_events", ctypes.POINTER(_vp)), ("n_stage_events", _i32),
        ("q_token_stride", _i64), ("k_token_stride", _i64), ("v_token_stride", _i64),
    ]


class ChunkBwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("beta", _vp),
        ("initial_state", _vp), ("cu_seqlens", _vp), ("dout", _vp), ("dht", _vp),
        ("dq", _vp), ("dk", _vp), ("dv", _vp), ("dg", _vp), ("dbeta", _vp), ("dh0", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("B", _i64), ("T", _i64), ("N", _i64),
        ("H", _i32), ("HV", _i32), ("K", _i32), ("V", _i32),
        ("qkv_dtype", _i32), ("cu_dtype", _i32),
        ("scale", ctypes.c_float),
        ("use_qk_l2norm", _i32), ("state_v_first", _i32),
    ]


class ChunkHArgs(ctypes.Structure):
    _fields_ = [
        ("k", _vp), ("w", _vp), ("u", _vp), ("g", _vp), ("gk", _vp), ("initial_state", _vp),
        ("h", _vp), ("v_new", _vp), ("final_state", _vp), ("cu_seqlens", _vp),
        ("B", _i64), ("T", _i64), ("N", _i64),
        ("Hg", _i32), ("H", _i32), ("K", _i32), ("V", _i32),
        ("dtype", _i32), ("cu_dtype", _i32), ("state_v_first", _i32),
    ]


class RecurrentArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("beta", _vp),
        ("initial_state", _vp), ("o", _vp), ("final_state", _vp), ("cu_seqlens", _vp),
        ("ssm_state_indices", _vp), ("num_accepted_tokens", _vp),
        ("B", _i64), ("T", _i64), ("N", _i64),
        ("H", _i32), ("HV", _i32), ("K", _i32), ("V", _i32),
        ("qkv_dtype", _i32), ("cu_dtype", _i32), ("idx_dtype", _i32), ("nacc_dtype", _i32),
        ("stride_init_state_token", _i64), ("stride_final_state_token", _i64),
        ("stride_indices_seq", _i64), ("stride_indices_tok", _i64),
        ("scale", ctypes.c_float),
        ("use_qk_l2norm", _i32), ("beta_per_v", _i32), ("inplace_final_state", _i32),
        ("num_slots", _i64), ("err", _vp), ("gk", _vp),
    ]


class RecurrentPlainArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("gk", _vp), ("gv", _vp), ("beta", _vp),
        ("initial_state", _vp), ("o", _vp), ("final_state", _vp), ("cu_seqlens", _vp),
        ("B", _i64), ("T", _i64), ("N", _i64),
        ("H", _i32), ("HV", _i32), ("K", _i32), ("V", _i32),
        ("qkv_dtype", _i32), ("cu_dtype", _i32),
        ("scale", ctypes.c_float),
        ("use_qk_l2norm", _i32), ("beta_per_v", _i32),
    ]


class Conv1dArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("weight", _vp), ("bias", _vp), ("residual", _vp), ("initial_state", _vp),
        ("y", _vp), ("cu_seqlens", _vp),
        ("B", _i64), ("T", _i64), ("N", _i64), ("D", _i64),
        ("W", _i32), ("x_dtype", _i32), ("w_dtype", _i32), ("state_dtype", _i32), ("cu_dtype", _i32),
        ("activation", _i32),
    ]


class Conv1dFnArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("out", _vp), ("weight", _vp), ("bias", _vp), ("conv_states", _vp),
        ("query_start_loc", _vp), ("cache_indices", _vp), ("has_initial_state", _vp),
        ("stride_x_token", _i64), ("stride_o_token", _i64),
        ("stride_state_seq", _i64), ("stride_state_tok", _i64), ("num_cache_lines", _i64),
        ("batch", _i64), ("dim", _i64), ("total_tokens", _i64),
        ("pad_slot_id", _i64), ("null_block_id", _i64),
        ("has_null_block", _i32), ("W", _i32),
        ("x_dtype", _i32), ("w_dtype", _i32), ("state_dtype", _i32), ("qsl_dtype", _i32), ("idx_dtype", _i32),
        ("activation", _i32),
        ("block_idx_first", _vp), ("block_idx_last", _vp), ("initial_state_idx", _vp),
        ("num_computed_tokens", _vp), ("stride_cache_indices", _i64), ("block_size_to_align", _i64),
        ("apc_dtype", _i32),
    ]


class Conv1dUpdateArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("cache", _vp), ("residual", _vp), ("weight", _vp), ("bias", _vp), ("y", _vp),
        ("stride_x_n", _i64), ("N", _i64), ("D", _i64),
        ("W", _i32), ("x_dtype", _i32), ("cache_dtype", _i32), ("w_dtype", _i32), ("activation", _i32),
    ]


_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python -m domesticated_torch_mlu_ops_b200.build` "
            "(the GDN ops have no CPU fallback)")
    lib = ctypes.CDLL(path)
    lib.gdn_chunk_workspace_size.argtypes = [ctypes.POINTER(ChunkArgs)]
    lib.gdn_chunk_workspace_size.restype = ctypes.c_size_t
    lib.gdn_chunk_fwd.argtypes = [ctypes.POINTER(ChunkArgs), _vp]
    lib.gdn_chunk_fwd.restype = ctypes.c_int
    lib.gdn_chunk_fwd_noalloc.argtypes = [ctypes.POINTER(ChunkArgs), _vp]
    lib.gdn_chunk_fwd_noalloc.restype = ctypes.c_int
    lib.gdn_chunk_noalloc_check_device_error.argtypes = [_vp]
    lib.gdn_chunk_noalloc_check_device_error.restype = ctypes.c_int
    lib.gdn_chunk_fwd_test_stall.argtypes = [ctypes.POINTER(ChunkArgs), _i64, _i64, _vp]
    lib.gdn_chunk_fwd_test_stall.restype = ctypes.c_int
    lib.gdn_chunk_check_device_error.argtypes = [_vp, _vp]
    lib.gdn_chunk_check_device_error.restype = ctypes.c_int
    lib.gdn_chunk_bwd_workspace_size.argtypes = [ctypes.POINTER(ChunkBwdArgs)]
    lib.gdn_chunk_bwd_workspace_size.restype = ctypes.c_size_t
    lib.gdn_chunk_bwd.argtypes = [ctypes.POINTER(ChunkBwdArgs), _vp]
    lib.gdn_chunk_bwd.restype = ctypes.c_int
    lib.gdn_chunk_fwd_host_buffer_size.argtypes = [ctypes.POINTER(ChunkArgs), _i64]
    lib.gdn_chunk_fwd_host_buffer_size.restype = ctypes.c_size_t
    lib.gdn_chunk_fwd_host.argtypes = [ctypes.POINTER(ChunkArgs), _i64, _vp]
    lib.gdn_chunk_fwd_host.restype = ctypes.c_int
    lib.gdn_chunk_fwd_h.argtypes = [ctypes.POINTER(ChunkHArgs), _vp]
    lib.gdn_chunk_fwd_h.restype = ctypes.c_int
    lib.gdn_fused_recurrent_fwd.argtypes = [ctypes.POINTER(RecurrentArgs), _vp]
    lib.gdn_fused_recurrent_fwd.restype = ctypes.c_int
    lib.gdn_recurrent_plain_fwd.argtypes = [ctypes.POINTER(RecurrentPlainArgs), _vp]
    lib.gdn_recurrent_plain_fwd.restype = ctypes.c_int
    lib.gdn_solve_tril.argtypes = [_vp, _vp, _i32, _vp, _i32, _i64, _i64, _i64, _i32, _i32, _vp]
    lib.gdn_solve_tril.restype = ctypes.c_int
    lib.gdn_causal_conv1d_fwd.argtypes = [ctypes.POINTER(Conv1dArgs), _vp]
    lib.gdn_causal_conv1d_fwd.restype = ctypes.c_int
    lib.gdn_causal_conv1d_fn.argtypes = [ctypes.POINTER(Conv1dFnArgs), _vp]
    lib.gdn_causal_conv1d_fn.restype = ctypes.c_int
    lib.gdn_causal_conv1d_update.argtypes = [ctypes.POINTER(Conv1dUpdateArgs), _vp]
    lib.gdn_causal_conv1d_update.restype = ctypes.c_int
    lib.gdn_conv_chunk_workspace_size.argtypes = [ctypes.POINTER(ChunkArgs)]
    lib.gdn_conv_chunk_workspace_size.restype = ctypes.c_size_t
    lib.gdn_conv_chunk_fwd.argtypes = [ctypes.POINTER(ChunkArgs), ctypes.POINTER(Conv1dFnArgs), _vp]
    lib.gdn_conv_chunk_fwd.restype = ctypes.c_int
    lib.gdn_last_error.argtypes = []
    lib.gdn_last_error.restype = ctypes.c_char_p
    lib.gdn_abi_version.argtypes = []
    lib.gdn_abi_version.restype = ctypes.c_int
    lib.gdn_kernel_launch_count.argtypes = []
    lib.gdn_kernel_launch_count.restype = ctypes.c_uint64
    _lib = lib
    return lib


class GdnError(RuntimeError):
    """A libgdn_b200 call returned a negative status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libgdn_b200 error {code}: {msg}")
        self.code = code


def check(code: int) -> None:
    if code == GDN_OK:
        return
    msg = load().gdn_last_error().decode(errors="replace")
    if code in (GDN_ERR_INVALID, GDN_ERR_UNSUPPORTED, GDN_ERR_WORKSPACE):
        raise ValueError(f"libgdn_b200 error {code}: {msg}")
    raise GdnError(code, msg)
