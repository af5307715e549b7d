"""ctypes binding of libflagattn_b200.so (the C ABI in include/flagattn_b200.h).

The library must have been built in-tree (``flagattention_b200.build``); there
is no fallback: if it is missing or fails to load, every operator raises.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# FA_LIB_PATH selects another build of the same library; by default the
# in-tree build is loaded.
LIB_PATH = os.environ.get("FA_LIB_PATH") or os.path.join(_HERE, "libflagattn_b200.so")

FA_OK = 0
FA_ERR_INVALID_ARGUMENT = -1
FA_ERR_UNSUPPORTED = -2
FA_ERR_CUDA = -3
FA_ERR_NO_DEVICE = -4

FA_DTYPE_BF16, FA_DTYPE_F16, FA_DTYPE_F32 = 0, 1, 2
FA_MLA_META_INTS = 8
FA_EXCHANGE_MAX_RANKS = 8
FA_IPC_HANDLE_BYTES = 64
FA_DEVICE_TIMEOUT_EXCHANGE = 4

_i32, _i64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class InvalidArgument(AssertionError, ValueError):
    """Rejected shape / stride / alignment (the reference raises AssertionError)."""


class Unsupported(NotImplementedError):
    """A valid request this build does not implement."""


class CudaError(RuntimeError):
    """A CUDA call inside the library failed."""


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("q_stride_b", _i64), ("q_stride_h", _i64), ("q_stride_m", _i64),
        ("k", _vp), ("v", _vp),
        ("k_stride_seq", _i64), ("k_stride_tok", _i64), ("k_stride_head", _i64),
        ("block_table", _vp), ("bt_stride", _i64), ("page_size", _i32),
        ("seq_lens", _vp), ("n_ctx", _i32),
        ("batch", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("m_q", _i32),
        ("d_qk", _i32), ("d_v", _i32), ("causal", _i32), ("dtype", _i32), ("scale", _f32),
        ("num_splits", _i32), ("partition_size", _i32),
        ("o", _vp), ("o_stride_b", _i64), ("o_stride_h", _i64), ("o_stride_m", _i64),
        ("lse", _vp), ("part_o", _vp), ("part_lse", _vp),
        ("num_pages", _i32), ("sched", _vp), ("status", _vp),
    ]


class MlaArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("q_stride_b", _i64), ("q_stride_s", _i64), ("q_stride_h", _i64),
        ("kcache", _vp), ("kv_stride_page", _i64), ("kv_stride_tok", _i64),
        ("num_pages", _i32), ("page_size", _i32),
        ("block_table", _vp), ("bt_stride", _i64),
        ("seq_lens", _vp), ("n_ctx", _i32),
        ("indices", _vp), ("idx_stride_b", _i64), ("idx_stride_s", _i64), ("topk", _i32),
        ("tile_meta", _vp), ("num_splits", _vp), ("num_sm_parts", _i32),
        ("out", _vp), ("o_stride_b", _i64), ("o_stride_s", _i64), ("o_stride_h", _i64),
        ("lse", _vp), ("part_o", _vp), ("part_lse", _vp),
        ("batch", _i32), ("s_q", _i32), ("h_q", _i32), ("d_qk", _i32), ("d_v", _i32),
        ("causal", _i32), ("dtype", _i32), ("out_dtype", _i32), ("scale", _f32),
        ("status", _vp),
    ]


# (name, restype, argtypes) of every exported entry point
SIGNATURES = [
    ("fa_version", _i32, []),
    ("fa_status_string", ctypes.c_char_p, [_i32]),
    ("fa_last_error", ctypes.c_char_p, []),
    ("fa_device_sm_count", _i32, [_i32, ctypes.POINTER(_i32)]),
    ("fa_paged_num_splits", _i32, [_i32, _i32, _i32, _i32, _i32, _i32,
                                   ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    ("fa_split_kv_num_splits", _i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                      ctypes.POINTER(_i32)]),
    ("fa_decode_uses_tensor_cores", _i32, [ctypes.POINTER(DecodeArgs)]),
    ("fa_decode_workspace_size", _i32, [ctypes.POINTER(DecodeArgs),
                                        ctypes.POINTER(ctypes.c_size_t),
                                        ctypes.POINTER(ctypes.c_size_t),
                                        ctypes.POINTER(ctypes.c_size_t)]),
    ("fa_paged_attention", _i32, [ctypes.POINTER(DecodeArgs), _vp]),
    ("fa_split_kv_attention", _i32, [ctypes.POINTER(DecodeArgs), _vp]),
    ("fa_lse_combine", _i32, [_vp, _vp, _i32, _i64, _i32, _vp, _i32, _vp, _vp]),
    ("fa_lse_combine_strided", _i32, [_vp, _i64, _vp, _i64, _i32, _i64, _i32, _vp, _i32, _vp,
                                      _vp]),
    ("fa_mla_num_sm_parts", _i32, [_i32, _i32, _i32, _i32, ctypes.POINTER(_i32)]),
    ("fa_mla_workspace_size", _i32, [_i32, _i32, _i32, _i32, _i32,
                                     ctypes.POINTER(ctypes.c_size_t),
                                     ctypes.POINTER(ctypes.c_size_t)]),
    ("fa_mla_get_metadata", _i32, [_vp, _i32, _i32, _i32, _vp, _vp, _vp]),
    ("fa_mla_decode", _i32, [ctypes.POINTER(MlaArgs), _vp]),
    ("fa_mla_decode_partial", _i32, [ctypes.POINTER(MlaArgs), _vp]),
    ("fa_mla_combine", _i32, [ctypes.POINTER(MlaArgs), _vp]),
    ("fa_mla_decode_static_workspace", _i32, [ctypes.POINTER(MlaArgs), _vp]),
    ("fa_mla_append_rows", _i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i32, _i32, _i32,
                                  _vp]),
    ("fa_selftest_wait_timeout", _i32, [_vp, _vp]),
    ("fa_ipc_export", _i32, [_vp, _vp, ctypes.POINTER(ctypes.c_uint64)]),
    ("fa_ipc_open", _i32, [_vp, ctypes.POINTER(_vp)]),
    ("fa_ipc_close", _i32, [_vp]),
    ("fa_mla_combine_push", _i32, [ctypes.POINTER(MlaArgs), _vp, _vp, _i32, _i32, _vp]),
    ("fa_lse_merge_wait", _i32, [_vp, _i32, _i64, _i32, _vp, ctypes.c_uint64, _vp, _i32, _vp,
                                 _vp, _i64, _vp]),
    ("fa_mla_combine_exchange", _i32, [ctypes.POINTER(MlaArgs), _vp, _vp, _i32, _i32,
                                       ctypes.c_uint64, _vp, _i32, _vp, _vp, _i64, _vp]),
]

_lib = None


def lib():
    """Load (once) and return the shared library; raises if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m flagattention_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status, what):
    if status == FA_OK:
        return
    msg = f"{what}: {lib().fa_status_string(status).decode()}: {lib().fa_last_error().decode()}"
    if status == FA_ERR_INVALID_ARGUMENT:
        raise InvalidArgument(msg)
    if status == FA_ERR_UNSUPPORTED:
        raise Unsupported(msg)
    raise CudaError(msg)
