"""ctypes binding of the C ABI declared in include/laprune_b200.h.

The library is built in-tree by ``python -m laprune_b200.build``.  There is no
fallback: if the library is missing or cannot be loaded, importing the CUDA
entry points raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblaprune_b200.so"

LP_OK, LP_ERR_INVALID, LP_ERR_CUDA, LP_ERR_UNSUPPORTED, LP_ERR_WORKSPACE = 0, 1, 2, 3, 4
LP_F32, LP_F16, LP_BF16, LP_F64, LP_U8, LP_I8, LP_I64, LP_I32 = range(8)
LP_SELECT_KV_GROUP, LP_SELECT_QUERY_HEAD = 0, 1
LP_DEVERR_WAIT_TIMEOUT, LP_DEVERR_TIE_OVERFLOW = 1, 2
LP_FLAG_NO_FUSED = 1
LP_FLAG_EXCHANGE_SELECT = 2
LP_FLAG_TEST_WAIT_TIMEOUT = 4

_c_i32, _c_i64, _c_p, _c_f = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float


class SparseDecodeArgs(ctypes.Structure):
    """Mirror of lp_sparse_decode_args."""
    _fields_ = [
        ("q", _c_p), ("q_dtype", _c_i32), ("_pad0", _c_i32),
        ("q_stride_b", _c_i64), ("q_stride_h", _c_i64),
        ("codebooks", _c_p), ("cb_per_kv_head", _c_i32), ("cb_dtype", _c_i32),
        ("codes", _c_p), ("codes_stride_b", _c_i64), ("codes_stride_h", _c_i64), ("codes_stride_t", _c_i64),
        ("keys", _c_p), ("vals", _c_p), ("kv_dtype", _c_i32), ("_pad2", _c_i32),
        ("k_stride_b", _c_i64), ("k_stride_h", _c_i64), ("k_stride_t", _c_i64),
        ("v_stride_b", _c_i64), ("v_stride_h", _c_i64), ("v_stride_t", _c_i64),
        ("B", _c_i32), ("Hkv", _c_i32), ("G", _c_i32), ("D", _c_i32), ("M", _c_i32), ("K", _c_i32),
        ("T_codes", _c_i32), ("T_total", _c_i32), ("sink", _c_i32), ("local", _c_i32),
        ("topk", _c_i32), ("select_mode", _c_i32),
        ("scale", _c_f), ("out_dtype", _c_i32),
        ("out", _c_p), ("out_stride_b", _c_i64), ("out_stride_h", _c_i64),
        ("head_scores", _c_p), ("topk_out", _c_p), ("stage_events", _c_p),
        ("flags", _c_i32), ("_pad3", _c_i32), ("phase_ns", _c_p),
        ("prefetch_ptr", _c_p * 2), ("prefetch_bytes", _c_i64 * 2),
        ("prefetch_count", _c_i64 * 2), ("prefetch_stride", _c_i64 * 2),
    ]


class EncodeArgs(ctypes.Structure):
    """Mirror of lp_encode_args."""
    _fields_ = [
        ("x", _c_p), ("x_dtype", _c_i32), ("cb_per_kv_head", _c_i32),
        ("x_stride_b", _c_i64), ("x_stride_h", _c_i64), ("x_stride_t", _c_i64),
        ("codebooks", _c_p), ("codes", _c_p),
        ("codes_stride_b", _c_i64), ("codes_stride_h", _c_i64), ("codes_stride_t", _c_i64),
        ("B", _c_i32), ("H", _c_i32), ("T", _c_i32), ("D", _c_i32), ("M", _c_i32), ("K", _c_i32),
        ("flags", _c_i32), ("icm_iters", _c_i32),
    ]


LP_ENCODE_FLAG_EXACT = 1


class LutGatherArgs(ctypes.Structure):
    """Mirror of lp_lut_gather_args."""
    _fields_ = [
        ("lut", _c_p), ("lut_dtype", _c_i32), ("code_mode", _c_i32),
        ("lut_stride_q", _c_i64),
        ("M_stride", _c_i32), ("K", _c_i32), ("m0", _c_i32), ("m1", _c_i32),
        ("codes", _c_p), ("codes_stride_h", _c_i64), ("codes_stride_t", _c_i64),
        ("Q", _c_i32), ("G", _c_i32), ("T", _c_i32), ("N", _c_i32),
        ("indices", _c_p), ("indices_stride_q", _c_i64),
        ("out", _c_p), ("out_dtype", _c_i32), ("_pad0", _c_i32),
        ("out_stride_q", _c_i64),
    ]


class LutBuildArgs(ctypes.Structure):
    """Mirror of lp_lut_build_args."""
    _fields_ = [
        ("q", _c_p), ("q_dtype", _c_i32), ("_pad0", _c_i32), ("q_stride", _c_i64),
        ("codebooks", _c_p), ("Q", _c_i32), ("M", _c_i32), ("K", _c_i32),
        ("D", _c_i32), ("lut", _c_p),
    ]


class GqaGatherArgs(ctypes.Structure):
    """Mirror of lp_gqa_gather_args."""
    _fields_ = [
        ("keys", _c_p), ("vals", _c_p), ("kv_dtype", _c_i32), ("_pad0", _c_i32),
        ("k_stride_b", _c_i64), ("k_stride_h", _c_i64), ("k_stride_t", _c_i64),
        ("v_stride_b", _c_i64), ("v_stride_h", _c_i64), ("v_stride_t", _c_i64),
        ("indices", _c_p), ("indices_stride_b", _c_i64), ("indices_stride_h", _c_i64),
        ("B", _c_i32), ("Hkv", _c_i32), ("G", _c_i32), ("T", _c_i32),
        ("D", _c_i32), ("N_explicit", _c_i32), ("tail_start", _c_i32),
        ("tail_count", _c_i32), ("out_k", _c_p), ("out_v", _c_p),
    ]

class RopeAppendArgs(ctypes.Structure):
    """Mirror of lp_rope_append_args."""
    _fields_ = [
        ("q", _c_p), ("k", _c_p), ("v", _c_p),
        ("q_stride_b", _c_i64), ("q_stride_h", _c_i64), ("k_stride_b", _c_i64), ("k_stride_h", _c_i64),
        ("v_stride_b", _c_i64), ("v_stride_h", _c_i64),
        ("cos", _c_p), ("sin", _c_p), ("cos_stride_b", _c_i64), ("sin_stride_b", _c_i64),
        ("q_out", _c_p), ("q_out_stride_b", _c_i64), ("q_out_stride_h", _c_i64),
        ("k_cache", _c_p), ("v_cache", _c_p),
        ("kc_stride_b", _c_i64), ("kc_stride_h", _c_i64), ("kc_stride_t", _c_i64),
        ("vc_stride_b", _c_i64), ("vc_stride_h", _c_i64), ("vc_stride_t", _c_i64),
        ("dtype", _c_i32), ("B", _c_i32), ("Hq", _c_i32), ("Hkv", _c_i32), ("D", _c_i32), ("pos", _c_i32),
    ]


# name -> (restype, argtypes) of every exported entry point
SIGNATURES = {
    "lp_last_error": (ctypes.c_char_p, []),
    "lp_version": (ctypes.c_int, []),
    "lp_sizeof_sparse_decode_args": (ctypes.c_size_t, []),
    "lp_sparse_decode_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(SparseDecodeArgs)]),
    "lp_sparse_decode": (ctypes.c_int, [ctypes.POINTER(SparseDecodeArgs), _c_p, ctypes.c_size_t, _c_p]),
    "lp_read_device_errors": (ctypes.c_int, [_c_p, ctypes.c_size_t, _c_p, ctypes.POINTER(ctypes.c_uint32)]),
    "lp_sparse_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(SparseDecodeArgs), _c_p,
                                                ctypes.POINTER(ctypes.c_uint32)]),
    "lp_sizeof_encode_args": (ctypes.c_size_t, []),
    "lp_encode_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(EncodeArgs)]),
    "lp_encode_keys": (ctypes.c_int, [ctypes.POINTER(EncodeArgs), _c_p, ctypes.c_size_t, _c_p]),
    "lp_encode_rows_per_cta": (ctypes.c_int, [ctypes.POINTER(EncodeArgs)]),
    "lp_lut_gather": (ctypes.c_int, [ctypes.POINTER(LutGatherArgs), _c_p]),
    "lp_lut_build": (ctypes.c_int, [ctypes.POINTER(LutBuildArgs), _c_p]),
    "lp_gqa_gather_kv": (ctypes.c_int, [ctypes.POINTER(GqaGatherArgs), _c_p]),
    "lp_sizeof_rope_append_args": (ctypes.c_size_t, []),
    "lp_rope_append": (ctypes.c_int, [ctypes.POINTER(RopeAppendArgs), _c_p]),
}
LP_NOALLOC_SCRATCH_BYTES = 32 << 20

_lib = None


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the CUDA library (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise ImportError(
                f"laprune_b200 CUDA library not found at {_LIB_PATH}; "
                "build it with `python -m laprune_b200.build`")
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.lp_sizeof_sparse_decode_args() != ctypes.sizeof(SparseDecodeArgs):
            raise ImportError("lp_sparse_decode_args layout mismatch between the binding and the library")
        if lib.lp_sizeof_encode_args() != ctypes.sizeof(EncodeArgs):
            raise ImportError("lp_encode_args layout mismatch between the binding and the library")
        if lib.lp_sizeof_rope_append_args() != ctypes.sizeof(RopeAppendArgs):
            raise ImportError("lp_rope_append_args layout mismatch between the binding and the library")
        _lib = lib
    return _lib


def check(status: int) -> None:
    if status != LP_OK:
        msg = load().lp_last_error()
        raise RuntimeError(msg.decode() if msg else f"laprune_b200 error {status}")
