"""ctypes binding of libstrata_cuda.so (include/strata_cuda.h).

Loading fails loudly when the library is missing: there is no CPU fallback for any entry.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = pathlib.Path(os.environ.get("STRATA_CUDA_LIB", PKG / "libstrata_cuda.so"))

OK, ERR_RANGE, ERR_LAYOUT, ERR_UNKNOWN, ERR_HANDLE, ERR_ALLOC, ERR_CUDA, ERR_DEVICE = range(8)
F32, I32, U32 = 0, 1, 2
ARG_BUF, ARG_I32, ARG_F32 = 0, 1, 2
MOE_EXACT, MOE_FAST = 0, 1

# Every symbol the header declares, with its ctypes signature.
_vp, _i, _u64, _sz, _d = C.c_void_p, C.c_int, C.c_uint64, C.c_size_t, C.c_double


class StrataArg(C.Structure):
    _fields_ = [("name", C.c_char_p), ("kind", C.c_int32), ("i32", C.c_int32), ("f32", C.c_float), ("buf", C.c_uint64)]


class StrataMoeLayer(C.Structure):
    _fields_ = [("width", C.c_int32), ("ff", C.c_int32), ("experts", C.c_int32), ("top_k", C.c_int32),
                ("router", C.c_uint64), ("router_bias", C.c_uint64), ("experts_blob", C.c_uint64),
                ("shared_blob", C.c_uint64), ("shared_gate", C.c_uint64)]


class StrataMoeLayerDev(C.Structure):
    _fields_ = [("width", C.c_int32), ("ff", C.c_int32), ("experts", C.c_int32), ("top_k", C.c_int32),
                ("router", C.c_void_p), ("router_bias", C.c_void_p), ("experts_blob", C.c_void_p),
                ("shared_blob", C.c_void_p), ("shared_gate", C.c_void_p)]


SIGNATURES = {
    "strata_create": ([_i, C.POINTER(_vp)], _i),
    "strata_destroy": ([_vp], _i),
    "strata_last_error": ([_vp, C.c_char_p, _sz], _i),
    "strata_stream": ([_vp, C.POINTER(_vp)], _i),
    "strata_alloc": ([_vp, _u64, _i, _i, C.POINTER(_u64)], _i),
    "strata_free": ([_vp, _u64], _i),
    "strata_write": ([_vp, _u64, _vp, _u64, _u64], _i),
    "strata_read": ([_vp, _u64, _vp, _u64, _u64], _i),
    "strata_copy": ([_vp, _u64, _u64, _u64, _u64, _u64], _i),
    "strata_zero": ([_vp, _u64], _i),
    "strata_buffer_info": ([_vp, _u64, C.POINTER(_u64), C.POINTER(_i), C.POINTER(_vp)], _i),
    "strata_run": ([_vp, C.c_char_p, C.POINTER(StrataArg), _i, C.POINTER(C.c_uint32)], _i),
    "strata_idle": ([_vp], _i),
    "strata_flush": ([_vp], _i),
    "strata_info": ([_vp, C.c_char_p, _sz], _i),
    "strata_profile": ([_vp, C.c_int32], _i),
    "strata_ple_gather_decode": ([_vp, _u64, _u64, C.c_int32, C.c_int32, _u64], _i),
    "strata_capture_begin": ([_vp], _i),
    "strata_capture_end": ([_vp, C.POINTER(C.c_uint64)], _i),
    "strata_graph_launch": ([_vp, _u64], _i),
    "strata_graph_free": ([_vp, _u64], _i),
    "strata_ep_unique_id": ([_vp, C.c_char_p, _sz], _i),
    "strata_ep_init": ([_vp, C.c_int32, C.c_int32, C.c_char_p], _i),
    "strata_ep_set_timeout": ([_vp, C.c_int32], _i),
    "strata_ep_set_placement": ([_vp, C.c_int32, C.POINTER(C.c_int32)], _i),
    "strata_ep_local_experts": ([_vp, C.c_int32, C.POINTER(C.c_int32)], _i),
    "strata_ep_loopback_create": ([_vp, C.c_int32, C.POINTER(_u64)], _i),
    "strata_ep_init_loopback": ([_vp, C.c_int32, _u64], _i),
    "strata_ep_loopback_release": ([_vp, _u64], _i),
    "strata_moe_ep_forward": ([_vp, C.POINTER(StrataMoeLayer), _u64, C.c_int32, _u64, _u64, _u64], _i),
    "strata_profile_read": ([_vp, C.POINTER(C.c_double), C.c_int32, C.POINTER(C.c_uint64)], _i),
    "strata_moe_forward": ([_vp, C.POINTER(StrataMoeLayer), _u64, C.c_int32, _u64, _u64, _u64, C.c_int32], _i),
    "strata_validate_experts": ([_vp, _u64, C.c_int32, C.c_int32, C.c_int32], _i),
    "strata_moe_forward_noalloc": ([C.POINTER(StrataMoeLayerDev), _vp, C.c_int32, _vp, _vp, _vp, _vp, C.c_char_p, _sz], _i),
    "strata_synth_blobs": ([_vp, _u64, _u64, _u64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32], _i),
    "strata_synth_normals": ([_vp, _u64, _u64, _u64, _u64, _u64, _u64, _u64, _d], _i),
}

_lib = None


def load() -> C.CDLL:
    """Load the in-tree library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `python -m stratacuda_b200.build` "
                                    "(there is no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib
