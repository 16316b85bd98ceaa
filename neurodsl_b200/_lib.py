"""ctypes binding of libneurodsl_b200.so (the C ABI in include/neurodsl_b200.h).

The shared library is the only compute path: if it is missing or fails to
load, every operation raises; nothing falls back to another implementation.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libneurodsl_b200.so")

ND_OK = 0
ND_ERR_INVALID_ARG = 1
ND_ERR_SHAPE = 2
ND_ERR_ALIGNMENT = 3
ND_ERR_UNSUPPORTED = 4
ND_ERR_CUDA = 5
ND_ERR_DEVICE = 6
ND_ERR_WORKSPACE = 7
ND_ERR_TIMEOUT = 8

ND_F32 = 0
ND_BF16 = 1
ND_I32 = 2
ND_I64 = 3

ND_ACT_NONE = 0
ND_ACT_GELU_SIGMOID = 1
ND_ACT_GELU_TANH = 2
ND_ACT_GELU_ERF = 3

# Every symbol the header declares, with its ctypes signature.
_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_fp = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t
_i64p = ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    "nd_version": (_i, []),
    "nd_last_error_string": (ctypes.c_char_p, []),
    "nd_device_check": (_i, [_i]),
    "nd_device_error": (_i, [ctypes.POINTER(_i)]),
    "nd_flash_attn_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _f, _i]),
    "nd_flash_attn_fwd_strided": (_i, [_vp, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _i,
                                       _vp, _vp, _i, _i, _i, _i, _i, _f, _i]),
    "nd_kv_decode_workspace_size": (_i, [_i, _i, _i, _i, ctypes.POINTER(_sz)]),
    "nd_kv_decode_attn": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _f,
                               _vp, _sz]),
    "nd_kv_decode_attn_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i,
                                       _i, _i, _f]),
    "nd_kv_decode_attn_qkv": (_i, [_vp, _vp, ctypes.c_int64, _vp, _vp, _vp, _i, _vp, _i, _i, _i,
                                   _i, _i, _f, _vp, _sz]),
    "nd_set_pdl": (_i, [_i, ctypes.POINTER(_i)]),
    "nd_set_sm_limit": (_i, [_i, ctypes.POINTER(_i)]),
    "nd_kv_append": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i]),
    "nd_gemm_bias_act": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i]),
    "nd_gemm_qkv_cache": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _i]),
    "nd_gemm_qkv_cache_peers": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, ctypes.POINTER(_vp),
                                     ctypes.POINTER(_vp), _i, _i, _i, _i, _i, _i, _i]),
    "nd_ln_gemm": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i]),
    "nd_gelu": (_i, [_vp, _vp, _vp, ctypes.c_int64, _i]),
    "nd_scale_mask": (_i, [_vp, _vp, _vp, _i, _i, _i]),
    "nd_softmax": (_i, [_vp, _vp, _vp, _i, _i]),
    "nd_add": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i]),
    "nd_layernorm": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _f]),
    "nd_convert_2d": (_i, [_vp, _vp, _i, _i, _vp, _i, _i, _i]),
    "nd_convert_2d_padded": (_i, [_vp, _vp, _i, _i, _vp, _i, _i, _i, _i]),
    "nd_gather_rows": (_i, [_vp, _vp, _i, ctypes.c_longlong, _i, _vp, _i, _i, _i, _i, _vp,
                            ctypes.c_longlong]),
    "nd_copy_2d": (_i, [_vp, _vp, ctypes.c_longlong, _vp, ctypes.c_longlong, _i, _i, _i]),
    "nd_copy_2d_batched": (_i, [_vp, _vp, ctypes.c_longlong, ctypes.c_longlong, _vp,
                                ctypes.c_longlong, ctypes.c_longlong, _i, _i, _i, _i]),
    "nd_embed": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "nd_argmax": (_i, [_vp, _vp, _i, ctypes.c_int64, _i, _i, _vp, _vp]),
    "nd_kv_store": (_i, [_vp, _vp, ctypes.c_int64, _i, _i, _vp, _vp, _i, _i, _i, _i, _i, _i]),
    "nd_add_layernorm": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _f]),
    "nd_comm_region_bytes": (_i, [_i, _i, ctypes.POINTER(_sz)]),
    "nd_comm_slot_offset": (_i, [_i, _i, _i, ctypes.POINTER(_sz)]),
    "nd_comm_alloc": (_i, [_sz, ctypes.POINTER(_vp), _vp]),
    "nd_comm_open": (_i, [_vp, ctypes.POINTER(_vp)]),
    "nd_comm_close": (_i, [_vp]),
    "nd_comm_free": (_i, [_vp]),
    "nd_allreduce_add_layernorm": (_i, [_vp, ctypes.POINTER(_vp), _i, _i, _sz, _i, _i, _vp, _vp,
                                        _vp, _vp, _vp, _vp, _i, _i, _f]),
    "nd_gemm_allreduce_add_layernorm": (_i, [_vp, _vp, _vp, _i, ctypes.POINTER(_vp), _i, _i, _sz,
                                             _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _f]),
}


class NeuroDSLError(RuntimeError):
    """A non-zero status from the C ABI (the reference raises error("❌ ...") )."""

    def __init__(self, status: int, message: str):
        super().__init__(f"❌ [status {status}] {message}")
        self.status = status


_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """Load the library once; raise if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise ImportError(
                    f"{path} is missing: build it with `python -m neurodsl_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int):
    if status != ND_OK:
        msg = load().nd_last_error_string().decode("utf-8", "replace")
        raise NeuroDSLError(status, msg)
