"""Host-side checks of the tensor-parallel exchange's shape rules, without a GPU:
the Python predicate that chooses the fused projection + exchange
(neurodsl_b200.comm.PeerReduce.fused_supported) agrees with the library's own
check in nd_gemm_allreduce_add_layernorm, which refuses unsupported shapes
with ND_ERR_UNSUPPORTED before touching any device (supported shapes get as
far as the device check instead)."""
import ctypes
import itertools
import types

import pytest


def _supported_by_library(lib, _lib, tp, rows, d, K, rows_max=32):
    fake = [ctypes.c_void_p(0x100000 * (r + 1)) for r in range(tp)]
    regions = (ctypes.c_void_p * tp)(*fake)
    nbytes = 1 << 40   # large enough for any shape here
    rc = lib.nd_gemm_allreduce_add_layernorm(None, ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000),
                                             K, regions, tp, 0, nbytes, rows_max, 0,
                                             ctypes.c_void_p(0x3000), None, None, None,
                                             ctypes.c_void_p(0x4000), ctypes.c_void_p(0x5000),
                                             rows, d, 1e-5)
    assert rc != _lib.ND_OK, "no launch can succeed on a host without a GPU"
    return rc != _lib.ND_ERR_UNSUPPORTED


def test_fused_projection_shape_rule_matches_the_library():
    from neurodsl_b200 import _lib
    from neurodsl_b200.comm import PeerReduce
    lib = _lib.load()
    for tp, rows, d, K in itertools.product((1, 2, 3, 4, 8), (1, 16, 32), (8, 100, 768, 1024, 1032),
                                            (32, 48, 1024)):
        fake = types.SimpleNamespace(tp=tp, rows_max=32, d=d)
        want = PeerReduce.fused_supported(fake, rows, K)
        assert _supported_by_library(lib, _lib, tp, rows, d, K) == want, (tp, rows, d, K)


def test_fused_projection_refuses_rows_beyond_the_slots():
    from neurodsl_b200 import _lib
    lib = _lib.load()
    regions = (ctypes.c_void_p * 2)(ctypes.c_void_p(0x100000), ctypes.c_void_p(0x200000))
    rc = lib.nd_gemm_allreduce_add_layernorm(None, None, None, 64, regions, 2, 0, 1 << 30, 8, 0,
                                             None, None, None, None, None, None, 9, 256, 1e-5)
    assert rc == _lib.ND_ERR_SHAPE
    assert b"rows_max" in lib.nd_last_error_string()
