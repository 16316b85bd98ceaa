"""Argument checks of the newer entry points, on the host (no GPU needed):
each refuses a bad call with its error code and message before any device
work — the SM cap, the batched 2-D copy and the QKV projection that writes
into the owning ranks' caches."""
import ctypes

import pytest


def _lib():
    from neurodsl_b200 import _lib
    return _lib, _lib.load()


def test_sm_limit_refuses_negative_and_reports_previous():
    m, lib = _lib()
    prev = ctypes.c_int(-7)
    assert lib.nd_set_sm_limit(-1, ctypes.byref(prev)) == m.ND_ERR_INVALID_ARG
    assert lib.nd_set_sm_limit(100, ctypes.byref(prev)) == m.ND_OK
    assert lib.nd_set_sm_limit(0, ctypes.byref(prev)) == m.ND_OK and prev.value == 100


def test_copy_2d_batched_checks():
    m, lib = _lib()
    p = ctypes.c_void_p(0x1000)
    # more views than a launch takes
    assert lib.nd_copy_2d_batched(None, p, 8, 8, p, 8, 8, 70000, 1, 8, 4) == m.ND_ERR_SHAPE
    # element size
    assert lib.nd_copy_2d_batched(None, p, 8, 8, p, 8, 8, 2, 1, 8, 8) == m.ND_ERR_UNSUPPORTED
    # row stride below the row length
    assert lib.nd_copy_2d_batched(None, p, 4, 8, p, 8, 8, 2, 1, 8, 4) == m.ND_ERR_SHAPE
    # nothing to copy is fine, without a device
    assert lib.nd_copy_2d_batched(None, None, 8, 8, None, 8, 8, 0, 1, 8, 4) == m.ND_OK


def test_qkv_cache_peers_checks():
    m, lib = _lib()
    p = ctypes.c_void_p(0x1000)
    caches = (ctypes.c_void_p * 2)(ctypes.c_void_p(0x100000), ctypes.c_void_p(0x200000))
    # 32 rows or fewer: the cache-writing epilogue needs more
    rc = lib.nd_gemm_qkv_cache_peers(None, p, p, None, p, 32, 64, caches, caches, 2, 1, 0, 32,
                                     1, 40, 0)
    assert rc == m.ND_ERR_UNSUPPORTED
    # M != B * S
    rc = lib.nd_gemm_qkv_cache_peers(None, p, p, None, p, 40, 64, caches, caches, 2, 1, 0, 41,
                                     1, 64, 0)
    assert rc == m.ND_ERR_SHAPE
    # positions beyond the cache
    rc = lib.nd_gemm_qkv_cache_peers(None, p, p, None, p, 40, 64, caches, caches, 2, 1, 0, 40,
                                     1, 39, 0)
    assert rc == m.ND_ERR_SHAPE
    # more ranks than the epilogue addresses
    many = (ctypes.c_void_p * 9)(*[ctypes.c_void_p(0x100000 * (i + 1)) for i in range(9)])
    rc = lib.nd_gemm_qkv_cache_peers(None, p, p, None, p, 40, 64, many, many, 9, 1, 0, 40,
                                     1, 64, 0)
    assert rc == m.ND_ERR_INVALID_ARG
