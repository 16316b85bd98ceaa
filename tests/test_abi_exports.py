"""CPU checks of the C ABI library: it loads without a GPU and exports every
function that include/neurodsl_b200.h declares (no compute call is made)."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "neurodsl_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\**\s*(nd_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("nd_flash_attn_fwd", "nd_kv_decode_attn", "nd_gemm_bias_act",
                     "nd_layernorm", "nd_last_error_string"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol():
    from neurodsl_b200 import _lib
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\bT (nd_\w+)", out))
    assert set(declared_functions()) <= exported
    # no stray exports beyond the header
    assert exported <= set(declared_functions()), exported - set(declared_functions())


def test_version_and_error_string_without_gpu():
    from neurodsl_b200 import _lib
    lib = _lib.load()
    assert lib.nd_version() >= 100
    assert isinstance(lib.nd_last_error_string(), bytes)


def test_argument_validation_runs_before_any_device_work():
    """Shape/dtype errors are reported on the host, even with no GPU present."""
    from neurodsl_b200 import _lib
    lib = _lib.load()
    rc = lib.nd_flash_attn_fwd(None, None, None, None, None, 0, None, None, 1, 1, 16, 16, 32,
                               0.125, 1)
    assert rc == _lib.ND_ERR_UNSUPPORTED
    assert b"head_dim" in lib.nd_last_error_string()
    rc = lib.nd_flash_attn_fwd(None, None, None, None, None, 0, None, None, 1, 1, 16, 20, 64,
                               0.125, 1)
    assert rc == _lib.ND_ERR_SHAPE
    rc = lib.nd_kv_decode_attn(None, None, None, None, None, None, None, 0, None, 1, 1, 9, 8, 64,
                               0.125, None, 0)
    assert rc == _lib.ND_ERR_SHAPE
    rc = lib.nd_gemm_bias_act(None, None, None, None, None, 0, None, 0, 4, 8, 12, 0)
    assert rc == _lib.ND_ERR_SHAPE
    rc = lib.nd_layernorm(None, None, 0, None, None, None, 0, None, None, 4, 0, 1e-5)
    assert rc == _lib.ND_ERR_SHAPE
    n = ctypes.c_size_t(0)
    assert lib.nd_kv_decode_workspace_size(64, 12, 1152, 64, ctypes.byref(n)) == 0
    assert n.value > 64 * 12 * 9 * 256


def test_pdl_switch_is_per_call_state_without_a_gpu():
    """nd_set_pdl only records the launch mode (no device work): it returns
    the previous setting, and the fused-QKV decode entry point checks its row
    stride before touching the device."""
    from neurodsl_b200 import _lib, ops
    assert ops.set_pdl(True) is False
    assert ops.set_pdl(False) is True
    with ops.pdl(True):
        assert ops.set_pdl(True) is True
    assert ops.set_pdl(False) is False
    lib = _lib.load()
    rc = lib.nd_kv_decode_attn_qkv(None, 16, 3 * 2 * 64 - 8, None, None, None, 1, None, 2, 2, 4,
                                   16, 64, 0.125, None, 0)
    assert rc == _lib.ND_ERR_SHAPE
    assert b"row stride" in lib.nd_last_error_string()
    # the unfused graph ops refuse bad arguments before touching the device
    assert lib.nd_gelu(None, None, None, 16, 0) == _lib.ND_ERR_UNSUPPORTED      # not a GELU form
    assert lib.nd_gelu(None, None, None, -1, 1) == _lib.ND_ERR_INVALID_ARG
    assert lib.nd_scale_mask(None, None, None, 4, 4, 0) == _lib.ND_ERR_INVALID_ARG  # d_head 0
    assert lib.nd_softmax(None, None, None, -2, 4) == _lib.ND_ERR_INVALID_ARG
    assert lib.nd_gelu(None, None, None, 0, 1) == _lib.ND_OK                     # empty
    # nd_ln_gemm: K must be a multiple of 32 up to 1024, at most 32 rows
    for M, K in ((4, 80), (4, 2048), (33, 64)):
        rc = lib.nd_ln_gemm(None, None, None, None, None, None, 1e-5, None, None, None, None, 1,
                            M, 8, K, 0)
        assert rc == _lib.ND_ERR_SHAPE, (M, K)


def test_missing_library_raises(tmp_path):
    from neurodsl_b200 import _lib
    with pytest.raises(ImportError):
        old = _lib._lib
        _lib._lib = None
        try:
            _lib.load(str(tmp_path / "nope.so"))
        finally:
            _lib._lib = old


def test_empty_inputs_are_accepted_without_a_device():
    """Zero-size shapes (an empty batch, no rows, no tokens) return ND_OK
    before any pointer is touched or the device is queried, so a caller's
    ragged batch that happens to be empty needs no special case."""
    from neurodsl_b200 import _lib
    lib = _lib.load()
    N = None
    calls = {
        "nd_flash_attn_fwd": lambda: lib.nd_flash_attn_fwd(N, N, N, N, N, 0, N, N, 0, 4, 128, 128,
                                                           64, 0.125, 1),
        "nd_kv_decode_attn": lambda: lib.nd_kv_decode_attn(N, N, N, N, N, N, N, 0, N, 0, 4, 5, 8,
                                                           64, 0.125, N, 0),
        "nd_kv_decode_attn_qkv": lambda: lib.nd_kv_decode_attn_qkv(N, N, 0, N, N, N, 0, N, 0, 4,
                                                                   5, 8, 64, 0.125, N, 0),
        "nd_gemm_bias_act": lambda: lib.nd_gemm_bias_act(N, N, N, N, N, 0, N, 0, 0, 64, 64, 0),
        "nd_gemm_qkv_cache": lambda: lib.nd_gemm_qkv_cache(N, N, N, N, N, 0, 64, N, N, 0, 7, 2,
                                                           16, 0),
        "nd_ln_gemm": lambda: lib.nd_ln_gemm(N, N, N, N, N, N, 1e-5, N, N, N, N, 1, 0, 64, 64, 0),
        "nd_layernorm": lambda: lib.nd_layernorm(N, N, 0, N, N, N, 0, N, N, 0, 64, 1e-5),
        "nd_add_layernorm": lambda: lib.nd_add_layernorm(N, N, N, 1, N, N, N, N, N, 0, 64, 1e-5),
        "nd_softmax": lambda: lib.nd_softmax(N, N, N, 0, 16),
        "nd_scale_mask": lambda: lib.nd_scale_mask(N, N, N, 0, 16, 64),
        "nd_argmax": lambda: lib.nd_argmax(N, N, 0, 64, 0, 64, N, N),
    }
    for name, call in calls.items():
        assert call() == _lib.ND_OK, (name, lib.nd_last_error_string())
