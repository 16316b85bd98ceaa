"""The allocation-free decode entry point, nd_kv_decode_attn_noalloc.

It serves callers that may not allocate device memory during decode (a host
runtime whose device memory all comes from its own pool, or a serving process
that reserves its HBM up front and forbids cudaMalloc/cudaFree and their
device-wide synchronisation on the token loop).  Its scratch is a fixed block
inside the library, so these tests check that it gives the same results as
nd_kv_decode_attn (which uses an allocated workspace) on two calls in a row —
the second call reuses the block the first one left behind — and that shapes
larger than the block are refused.  The file sorts last so that a run that
stops at its first failure has run every other test before this one.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2   # the bf16 decode tolerance used by the other decode tests
REL_L2 = 1e-2


def _lib():
    from neurodsl_b200 import _lib
    return _lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _call_reference_entry(lib, q, kc, vc, L, kn, vn, out, lse):
    B, H, D = q.shape
    rc = lib.nd_kv_decode_attn(_stream(), _p(q), _p(kn), _p(vn), _p(kc), _p(vc), _p(out), 1,
                               _p(lse), B, H, L, kc.shape[2], D, 1.0 / 8.0, None, 0)
    assert rc == 0, lib.nd_last_error_string()


def _call_noalloc(lib, q, kc, vc, L, kn, vn, out, lse):
    B, H, D = q.shape
    rc = lib.nd_kv_decode_attn_noalloc(_stream(), _p(q), _p(kn), _p(vn), _p(kc), _p(vc), _p(out),
                                       1, _p(lse), B, H, L, kc.shape[2], D, 1.0 / 8.0)
    assert rc == 0, lib.nd_last_error_string()


def _close(a, b):
    a = a.float().cpu().numpy().astype(np.float64)
    b = b.float().cpu().numpy().astype(np.float64)
    err = float(np.abs(a - b).max())
    rel = float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
    assert err <= MAX_ABS and rel <= REL_L2, (err, rel)


def test_noalloc_matches_workspace_entry_two_calls_in_a_row():
    L_ = _lib()
    lib = L_.load()
    gen = torch.Generator(device="cuda").manual_seed(42)
    # two consecutive calls with different shapes: the second reuses the
    # fixed scratch block (tickets and partials) left by the first
    for (B, H, L, L_max, append) in [(64, 12, 1025, 1152, True), (8, 12, 700, 1024, False)]:
        D = 64
        q = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
        kc = torch.randn(B, H, L_max, D, device="cuda", generator=gen).bfloat16()
        vc = torch.randn(B, H, L_max, D, device="cuda", generator=gen).bfloat16()
        kn = vn = None
        if append:
            kn = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
            vn = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
        kc2, vc2 = kc.clone(), vc.clone()
        out_ref = torch.empty(B, H, D, device="cuda", dtype=torch.bfloat16)
        lse_ref = torch.empty(B, H, device="cuda")
        out = torch.empty_like(out_ref)
        lse = torch.empty_like(lse_ref)
        _call_reference_entry(lib, q, kc, vc, L, kn, vn, out_ref, lse_ref)
        _call_noalloc(lib, q, kc2, vc2, L, kn, vn, out, lse)
        torch.cuda.synchronize()
        _close(out, out_ref)
        np.testing.assert_allclose(lse.cpu().numpy(), lse_ref.cpu().numpy(), atol=2e-3, rtol=1e-3)
        # the fused append wrote the same token into both caches
        assert torch.equal(kc2, kc) and torch.equal(vc2, vc)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    L_ = _lib()
    lib = L_.load()
    # 64 x 12 heads x 100 chunks of partials is far more than the fixed block
    B, H, L, L_max, D = 64, 12, 12800, 12800, 64
    q = torch.zeros(B, H, D, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(1, device="cuda", dtype=torch.bfloat16)  # never touched: refused first
    out = torch.empty(B, H, D, device="cuda", dtype=torch.bfloat16)
    rc = lib.nd_kv_decode_attn_noalloc(_stream(), _p(q), None, None, _p(kc), _p(kc), _p(out), 1,
                                       None, B, H, L, L_max, D, 0.125)
    assert rc == L_.ND_ERR_WORKSPACE
    assert b"fixed block" in lib.nd_last_error_string()
