"""The allocation-free decode entry point, nd_kv_decode_attn_noalloc.

It serves callers that may not allocate device memory during decode (a host
runtime whose device memory all comes from its own pool, or a serving process
that reserves its HBM up front and forbids cudaMalloc/cudaFree and their
device-wide synchronisation on the token loop).  Its scratch is a fixed block
inside the library, so these tests check that it gives the same results as
nd_kv_decode_attn (which uses an allocated workspace) on two calls in a row —
the second call reuses the block the first one left behind — and that shapes
larger than the block are refused.  Both entry points run the same kernel on
the same inputs, so their outputs must be identical bit for bit; the decode
tolerance (max-abs 2e-2, rel-L2 1e-2 against the oracle) is what the other
decode tests hold that kernel to.  The tests also cover a single-chunk call
(no scratch needed), a call on a side stream, and the property the entry
point exists for: free device memory is the same before and after a call at
a new, larger shape.  The file sorts last so that a run that stops at its
first failure has run every other test before this one.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _lib():
    from neurodsl_b200 import _lib
    return _lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _call_reference_entry(lib, q, kc, vc, L, kn, vn, out, lse):
    B, H, D = q.shape
    rc = lib.nd_kv_decode_attn(_stream(), _p(q), _p(kn), _p(vn), _p(kc), _p(vc), _p(out), 1,
                               _p(lse), B, H, L, kc.shape[2], D, 1.0 / 8.0, None, 0)
    assert rc == 0, lib.nd_last_error_string()


def _call_noalloc(lib, q, kc, vc, L, kn, vn, out, lse, stream=None):
    B, H, D = q.shape
    rc = lib.nd_kv_decode_attn_noalloc(_stream(stream), _p(q), _p(kn), _p(vn), _p(kc), _p(vc),
                                       _p(out), 1, _p(lse), B, H, L, kc.shape[2], D, 1.0 / 8.0)
    assert rc == 0, lib.nd_last_error_string()


def _inputs(gen, B, H, L_max, append):
    D = 64
    q = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
    kc = torch.randn(B, H, L_max, D, device="cuda", generator=gen).bfloat16()
    vc = torch.randn(B, H, L_max, D, device="cuda", generator=gen).bfloat16()
    kn = vn = None
    if append:
        kn = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
        vn = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
    return q, kc, vc, kn, vn


def _compare(lib, gen, B, H, L, L_max, append, stream=None):
    """One call of each entry point on the same inputs: identical outputs,
    log-sum-exp values and cache writes."""
    q, kc, vc, kn, vn = _inputs(gen, B, H, L_max, append)
    kc2, vc2 = kc.clone(), vc.clone()
    out_ref = torch.empty(B, H, 64, device="cuda", dtype=torch.bfloat16)
    lse_ref = torch.empty(B, H, device="cuda")
    out = torch.empty_like(out_ref)
    lse = torch.empty_like(lse_ref)
    _call_reference_entry(lib, q, kc, vc, L, kn, vn, out_ref, lse_ref)
    torch.cuda.synchronize()
    if stream is not None:
        stream.wait_stream(torch.cuda.current_stream())
    _call_noalloc(lib, q, kc2, vc2, L, kn, vn, out, lse, stream)
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref)
    assert torch.equal(lse, lse_ref)
    # the fused append wrote the same token into both caches
    assert torch.equal(kc2, kc) and torch.equal(vc2, vc)


def test_noalloc_matches_workspace_entry_two_calls_in_a_row():
    lib = _lib().load()
    gen = torch.Generator(device="cuda").manual_seed(42)
    # two consecutive calls with different shapes: the second reuses the
    # fixed scratch block (tickets and partials) left by the first
    for (B, H, L, L_max, append) in [(64, 12, 1025, 1152, True), (8, 12, 700, 1024, False)]:
        _compare(lib, gen, B, H, L, L_max, append)


def test_noalloc_single_chunk_and_side_stream():
    """L <= 128 is one chunk per head (no scratch is used at all); a call on
    a non-default stream orders its own work on that stream."""
    lib = _lib().load()
    gen = torch.Generator(device="cuda").manual_seed(7)
    _compare(lib, gen, 4, 12, 100, 128, True)
    _compare(lib, gen, 4, 12, 128, 256, False)
    side = torch.cuda.Stream()
    _compare(lib, gen, 16, 12, 900, 1024, True, stream=side)
    _compare(lib, gen, 16, 12, 60, 1024, False, stream=side)


def test_noalloc_allocates_no_device_memory():
    """A call at a new, larger shape (one that would make the workspace entry
    point grow its own buffer) leaves free device memory unchanged: every
    tensor is created first, then free memory is read around the call."""
    lib = _lib().load()
    gen = torch.Generator(device="cuda").manual_seed(3)
    small = _inputs(gen, 2, 12, 512, False)
    big = _inputs(gen, 96, 12, 2048, True)      # 96 x 12 heads x 16 chunks of partials
    out_s = torch.empty(2, 12, 64, device="cuda", dtype=torch.bfloat16)
    out_b = torch.empty(96, 12, 64, device="cuda", dtype=torch.bfloat16)
    q, kc, vc, kn, vn = small
    _call_noalloc(lib, q, kc, vc, 300, kn, vn, out_s, None)   # set-up done, module loaded
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    q, kc, vc, kn, vn = big
    for L in (2000, 2048):
        _call_noalloc(lib, q, kc, vc, L, kn, vn, out_b, None)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert torch.isfinite(out_b.float()).all()


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
