"""GPU parity of nd_flash_attn_fwd_strided: attention read from and written
to token-major [B][S][H][64] tensors (the layout of (S, H·64) projections)
through strides, against the CPU oracle and against the head-major entry
point on the same values.

Tolerance for the bf16 tensor-core path: max-abs <= 2e-2 and relative L2
<= 1e-2 on O against the fp32 oracle fed the same bf16-rounded inputs; the
strided and head-major kernels compute identical values (compared exactly).
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _ops():
    from neurodsl_b200 import ops
    return ops


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _token_major(B, S, H, seed, D=64):
    rng = np.random.default_rng(seed)
    x = oracle.bf16_round(rng.standard_normal((B, S, H, D), dtype=np.float32))
    return x, torch.from_numpy(x).cuda().to(torch.bfloat16)


@pytest.mark.parametrize("S,causal", [(128, True), (200, True), (333, False), (1024, True)])
@pytest.mark.parametrize("out_f32", [False, True])
def test_token_major_matches_oracle_and_head_major(S, causal, out_f32):
    ops = _ops()
    B, H = 2, 3
    qn, q = _token_major(B, S, H, 1)
    kn, k = _token_major(B, S, H, 2)
    vn, v = _token_major(B, S, H, 3)
    odt = torch.float32 if out_f32 else torch.bfloat16
    out = torch.full((B, S, H, 64), float("nan"), device="cuda", dtype=odt)
    view = lambda t: t.permute(0, 2, 1, 3)   # [B][H][S][D] view, token-major strides
    _, lse, m = ops.flash_attn_fwd(view(q), view(k), view(v), causal=causal, out=view(out))
    # head-major reference launch on copies
    hm = lambda t: view(t).contiguous()
    O2, lse2, m2 = ops.flash_attn_fwd(hm(q), hm(k), hm(v), causal=causal, out_dtype=odt)
    torch.cuda.synchronize()
    assert torch.equal(view(out), O2), "strided and head-major kernels differ"
    assert torch.equal(lse, lse2) and torch.equal(m, m2)
    O = out.float().cpu().numpy()
    for b in range(B):
        for h in range(H):
            Or, lr, mr = oracle.attn_simple(qn[b, :, h], kn[b, :, h], vn[b, :, h], causal=causal)
            err = float(np.abs(O[b, :, h] - Or).max())
            assert err <= MAX_ABS, f"b={b} h={h} max-abs {err}"
            assert rel_l2(O[b, :, h], Or) <= REL_L2
            np.testing.assert_allclose(lse[b, h].cpu().numpy(), lr, atol=2e-3, rtol=1e-3)
            np.testing.assert_allclose(m[b, h].cpu().numpy(), mr, atol=2e-3, rtol=1e-3)


def test_fused_qkv_projection_layout():
    """Q, K, V as the three column blocks of one (S, 3·H·64) projection."""
    ops = _ops()
    S, H = 256, 4
    rng = np.random.default_rng(7)
    qkv_n = oracle.bf16_round(rng.standard_normal((S, 3 * H * 64), dtype=np.float32))
    qkv = torch.from_numpy(qkv_n).cuda().to(torch.bfloat16)
    parts = qkv.view(S, 3, H, 64).permute(1, 2, 0, 3).unsqueeze(1)   # [3][1][H][S][64]
    out = torch.empty((S, H * 64), device="cuda", dtype=torch.bfloat16)
    ops.flash_attn_fwd(parts[0], parts[1], parts[2], causal=True,
                       out=out.view(S, H, 64).permute(1, 0, 2).unsqueeze(0))
    torch.cuda.synchronize()
    O = out.float().cpu().numpy().reshape(S, H, 64)
    x = qkv_n.reshape(S, 3, H, 64)
    for h in range(H):
        Or, _, _ = oracle.attn_simple(x[:, 0, h], x[:, 1, h], x[:, 2, h], causal=True)
        assert float(np.abs(O[:, h] - Or).max()) <= MAX_ABS
        assert rel_l2(O[:, h], Or) <= REL_L2


def _strided_call(q, qs, k, ks, v, vs, o, os_, B=1, H=1, S=128):
    from neurodsl_b200 import _lib
    lib = _lib.load()
    arr = lambda t: (ctypes.c_int64 * 3)(*t)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    return lib.nd_flash_attn_fwd_strided(None, p(q), arr(qs), p(k), arr(ks), p(v), arr(vs), p(o),
                                         arr(os_), 1, None, None, B, H, S, S, 64, 0.125, 1)


def test_rejects_bad_strides():
    t = torch.zeros((4, 128, 64), device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(t)
    B, H = 2, 2
    hm = (64, 128 * 64, H * 128 * 64)
    tm = (H * 64, 64, 128 * H * 64)
    assert _strided_call(t, hm, t, hm, t, hm, o, hm, B, H) == 0
    assert _strided_call(t, tm, t, tm, t, tm, o, tm, B, H) == 0
    torch.cuda.synchronize()
    # stride not a multiple of 8 elements
    assert _strided_call(t, (60, 128 * 64, H * 128 * 64), t, hm, t, hm, o, hm, B, H) == 2
    # batch stride inside a head (only checked when B > 1)
    assert _strided_call(t, (64, 128 * 64, 64), t, hm, t, hm, o, hm, B, H) == 2
    # K head-major, V token-major
    assert _strided_call(t, hm, t, hm, t, tm, o, hm, B, H) == 2


@pytest.mark.parametrize("B,H,S", [(16, 12, 512), (13, 12, 300)])
@pytest.mark.parametrize("token_major", [True, False])
def test_many_light_items_per_cta(B, H, S, token_major):
    """More (batch, head) pairs than SMs with short sequences: a persistent CTA
    processes several consecutive items of only one or two K/V tiles, whose
    ring stages must be released in order (the first query tile skips the
    last K/V tile of every item).  The kernel completes without a wait
    deadline (device error word 0) and matches the oracle on the first and
    last batch entries."""
    ops = _ops()
    ops.device_error()
    q_np, q = _token_major(B, S, H, 31)
    k_np, k = _token_major(B, S, H, 32)
    v_np, v = _token_major(B, S, H, 33)
    tr = lambda t: t.permute(0, 2, 1, 3)
    if token_major:
        o = torch.empty(B, S, H, 64, device="cuda", dtype=torch.bfloat16)
        ops.flash_attn_fwd(tr(q), tr(k), tr(v), causal=True, out=tr(o))
        got = tr(o)
    else:
        got = torch.empty(B, H, S, 64, device="cuda", dtype=torch.bfloat16)
        ops.flash_attn_fwd(tr(q).contiguous(), tr(k).contiguous(), tr(v).contiguous(),
                           causal=True, out=got)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for b in (0, B - 1):
        sel = lambda a: np.ascontiguousarray(a[b:b + 1].transpose(0, 2, 1, 3))
        ref, _, _ = oracle.attn_bhsd(sel(q_np), sel(k_np), sel(v_np), causal=True)
        g = got[b:b + 1].float().cpu().numpy()
        assert np.abs(g - ref).max() <= MAX_ABS
        assert rel_l2(g, ref) <= REL_L2
