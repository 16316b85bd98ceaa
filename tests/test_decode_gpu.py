"""GPU parity of nd_kv_decode_attn / nd_kv_append against the oracle's
single-query attention (flash_attn_fwd_cpu_simple! with one row), through the
C ABI.  Same bf16 tolerance as the prefill path."""
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


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)


def check(out, ref, lse=None, lse_ref=None):
    err = float(np.abs(out - ref).max())
    rel = float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30))
    assert err <= MAX_ABS and rel <= REL_L2, (err, rel)
    if lse is not None:
        np.testing.assert_allclose(lse, lse_ref, atol=2e-3, rtol=1e-3)


def test_golden_fixture(golden):
    g = golden("kv_decode")
    ops = _ops()
    out, lse = ops.kv_decode_attn(_t(g["q"]), _t(g["k_cache"]), _t(g["v_cache"]), int(g["L"]))
    check(out.float().cpu().numpy(), g["out"], lse.cpu().numpy(), g["lse"])


@pytest.mark.parametrize("L", [1, 5, 127, 128, 129, 511, 1025, 1152])
@pytest.mark.parametrize("fused_append", [False, True])
def test_lengths(L, fused_append):
    ops = _ops()
    rng = np.random.default_rng(L)
    B, H, D, L_max = 3, 4, 64, 1160
    q = oracle.bf16_round(rng.standard_normal((B, H, D), dtype=np.float32))
    kc = oracle.bf16_round(rng.standard_normal((B, H, L_max, D), dtype=np.float32))
    vc = oracle.bf16_round(rng.standard_normal((B, H, L_max, D), dtype=np.float32))
    kn = oracle.bf16_round(rng.standard_normal((B, H, D), dtype=np.float32))
    vn = oracle.bf16_round(rng.standard_normal((B, H, D), dtype=np.float32))
    kc_g, vc_g = _t(kc), _t(vc)
    if fused_append:
        out, lse = ops.kv_decode_attn(_t(q), kc_g, vc_g, L, k_new=_t(kn), v_new=_t(vn))
        kc[:, :, L - 1] = kn
        vc[:, :, L - 1] = vn
    else:
        out, lse = ops.kv_decode_attn(_t(q), kc_g, vc_g, L)
    torch.cuda.synchronize()
    ref, lse_ref = oracle.kv_decode(q, kc, vc, L)
    check(out.float().cpu().numpy(), ref, lse.cpu().numpy(), lse_ref)
    # the caches now hold the appended token and nothing else changed
    np.testing.assert_array_equal(kc_g.float().cpu().numpy(), kc)
    np.testing.assert_array_equal(vc_g.float().cpu().numpy(), vc)


def test_caller_workspace_and_fp32_out():
    ops = _ops()
    rng = np.random.default_rng(3)
    B, H, D, L_max, L = 2, 12, 64, 1024, 1000
    q = oracle.bf16_round(rng.standard_normal((B, H, D), dtype=np.float32))
    kc = oracle.bf16_round(rng.standard_normal((B, H, L_max, D), dtype=np.float32))
    vc = oracle.bf16_round(rng.standard_normal((B, H, L_max, D), dtype=np.float32))
    n = ops.kv_decode_workspace_size(B, H, L)
    assert n > 0
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    ref, lse_ref = oracle.kv_decode(q, kc, vc, L)
    for _ in range(3):  # the workspace tickets must reset between calls
        out, lse = ops.kv_decode_attn(_t(q), _t(kc), _t(vc), L, out_dtype=torch.float32,
                                      workspace=ws)
        torch.cuda.synchronize()
        check(out.cpu().numpy(), ref, lse.cpu().numpy(), lse_ref)
    from neurodsl_b200._lib import NeuroDSLError
    with pytest.raises(NeuroDSLError):
        ops.kv_decode_attn(_t(q), _t(kc), _t(vc), L, workspace=ws[: n // 2])


def test_library_workspace_across_shapes():
    """Calls of different (B, H, L) share the library-owned scratch buffer;
    each must see a clean ticket region."""
    ops = _ops()
    rng = np.random.default_rng(21)
    for (B, H, L) in [(2, 12, 511), (3, 4, 129), (1, 12, 1025), (3, 4, 129), (64, 12, 1152),
                      (2, 2, 300)]:
        L_max = L + 3
        q = oracle.bf16_round(rng.standard_normal((B, H, 64), dtype=np.float32))
        kc = oracle.bf16_round(rng.standard_normal((B, H, L_max, 64), dtype=np.float32))
        vc = oracle.bf16_round(rng.standard_normal((B, H, L_max, 64), dtype=np.float32))
        out, lse = ops.kv_decode_attn(_t(q), _t(kc), _t(vc), L)
        torch.cuda.synchronize()
        ref, lse_ref = oracle.kv_decode(q, kc, vc, L)
        check(out.float().cpu().numpy(), ref, lse.cpu().numpy(), lse_ref)


def test_append_kernel():
    ops = _ops()
    B, H, D, L_max = 2, 3, 64, 10
    kc = torch.zeros(B, H, L_max, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kn = torch.randn(B, H, D, device="cuda").bfloat16()
    vn = torch.randn(B, H, D, device="cuda").bfloat16()
    ops.kv_append(kn, vn, kc, vc, 7)
    torch.cuda.synchronize()
    assert torch.equal(kc[:, :, 7], kn) and torch.equal(vc[:, :, 7], vn)
    assert kc[:, :, :7].abs().sum() == 0 and kc[:, :, 8:].abs().sum() == 0


def test_decode_config_sequence():
    """Batch 64, 12 heads, head_dim 64, cache prefilled to 1024, 128 decode
    steps each appending one token; steps 1, 64 and 128 checked against the
    oracle, every step checked for finiteness."""
    ops = _ops()
    B, H, D, L0, T = 64, 12, 64, 1024, 128
    L_max = L0 + T
    gen = torch.Generator(device="cuda").manual_seed(1)
    kc = torch.randn(B, H, L_max, D, device="cuda", generator=gen).bfloat16()
    vc = torch.randn(B, H, L_max, D, device="cuda", generator=gen).bfloat16()
    for t in range(1, T + 1):
        L = L0 + t
        q = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
        kn = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
        vn = torch.randn(B, H, D, device="cuda", generator=gen).bfloat16()
        out, lse = ops.kv_decode_attn(q, kc, vc, L, k_new=kn, v_new=vn)
        if t in (1, 64, 128):
            torch.cuda.synchronize()
            sel = slice(0, 8)  # 8 sequences x 12 heads against the oracle
            ref, lse_ref = oracle.kv_decode(q[sel].float().cpu().numpy(),
                                            kc[sel].float().cpu().numpy(),
                                            vc[sel].float().cpu().numpy(), L)
            check(out[sel].float().cpu().numpy(), ref, lse[sel].cpu().numpy(), lse_ref)
            assert torch.equal(kc[:, :, L - 1], kn)
        assert torch.isfinite(out.float()).all()


def test_rejects_bad_arguments():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    q = torch.zeros(1, 1, 64, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(1, 1, 8, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(NeuroDSLError):
        ops.kv_decode_attn(q, kc, kc, 9)  # L > L_max
    with pytest.raises(NeuroDSLError):
        ops.kv_decode_attn(q, kc, kc, 0)
