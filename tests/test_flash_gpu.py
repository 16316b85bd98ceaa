"""GPU parity of nd_flash_attn_fwd against the CPU oracle (the reference's
Float32 attention restated), through the C ABI.

Tolerance for the bf16 tensor-core path: max-abs <= 2e-2 and relative L2
<= 1e-2 on O against the fp32 oracle fed the same bf16-rounded inputs.
"""
import math

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


def check_close(O, O_ref, lse=None, lse_ref=None, m=None, m_ref=None):
    err = float(np.abs(O - O_ref).max()) if O.size else 0.0
    assert err <= MAX_ABS, f"max-abs {err}"
    if O.size:
        assert rel_l2(O, O_ref) <= REL_L2, f"rel-L2 {rel_l2(O, O_ref)}"
    if lse is not None:
        np.testing.assert_allclose(lse, lse_ref, atol=2e-3, rtol=1e-3)
    if m is not None:
        np.testing.assert_allclose(m, m_ref, atol=2e-3, rtol=1e-3)


def run_gpu(Q, K, V, causal, out_dtype=None):
    ops = _ops()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)
    out_dtype = out_dtype or torch.bfloat16
    O, lse, m = ops.flash_attn_fwd(t(Q), t(K), t(V), causal=causal, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return O.float().cpu().numpy(), lse.cpu().numpy(), m.cpu().numpy()


def rand_bhsd(rng, B, H, S, D=64):
    return oracle.bf16_round(rng.standard_normal((B, H, S, D), dtype=np.float32))


@pytest.mark.parametrize("name", ["attn_causal_bhsd", "attn_noncausal_bhsd"])
def test_golden_fixture(golden, name):
    g = golden(name)
    O, lse, m = run_gpu(g["Q"], g["K"], g["V"], bool(g["causal"]))
    check_close(O, g["O"], lse, g["lse"], m, g["m"])


@pytest.mark.parametrize("S", [1, 7, 64, 127, 128, 129, 256, 300, 515])
def test_causal_shapes(S):
    rng = np.random.default_rng(S)
    Q, K, V = (rand_bhsd(rng, 1, 2, S) for _ in range(3))
    O_ref, lse_ref, m_ref = oracle.attn_bhsd(Q, K, V, causal=True)
    O, lse, m = run_gpu(Q, K, V, True)
    check_close(O, O_ref, lse, lse_ref, m, m_ref)


@pytest.mark.parametrize("Sq,Sk", [(1, 1), (1, 300), (128, 64), (200, 129), (64, 1000)])
def test_noncausal_shapes(Sq, Sk):
    rng = np.random.default_rng(Sq * 1000 + Sk)
    Q = rand_bhsd(rng, 2, 1, Sq)
    K = rand_bhsd(rng, 2, 1, Sk)
    V = rand_bhsd(rng, 2, 1, Sk)
    O_ref, lse_ref, m_ref = oracle.attn_bhsd(Q, K, V, causal=False)
    O, lse, m = run_gpu(Q, K, V, False)
    check_close(O, O_ref, lse, lse_ref, m, m_ref)


def test_fp32_output():
    rng = np.random.default_rng(5)
    Q, K, V = (rand_bhsd(rng, 1, 3, 333) for _ in range(3))
    O_ref, lse_ref, _ = oracle.attn_bhsd(Q, K, V, causal=True)
    O, lse, _ = run_gpu(Q, K, V, True, out_dtype=torch.float32)
    check_close(O, O_ref, lse, lse_ref)


def test_large_logits_rescaling():
    """Rows whose max grows across key tiles exercise the running-max update."""
    rng = np.random.default_rng(11)
    S = 640
    Q, K, V = (rand_bhsd(rng, 1, 1, S) for _ in range(3))
    ramp = np.linspace(0.2, 4.0, S, dtype=np.float32)[None, None, :, None]
    K = oracle.bf16_round(K * ramp)
    Q = oracle.bf16_round(Q * 2.0)
    O_ref, lse_ref, m_ref = oracle.attn_bhsd(Q, K, V, causal=True)
    O, lse, m = run_gpu(Q, K, V, True)
    check_close(O, O_ref, lse, lse_ref, m, m_ref)


def test_prefill_config_full_size():
    """Causal prefill at batch 8, 16 heads, head_dim 64, seq 2048: eight heads
    against the oracle, every head checked for normalisation properties."""
    ops = _ops()
    B, H, S, D = 8, 16, 2048, 64
    gen = torch.Generator(device="cuda").manual_seed(0)
    Q = torch.randn(B, H, S, D, device="cuda", generator=gen).bfloat16()
    K = torch.randn(B, H, S, D, device="cuda", generator=gen).bfloat16()
    V = torch.randn(B, H, S, D, device="cuda", generator=gen).bfloat16()
    O, lse, m = ops.flash_attn_fwd(Q, K, V, causal=True)
    torch.cuda.synchronize()
    assert torch.isfinite(O.float()).all() and torch.isfinite(lse).all()
    # lse >= m (log of a sum that contains exp(0)) and lse <= m + log(i+1)
    pos = torch.arange(S, device="cuda").float()
    assert (lse >= m - 1e-4).all()
    assert (lse <= m + torch.log(pos + 1) + 1e-3).all()
    # row 0 attends only to key 0: O[...,0,:] == V[...,0,:]
    assert torch.allclose(O[:, :, 0].float(), V[:, :, 0].float(), atol=1e-2)
    Qn, Kn, Vn = (x.float().cpu().numpy() for x in (Q, K, V))
    for (b, h) in [(0, 0), (1, 5), (3, 15), (7, 7), (4, 2), (2, 11), (6, 0), (5, 9)]:
        o_ref, l_ref, m_ref = oracle.attn_simple(Qn[b, h], Kn[b, h], Vn[b, h], causal=True)
        check_close(O[b, h].float().cpu().numpy(), o_ref, lse[b, h].cpu().numpy(), l_ref,
                    m[b, h].cpu().numpy(), m_ref)


def test_rejects_bad_arguments():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    q = torch.zeros(1, 1, 16, 32, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(NeuroDSLError):
        ops.flash_attn_fwd(q, q, q, causal=True)  # head_dim 32 unsupported
    q = torch.zeros(1, 1, 16, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 1, 20, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(NeuroDSLError):
        ops.flash_attn_fwd(q, k, k, causal=True)  # causal needs Sq == Sk
    assert ops.device_error() == 0


def test_empty_batch_is_noop():
    ops = _ops()
    q = torch.zeros(0, 2, 16, 64, device="cuda", dtype=torch.bfloat16)
    O, lse, m = ops.flash_attn_fwd(q, q, q, causal=True)
    assert O.shape == (0, 2, 16, 64)
