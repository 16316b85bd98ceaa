"""CPU tests of the oracle: the reference's own equivalence test, float64
cross-checks, the reference's softmax property test and golden regressions."""
import numpy as np
import pytest

import oracle


def np_attention64(Q, K, V, d_head, causal):
    """float64 restatement of flash_attn_fwd_cpu_simple! for cross-checking."""
    Q, K, V = (np.asarray(a, np.float64) for a in (Q, K, V))
    S = Q @ K.T / np.sqrt(d_head)
    if causal:
        n = Q.shape[0]
        S[np.triu(np.ones((n, S.shape[1]), bool), k=1)] = -np.inf
    m = S.max(axis=1)
    E = np.exp(S - m[:, None])
    l = E.sum(axis=1)
    return (E / l[:, None]) @ V, np.log(l) + m, m


def test_tiled_matches_simple_reference_test():
    """test/test_runtime_optimizations.jl:55-69: N=8, D=16, d_head=8, causal,
    atol 1e-5 / rtol 1e-6 on out, LSE and m."""
    rng = np.random.default_rng(1234)
    Q, K, V = (rng.random((8, 16), dtype=np.float32) for _ in range(3))
    o1, l1, m1 = oracle.attn_tiled(Q, K, V, d_head=8, causal=True)
    o2, l2, m2 = oracle.attn_simple(Q, K, V, d_head=8, causal=True)
    np.testing.assert_allclose(o1, o2, atol=1e-5, rtol=1e-6)
    np.testing.assert_allclose(l1, l2, atol=1e-5, rtol=1e-6)
    np.testing.assert_allclose(m1, m2, atol=1e-5, rtol=1e-6)


@pytest.mark.parametrize("N,D,causal", [(1, 64, True), (63, 64, True), (130, 64, True),
                                        (200, 32, False), (64, 64, False)])
def test_tiled_matches_simple_shapes(N, D, causal):
    rng = np.random.default_rng(N * 7 + D)
    Q, K, V = (rng.standard_normal((N, D), dtype=np.float32) for _ in range(3))
    o1, l1, m1 = oracle.attn_tiled(Q, K, V, causal=causal)
    o2, l2, m2 = oracle.attn_simple(Q, K, V, causal=causal)
    np.testing.assert_allclose(o1, o2, atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(l1, l2, atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(m1, m2, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("N,Nk,D,causal", [(37, 37, 64, True), (5, 91, 64, False),
                                           (128, 128, 64, True)])
def test_simple_matches_float64(N, Nk, D, causal):
    rng = np.random.default_rng(N + Nk + D)
    Q = rng.standard_normal((N, D), dtype=np.float32)
    K = rng.standard_normal((Nk, D), dtype=np.float32)
    V = rng.standard_normal((Nk, D), dtype=np.float32)
    O, lse, m = oracle.attn_simple(Q, K, V, causal=causal)
    O64, lse64, m64 = np_attention64(Q, K, V, D, causal)
    np.testing.assert_allclose(O, O64, atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(lse, lse64, atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(m, m64, atol=1e-5, rtol=1e-5)


def test_causal_requires_square():
    Q = np.zeros((4, 8), np.float32)
    K = np.zeros((5, 8), np.float32)
    with pytest.raises(ValueError):
        oracle.attn_simple(Q, K, K, causal=True)


def test_empty_sequence():
    Q = np.zeros((0, 64), np.float32)
    O, lse, m = oracle.attn_simple(Q, Q, Q, causal=True)
    assert O.shape == (0, 64) and lse.shape == (0,)


def test_bhsd_matches_per_head():
    rng = np.random.default_rng(9)
    Q, K, V = (rng.standard_normal((2, 3, 50, 64), dtype=np.float32) for _ in range(3))
    O, lse, m = oracle.attn_bhsd(Q, K, V, causal=True)
    for b in range(2):
        for h in range(3):
            o, l, mm = oracle.attn_simple(Q[b, h], K[b, h], V[b, h], causal=True)
            np.testing.assert_array_equal(O[b, h], o)
            np.testing.assert_array_equal(lse[b, h], l)
            np.testing.assert_array_equal(m[b, h], mm)


def test_decode_is_single_row_attention():
    rng = np.random.default_rng(11)
    B, H, Lm, D, L = 2, 2, 40, 64, 33
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    kc = rng.standard_normal((B, H, Lm, D), dtype=np.float32)
    vc = rng.standard_normal((B, H, Lm, D), dtype=np.float32)
    out, lse = oracle.kv_decode(q, kc, vc, L)
    for b in range(B):
        for h in range(H):
            o, l, _ = np_attention64(q[b, h][None], kc[b, h, :L], vc[b, h, :L], D, False)
            np.testing.assert_allclose(out[b, h], o[0], atol=1e-5, rtol=1e-4)
            np.testing.assert_allclose(lse[b, h], l[0], atol=1e-5, rtol=1e-5)


def test_softmax_rows_sum_to_one():
    """test/test_kernels.jl:32-39: softmax rows sum to 1."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 10), dtype=np.float32)
    p = oracle.softmax(x)
    np.testing.assert_allclose(p.sum(axis=1), 1.0, atol=1e-6)


def test_scale_mask_then_softmax_equals_attention_probs():
    """The naive MultiHeadAttention path (src/layers.jl:62-72) gives the same
    probabilities as the flash path."""
    rng = np.random.default_rng(5)
    Q, K, V = (rng.standard_normal((12, 16), dtype=np.float32) for _ in range(3))
    P = oracle.softmax(oracle.scale_mask(Q @ K.T, 16))
    O, _, _ = oracle.attn_simple(Q, K, V, causal=True)
    np.testing.assert_allclose(P @ V, O, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("act", ["none", "sigmoid", "tanh", "erf"])
@pytest.mark.parametrize("trans_w", [True, False])
def test_linear_matches_float64(act, trans_w):
    import math
    rng = np.random.default_rng(21)
    M, N, K = 9, 17, 40
    A = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K) if trans_w else (K, N), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    R = rng.standard_normal((M, N), dtype=np.float32)
    Y = oracle.linear(A, W, b, residual=R, trans_w=trans_w, act=act)
    z = A.astype(np.float64) @ (W.T if trans_w else W).astype(np.float64) + b
    if act == "sigmoid":
        z = z / (1 + np.exp(-1.702 * z))
    elif act == "tanh":
        z = 0.5 * z * (1 + np.tanh(math.sqrt(2 / math.pi) * (z + 0.044715 * z ** 3)))
    elif act == "erf":
        from scipy.special import erf
        z = 0.5 * z * (1 + erf(z / math.sqrt(2)))
    np.testing.assert_allclose(Y, z + R, atol=1e-4, rtol=1e-4)


def test_layernorm_matches_float64():
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((7, 300)) * 2 + 1).astype(np.float32)
    g = rng.standard_normal(300).astype(np.float32)
    b = rng.standard_normal(300).astype(np.float32)
    y, mu, rs = oracle.layernorm(x, g, b, eps=1e-5)
    x64 = x.astype(np.float64)
    mu64 = x64.mean(1)
    var64 = ((x64 - mu64[:, None]) ** 2).mean(1)
    y64 = (x64 - mu64[:, None]) / np.sqrt(var64[:, None] + 1e-5) * g + b
    np.testing.assert_allclose(y, y64, atol=1e-4, rtol=1e-4)
    np.testing.assert_allclose(mu, mu64, rtol=1e-5, atol=1e-6)


def test_rmsnorm_template():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((3, 64)).astype(np.float32)
    g = np.ones(64, np.float32)
    y, inv = oracle.rmsnorm(x, g)
    np.testing.assert_allclose(inv, 1 / np.sqrt((x.astype(np.float64) ** 2).mean(1) + 1e-6),
                               rtol=1e-5)


def test_bf16_round_ties_to_even():
    a = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38], np.float32)
    r = oracle.bf16_round(a)
    import torch
    t = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(r, t)


# ---- golden regressions: the oracle reproduces the committed fixtures --------

def test_golden_attn_ref_shape(golden):
    g = golden("attn_ref_shape")
    O, lse, m = oracle.attn_simple(g["Q"], g["K"], g["V"], d_head=int(g["d_head"]), causal=True)
    np.testing.assert_allclose(O, g["O"], atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(lse, g["lse"], atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(m, g["m"], atol=1e-6, rtol=1e-6)
    # and the tiled form agrees with the stored result at the reference's tolerance
    O2, lse2, m2 = oracle.attn_tiled(g["Q"], g["K"], g["V"], d_head=int(g["d_head"]), causal=True)
    np.testing.assert_allclose(O2, g["O"], atol=1e-5, rtol=1e-6)


@pytest.mark.parametrize("name", ["attn_causal_bhsd", "attn_noncausal_bhsd"])
def test_golden_attn_bhsd(golden, name):
    g = golden(name)
    O, lse, m = oracle.attn_bhsd(g["Q"], g["K"], g["V"], causal=bool(g["causal"]))
    np.testing.assert_allclose(O, g["O"], atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(lse, g["lse"], atol=1e-6, rtol=1e-6)


def test_golden_kv_decode(golden):
    g = golden("kv_decode")
    out, lse = oracle.kv_decode(g["q"], g["k_cache"], g["v_cache"], int(g["L"]))
    np.testing.assert_allclose(out, g["out"], atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(lse, g["lse"], atol=1e-6, rtol=1e-6)


def test_golden_linear_gelu(golden):
    g = golden("linear_gelu")
    for act in ("sigmoid", "tanh", "erf"):
        Y = oracle.linear(g["A"], g["W"], g["bias"], act=act)
        np.testing.assert_allclose(Y, g["Y_" + act], atol=1e-6, rtol=1e-5)
    Y = oracle.linear(g["A"], g["W"], g["bias"], residual=g["residual"])
    np.testing.assert_allclose(Y, g["Y_residual"], atol=1e-6, rtol=1e-5)


def test_golden_layernorm(golden):
    g = golden("layernorm")
    for d in (1024, 100):
        y, mu, rs = oracle.layernorm(g[f"x{d}"], g[f"gamma{d}"], g[f"beta{d}"], eps=1e-5)
        np.testing.assert_allclose(y, g[f"y{d}"], atol=1e-6, rtol=1e-6)
        np.testing.assert_allclose(rs, g[f"rstd{d}"], rtol=1e-6)


def test_golden_fixtures_regenerate_bit_for_bit(tmp_path, golden):
    """The committed fixtures are what the committed generator and oracle
    produce: tests/golden/make_golden.py, run into a scratch folder, gives
    every array of every fixture bit for bit."""
    import importlib.util
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(root, "tests", "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    mg.OUT = str(tmp_path)
    mg.main()
    made = sorted(f[:-4] for f in os.listdir(tmp_path) if f.endswith(".npz"))
    assert made == ["attn_causal_bhsd", "attn_noncausal_bhsd", "attn_ref_shape", "kv_decode",
                    "layernorm", "linear_gelu"]
    for name in made:
        new = dict(np.load(os.path.join(tmp_path, name + ".npz")))
        old = golden(name)
        assert sorted(new) == sorted(old), name
        for k in old:
            np.testing.assert_array_equal(new[k], old[k], err_msg=f"{name}:{k}")
