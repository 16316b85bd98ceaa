"""The reference's operator API driving the B200 kernels: graphs built with
GraphRule / addrule / set_ and evaluated with demand, checked against the CPU
oracle.  Mirrors test/test_runtime_optimizations.jl:55-69 (flash attention on
a small graph) and the pre-LN block configuration (batch 1, seq 128, dim
1024, 16 heads x 64, MLP 4096 GELU)."""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def G():
    from neurodsl_b200 import graph
    return graph


def check(got, ref, max_abs=MAX_ABS, rel_l2=REL_L2):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = float(np.abs(got - ref).max())
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    assert err <= max_abs and rel <= rel_l2, (err, rel)


def test_flash_attn_rule_on_graph():
    """GraphRule(:ao, [:Q,:K,:V], :flash_attn; d_head=64, causal=true)."""
    g_ = G()
    rng = np.random.default_rng(1234)
    N, D = 96, 64
    Q, K, V = (oracle.bf16_round(rng.random((N, D), dtype=np.float32)) for _ in range(3))
    g = g_.NeuroGraph()
    for s, a in (("Q", Q), ("K", K), ("V", V)):
        g_.set_(g, s, a)
    g_.addrule(g, g_.GraphRule("ao", ["Q", "K", "V"], "flash_attn",
                               {"d_head": D, "causal": True}))
    ctx = g_.CtxStore()
    out = g_.demand(g, "ao", ctx_store=ctx)
    torch.cuda.synchronize()
    O_ref, l_ref, m_ref = oracle.attn_simple(Q, K, V, d_head=D, causal=True)
    check(out.cpu().numpy(), O_ref)
    nd = g.nodes["default"]["ao"]
    np.testing.assert_allclose(nd.aux_data["flash_l"].cpu().numpy(), l_ref, atol=2e-3, rtol=1e-3)
    np.testing.assert_allclose(nd.aux_data["flash_m"].cpu().numpy(), m_ref, atol=2e-3, rtol=1e-3)
    assert set(ctx["ao"]) == {"Q", "K", "V", "out", "l", "m", "d_head", "causal"}
    assert out.dtype == torch.float32 and tuple(out.shape) == (N, D)


def test_multihead_flash_attention_rule():
    g_ = G()
    rng = np.random.default_rng(2)
    S, Hh, D = 130, 4, 64
    q, k, v = (oracle.bf16_round(rng.standard_normal((S, Hh * D), dtype=np.float32))
               for _ in range(3))
    g = g_.NeuroGraph()
    for s, a in (("q", q), ("k", k), ("v", v)):
        g_.set_(g, s, a)
    g_.addrule(g, g_.GraphRule("attn", ["q", "k", "v"], "flash_attention",
                               {"n_heads": Hh, "causal": True}))
    out = g_.demand(g, "attn").cpu().numpy()
    for h in range(Hh):
        sl = slice(h * D, (h + 1) * D)
        o_ref, _, _ = oracle.attn_simple(q[:, sl], k[:, sl], v[:, sl], causal=True)
        check(out[:, sl], o_ref)


def test_multihead_flash_attention_fused_qkv():
    """One (S, 3·H·D) projection as the single input: q, k, v are read from
    its column blocks in place."""
    g_ = G()
    rng = np.random.default_rng(5)
    S, Hh, D = 200, 4, 64
    qkv = oracle.bf16_round(rng.standard_normal((S, 3 * Hh * D), dtype=np.float32))
    g = g_.NeuroGraph()
    g_.set_(g, "qkv", qkv)
    g_.addrule(g, g_.GraphRule("attn", ["qkv"], "flash_attention",
                               {"n_heads": Hh, "causal": True}))
    out = g_.demand(g, "attn").cpu().numpy()
    assert out.shape == (S, Hh * D)
    d = Hh * D
    for h in range(Hh):
        sl = slice(h * D, (h + 1) * D)
        o_ref, _, _ = oracle.attn_simple(qkv[:, sl], qkv[:, d:][:, sl], qkv[:, 2 * d:][:, sl],
                                         causal=True)
        check(out[:, sl], o_ref)


def build_block(g_, g, x, params, n_heads):
    """Pre-LN causal block from GraphRules:
    LN -> Q,K,V linear -> multi-head causal flash attention -> out-proj + x
    -> LN -> linear + GELU -> linear + residual."""
    R = g_.GraphRule
    g_.set_(g, "x", x)
    for k, v in params.items():
        g_.set_(g, k, v, is_param=True)
    g_.addrule(g, R("ln1", ["x", "ln1_g", "ln1_b"], "layernorm", {"eps": 1e-5}))
    for p in ("q", "k", "v"):
        g_.addrule(g, R(p, ["ln1", f"W{p}", f"b{p}"], "linear"))
    g_.addrule(g, R("attn", ["q", "k", "v"], "flash_attention", {"n_heads": n_heads,
                                                                 "causal": True}))
    g_.addrule(g, R("h1", ["attn", "Wo", "bo", "x"], "fused_linear_residual"))
    g_.addrule(g, R("ln2", ["h1", "ln2_g", "ln2_b"], "layernorm", {"eps": 1e-5}))
    g_.addrule(g, R("up", ["ln2", "W1", "b1"], "fused_linear_gelu",
                    {"trans_b": True, "approx": "sigmoid"}))
    g_.addrule(g, R("y", ["up", "W2", "b2", "h1"], "fused_linear_residual"))


def oracle_block(x, p, n_heads):
    S, d = x.shape
    D = d // n_heads
    ln1, _, _ = oracle.layernorm(x, p["ln1_g"], p["ln1_b"], eps=1e-5)
    q = oracle.linear(ln1, p["Wq"], p["bq"])
    k = oracle.linear(ln1, p["Wk"], p["bk"])
    v = oracle.linear(ln1, p["Wv"], p["bv"])
    attn = np.zeros_like(q)
    for h in range(n_heads):
        sl = slice(h * D, (h + 1) * D)
        attn[:, sl], _, _ = oracle.attn_simple(q[:, sl], k[:, sl], v[:, sl], causal=True)
    h1 = oracle.linear(attn, p["Wo"], p["bo"], residual=x)
    ln2, _, _ = oracle.layernorm(h1, p["ln2_g"], p["ln2_b"], eps=1e-5)
    up = oracle.linear(ln2, p["W1"], p["b1"], act="sigmoid")
    return oracle.linear(up, p["W2"], p["b2"], residual=h1)


def block_params(rng, d, f):
    w = lambda o, i: oracle.bf16_round((0.02 * rng.standard_normal((o, i))).astype(np.float32))
    z = lambda n: np.zeros(n, np.float32)
    return {"ln1_g": np.ones(d, np.float32), "ln1_b": z(d), "ln2_g": np.ones(d, np.float32),
            "ln2_b": z(d), "Wq": w(d, d), "bq": z(d), "Wk": w(d, d), "bk": z(d), "Wv": w(d, d),
            "bv": z(d), "Wo": w(d, d), "bo": z(d), "W1": w(f, d), "b1": z(f), "W2": w(d, f),
            "b2": z(d)}


def test_pre_ln_block_config():
    """Batch 1, seq 128, dim 1024, 16 heads x 64, MLP 1024->4096->1024 with
    GELU; x ~ N(0,1), weights ~ N(0,0.02), biases 0, LayerNorm gamma=1 beta=0."""
    g_ = G()
    rng = np.random.default_rng(0)
    S, d, f, nh = 128, 1024, 4096, 16
    x = rng.standard_normal((S, d)).astype(np.float32)
    p = block_params(rng, d, f)
    g = g_.NeuroGraph()
    build_block(g_, g, x, p, nh)
    y = g_.demand(g, "y")
    torch.cuda.synchronize()
    y_ref = oracle_block(x, p, nh)
    check(y.cpu().numpy(), y_ref)
    # incremental: a new input invalidates and recomputes the whole block
    x2 = rng.standard_normal((S, d)).astype(np.float32)
    g_.set_(g, "x", x2)
    assert not g.nodes["default"]["y"].valid
    y2 = g_.demand(g, "y")
    check(y2.cpu().numpy(), oracle_block(x2, p, nh))


def test_kv_decode_rule_with_append():
    g_ = G()
    rng = np.random.default_rng(5)
    Bt, Hh, D, L_max, L = 4, 12, 64, 300, 200
    kc = torch.from_numpy(oracle.bf16_round(
        rng.standard_normal((Bt, Hh, L_max, D), dtype=np.float32))).cuda().bfloat16()
    vc = torch.from_numpy(oracle.bf16_round(
        rng.standard_normal((Bt, Hh, L_max, D), dtype=np.float32))).cuda().bfloat16()
    q = oracle.bf16_round(rng.standard_normal((Bt, Hh * D), dtype=np.float32))
    kn = oracle.bf16_round(rng.standard_normal((Bt, Hh * D), dtype=np.float32))
    vn = oracle.bf16_round(rng.standard_normal((Bt, Hh * D), dtype=np.float32))
    kc_np = kc.float().cpu().numpy()
    vc_np = vc.float().cpu().numpy()
    g = g_.NeuroGraph()
    g_.set_(g, "q", q)
    g_.set_(g, "kc", kc)
    g_.set_(g, "vc", vc)
    g_.set_(g, "kn", kn)
    g_.set_(g, "vn", vn)
    g_.addrule(g, g_.GraphRule("o", ["q", "kc", "vc", "kn", "vn"], "kv_decode_attn",
                               {"n_heads": Hh, "d_head": D, "cache_len": L}))
    out = g_.demand(g, "o").cpu().numpy()
    kc_np[:, :, L - 1] = kn.reshape(Bt, Hh, D)
    vc_np[:, :, L - 1] = vn.reshape(Bt, Hh, D)
    ref, _ = oracle.kv_decode(q.reshape(Bt, Hh, D), kc_np, vc_np, L)
    check(out, ref.reshape(Bt, Hh * D))


def test_matmul_trans_b_false_and_linear_alias():
    g_ = G()
    rng = np.random.default_rng(8)
    A = oracle.bf16_round(rng.standard_normal((40, 64), dtype=np.float32))
    B = oracle.bf16_round(rng.standard_normal((64, 48), dtype=np.float32))
    g = g_.NeuroGraph()
    g_.set_(g, "A", A)
    g_.set_(g, "B", B)
    g_.addrule(g, g_.GraphRule("C", ["A", "B"], "matmul"))
    g_.addrule(g, g_.GraphRule("Ct", ["A", "Bt"], "matmul", {"trans_b": True}))
    g_.set_(g, "Bt", np.ascontiguousarray(B.T))
    C = g_.demand(g, "C").cpu().numpy()
    Ct = g_.demand(g, "Ct").cpu().numpy()
    ref = A.astype(np.float64) @ B
    check(C, ref)
    check(Ct, ref)


def test_embedding_op_on_the_device():
    """:embedding (src/dispatch.jl:476-491) gathers Float32 rows of E by
    1-based Float32 indices on the device (nd_gather_rows), exactly, with the
    reference's ctx {idx, E_size}.  An index past the table, or one that is
    not an integer, gives a zero row and sets the device error word (16)
    instead of synchronising the host; good calls leave the word at 0."""
    from neurodsl_b200 import ops
    g_ = G()
    ops.device_error()
    rng = np.random.default_rng(21)
    E = rng.standard_normal((50, 64)).astype(np.float32)
    idx = np.array([3, 50, 1, 7, 7], np.float32)
    g = g_.NeuroGraph()
    g_.set_(g, "E", E, is_param=True)
    g_.set_(g, "idx", idx)
    g_.addrule(g, g_.GraphRule("emb", ["E", "idx"], "embedding"))
    ctx = g_.CtxStore()
    out = g_.demand(g, "emb", ctx_store=ctx)
    assert out.is_cuda
    np.testing.assert_array_equal(out.cpu().numpy(), E[idx.astype(np.int64) - 1])
    assert ctx["emb"]["E_size"] == (50, 64)
    assert ctx["emb"]["idx"].cpu().tolist() == [3, 50, 1, 7, 7]
    assert ops.device_error() == 0
    for bad in ([51.0], [0.0], [2.5]):
        g_.set_(g, "idx", np.array([1.0] + bad, np.float32))
        out = g_.demand(g, "emb").cpu().numpy()
        np.testing.assert_array_equal(out[0], E[0])
        assert not out[1].any()
        assert ops.device_error() == 16


def test_copy_ops_run_on_the_library():
    """:slice_cols, :hcat_heads and :identity (src/dispatch.jl:544-553,
    :349-361) are device copies by nd_copy_2d: the sliced columns, the heads
    side by side and the input itself, bit for bit; odd widths and offsets
    take the narrower copy units."""
    g_ = G()
    rng = np.random.default_rng(22)
    X = rng.standard_normal((37, 130)).astype(np.float32)
    g = g_.NeuroGraph()
    g_.set_(g, "X", X)
    g_.addrule(g, g_.GraphRule("s1", ["X"], "slice_cols", {"start_col": 1, "end_col": 64}))
    g_.addrule(g, g_.GraphRule("s2", ["X"], "slice_cols", {"start_col": 66, "end_col": 130}))
    g_.addrule(g, g_.GraphRule("s3", ["X"], "slice_cols", {"start_col": 3, "end_col": 3}))
    g_.addrule(g, g_.GraphRule("cat", ["s1", "s2", "s3"], "hcat_heads"))
    g_.addrule(g, g_.GraphRule("same", ["X"], "identity"))
    cat = g_.demand(g, "cat").cpu().numpy()
    np.testing.assert_array_equal(cat, np.concatenate([X[:, :64], X[:, 65:130], X[:, 2:3]], axis=1))
    np.testing.assert_array_equal(g_.demand(g, "same").cpu().numpy(), X)


def test_linear_weight_converted_once_and_refreshed_on_change():
    """A :linear weight node's bf16 copy is made once and reused by later
    runs; replacing the node's value (set!) or writing the tensor in place
    makes the next run convert again, so results follow the weight.  K = 13
    is padded to 16 in the same conversion."""
    from neurodsl_b200 import graph as GR
    g_ = G()
    rng = np.random.default_rng(23)
    X = oracle.bf16_round(rng.standard_normal((64, 13)).astype(np.float32))
    W = oracle.bf16_round((0.1 * rng.standard_normal((24, 13))).astype(np.float32))
    g = g_.NeuroGraph()
    g_.set_(g, "X", X)
    g_.set_(g, "W", W, is_param=True)
    g_.addrule(g, g_.GraphRule("Y", ["X", "W"], "linear"))
    y1 = g_.demand(g, "Y").cpu().numpy()
    Wt = g.nodes["default"]["W"].value
    hit = GR._WEIGHT_CACHE.get(id(Wt))
    assert hit is not None and hit[3].shape == (24, 16)
    conv = hit[3]
    g_.set_(g, "X", X * 2)                 # recompute with the same weight
    y2 = g_.demand(g, "Y").cpu().numpy()
    assert GR._WEIGHT_CACHE[id(Wt)][3] is conv
    np.testing.assert_allclose(y2, 2 * y1, rtol=1e-5, atol=1e-6)
    Wt.mul_(2)                             # in place: the version moves
    g_.set_(g, "X", X)
    y3 = g_.demand(g, "Y").cpu().numpy()
    np.testing.assert_allclose(y3, 2 * y1, rtol=1e-5, atol=1e-6)
    g_.set_(g, "W", -W, is_param=True)     # a new tensor
    y4 = g_.demand(g, "Y").cpu().numpy()
    np.testing.assert_allclose(y4, -y1, rtol=1e-5, atol=1e-6)
