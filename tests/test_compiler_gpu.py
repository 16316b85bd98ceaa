"""GPU checks of graphs compiled by the rewrite rules: each graph runs once as
written (unfused ops, each a library kernel) and once compiled onto the fused
operators; both are compared with the oracle (bf16-operand tolerance:
max-abs 2e-2, rel-L2 1e-2) and with each other."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2


def _mods():
    from neurodsl_b200 import compiler as C
    from neurodsl_b200 import graph as G
    return C, G


def check(out, ref, max_abs=MAX_ABS, rel_l2=REL_L2):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    err = float(np.abs(out - ref).max())
    rel = float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30))
    assert err <= max_abs and rel <= rel_l2, (err, rel)


def _run(build, compiled, out):
    C, G = _mods()
    g = G.NeuroGraph()
    build(G, g)
    fused = {}
    if compiled:
        fused = C.compile(g, C.CompilerConfig(training=False)).fused_ops
    y = G.demand(g, out)
    torch.cuda.synchronize()
    return y.float().cpu().numpy(), fused, g


def test_unfused_elementwise_ops_match_oracle():
    _, G = _mods()
    rng = np.random.default_rng(0)
    s = rng.standard_normal((96, 96)).astype(np.float32) * 4
    x = rng.standard_normal((37, 50)).astype(np.float32)
    g = G.NeuroGraph()
    G.set_(g, "s", s)
    G.set_(g, "x", x)
    G.addrule(g, G.GraphRule("sm", ["s"], "scale_mask", attrs={"d_head": 64}))
    G.addrule(g, G.GraphRule("p", ["sm"], "softmax"))
    G.addrule(g, G.GraphRule("ge", ["x"], "gelu", attrs={"approx": "tanh"}))
    p = G.demand(g, "p").cpu().numpy()
    ge = G.demand(g, "ge").cpu().numpy()
    np.testing.assert_allclose(p, oracle.softmax(oracle.scale_mask(s, 64)), atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(np.triu(p, 1), 0.0)
    # the oracle's GELU through an identity matrix (x·I is exact in fp32)
    ge_ref = oracle.linear(x, np.eye(x.shape[1], dtype=np.float32), act="tanh")
    np.testing.assert_allclose(ge, ge_ref, atol=1e-5, rtol=1e-5)


def test_matmul_gelu_compiles_to_the_fused_gemm():
    rng = np.random.default_rng(1)
    x = oracle.bf16_round(rng.standard_normal((128, 256)).astype(np.float32))
    W = oracle.bf16_round((0.05 * rng.standard_normal((256, 384))).astype(np.float32))

    def build(G, g):
        G.set_(g, "x", x)
        G.set_(g, "W", W, is_param=True)
        G.addrule(g, G.GraphRule("u", ["x", "W"], "matmul", attrs={"trans_b": False}))
        G.addrule(g, G.GraphRule("v", ["u"], "gelu", attrs={"approx": "sigmoid"}))
    y0, _, _ = _run(build, False, "v")
    y1, fused, g = _run(build, True, "v")
    assert fused == {"v": "fused_linear_gelu"} and "u" not in g.nodes["default"]
    ref = oracle.linear(x, W, trans_w=False, act="sigmoid")
    check(y0, ref)
    check(y1, ref)


@pytest.mark.parametrize("rows,dtype", [(64, torch.float32), (16, torch.bfloat16)])
def test_layernorm_linear_compiles_to_the_fused_op(rows, dtype):
    rng = np.random.default_rng(rows)
    d, n = 512, 384
    x = rng.standard_normal((rows, d)).astype(np.float32)
    gm = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    bt = (0.1 * rng.standard_normal(d)).astype(np.float32)
    W = oracle.bf16_round((0.05 * rng.standard_normal((n, d))).astype(np.float32))
    b = (0.1 * rng.standard_normal(n)).astype(np.float32)

    def build(G, g):
        G.set_(g, "x", torch.from_numpy(x).to(dtype))
        G.set_(g, "g", gm, is_param=True)
        G.set_(g, "b", bt, is_param=True)
        G.set_(g, "W", W, is_param=True)
        G.set_(g, "bw", b, is_param=True)
        G.addrule(g, G.GraphRule("h", ["x", "g", "b"], "layernorm", attrs={"eps": 1e-5}))
        G.addrule(g, G.GraphRule("y", ["h", "W", "bw"], "linear"))
    y0, _, _ = _run(build, False, "y")
    y1, fused, _ = _run(build, True, "y")
    assert fused == {"y": "fused_layernorm_linear"}
    xin = torch.from_numpy(x).to(dtype).float().numpy()
    h, _, _ = oracle.layernorm(xin, gm, bt, 1e-5)
    ref = oracle.linear(oracle.bf16_round(h), W, b)
    check(y0, ref)
    check(y1, ref)
    if dtype == torch.float32:
        # the fused op's LayerNorm writes bf16 directly, the same values the
        # unfused :linear gets by converting the fp32 LayerNorm output
        np.testing.assert_array_equal(y0, y1)


def test_naive_attention_compiles_to_flash_attn():
    rng = np.random.default_rng(3)
    S, D = 256, 64
    q, k, v = (oracle.bf16_round(rng.standard_normal((S, D)).astype(np.float32)) for _ in range(3))

    def build(G, g):
        for name, a in (("q", q), ("k", k), ("v", v)):
            G.set_(g, name, a)
        G.addrule(g, G.GraphRule("sc", ["q", "k"], "matmul", attrs={"trans_b": True}))
        G.addrule(g, G.GraphRule("sk", ["sc"], "scale_mask", attrs={"d_head": D}))
        G.addrule(g, G.GraphRule("pr", ["sk"], "softmax"))
        G.addrule(g, G.GraphRule("ao", ["pr", "v"], "matmul"))
    y0, _, _ = _run(build, False, "ao")
    y1, fused, g = _run(build, True, "ao")
    assert fused == {"ao": "flash_attn"} and set(g.rules["default"]) == {"ao"}
    ref, _, _ = oracle.attn_simple(q, k, v, D, causal=True)
    check(y0, ref)
    check(y1, ref)


def test_linear_add_compiles_to_the_residual_gemm():
    rng = np.random.default_rng(4)
    x = oracle.bf16_round(rng.standard_normal((96, 256)).astype(np.float32))
    W = oracle.bf16_round((0.05 * rng.standard_normal((128, 256))).astype(np.float32))
    b = (0.1 * rng.standard_normal(128)).astype(np.float32)
    r = rng.standard_normal((96, 128)).astype(np.float32)

    def build(G, g):
        G.set_(g, "x", x)
        G.set_(g, "W", W, is_param=True)
        G.set_(g, "b", b, is_param=True)
        G.set_(g, "r", r)
        G.addrule(g, G.GraphRule("y", ["x", "W", "b"], "linear"))
        G.addrule(g, G.GraphRule("z", ["r", "y"], "add"))
    y0, _, _ = _run(build, False, "z")
    y1, fused, _ = _run(build, True, "z")
    assert fused == {"z": "fused_linear_residual"}
    ref = oracle.linear(x, W, b, residual=r)
    check(y0, ref)
    check(y1, ref)


def test_pooled_plan_reuses_buffers_and_matches_demand():
    """A compiled plan run with its buffer pool gives the bits of an unpooled
    demand; intermediates return their buffers (value None, invalid), the
    output stays, and a second run takes every buffer from the pool."""
    C, G = _mods()
    rng = np.random.default_rng(6)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    gm = np.ones(256, np.float32)
    bt = np.zeros(256, np.float32)
    W1 = (0.05 * rng.standard_normal((512, 256))).astype(np.float32)
    W2 = (0.05 * rng.standard_normal((256, 512))).astype(np.float32)

    def build(G, g):
        G.set_(g, "x", x)
        for name, a in (("g", gm), ("b", bt), ("W1", W1), ("W2", W2)):
            G.set_(g, name, a, is_param=True)
        G.addrule(g, G.GraphRule("h", ["x", "g", "b"], "layernorm"))
        G.addrule(g, G.GraphRule("u", ["h", "W1"], "linear"))
        G.addrule(g, G.GraphRule("v", ["u"], "gelu", attrs={"approx": "tanh"}))
        G.addrule(g, G.GraphRule("y", ["v", "W2"], "linear"))
        G.addrule(g, G.GraphRule("z", ["y", "x"], "add"))
    ref, _, _ = _run(build, True, "z")           # compiled, unpooled demand
    g = G.NeuroGraph()
    build(G, g)
    plan = C.compile(g, C.CompilerConfig(training=False))
    assert plan.fused_ops == {"u": "fused_layernorm_linear", "z": "fused_linear_residual"}
    out = plan(g, "z").cpu().numpy()
    np.testing.assert_array_equal(out, ref)
    ns = g.nodes["default"]
    computed = [s for s in plan.memory_plan.order if s in g.rules["default"] and s != "z"]
    assert computed and all(ns[s].value is None and not ns[s].valid for s in computed)
    assert ns["z"].valid and ns["x"].value is not None
    st = plan.pool.stats()
    G.set_(g, "x", x)                               # invalidates everything downstream
    out2 = plan(g, "z").cpu().numpy()
    np.testing.assert_array_equal(out2, ref)
    st2 = plan.pool.stats()
    # the intermediates' buffers come back from the pool; the kept output's
    # own buffer is reused in place
    assert st2["allocs"] == st["allocs"] and st2["hits"] == st["hits"] + len(computed)


def test_add_op_broadcasts_like_the_reference():
    """:add on the library kernel: same shapes, a vector per column
    (preferred when both lengths match), a vector per row, and the vector
    first — each the fp32 sums NumPy gives, bit for bit."""
    _, G = _mods()
    rng = np.random.default_rng(11)
    a = rng.standard_normal((6, 9)).astype(np.float32)
    sq = rng.standard_normal((5, 5)).astype(np.float32)
    cases = {
        "same": (a, rng.standard_normal((6, 9)).astype(np.float32)),
        "per_col": (a, rng.standard_normal(9).astype(np.float32)),
        "per_row": (a, rng.standard_normal(6).astype(np.float32)),
        "square_prefers_cols": (sq, rng.standard_normal(5).astype(np.float32)),
    }
    for name, (x, y) in cases.items():
        for first, second in ((x, y), (y, x)):
            g = G.NeuroGraph()
            G.set_(g, "p", first)
            G.set_(g, "q", second)
            G.addrule(g, G.GraphRule("z", ["p", "q"], "add"))
            z = G.demand(g, "z").cpu().numpy()
            m, v = (first, second) if first.ndim == 2 else (second, first)
            if v.ndim == 1 and v.shape[0] == m.shape[1]:
                ref = m + v.reshape(1, -1)
            elif v.ndim == 1:
                ref = m + v.reshape(-1, 1)
            else:
                ref = m + v
            np.testing.assert_array_equal(z, ref, err_msg=name)


def test_add_op_matrix_broadcasts():
    """:add of a matrix and a (1, cols) row, a (rows, 1) column or a (1, 1)
    value — the reference's general broadcast branch (src/dispatch.jl:409-410),
    which its compiler tests use for a (1, 5) bias — each the fp32 sums NumPy
    gives, bit for bit."""
    _, G = _mods()
    rng = np.random.default_rng(12)
    a = rng.standard_normal((6, 9)).astype(np.float32)
    for shape in ((1, 9), (6, 1), (1, 1)):
        b = rng.standard_normal(shape).astype(np.float32)
        g = G.NeuroGraph()
        G.set_(g, "p", a)
        G.set_(g, "q", b)
        G.addrule(g, G.GraphRule("z", ["p", "q"], "add"))
        z = G.demand(g, "z").cpu().numpy()
        assert z.shape == a.shape
        np.testing.assert_array_equal(z, a + b, err_msg=str(shape))


def test_reference_matmul_add_rule_with_row_bias():
    """The reference's compiler test of a user rule (:matmul, :add) ->
    :fused_matmul_add with x (4, 3), W (3, 5) and a (1, 5) bias
    (test/test_compiler.jl:34-56): the rule applies, and the compiled plan
    gives the unfused graph's values (the reference's atol 1e-5) and the
    oracle's within the bf16-operand tolerance.  K = 3 runs on the same GEMM
    with the inner dimension zero-padded."""
    C, G = _mods()
    rng = np.random.default_rng(13)
    x = oracle.bf16_round(rng.standard_normal((4, 3)).astype(np.float32))
    W = oracle.bf16_round(rng.standard_normal((3, 5)).astype(np.float32))
    b = rng.standard_normal((1, 5)).astype(np.float32)

    def build(G, g):
        G.set_(g, "x", x, is_param=True)
        G.set_(g, "W", W)
        G.set_(g, "b", b)
        G.addrule(g, G.GraphRule("h", ["x", "W"], "matmul"))
        G.addrule(g, G.GraphRule("z", ["h", "b"], "add"))
    rule = C.RewriteRule("t_matmul_add", ("matmul", "add"), "fused_matmul_add", cost_delta=0.2)
    g = G.NeuroGraph()
    build(G, g)
    n_before = len(g.rules["default"])
    plan = C.compile(g, C.CompilerConfig(rules=[rule], training=False))
    assert len(g.rules["default"]) < n_before
    assert g.rules["default"]["z"].op == "fused_matmul_add" and len(plan.fused_ops) == 1
    out_fused = plan(g, "z").cpu().numpy()
    gref = G.NeuroGraph()
    build(G, gref)
    out_ref = G.demand(gref, "z", ctx_store=G.CtxStore()).cpu().numpy()
    np.testing.assert_allclose(out_fused, out_ref, atol=1e-5, rtol=0)
    check(out_fused, oracle.linear(x, W, b.reshape(-1), trans_w=False))


def test_multihead_layer_runs_unfused_and_folded():
    """The graph MultiHeadFlashAttention builds (src/flash_attention.jl:232-256:
    projections, per head three :slice_cols and a causal :flash_attn,
    :hcat_heads, output projection) runs as written — the slices and the
    concatenation as device copies — and compiled, where the layer folds
    into one strided :flash_attention; both match the oracle."""
    rng = np.random.default_rng(14)
    S, H, D = 130, 4, 64
    d = H * D
    x = oracle.bf16_round(rng.standard_normal((S, d)).astype(np.float32))
    Ws = {n: oracle.bf16_round((0.06 * rng.standard_normal((d, d))).astype(np.float32))
          for n in ("Wq", "Wk", "Wv", "Wo")}

    def build(G, g):
        G.set_(g, "x", x)
        for n, w in Ws.items():
            G.set_(g, n, w, is_param=True)
        heads = []
        for p in "qkv":
            G.addrule(g, G.GraphRule(f"a_{p}", ["x", f"W{p}"], "linear"))
        for h in range(H):
            for p in "qkv":
                G.addrule(g, G.GraphRule(f"a_{p}_h{h}", [f"a_{p}"], "slice_cols",
                                         attrs={"start_col": h * D + 1, "end_col": (h + 1) * D}))
            G.addrule(g, G.GraphRule(f"a_ao_h{h}", [f"a_q_h{h}", f"a_k_h{h}", f"a_v_h{h}"],
                                     "flash_attn", attrs={"d_head": D, "causal": True}))
            heads.append(f"a_ao_h{h}")
        G.addrule(g, G.GraphRule("a_concat", heads, "hcat_heads"))
        G.addrule(g, G.GraphRule("a_output", ["a_concat", "Wo"], "linear"))
    y0, _, _ = _run(build, False, "a_output")
    y1, fused, g = _run(build, True, "a_output")
    assert fused == {"a_concat": "flash_attention"}
    assert g.rules["default"]["a_concat"].inputs == ["a_q", "a_k", "a_v"]
    proj = {p: oracle.linear(x, Ws[f"W{p}"]) for p in "qkv"}
    cat = np.zeros((S, d), np.float32)
    for h in range(H):
        sl = slice(h * D, (h + 1) * D)
        o, _, _ = oracle.attn_simple(*(oracle.bf16_round(proj[p][:, sl]) for p in "qkv"), D,
                                     causal=True)
        cat[:, sl] = o
    ref = oracle.linear(oracle.bf16_round(cat), Ws["Wo"])
    check(y0, ref)
    check(y1, ref)
    np.testing.assert_allclose(y0, y1, atol=2e-3, rtol=0)
