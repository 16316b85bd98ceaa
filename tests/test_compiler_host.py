"""Host tests of the rewrite-rule compiler (no GPU): rule matching on graphs
that carry no values, and recompilation and pooling on graphs whose ops the
test registers on a CPU device tag.  The logic follows the reference's
scan_graph / _apply_fusion! / recompile! / plan call
(src/compiler_rules.jl:575-623, src/compiler.jl:16-240)."""
import pytest

pytest.importorskip("torch")

from neurodsl_b200 import compiler as C  # noqa: E402
from neurodsl_b200 import graph as G  # noqa: E402


def _graph(inputs):
    g = G.NeuroGraph()
    for name in inputs:
        g.nodes["default"][name] = G.GraphNode(name, None, is_param=True)
    return g


def _rule(g, out, ins, op, **attrs):
    G.addrule(g, G.GraphRule(out, list(ins), op, attrs=dict(attrs)))


def test_layernorm_linear_gelu_chain():
    """LN -> linear -> gelu: the higher-scored LN+linear fusion applies first,
    which leaves the linear+gelu match stale (its first node now has another
    op) — the gelu stays."""
    g = _graph(["x", "g", "b", "W", "bw"])
    _rule(g, "h", ["x", "g", "b"], "layernorm", eps=1e-6)
    _rule(g, "y", ["h", "W", "bw"], "linear")
    _rule(g, "z", ["y"], "gelu", approx="tanh")
    plan = C.compile(g, C.CompilerConfig(training=False))
    assert plan.fused_ops == {"y": "fused_layernorm_linear"}
    r = g.rules["default"]["y"]
    assert r.op == "fused_layernorm_linear"
    assert r.inputs == ["x", "g", "b", "W", "bw"]
    assert r.attrs == {"eps": 1e-6, "trans_b": True}
    assert "h" not in g.nodes["default"] and "h" not in g.rules["default"]
    assert g.rules["default"]["z"].op == "gelu"
    assert plan.order.index("y") < plan.order.index("z")


def test_matmul_gelu_and_linear_residual():
    g = _graph(["x", "W1", "W2", "b2", "r"])
    _rule(g, "u", ["x", "W1"], "matmul", trans_b=False)
    _rule(g, "v", ["u"], "gelu", approx="sigmoid")
    _rule(g, "w", ["v", "W2", "b2"], "linear")
    _rule(g, "out", ["r", "w"], "add")
    plan = C.compile(g, C.CompilerConfig(training=False))
    assert plan.fused_ops == {"v": "fused_linear_gelu", "out": "fused_linear_residual"}
    v = g.rules["default"]["v"]
    assert (v.op, v.inputs, v.attrs) == ("fused_linear_gelu", ["x", "W1"],
                                         {"trans_b": False, "approx": "sigmoid"})
    o = g.rules["default"]["out"]
    # external inputs in rule order: the linear's, then the add's other operand
    assert (o.op, o.inputs) == ("fused_linear_residual", ["v", "W2", "b2", "r"])


def test_naive_attention_becomes_flash_attn():
    g = _graph(["q", "k", "v"])
    _rule(g, "sc", ["q", "k"], "matmul", trans_b=True)
    _rule(g, "sk", ["sc"], "scale_mask", d_head=64)
    _rule(g, "pr", ["sk"], "softmax")
    _rule(g, "ao", ["pr", "v"], "matmul")
    plan = C.compile(g, C.CompilerConfig(training=False))
    assert plan.fused_ops == {"ao": "flash_attn"}
    r = g.rules["default"]["ao"]
    assert r.op == "flash_attn" and r.inputs == ["q", "k", "v"]
    assert r.attrs["d_head"] == 64 and r.attrs["causal"] is True
    assert set(g.rules["default"]) == {"ao"}


def test_attention_variants_that_do_not_match():
    # keys not transposed in the score matmul
    g = _graph(["q", "k", "v"])
    _rule(g, "sc", ["q", "k"], "matmul", trans_b=False)
    _rule(g, "sk", ["sc"], "scale_mask", d_head=64)
    _rule(g, "pr", ["sk"], "softmax")
    _rule(g, "ao", ["pr", "v"], "matmul")
    assert C.compile(g, C.CompilerConfig(training=False)).fused_ops == {}
    # probabilities as the second operand of the last matmul
    g = _graph(["q", "k", "v"])
    _rule(g, "sc", ["q", "k"], "matmul", trans_b=True)
    _rule(g, "sk", ["sc"], "scale_mask", d_head=64)
    _rule(g, "pr", ["sk"], "softmax")
    _rule(g, "ao", ["v", "pr"], "matmul")
    assert C.compile(g, C.CompilerConfig(training=False)).fused_ops == {}


def test_shared_intermediate_blocks_fusion():
    """An intermediate with two consumers cannot be fused away."""
    g = _graph(["x", "W"])
    _rule(g, "u", ["x", "W"], "matmul", trans_b=True)
    _rule(g, "v", ["u"], "gelu")
    _rule(g, "w", ["u"], "gelu")
    assert C.scan_graph(g, C.B200_RULES) == []
    assert C.compile(g, C.CompilerConfig(training=False)).fused_ops == {}


def test_training_refuses_inference_only_fusions():
    """Like the reference's training guard (src/compiler.jl:19-24): no fused
    B200 op has a backward rule."""
    g = _graph(["x", "W"])
    _rule(g, "u", ["x", "W"], "matmul", trans_b=True)
    _rule(g, "v", ["u"], "gelu")
    assert len(C.scan_graph(g)) == 1
    assert C.compile(g, C.CompilerConfig(training=True)).fused_ops == {}
    assert g.rules["default"]["v"].op == "gelu"


def test_two_input_layernorm_is_left_alone():
    g = _graph(["x", "g", "W"])
    _rule(g, "h", ["x", "g"], "layernorm")
    _rule(g, "y", ["h", "W"], "matmul")
    assert C.compile(g, C.CompilerConfig(training=False)).fused_ops == {}


def test_failing_condition_makes_rule_inapplicable():
    def boom(g, chain, ns):
        raise RuntimeError("condition error")
    rule = C.RewriteRule("x", ("matmul", "gelu"), "fused_linear_gelu", condition=boom)
    g = _graph(["x", "W"])
    _rule(g, "u", ["x", "W"], "matmul")
    _rule(g, "v", ["u"], "gelu")
    assert C.scan_graph(g, [rule]) == []


# ------------------------------------------------------------ memory plan ---

def _atom_chain(atom):
    g = _graph(["x", "W"])
    for out, ins, op in (("a", ["x", "W"], "matmul"), ("b", ["a"], "gelu"),
                         ("c", ["b"], "gelu"), ("d", ["a", "c"], "add")):
        G.addrule(g, G.GraphRule(out, ins, op, atom_type=atom))
    return g


def test_liveness_of_a_backpropagable_chain_extends_to_the_end():
    """src/liveness.jl:101-108: parameters and backpropagable (Quantom, the
    default atom type) nodes live to the last step of the order, whatever
    their last reader."""
    from neurodsl_b200 import liveness as L
    g = _atom_chain(G.Quantom)
    order = G.topo_order(g)
    n = len(order)
    live = L.compute_liveness(g)
    pos = {s: i + 1 for i, s in enumerate(order)}
    for s in ("a", "b", "c", "d"):
        assert live[s] == L.LivenessInterval(pos[s], n), s
    assert live["W"].last_use == n
    # every intermediate alive at once: one slot each
    slot = L.greedy_interval_coloring(live, order)
    assert len({slot[s] for s in ("a", "b", "c", "d")}) == 4


def test_liveness_and_slots_of_a_chain():
    """Datom chain x -> a -> b -> c, plus d = f(a, c): a lives until d; b's
    slot is free again when c starts only if b's last use is before c's first
    step."""
    from neurodsl_b200 import liveness as L
    g = _atom_chain(G.Datom)
    order = G.topo_order(g)
    live = L.compute_liveness(g)
    pos = {s: i + 1 for i, s in enumerate(order)}
    assert live["a"] == L.LivenessInterval(pos["a"], pos["d"])
    assert live["b"] == L.LivenessInterval(pos["b"], pos["c"])
    assert live["W"].last_use == len(order)          # parameter: to the end
    slot = L.greedy_interval_coloring(live, order)
    # nodes alive at the same step never share a slot
    for s in order:
        for t in order:
            if s < t and slot[s] == slot[t]:
                a, b = live[s], live[t]
                assert a.last_use < b.first_use or b.last_use < a.first_use
    plan = L.plan_memory(g)
    assert plan.n_slots == max(slot.values()) and plan.order == order


def test_buffer_pool_buckets_by_shape_and_dtype():
    import torch
    from neurodsl_b200 import liveness as L
    pool = L.BufferPool(torch.device("cpu"))
    a = pool.acquire((4, 8))
    pool.release(a)
    assert pool.acquire((4, 8)) is a                 # reused
    b = pool.acquire((4, 8), torch.bfloat16)         # other dtype: a new buffer
    assert b is not a and b.dtype == torch.bfloat16
    assert pool.stats() == {"allocs": 2, "hits": 1, "hit_rate_pct": 33.3}


def test_compile_attaches_a_memory_plan():
    g = _graph(["x", "W"])
    _rule(g, "u", ["x", "W"], "matmul", trans_b=True)
    _rule(g, "v", ["u"], "gelu")
    plan = C.compile(g, C.CompilerConfig(training=False))
    assert plan.memory_plan is not None and plan.pool is not None
    assert set(plan.memory_plan.order) == {"x", "W", "v"}


# ------------------------------------- recompilation and pooling semantics ---
# Restatements of the reference's compiler tests (test/test_compiler.jl:147-292)
# on the host: the ops are registered by the test on a CPU device tag, under
# names of its own, so the executor runs without a kernel.

import torch  # noqa: E402


class _HostDevice:
    torch_device = torch.device("cpu")


@pytest.fixture
def cpu_ops():
    saved = dict(G.CUSTOM_OPS)

    def mm(dev, out, ins, attrs, sym, node, ctx):
        out.copy_(ins[0] @ ins[1])

    def addb(dev, out, ins, attrs, sym, node, ctx):
        out.copy_(ins[0] + ins[1])

    def relu(dev, out, ins, attrs, sym, node, ctx):
        out.copy_(torch.relu(ins[0]))

    def mm_add_relu(dev, out, ins, attrs, sym, node, ctx):
        out.copy_(torch.relu(ins[0] @ ins[1] + ins[2]))

    for name, fn in (("t_mm", mm), ("t_addb", addb), ("t_relu", relu),
                     ("t_mm_add_relu", mm_add_relu)):
        G.register_op(name, fn)
    yield
    G.CUSTOM_OPS.clear()
    G.CUSTOM_OPS.update(saved)


def _chain(seed=0):
    """x·W + b, then relu (the reference's build_chain with square operands,
    since the test ops get the first input's shape)."""
    gen = torch.Generator().manual_seed(seed)
    g = G.NeuroGraph(device=_HostDevice())
    G.set_(g, "x", torch.randn(4, 4, generator=gen), is_param=True)
    G.set_(g, "W", torch.randn(4, 4, generator=gen))
    G.set_(g, "b", torch.randn(1, 4, generator=gen))
    _rule(g, "h", ["x", "W"], "t_mm")
    _rule(g, "y", ["h", "b"], "t_addb")
    _rule(g, "z", ["y"], "t_relu")
    return g


def _fusion():
    return C.RewriteRule("t_mar", ("t_mm", "t_addb", "t_relu"), "t_mm_add_relu", cost_delta=0.5)


_quiet_shapes = pytest.mark.filterwarnings("ignore:Shape inference")


@_quiet_shapes
def test_plan_starts_clean_and_set_marks_it_dirty(cpu_ops):
    g = _chain()
    plan = C.compile(g, C.CompilerConfig(rules=[_fusion()], training=False))
    assert g.rules["default"]["z"].op == "t_mm_add_relu"
    assert not C.is_dirty(plan) and plan.n_recompiles == 0
    G.set_(g, "x", torch.randn(4, 4), is_param=True)
    assert C.is_dirty(plan)


@_quiet_shapes
def test_recompile_is_a_no_op_on_a_clean_plan(cpu_ops):
    g = _chain()
    plan = C.compile(g, C.CompilerConfig(rules=[_fusion()], training=False))
    C.recompile(plan, g)
    C.recompile(plan, g)
    assert plan.n_recompiles == 0


@_quiet_shapes
def test_calling_a_dirty_plan_recompiles_and_recomputes(cpu_ops):
    g = _chain()
    plan = C.compile(g, C.CompilerConfig(rules=[_fusion()], training=False))
    plan(g, "z")
    assert plan.n_recompiles == 0
    x_new = torch.randn(4, 4, generator=torch.Generator().manual_seed(9))
    G.set_(g, "x", x_new, is_param=True)
    assert C.is_dirty(plan)
    out = plan(g, "z").clone()
    assert plan.n_recompiles == 1 and not C.is_dirty(plan)
    ref = G.NeuroGraph(device=_HostDevice())
    G.set_(ref, "x", x_new)
    G.set_(ref, "W", g.nodes["default"]["W"].value)
    G.set_(ref, "b", g.nodes["default"]["b"].value)
    _rule(ref, "h", ["x", "W"], "t_mm")
    _rule(ref, "y", ["h", "b"], "t_addb")
    _rule(ref, "z", ["y"], "t_relu")
    torch.testing.assert_close(out, G.demand(ref, "z", ctx_store=G.CtxStore()), atol=1e-5,
                               rtol=0)


@_quiet_shapes
def test_recompile_picks_up_a_rule_added_after_compilation(cpu_ops):
    """A graph that gained nodes since the last compilation is compiled
    afresh on the next call (src/compiler.jl:146-158)."""
    g = _chain()
    plan = C.compile(g, C.CompilerConfig(rules=[_fusion()], training=False))
    _rule(g, "w", ["z"], "t_relu")
    plan.dirty_nodes.add("z")
    out = plan(g, "w")
    assert plan.n_recompiles == 1 and "w" in plan.order
    ns = g.nodes["default"]
    x, W, b = ns["x"].value, ns["W"].value, ns["b"].value
    torch.testing.assert_close(out, torch.relu(x @ W + b), atol=1e-5, rtol=0)


def _mlp(atom):
    gen = torch.Generator().manual_seed(3)
    g = G.NeuroGraph(device=_HostDevice())
    G.set_(g, "x", torch.randn(6, 6, generator=gen), is_param=True)
    for w in ("W1", "W2", "W3"):
        G.set_(g, w, torch.randn(6, 6, generator=gen), is_param=True)
    for out, ins, op in (("h1", ["x", "W1"], "t_mm"), ("h2", ["h1"], "t_relu"),
                         ("h3", ["h2", "W2"], "t_mm"), ("h4", ["h3"], "t_relu"),
                         ("out", ["h4", "W3"], "t_mm")):
        G.addrule(g, G.GraphRule(out, ins, op, atom_type=atom))
    return g


@_quiet_shapes
def test_inference_pooling_recycles_intermediates(cpu_ops):
    g = _mlp(G.Datom)
    plan = C.compile(g, C.CompilerConfig(rules=[], training=False))
    plan(g, "out")
    st = plan.pool.stats()
    assert st["allocs"] + st["hits"] > 0
    assert g.nodes["default"]["h1"].value is None


@_quiet_shapes
def test_training_pooling_keeps_backpropagable_intermediates(cpu_ops):
    g = _mlp(G.Quantom)
    plan = C.compile(g, C.CompilerConfig(rules=[], training=True))
    plan(g, "out")
    assert all(g.nodes["default"][s].value is not None for s in ("h1", "h2", "h3", "h4"))


@_quiet_shapes
def test_params_and_requested_output_never_recycled(cpu_ops):
    for atom, training in ((G.Datom, False), (G.Quantom, True)):
        g = _mlp(atom)
        plan = C.compile(g, C.CompilerConfig(rules=[], training=training))
        plan(g, "out")
        for s in ("W1", "W2", "W3", "out"):
            assert g.nodes["default"][s].value is not None, (s, training)


def test_training_guard_refuses_then_allows_a_made_up_op():
    """test/test_compiler.jl:147-167: a rule into an op without a backward
    rule is refused by default and applied with training=False."""
    made_up = C.RewriteRule("made_up_fusion", ("matmul", "gelu"), "made_up_op_no_grad",
                            cost_delta=0.9)
    g = _graph(["x", "W"])
    _rule(g, "h", ["x", "W"], "matmul")
    _rule(g, "z", ["h"], "gelu")
    C.compile(g, C.CompilerConfig(rules=[made_up]))
    assert g.rules["default"]["z"].op == "gelu"
    g2 = _graph(["x", "W"])
    _rule(g2, "h", ["x", "W"], "matmul")
    _rule(g2, "z", ["h"], "gelu")
    C.compile(g2, C.CompilerConfig(rules=[made_up], training=False))
    assert g2.rules["default"]["z"].op == "made_up_op_no_grad"


def test_cheapest_of_two_alternative_rules_at_one_root():
    """test/test_compiler.jl:294-326: of an sdpa_fusion and a flash_attention
    match at the same root only the cheaper under the cost function stays;
    matches at different roots both stay."""
    g = G.NeuroGraph(device=_HostDevice())
    G.set_(g, "root", torch.randn(8, 8))
    cheap = C.RewriteRule("sdpa_fusion", ("matmul",), "fused_sdpa", cost_delta=0.1)
    dear = C.RewriteRule("flash_attention", ("matmul",), "flash_attention_dummy", cost_delta=0.1)

    def cost_fn(op, shapes, rule_cost_delta=0.0):
        return 1.0 if op == "fused_sdpa" else 100.0
    kept = C.choose_cheapest_alternative(
        g, [C.RuleMatch(cheap, ["root"], "default", 0.1),
            C.RuleMatch(dear, ["root"], "default", 0.1)], cost_fn)
    assert len(kept) == 1 and kept[0].rule.result == "fused_sdpa"
    G.set_(g, "root_b", torch.randn(8, 8))
    kept = C.choose_cheapest_alternative(
        g, [C.RuleMatch(cheap, ["root"], "default", 0.1),
            C.RuleMatch(dear, ["root_b"], "default", 0.1)], cost_fn)
    assert len(kept) == 2


def test_default_cost_model():
    assert C.symbolic_cost("matmul", [(128, 1024), (1024, 4096)]) == 128 * 1024 * 4096 / 1e9
    assert C.symbolic_cost("gelu", [(10, 10)]) == 100 / 1e8
    assert C.symbolic_cost("layernorm", [(10, 10)]) == 100 / 5e7
    assert C.symbolic_cost("flash_attention", [(2048, 64)]) == 2048 * 2048 * 64 / 1e9
    assert C.symbolic_cost("identity", [(10, 10)]) == 0.0
    assert C.default_cost("gelu", [(10, 10)], rule_cost_delta=1.0) == 0.0
    assert C.CompilerConfig().cost_fn is C.default_cost


def _mha_graph(H=4, D=64, order=None, extra_reader=False):
    """The rules MultiHeadFlashAttention adds (src/flash_attention.jl:232-256):
    three bias-free projections, per head three :slice_cols and a causal
    :flash_attn, the :hcat_heads of the heads and the output projection."""
    g = _graph(["x", "Wq", "Wk", "Wv", "Wo"])
    for p in "qkv":
        _rule(g, f"a_{p}", ["x", f"W{p}"], "linear")
    heads = []
    for h in range(H):
        for p in "qkv":
            _rule(g, f"a_{p}_h{h}", [f"a_{p}"], "slice_cols", start_col=h * D + 1,
                  end_col=(h + 1) * D)
        _rule(g, f"a_ao_h{h}", [f"a_q_h{h}", f"a_k_h{h}", f"a_v_h{h}"], "flash_attn", d_head=D,
              causal=True)
        heads.append(f"a_ao_h{h}")
    if order is not None:
        heads = [heads[i] for i in order]
    _rule(g, "a_concat", heads, "hcat_heads")
    _rule(g, "a_output", ["a_concat", "Wo"], "linear")
    if extra_reader:
        _rule(g, "peek", ["a_q_h0"], "gelu")
    return g


def test_multihead_layer_folds_into_flash_attention():
    g = _mha_graph()
    plan = C.compile(g, C.CompilerConfig(training=False))
    r = g.rules["default"]["a_concat"]
    assert (r.op, r.inputs) == ("flash_attention", ["a_q", "a_k", "a_v"])
    assert r.attrs == {"n_heads": 4, "d_head": 64, "causal": True}
    assert plan.fused_ops["a_concat"] == "flash_attention"
    assert not [s for s in g.rules["default"] if "_h" in s]
    assert not [s for s in g.nodes["default"] if "_h" in s]
    assert plan.order.index("a_concat") < plan.order.index("a_output")


def test_multihead_fold_needs_the_layer_exactly():
    # heads concatenated out of order, a slice read elsewhere, training mode
    for g, cfg in ((_mha_graph(order=[1, 0, 2, 3]), C.CompilerConfig(training=False)),
                   (_mha_graph(extra_reader=True), C.CompilerConfig(training=False)),
                   (_mha_graph(), C.CompilerConfig(training=True))):
        C.compile(g, cfg)
        assert g.rules["default"]["a_concat"].op == "hcat_heads"
        assert "a_q_h1" in g.rules["default"]


@_quiet_shapes
def test_memory_planning_like_the_reference(cpu_ops):
    """test/test_runtime_optimizations.jl:20-36: plan_memory! gives at most
    one slot per node and an untouched pool; after invalidate_all! the planned
    demand recomputes the output."""
    from neurodsl_b200 import liveness as L
    g = G.NeuroGraph(device=_HostDevice())
    G.set_(g, "x", torch.rand(2, 2), is_param=True)
    G.set_(g, "w", torch.rand(2, 2), is_param=True)
    _rule(g, "h", ["x", "w"], "t_mm")
    _rule(g, "out", ["h"], "t_relu")
    plan, pool = L.plan_memory_pool(g)
    assert plan.n_slots <= len(plan.order)
    assert pool.n_alloc >= 0 and pool.n_hits == 0
    G.invalidate_all(g)
    assert not g.nodes["default"]["h"].valid and g.nodes["default"]["x"].valid
    val = L.demand_planned(g, "out", plan, pool)
    x, w = g.nodes["default"]["x"].value, g.nodes["default"]["w"].value
    torch.testing.assert_close(val, torch.relu(x @ w))
    assert L.demand_planned(g, "out", plan, pool) is val          # valid: no recompute
    assert L.pool_stats(pool)["allocs"] == 2


def test_rule_names_shared_with_the_reference_keep_its_patterns():
    """src/compiler_config.jl:154-172: linear_gelu_fusion is (:matmul, :gelu)
    and layernorm_linear_fusion is (:layernorm, :matmul), so a caller that
    selects or drops rules by name gets the same fusions."""
    by_name = {r.name: r for r in C.B200_RULES}
    assert by_name["linear_gelu_fusion"].pattern == ("matmul", "gelu")
    assert by_name["linear_gelu_fusion"].result == "fused_linear_gelu"
    assert by_name["layernorm_linear_fusion"].pattern == ("layernorm", "matmul")
    assert by_name["layernorm_linear_fusion"].result == "fused_layernorm_linear"
    assert len(by_name) == len(C.B200_RULES)


def test_compiler_config_fields_of_the_reference():
    """budget bounds the fusions applied, verify_rules warns for unverified
    rules, only the GPU target and the symbolic cost mode are accepted."""
    g = _graph(["x", "W1", "W2"])
    _rule(g, "u", ["x", "W1"], "matmul")
    _rule(g, "v", ["u"], "gelu")
    _rule(g, "w", ["v", "W2"], "matmul")
    _rule(g, "z", ["w"], "gelu")
    assert C.compile(g, C.CompilerConfig(training=False, budget=1)).fused_ops == \
        {"v": "fused_linear_gelu"}
    g = _graph(["x", "W"])
    _rule(g, "u", ["x", "W"], "matmul")
    _rule(g, "v", ["u"], "gelu")
    with pytest.warns(UserWarning, match="linear_gelu_fusion"):
        C.compile(g, C.CompilerConfig(training=False, verify_rules=True))
    with pytest.raises(ValueError):
        C.CompilerConfig(target="cpu")
    with pytest.raises(ValueError):
        C.CompilerConfig(cost_mode="profiled")


@_quiet_shapes
def test_non_incremental_recompilation_is_a_full_compile(cpu_ops):
    g = _chain()
    plan = C.compile(g, C.CompilerConfig(rules=[_fusion()], training=False, incremental=False))
    G.set_(g, "x", torch.randn(4, 4, generator=torch.Generator().manual_seed(5)), is_param=True)
    out = plan(g, "z")
    assert plan.n_recompiles == 1 and not C.is_dirty(plan)
    ns = g.nodes["default"]
    torch.testing.assert_close(out, torch.relu(ns["x"].value @ ns["W"].value + ns["b"].value))


def test_memory_plan_summary():
    from neurodsl_b200 import liveness as L
    g = _graph(["x", "W"])
    _rule(g, "a", ["x", "W"], "matmul")
    _rule(g, "b", ["a"], "gelu")
    _rule(g, "c", ["b"], "gelu")
    plan = L.plan_memory(g)
    text = str(plan)
    assert text.startswith("MemoryPlan:") and f"Slots     : {plan.n_slots}" in text
    assert 1 <= plan.peak_live() <= len(plan.order)
    assert f"Nodes     : {len(plan.order)}" in text and "Reduction : -" in text
