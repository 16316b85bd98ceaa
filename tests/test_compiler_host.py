"""Host tests of the rewrite-rule compiler (no GPU: graphs carry no values,
only rules).  The matching and application logic follows the reference's
scan_graph / _apply_fusion! (src/compiler_rules.jl:575-623,
src/compiler.jl:16-66)."""
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

def test_liveness_and_slots_of_a_chain():
    """x -> a -> b -> c, plus d = f(a, c): a lives until d; b's slot is free
    again when c starts only if b's last use is before c's first step."""
    from neurodsl_b200 import liveness as L
    g = _graph(["x", "W"])
    _rule(g, "a", ["x", "W"], "matmul")
    _rule(g, "b", ["a"], "gelu")
    _rule(g, "c", ["b"], "gelu")
    _rule(g, "d", ["a", "c"], "add")
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
