"""CPU tests of the operator-API mirror (no GPU): topo order, invalidation,
demand! semantics, register_op! fall-through, shape inference and error
behaviour, modelled on the reference's test/test_graph_api.jl:4-36.  The
executor is exercised with ops registered by the test on a host device tag,
so no kernel is called."""
import pytest
import torch

from neurodsl_b200 import graph as G
from neurodsl_b200._lib import NeuroDSLError


class HostDevice:
    torch_device = torch.device("cpu")


def _host_copy(dev, out, inputs, attrs, out_sym, nd, ctx):
    out.copy_(inputs[0])


def host_graph():
    return G.NeuroGraph(device=HostDevice())


@pytest.fixture(autouse=True)
def _restore_custom_ops():
    # the built-in :identity runs a library kernel; host graphs use this copy
    saved = dict(G.CUSTOM_OPS)
    G.register_op("host_copy", _host_copy)
    yield
    G.CUSTOM_OPS.clear()
    G.CUSTOM_OPS.update(saved)


def test_set_and_demand_with_custom_op():
    calls = []

    def double(dev, out, inputs, attrs, out_sym, nd, ctx):
        calls.append(out_sym)
        out.copy_(inputs[0] * attrs.get("factor", 2.0))
        if ctx is not None:
            ctx[out_sym] = {"x": inputs[0]}

    G.register_op("twice", double)
    g = host_graph()
    G.set_(g, "x", torch.ones(2, 3))
    G.addrule(g, G.GraphRule("y", ["x"], "twice", {"factor": 3.0}))
    G.addrule(g, G.GraphRule("z", ["y"], "twice"))
    ctx = G.CtxStore()
    z = G.demand(g, "z", ctx_store=ctx)
    assert torch.equal(z, torch.full((2, 3), 6.0))
    assert calls == ["y", "z"] and set(ctx) == {"y", "z"}
    # valid nodes are not recomputed
    G.demand(g, "z")
    assert calls == ["y", "z"]
    # set! invalidates downstream only
    G.set_(g, "x", torch.full((2, 3), 2.0))
    assert not g.nodes["default"]["y"].valid and not g.nodes["default"]["z"].valid
    assert torch.equal(G.demand(g, "z"), torch.full((2, 3), 12.0))
    assert calls == ["y", "z", "y", "z"]


def test_output_buffer_is_reused_in_place():
    def fill(dev, out, inputs, attrs, out_sym, nd, ctx):
        out.copy_(inputs[0] + 1)

    G.register_op("inc", fill)
    g = host_graph()
    G.set_(g, "x", torch.zeros(4))
    G.addrule(g, G.GraphRule("y", ["x"], "host_copy"))
    G.addrule(g, G.GraphRule("w", ["x"], "inc"))
    y1 = G.demand(g, "w")
    ptr = y1.data_ptr()
    G.set_(g, "x", torch.ones(4))
    y2 = G.demand(g, "w")
    assert y2.data_ptr() == ptr and torch.equal(y2, torch.full((4,), 2.0))


def test_topo_order_and_namespaces():
    g = host_graph()
    G.set_(g, "a", torch.zeros(1))
    G.addrule(g, G.GraphRule("b", ["a"], "host_copy"))
    G.addrule(g, G.GraphRule("c", ["b", "a"], "add"))
    order = G.topo_order(g)
    assert order.index("a") < order.index("b") < order.index("c")
    G.set_(g, "a", torch.zeros(1), namespace="other")
    assert "b" not in g.nodes["other"]


def test_cycle_detected():
    g = host_graph()
    G.addrule(g, G.GraphRule("p", ["q"], "host_copy"))
    G.addrule(g, G.GraphRule("q", ["p"], "host_copy"))
    with pytest.raises(NeuroDSLError):
        G.topo_order(g)


def test_unknown_op_raises_like_reference():
    g = host_graph()
    G.set_(g, "x", torch.zeros(2, 2))
    G.addrule(g, G.GraphRule("y", ["x"], "gelu_unknown"))
    with pytest.raises(NeuroDSLError, match="register_op"):
        G.demand(g, "y")


def test_missing_node_raises():
    g = host_graph()
    with pytest.raises(NeuroDSLError):
        G.demand(g, "nope")


def test_shape_inference_for_b200_ops():
    X = torch.zeros(128, 1024)
    W = torch.zeros(4096, 1024)
    assert G._infer_output_shape("fused_linear_gelu", [X, W], {"trans_b": True}) == (128, 4096)
    assert G._infer_output_shape("fused_linear_gelu", [X, W.T], {}) == (128, 4096)
    assert G._infer_output_shape("linear", [X, W], {}) == (128, 4096)
    assert G._infer_output_shape("fused_linear_residual", [X, W], {}) == (128, 4096)
    assert G._infer_output_shape("flash_attention", [X, X, X], {"n_heads": 16}) == (128, 1024)
    assert G._infer_output_shape("layernorm", [X], {}) == (128, 1024)
    assert G._infer_output_shape("hcat_heads", [torch.zeros(5, 64)] * 3, {}) == (5, 192)
    with pytest.warns(UserWarning):
        assert G._infer_output_shape("no_such_op", [X], {}) == (128, 1024)


def test_shape_inference_for_unfused_and_compiled_ops():
    """The unfused ops keep their input's shape; :add takes the matrix's shape
    whichever operand the vector is; the compiled LayerNorm + linear takes the
    weight's output dimension in either orientation; a fused (S, 3d) QKV
    projection gives (S, d)."""
    X = torch.zeros(64, 512)
    for op in ("gelu", "scale_mask", "softmax", "identity"):
        assert G._infer_output_shape(op, [X], {}) == (64, 512)
    v = torch.zeros(512)
    assert G._infer_output_shape("add", [X, v], {}) == (64, 512)
    assert G._infer_output_shape("add", [v, X], {}) == (64, 512)
    assert G._infer_output_shape("add", [X, X], {}) == (64, 512)
    g, b = torch.zeros(512), torch.zeros(512)
    W = torch.zeros(384, 512)
    assert G._infer_output_shape("fused_layernorm_linear", [X, g, b, W],
                                 {"trans_b": True}) == (64, 384)
    assert G._infer_output_shape("fused_layernorm_linear", [X, g, b, W.T], {}) == (64, 384)
    assert G._infer_output_shape("flash_attention", [torch.zeros(128, 3 * 512)],
                                 {"n_heads": 8}) == (128, 512)
    assert G._infer_output_shape("slice_cols", [X], {"start_col": 65, "end_col": 128}) == (64, 64)
    assert G._infer_output_shape("matmul", [X, W], {"trans_b": True}) == (64, 384)
    assert G._infer_output_shape("matmul", [X, W.T], {}) == (64, 384)


def test_b200_ops_registered():
    for op in ("flash_attn", "flash_attention", "kv_decode_attn", "fused_linear_gelu",
               "fused_linear_residual", "layernorm", "add", "gelu", "scale_mask", "softmax",
               "fused_layernorm_linear"):
        assert op in G.CUSTOM_OPS


def test_aliased_output_goes_through_a_kept_side_buffer():
    """An output buffer that is also an input (the buffer pool can hand out
    such a pair) is redirected to aux_data[:_alias_buf], kept for the next
    call of the same shape and dtype and replaced when either changes
    (src/dispatch.jl:220-231)."""
    node = G.GraphNode("y", None)
    x = torch.zeros(4, 8)
    other = torch.zeros(4, 8)
    buf, aliased = G._alias_safe(other, node, [x])
    assert buf is other and not aliased and "_alias_buf" not in node.aux_data
    buf, aliased = G._alias_safe(x, node, [x, other])
    assert aliased and buf is not x and buf.shape == x.shape
    assert buf.data_ptr() != x.data_ptr()
    again, _ = G._alias_safe(x, node, [x])
    assert again is buf                                   # reused
    xb = torch.zeros(4, 8, dtype=torch.bfloat16)
    third, aliased = G._alias_safe(xb, node, [xb])
    assert aliased and third is not buf and third.dtype == torch.bfloat16


def test_graph_api_like_the_reference():
    """test/test_graph_api.jl:4-36 restated: node / is_backpropable / params,
    topological order, invalidation on set_, and namespace isolation with
    activate."""
    g = G.NeuroGraph(namespace="t", device=HostDevice())
    G.set_(g, "x", torch.ones(2, 2), is_param=True, namespace="t")
    G.set_(g, "d", torch.tensor([1, 2]), atom_type=G.Datom, namespace="t")
    assert G.is_backpropable(G.node(g, "x", namespace="t"))
    assert not G.is_backpropable(G.node(g, "d", namespace="t"))
    assert len(G.params(g, namespace="t")) == 1
    G.set_(g, "W", torch.ones(2, 2), is_param=True, namespace="t")
    G.addrule(g, G.GraphRule("out", ["x", "W"], "matmul", attrs={"trans_b": False},
                             namespace="t"))
    order = G.topo_order(g, "t")
    assert "out" in order and order.index("x") < order.index("out")
    G.set_(g, "x", torch.zeros(2, 2), namespace="t")
    assert not G.node(g, "out", namespace="t").valid
    G.activate(g, "other")
    assert g.active_ns == "other" and set(G.namespaces(g)) == {"t", "other"}
    G.set_(g, "x", torch.ones(2, 2), namespace="other")
    assert "out" not in g.nodes["other"]
    with pytest.raises(NeuroDSLError):
        G.node(g, "out")                      # the active namespace has no :out


def test_defop_decorator_registers_an_op():
    @G.defop("twice_plus_one")
    def _op(dev, out, inputs, attrs, out_sym, nd, ctx):
        out.copy_(2 * inputs[0] + 1)
    g = host_graph()
    G.set_(g, "x", torch.arange(4.0).reshape(2, 2))
    G.addrule(g, G.GraphRule("y", ["x"], "host_copy"))
    G.addrule(g, G.GraphRule("z", ["y"], "twice_plus_one"))
    assert G.CUSTOM_OPS["twice_plus_one"] is _op
    with pytest.warns(UserWarning):
        z = G.demand(g, "z")
    torch.testing.assert_close(z, 2 * torch.arange(4.0).reshape(2, 2) + 1)


def test_on_change_callback_gets_graph_symbol_and_namespace():
    """A node's on_change callback fires when an upstream set_ invalidates it,
    with the reference's (g, sym, ns) arguments (src/graph_api.jl:52-54)."""
    g = host_graph()
    G.set_(g, "x", torch.ones(2, 2))
    G.addrule(g, G.GraphRule("y", ["x"], "host_copy"))
    seen = []
    g.nodes["default"]["y"].on_change = lambda gg, sym, ns: seen.append((gg, sym, ns))
    G.set_(g, "x", torch.zeros(2, 2))
    assert seen == [(g, "y", "default")]


def test_watchers_are_invalidated_with_what_they_observe():
    g = host_graph()
    G.set_(g, "x", torch.ones(2, 2))
    G.set_(g, "stats", torch.zeros(1))
    G.addrule(g, G.GraphRule("y", ["x"], "host_copy"))
    G.demand(g, "y")
    G.watch(g, "stats", "y")
    assert g.nodes["default"]["stats"].valid
    G.set_(g, "x", torch.zeros(2, 2))
    assert not g.nodes["default"]["y"].valid and not g.nodes["default"]["stats"].valid
    assert g.nodes["default"]["x"].valid


def test_graph_summary_counts_per_namespace(capsys):
    g = host_graph()
    G.set_(g, "x", torch.ones(2, 2))
    G.set_(g, "W", torch.ones(2, 2), is_param=True)
    G.addrule(g, G.GraphRule("y", ["x", "W"], "matmul"))
    text = G.graph_summary(g)
    assert "[:default]  nodes=3  rules=1  params=1" in text
    assert "Device    : CPU" in text and text in capsys.readouterr().out
