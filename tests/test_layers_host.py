"""Host tests of the layer builders (no GPU): the rules and parameter nodes
each builder adds, named as the reference's layers name them
(src/layers.jl:15-80, src/flash_attention.jl:225-256), and the compiled form
of both multi-head layers — one strided :flash_attention."""
import math

import pytest
import torch

from neurodsl_b200 import compiler as C
from neurodsl_b200 import graph as G
from neurodsl_b200 import layers as Ly


class _HostDevice:
    torch_device = torch.device("cpu")


def _graph():
    g = G.NeuroGraph(device=_HostDevice())
    G.set_(g, "x", torch.zeros(16, 256))
    return g


def test_linear_with_and_without_bias():
    g = _graph()
    gen = torch.Generator().manual_seed(0)
    out = Ly.Linear(256, 96)(g, "x", "fc", generator=gen)
    ns = g.nodes["default"]
    assert out == "fc_out" and g.rules["default"]["fc_out"].op == "linear"
    assert g.rules["default"]["fc_out"].inputs == ["x", "fc_W", "fc_b"]
    W = ns["fc_W"].value
    assert tuple(W.shape) == (96, 256) and ns["fc_W"].is_param
    assert float(W.abs().max()) <= 1 / math.sqrt(256)
    assert tuple(ns["fc_b"].value.shape) == (96,)
    out = Ly.Linear(256, 64, bias=False)(g, "x", "nb", generator=gen)
    r = g.rules["default"][out]
    assert (r.op, r.inputs, r.attrs) == ("matmul", ["x", "nb_W"], {"trans_b": True})


@pytest.mark.parametrize("layer", [Ly.MultiHeadFlashAttention, Ly.MultiHeadAttention])
def test_multihead_layers_build_the_reference_graph_and_compile_to_one_launch(layer):
    g = _graph()
    out = layer(256, 4)(g, "x", "mha", generator=torch.Generator().manual_seed(1))
    rules = g.rules["default"]
    assert out == "mha_output_out"
    for p in "qkv":
        assert rules[f"mha_{p}_out"].op == "matmul"
        for h in range(1, 5):
            r = rules[f"mha_{p}_h{h}"]
            assert (r.op, r.inputs) == ("slice_cols", [f"mha_{p}_out"])
            assert r.attrs == {"start_col": (h - 1) * 64 + 1, "end_col": h * 64}
    assert rules["mha_concat"].inputs == [f"mha_ao_h{h}" for h in range(1, 5)]
    plan = C.compile(g, C.CompilerConfig(training=False))
    r = g.rules["default"]["mha_concat"]
    assert (r.op, r.inputs) == ("flash_attention", ["mha_q_out", "mha_k_out", "mha_v_out"])
    assert r.attrs == {"n_heads": 4, "d_head": 64, "causal": True}
    assert plan.fused_ops["mha_concat"] == "flash_attention"
    assert not [s for s in g.rules["default"] if "_h" in s]
    assert g.rules["default"]["mha_output_out"].inputs == ["mha_concat", "mha_output_W"]


@pytest.mark.parametrize("layer", [Ly.MultiHeadFlashAttention, Ly.MultiHeadAttention])
def test_heads_the_kernels_do_not_take_stay_unfused(layer):
    """test/test_layers.jl:23-29 builds MultiHeadAttention(16, 2): heads of 8.
    The attention kernels take heads of 64 only, so compile leaves such a
    layer as written (its GEMM-based ops run any head width)."""
    g = G.NeuroGraph(device=_HostDevice())
    G.set_(g, "x", torch.zeros(4, 16))
    layer(16, 2)(g, "x", "mha", generator=torch.Generator().manual_seed(2))
    before = {k: r.op for k, r in g.rules["default"].items()}
    plan = C.compile(g, C.CompilerConfig(training=False))
    assert plan.fused_ops == {} and {k: r.op for k, r in g.rules["default"].items()} == before
