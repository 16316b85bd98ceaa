"""Layer builders of the operator API: each call adds parameter nodes and rules
to a graph and returns the output symbol, as the reference's layer structs do.

  reference (Julia)                                    here
  ---------------------------------------------------  ---------------------------
  Linear  src/layers.jl:15-34                           Linear
  MultiHeadAttention  src/layers.jl:37-80               MultiHeadAttention
  MultiHeadFlashAttention  src/flash_attention.jl:225-256
                                                        MultiHeadFlashAttention

Node names follow the reference (`<prefix>_W`, `<prefix>_out`,
`<prefix>_q_h<h>`, `<prefix>_concat`, ...), heads counted from 1, so graphs
and CtxStores read the same.  The rules run on the library's kernels; with
`compiler.compile(g, CompilerConfig(training=False))` a multi-head layer of
either kind becomes one strided :flash_attention over its three projections
(the naive per-head chain first becomes :flash_attn by rewrite rule).
Weights are uniform in ±1/√in_features like the reference's initialisation,
drawn from torch's generator on the graph's device (the reference's Julia
random stream cannot be reproduced).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import graph as G


def _uniform(g, *shape, k, generator=None):
    dev = g.device.torch_device
    return (torch.rand(*shape, generator=generator, device=dev) - 0.5) * (2 * k)


@dataclass
class Linear:
    """Y = X·Wᵀ (+ b) with W (out_features, in_features): a :linear rule with
    a bias, else :matmul with trans_b=true (src/layers.jl:15-34)."""
    in_features: int
    out_features: int
    bias: bool = True

    def __call__(self, g, input_sym: str, prefix: str, namespace: Optional[str] = None,
                 generator=None) -> str:
        ns = namespace or g.active_ns
        wn, on = f"{prefix}_W", f"{prefix}_out"
        k = 1.0 / math.sqrt(self.in_features)
        G.set_(g, wn, _uniform(g, self.out_features, self.in_features, k=k,
                               generator=generator), is_param=True, namespace=ns)
        if self.bias:
            bn = f"{prefix}_b"
            G.set_(g, bn, _uniform(g, self.out_features, k=k, generator=generator),
                   is_param=True, namespace=ns)
            G.addrule(g, G.GraphRule(on, [input_sym, wn, bn], "linear", namespace=ns))
        else:
            G.addrule(g, G.GraphRule(on, [input_sym, wn], "matmul", attrs={"trans_b": True},
                                     namespace=ns))
        return on


def _projections(g, dim, x_sym, prefix, ns, generator):
    return [Linear(dim, dim, bias=False)(g, x_sym, f"{prefix}_{p}", ns, generator)
            for p in "qkv"]


def _head_slices(g, h, d_head, full, prefix, ns):
    start, end = (h - 1) * d_head + 1, h * d_head
    names = []
    for p, src in zip("qkv", full):
        name = f"{prefix}_{p}_h{h}"
        G.addrule(g, G.GraphRule(name, [src], "slice_cols",
                                 attrs={"start_col": start, "end_col": end}, namespace=ns))
        names.append(name)
    return names


@dataclass
class MultiHeadAttention:
    """The naive multi-head layer (src/layers.jl:37-80): per head the column
    slices of the three bias-free projections, scores Q·Kᵀ, :scale_mask
    (1/√d_head and the causal mask), :softmax and P·V; :hcat_heads; the
    output projection."""
    dim: int
    n_heads: int
    d_head: Optional[int] = None

    def __post_init__(self):
        if self.d_head is None:
            self.d_head = self.dim // self.n_heads

    def __call__(self, g, x_sym: str, prefix: str, namespace: Optional[str] = None,
                 generator=None) -> str:
        ns = namespace or g.active_ns
        full = _projections(g, self.dim, x_sym, prefix, ns, generator)
        heads = []
        for h in range(1, self.n_heads + 1):
            qh, kh, vh = _head_slices(g, h, self.d_head, full, prefix, ns)
            sc, sk, pr, ao = (f"{prefix}_{n}_h{h}" for n in ("sc", "sk", "pr", "ao"))
            G.addrule(g, G.GraphRule(sc, [qh, kh], "matmul", attrs={"trans_b": True},
                                     namespace=ns))
            G.addrule(g, G.GraphRule(sk, [sc], "scale_mask", attrs={"d_head": self.d_head},
                                     namespace=ns))
            G.addrule(g, G.GraphRule(pr, [sk], "softmax", namespace=ns))
            G.addrule(g, G.GraphRule(ao, [pr, vh], "matmul", namespace=ns))
            heads.append(ao)
        concat = f"{prefix}_concat"
        G.addrule(g, G.GraphRule(concat, heads, "hcat_heads", namespace=ns))
        return Linear(self.dim, self.dim, bias=False)(g, concat, f"{prefix}_output", ns,
                                                      generator)


@dataclass
class MultiHeadFlashAttention:
    """The flash multi-head layer (src/flash_attention.jl:225-256): per head
    the column slices of the three projections and a causal :flash_attn;
    :hcat_heads; the output projection."""
    dim: int
    n_heads: int
    d_head: Optional[int] = None

    def __post_init__(self):
        if self.d_head is None:
            self.d_head = self.dim // self.n_heads

    def __call__(self, g, x_sym: str, prefix: str, namespace: Optional[str] = None,
                 generator=None) -> str:
        ns = namespace or g.active_ns
        full = _projections(g, self.dim, x_sym, prefix, ns, generator)
        heads = []
        for h in range(1, self.n_heads + 1):
            qh, kh, vh = _head_slices(g, h, self.d_head, full, prefix, ns)
            ao = f"{prefix}_ao_h{h}"
            G.addrule(g, G.GraphRule(ao, [qh, kh, vh], "flash_attn",
                                     attrs={"d_head": self.d_head, "causal": True}, namespace=ns))
            heads.append(ao)
        concat = f"{prefix}_concat"
        G.addrule(g, G.GraphRule(concat, heads, "hcat_heads", namespace=ns))
        return Linear(self.dim, self.dim, bias=False)(g, concat, f"{prefix}_output", ns,
                                                      generator)
