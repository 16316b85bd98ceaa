"""NeuroDSL's operator API (GraphRule / register_op! / demand!) over the B200 library.

A Python mirror of the reference's graph executor for the hot path, so that a
graph written against NeuroDSL's operator API runs on libneurodsl_b200.so with
the same op symbols, attrs, output-buffer ownership and CtxStore contents:

  reference (Julia)                         here
  ---------------------------------------   ------------------------------------
  NeuroGraph / GraphNode / GraphRule        NeuroGraph / GraphNode / GraphRule
    src/types.jl:12-69
  set!(g, sym, value; is_param)             set_(g, sym, value, is_param=...)
    src/graph_api.jl:12-35
  addrule!(g, rule)  src/graph_api.jl:152   addrule(g, rule)
  topo_order!        src/graph_api.jl:163   topo_order(g)
  invalidate_all!    src/graph_api.jl:222   invalidate_all(g)
  activate! / namespaces / node / params    activate / namespaces / node / params
  graph_summary  src/graph_api.jl:228       graph_summary
    src/graph_api.jl:9-10,146-150,225-226   (is_backpropable: src/types.jl:35)
  demand!(g, sym; ctx_store)                demand(g, sym, ctx_store=...)
    src/dispatch.jl:592-615
  execute_rule!      src/dispatch.jl:106    execute_rule(g, rule, ...)
  _infer_output_shape  src/dispatch.jl:36   _infer_output_shape(op, inputs, attrs)
  _dispatch_op       src/dispatch.jl:212    _dispatch_op(dev, out, op, inputs, ...)
  register_op! / CUSTOM_OPS  :587-588       register_op / CUSTOM_OPS
  @defop  src/dsl_macros.jl:9-26            @defop(name) decorator

Op symbols are strings ("flash_attn" for :flash_attn).  Node values are torch
CUDA tensors on the graph's B200Device: float32 (the reference's Float32
typing) or bfloat16 (device storage for tensor-core operands).  Every op
writes in place into the output buffer that execute_rule allocated, as the
reference's ops do, and stores the same CtxStore keys.  There is no CPU
device and no fallback: an op whose kernel is missing raises.
"""
from __future__ import annotations

import math
import warnings
from collections import deque
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional
import weakref

import torch

from . import ops
from ._lib import NeuroDSLError

CtxStore = dict  # src/types.jl:3


class NeurAtom:
    pass


class Datom(NeurAtom):
    pass


class Quantom(NeurAtom):
    pass


@dataclass
class B200Device:
    """The device tag of a graph whose ops run on libneurodsl_b200.so
    (the counterpart of Backend.CUDADevice, src/backend.jl:6-9)."""
    index: int = 0

    @property
    def torch_device(self):
        return torch.device("cuda", self.index)


def zeros32(dev: B200Device, *shape):
    """Backend.zeros32 (src/backend.jl:11-12) on the B200 device."""
    return torch.zeros(*shape, dtype=torch.float32, device=dev.torch_device)


def to_device(dev: B200Device, x):
    """Backend.to_device (src/backend.jl:20-26)."""
    if isinstance(x, torch.Tensor):
        return x.to(dev.torch_device)
    import numpy as np
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x)).to(dev.torch_device)
    return x


@dataclass
class GraphNode:
    """src/types.jl:12-31."""
    name: str
    value: Optional[torch.Tensor]
    gradient: Optional[torch.Tensor] = None
    valid: bool = True
    backwarded: bool = False
    atom_type: type = Quantom
    is_param: bool = False
    namespace: str = "default"
    aux_data: Dict[str, Any] = field(default_factory=dict)
    watchers: List[str] = field(default_factory=list)
    on_change: Optional[Callable] = None


@dataclass
class GraphRule:
    """GraphRule(output, inputs, op; attrs, namespace, atom_type), src/types.jl:37-46."""
    output: str
    inputs: List[str]
    op: str
    attrs: Dict[str, Any] = field(default_factory=dict)
    namespace: str = "default"
    atom_type: type = Quantom


class NeuroGraph:
    """src/types.jl:51-69 — nodes and rules per namespace, cached topo order."""

    def __init__(self, namespace: str = "default", device: Optional[B200Device] = None):
        self.nodes: Dict[str, Dict[str, GraphNode]] = {}
        self.rules: Dict[str, Dict[str, GraphRule]] = {}
        self.grad_registry: Dict[str, Callable] = {}
        self._topo_cache: Dict[str, Optional[List[str]]] = {}
        self.active_ns = namespace
        self.device = device if device is not None else B200Device(0)
        self._ensure_namespace(namespace)

    def _ensure_namespace(self, ns):
        self.nodes.setdefault(ns, {})
        self.rules.setdefault(ns, {})
        self._topo_cache.setdefault(ns, None)


def activate(g: NeuroGraph, ns: str) -> NeuroGraph:
    """activate!(g, ns) (src/graph_api.jl:9): later calls without a namespace
    use `ns`."""
    g._ensure_namespace(ns)
    g.active_ns = ns
    return g


def namespaces(g: NeuroGraph) -> List[str]:
    return list(g.nodes)


def graph_summary(g: NeuroGraph) -> str:
    """graph_summary(g) (src/graph_api.jl:228-237): the device and, per
    namespace, the node, rule and parameter counts; printed and returned."""
    dev = g.device.torch_device
    lines = ["NeuroGraph — neurodsl_b200",
             f"  Device    : {'B200 (cuda:%d)' % dev.index if dev.type == 'cuda' else dev.type.upper()}"]
    for ns in namespaces(g):
        n_p = sum(1 for nd in g.nodes[ns].values() if nd.is_param)
        lines.append(f"  [:{ns}]  nodes={len(g.nodes[ns])}  rules={len(g.rules[ns])}  params={n_p}")
    text = "\n".join(lines)
    print(text)
    return text


def is_backpropable(nd: "GraphNode") -> bool:
    """A Quantom node carries gradients (src/types.jl:35)."""
    return issubclass(nd.atom_type, Quantom)


def node(g: NeuroGraph, name: str, namespace: Optional[str] = None) -> "GraphNode":
    """node(g, name) (src/graph_api.jl:146-150)."""
    ns = namespace or g.active_ns
    if ns not in g.nodes or name not in g.nodes[ns]:
        raise NeuroDSLError(1, f"Nœud :{name} introuvable dans :{ns}")
    return g.nodes[ns][name]


def params(g: NeuroGraph, namespace: Optional[str] = None) -> List["GraphNode"]:
    """The backpropagable parameter nodes (src/graph_api.jl:225-226)."""
    ns = namespace or g.active_ns
    return [nd for nd in g.nodes[ns].values() if nd.is_param and is_backpropable(nd)]


def _consumers(g, ns):
    cons: Dict[str, List[str]] = {}
    for out, r in g.rules[ns].items():
        for s in r.inputs:
            cons.setdefault(s, []).append(out)
    return cons


def _invalidate_downstream(g, sym, ns):
    """BFS from `sym` over its consumers and watchers (src/graph_api.jl:37-71):
    every node reached is invalidated and its on_change callback called with
    the reference's (g, sym, ns).  `sym` itself keeps its new value (valid)
    but its callback fires too.  Unlike the reference, consumers that are
    already invalid are still followed: a compiled plan's released
    intermediates are invalid while the output computed from them is valid,
    and must be recomputed."""
    cons = _consumers(g, ns)
    q = deque([sym])
    seen = set()
    while q:
        s = q.popleft()
        if s in seen:
            continue
        seen.add(s)
        nd = g.nodes[ns].get(s)
        if nd is not None:
            if s != sym:
                nd.valid = False
            if nd.on_change is not None:
                nd.on_change(g, s, ns)
            q.extend(w for w in nd.watchers if w not in seen)
        q.extend(cons.get(s, []))


def watch(g: NeuroGraph, observer: str, observed: str, namespace: Optional[str] = None):
    """_watch!(g, observer, observed) (src/graph_api.jl:72-80): invalidating
    `observed` invalidates `observer` too."""
    ns = namespace or g.active_ns
    g.nodes[ns][observed].watchers.append(observer)


def set_(g: NeuroGraph, name: str, value, is_param: bool = False, namespace: Optional[str] = None,
         atom_type=Quantom):
    """set!(g, name, value; is_param, namespace) — src/graph_api.jl:12-35."""
    ns = namespace or g.active_ns
    g._ensure_namespace(ns)
    v = to_device(g.device, value)
    nd = g.nodes[ns].get(name)
    if nd is None:
        g.nodes[ns][name] = GraphNode(name, v, is_param=is_param, namespace=ns, atom_type=atom_type)
        g._topo_cache[ns] = None
    else:
        nd.value = v
        nd.valid = True
        nd.is_param = nd.is_param or is_param
    _invalidate_downstream(g, name, ns)
    return g.nodes[ns][name]


def addrule(g: NeuroGraph, rule: GraphRule):
    """addrule!(g, rule) — src/graph_api.jl:152-160."""
    ns = rule.namespace
    g._ensure_namespace(ns)
    g.rules[ns][rule.output] = rule
    if rule.output not in g.nodes[ns]:
        g.nodes[ns][rule.output] = GraphNode(rule.output, None, valid=False, namespace=ns,
                                             atom_type=rule.atom_type)
    else:
        g.nodes[ns][rule.output].valid = False
    g._topo_cache[ns] = None
    return rule


def topo_order(g: NeuroGraph, namespace: Optional[str] = None) -> List[str]:
    """topo_order! — iterative DFS, cached per namespace (src/graph_api.jl:163-209)."""
    ns = namespace or g.active_ns
    cached = g._topo_cache.get(ns)
    if cached is not None:
        return cached
    order: List[str] = []
    state: Dict[str, int] = {}
    for root in list(g.nodes[ns].keys()):
        if state.get(root):
            continue
        stack = [(root, False)]
        while stack:
            s, done = stack.pop()
            if done:
                state[s] = 2
                order.append(s)
                continue
            st = state.get(s, 0)
            if st == 2:
                continue
            if st == 1:
                raise NeuroDSLError(2, f"cycle detected at :{s}")
            state[s] = 1
            stack.append((s, True))
            r = g.rules[ns].get(s)
            if r is not None:
                for inp in reversed(r.inputs):
                    if state.get(inp, 0) == 0:
                        stack.append((inp, False))
                    elif state.get(inp) == 1:
                        raise NeuroDSLError(2, f"cycle detected at :{inp}")
    g._topo_cache[ns] = order
    return order


def _store_ctx(ctx_store, sym, d):
    """_store_ctx! (src/dispatch.jl:29-33)."""
    if ctx_store is not None:
        ctx_store[sym] = d


# ----------------------------------------------------------------- shapes ---

def _infer_output_shape(op: str, inputs, attrs):
    """_infer_output_shape (src/dispatch.jl:36-97) with entries for the new ops."""
    if op in ("matmul", "fused_matmul_add", "fused_linear_gelu", "fused_matmul_relu"):
        A, B = inputs[0], inputs[1]
        tb = attrs.get("trans_b", False)
        return (A.shape[0], B.shape[0] if tb else B.shape[1])
    if op in ("linear", "fused_linear_residual"):
        X, W = inputs[0], inputs[1]
        return (X.shape[0], W.shape[0])
    if op == "fused_layernorm_linear":                       # [x, gamma, beta, W(, b)]
        W = inputs[3]
        return (inputs[0].shape[0], W.shape[0] if attrs.get("trans_b", False) else W.shape[1])
    if op == "hcat_heads":
        return (inputs[0].shape[0], sum(x.shape[1] for x in inputs))
    if op == "slice_cols":
        s, e = attrs.get("start_col", 1), attrs.get("end_col", inputs[0].shape[1])
        return (inputs[0].shape[0], e - s + 1)
    if op == "flash_attention" and len(inputs) == 1:
        return (inputs[0].shape[0], inputs[0].shape[1] // 3)   # fused (S, 3d) projection
    if op == "add":
        a, b = inputs[0], inputs[1]
        return tuple(b.shape) if (a.dim() == 1 and b.dim() == 2) else tuple(a.shape)
    if op in ("identity", "flash_attn", "flash_attention", "layernorm", "gelu",
              "scale_mask", "softmax"):
        return tuple(inputs[0].shape)
    if op == "kv_decode_attn":
        return tuple(inputs[0].shape)
    if op == "embedding":                                    # [E, idx]
        return (inputs[1].numel(), inputs[0].shape[1])
    # the reference warns and falls back to the first input's shape (:93-96)
    warnings.warn(f"Shape inference non implémentée pour :{op}, utilisation de la forme du "
                  "premier argument")
    return tuple(inputs[0].shape)


# ------------------------------------------------------------------- exec ---

def execute_rule(g: NeuroGraph, rule: GraphRule, ctx_store=None, namespace=None):
    """execute_rule! (src/dispatch.jl:106-152): gather inputs, (re)allocate the
    output buffer when its shape changed, run the op in place, mark valid."""
    dev = g.device
    ns = rule.namespace
    out_node = g.nodes[ns][rule.output]
    inputs = []
    for s in rule.inputs:
        v = g.nodes[ns][s].value
        if not isinstance(v, torch.Tensor):
            raise NeuroDSLError(1, f":{s} has no value (input of :{rule.output})")
        inputs.append(v)
    shape = _infer_output_shape(rule.op, inputs, rule.attrs)
    out_dtype = rule.attrs.get("out_dtype", torch.float32)
    if (out_node.value is None or tuple(out_node.value.shape) != tuple(shape)
            or out_node.value.dtype != out_dtype):
        out_node.value = torch.zeros(shape, dtype=out_dtype, device=dev.torch_device)
    _dispatch_op(dev, out_node.value, rule.op, inputs, rule.attrs, rule.output, out_node, ctx_store)
    out_node.valid = True
    return out_node.value


def invalidate_all(g: NeuroGraph, namespace: Optional[str] = None):
    """invalidate_all!(g) (src/graph_api.jl:222-223): every node that is not a
    parameter is marked for recomputation."""
    ns = namespace or g.active_ns
    for nd in g.nodes[ns].values():
        if not nd.is_param:
            nd.valid = False


def demand(g: NeuroGraph, name: str, ctx_store=None, namespace=None):
    """demand!(g, name; ctx_store) — src/dispatch.jl:592-615."""
    ns = namespace or g.active_ns
    if ns not in g.nodes or name not in g.nodes[ns]:
        raise NeuroDSLError(1, f":{name} introuvable dans :{ns}")
    nd = g.nodes[ns][name]
    if nd.valid and nd.value is not None:
        return nd.value
    for sym in topo_order(g, ns):
        ndi = g.nodes[ns][sym]
        if ndi.valid and ndi.value is not None:
            continue
        if sym not in g.rules[ns]:
            continue
        execute_rule(g, g.rules[ns][sym], ctx_store=ctx_store, namespace=ns)
        if sym == name:
            break
    return g.nodes[ns][name].value


CUSTOM_OPS: Dict[str, Callable] = {}


def register_op(name: str, fn: Callable):
    """register_op!(name, fn) — src/dispatch.jl:587-588."""
    CUSTOM_OPS[name] = fn
    return fn


def defop(name: str):
    """The @defop macro's function form (src/dsl_macros.jl:9-26) as a
    decorator: the function (dev, out, inputs, attrs, out_sym, node, ctx)
    writes its result into `out` and is registered under `name`."""
    def deco(fn: Callable) -> Callable:
        return register_op(name, fn)
    return deco


# ----------------------------------------------------------- op helpers ---

def _ceil8(k):
    return (k + 7) // 8 * 8


def _bf16_rows(x):
    """A 2-D GEMM operand as contiguous bf16 rows whose length is a multiple
    of 8 (converted on the device by the library, the zero columns of an
    inner dimension that is not a multiple of 8 written in the same pass:
    the GEMM moves rows in 16-byte pieces, and zero columns add nothing to
    the dot products, so graphs with any inner dimension — the reference's
    tests use K = 3 — run on the same kernel)."""
    rows, cols = x.shape
    if x.dtype == torch.bfloat16 and x.is_contiguous() and cols % 8 == 0:
        return x
    return ops.convert_2d_padded(x.contiguous(), rows, cols, False, torch.bfloat16, _ceil8(cols))


def _convert_weight_nk(W, trans_b):
    if trans_b:
        return _bf16_rows(W)
    K, N = W.shape
    return ops.convert_2d_padded(W.contiguous(), N, K, True, torch.bfloat16, _ceil8(K))


# bf16 [N][K] copies of Float32 weights, per weight tensor: a node's value is
# converted once and reused by every later call until the tensor is replaced
# (set!) or written in place (its version counter moves).
_WEIGHT_CACHE = {}


def _weight_nk(W, trans_b):
    """The weight as [N][K] bf16 (K padded to a multiple of 8): trans_b=true
    weights already are; a (K, N) row-major matrix is the column-major (N, K)
    one and is converted.  Cached per tensor (see _WEIGHT_CACHE)."""
    if W.dtype == torch.bfloat16 and trans_b and W.is_contiguous() and W.shape[1] % 8 == 0:
        return W
    key = id(W)
    hit = _WEIGHT_CACHE.get(key)
    if hit is not None:
        ref, version, tb, conv = hit
        if ref() is W and version == W._version and tb == trans_b:
            return conv
    conv = _convert_weight_nk(W, trans_b)
    try:
        ref = weakref.ref(W, lambda _r, k=key: _WEIGHT_CACHE.pop(k, None))
    except TypeError:
        return conv
    _WEIGHT_CACHE[key] = (ref, W._version, trans_b, conv)
    return conv


def _bias_vec(b):
    if b is None:
        return None
    return b.reshape(-1).to(torch.float32).contiguous()


def _gemm_into(out, X, Wnk, bias=None, residual=None, act="none"):
    if out.dtype not in (torch.float32, torch.bfloat16) or not out.is_contiguous():
        raise NeuroDSLError(4, "output buffer must be contiguous fp32 or bf16")
    ops.linear(_bf16_rows(X), Wnk, _bias_vec(bias), residual=residual, act=act, out=out)


def _copy_back(buf, out):
    """The side buffer of an aliased output copied into the node's buffer."""
    rows = out.shape[0] if out.dim() else 1
    ops.copy_2d(buf.reshape(rows, -1), out.view(rows, -1))


def _alias_safe(out, out_node, inputs):
    """Output buffer aliasing an input is redirected through aux_data[:_alias_buf]
    (src/dispatch.jl:220-231, :366-376)."""
    if any(out.data_ptr() == x.data_ptr() for x in inputs):
        buf = out_node.aux_data.get("_alias_buf")
        if buf is None or buf.shape != out.shape or buf.dtype != out.dtype:
            buf = torch.empty_like(out)
            out_node.aux_data["_alias_buf"] = buf
        return buf, True
    return out, False


# ------------------------------------------------------------- dispatch ---

def _dispatch_op(dev, output_buffer, op: str, inputs, attrs, out_sym, out_node, ctx_store):
    """_dispatch_op (src/dispatch.jl:212-585) for the ops on the inference hot
    path; custom ops (CUSTOM_OPS) are looked up after the built-ins, like the
    reference's fall-through at :571-573."""
    if op == "matmul":
        A, B = inputs[0], inputs[1]
        tb = attrs.get("trans_b", False)
        kA = A.shape[1]
        kB = B.shape[1] if tb else B.shape[0]
        if kA != kB:
            raise NeuroDSLError(2, f"[{out_sym}] matmul incompatible A={tuple(A.shape)} "
                                   f"B={tuple(B.shape)} trans_b={tb}")
        buf, aliased = _alias_safe(output_buffer, out_node, inputs)
        _gemm_into(buf, A, _weight_nk(B, tb))
        if aliased:
            _copy_back(buf, output_buffer)
        _store_ctx(ctx_store, out_sym, {"trans_b": tb, "A": A.clone() if ctx_store is not None else A,
                                        "B": B})
        return output_buffer
    if op == "fused_matmul_add":
        A, B, bias = inputs[0], inputs[1], inputs[2]
        tb = attrs.get("trans_b", False)
        _gemm_into(output_buffer, A, _weight_nk(B, tb), bias=bias)
        _store_ctx(ctx_store, out_sym, {"trans_b": tb, "A": A, "B": B})
        return output_buffer
    if op == "linear":
        X, W = inputs[0], inputs[1]
        bias = inputs[2] if len(inputs) == 3 else None
        buf, aliased = _alias_safe(output_buffer, out_node, inputs)
        _gemm_into(buf, X, _weight_nk(W, True), bias=bias)
        if aliased:
            _copy_back(buf, output_buffer)
        _store_ctx(ctx_store, out_sym, {"X": X, "W": W, "n_inputs": len(inputs)})
        return output_buffer
    if op == "slice_cols":
        # columns start_col..end_col (1-based, inclusive) of an (N, d) node,
        # src/dispatch.jl:544-553: a device copy.  compile() folds the slices
        # of a multi-head layer into the strided :flash_attention instead.
        x = inputs[0]
        s, e = attrs.get("start_col", 1), attrs.get("end_col", x.shape[1])
        ops.copy_2d(x[:, s - 1:e], output_buffer)
        _store_ctx(ctx_store, out_sym, {"start_col": s, "end_col": e})
        return output_buffer
    if op == "embedding":
        # rows idx[i] (1-based, as the reference's Julia indices) of the table
        # E (vocab, d), src/dispatch.jl:476-491, gathered on the device where
        # the reference copies through the host; ctx {idx, E_size}
        # (nd_gather_rows: an index outside 1..vocab gives a zero row and sets
        # the device error word, read by ops.device_error(); no host sync)
        E, idx = inputs[0], inputs[1]
        if idx.device != E.device:
            raise NeuroDSLError(2, f"[{out_sym}] embedding indices must be on the table's device")
        ops.gather_rows(E, idx, index_base=1, out=output_buffer)
        _store_ctx(ctx_store, out_sym, {"idx": idx.reshape(-1), "E_size": tuple(E.shape)})
        return output_buffer
    if op == "hcat_heads":
        # the heads' (N, d_h) outputs side by side, src/dispatch.jl:349-361
        off = 0
        for x in inputs:
            ops.copy_2d(x, output_buffer[:, off:off + x.shape[1]])
            off += x.shape[1]
        _store_ctx(ctx_store, out_sym, {"n_heads": len(inputs), "d_head": inputs[0].shape[1]})
        return output_buffer
    if op in CUSTOM_OPS:
        CUSTOM_OPS[op](dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store)
        return output_buffer
    if op == "identity":
        x = inputs[0]
        ops.copy_2d(x.reshape(x.shape[0], -1), output_buffer.view(x.shape[0], -1))
        return output_buffer
    raise NeuroDSLError(4, f"Opérateur inconnu : :{op}. Utilisez register_op! pour enregistrer "
                           "un op custom.")


# ------------------------------------------------ B200 custom operators ---

def _dispatch_flash_attn(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:flash_attn on one head, Q/K/V (N, D) — _dispatch_flash_attn!
    (src/flash_attention.jl:175-200): aux_data[:flash_l] = log-sum-exp,
    aux_data[:flash_m] = row max, ctx {Q,K,V,out,l,m,d_head,causal}."""
    Q, K, V = inputs[0], inputs[1], inputs[2]
    d_head = attrs.get("d_head", Q.shape[1])
    causal = attrs.get("causal", True)
    N, D = Q.shape
    Nk = K.shape[0]
    l_buf = out_node.aux_data.get("flash_l")
    if l_buf is None or l_buf.numel() != N:
        l_buf = torch.zeros(N, dtype=torch.float32, device=dev.torch_device)
        m_buf = torch.full((N,), -math.inf, dtype=torch.float32, device=dev.torch_device)
        out_node.aux_data["flash_l"] = l_buf
        out_node.aux_data["flash_m"] = m_buf
    m_buf = out_node.aux_data["flash_m"]
    q4 = _bf16_rows(Q).view(1, 1, N, D)
    k4 = _bf16_rows(K).view(1, 1, Nk, D)
    v4 = _bf16_rows(V).view(1, 1, Nk, D)
    ops.flash_attn_fwd(q4, k4, v4, causal=causal, scale=1.0 / math.sqrt(d_head),
                       out=output_buffer.view(1, 1, N, D), lse=l_buf.view(1, 1, N),
                       row_max=m_buf.view(1, 1, N))
    _store_ctx(ctx_store, out_sym, {"Q": Q, "K": K, "V": V, "out": output_buffer, "l": l_buf,
                                    "m": m_buf, "d_head": d_head, "causal": causal})
    return output_buffer


def _token_major_view(x, S, H, D):
    """An (S, H·D) row-major matrix seen as [1][H][S][D] without copying: the
    per-head :slice_cols of src/flash_attention.jl:241-246 become strides."""
    return x.view(S, H, D).permute(1, 0, 2).unsqueeze(0)


def _dispatch_flash_attention(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:flash_attention — all heads of q_full/k_full/v_full (S, H·D) in one
    launch; replaces H × (3 :slice_cols + :flash_attn) and :hcat_heads
    (src/flash_attention.jl:232-256).  The kernel reads the projections and
    writes the (S, H·D) output in place through strides."""
    H = attrs["n_heads"]
    causal = attrs.get("causal", True)
    if len(inputs) == 1:
        # one fused projection [q | k | v] of shape (S, 3·H·D)
        qkv = _bf16_rows(inputs[0])
        S, d3 = qkv.shape
        d = d3 // 3
        D = attrs.get("d_head", d // H)
        if 3 * H * D != d3:
            raise NeuroDSLError(2, f"fused qkv width {d3} != 3 x n_heads {H} x d_head {D}")
        parts = qkv.view(S, 3, H, D).permute(1, 2, 0, 3).unsqueeze(1)  # [3][1][H][S][D]
        q4, k4, v4 = parts[0], parts[1], parts[2]
        q = k = v = inputs[0]
        Sk = S
    else:
        q, k, v = inputs[0], inputs[1], inputs[2]
        S, d = q.shape
        D = attrs.get("d_head", d // H)
        if H * D != d:
            raise NeuroDSLError(2, f"n_heads {H} x d_head {D} != dim {d}")
        Sk = k.shape[0]
        q4 = _token_major_view(_bf16_rows(q), S, H, D)
        k4 = _token_major_view(_bf16_rows(k), Sk, H, D)
        v4 = _token_major_view(_bf16_rows(v), Sk, H, D)
    lse = out_node.aux_data.get("flash_l")
    if lse is None or tuple(lse.shape) != (H, S):
        lse = torch.empty((H, S), dtype=torch.float32, device=dev.torch_device)
        out_node.aux_data["flash_l"] = lse
        out_node.aux_data["flash_m"] = torch.empty_like(lse)
    m = out_node.aux_data["flash_m"]
    buf, aliased = _alias_safe(output_buffer, out_node, inputs)
    ops.flash_attn_fwd(q4, k4, v4, causal=causal, scale=1.0 / math.sqrt(D),
                       out=_token_major_view(buf, S, H, D), lse=lse.view(1, H, S),
                       row_max=m.view(1, H, S))
    if aliased:
        _copy_back(buf, output_buffer)
    _store_ctx(ctx_store, out_sym, {"Q": q, "K": k, "V": v, "out": output_buffer,
                                    "l": lse, "m": m, "d_head": D, "causal": causal,
                                    "n_heads": H})
    return output_buffer


def _dispatch_kv_decode_attn(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:kv_decode_attn — inputs [q (B, H·D), k_cache, v_cache ([B][H][L_max][D])]
    (+ optional [k_new, v_new] (B, H·D) appended at cache_len-1), attrs
    :n_heads, :d_head, :cache_len.  Output (B, H·D)."""
    q, kc, vc = inputs[0], inputs[1], inputs[2]
    B, d = q.shape
    H = attrs["n_heads"]
    D = attrs.get("d_head", d // H)
    L = attrs["cache_len"]
    kn = vn = None
    if len(inputs) == 5:
        kn = _bf16_rows(inputs[3]).view(B, H, D)
        vn = _bf16_rows(inputs[4]).view(B, H, D)
    out, lse = ops.kv_decode_attn(_bf16_rows(q).view(B, H, D), kc, vc, L, k_new=kn, v_new=vn,
                                  scale=1.0 / math.sqrt(D), out_dtype=output_buffer.dtype,
                                  out=output_buffer.view(B, H, D))
    out_node.aux_data["decode_lse"] = lse
    _store_ctx(ctx_store, out_sym, {"q": q, "cache_len": L, "l": lse, "n_heads": H, "d_head": D})
    return output_buffer


_GELU_APPROX = {"sigmoid": "sigmoid", "tanh": "tanh", "erf": "erf"}


def _dispatch_fused_linear_gelu(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:fused_linear_gelu — inputs [A, W(, b)], attrs :trans_b, :approx.
    The reference's notebook @defop (notebook/compiler.ipynb cell 15) is
    z·σ(1.702 z) of A·B(ᵀ) with no bias; the default approx is that one."""
    A, W = inputs[0], inputs[1]
    b = inputs[2] if len(inputs) > 2 else None
    tb = attrs.get("trans_b", False)
    approx = _GELU_APPROX[str(attrs.get("approx", "sigmoid")).lstrip(":")]
    _gemm_into(output_buffer, A, _weight_nk(W, tb), bias=b, act=approx)
    _store_ctx(ctx_store, out_sym, {"trans_b": tb, "A": A, "B": W, "output": output_buffer})
    return output_buffer


def _dispatch_fused_linear_residual(dev, output_buffer, inputs, attrs, out_sym, out_node,
                                    ctx_store):
    """:fused_linear_residual — X·Wᵀ (+ b) + R, inputs [X, W, (b,) R]: the
    :linear rule followed by the residual :add (src/dispatch.jl:363-417) in
    one GEMM epilogue."""
    if len(inputs) == 4:
        X, W, b, R = inputs
    else:                                   # a :linear without bias, then the :add
        (X, W, R), b = inputs, None
    res = R if R.is_contiguous() else R.contiguous()
    _gemm_into(output_buffer, X, _bf16_rows(W), bias=b, residual=res)
    _store_ctx(ctx_store, out_sym, {"X": X, "W": W, "n_inputs": 4})
    return output_buffer


def _dispatch_layernorm(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:layernorm — inputs [x, gamma(, beta)], attr :eps (default 1e-5).
    aux_data[:ln_mean], [:ln_rstd] and ctx {x, gamma, beta, mean, rstd}
    mirror :rmsnorm's aux_data[:rms_inv] (src/dispatch.jl:426-438)."""
    x = inputs[0]
    gamma = inputs[1] if len(inputs) > 1 else None
    beta = inputs[2] if len(inputs) > 2 else None
    eps = float(attrs.get("eps", 1e-5))
    rows = x.shape[0]
    mean = out_node.aux_data.get("ln_mean")
    if mean is None or mean.numel() != rows:
        mean = torch.zeros(rows, dtype=torch.float32, device=dev.torch_device)
        out_node.aux_data["ln_mean"] = mean
        out_node.aux_data["ln_rstd"] = torch.zeros_like(mean)
    rstd = out_node.aux_data["ln_rstd"]
    g = None if gamma is None else gamma.reshape(-1).float().contiguous()
    bt = None if beta is None else beta.reshape(-1).float().contiguous()
    ops.layernorm(x.contiguous(), g, bt, eps=eps, out=output_buffer, mean=mean, rstd=rstd)
    _store_ctx(ctx_store, out_sym, {"x": x, "gamma": gamma, "beta": beta, "mean": mean,
                                    "rstd": rstd})
    return output_buffer


def _dispatch_add(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:add (src/dispatch.jl:386-417): same shapes, or a matrix and a vector
    broadcast per column (preferred when the lengths match, as in the
    reference) or per row, in either operand order; and, as the reference's
    general broadcast, a matrix plus a (1, cols) row, a (rows, 1) column or a
    single value (nd_add)."""
    a, b = _f32(inputs[0]), _f32(inputs[1])
    if a.dim() == 1 and b.dim() == 2:
        a, b = b, a
    ops.add(a, b, out=output_buffer)
    return output_buffer


def _f32(x):
    return x if x.dtype == torch.float32 and x.is_contiguous() else x.float().contiguous()


def _dispatch_gelu(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:gelu — elementwise GELU in the form of attr :approx (default :sigmoid,
    the z·σ(1.702 z) of the reference's fused_linear_gelu notebook op); the
    compiler fuses a :matmul / :linear followed by it into
    :fused_linear_gelu."""
    approx = _GELU_APPROX[str(attrs.get("approx", "sigmoid")).lstrip(":")]
    ops.gelu(_f32(inputs[0]), act=approx, out=output_buffer)
    _store_ctx(ctx_store, out_sym, {"x": inputs[0], "approx": approx})
    return output_buffer


def _dispatch_scale_mask(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:scale_mask — scores / sqrt(d_head) plus the causal mask
    (src/dispatch.jl:464-474); ctx {scale}."""
    scores = inputs[0]
    d_head = int(attrs.get("d_head", scores.shape[1]))
    ops.scale_mask(_f32(scores), d_head, out=output_buffer)
    _store_ctx(ctx_store, out_sym, {"scale": 1.0 / math.sqrt(d_head)})
    return output_buffer


def _dispatch_softmax(dev, output_buffer, inputs, attrs, out_sym, out_node, ctx_store):
    """:softmax — row softmax (src/kernels.jl:269-287); ctx {output}."""
    ops.softmax(_f32(inputs[0]), out=output_buffer)
    _store_ctx(ctx_store, out_sym, {"output": output_buffer})
    return output_buffer


def _dispatch_fused_layernorm_linear(dev, output_buffer, inputs, attrs, out_sym, out_node,
                                     ctx_store):
    """:fused_layernorm_linear — LayerNorm(x; gamma, beta, :eps) · W (+ b),
    inputs [x, gamma, beta, W(, b)], attr :trans_b (true for a :linear weight
    (out, in)).  At most 32 bf16 rows with K % 32 == 0 and K <= 1024 take
    nd_ln_gemm (one launch, the LayerNorm in the GEMM prologue); otherwise the
    LayerNorm goes to a bf16 buffer (aux_data[:_ln_buf]) read by the GEMM."""
    x, gamma, beta, W = inputs[:4]
    b = inputs[4] if len(inputs) > 4 else None
    eps = float(attrs.get("eps", 1e-5))
    Wnk = _weight_nk(W, attrs.get("trans_b", False))
    g = gamma.reshape(-1).float().contiguous()
    bt = beta.reshape(-1).float().contiguous()
    rows, K = x.shape
    if x.dtype == torch.bfloat16 and rows <= 32 and K % 32 == 0 and K <= 1024:
        ops.ln_linear(x.contiguous(), Wnk, gamma=g, beta=bt, eps=eps, bias=_bias_vec(b),
                      out=output_buffer)
    else:
        h = out_node.aux_data.get("_ln_buf")
        if h is None or tuple(h.shape) != (rows, K):
            h = torch.empty((rows, K), dtype=torch.bfloat16, device=dev.torch_device)
            out_node.aux_data["_ln_buf"] = h
        ops.layernorm(x.contiguous(), g, bt, eps=eps, out=h, stats=False)
        ops.linear(_bf16_rows(h), Wnk, _bias_vec(b), out=output_buffer)
    _store_ctx(ctx_store, out_sym, {"x": x, "gamma": gamma, "beta": beta, "W": W})
    return output_buffer


def register_b200_ops():
    """Register the B200 operators (the @defop / register_op! plugin form)."""
    register_op("flash_attn", _dispatch_flash_attn)
    register_op("flash_attention", _dispatch_flash_attention)
    register_op("kv_decode_attn", _dispatch_kv_decode_attn)
    register_op("fused_linear_gelu", _dispatch_fused_linear_gelu)
    register_op("fused_linear_residual", _dispatch_fused_linear_residual)
    register_op("layernorm", _dispatch_layernorm)
    register_op("add", _dispatch_add)
    register_op("gelu", _dispatch_gelu)
    register_op("scale_mask", _dispatch_scale_mask)
    register_op("softmax", _dispatch_softmax)
    register_op("fused_layernorm_linear", _dispatch_fused_layernorm_linear)


register_b200_ops()
