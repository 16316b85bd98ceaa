"""NeuroDSL's rewrite-rule compiler, restated over the operator-API mirror, with
rules that map unfused transformer graphs onto the B200 fused operators.

  reference (Julia)                               here
  ---------------------------------------------   ---------------------------------
  RewriteRule  src/compiler_config.jl:75-97       RewriteRule (+ optional `attrs`)
  CompilerConfig  src/compiler_config.jl:349-359  CompilerConfig
  op_of / single_consumer                         op_of / single_consumer
    src/compiler_rules.jl:56-72
  _is_fuseable_chain  src/compiler_rules.jl:121   _is_fuseable_chain
  scan_graph  src/compiler_rules.jl:575-623       scan_graph
  _apply_fusion!  src/compiler.jl:16-66           _apply_fusion
  compile  src/compiler.jl:70-124                 compile -> CompiledPlan
  dirty tracking / recompile!  src/compiler.jl:126-191
                                                  _register_dirty_tracking,
                                                  is_dirty, recompile
  plan(g, out)  src/compiler.jl:204-240           CompiledPlan.__call__
  symbolic_cost / default_cost                    symbolic_cost / default_cost
    src/compiler_config.jl:230-283
  _choose_cheapest_alternative                    choose_cheapest_alternative
    src/compiler_rules.jl:696-750
  (B200) MultiHeadFlashAttention layer            fold_multihead_attention
    src/flash_attention.jl:232-256 -> :flash_attention
  _flash_condition  src/compiler_config.jl:107    _flash_condition
  memory plan + BufferPool (liveness.jl)          neurodsl_b200/liveness.py

Matching follows the reference: for each rule, every node produced by the
pattern's first op starts a chain that follows single consumers through the
pattern; intermediate nodes must have exactly one consumer; the optional
condition must hold; matches apply in decreasing `cost_delta`.  A fusion
merges the chain's attrs, takes the chain's external inputs in rule order,
deletes the intermediate nodes and re-registers the last node's output
with the fused op.  As in the reference, `training=True` refuses a fusion
into an op without a backward rule; the B200 operators are inference-only,
so inference graphs compile with `CompilerConfig(training=False)`.

B200 extension: a rule may carry `attrs` merged into the fused rule (the
:linear weight is (out, in), so a :linear chain sets `trans_b=True` for ops
that take a :matmul-style weight), and a condition receives the graph, the
chain and the namespace like the reference's.
"""
from __future__ import annotations

import time
import warnings
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Set, Tuple

from . import graph as G
from . import liveness as L


@dataclass
class RewriteRule:
    name: str
    pattern: Tuple[str, ...]
    result: str
    condition: Optional[Callable] = None
    cost_delta: float = 1.0
    verified: bool = False
    attrs: Dict[str, Any] = field(default_factory=dict)


@dataclass
class RuleMatch:
    rule: RewriteRule
    nodes: List[str]
    namespace: str
    score: float


def producer(g, sym, ns):
    return g.rules[ns].get(sym)


def op_of(g, sym, ns) -> Optional[str]:
    r = producer(g, sym, ns)
    return None if r is None else r.op


def consumers(g, sym, ns) -> List[str]:
    return [out for out, r in g.rules[ns].items() if sym in r.inputs]


def single_consumer(g, sym, ns) -> Optional[str]:
    c = consumers(g, sym, ns)
    return c[0] if len(c) == 1 else None


def _is_fuseable_chain(g, chain, ns) -> bool:
    if len(chain) < 2:
        return False
    return all(single_consumer(g, s, ns) is not None for s in chain[:-1])


# ------------------------------------------------------------- conditions ---

def _flash_condition(g, chain, ns) -> bool:
    """The reference's condition on :flash_attention: the first node's value
    has at least 2 dims and more than 512 rows (src/compiler_config.jl:107-112)."""
    nd = g.nodes[ns].get(chain[0])
    v = None if nd is None else nd.value
    return v is not None and v.dim() >= 2 and v.shape[0] > 512


def _naive_attention_condition(g, chain, ns) -> bool:
    """matmul(Q, K; trans_b=true) -> scale_mask -> softmax -> matmul(P, V): the
    per-head naive attention of MultiHeadAttention (src/layers.jl:62-72),
    which is causal softmax(Q·Kᵀ/√d_head)·V — the :flash_attn op.  The last
    matmul must take the probabilities as its first operand, without
    transposition."""
    qk = producer(g, chain[0], ns)
    pv = producer(g, chain[3], ns)
    return (bool(qk.attrs.get("trans_b", False)) and len(qk.inputs) == 2
            and len(pv.inputs) == 2 and pv.inputs[0] == chain[2]
            and not pv.attrs.get("trans_b", False)
            and _head_dim(g, chain, qk, ns) == FLASH_HEAD_DIM)


# The attention kernels' head dimension: a rewrite onto :flash_attn or
# :flash_attention only applies to heads of this width, so a graph with
# other heads keeps its (GEMM-based) unfused form and still runs.
FLASH_HEAD_DIM = 64


def _head_dim(g, chain, qk, ns):
    """The head width of a naive attention chain: the :scale_mask's d_head
    attr, else the columns of Q's value when it is known, else None."""
    sm = producer(g, chain[1], ns)
    if "d_head" in sm.attrs:
        return int(sm.attrs["d_head"])
    nd = g.nodes[ns].get(qk.inputs[0])
    v = None if nd is None else nd.value
    return int(v.shape[1]) if v is not None and v.dim() == 2 else None


def _three_input_layernorm(g, chain, ns) -> bool:
    """:layernorm with [x, gamma, beta], so the fused op's inputs are
    [x, gamma, beta, W(, b)]."""
    return len(producer(g, chain[0], ns).inputs) == 3


# ------------------------------------------------------------------ rules ---

B200_RULES: List[RewriteRule] = [
    RewriteRule("naive_attention_to_flash", ("matmul", "scale_mask", "softmax", "matmul"),
                "flash_attn", condition=_naive_attention_condition, cost_delta=0.70,
                attrs={"causal": True}),
    # the reference's names (src/compiler_config.jl:154-172) keep their
    # patterns; the :linear forms (weight (out, in), optional bias) are extra
    RewriteRule("layernorm_linear_fusion", ("layernorm", "matmul"), "fused_layernorm_linear",
                condition=_three_input_layernorm, cost_delta=0.40),
    RewriteRule("layernorm_linear_bias_fusion", ("layernorm", "linear"),
                "fused_layernorm_linear", condition=_three_input_layernorm, cost_delta=0.40,
                attrs={"trans_b": True}),
    RewriteRule("linear_gelu_fusion", ("matmul", "gelu"), "fused_linear_gelu", cost_delta=0.35),
    RewriteRule("linear_bias_gelu_fusion", ("linear", "gelu"), "fused_linear_gelu",
                cost_delta=0.35, attrs={"trans_b": True}),
    RewriteRule("linear_residual_fusion", ("linear", "add"), "fused_linear_residual",
                cost_delta=0.30),
]

# fused ops with a backward rule (none of the B200 operators has one)
BACKWARD_SUPPORT = {"identity"}


# ------------------------------------------------------------------- cost ---

_GEMM_OPS = {"matmul", "fused_matmul_relu", "fused_linear_gelu", "fused_matmul_sigmoid",
             "scaled_matmul", "fused_rmsnorm_linear", "fused_layernorm_linear",
             "fused_matmul_add", "fused_linear_residual", "linear"}
_ELEMENTWISE_OPS = {"relu", "gelu", "sigmoid", "tanh", "softmax", "scale", "add", "wsum", "nsum",
                    "scale_add", "scale_mask"}
_ATTENTION_OPS = {"softmax_attn", "flash_attention", "flash_attn"}


def _numel(shape) -> int:
    n = 1
    for x in shape:
        n *= int(x)
    return n


def symbolic_cost(op: str, shapes) -> float:
    """A size-based cost of `op` on inputs of the given shapes, in the units of
    the reference's symbolic model (src/compiler_config.jl:230-267): GEMMs
    M·K·N / 1e9 from the first two operands, elementwise ops volume / 1e8,
    norms volume / 5e7, attention S²·d / 1e9, pure restructuring 0, anything
    else volume / 5e7.  The B200 ops are placed in the matching class."""
    shapes = [tuple(s) for s in shapes]
    if not shapes:
        return 0.0
    if op in _GEMM_OPS:
        if len(shapes) < 2:
            return 0.0
        a, b = shapes[0], shapes[1]
        M = a[0] if len(a) >= 1 else 1
        K = a[1] if len(a) >= 2 else 1
        N = b[1] if len(b) >= 2 else (b[0] if len(b) >= 1 else 1)
        return M * K * N / 1e9
    if op in _ELEMENTWISE_OPS:
        return _numel(shapes[0]) / 1e8
    if op in ("layernorm", "rmsnorm"):
        return _numel(shapes[0]) / 5e7
    if op in _ATTENTION_OPS:
        s = shapes[0]
        seq = s[0] if len(s) >= 1 else 1
        d = s[1] if len(s) >= 2 else 1
        return seq * seq * d / 1e9
    if op in ("transpose", "identity", "double_transpose_elim"):
        return 0.0
    return _numel(shapes[0]) / 5e7


def default_cost(op: str, shapes, rule_cost_delta: float = 0.0) -> float:
    """symbolic_cost less the rule's declared saving, never below zero
    (src/compiler_config.jl:278-283)."""
    return max(0.0, symbolic_cost(op, shapes) - rule_cost_delta)


# Rule pairs that rewrite the same pattern instance into alternative ops; when
# both match at the same root node only the cheaper survives
# (src/compiler_rules.jl:696).
ALTERNATIVE_RULE_PAIRS: List[Tuple[str, str]] = [("sdpa_fusion", "flash_attention")]


@dataclass
class CompilerConfig:
    """The reference's CompilerConfig fields (src/compiler_config.jl:349-359)
    plus `pooled`.  `budget` bounds the fusions one compilation applies;
    `incremental=False` makes every recompilation a full one; `verify_rules`
    warns for each applied rule not marked verified.  Only the GPU target and
    the symbolic cost mode exist here; `inspect` keeps no e-graph (the
    matching is direct) and is accepted for compatibility."""
    rules: List[RewriteRule] = field(default_factory=lambda: list(B200_RULES))
    training: bool = True
    pooled: bool = True      # run with the memory plan's buffer pool
    cost_fn: Callable = default_cost   # (op, shapes, rule_cost_delta=...) -> float
    budget: int = 1000
    target: str = "gpu"
    incremental: bool = True
    inspect: bool = False
    cost_mode: str = "symbolic"
    verify_rules: bool = False

    def __post_init__(self):
        if str(self.target).lstrip(":") != "gpu":
            raise ValueError(f"target {self.target!r}: this library runs on the GPU only")
        if str(self.cost_mode).lstrip(":") != "symbolic":
            raise ValueError(f"cost_mode {self.cost_mode!r}: only the symbolic cost model exists")
        if self.budget < 0:
            raise ValueError("budget must be >= 0")


@dataclass
class CompiledPlan:
    namespace: str
    order: List[str]
    fused_ops: Dict[str, str]
    config: CompilerConfig
    memory_plan: Optional[L.MemoryPlan] = None
    pool: Optional[L.BufferPool] = None
    dirty_nodes: Set[str] = field(default_factory=set)
    n_recompiles: int = 0
    compiled_at: float = 0.0

    def is_dirty(self) -> bool:
        return bool(self.dirty_nodes)

    def __call__(self, g, output_sym, ctx_store=None):
        """Run the compiled graph up to `output_sym` (the reference's
        plan(g, output_sym), src/compiler.jl:204-240), recompiling first when
        a set_ since the last compilation invalidated one of its nodes.  With
        the buffer pool, every intermediate's buffer returns to the pool when
        its liveness interval ends and later nodes reuse it — except, with
        `training=True`, a backpropagable (Quantom) node, whose forward value
        a backward pass needs (a CtxStore holds buffers that later nodes
        overwrite: keep it for unpooled runs)."""
        if self.is_dirty():
            recompile(self, g)
        if self.config.pooled and self.memory_plan is not None:
            return L.run_planned(g, self.memory_plan, self.pool, output_sym, self.namespace,
                                 ctx_store, training=self.config.training)
        return G.demand(g, output_sym, ctx_store=ctx_store, namespace=self.namespace)


def scan_graph(g, rules=None, namespace=None) -> List[RuleMatch]:
    ns = namespace or g.active_ns
    rules = B200_RULES if rules is None else rules
    if ns not in g.rules:
        return []
    matches: List[RuleMatch] = []
    for rule in rules:
        if not rule.pattern:
            continue
        for sym, r in list(g.rules[ns].items()):
            if r.op != rule.pattern[0]:
                continue
            chain = [sym]
            ok = True
            for expected in rule.pattern[1:]:
                nxt = single_consumer(g, chain[-1], ns)
                if nxt is None or op_of(g, nxt, ns) != expected:
                    ok = False
                    break
                chain.append(nxt)
            if not ok:
                continue
            if len(chain) > 1 and not _is_fuseable_chain(g, chain, ns):
                continue
            if rule.condition is not None:
                try:
                    if not rule.condition(g, chain, ns):
                        continue
                except Exception:   # a failing condition makes the rule inapplicable
                    continue
            matches.append(RuleMatch(rule, chain, ns, rule.cost_delta))
    matches.sort(key=lambda m: -m.score)
    return matches


def _match_cost(g, m: RuleMatch, cost_fn, ns) -> float:
    """cost_fn of the match's result on the shapes of its nodes' current
    values; a match with no known shape never wins (src/compiler_rules.jl:704-713)."""
    shapes = [tuple(nd.value.shape) for nd in (g.nodes[ns].get(s) for s in m.nodes)
              if nd is not None and nd.value is not None]
    if not shapes:
        return float("inf")
    return float(cost_fn(m.rule.result, shapes, rule_cost_delta=m.rule.cost_delta))


def choose_cheapest_alternative(g, matches: List[RuleMatch], cost_fn=default_cost,
                                namespace=None) -> List[RuleMatch]:
    """For each pair in ALTERNATIVE_RULE_PAIRS, of two matches (one of each
    rule) with the same root node keep the one of lower cost — the first on a
    tie; every other match stays (src/compiler_rules.jl:725-750)."""
    ns = namespace or g.active_ns
    drop = set()
    for name_a, name_b in ALTERNATIVE_RULE_PAIRS:
        ia_all = [i for i, m in enumerate(matches) if m.rule.name == name_a]
        ib_all = [i for i, m in enumerate(matches) if m.rule.name == name_b]
        for ia in ia_all:
            for ib in ib_all:
                if ia in drop or ib in drop or matches[ia].nodes[0] != matches[ib].nodes[0]:
                    continue
                ca = _match_cost(g, matches[ia], cost_fn, ns)
                cb = _match_cost(g, matches[ib], cost_fn, ns)
                drop.add(ib if ca <= cb else ia)
    return [m for i, m in enumerate(matches) if i not in drop]


def _apply_fusion(g, ns, chain, rule: RewriteRule, training=True) -> bool:
    fused_op = rule.result
    if training and fused_op != "identity" and fused_op not in BACKWARD_SUPPORT:
        return False
    if any(s not in g.rules[ns] or g.rules[ns][s].op != op
           for s, op in zip(chain, rule.pattern)):
        return False       # an earlier fusion took or rewrote part of this chain
    for a, b in zip(chain[:-1], chain[1:]):
        users = consumers(g, a, ns)
        if len(users) != 1 or users[0] != b:
            return False
    rules = [g.rules[ns][s] for s in chain]
    merged: Dict[str, Any] = {}
    for r in rules:
        merged.update(r.attrs)
    merged.update(rule.attrs)
    intermediate = {r.output for r in rules[:-1]}
    fused_inputs: List[str] = []
    for r in rules:
        for inp in r.inputs:
            if inp not in intermediate and inp not in fused_inputs:
                fused_inputs.append(inp)
    out = rules[-1].output
    for s in chain[:-1]:
        del g.rules[ns][s]
        del g.nodes[ns][s]
    del g.rules[ns][chain[-1]]
    G.addrule(g, G.GraphRule(out, fused_inputs, fused_op, attrs=merged, namespace=ns))
    G._invalidate_downstream(g, out, ns)
    return True


def _multihead_sources(g, ns, heads):
    """If the :hcat_heads inputs `heads` are the per-head :flash_attn nodes of
    a MultiHeadFlashAttention layer (src/flash_attention.jl:232-256) — head h
    reads columns h·D+1 .. (h+1)·D of the same three projections through
    :slice_cols, every intermediate read only by the next step — return
    ((q_full, k_full, v_full), D, causal, nodes to delete); else None."""
    rules = g.rules[ns]
    full: List[Optional[str]] = [None, None, None]
    D = None
    causal = None
    dead: Dict[str, None] = {}
    for h, sym in enumerate(heads):
        fa = rules.get(sym)
        if fa is None or fa.op != "flash_attn" or len(fa.inputs) != 3 or sym in dead:
            return None
        if len(consumers(g, sym, ns)) != 1:
            return None
        c = bool(fa.attrs.get("causal", True))
        if causal is not None and c != causal:
            return None
        causal = c
        for j, sl in enumerate(fa.inputs):
            sr = rules.get(sl)
            if sr is None or sr.op != "slice_cols" or len(sr.inputs) != 1:
                return None
            if consumers(g, sl, ns) != [sym]:
                return None
            if "start_col" not in sr.attrs or "end_col" not in sr.attrs:
                return None
            start, end = int(sr.attrs["start_col"]), int(sr.attrs["end_col"])
            if D is None:
                D = end - start + 1
            if D <= 0 or end - start + 1 != D or start != h * D + 1:
                return None
            if full[j] is None:
                full[j] = sr.inputs[0]
            elif full[j] != sr.inputs[0]:
                return None
            dead[sl] = None
        if int(fa.attrs.get("d_head", D)) != D:
            return None
        dead[sym] = None
    if D != FLASH_HEAD_DIM:
        return None
    return (full[0], full[1], full[2]), D, causal, list(dead)


def fold_multihead_attention(g, namespace=None) -> Dict[str, str]:
    """Rewrite each MultiHeadFlashAttention layer — 3·H :slice_cols, H
    :flash_attn and the :hcat_heads of their outputs — into one
    :flash_attention over the three projections: the kernel reads every head
    in place through strides and writes the concatenated output, so the
    3·H + 1 copies disappear.  The output keeps the :hcat_heads node's name.
    Returns {output: "flash_attention"} for each layer folded."""
    ns = namespace or g.active_ns
    folded: Dict[str, str] = {}
    for out, r in list(g.rules[ns].items()):
        if r.op != "hcat_heads" or not r.inputs:
            continue
        found = _multihead_sources(g, ns, r.inputs)
        if found is None:
            continue
        (q_full, k_full, v_full), D, causal, dead = found
        n_heads = len(r.inputs)
        for s in dead:
            del g.rules[ns][s]
            del g.nodes[ns][s]
        del g.rules[ns][out]
        G.addrule(g, G.GraphRule(out, [q_full, k_full, v_full], "flash_attention",
                                 attrs={"n_heads": n_heads, "d_head": D, "causal": causal},
                                 namespace=ns))
        G._invalidate_downstream(g, out, ns)
        folded[out] = "flash_attention"
    return folded


def _warn_unverified(config: CompilerConfig, rule: RewriteRule):
    if config.verify_rules and not rule.verified:
        warnings.warn(f"rewrite rule :{rule.name} is not verified")


def _fold_allowed(training) -> bool:
    # the same training guard as the rewrite rules
    return not training or "flash_attention" in BACKWARD_SUPPORT


def compile(g, config: Optional[CompilerConfig] = None, namespace=None) -> CompiledPlan:
    """Scan, apply the matches in decreasing score, fold multi-head layers
    into :flash_attention, recompute the order."""
    config = config or CompilerConfig()
    ns = namespace or g.active_ns
    fused_ops: Dict[str, str] = {}
    matches = choose_cheapest_alternative(g, scan_graph(g, config.rules, ns), config.cost_fn, ns)
    for m in matches:
        if len(fused_ops) >= config.budget:
            break
        if _apply_fusion(g, ns, m.nodes, m.rule, training=config.training):
            fused_ops[m.nodes[-1]] = m.rule.result
            _warn_unverified(config, m.rule)
    if _fold_allowed(config.training):
        fused_ops.update(fold_multihead_attention(g, ns))
    g._topo_cache[ns] = None
    order = G.topo_order(g, ns)
    memory_plan = L.plan_memory(g, ns)
    plan = CompiledPlan(ns, order, fused_ops, config, memory_plan, L.BufferPool(g.device),
                        compiled_at=time.time())
    _register_dirty_tracking(plan, g, ns)
    return plan


def _register_dirty_tracking(plan: CompiledPlan, g, ns):
    """Every node of the plan reports its invalidation (a set_ upstream) into
    plan.dirty_nodes (src/compiler.jl:126-131)."""
    def mark(_g, sym, _ns, plan=plan):
        plan.dirty_nodes.add(sym)
    for sym in plan.order:
        nd = g.nodes[ns].get(sym)
        if nd is not None:
            nd.on_change = mark


def is_dirty(plan: CompiledPlan) -> bool:
    return plan.is_dirty()


def recompile(plan: CompiledPlan, g) -> CompiledPlan:
    """recompile!(plan, g) (src/compiler.jl:142-191): a no-op for a clean
    plan; otherwise the rules are applied again, but only to matches that
    touch the region downstream of the dirty nodes, and the order and memory
    plan are recomputed.  A graph that gained nodes since the last
    compilation is compiled afresh."""
    if not plan.is_dirty():
        return plan
    ns = plan.namespace
    if not plan.config.incremental or len(g.nodes[ns]) != len(plan.order):
        fresh = compile(g, plan.config, namespace=ns)
        plan.order, plan.memory_plan = fresh.order, fresh.memory_plan
        plan.pool, plan.fused_ops = fresh.pool, fresh.fused_ops
        _register_dirty_tracking(plan, g, ns)
    else:
        affected: Set[str] = set()
        queue = list(plan.dirty_nodes)
        while queue:
            sym = queue.pop()
            if sym in affected:
                continue
            affected.add(sym)
            queue.extend(consumers(g, sym, ns))
        matches = choose_cheapest_alternative(g, scan_graph(g, plan.config.rules, ns),
                                              plan.config.cost_fn, ns)
        for m in matches:
            if not affected.intersection(m.nodes):
                continue
            if _apply_fusion(g, ns, m.nodes, m.rule, training=plan.config.training):
                plan.fused_ops[m.nodes[-1]] = m.rule.result
                _warn_unverified(plan.config, m.rule)
        if _fold_allowed(plan.config.training):
            plan.fused_ops.update(fold_multihead_attention(g, ns))
        g._topo_cache[ns] = None
        plan.order = G.topo_order(g, ns)
        plan.memory_plan = L.plan_memory(g, ns)
        _register_dirty_tracking(plan, g, ns)
    plan.dirty_nodes.clear()
    plan.n_recompiles += 1
    plan.compiled_at = time.time()
    return plan
