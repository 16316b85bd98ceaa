"""Liveness, slot assignment and the buffer pool of a compiled graph
(src/liveness.jl restated over the operator-API mirror).

  reference (Julia)                                here
  -----------------------------------------------  -----------------------------
  LivenessInterval  src/liveness.jl:20-24          LivenessInterval
  BufferPool / acquire! / release! / pool_stats    BufferPool.acquire / release /
    src/liveness.jl:29-68                            stats
  compute_liveness  src/liveness.jl:83-113         compute_liveness
  greedy_interval_coloring  :130-158               greedy_interval_coloring
  MemoryPlan                                       MemoryPlan
  plan_memory!  src/liveness.jl:198-207            plan_memory_pool (plan_memory
                                                   returns the plan alone)
  demand_planned!  src/liveness.jl:217-257         demand_planned

A node lives from the topological step that computes it to the last step
that reads it; parameters live to the end.  The greedy sweep gives every node
the lowest slot free at its first step, so the slot count bounds how many
intermediate buffers a run holds at once.  The pool hands out device buffers
keyed by (shape, dtype) and takes them back when a node's interval has ended;
a second run of the same plan reuses every buffer instead of allocating.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Tuple

import torch

from . import graph as G


@dataclass(frozen=True)
class LivenessInterval:
    first_use: int
    last_use: int

    def is_alive_at(self, t: int) -> bool:
        return self.first_use <= t <= self.last_use


class BufferPool:
    """Reusable device buffers bucketed by (shape, dtype)."""

    def __init__(self, device):
        self.device = device if isinstance(device, torch.device) else device.torch_device
        self.buckets: Dict[Tuple, List[torch.Tensor]] = {}
        self.n_alloc = 0
        self.n_hits = 0

    def acquire(self, shape, dtype=torch.float32) -> torch.Tensor:
        key = (tuple(shape), dtype)
        b = self.buckets.get(key)
        if b:
            self.n_hits += 1
            return b.pop()
        self.n_alloc += 1
        return torch.zeros(tuple(shape), dtype=dtype, device=self.device)

    def release(self, buf: torch.Tensor):
        self.buckets.setdefault((tuple(buf.shape), buf.dtype), []).append(buf)

    def stats(self):
        """pool_stats (src/liveness.jl:64-68): allocations, hits and the hit
        rate in percent."""
        total = self.n_alloc + self.n_hits
        rate = round(100.0 * self.n_hits / total, 1) if total else 0.0
        return {"allocs": self.n_alloc, "hits": self.n_hits, "hit_rate_pct": rate}


def compute_liveness(g, namespace=None) -> Dict[str, LivenessInterval]:
    ns = namespace or g.active_ns
    order = G.topo_order(g, ns)
    n = len(order)
    idx = {s: i + 1 for i, s in enumerate(order)}
    last = {s: idx[s] for s in order}
    for out, r in g.rules[ns].items():
        j = idx.get(out, 0)
        for s in r.inputs:
            if s in last and j > last[s]:
                last[s] = j
    live = {}
    for s in order:
        nd = g.nodes[ns].get(s)
        lu = last[s]
        # parameters live for the whole pass; a backpropagable (Quantom) node's
        # forward value is read by the backward pass, so it lives to the end as
        # well (src/liveness.jl:101-108) — in inference its buffer goes back to
        # the pool at the last step; Datom intermediates end at their last reader
        if nd is not None and (nd.is_param or G.is_backpropable(nd)):
            lu = n
        live[s] = LivenessInterval(idx[s], lu)
    return live


def greedy_interval_coloring(liveness: Dict[str, LivenessInterval], order: List[str]):
    slot_of: Dict[str, int] = {}
    free: List[int] = []
    active: Dict[str, int] = {}
    next_slot = 1
    for s in sorted(order, key=lambda x: liveness[x].first_use):
        iv = liveness[s]
        for a in [a for a, lu in active.items() if lu < iv.first_use]:
            free.append(slot_of[a])
            del active[a]
        free.sort()
        slot = free.pop(0) if free else next_slot
        next_slot = max(next_slot, slot + 1)
        slot_of[s] = slot
        active[s] = iv.last_use
    return slot_of


@dataclass
class MemoryPlan:
    slot_of: Dict[str, int]
    liveness: Dict[str, LivenessInterval]
    n_slots: int
    order: List[str] = field(default_factory=list)

    def peak_live(self) -> int:
        """Most nodes alive at one step of the order."""
        return max((sum(1 for s in self.order if self.liveness[s].is_alive_at(t))
                    for t in range(1, len(self.order) + 1)), default=0)

    def __str__(self):
        """The reference's summary of a plan (src/liveness.jl:172-185): nodes,
        slots, peak of simultaneously live nodes, and the reduction against
        one buffer per node."""
        n = len(self.order)
        return (f"MemoryPlan:\n  Nodes     : {n}\n"
                f"  Slots     : {self.n_slots}  (distinct physical buffers)\n"
                f"  Peak live : {self.peak_live()}  nodes at once\n"
                f"  Reduction : -{100 * (1 - self.n_slots / max(1, n)):.0f}% vs naive "
                "(1 buffer / node)")


def plan_memory(g, namespace=None) -> MemoryPlan:
    ns = namespace or g.active_ns
    order = G.topo_order(g, ns)
    live = compute_liveness(g, ns)
    slot_of = greedy_interval_coloring(live, order)
    return MemoryPlan(slot_of, live, max(slot_of.values(), default=0), order)


def execute_rule_pooled(g, rule, pool: BufferPool, ctx_store=None):
    """execute_rule_pooled! (src/dispatch.jl:163): the output buffer comes
    from the pool instead of a fresh allocation; the op overwrites it."""
    ns = rule.namespace
    out_node = g.nodes[ns][rule.output]
    inputs = []
    for s in rule.inputs:
        v = g.nodes[ns][s].value
        if not isinstance(v, torch.Tensor):
            raise G.NeuroDSLError(1, f":{s} has no value (input of :{rule.output})")
        inputs.append(v)
    shape = G._infer_output_shape(rule.op, inputs, rule.attrs)
    dtype = rule.attrs.get("out_dtype", torch.float32)
    v = out_node.value
    if v is None or tuple(v.shape) != tuple(shape) or v.dtype != dtype:
        if v is not None:
            pool.release(v)
        out_node.value = pool.acquire(shape, dtype)
    G._dispatch_op(g.device, out_node.value, rule.op, inputs, rule.attrs, rule.output, out_node,
                   ctx_store)
    out_node.valid = True
    return out_node.value


def run_planned(g, plan: MemoryPlan, pool: BufferPool, output_sym, namespace=None,
                ctx_store=None, training=False):
    """Run the graph in plan order up to `output_sym` with pooled outputs and
    return every computed node's buffer to the pool once its interval has
    ended (the reference's CompiledPlan call, src/compiler.jl:204-240).  The
    requested output stays; nodes without a rule (inputs, parameters) are
    never released, since their values belong to the caller; with
    `training`, neither is a backpropagable (Quantom) node, whose forward
    value a backward pass reads (src/compiler.jl:233)."""
    ns = namespace or g.active_ns
    held: List[str] = []
    for step, sym in enumerate(plan.order, start=1):
        nd = g.nodes[ns][sym]
        if not (nd.valid and nd.value is not None) and sym in g.rules[ns]:
            execute_rule_pooled(g, g.rules[ns][sym], pool, ctx_store)
            if not (training and issubclass(nd.atom_type, G.Quantom)):
                held.append(sym)
        for prev in list(held):
            if prev == output_sym:
                continue
            if plan.liveness[prev].last_use <= step:
                pnd = g.nodes[ns][prev]
                pool.release(pnd.value)
                pnd.value = None
                pnd.valid = False
                held.remove(prev)
        if sym == output_sym:
            break
    return g.nodes[ns][output_sym].value


def pool_stats(pool: BufferPool):
    return pool.stats()


def plan_memory_pool(g, namespace=None):
    """plan_memory!(g) (src/liveness.jl:198-207): the memory plan and an empty
    buffer pool on the graph's device."""
    return plan_memory(g, namespace), BufferPool(g.device)


def demand_planned(g, sym, plan: MemoryPlan, pool: BufferPool, ctx_store=None,
                   namespace=None):
    """demand_planned!(g, sym, plan, pool) (src/liveness.jl:217-257): a valid
    node's value as is, otherwise the planned run up to `sym` with pooled
    buffers, each released once its interval has ended."""
    ns = namespace or g.active_ns
    if ns not in g.nodes or sym not in g.nodes[ns]:
        raise G.NeuroDSLError(1, f":{sym} introuvable dans :{ns}")
    nd = g.nodes[ns][sym]
    if nd.valid and nd.value is not None:
        return nd.value
    return run_planned(g, plan, pool, sym, ns, ctx_store)
