"""Benchmark of the NeuroDSL B200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one step): causal attention prefill at batch 8, 16 heads, head_dim
64, sequence 2048, bf16 Q/K/V ~ N(0,1), fp32 accumulation — one call of the
library's prefill kernel over all 128 (batch, head) pairs.  Metric: attention
TFLOP/s with the algorithmic causal count 4·B·H·D·S(S+1)/2 per step.  The same
JSON line carries the KV-cache decode workload (batch 64, 12 heads, head_dim
64, cache 1024 -> 1152 over 128 appending steps) as tokens/s, each with its
roofline against the measured B200 peaks, the fused GEMM + bias + GELU and
LayerNorm kernels on their own shapes, and two whole decoders assembled from
the library (prefill tokens/s and greedy-decode tokens/s): GPT-2 small
(batch 16, prompt 512, 256 tokens; one replica per GPU) and a 24-layer d=1024
model (batch 32, prompt 2048, 512 tokens; tensor-parallel over all GPUs).
The decoders' prefill is replayed from one CUDA graph and their decode steps
from graphs of several steps each; token ids stay on the device throughout.

Multi-GPU: one process per GPU (torchrun); every rank runs its own full
workload (independent batches, no collective on the data path) and the job
value is the sum over ranks divided by the slowest rank's time (weak scaling).

--impl reference times the reference's CPU path restated by the oracle
(the Julia reference cannot run on this machine) on all host threads, on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from neurodsl_b200.ranks import dist_env  # noqa: E402  (no CUDA library load)

B, H, S, D = 8, 16, 2048, 64
FLOPS_PER_STEP = 4 * B * H * D * S * (S + 1) // 2          # 68,753,031,168
DEC_B, DEC_H, DEC_L0, DEC_T = 64, 12, 1024, 128
METRIC = "Attn prefill TFLOP/s + KV-decode tokens/s (dim 1024), % of B200 roofline"
N_SETS = 3  # rotating input sets: 3 x 134 MB > 126 MB L2


def dec_bytes(L):
    """Algorithmic HBM bytes of one decode step over L keys: K and V read,
    q read, new K/V written, output written (bf16)."""
    return 2 * DEC_B * DEC_H * L * D * 2 + DEC_B * DEC_H * D * 2 * 4


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"],
                "bf16_tflops_sustained": j.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic(name):
    """Per-launch DRAM bytes from a committed ncu summary (profiles/<name>.md,
    line 'dram_bytes_per_launch = <int>'), or None."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("dram_bytes_per_launch"):
            try:
                return int(float(line.split("=")[1].strip().split()[0]))
            except (IndexError, ValueError):
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        return self.summarise(self.lines)

    @staticmethod
    def summarise(lines):
        """Median SM clock under load, the max clock and every throttle
        reason seen Active in the sampled CSV lines."""
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() in ("active", "1"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def barrier():
    """Barrier over all ranks (a no-op for one process)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def max_over_ranks(x, device=None):
    """Max of a per-rank time over all ranks (identity for one process)."""
    from neurodsl_b200 import ranks
    return ranks.max_over_ranks(x, device=device)


def cpu_model():
    """The host CPU's model name (first 'model name' line of /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# --------------------------------------------------------------- CPU arm ---

def cpu_prefill_sample(min_seconds=10.0, nthreads=0):
    """Time the oracle's restatement of the reference CPU attention on a bounded
    sample of (batch, head) pairs of the prefill workload; returns
    (TFLOP/s with the algorithmic causal count, threads, sample description)."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(0)
    nh = 8
    Q = oracle.bf16_round(rng.standard_normal((1, nh, S, D), dtype=np.float32))
    K = oracle.bf16_round(rng.standard_normal((1, nh, S, D), dtype=np.float32))
    V = oracle.bf16_round(rng.standard_normal((1, nh, S, D), dtype=np.float32))
    threads = nthreads or os.cpu_count() or 1
    oracle.attn_bhsd(Q[:, :1], K[:, :1], V[:, :1], causal=True, nthreads=threads)  # warm
    reps = 0
    t0 = time.perf_counter()
    while True:
        oracle.attn_bhsd(Q, K, V, causal=True, nthreads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or reps >= 64:
            break
    flops = reps * nh * 4 * D * S * (S + 1) // 2
    return flops / el / 1e12, threads, f"{reps}x{nh} heads of S={S}, D={D} (causal), {el:.1f}s"


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    vals = []
    desc = ""
    # each step is a bounded sample; the whole run stays within ~2 minutes
    per_step = min(args.ref_seconds, 120.0 / max(1, args.warmup + args.steps))
    for i in range(args.warmup + args.steps):
        v, threads, desc = cpu_prefill_sample(min_seconds=per_step, nthreads=threads)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": FLOPS_PER_STEP / (value * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), bf16-rounded)",
        "config": {"workload": f"causal attention prefill B={B} H={H} S={S} D={D}",
                   "path": "oracle restatement of flash_attn_fwd_cpu_simple! "
                           "(src/flash_attention.jl:49-69); Julia reference not runnable here"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(), "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------- GPU arm ---

def _gather_vocab(logits, V, tp, group):
    """Full-vocabulary logits [rows][V] from the ranks' slices of a
    tensor-parallel LM head (rank r holds rows [r·ceil(V/tp), ...))."""
    import torch
    w = (V + tp - 1) // tp
    pad = torch.full((logits.shape[0], w), float("nan"), device=logits.device)
    pad[:, :logits.shape[1]] = logits
    parts = [torch.empty_like(pad) for _ in range(tp)]
    torch.distributed.all_gather(parts, pad, group=group)
    return torch.cat(parts, dim=1)[:, :V]


def tp_parity(model, cfg, ids, group, tp, dev, steps=16):
    """Tensor-parallel decoder against the one-GPU model of the same seed on
    the same prompts: logits of the last prompt position (max-abs and
    relative L2 over the full vocabulary), the first `steps` greedy tokens of
    every row, and — so that a differing token can be told from a near tie —
    the largest logit difference over the steps before the first differing
    token and the one-GPU model's top-2 margin of each row where the tokens
    first differ.  Collective over the model's group; the one-GPU model runs
    on the group's first rank, which returns the result (others None)."""
    import torch
    import torch.distributed as dist

    from neurodsl_b200.model import GPT
    model.release_graphs()
    lgs = [_gather_vocab(model.prefill(ids, steps), cfg.vocab, tp, group)]
    for t in range(steps - 1):
        lgs.append(_gather_vocab(model.decode_step(t), cfg.vocab, tp, group))
    toks = model.tokens().clone()
    out = None
    if dist.get_rank(group) == 0:
        ref = GPT(cfg, seed=0, device=dev)
        rls = [ref.prefill(ids, steps).clone()]
        for t in range(steps - 1):
            rls.append(ref.decode_step(t).clone())
        rt = ref.tokens().clone()
        torch.cuda.synchronize()
        full, rl = lgs[0], rls[0]
        eq = (toks == rt)
        first = None
        margins = []
        dev_before = 0.0
        if not bool(eq.all()):
            bad = (~eq).nonzero()
            first = int(bad[:, 1].min())
            for r in bad[bad[:, 1] == first][:, 0].tolist():
                top2 = torch.topk(rls[first][r], 2).values
                margins.append(float(top2[0] - top2[1]))
        for k in range(first if first is not None else steps):
            dev_before = max(dev_before, float((lgs[k] - rls[k]).abs().max()))
        out = {"reference": "one-GPU model, same seed and prompts",
               "logits_max_abs": float((full - rl).abs().max()),
               "logits_rel_l2": float((full - rl).norm() / rl.norm()),
               "tokens_equal": bool(eq.all()), "tokens_checked": int(eq.numel()),
               "first_differing_step": first,
               "decode_logits_max_abs_before_first_difference": dev_before,
               "one_gpu_top2_margin_where_first_different": margins}
        del ref
        torch.cuda.empty_cache()
    return out


def model_line(name, cfg, B, S, steps, tp, groups, dev, peaks, reps, chunk, parity,
               split_batch=False):
    """Prefill and greedy decode of a GPT-style decoder built from the library
    (neurodsl_b200.model).  The world is split into world/tp groups of tp
    consecutive ranks; each group runs one tensor-parallel model (prompt-
    sharded prefill writing the keys/values into the owning ranks' caches;
    decode with the row-parallel projection fused with the NVLink exchange)
    on its own batch.  tp == world: one model over all GPUs (strong scaling);
    tp == 1: one replica per GPU (weak scaling), or with split_batch one
    global batch of B·world prompts split over the replicas (strong)."""
    import torch
    import torch.distributed as dist

    from neurodsl_b200.model import GPT, decode_weight_bytes, flops_prefill
    rank, world, _ = dist_env()
    dp = world // tp
    gi = rank // tp
    group = groups.get((tp, gi)) if tp > 1 else None
    model = GPT(cfg, seed=0, device=dev, tp=tp, rank=rank % tp if tp > 1 else 0, group=group,
                nvlink_rows=B if tp > 1 else 0)
    gen = torch.Generator(device=dev).manual_seed(99 + (gi if tp > 1 else rank))
    ids = torch.randint(0, cfg.vocab, (B, S), device=dev, dtype=torch.int32, generator=gen)
    graphs = True
    try:
        model.generate(ids, steps, graph_chunk=chunk, graph_prefill=True)
    except Exception:  # collectives that cannot be captured: run eagerly
        graphs = False
        model.release_graphs()
        torch.cuda.synchronize()
        model.generate(ids, steps)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    tp_ms, td_ms = [], []
    for _ in range(reps):
        barrier()
        torch.cuda.synchronize()
        ev[0].record()
        if graphs:
            model.prefill_graphed(ids, steps)
        else:
            model.prefill(ids, steps)
        ev[1].record()
        if graphs:
            for g in model._graphs:
                g.replay()
        else:
            for t in range(steps - 1):
                model.decode_step(t)
        ev[2].record()
        torch.cuda.synchronize()
        tp_ms.append(ev[0].elapsed_time(ev[1]))
        td_ms.append(ev[1].elapsed_time(ev[2]))
    p_ms = max_over_ranks(min(tp_ms), dev)
    d_ms = max_over_ranks(min(td_ms), dev)
    tokens = model.tokens()[:, :4].cpu().tolist()
    # tensor-parallel models prefill with the prompts sharded over the ranks;
    # the Megatron prefill (sharded weights, two all-reduces per layer,
    # overlapped in two sequence groups) is timed beside it
    p_ms_tp = None
    if tp > 1 and model.prefill_mode == "dp" and B % tp == 0:
        model.prefill_mode = "tp"
        model._prefill_graph, model._prefill_key = None, None
        t_tp = []
        for _ in range(reps):
            barrier()
            torch.cuda.synchronize()
            ev[0].record()
            if graphs:
                model.prefill_graphed(ids, steps)
            else:
                model.prefill(ids, steps)
            ev[1].record()
            torch.cuda.synchronize()
            t_tp.append(ev[0].elapsed_time(ev[1]))
        p_ms_tp = max_over_ranks(min(t_tp), dev)
        model.prefill_mode = "dp"
        model._prefill_graph, model._prefill_key = None, None
    par = None
    if parity and tp > 1:
        if gi == 0:
            par = tp_parity(model, cfg, ids, group, tp, dev)
        barrier()
    model.close()
    del model
    torch.cuda.synchronize()
    n_dec = steps - 1
    fl = flops_prefill(cfg, B, S)
    kv = sum(2 * B * cfg.n_layer * cfg.n_head * (S + t + 1) * 64 * 2 for t in range(n_dec))
    dec_bytes = decode_weight_bytes(cfg) * n_dec + kv   # one model, all its ranks together
    p_tflops = dp * fl / (p_ms * 1e-3) / 1e12
    d_gbs = dp * dec_bytes / (d_ms * 1e-3) / 1e9
    if tp == 1 and split_batch:
        layout = f"dp{world} replicas, global batch {B * world} split over them"
    elif tp == 1:
        layout = f"dp{world} replicas"
    elif dp == 1:
        layout = f"tp{tp}"
    else:
        layout = f"tp{tp} x dp{dp}"
    line = {
        "workload": f"{name}: {cfg.n_layer} layers d={cfg.d_model} {cfg.n_head}x64 heads "
                    f"F={cfg.d_ff} vocab {cfg.vocab}, batch {B} per model, prompt {S}, "
                    f"{steps} greedy tokens",
        "parallelism": layout,
        "reduction": ("prefill: prompts sharded over the ranks, keys/values to their heads' "
                      "ranks by one NCCL all-to-all per layer; decode: row-parallel projection "
                      "fused with the NVLink peer exchange, residual and LayerNorm")
                     if tp > 1 else None,
        "scaling": "strong" if ((tp > 1 and dp == 1) or split_batch) else "weak",
        "prefill": {"value": dp * B * S / (p_ms * 1e-3), "unit": "tokens/s", "ms": p_ms,
                    "launch": "one CUDA graph" if graphs else "eager launches",
                    "roofline": {"bound": "tensor", "achieved": p_tflops / world,
                                 "peak": peaks["bf16_tflops"], "unit": "TFLOP/s per GPU",
                                 "frac": p_tflops / world / peaks["bf16_tflops"]}},
        "decode": {"value": dp * B * n_dec / (d_ms * 1e-3), "unit": "tokens/s", "ms": d_ms,
                   "us_per_step": d_ms * 1e3 / n_dec,
                   "launch": "CUDA graphs" if graphs else "eager launches",
                   "roofline": {"bound": "hbm", "achieved": d_gbs / world,
                                "peak": peaks["hbm_gbs"], "unit": "GB/s per GPU",
                                "frac": d_gbs / world / peaks["hbm_gbs"],
                                "bytes": "bf16 weights + K/V read per step"}},
        "first_tokens": tokens[0],
    }
    if p_ms_tp is not None:
        line["prefill_tensor_parallel"] = {
            "value": dp * B * S / (p_ms_tp * 1e-3), "unit": "tokens/s", "ms": p_ms_tp,
            "how": "Megatron shards, NCCL all-reduce after the output and down projections, "
                   "two sequence groups on two streams"}
    if par is not None or (parity and tp > 1):
        line["tp_parity"] = par
    return line


def run_ours(args):
    import torch

    from neurodsl_b200 import ops
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    groups = {}
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        pg = dist
        # tensor-parallel groups of tp consecutive ranks (every rank creates
        # every group, in the same order)
        for tp in sorted({world, min(world, 4)}):
            for g in range(world // tp):
                members = list(range(g * tp, (g + 1) * tp))
                groups[(tp, g)] = dist.group.WORLD if tp == world else dist.new_group(members)

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = []
    for _ in range(N_SETS):
        q = torch.randn(B, H, S, D, device=dev, generator=gen).bfloat16()
        k = torch.randn(B, H, S, D, device=dev, generator=gen).bfloat16()
        v = torch.randn(B, H, S, D, device=dev, generator=gen).bfloat16()
        o = torch.empty(B, H, S, D, device=dev, dtype=torch.bfloat16)
        lse = torch.empty(B, H, S, device=dev)
        m = torch.empty(B, H, S, device=dev)
        sets.append((q, k, v, o, lse, m))
    stream = torch.cuda.current_stream()

    def step(i):
        q, k, v, o, lse, m = sets[i % N_SETS]
        ops.flash_attn_fwd(q, k, v, causal=True, out=o, lse=lse, row_max=m)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    # soak so the clock record covers steady-state load around the timed region
    t_end = time.time() + args.soak
    i = 0
    while time.time() < t_end:
        step(i)
        i += 1
        if i % 64 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()

    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_local = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms_local, dev)
    value = world * FLOPS_PER_STEP / (ms * 1e-3) / 1e12
    kernel_tflops = FLOPS_PER_STEP / (ms_local * 1e-3) / 1e12

    # ---- decode workload (128 appending steps per "step" of the decode line)
    L_max = DEC_L0 + DEC_T
    kc = torch.randn(DEC_B, DEC_H, L_max, D, device=dev, generator=gen).bfloat16()
    vc = torch.randn(DEC_B, DEC_H, L_max, D, device=dev, generator=gen).bfloat16()
    qs = torch.randn(DEC_T, DEC_B, DEC_H, D, device=dev, generator=gen).bfloat16()
    kns = torch.randn(DEC_T, DEC_B, DEC_H, D, device=dev, generator=gen).bfloat16()
    vns = torch.randn(DEC_T, DEC_B, DEC_H, D, device=dev, generator=gen).bfloat16()
    dout = torch.empty(DEC_B, DEC_H, D, device=dev, dtype=torch.bfloat16)
    dlse = torch.empty(DEC_B, DEC_H, device=dev)

    def decode_pass():
        for t in range(1, DEC_T + 1):
            ops.kv_decode_attn(qs[t - 1], kc, vc, DEC_L0 + t, k_new=kns[t - 1], v_new=vns[t - 1],
                               out=dout, lse=dlse)

    # warm-up outside capture (sizes the library's decode scratch), then the
    # 128 launch-bound steps are captured once in a CUDA graph and replayed
    for _ in range(max(1, args.warmup)):
        decode_pass()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        decode_pass()
    graph.replay()
    torch.cuda.synchronize()
    barrier()
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    dec_reps = max(1, args.decode_reps)
    d0.record(stream)
    for _ in range(dec_reps):
        graph.replay()
    d1.record(stream)
    torch.cuda.synchronize()
    barrier()
    dec_ms_local = d0.elapsed_time(d1) / dec_reps
    dec_ms = max_over_ranks(dec_ms_local, dev)
    dec_bytes_total = sum(dec_bytes(DEC_L0 + t) for t in range(1, DEC_T + 1))
    dec_tokens = world * DEC_B * DEC_T / (dec_ms * 1e-3)
    dec_gbs = dec_bytes_total / (dec_ms_local * 1e-3) / 1e9
    del graph

    # ---- fused linear + bias + GELU (the MLP-up of the 24-layer dim-1024
    # model's prefill: 32 x 2048 tokens, 1024 -> 4096) and LayerNorm over the
    # same tokens; each timed over `args.aux_reps` calls
    # Two rotating sets of inputs and outputs each (every set is larger than
    # the 126 MB L2), so no call finds its operands in L2 from the call before.
    gm, gn, gk = 65536, 4096, 1024
    gsets = [(torch.randn(gm, gk, device=dev, generator=gen).bfloat16(),
              (0.02 * torch.randn(gn, gk, device=dev, generator=gen)).bfloat16(),
              torch.empty(gm, gn, device=dev, dtype=torch.bfloat16)) for _ in range(2)]
    gb = torch.zeros(gn, device=dev)
    lsets = [(torch.randn(gm, gk, device=dev, generator=gen),
              torch.empty(gm, gk, device=dev, dtype=torch.bfloat16),
              torch.empty(gm, device=dev), torch.empty(gm, device=dev)) for _ in range(2)]

    def time_calls(fn, reps):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for i in range(reps):
            fn(i)
        a1.record(stream)
        torch.cuda.synchronize()
        return a0.elapsed_time(a1) / reps

    def gemm_call(i):
        ga, gw, gy = gsets[i & 1]
        ops.linear(ga, gw, gb, act="sigmoid", out=gy)

    def ln_call(i):
        lx, ly, lmean, lrstd = lsets[i & 1]
        ops.layernorm(lx, out=ly, mean=lmean, rstd=lrstd)

    gemm_ms = time_calls(gemm_call, args.aux_reps)
    gemm_tflops = 2.0 * gm * gn * gk / (gemm_ms * 1e-3) / 1e12
    ln_ms = time_calls(ln_call, args.aux_reps)
    ln_bytes = gm * gk * (4 + 2) + gm * 8
    ln_gbs = ln_bytes / (ln_ms * 1e-3) / 1e9
    del gsets, lsets
    clocks = sampler.stop()

    # ---- end to end through the public API with host buffers (pinned)
    hq = torch.randn(B, H, S, D, generator=torch.Generator().manual_seed(7)).bfloat16().pin_memory()
    hk = torch.randn(B, H, S, D, generator=torch.Generator().manual_seed(8)).bfloat16().pin_memory()
    hv = torch.randn(B, H, S, D, generator=torch.Generator().manual_seed(9)).bfloat16().pin_memory()
    ho = torch.empty(B, H, S, D, dtype=torch.bfloat16).pin_memory()
    # Steps are pipelined over two device buffer sets and three streams: the
    # inputs of step i+1 go host -> device while step i computes and step
    # i-1's output comes back, as a serving loop would run; every step still
    # copies its own inputs in and its output out inside the timed region.
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]
    out_done = [torch.cuda.Event(), torch.cuda.Event()]
    in_done = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_run(n):
        for i in range(n):
            j = i & 1
            dq, dk, dv, do, dl, dm = sets[j]
            with torch.cuda.stream(s_in):
                if i >= 2:   # set j is free once step i-2 computed and was read back
                    s_in.wait_event(comp_done[j])
                    s_in.wait_event(out_done[j])
                dq.copy_(hq, non_blocking=True)
                dk.copy_(hk, non_blocking=True)
                dv.copy_(hv, non_blocking=True)
                in_done[j].record(s_in)
            stream.wait_event(in_done[j])
            ops.flash_attn_fwd(dq, dk, dv, causal=True, out=do, lse=dl, row_max=dm)
            comp_done[j].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[j])
                ho.copy_(do, non_blocking=True)
                out_done[j].record(s_out)

    def joined_run(n):
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        e2e_run(n)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)

    joined_run(2)
    torch.cuda.synchronize()
    barrier()
    x0 = torch.cuda.Event(enable_timing=True)
    x1 = torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 20))
    x0.record(stream)
    joined_run(e2e_steps)
    x1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(x0.elapsed_time(x1) / e2e_steps, dev)
    e2e_value = world * FLOPS_PER_STEP / (e2e_ms * 1e-3) / 1e12
    h2d = 3 * B * H * S * D * 2
    d2h = B * H * S * D * 2

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, thr, desc = cpu_prefill_sample(min_seconds=args.cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": thr, "kind": "port",
               "cpu_model": cpu_model(), "sample": desc}

    peaks = load_peaks()
    models = {}
    if not args.no_model:
        from neurodsl_b200.model import GPT2_SMALL, GPT_24L_1024
        models["gpt2_small"] = model_line("GPT-2 small", GPT2_SMALL, 16, 512, 256, 1, groups, dev,
                                          peaks, 2, 32, False)
        if world > 1:
            # 12 heads: tensor parallel over at most 4 GPUs, data parallel beyond
            models["gpt2_small_tp"] = model_line("GPT-2 small", GPT2_SMALL, 16, 512, 256,
                                                 min(world, 4), groups, dev, peaks, 2, 32, True)
        models["gpt_24l_1024"] = model_line("24-layer", GPT_24L_1024, 32, 2048, 512, world, groups,
                                            dev, peaks, 2, 64, True)
        if world > 1 and 32 % world == 0:
            # the same 32 prompts as replicas of the whole model, 32/N per GPU
            # (no collective on the data path): the data-parallel counterpart
            models["gpt_24l_1024_dp"] = model_line("24-layer", GPT_24L_1024, 32 // world, 2048,
                                                   512, 1, groups, dev, peaks, 2, 64, False,
                                                   split_batch=True)
    traffic = load_traffic("flash_fwd_causal_b8_h16_s2048_d64")
    dec_traffic = load_traffic("kv_decode_b64_h12_l1024_d64")
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": f"causal attention prefill B={B} H={H} S={S} D={D} per GPU",
                       "flops_per_step": FLOPS_PER_STEP,
                       "l2": f"{N_SETS} rotating input sets of 134 MB (> 126 MB L2)",
                       "parallelism": f"dp{world} over independent batches"},
            "roofline": {"bound": "tensor", "achieved": kernel_tflops,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": kernel_tflops / peaks["bf16_tflops"],
                         "traffic": traffic, "peak_source": peaks["source"] + " burst bf16"},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "decode": {
                "workload": f"KV decode B={DEC_B} H={DEC_H} D={D} cache {DEC_L0}->{DEC_L0 + DEC_T}, "
                            f"{DEC_T} appending steps",
                "value": dec_tokens, "unit": "tokens/s", "ms_per_pass": dec_ms,
                "us_per_token_step": dec_ms * 1e3 / DEC_T,
                "gpu_launches": dec_reps * DEC_T,
                "launch": f"{DEC_T} steps captured in one CUDA graph, replayed; one "
                          f"kv_decode_kernel launch per step, {dec_reps} timed passes",
                "roofline": {"bound": "hbm", "achieved": dec_gbs, "peak": peaks["hbm_gbs"],
                             "unit": "GB/s", "frac": dec_gbs / peaks["hbm_gbs"],
                             "traffic": dec_traffic,
                             "bytes_per_pass": dec_bytes_total},
            },
            "gemm_bias_gelu": {
                "workload": f"Y = gelu_sigmoid(X W^T + b), X [{gm}][{gk}], W [{gn}][{gk}] bf16",
                "value": gemm_tflops, "unit": "TFLOP/s", "ms_per_call": gemm_ms,
                "gpu_launches": args.aux_reps,
                "roofline": {"bound": "tensor", "achieved": gemm_tflops,
                             "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": gemm_tflops / peaks["bf16_tflops"],
                             "traffic": load_traffic("gemm_bias_gelu_m65536_n4096_k1024")},
            },
            "layernorm": {
                "workload": f"LayerNorm rows={gm} d={gk}, fp32 in, bf16 out, fp32 stats",
                "value": ln_gbs, "unit": "GB/s", "ms_per_call": ln_ms,
                "gpu_launches": args.aux_reps,
                "roofline": {"bound": "hbm", "achieved": ln_gbs, "peak": peaks["hbm_gbs"],
                             "unit": "GB/s", "frac": ln_gbs / peaks["hbm_gbs"],
                             "traffic": load_traffic("layernorm_rows65536_d1024")},
            },
        }
        line.update(models)
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# entry points of neurodsl_b200.ops that a decode step calls
_STEP_OPS = ("embed", "layernorm", "add_layernorm", "linear", "ln_linear", "kv_decode_attn_qkv",
             "allreduce_add_layernorm", "gemm_allreduce_add_layernorm", "argmax")


def _op_times_of_step(model, t, dev):
    """Per-operation device times of decode step t: every call of the ops in
    _STEP_OPS (and the LM head's all-gathers) is bracketed by CUDA events.
    A sleep kernel holds the stream while the host enqueues the step, so the
    launches and events run back to back without host gaps; the events are
    then the only addition to the step.  Returns {op: [calls, us]}, the
    step's event-to-event time and the sum over ops."""
    import collections

    import torch
    import torch.distributed as dist

    from neurodsl_b200 import ops
    rec = []

    def wrap(name, fn):
        def timed(*a, **k):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            r = fn(*a, **k)
            e1.record()
            rec.append((name, e0, e1))
            return r
        return timed

    saved = {n: getattr(ops, n) for n in _STEP_OPS}
    saved_ag = dist.all_gather_into_tensor
    try:
        for n, fn in saved.items():
            setattr(ops, n, wrap(n, fn))
        dist.all_gather_into_tensor = wrap("all_gather (LM head max, index)", saved_ag)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)   # ~10 ms at 2 GHz: the host enqueues the step meanwhile
        s0.record()
        model.decode_step(t)
        s1.record()
    finally:
        for n, fn in saved.items():
            setattr(ops, n, fn)
        dist.all_gather_into_tensor = saved_ag
    torch.cuda.synchronize(dev)
    agg = collections.OrderedDict()
    for name, e0, e1 in rec:
        a = agg.setdefault(name, [0, 0.0])
        a[0] += 1
        a[1] += e0.elapsed_time(e1) * 1e3
    return agg, s0.elapsed_time(s1) * 1e3


def run_decoder_only(args):
    """A short eager run of one decoder (prefill, then `--decoder-steps`
    greedy decode steps, one launch per kernel, no CUDA graphs) for ncu
    captures of the decode-step kernels; prints one line of step times.
    Under torchrun the decoder is tensor-parallel over all ranks (decode
    reductions over NVLink).  With --op-times the last step is timed per
    operation (CUDA events, programmatic dependent launch off) and the table
    of rank 0 and the per-op maximum over ranks is printed too."""
    import datetime

    import torch
    import torch.distributed as dist

    from neurodsl_b200.model import GPT, GPT2_SMALL, GPT_24L_1024
    cfg, B, S = {"gpt2_small": (GPT2_SMALL, 16, 512),
                 "gpt_24l_1024": (GPT_24L_1024, 32, 2048)}[args.decoder_only]
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
        group = dist.group.WORLD
    model = GPT(cfg, seed=0, device=dev, tp=world, rank=rank, group=group,
                nvlink_rows=B if world > 1 else 0, pdl=not args.op_times)
    gen = torch.Generator(device=dev).manual_seed(99)
    ids = torch.randint(0, cfg.vocab, (B, S), device=dev, dtype=torch.int32, generator=gen)
    n = max(2, args.decoder_steps)
    model.prefill(ids, n + 1)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
    ev[0].record()
    for t in range(n - 1 if args.op_times else n):
        model.decode_step(t)
        ev[t + 1].record()
    torch.cuda.synchronize()
    steps = n - 1 if args.op_times else n
    us = [ev[t].elapsed_time(ev[t + 1]) * 1e3 for t in range(steps)]
    out = {"decoder": args.decoder_only, "batch": B, "prompt": S, "tp": world,
           "eager_decode_step_us": us}
    if args.op_times:
        barrier()
        agg, step_us = _op_times_of_step(model, n - 1, dev)
        names = list(agg)
        worst = {nm: round(max_over_ranks(agg[nm][1], dev), 1) for nm in names}
        out["op_times_step"] = {"pdl": False, "step_us": round(step_us, 1),
                                "step_us_max_over_ranks": round(max_over_ranks(step_us, dev), 1),
                                "sum_of_ops_us": round(sum(v[1] for v in agg.values()), 1),
                                "ops": {nm: {"calls": agg[nm][0], "us": round(agg[nm][1], 1),
                                             "us_max_over_ranks": worst[nm]} for nm in names}}
    if rank == 0:
        print(json.dumps(out), flush=True)
    model.close()
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


def run_comm_bench(args):
    """The tensor-parallel reduction of a decode step on its own (torchrun,
    one rank per GPU): rows x d bf16 partial sums combined with the residual
    add, bias and LayerNorm by the NVLink kernel (nd_allreduce_add_layernorm),
    against an NCCL all-reduce of the same bytes followed by the library's
    add + LayerNorm; then the same with the row-parallel projection that
    produces the partials (nd_gemm_allreduce_add_layernorm, one launch).
    CUDA-event times over back-to-back calls, max over ranks.  Prints one
    JSON line on rank 0."""
    import datetime

    import torch
    import torch.distributed as dist

    from neurodsl_b200 import ops
    from neurodsl_b200.comm import PeerReduce
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # one process without torchrun: a one-rank group (the tp = 1 kernels)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    rows, d, n = 32, 1024, args.comm_iters
    x = torch.randn(rows, d, device=dev).bfloat16()
    h = torch.empty_like(x)
    bias = torch.zeros(d, device=dev)
    g = torch.ones(d, device=dev)
    bt = torch.zeros(d, device=dev)
    pr = PeerReduce(rows, d, device=dev)
    for _ in range(2):
        pr.partial(rows).copy_(x)
        pr.k ^= 1
    buf = torch.randn(rows, d, device=dev).bfloat16()

    def timed(fn):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) * 1e3 / n, dev)

    def nvlink():
        pr.add_layernorm(x, bias, g, bt, 1e-5, x, h)

    def nccl():
        dist.all_reduce(buf)
        ops.add_layernorm(x, buf, bias, g, bt, 1e-5, s_out=x, out=h)

    res = {"workload": f"tensor-parallel reduction of {rows} x {d} bf16 partial sums + residual "
                       f"+ bias + LayerNorm, {world} ranks",
           "nvlink_fused_us": timed(nvlink)}
    with ops.pdl(True):
        res["nvlink_fused_pdl_us"] = timed(nvlink)
    res["nccl_allreduce_then_add_layernorm_us"] = timed(nccl)
    # the MLP-down projection of the 24-layer d=1024 decoder (d_ff 4096 split
    # over the ranks) with its reduction: one fused launch, against the
    # projection into this rank's slot followed by the reduction kernel
    K = 4096 // world
    a = (torch.randn(rows, K, device=dev) * 0.05).bfloat16()
    w = (torch.randn(d, K, device=dev) * 0.02).bfloat16()

    def fused_projection():
        pr.linear_add_layernorm(a, w, x, bias, g, bt, 1e-5, x, h)

    def projection_then_reduce():
        ops.linear(a, w, out=pr.partial(rows))
        pr.add_layernorm(x, bias, g, bt, 1e-5, x, h)

    def projection_then_nccl():
        ops.linear(a, w, out=buf)
        dist.all_reduce(buf)
        ops.add_layernorm(x, buf, bias, g, bt, 1e-5, s_out=x, out=h)

    res["projection_k"] = K
    with ops.pdl(True):
        res["projection_fused_pdl_us"] = timed(fused_projection)
        res["projection_then_nvlink_reduce_pdl_us"] = timed(projection_then_reduce)
    res["projection_then_nccl_us"] = timed(projection_then_nccl)
    res["device_error"] = ops.device_error()
    pr.close()
    if rank == 0:
        print(json.dumps(res), flush=True)
    barrier()
    dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--soak", type=float, default=2.0, help="seconds of load before timing")
    ap.add_argument("--decode-reps", type=int, default=5)
    ap.add_argument("--aux-reps", type=int, default=10, help="timed GEMM / LayerNorm calls")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the GPT-2-small and 24-layer decoder lines")
    ap.add_argument("--decoder-only", choices=["gpt2_small", "gpt_24l_1024"],
                    help="only a short eager run of this decoder (for kernel profiles)")
    ap.add_argument("--decoder-steps", type=int, default=4)
    ap.add_argument("--op-times", action="store_true",
                    help="with --decoder-only: per-operation times of one decode step")
    ap.add_argument("--comm-iters", type=int, default=500,
                    help="timed calls per variant of --comm-bench")
    ap.add_argument("--comm-bench", action="store_true",
                    help="only the tensor-parallel reduction microbenchmark (torchrun)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.decoder_only:
        return run_decoder_only(args)
    if args.comm_bench:
        return run_comm_bench(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
