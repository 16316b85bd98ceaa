"""GPT-style decoder built from the library's entry points (prefill and
greedy KV-cache decode), optionally tensor-parallel over ranks.

This is the GPU form of the reference's GPT-2 graph (notebook/GPT2.ipynb
cells 4 and 10: token + position :embedding, per block a pre-norm, the
multi-head flash attention of src/flash_attention.jl:225-256, residual :add,
pre-norm MLP with GELU, residual :add; a final norm and the LM head
:matmul trans_b against the token embedding) with LayerNorm as the norm and
one of the GELU forms of fused_linear_gelu as the activation.  Every op runs
in libneurodsl_b200.so:

  embedding             nd_embed
  LayerNorm             nd_layernorm, then nd_add_layernorm (residual add,
                        bias and the next LayerNorm in one pass); one-GPU
                        decode folds both into the next linear layer
                        (nd_ln_gemm)
  QKV / out / MLP       nd_gemm_bias_act (bias and GELU in the epilogue)
  prefill attention     nd_flash_attn_fwd_strided on the fused QKV projection
                        (no per-head copies); the projection's epilogue also
                        writes K/V into the caches (nd_gemm_qkv_cache)
  decode attention      nd_kv_decode_attn_qkv straight from the fused QKV
                        projection, the new token appended in place
  greedy token          nd_argmax on the LM-head logits

Tensor parallelism (Megatron layout): rank r of `tp` holds heads
[r·H/tp, (r+1)·H/tp) with their Q/K/V rows, output-projection columns and
decode caches, MLP columns [r·F/tp, (r+1)·F/tp) of the up projection and the
matching columns of the down projection, and vocabulary rows [r·V/tp, ...)
of the LM head.  In decode the output and down projections produce partial
sums that are reduced before the fused residual + LayerNorm — for batches of
up to `nvlink_rows` rows by one kernel that computes this rank's projection
tile, pushes it to every rank over NVLink and applies the residual and
LayerNorm to the sum (neurodsl_b200.comm, nd_gemm_allreduce_add_layernorm;
nd_allreduce_add_layernorm after a separate projection where the fused
kernel does not take the shapes), else with NCCL.  The prefill shards the
prompts instead (prefill_mode "dp", the default when the batch divides by
tp): each rank runs whole layers with the full weights for its prompts and
its QKV projection's epilogue writes every head's keys and values into the
owning rank's cache over NVLink (nd_gemm_qkv_cache_peers); prefill_mode "tp"
is the Megatron prefill with NCCL all-reduces, overlapped with compute in
stream groups.  The LM head gives a local (max, index) per row that is
all-gathered and reduced to the global first maximum.  Weights are generated
from one seed on every rank and sliced, so any `tp` computes the same model.

Decode steps run with programmatic dependent launch (nd_set_pdl): each
kernel's weight loads, and the decode attention's cache reads, overlap the
previous kernel, which matters because a decode step of a few rows is some
ten kernels per layer of a few microseconds each.
"""
import math
from dataclasses import dataclass

import torch

from . import ops


@dataclass(frozen=True)
class GPTConfig:
    n_layer: int
    d_model: int
    n_head: int
    d_ff: int
    vocab: int
    n_pos: int
    act: str = "tanh"      # GELU form: "sigmoid" (z·σ(1.702 z)), "tanh" or "erf"
    eps: float = 1e-5

    @property
    def d_head(self):
        return self.d_model // self.n_head


# The GPT-2-small shape and a 24-layer d=1024 model (16 heads x 64, MLP 4096).
GPT2_SMALL = GPTConfig(n_layer=12, d_model=768, n_head=12, d_ff=3072, vocab=50257, n_pos=1024)
GPT_24L_1024 = GPTConfig(n_layer=24, d_model=1024, n_head=16, d_ff=4096, vocab=50257, n_pos=4096)


def _shard(n, tp, rank):
    if n % tp:
        raise ValueError(f"{n} is not divisible by tp={tp}")
    k = n // tp
    return rank * k, (rank + 1) * k


class GPT:
    """Weights of one rank plus the buffers of one (batch, length) shape."""

    def __init__(self, cfg: GPTConfig, seed=0, device=None, tp=1, rank=0, group=None,
                 weight_std=0.02, bias_std=0.0, nvlink_rows=0, pdl=True, fused_projection=True,
                 prefill_groups=2, overlap_reserve_sms=16, prefill_mode="dp"):
        if cfg.d_head != 64:
            raise ValueError("head_dim must be 64")
        self.cfg = cfg
        # decode steps launch with programmatic dependent launch: their weights
        # and earlier cache entries are written by no kernel of the step
        self.pdl = pdl
        # NVLink decode reductions compute the row-parallel projection in the
        # same launch where the shapes allow it
        self.fused_projection = fused_projection
        # tensor-parallel prefill: the batch runs as `prefill_groups` groups of
        # sequences on as many streams, so one group's all-reduce overlaps the
        # others' compute; the persistent kernels leave overlap_reserve_sms
        # SMs to the collective
        self.prefill_groups = prefill_groups
        self.overlap_reserve_sms = overlap_reserve_sms
        self._side_streams = []
        # tensor-parallel models prefill with the prompts sharded by default: each
        # rank runs whole layers (full weights) for B/tp prompts and sends the
        # keys/values of the other ranks' heads to them ("dp"); "tp" prefills
        # with the sharded weights and all-reduces
        if prefill_mode not in ("dp", "tp"):
            raise ValueError(f"prefill_mode {prefill_mode!r} (dp or tp)")
        self.prefill_mode = prefill_mode
        self.tp, self.rank, self.group = tp, rank, group
        self.device = torch.device(device or "cuda")
        dev = self.device
        d, F, V = cfg.d_model, cfg.d_ff, cfg.vocab
        h0, h1 = _shard(cfg.n_head, tp, rank)
        self.n_head_local = h1 - h0
        self.d_local = self.n_head_local * 64
        f0, f1 = _shard(F, tp, rank)
        self.v0 = rank * ((V + tp - 1) // tp)
        self.v1 = min(V, self.v0 + (V + tp - 1) // tp)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)

        def randn(*shape, std=weight_std):
            return (torch.randn(*shape, generator=g, device=dev) * std)

        def bias(n):
            return randn(n, std=bias_std) if bias_std else torch.zeros(n, device=dev)

        bf = torch.bfloat16
        self.wte = randn(V, d).to(bf)
        self.wpe = randn(cfg.n_pos, d).to(bf)
        self.layers = []
        self.full_layers = []          # full bf16 weights of each layer (tp > 1)
        cols = slice(h0 * 64, h1 * 64)
        for _ in range(cfg.n_layer):
            ln1_g = 1 + randn(d, std=0.1) if bias_std else torch.ones(d, device=dev)
            ln1_b = bias(d)
            w_qkv = randn(3 * d, d)
            b_qkv = bias(3 * d)
            w_o = randn(d, d)
            b_o = bias(d)
            ln2_g = 1 + randn(d, std=0.1) if bias_std else torch.ones(d, device=dev)
            ln2_b = bias(d)
            w_1 = randn(F, d)
            b_1 = bias(F)
            w_2 = randn(d, F)
            b_2 = bias(d)
            q, k, v = w_qkv.view(3, d, d)
            bq, bk, bv = b_qkv.view(3, d)
            self.layers.append({
                "ln1_g": ln1_g, "ln1_b": ln1_b,
                # local Q, K, V rows stacked: [3·d_local][d]
                "w_qkv": torch.cat([q[cols], k[cols], v[cols]]).to(bf).contiguous(),
                "b_qkv": torch.cat([bq[cols], bk[cols], bv[cols]]).contiguous(),
                "w_o": w_o[:, cols].to(bf).contiguous(), "b_o": b_o,
                "ln2_g": ln2_g, "ln2_b": ln2_b,
                "w_1": w_1[f0:f1].to(bf).contiguous(), "b_1": b_1[f0:f1].contiguous(),
                "w_2": w_2[:, f0:f1].to(bf).contiguous(), "b_2": b_2,
            })
            if tp > 1:
                self.full_layers.append({"w_qkv": w_qkv.to(bf), "b_qkv": b_qkv,
                                         "w_o": w_o.to(bf), "w_1": w_1.to(bf), "b_1": b_1,
                                         "w_2": w_2.to(bf)})
        self.lnf_g = torch.ones(d, device=dev)
        self.lnf_b = torch.zeros(d, device=dev)
        self.w_head = self.wte[self.v0:self.v1]           # tied LM head, local vocab rows
        self._shape = None
        # Decode batches of up to nvlink_rows rows reduce over NVLink peer
        # memory (one fused kernel per reduction) instead of NCCL.
        self.comm = None
        if tp > 1 and nvlink_rows > 0:
            from .comm import PeerReduce
            self.comm = PeerReduce(nvlink_rows, d, group=group, device=dev)

    # ------------------------------------------------------------- buffers
    def _alloc(self, B, S, steps):
        """Buffers for prompts of S tokens and `steps` decode steps, batch B."""
        if self._shape == (B, S, steps):
            return
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        d, dl, Fl = cfg.d_model, self.d_local, self.layers[0]["w_1"].shape[0]
        L_max = S + steps
        if L_max > cfg.n_pos:
            raise ValueError(f"prompt {S} + steps {steps} exceeds n_pos {cfg.n_pos}")
        T = B * S
        self.buf = {
            "x": torch.empty(T, d, device=dev, dtype=bf), "h": torch.empty(T, d, device=dev, dtype=bf),
            "qkv": torch.empty(T, 3 * dl, device=dev, dtype=bf),
            "attn": torch.empty(T, dl, device=dev, dtype=bf),
            "part": torch.empty(T, d, device=dev, dtype=bf),
            "u": torch.empty(T, Fl, device=dev, dtype=bf),
            "last": torch.empty(B, d, device=dev, dtype=bf),
            "xd": torch.empty(B, d, device=dev, dtype=bf), "hd": torch.empty(B, d, device=dev, dtype=bf),
            "xd2": torch.empty(B, d, device=dev, dtype=bf),
            "qkvd": torch.empty(B, 3 * dl, device=dev, dtype=bf),
            "ad": torch.empty(B, dl, device=dev, dtype=bf),
            "pd": torch.empty(B, d, device=dev, dtype=bf), "ud": torch.empty(B, Fl, device=dev, dtype=bf),
            "logits": torch.empty(B, self.v1 - self.v0, device=dev, dtype=torch.float32),
            "val": torch.empty(B, device=dev, dtype=torch.float32),
            "idx": torch.empty(B, device=dev, dtype=torch.int32),
            # ids of step t in row t; row t+1 is written by step t's argmax
            "ids": torch.zeros(steps + 1, B, device=dev, dtype=torch.int32),
            "pos_prefill": torch.arange(S, device=dev, dtype=torch.int32).repeat(B),
            "pos_decode": (S + torch.arange(steps, device=dev, dtype=torch.int32))
            .view(steps, 1).repeat(1, B).contiguous(),
        }
        ws = ops.kv_decode_workspace_size(B, self.n_head_local, L_max)
        # decode scratch owned here (zero-filled once, left ready by every call)
        self.buf["ws"] = torch.zeros(max(ws, 16), device=dev, dtype=torch.uint8)
        self._alloc_caches(B, L_max)
        if self.tp > 1:
            self.buf["gval"] = torch.empty(self.tp, B, device=dev, dtype=torch.float32)
            self.buf["gidx"] = torch.empty(self.tp, B, device=dev, dtype=torch.int32)
        self._shape = (B, S, steps)

    def _alloc_caches(self, B, L_max):
        """Decode caches [B][H_local][L_max][64] per layer.  Tensor-parallel
        models keep all of a rank's caches in one region shared with the other
        ranks (CUDA IPC), so a prompt-sharded prefill writes each head's keys
        and values straight into its owner's cache; every rank maps the
        others' regions."""
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        shape = (B, self.n_head_local, L_max, 64)
        self._free_cache_region()
        if self.tp == 1:
            self.k_cache = [torch.zeros(shape, device=dev, dtype=bf) for _ in range(cfg.n_layer)]
            self.v_cache = [torch.zeros_like(c) for c in self.k_cache]
            return
        import torch.distributed as dist

        from .comm import _DeviceArray
        n = B * self.n_head_local * L_max * 64          # elements per cache
        nbytes = 2 * cfg.n_layer * n * 2
        ptr, handle = ops.comm_alloc(nbytes)            # zero-filled
        handles = [None] * self.tp
        dist.all_gather_object(handles, handle, group=self.group)
        bases = [ptr if q == self.rank else ops.comm_open(handles[q]) for q in range(self.tp)]
        self._cache_region = (ptr, bases)
        region = torch.as_tensor(_DeviceArray(ptr, (2 * cfg.n_layer * n,), "<i2"),
                                 device=dev).view(bf)
        self.k_cache = [region[(2 * i) * n:(2 * i + 1) * n].view(shape) for i in range(cfg.n_layer)]
        self.v_cache = [region[(2 * i + 1) * n:(2 * i + 2) * n].view(shape)
                        for i in range(cfg.n_layer)]
        # every rank's cache of layer i, as this process sees it
        self._peer_k = [[base + 2 * (2 * i) * n for base in bases] for i in range(cfg.n_layer)]
        self._peer_v = [[base + 2 * (2 * i + 1) * n for base in bases] for i in range(cfg.n_layer)]
        self._cache_sync = torch.zeros(1, device=dev)

    def _free_cache_region(self):
        """Unmap the peers' cache regions and free this rank's once no rank
        uses them (collective over the model's group)."""
        region = getattr(self, "_cache_region", None)
        if region is None:
            return
        import torch.distributed as dist
        ptr, bases = region
        self.k_cache = self.v_cache = []
        self._peer_k = self._peer_v = None
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)       # no rank writes or reads any cache any more
        for q, base in enumerate(bases):
            if q != self.rank:
                ops.comm_close(base)
        dist.barrier(group=self.group)       # every mapping of this region is closed
        ops.comm_free(ptr)
        self._cache_region = None

    def _all_reduce(self, t):
        if self.tp > 1:
            torch.distributed.all_reduce(t, group=self.group)

    def _next_token(self, h_rows, out_ids):
        """Greedy token of each row of h_rows [B][d] into out_ids [B]."""
        b = self.buf
        ops.linear(h_rows, self.w_head, out=b["logits"])
        if self.tp == 1:
            ops.argmax(b["logits"], idx=out_ids)
            return
        ops.argmax(b["logits"], idx=b["idx"], val=b["val"])
        b["idx"] += self.v0
        torch.distributed.all_gather_into_tensor(b["gval"], b["val"], group=self.group)
        torch.distributed.all_gather_into_tensor(b["gidx"], b["idx"], group=self.group)
        # ranks hold increasing vocabulary ranges: the first rank with the
        # maximum has the smallest index among equal values
        best = torch.argmax(b["gval"], dim=0)
        out_ids.copy_(b["gidx"].gather(0, best.view(1, -1)).view(-1))

    # ------------------------------------------------------------- prefill
    def prefill(self, ids, steps=0):
        """Run the prompt ids [B][S] (int32, device); fill the caches and
        write the first generated token into row 1 of the ids table.
        Returns the logits of the last position (local vocabulary slice)."""
        B, S = ids.shape
        self._alloc(B, S, max(steps, 1))
        cfg, b = self.cfg, self.buf
        if self.tp > 1 and self.prefill_mode == "dp" and B % self.tp == 0:
            self._prefill_sharded_prompts(ids, B, S)
        else:
            x, h = b["x"], b["h"]
            ops.embed(ids.reshape(-1), self.wte, self.wpe, b["pos_prefill"], out=x)
            ops.layernorm(x, self.layers[0]["ln1_g"], self.layers[0]["ln1_b"], eps=cfg.eps,
                          out=h, stats=False)
            G = self.prefill_groups if self.tp > 1 else 1
            if G > 1 and B % G == 0:
                self._prefill_layers_overlapped(B, S, G)
            else:
                for i in range(cfg.n_layer):
                    for sub in self._prefill_sublayers(i, self._prefill_group(0, B, S)):
                        sub()
            b["last"].copy_(h.view(B, S, -1)[:, -1])
        self._next_token(b["last"], b["ids"][1])
        b["ids"][0].copy_(ids[:, -1])
        return b["logits"]

    def _shard_buffers(self, B, S):
        """Buffers of the prompt-sharded prefill for this rank's B/tp prompts."""
        key = (B, S)
        if getattr(self, "_shard_key", None) != key:
            cfg, dev, bf = self.cfg, self.device, torch.bfloat16
            d, F, tp, dl = cfg.d_model, cfg.d_ff, self.tp, self.d_local
            T = B // tp * S
            self._shard = {
                "x": torch.empty(T, d, device=dev, dtype=bf), "h": torch.empty(T, d, device=dev, dtype=bf),
                "qkv": torch.empty(T, 3 * d, device=dev, dtype=bf),
                "attn": torch.empty(T, d, device=dev, dtype=bf),
                "part": torch.empty(T, d, device=dev, dtype=bf),
                "u": torch.empty(T, F, device=dev, dtype=bf),
                "last": torch.empty(B // tp, d, device=dev, dtype=bf),
                # keys and values of this rank's tokens for rank q: send[q][t][k | v][dl]
                "send": torch.empty(tp, T, 2, dl, device=dev, dtype=bf),
                # every rank's tokens (global token order) for this rank's heads
                "recv": torch.empty(B * S, 2 * dl, device=dev, dtype=bf),
            }
            self._shard_key = key
        return self._shard

    def _prefill_sharded_prompts(self, ids, B, S):
        """Prefill of a tensor-parallel model with the prompts sharded over the
        ranks: rank r runs every layer with the full weights for prompts
        [r·B/tp, (r+1)·B/tp) — the one-GPU prefill of those prompts, with no
        reduction — and after each layer's QKV projection sends the keys and
        values of rank q's heads to rank q (one all-to-all, on a side stream
        so it overlaps the rest of the layer), which writes them into its
        head-sharded decode caches — or, for more than 32 rows, the QKV
        projection's epilogue stores them straight into the owners' caches
        over NVLink (nd_gemm_qkv_cache_peers), with no copy, collective or
        extra launch.  The last positions' hidden states are all-gathered for
        the vocabulary-sharded LM head.  The caches and the
        LM head's input are those of the one-GPU model bit for bit; the
        communication is the keys and values once, instead of two all-reduces
        of the activations per layer."""
        cfg, b = self.cfg, self.buf
        tp, r, dl, H, d = self.tp, self.rank, self.d_local, cfg.n_head, cfg.d_model
        Bl = B // tp
        T = Bl * S
        sp = self._shard_buffers(B, S)
        x, h, qkv, attn = (sp[k] for k in ("x", "h", "qkv", "attn"))
        dev = self.device
        main = torch.cuda.current_stream(dev)
        if not self._side_streams:
            self._side_streams.append(torch.cuda.Stream(dev))
        side = self._side_streams[0]
        side.wait_stream(main)               # the side stream joins this prefill (or its capture)
        ops.embed(ids[r * Bl:(r + 1) * Bl].reshape(-1), self.wte, self.wpe,
                  b["pos_prefill"][:T], out=x)
        ops.layernorm(x, self.layers[0]["ln1_g"], self.layers[0]["ln1_b"], eps=cfg.eps, out=h,
                      stats=False)
        parts = qkv.view(Bl, S, 3, H, 64).permute(2, 0, 3, 1, 4)   # [3][Bl][H][S][64]
        o4 = attn.view(Bl, S, H, 64).permute(0, 2, 1, 3)
        # the K (then V) columns of rank q's heads: [tp][T][dl] views of qkv
        cols = [qkv[:, (1 + kv) * d:(2 + kv) * d].view(T, tp, dl).permute(1, 0, 2) for kv in (0, 1)]
        # no rank still reads its caches (an earlier decode) when the others
        # start writing into them
        torch.distributed.all_reduce(self._cache_sync, group=self.group)
        # the all-to-all form (few rows) leaves SMs to the collective; the
        # direct form needs none (its transfers are the GEMM's own stores)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        reserve = self.overlap_reserve_sms if T <= 32 else 0
        with ops.sm_limit(max(1, sms - reserve) if reserve > 0 else 0):
            self._sharded_layers(cfg, sp, cols, parts, o4, side, main, B, S, dl)
        sp["last"].copy_(h.view(Bl, S, -1)[:, -1])
        torch.distributed.all_gather_into_tensor(b["last"], sp["last"], group=self.group)
        main.wait_stream(side)

    def _sharded_layers(self, cfg, sp, cols, parts, o4, side, main, B, S, dl):
        """The layers of the prompt-sharded prefill (see _prefill_sharded_prompts)."""
        x, h, qkv, attn, part, u = (sp[k] for k in ("x", "h", "qkv", "attn", "part", "u"))
        Bl = B // self.tp
        L_max = self.k_cache[0].shape[2]
        # more than 32 rows: the projection's epilogue writes every head's keys
        # and values into its owner's cache over NVLink; else an all-to-all
        direct = Bl * S > 32
        for i, (L, FL) in enumerate(zip(self.layers, self.full_layers)):
            if direct:
                ops.linear_qkv_cache_peers(h, FL["w_qkv"], FL["b_qkv"], qkv, self._peer_k[i],
                                           self._peer_v[i], self.n_head_local, L_max, Bl,
                                           self.rank * Bl, S)
            else:
                ops.linear(h, FL["w_qkv"], FL["b_qkv"], out=qkv)
                main.wait_stream(side)           # the previous layer's all-to-all has read send
                for kv in (0, 1):
                    ops.copy_2d_batched(cols[kv], sp["send"][:, :, kv, :])
                side.wait_stream(main)
                with torch.cuda.stream(side):
                    torch.distributed.all_to_all_single(sp["recv"].view(-1), sp["send"].view(-1),
                                                        group=self.group)
                    ops.kv_store(sp["recv"], 0, dl, self.k_cache[i], self.v_cache[i], B, S)
            ops.flash_attn_fwd(parts[0], parts[1], parts[2], causal=True, out=o4)
            ops.linear(attn, FL["w_o"], out=part)
            ops.add_layernorm(x, part, L["b_o"], L["ln2_g"], L["ln2_b"], cfg.eps, s_out=x, out=h)
            ops.linear(h, FL["w_1"], FL["b_1"], act=cfg.act, out=u)
            ops.linear(u, FL["w_2"], out=part)
            nxt = self.layers[i + 1] if i + 1 < len(self.layers) else None
            g_, b_ = (nxt["ln1_g"], nxt["ln1_b"]) if nxt else (self.lnf_g, self.lnf_b)
            ops.add_layernorm(x, part, L["b_2"], g_, b_, cfg.eps, s_out=x, out=h)

    def _prefill_group(self, b0, b1, S):
        """Views of the prefill buffers and caches for sequences [b0, b1)."""
        b, H = self.buf, self.n_head_local
        n = b1 - b0
        r0, r1 = b0 * S, b1 * S
        qkv = b["qkv"][r0:r1]
        return {"n": n, "S": S, "x": b["x"][r0:r1], "h": b["h"][r0:r1], "qkv": qkv,
                "attn": b["attn"][r0:r1], "part": b["part"][r0:r1], "u": b["u"][r0:r1],
                "parts": qkv.view(n, S, 3, H, 64).permute(2, 0, 3, 1, 4),   # [3][n][H][S][64]
                "o4": b["attn"][r0:r1].view(n, S, H, 64).permute(0, 2, 1, 3),
                "b0": b0, "b1": b1}

    def _prefill_sublayers(self, i, g):
        """Layer i of the prefill over one group of sequences as two launch
        sequences, each ending in its tensor-parallel all-reduce: attention
        (QKV projection filling the caches, causal attention, output
        projection) and the MLP (residual + LN2, up, down), the residual + next
        LayerNorm opening the following one."""
        cfg, L = self.cfg, self.layers[i]
        x, h, part = g["x"], g["h"], g["part"]
        nxt = self.layers[i + 1] if i + 1 < len(self.layers) else None
        g_, b_ = (nxt["ln1_g"], nxt["ln1_b"]) if nxt else (self.lnf_g, self.lnf_b)

        def attention():
            ops.linear_qkv_cache(h, L["w_qkv"], L["b_qkv"], g["qkv"],
                                 self.k_cache[i][g["b0"]:g["b1"]],
                                 self.v_cache[i][g["b0"]:g["b1"]], g["n"], g["S"])
            p = g["parts"]
            ops.flash_attn_fwd(p[0], p[1], p[2], causal=True, out=g["o4"])
            ops.linear(g["attn"], L["w_o"], out=part)
            self._all_reduce(part)

        def mlp():
            ops.add_layernorm(x, part, L["b_o"], L["ln2_g"], L["ln2_b"], cfg.eps, s_out=x, out=h)
            ops.linear(h, L["w_1"], L["b_1"], act=cfg.act, out=g["u"])
            ops.linear(g["u"], L["w_2"], out=part)
            self._all_reduce(part)

        def close():
            ops.add_layernorm(x, part, L["b_2"], g_, b_, cfg.eps, s_out=x, out=h)

        return attention, mlp, close

    def _prefill_layers_overlapped(self, B, S, G):
        """Tensor-parallel prefill with the all-reduces overlapped: the batch
        is split into G groups of sequences (independent through every
        layer), group k's launches go to stream k, and the launch sequences
        are issued round-robin, so while one group's all-reduce runs (on the
        process group's stream, after that group's projection) the next
        group's GEMMs and attention run beside it.  The persistent kernels are
        capped to leave overlap_reserve_sms SMs to the collective's CTAs.  The
        groups share no data and every kernel computes a row from that row's
        inputs, so at tp = 2 the results are the one-stream prefill's bits; with
        more ranks the collective may add the smaller messages' partial sums
        in another order."""
        dev = self.device
        main = torch.cuda.current_stream(dev)
        while len(self._side_streams) < G - 1:
            self._side_streams.append(torch.cuda.Stream(dev))
        streams = [main] + self._side_streams[:G - 1]
        for s in streams[1:]:
            s.wait_stream(main)
        groups = [self._prefill_group(k * B // G, (k + 1) * B // G, S) for k in range(G)]
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        with ops.sm_limit(max(1, sms - self.overlap_reserve_sms)):
            for i in range(self.cfg.n_layer):
                seqs = [self._prefill_sublayers(i, g) for g in groups]
                for part in range(3):
                    for k, s in enumerate(streams):
                        with torch.cuda.stream(s):
                            seqs[k][part]()
        for s in streams[1:]:
            main.wait_stream(s)

    # -------------------------------------------------------------- decode
    def decode_step(self, t):
        """Decode step t (0-based): the token in row t of the ids table is
        appended at position S + t and attended; the greedy next token goes to
        row t + 1.  Launches only (no host synchronisation)."""
        cfg, b = self.cfg, self.buf
        B, S, steps = self._shape
        if not 0 <= t < steps:
            raise ValueError(f"step {t} outside [0, {steps})")
        H = self.n_head_local
        xd, hd = b["xd"], b["hd"]
        out_ids = b["ids"][t + 2] if t + 2 <= steps else b["idx"]
        Lc = S + t + 1
        with ops.pdl(self.pdl):
            ops.embed(b["ids"][t + 1], self.wte, self.wpe, b["pos_decode"][t], out=xd)
            if self.tp == 1:
                self._decode_layers_fused(B, H, Lc, out_ids)
                return b["logits"]
            ops.layernorm(xd, self.layers[0]["ln1_g"], self.layers[0]["ln1_b"], eps=cfg.eps,
                          out=hd, stats=False)
            peer = self.comm is not None and B <= self.comm.rows_max
            for i, L in enumerate(self.layers):
                ops.linear(hd, L["w_qkv"], L["b_qkv"], out=b["qkvd"])
                ops.kv_decode_attn_qkv(b["qkvd"], self.k_cache[i], self.v_cache[i], Lc,
                                       out=b["ad"].view(B, H, 64), workspace=b["ws"])
                nxt = self.layers[i + 1] if i + 1 < len(self.layers) else None
                g_, b_ = (nxt["ln1_g"], nxt["ln1_b"]) if nxt else (self.lnf_g, self.lnf_b)
                if peer:
                    self._peer_projection(b["ad"], L["w_o"], L["b_o"], L["ln2_g"], L["ln2_b"])
                    ops.linear(hd, L["w_1"], L["b_1"], act=cfg.act, out=b["ud"])
                    self._peer_projection(b["ud"], L["w_2"], L["b_2"], g_, b_)
                    continue
                ops.linear(b["ad"], L["w_o"], out=b["pd"])
                self._all_reduce(b["pd"])
                ops.add_layernorm(xd, b["pd"], L["b_o"], L["ln2_g"], L["ln2_b"], cfg.eps, s_out=xd,
                                  out=hd)
                ops.linear(hd, L["w_1"], L["b_1"], act=cfg.act, out=b["ud"])
                ops.linear(b["ud"], L["w_2"], out=b["pd"])
                self._all_reduce(b["pd"])
                ops.add_layernorm(xd, b["pd"], L["b_2"], g_, b_, cfg.eps, s_out=xd, out=hd)
            self._next_token(hd, out_ids)
        return b["logits"]

    def _peer_projection(self, a, w, bias, gamma, beta):
        """Row-parallel projection a · wᵀ, summed over the ranks through NVLink
        peer memory, + residual + bias, LayerNorm: one launch where the shapes
        allow it (nd_gemm_allreduce_add_layernorm), else the projection into
        this rank's slot and nd_allreduce_add_layernorm."""
        b, eps = self.buf, self.cfg.eps
        xd, hd = b["xd"], b["hd"]
        if self.fused_projection and self.comm.fused_supported(a.shape[0], a.shape[1]):
            self.comm.linear_add_layernorm(a, w, xd, bias, gamma, beta, eps, xd, hd)
            return
        ops.linear(a, w, out=self.comm.partial(a.shape[0]))
        self.comm.add_layernorm(xd, bias, gamma, beta, eps, xd, hd)

    def _decode_layers_fused(self, B, H, Lc, out_ids):
        """One GPU: five launches per layer — residual + LN1 + QKV projection,
        attention, output projection, residual + LN2 + up projection, down
        projection (nd_ln_gemm folds each residual add and LayerNorm into the
        linear layer after it; above 16 rows the two go as separate launches)
        — then residual + final LN + LM head, argmax.
        The residual stream alternates between two buffers: each fused launch
        reads one and writes the updated stream to the other, since all its
        CTAs read the old stream while one writes the new."""
        cfg, b = self.cfg, self.buf
        xa, xb = b["xd"], b["xd2"]
        p = pb = None

        def ln_linear(x, W, p, p_bias, gamma, beta, s_out, bias, out, act="none"):
            # Above 16 rows the residual + LayerNorm goes first in its own
            # launch (a warp per row) and the projection reads it: every CTA
            # of the fused form repeats the LayerNorm of all rows, which at 32
            # rows costs more than the extra launch (24-layer QKV projection:
            # 11.0 vs 12.5 us).  Same bits either way.
            if x.shape[0] <= 16:
                ops.ln_linear(x, W, p=p, p_bias=p_bias, gamma=gamma, beta=beta, eps=cfg.eps,
                              s_out=s_out, bias=bias, act=act, out=out)
            elif p is None:
                ops.layernorm(x, gamma, beta, eps=cfg.eps, out=b["hd"], stats=False)
                ops.linear(b["hd"], W, bias, act=act, out=out)
            else:
                ops.add_layernorm(x, p, p_bias, gamma, beta, cfg.eps, s_out=s_out, out=b["hd"])
                ops.linear(b["hd"], W, bias, act=act, out=out)

        for i, L in enumerate(self.layers):
            ln_linear(xa, L["w_qkv"], p, pb, L["ln1_g"], L["ln1_b"], None if p is None else xb,
                      L["b_qkv"], b["qkvd"])
            if p is not None:
                xa, xb = xb, xa
            ops.kv_decode_attn_qkv(b["qkvd"], self.k_cache[i], self.v_cache[i], Lc,
                                   out=b["ad"].view(B, H, 64), workspace=b["ws"])
            ops.linear(b["ad"], L["w_o"], out=b["pd"])
            ln_linear(xa, L["w_1"], b["pd"], L["b_o"], L["ln2_g"], L["ln2_b"], xb, L["b_1"],
                      b["ud"], act=cfg.act)
            xa, xb = xb, xa
            ops.linear(b["ud"], L["w_2"], out=b["pd"])
            p, pb = b["pd"], L["b_2"]
        ops.ln_linear(xa, self.w_head, p=p, p_bias=pb, gamma=self.lnf_g, beta=self.lnf_b,
                      eps=cfg.eps, out=b["logits"], out_dtype=torch.float32)
        ops.argmax(b["logits"], idx=out_ids)

    def tokens(self):
        """Generated tokens so far: [B][steps] (prefill's token first)."""
        return self.buf["ids"][1:].t()

    def prefill_graphed(self, ids, steps=0):
        """prefill(ids, steps) replayed from a CUDA graph captured on the first
        call for this (prompt shape, steps): the prompt is copied into a static
        buffer and the ~10 launches per layer replay without host work in
        between.  Returns the logits like prefill."""
        key = (tuple(ids.shape), max(steps, 1))
        if getattr(self, "_prefill_key", None) != key:
            self._prefill_graph = None
            self._prefill_ids = torch.empty_like(ids)
            self._prefill_ids.copy_(ids)
            self.prefill(self._prefill_ids, steps)   # buffers allocated outside the capture
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.prefill(self._prefill_ids, steps)
            torch.cuda.current_stream(self.device).wait_stream(s)
            self._prefill_graph, self._prefill_key = g, key
        self._prefill_ids.copy_(ids)
        self._prefill_graph.replay()
        return self.buf["logits"]

    def generate(self, ids, steps, graph_chunk=0, graph_prefill=False):
        """Greedy generation of `steps` tokens after the prompt ids [B][S].
        graph_chunk > 0 captures that many decode steps per CUDA graph (the
        graphs are kept and replayed by later calls of the same shape);
        graph_prefill replays the prefill from a CUDA graph too."""
        if graph_prefill:
            self.prefill_graphed(ids, steps)
        else:
            self.prefill(ids, steps)
        n_dec = steps - 1
        if graph_chunk <= 0:
            for t in range(n_dec):
                self.decode_step(t)
            return self.tokens()
        key = (self._shape, graph_chunk)
        if getattr(self, "_graphs_key", None) != key:
            self._graphs = []
            self._graphs_key = key
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            for t0 in range(0, n_dec, graph_chunk):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for t in range(t0, min(n_dec, t0 + graph_chunk)):
                        self.decode_step(t)
                self._graphs.append(g)
            torch.cuda.current_stream(self.device).wait_stream(s)
        for g in self._graphs:
            g.replay()
        return self.tokens()

    def release_graphs(self):
        """Drop captured graphs (those holding NCCL calls go before the
        process group is destroyed)."""
        self._graphs = []
        self._graphs_key = None
        self._prefill_graph = None
        self._prefill_key = None

    def close(self):
        """Release graphs and the NVLink reduction regions (collective when
        tensor-parallel: every rank calls it before the group is destroyed)."""
        self.release_graphs()
        self._free_cache_region()
        self._shape = None
        if self.comm is not None:
            self.comm.close()
            self.comm = None


def flops_prefill(cfg: GPTConfig, B, S):
    """Algorithmic FLOPs of a prefill of B prompts of S tokens: the layer
    GEMMs, causal attention (QKᵀ and P·V over the unmasked triangle) and the
    LM head for the last position of each prompt."""
    d, F, n = cfg.d_model, cfg.d_ff, cfg.n_layer
    gemm = 2 * B * S * (3 * d * d + d * d + 2 * d * F) * n
    attn = 4 * B * cfg.n_head * 64 * (S * (S + 1) // 2) * n
    return gemm + attn + 2 * B * d * cfg.vocab


def decode_weight_bytes(cfg: GPTConfig):
    """bf16 weight bytes read by one decode step (layers and the LM head)."""
    d, F, n = cfg.d_model, cfg.d_ff, cfg.n_layer
    return 2 * (n * (4 * d * d + 2 * d * F) + cfg.vocab * d)
