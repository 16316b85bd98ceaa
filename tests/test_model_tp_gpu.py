"""Tensor-parallel decoder on two GPUs (NCCL): the tp=2 model built from the
same seed must reproduce the one-GPU model — LM-head logits within relative
L2 1e-2 and max-abs 5e-2 (logits spread ~0.8 here; each rank's partial sum
is rounded to bf16 before the all-reduce, one extra rounding per sub-layer)
and the greedy tokens wherever the one-GPU top-2 margin exceeds 5e-2 — and
its graph-captured decode must give the same tokens as its eager decode.  Its
tensor-parallel prefill with the batch split into two sequence groups on two
streams (each group's all-reduces overlapping the other's compute) gives the
one-stream prefill's bits, and its default prefill with the prompts sharded
over the ranks (whole layers per rank, keys/values sent to their heads' ranks)
gives the one-GPU model's prefill logits and caches bit for bit.
The same holds for the tp=2 model whose decode reductions run over NVLink
peer memory instead of NCCL, with the row-parallel projection fused into the
exchange (nd_gemm_allreduce_add_layernorm); the same model with the
projection as a separate launch before nd_allreduce_add_layernorm gives
bit-identical logits.  Skipped with fewer than 2 GPUs.
Each rank runs the same collectives in the same order; the process group has
a 60 s timeout so a lost rank ends the others with an error.
"""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from _gpt_util import top2_margin  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = dict(n_layer=2, d_model=256, n_head=4, d_ff=1024, vocab=1000, n_pos=64, act="tanh")
B, S, STEPS = 2, 24, 6


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompt():
    return np.random.default_rng(9).integers(0, CFG["vocab"], (B, S)).astype(np.int32)


LONG = 40   # prompts long enough that every GEMM of a one-prompt shard keeps the many-row kernel


def _long_prompt():
    return np.random.default_rng(4).integers(0, CFG["vocab"], (B, LONG)).astype(np.int32)


def _run(model, ids):
    logits = [model.prefill(ids, STEPS).clone()]
    for t in range(STEPS - 1):
        logits.append(model.decode_step(t).clone())
    return logits, model.tokens().clone()


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist
    from neurodsl_b200.model import GPT, GPTConfig
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        m = GPT(GPTConfig(**CFG), seed=21, device=dev, tp=world, rank=rank,
                group=dist.group.WORLD, weight_std=0.05, bias_std=0.02)
        # the prefill with its two sequence groups on two streams (all-reduces
        # overlapped with the other group's compute) against one stream, on
        # prompts long enough that a group's GEMMs keep the many-row kernel
        long_ids = torch.from_numpy(_long_prompt()).to(dev)
        m.prefill_mode = "tp"
        m.prefill_groups = 1
        one_stream = m.prefill(long_ids, STEPS).clone()
        caches = [c[:, :, :LONG].clone() for c in m.k_cache + m.v_cache]
        m.prefill_groups = 2
        assert torch.equal(m.prefill(long_ids, STEPS), one_stream)
        for c, ref in zip(m.k_cache + m.v_cache, caches):
            assert torch.equal(c[:, :, :LONG], ref)
        # the prompt-sharded prefill (the default): each rank runs whole layers
        # for its prompts, keys/values go to their heads' ranks by all-to-all
        m.prefill_mode = "dp"
        sharded = m.prefill(long_ids, STEPS)
        parts = [torch.empty_like(sharded) for _ in range(world)]
        dist.all_gather(parts, sharded)
        np.save(os.path.join(out_dir, f"sharded_caches_{rank}.npy"),
                np.stack([c[:, :, :LONG].float().cpu().numpy() for c in m.k_cache + m.v_cache]))
        if rank == 0:
            np.save(os.path.join(out_dir, "sharded_logits.npy"),
                    torch.cat(parts, dim=1).cpu().numpy())
        ids = torch.from_numpy(_prompt()).to(dev)
        logits, tokens = _run(m, ids)
        full = []
        for lg in logits:
            parts = [torch.empty_like(lg) for _ in range(world)]
            dist.all_gather(parts, lg)
            full.append(torch.cat(parts, dim=1).cpu().numpy())
        graphed = m.generate(ids, STEPS, graph_chunk=2).clone()
        torch.cuda.synchronize()
        m.close()
        if rank == 0:
            np.save(os.path.join(out_dir, "logits.npy"), np.stack(full))
            np.save(os.path.join(out_dir, "tokens.npy"), tokens.cpu().numpy())
            np.save(os.path.join(out_dir, "graphed.npy"), graphed.cpu().numpy())
        # decode reductions over NVLink peer memory: the projection fused with
        # the exchange (default), and the projection as its own launch
        from neurodsl_b200 import ops
        for tag, fused in (("nv", True), ("nvsep", False)):
            m2 = GPT(GPTConfig(**CFG), seed=21, device=dev, tp=world, rank=rank,
                     group=dist.group.WORLD, weight_std=0.05, bias_std=0.02, nvlink_rows=8,
                     fused_projection=fused)
            logits2, tokens2 = _run(m2, ids)
            full2 = []
            for lg in logits2:
                parts = [torch.empty_like(lg) for _ in range(world)]
                dist.all_gather(parts, lg)
                full2.append(torch.cat(parts, dim=1).cpu().numpy())
            graphed2 = m2.generate(ids, STEPS, graph_chunk=2).clone()
            again2 = m2.generate(ids, STEPS, graph_chunk=2).clone()
            torch.cuda.synchronize()
            err = ops.device_error()
            m2.close()
            if rank == 0:
                np.save(os.path.join(out_dir, f"logits_{tag}.npy"), np.stack(full2))
                np.save(os.path.join(out_dir, f"tokens_{tag}.npy"), tokens2.cpu().numpy())
                np.save(os.path.join(out_dir, f"graphed_{tag}.npy"),
                        np.stack([graphed2.cpu().numpy(), again2.cpu().numpy()]))
                np.save(os.path.join(out_dir, f"err_{tag}.npy"), np.array([err]))
            dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_single_gpu(tmp_path):
    import torch.multiprocessing as mp
    from neurodsl_b200.model import GPT, GPTConfig
    mp.start_processes(_rank_main, args=(2, _port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    ref = GPT(GPTConfig(**CFG), seed=21, device="cuda:0", weight_std=0.05, bias_std=0.02)
    # the prompt-sharded prefill computes the one-GPU prefill: same logits and
    # caches (each rank's heads), bit for bit
    ref_long = ref.prefill(torch.from_numpy(_long_prompt()).cuda(), STEPS).cpu().numpy()
    np.testing.assert_array_equal(np.load(tmp_path / "sharded_logits.npy"), ref_long)
    hl = CFG["n_head"] // 2
    for r in range(2):
        got = np.load(tmp_path / f"sharded_caches_{r}.npy")
        want = np.stack([c[:, r * hl:(r + 1) * hl, :LONG].float().cpu().numpy()
                         for c in ref.k_cache + ref.v_cache])
        np.testing.assert_array_equal(got, want)
    ref_logits, ref_tokens = _run(ref, torch.from_numpy(_prompt()).cuda())
    ref_logits = np.stack([x.cpu().numpy() for x in ref_logits])
    ref_tokens = ref_tokens.cpu().numpy()
    logits = np.load(tmp_path / "logits.npy")
    tokens = np.load(tmp_path / "tokens.npy")
    graphed = np.load(tmp_path / "graphed.npy")
    np.testing.assert_array_equal(graphed, tokens)
    def close(a, b):
        rel = float(np.linalg.norm(a - b) / np.linalg.norm(b))
        return float(np.abs(a - b).max()) <= 5e-2 and rel <= 1e-2

    # the first step sees the same prompt on both sides
    assert close(logits[0], ref_logits[0])
    for k in range(STEPS):
        clear = top2_margin(ref_logits[k]) > 5e-2
        if (tokens[:, :k] == ref_tokens[:, :k]).all():
            assert close(logits[k], ref_logits[k]), k
            np.testing.assert_array_equal(tokens[clear, k], ref_tokens[clear, k])
    # the NVLink-reduced decode
    assert int(np.load(tmp_path / "err_nv.npy")[0]) == 0
    logits_nv = np.load(tmp_path / "logits_nv.npy")
    tokens_nv = np.load(tmp_path / "tokens_nv.npy")
    g_nv = np.load(tmp_path / "graphed_nv.npy")
    np.testing.assert_array_equal(g_nv[0], tokens_nv)
    np.testing.assert_array_equal(g_nv[1], tokens_nv)
    for k in range(STEPS):
        clear = top2_margin(ref_logits[k]) > 5e-2
        if (tokens_nv[:, :k] == ref_tokens[:, :k]).all():
            assert close(logits_nv[k], ref_logits[k]), k
            np.testing.assert_array_equal(tokens_nv[clear, k], ref_tokens[clear, k])
    # the fused projection + exchange gives the bits of the separate launches
    assert int(np.load(tmp_path / "err_nvsep.npy")[0]) == 0
    np.testing.assert_array_equal(np.load(tmp_path / "logits_nvsep.npy"), logits_nv)
    np.testing.assert_array_equal(np.load(tmp_path / "tokens_nvsep.npy"), tokens_nv)
    np.testing.assert_array_equal(np.load(tmp_path / "graphed_nvsep.npy")[0], tokens_nv)
