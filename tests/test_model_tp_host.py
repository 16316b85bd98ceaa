"""Tensor-parallel decomposition of the decoder on CPU: two gloo ranks each
hold the shard of neurodsl_b200.model.GPT that rank would hold on a GPU
(heads, MLP columns, LM-head vocabulary rows), run the oracle's decoder on it
with the partial sums all-reduced over gloo and the local logits gathered,
and must reproduce the one-rank model's logits (bf16 partial sums: max-abs
2e-2) and its greedy tokens wherever the top-2 margin exceeds 2e-2.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from _gpt_util import top2_margin, weights_of

CFG = dict(n_layer=2, d_model=128, n_head=2, d_ff=512, vocab=1001, n_pos=64, act="tanh")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, ids, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from neurodsl_b200.model import GPT, GPTConfig
        m = GPT(GPTConfig(**CFG), seed=7, device="cpu", tp=world, rank=rank, weight_std=0.05,
                bias_std=0.02)

        def reduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            dist.all_reduce(t)
            return t.numpy()

        local = oracle.gpt_last_logits(weights_of(m), ids, reduce=reduce)
        parts = [None] * world
        dist.all_gather_object(parts, local)
        if rank == 0:
            np.save(out_path, np.concatenate(parts, axis=1))
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_reproduce_one_rank_model(tmp_path):
    from neurodsl_b200.model import GPT, GPTConfig
    rng = np.random.default_rng(1)
    ids = rng.integers(0, CFG["vocab"], (2, 12)).astype(np.int32)
    full = GPT(GPTConfig(**CFG), seed=7, device="cpu", tp=1, rank=0, weight_std=0.05,
               bias_std=0.02)
    ref = oracle.gpt_last_logits(weights_of(full), ids)
    out = str(tmp_path / "tp2.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), ids, out), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(out)
    assert got.shape == ref.shape
    assert float(np.abs(got - ref).max()) <= 2e-2
    clear = top2_margin(ref) > 2e-2
    np.testing.assert_array_equal(got.argmax(-1)[clear], ref.argmax(-1)[clear])


def test_shards_partition_the_weights():
    from neurodsl_b200.model import GPT, GPTConfig
    cfg = GPTConfig(**CFG)
    full = GPT(cfg, seed=7, device="cpu", tp=1)
    shards = [GPT(cfg, seed=7, device="cpu", tp=2, rank=r) for r in range(2)]
    d, dl = cfg.d_model, cfg.d_model // 2
    L = [s.layers[0] for s in shards]
    F = full.layers[0]
    # Q rows of the two ranks' heads, in order, are the full Q rows
    q = torch.cat([x["w_qkv"][:dl] for x in L])
    assert torch.equal(q, F["w_qkv"][:d])
    assert torch.equal(torch.cat([x["w_o"] for x in L], dim=1), F["w_o"])
    assert torch.equal(torch.cat([x["w_1"] for x in L]), F["w_1"])
    assert torch.equal(torch.cat([x["w_2"] for x in L], dim=1), F["w_2"])
    assert torch.equal(torch.cat([s.w_head for s in shards]), full.w_head)
