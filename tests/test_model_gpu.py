"""GPU parity of the decoder assembled from the library (neurodsl_b200.model):
prefill and greedy KV-cache decode against the oracle's restatement of the
reference's GPT-2 graph, teacher-forced with the GPU's own tokens.

Tolerance: LM-head logits within max-abs 2e-2 and relative L2 2e-2 of the
oracle (bf16 activations on both sides, rounded at the same points); the
greedy token must agree wherever the oracle's top-2 margin exceeds 2e-2.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from _gpt_util import top2_margin, weights_of  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = dict(n_layer=2, d_model=128, n_head=2, d_ff=512, vocab=1000, n_pos=64, act="tanh")


def _model(**kw):
    from neurodsl_b200.model import GPT, GPTConfig
    cfg = GPTConfig(**{**CFG, **kw})
    return GPT(cfg, seed=11, weight_std=0.05, bias_std=0.02), cfg


def _prompt(B, S, V, seed=3):
    rng = np.random.default_rng(seed)
    return rng.integers(0, V, (B, S)).astype(np.int32)


@pytest.mark.parametrize("act", ["tanh", "sigmoid"])
def test_prefill_and_decode_match_oracle(act):
    model, cfg = _model(act=act)
    B, S, steps = 2, 20, 6
    ids = _prompt(B, S, cfg.vocab)
    logits = [model.prefill(torch.from_numpy(ids).cuda(), steps).clone()]
    for t in range(steps - 1):
        logits.append(model.decode_step(t).clone())
    torch.cuda.synchronize()
    tokens = model.tokens().cpu().numpy()
    W = weights_of(model)
    for k in range(steps):
        seq = np.concatenate([ids, tokens[:, :k]], axis=1)
        ref = oracle.gpt_last_logits(W, seq, act=act, eps=cfg.eps)
        got = logits[k].cpu().numpy()
        err = float(np.abs(got - ref).max())
        rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        assert err <= 2e-2 and rel <= 2e-2, f"step {k}: max-abs {err}, rel-L2 {rel}"
        clear = top2_margin(ref) > 2e-2
        np.testing.assert_array_equal(tokens[clear, k], ref.argmax(-1)[clear])


def test_graph_replay_gives_the_eager_tokens():
    model, cfg = _model()
    ids = torch.from_numpy(_prompt(3, 17, cfg.vocab, seed=5)).cuda()
    eager = model.generate(ids, 9).clone()
    g1 = model.generate(ids, 9, graph_chunk=3).clone()
    g2 = model.generate(ids, 9, graph_chunk=3).clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, g1) and torch.equal(g1, g2)
    model.release_graphs()


def test_rejects_sequences_past_the_position_table():
    model, cfg = _model()
    with pytest.raises(ValueError):
        model.prefill(torch.zeros((1, 60), dtype=torch.int32, device="cuda"), steps=10)


def test_graphed_prefill_matches_eager():
    """prefill_graphed (a captured CUDA graph, replayed with a new prompt
    copied into its static buffer) gives the eager prefill's logits and first
    token, on a second prompt too."""
    from neurodsl_b200.model import GPT, GPTConfig
    cfg = GPTConfig(n_layer=2, d_model=256, n_head=4, d_ff=1024, vocab=3001, n_pos=256)
    m = GPT(cfg, seed=3)
    gen = torch.Generator(device="cuda").manual_seed(8)
    for _ in range(2):
        ids = torch.randint(0, cfg.vocab, (3, 48), device="cuda", dtype=torch.int32, generator=gen)
        eager = m.prefill(ids, 4).clone()
        first = m.buf["ids"][1].clone()
        graphed = m.prefill_graphed(ids, 4).clone()
        torch.cuda.synchronize()
        assert torch.equal(eager, graphed)
        assert torch.equal(first, m.buf["ids"][1])
    m.release_graphs()
