"""Greedy-decode parity of the decoders at the sizes the benchmark runs.

GPT-2 small (12 layers, d 768, 12 heads x 64, MLP 3072, vocab 50257) and a
2-layer prefix of the 24-layer d=1024 model (16 heads x 64, MLP 4096, vocab
50257), random N(0, 0.02) bf16 weights, are prefilled with a batch of 2
prompts of 512 uniform token ids and decode 8 greedy tokens with the KV
cache.  The oracle (the reference's GPT-2 graph restated on the CPU,
notebook/GPT2.ipynb cells 4 and 10 with the LM head :matmul trans_b of
src/dispatch.jl:213-243) runs once, teacher-forced, over the prompt plus the
GPU's own tokens, and gives the logits after every decoded position.

Tolerance.  Both sides round to bf16 at the same points, but they sum in
different orders, so a few intermediates land one bf16 ulp apart, and a deep
random-init model carries such flips to its logits: in the oracle itself,
flipping 1% of the position-embedding values of GPT-2 small by one bf16 ulp
moves the logits by relative L2 1.1e-2 and max-abs 2.8e-2 (one layer: 4.8e-3
and 1.3e-2; tests/test_oracle_sensitivity.py measures it at a smaller size).
That floor is the north-star bound for one kernel (max-abs 2e-2, rel-L2 1e-2)
already, so a whole decoder is held to twice it: every step's logits within
max-abs 5e-2 and relative L2 2e-2.  Every greedy token must equal the
oracle's argmax, except in a near tie — a row whose oracle top-2 margin is
below the logits' observed error — where a different token can be the
larger one on either side; such a row is still checked, not skipped: the
GPU's token must then have an oracle logit within that error of the
oracle's maximum.  The output reports the top-2 margins, the near ties and
how many tokens differ from the oracle's argmax.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from _gpt_util import weights_of  # noqa: E402

pytestmark = pytest.mark.gpu

B, S, STEPS = 2, 512, 8


def _run(cfg, seed):
    from neurodsl_b200.model import GPT
    model = GPT(cfg, seed=seed)
    ids = np.random.default_rng(seed + 1).integers(0, cfg.vocab, (B, S)).astype(np.int32)
    logits = [model.prefill(torch.from_numpy(ids).cuda(), STEPS).clone()]
    for t in range(STEPS - 1):
        logits.append(model.decode_step(t).clone())
    torch.cuda.synchronize()
    got = np.stack([x.cpu().numpy() for x in logits], axis=1)       # [B][STEPS][V]
    tokens = model.tokens().cpu().numpy()                             # [B][STEPS]
    W = weights_of(model)
    del model
    torch.cuda.empty_cache()
    seq = np.concatenate([ids, tokens[:, :STEPS - 1]], axis=1)
    ref = oracle.gpt_last_logits(W, seq, act=cfg.act, eps=cfg.eps, last_k=STEPS)
    return got, ref, tokens


MAX_ABS, REL_L2 = 5e-2, 2e-2


def _check(name, got, ref, tokens):
    err = np.abs(got - ref)
    rel = [float(np.linalg.norm(got[:, k] - ref[:, k]) / np.linalg.norm(ref[:, k]))
           for k in range(STEPS)]
    srt = np.sort(ref, axis=-1)
    margin = srt[..., -1] - srt[..., -2]
    near = int((margin < err.max()).sum())
    agree = tokens == ref.argmax(-1)
    tie = margin < err.max()
    # the oracle's logit of the GPU's token, against the oracle's maximum
    gap = srt[..., -1] - np.take_along_axis(ref, tokens[..., None].astype(np.int64), -1)[..., 0]
    print(f"\n{name}: max-abs {err.max():.3e}, rel-L2 max {max(rel):.3e}, "
          f"top-2 margin min {margin.min():.3e} median {np.median(margin):.3e}, "
          f"near ties (margin < max-abs error) {near} of {margin.size}, "
          f"greedy tokens equal to the oracle's argmax {int(agree.sum())} of {agree.size}"
          f" (others: oracle-logit gap {gap[~agree].tolist()})")
    assert (agree | (tie & (gap <= err.max()))).all(), (tokens, ref.argmax(-1), margin, gap)
    assert err.max() <= MAX_ABS, err.max()
    assert max(rel) <= REL_L2, rel


def test_gpt2_small_greedy_decode_matches_oracle():
    from neurodsl_b200.model import GPT2_SMALL
    got, ref, tokens = _run(GPT2_SMALL, seed=5)
    _check("GPT-2 small", got, ref, tokens)


def test_24_layer_model_prefix_greedy_decode_matches_oracle():
    from neurodsl_b200.model import GPT_24L_1024, GPTConfig
    cfg = GPTConfig(**{**GPT_24L_1024.__dict__, "n_layer": 2})
    got, ref, tokens = _run(cfg, seed=7)
    _check("24-layer d=1024 model, first 2 layers", got, ref, tokens)
