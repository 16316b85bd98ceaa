"""The rounding noise floor of a decoder's logits, measured on the oracle alone.

Both the GPU path and the oracle round activations to bf16 at the same points
but sum in different orders, so a few intermediates end up one bf16 ulp
apart.  This test measures how far such flips move a random-init decoder's
logits in the oracle itself: GPT-2-small widths (d 768, 12 heads, MLP 3072),
N(0, 0.02) bf16 weights, with one bf16 ulp added to 1% of the position
embeddings.  The decoder parity tests (tests/test_model_config_gpu.py) take
their tolerance from this floor; it is asserted here to stay well above the
1e-3 level a kernel-level tolerance would assume.
"""
import numpy as np

import oracle


def _weights(rng, L, d=768, F=3072, V=4096, n_pos=256):
    bf = oracle.bf16_round
    r = lambda *s: bf((rng.standard_normal(s, dtype=np.float32) * 0.02).astype(np.float32))
    one, zero = (lambda n: np.ones(n, np.float32)), (lambda n: np.zeros(n, np.float32))
    W = {"wte": r(V, d), "wpe": r(n_pos, d), "lnf_g": one(d), "lnf_b": zero(d), "layers": []}
    W["w_head"] = W["wte"]
    for _ in range(L):
        W["layers"].append({"ln1_g": one(d), "ln1_b": zero(d), "w_qkv": r(3 * d, d),
                            "b_qkv": zero(3 * d), "w_o": r(d, d), "b_o": zero(d),
                            "ln2_g": one(d), "ln2_b": zero(d), "w_1": r(F, d), "b_1": zero(F),
                            "w_2": r(d, F), "b_2": zero(d)})
    return W


def test_one_ulp_flips_move_decoder_logits_by_about_one_percent():
    rng = np.random.default_rng(0)
    W = _weights(rng, L=2)
    ids = rng.integers(0, W["wte"].shape[0], (2, 64))
    a = oracle.gpt_last_logits(W, ids)
    wpe = W["wpe"].copy()
    bits = wpe.view(np.uint32)
    bits[rng.random(wpe.shape) < 0.01] += np.uint32(1 << 16)     # one bf16 ulp up
    b = oracle.gpt_last_logits({**W, "wpe": wpe}, ids)
    rel = float(np.linalg.norm(a - b) / np.linalg.norm(a))
    print(f"\nrel-L2 {rel:.3e}, max-abs {np.abs(a - b).max():.3e}")
    assert 2e-3 < rel < 5e-2
