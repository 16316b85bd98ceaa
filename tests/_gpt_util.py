"""Test helpers: the weights of a neurodsl_b200.model.GPT rank as the float32
NumPy dict that oracle.gpt_last_logits takes."""
import numpy as np


def weights_of(model):
    f = lambda t: t.detach().float().cpu().numpy()
    W = {"wte": f(model.wte), "wpe": f(model.wpe), "w_head": f(model.w_head),
         "lnf_g": f(model.lnf_g), "lnf_b": f(model.lnf_b), "layers": []}
    for L in model.layers:
        W["layers"].append({k: f(v) for k, v in L.items()})
    return W


def top2_margin(logits):
    s = np.sort(logits, axis=-1)
    return s[..., -1] - s[..., -2]
