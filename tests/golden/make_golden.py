"""Generate the committed golden fixtures for the hot-path parity tests.

Run from the repository root:  python tests/golden/make_golden.py

Each fixture is a compressed .npz holding seeded inputs and the CPU oracle's
outputs for them (the oracle restates the reference's Float32 CPU path).  The
reference publishes no golden vectors and its Julia RNG stream cannot be
reproduced without Julia, so the seeds here are NumPy PCG64 seeds, one
generator per fixture, tensors drawn in a fixed order.

Tensor-core fixtures hold bf16-rounded inputs (stored as float32) so that the
CUDA path and the oracle see identical values.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def save(name, **arrays):
    path = os.path.join(OUT, name + ".npz")
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def main():
    # 1. the reference's own test shape (test/test_runtime_optimizations.jl:55-69):
    #    rand(Float32, 8, 16) for Q, K, V; d_head = 8; causal.
    g = np.random.Generator(np.random.PCG64(1))
    Q = g.random((8, 16), dtype=np.float32)
    K = g.random((8, 16), dtype=np.float32)
    V = g.random((8, 16), dtype=np.float32)
    O, lse, m = oracle.attn_simple(Q, K, V, d_head=8, causal=True)
    save("attn_ref_shape", Q=Q, K=K, V=V, d_head=np.int32(8), causal=np.int32(1), O=O, lse=lse, m=m)

    # 2. multi-head causal prefill, head_dim 64, ragged sequence (not a tile multiple)
    g = np.random.Generator(np.random.PCG64(2))
    B, H, S, D = 1, 2, 200, 64
    Qb = oracle.bf16_round(g.standard_normal((B, H, S, D), dtype=np.float32))
    Kb = oracle.bf16_round(g.standard_normal((B, H, S, D), dtype=np.float32))
    Vb = oracle.bf16_round(g.standard_normal((B, H, S, D), dtype=np.float32))
    O, lse, m = oracle.attn_bhsd(Qb, Kb, Vb, causal=True)
    save("attn_causal_bhsd", Q=Qb, K=Kb, V=Vb, causal=np.int32(1), O=O, lse=lse, m=m)

    # 3. non-causal prefill
    g = np.random.Generator(np.random.PCG64(3))
    B, H, S, D = 2, 1, 160, 64
    Qb = oracle.bf16_round(g.standard_normal((B, H, S, D), dtype=np.float32))
    Kb = oracle.bf16_round(g.standard_normal((B, H, S, D), dtype=np.float32))
    Vb = oracle.bf16_round(g.standard_normal((B, H, S, D), dtype=np.float32))
    O, lse, m = oracle.attn_bhsd(Qb, Kb, Vb, causal=False)
    save("attn_noncausal_bhsd", Q=Qb, K=Kb, V=Vb, causal=np.int32(0), O=O, lse=lse, m=m)

    # 4. KV-cache decode: cache prefilled to L-1, one new token appended at L-1
    g = np.random.Generator(np.random.PCG64(4))
    B, H, L_max, D, L = 2, 3, 96, 64, 77
    q = oracle.bf16_round(g.standard_normal((B, H, D), dtype=np.float32))
    kc = oracle.bf16_round(g.standard_normal((B, H, L_max, D), dtype=np.float32))
    vc = oracle.bf16_round(g.standard_normal((B, H, L_max, D), dtype=np.float32))
    kc[:, :, L:, :] = 0.0
    vc[:, :, L:, :] = 0.0
    out, lse = oracle.kv_decode(q, kc, vc, L)
    save("kv_decode", q=q, k_cache=kc, v_cache=vc, L=np.int32(L), out=out, lse=lse)

    # 5. fused linear + bias + GELU, every variant, and linear + bias + residual
    g = np.random.Generator(np.random.PCG64(5))
    M, N, K = 33, 72, 64
    A = oracle.bf16_round(g.standard_normal((M, K), dtype=np.float32))
    W = oracle.bf16_round((0.02 * g.standard_normal((N, K))).astype(np.float32) * 10)
    b = g.standard_normal(N).astype(np.float32) * 0.1
    R = g.standard_normal((M, N)).astype(np.float32)
    arrays = dict(A=A, W=W, bias=b, residual=R)
    for name in ("sigmoid", "tanh", "erf"):
        arrays["Y_" + name] = oracle.linear(A, W, b, act=name)
    arrays["Y_residual"] = oracle.linear(A, W, b, residual=R)
    save("linear_gelu", **arrays)

    # 6. LayerNorm (fp32): d = 1024 and a ragged d
    g = np.random.Generator(np.random.PCG64(6))
    arrays = {}
    for d in (1024, 100):
        x = g.standard_normal((5, d)).astype(np.float32) * 3 + 0.5
        gam = g.standard_normal(d).astype(np.float32)
        bet = g.standard_normal(d).astype(np.float32)
        y, mu, rs = oracle.layernorm(x, gam, bet, eps=1e-5)
        arrays.update({f"x{d}": x, f"gamma{d}": gam, f"beta{d}": bet, f"y{d}": y, f"mean{d}": mu,
                       f"rstd{d}": rs})
    save("layernorm", **arrays)


if __name__ == "__main__":
    main()
