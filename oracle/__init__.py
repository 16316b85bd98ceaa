"""CPU oracle for the NeuroDSL hot path — test infrastructure only.

NumPy-facing wrappers over ``liboracle.so`` (built from ``neurodsl_oracle.c``
by ``oracle/Makefile``).  Only the test suite, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg import this package, as the checker or as the
timed CPU baseline; the library in ``neurodsl_b200`` never does.

Parity status: unpinned against reference outputs (the Julia reference cannot
run here and its tests hold no golden vectors); the reference's own tiled-vs-
simple equivalence test is re-asserted on this restatement by the test suite.

All arrays are C row-major float32.  Each function names the reference
function it restates (file:line inside the NeuroDSL project).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

GELU_NONE, GELU_SIGMOID, GELU_TANH, GELU_ERF = 0, 1, 2, 3
GELU_BY_NAME = {"none": GELU_NONE, "sigmoid": GELU_SIGMOID, "tanh": GELU_TANH, "erf": GELU_ERF}


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, no GPU needed)."""
    src = os.path.join(_HERE, "neurodsl_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        i = ctypes.c_int
        L.oracle_attn_simple.argtypes = [fp, fp, fp, fp, fp, fp, i, i, i, i, i, fp]
        L.oracle_attn_tiled.argtypes = [fp, fp, fp, fp, fp, fp, i, i, i, i, i, i, fp, fp, fp]
        L.oracle_attn_simple_bhsd.argtypes = [fp, fp, fp, fp, fp, fp, i, i, i, i, i, i, i]
        L.oracle_kv_decode.argtypes = [fp, fp, fp, fp, fp, i, i, i, i, i, i]
        L.oracle_linear.argtypes = [fp, fp, fp, fp, fp, i, i, i, i, i, i]
        L.oracle_layernorm.argtypes = [fp, fp, fp, fp, fp, fp, i, i, ctypes.c_float]
        L.oracle_rmsnorm.argtypes = [fp, fp, fp, fp, i, i, ctypes.c_float]
        L.oracle_softmax.argtypes = [fp, fp, i, i]
        L.oracle_scale_mask.argtypes = [fp, fp, i, i]
        for f in ("oracle_attn_simple", "oracle_attn_tiled", "oracle_attn_simple_bhsd",
                  "oracle_kv_decode", "oracle_linear", "oracle_layernorm", "oracle_rmsnorm",
                  "oracle_softmax", "oracle_scale_mask"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    if a is None:
        return None
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _check(rc, name):
    if rc != 0:
        raise ValueError(f"oracle {name} failed with status {rc}")


def attn_simple(Q, K, V, d_head=None, causal=True):
    """flash_attn_fwd_cpu_simple! (src/flash_attention.jl:49-69) on one head.

    Q (N,D), K/V (Nk,D).  Returns (O, lse, m) like the reference.
    """
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    N, D = Q.shape
    Nk = K.shape[0]
    d_head = D if d_head is None else d_head
    O = np.zeros((N, D), np.float32)
    lse = np.zeros(N, np.float32)
    m = np.zeros(N, np.float32)
    work = np.zeros(max(N * Nk, 1), np.float32)
    _check(lib().oracle_attn_simple(_p(Q), _p(K), _p(V), _p(O), _p(lse), _p(m), N, Nk, D,
                                    d_head, int(bool(causal)), _p(work)), "attn_simple")
    return O, lse, m


def attn_tiled(Q, K, V, d_head=None, causal=True, block_size=64):
    """flash_attn_fwd_cpu! (src/flash_attention.jl:9-46), FLASH_BLOCK = 64."""
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    N, D = Q.shape
    Nk = K.shape[0]
    d_head = D if d_head is None else d_head
    O = np.zeros((N, D), np.float32)
    lse = np.zeros(N, np.float32)
    m = np.zeros(N, np.float32)
    work = np.zeros(max(N * block_size, 1), np.float32)
    lb = np.zeros(max(N, 1), np.float32)
    mb = np.zeros(max(N, 1), np.float32)
    _check(lib().oracle_attn_tiled(_p(Q), _p(K), _p(V), _p(O), _p(lse), _p(m), N, Nk, D, d_head,
                                   int(bool(causal)), block_size, _p(work), _p(lb), _p(mb)),
           "attn_tiled")
    return O, lse, m


def attn_bhsd(Q, K, V, causal=True, nthreads=0):
    """a1 over every head of head-major [B][H][S][D] tensors.  Returns (O, lse, m)."""
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    B, H, S, D = Q.shape
    Sk = K.shape[2]
    O = np.zeros((B, H, S, D), np.float32)
    lse = np.zeros((B, H, S), np.float32)
    m = np.zeros((B, H, S), np.float32)
    _check(lib().oracle_attn_simple_bhsd(_p(Q), _p(K), _p(V), _p(O), _p(lse), _p(m), B, H, S, Sk,
                                         D, int(bool(causal)), int(nthreads)), "attn_bhsd")
    return O, lse, m


def kv_decode(q, k_cache, v_cache, L, nthreads=0):
    """Single-token decode: a1 with one query row, causal=false, over keys [0, L).

    q [B][H][D]; caches [B][H][L_max][D].  Returns (out [B][H][D], lse [B][H]).
    """
    q, k_cache, v_cache = _f32(q), _f32(k_cache), _f32(v_cache)
    B, H, D = q.shape
    L_max = k_cache.shape[2]
    out = np.zeros((B, H, D), np.float32)
    lse = np.zeros((B, H), np.float32)
    _check(lib().oracle_kv_decode(_p(q), _p(k_cache), _p(v_cache), _p(out), _p(lse), B, H, int(L),
                                  L_max, D, int(nthreads)), "kv_decode")
    return out, lse


def linear(A, W, bias=None, residual=None, trans_w=True, act="none", nthreads=0):
    """act(A·op(W) + bias) + residual — :linear / :fused_matmul_add / fused_linear_gelu."""
    A, W = _f32(A), _f32(W)
    M, K = A.shape
    N = W.shape[0] if trans_w else W.shape[1]
    Y = np.zeros((M, N), np.float32)
    b = None if bias is None else _f32(bias).reshape(-1)
    r = None if residual is None else _f32(residual)
    _check(lib().oracle_linear(_p(A), _p(W), _p(b), _p(r), _p(Y), M, N, K, int(bool(trans_w)),
                               GELU_BY_NAME[act] if isinstance(act, str) else int(act),
                               int(nthreads)), "linear")
    return Y


def layernorm(x, gamma=None, beta=None, eps=1e-5):
    """LayerNorm per row; returns (y, mean, rstd)."""
    x = _f32(x)
    rows, d = x.shape
    y = np.zeros_like(x)
    mean = np.zeros(rows, np.float32)
    rstd = np.zeros(rows, np.float32)
    g = None if gamma is None else _f32(gamma)
    b = None if beta is None else _f32(beta)
    _check(lib().oracle_layernorm(_p(x), _p(g), _p(b), _p(y), _p(mean), _p(rstd), rows, d,
                                  float(eps)), "layernorm")
    return y, mean, rstd


def rmsnorm(x, gamma, eps=1e-6):
    """rmsnorm_fwd! (src/kernels.jl:48-64); returns (y, rms_inv)."""
    x, gamma = _f32(x), _f32(gamma)
    rows, d = x.shape
    y = np.zeros_like(x)
    inv = np.zeros(rows, np.float32)
    _check(lib().oracle_rmsnorm(_p(x), _p(gamma), _p(y), _p(inv), rows, d, float(eps)), "rmsnorm")
    return y, inv


def softmax(x):
    """softmax_fwd! CPU (src/kernels.jl:269-287)."""
    x = _f32(x)
    out = np.zeros_like(x)
    _check(lib().oracle_softmax(_p(x), _p(out), x.shape[0], x.shape[1]), "softmax")
    return out


def scale_mask(scores, d_head):
    """scale_mask_fwd! with the causal mask (src/kernels.jl:427-430)."""
    s = _f32(scores)
    out = np.zeros_like(s)
    _check(lib().oracle_scale_mask(_p(s), _p(out), s.shape[0], int(d_head)), "scale_mask")
    return out


def bf16_round(a):
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32.

    Inputs fed to the bf16 tensor-core kernels are rounded this way before the
    oracle sees them, so only accumulation order and precision differ.
    """
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def gpt_last_logits(W, ids, act="tanh", eps=1e-5, reduce=None, last_k=1):
    """LM-head logits of the last position of each sequence ids [B][T] for a
    pre-LayerNorm GPT decoder — the composition of the reference's GPT-2 graph
    (notebook/GPT2.ipynb cells 4 and 10): token + position :embedding
    (src/dispatch.jl:476-491) and :add, per block LayerNorm -> Q/K/V :linear
    (:363-384) -> causal attention per head (flash_attn_fwd_cpu_simple!,
    src/flash_attention.jl:49-69) -> output :linear -> residual :add
    (:386-417) -> LayerNorm -> :linear + GELU (fused_linear_gelu) -> :linear
    -> residual :add; final LayerNorm and the LM head :matmul trans_b
    (:213-243) against the embedding rows.

    W holds float32 arrays (the bf16 weight values): wte [V][d], wpe, w_head
    [V_local][d] (LM-head rows), lnf_g, lnf_b and layers: a list of dicts with
    ln1_g, ln1_b, w_qkv [3·d_local][d] (Q, K, V rows of the local heads),
    b_qkv, w_o [d][d_local], b_o, ln2_g, ln2_b, w_1 [F_local][d], b_1,
    w_2 [d][F_local], b_2.  `reduce(x)` sums a partial result over the ranks
    of a tensor-parallel split (identity for one rank).  Values that the GPU
    path stores in bf16 are rounded to bf16 at the same points, so the two
    differ only in accumulation order and approximate functions.

    Returns the logits of the last position of each sequence, [B][V_local];
    with last_k > 1, those of the last last_k positions, [B][last_k][V_local]
    (the causal model's predictions after each of those positions, so one
    pass over a prompt plus generated tokens checks every decode step).
    """
    ids = np.asarray(ids)
    B, T = ids.shape
    red = reduce if reduce is not None else (lambda a: a)
    x = bf16_round(W["wte"][ids.reshape(-1)] + W["wpe"][np.tile(np.arange(T), B)])
    L0 = W["layers"][0]
    h = bf16_round(layernorm(x, L0["ln1_g"], L0["ln1_b"], eps)[0])
    n = len(W["layers"])
    for i, L in enumerate(W["layers"]):
        dl = L["w_qkv"].shape[0] // 3
        H = dl // 64
        qkv = bf16_round(linear(h, L["w_qkv"], L["b_qkv"])).reshape(B, T, 3, H, 64)
        attn = np.zeros((B, T, H, 64), np.float32)
        for b in range(B):
            for hh in range(H):
                o, _, _ = attn_simple(qkv[b, :, 0, hh], qkv[b, :, 1, hh], qkv[b, :, 2, hh],
                                      causal=True)
                attn[b, :, hh] = o
        attn = bf16_round(attn.reshape(B * T, dl))
        part = bf16_round(red(bf16_round(linear(attn, L["w_o"]))))
        x = bf16_round(x + (part + L["b_o"]))
        h = bf16_round(layernorm(x, L["ln2_g"], L["ln2_b"], eps)[0])
        u = bf16_round(linear(h, L["w_1"], L["b_1"], act=act))
        part = bf16_round(red(bf16_round(linear(u, L["w_2"]))))
        x = bf16_round(x + (part + L["b_2"]))
        nxt = W["layers"][i + 1] if i + 1 < n else None
        g, be = (nxt["ln1_g"], nxt["ln1_b"]) if nxt else (W["lnf_g"], W["lnf_b"])
        h = bf16_round(layernorm(x, g, be, eps)[0])
    if last_k == 1:
        return linear(h.reshape(B, T, -1)[:, -1], W["w_head"])
    last = h.reshape(B, T, -1)[:, -last_k:].reshape(B * last_k, -1)
    return linear(last, W["w_head"]).reshape(B, last_k, -1)
