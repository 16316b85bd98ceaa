"""Torch-tensor front end of the C ABI: one function per hot-path kernel.

Tensors are CUDA tensors (torch is used only to own device memory and to
name the current stream); each call validates dtype/shape/contiguity here
and then calls the corresponding nd_* entry point, which validates again.
Outputs are allocated here when the caller passes none.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import check

_DT = {torch.float32: _lib.ND_F32, torch.bfloat16: _lib.ND_BF16}
ACT = {"none": _lib.ND_ACT_NONE, "sigmoid": _lib.ND_ACT_GELU_SIGMOID,
       "tanh": _lib.ND_ACT_GELU_TANH, "erf": _lib.ND_ACT_GELU_ERF}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _need(t, name, dtype=None, dims=None, contiguous=True):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if dims is not None and t.dim() != dims:
        raise ValueError(f"{name} must have {dims} dims, got shape {tuple(t.shape)}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _row_strides(t, name):
    """{row, head, batch} element strides of a [B][H][S][64] view, D contiguous."""
    if t.stride(3) != 1:
        raise ValueError(f"{name}: the 64 head dims of a row must be contiguous")
    return (ctypes.c_int64 * 3)(t.stride(2), t.stride(1), t.stride(0))


def flash_attn_fwd(Q, K, V, causal=True, scale=None, out=None, out_dtype=torch.bfloat16,
                   lse=None, row_max=None, stream=None):
    """O = softmax(Q·Kᵀ·scale [causal]) · V for [B][H][S][64] bf16 tensors.

    Mirrors flash_attn_fwd!(dev, out, Q, K, V, d_head; causal)
    (src/flash_attention.jl:113-134); returns (O, lse, row_max) like the
    reference's (out, l, m).  Q, K, V and `out` may be strided views, e.g.
    token-major slices of an (S, 3·H·64) QKV projection viewed as
    [B][H][S][64]; they are then read and written in place
    (nd_flash_attn_fwd_strided) instead of being copied per head.
    """
    for n, t in (("Q", Q), ("K", K), ("V", V)):
        _need(t, n, torch.bfloat16, 4, contiguous=False)
    B, H, Sq, D = Q.shape
    Sk = K.shape[2]
    if K.shape != (B, H, Sk, D) or V.shape != K.shape:
        raise ValueError(f"shape mismatch Q{tuple(Q.shape)} K{tuple(K.shape)} V{tuple(V.shape)}")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, H, Sq, D), dtype=out_dtype, device=Q.device)
    _need(out, "out", None, 4, contiguous=False)
    if tuple(out.shape) != (B, H, Sq, D):
        raise ValueError(f"out{tuple(out.shape)} != {(B, H, Sq, D)}")
    if lse is None:
        lse = torch.empty((B, H, Sq), dtype=torch.float32, device=Q.device)
    if row_max is None:
        row_max = torch.empty((B, H, Sq), dtype=torch.float32, device=Q.device)
    lib = _lib.load()
    if all(t.is_contiguous() for t in (Q, K, V, out)):
        check(lib.nd_flash_attn_fwd(_stream(stream), _ptr(Q), _ptr(K), _ptr(V), _ptr(out),
                                    _DT[out.dtype], _ptr(lse), _ptr(row_max), B, H, Sq, Sk,
                                    D, float(scale), int(bool(causal))))
    else:
        check(lib.nd_flash_attn_fwd_strided(
            _stream(stream), _ptr(Q), _row_strides(Q, "Q"), _ptr(K), _row_strides(K, "K"),
            _ptr(V), _row_strides(V, "V"), _ptr(out), _row_strides(out, "out"), _DT[out.dtype],
            _ptr(lse), _ptr(row_max), B, H, Sq, Sk, D, float(scale), int(bool(causal))))
    return out, lse, row_max


def kv_decode_workspace_size(B, H, L, D=64):
    n = ctypes.c_size_t(0)
    check(_lib.load().nd_kv_decode_workspace_size(B, H, L, D, ctypes.byref(n)))
    return n.value


def kv_decode_attn(q, k_cache, v_cache, L, k_new=None, v_new=None, scale=None, out=None,
                   out_dtype=torch.bfloat16, lse=None, workspace=None, want_lse=True,
                   stream=None):
    """Single-token decode over keys [0, L) of [B][H][L_max][64] bf16 caches.

    With k_new/v_new the token at L-1 is appended to the caches in the same
    pass.  Returns (out [B][H][64], lse [B][H]).
    """
    _need(q, "q", torch.bfloat16, 3)
    _need(k_cache, "k_cache", torch.bfloat16, 4)
    _need(v_cache, "v_cache", torch.bfloat16, 4)
    B, H, D = q.shape
    L_max = k_cache.shape[2]
    if k_cache.shape != (B, H, L_max, D) or v_cache.shape != k_cache.shape:
        raise ValueError("cache shape mismatch")
    if (k_new is None) != (v_new is None):
        raise ValueError("k_new and v_new go together")
    if k_new is not None:
        _need(k_new, "k_new", torch.bfloat16, 3)
        _need(v_new, "v_new", torch.bfloat16, 3)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, H, D), dtype=out_dtype, device=q.device)
    if lse is None and want_lse:
        lse = torch.empty((B, H), dtype=torch.float32, device=q.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(_lib.load().nd_kv_decode_attn(_stream(stream), _ptr(q), _ptr(k_new), _ptr(v_new),
                                        _ptr(k_cache), _ptr(v_cache), _ptr(out), _DT[out.dtype],
                                        _ptr(lse), B, H, int(L), L_max, D, float(scale),
                                        _ptr(workspace), ws_bytes))
    return out, lse


def kv_decode_attn_qkv(qkv, k_cache, v_cache, L, scale=None, out=None, out_dtype=torch.bfloat16,
                       lse=None, workspace=None, want_lse=False, stream=None):
    """Decode attention from a fused QKV projection qkv [B][3*H*64] (bf16,
    unit column stride; rows may be padded): q, k_new and v_new are its three
    column blocks, and k_new / v_new are appended at position L-1.
    Returns (out [B][H][64], lse [B][H] or None)."""
    if not isinstance(qkv, torch.Tensor) or qkv.dtype != torch.bfloat16 or qkv.dim() != 2:
        raise ValueError("qkv must be a 2-D bf16 tensor")
    if not qkv.is_cuda or qkv.stride(1) != 1:
        raise ValueError("qkv must be a CUDA tensor with unit column stride")
    _need(k_cache, "k_cache", torch.bfloat16, 4)
    _need(v_cache, "v_cache", torch.bfloat16, 4)
    B = qkv.shape[0]
    _, H, L_max, D = k_cache.shape
    if k_cache.shape[0] != B or v_cache.shape != k_cache.shape or qkv.shape[1] != 3 * H * D:
        raise ValueError("qkv / cache shape mismatch")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, H, D), dtype=out_dtype, device=qkv.device)
    if lse is None and want_lse:
        lse = torch.empty((B, H), dtype=torch.float32, device=qkv.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(_lib.load().nd_kv_decode_attn_qkv(_stream(stream), _ptr(qkv), qkv.stride(0),
                                            _ptr(k_cache), _ptr(v_cache), _ptr(out),
                                            _DT[out.dtype], _ptr(lse), B, H, int(L), L_max, D,
                                            float(scale), _ptr(workspace), ws_bytes))
    return out, lse


def set_pdl(enable):
    """Programmatic dependent launch for this thread's decode-step kernels
    (nd_set_pdl); returns the previous setting."""
    prev = ctypes.c_int(0)
    check(_lib.load().nd_set_pdl(1 if enable else 0, ctypes.byref(prev)))
    return bool(prev.value)


class pdl:
    """Context manager: launches inside run with programmatic dependent
    launch on (or off), restoring the previous setting on exit."""

    def __init__(self, enable=True):
        self.enable = enable

    def __enter__(self):
        self.prev = set_pdl(self.enable)
        return self

    def __exit__(self, *exc):
        set_pdl(self.prev)
        return False


def set_sm_limit(sms):
    """Cap the SMs this thread's persistent GEMM / prefill-attention launches
    occupy (nd_set_sm_limit; 0 = all); returns the previous setting."""
    prev = ctypes.c_int(0)
    check(_lib.load().nd_set_sm_limit(int(sms), ctypes.byref(prev)))
    return prev.value


class sm_limit:
    """Context manager: launches inside leave all but `sms` SMs to other
    streams' kernels (0 = no cap), restoring the previous cap on exit."""

    def __init__(self, sms):
        self.sms = sms

    def __enter__(self):
        self.prev = set_sm_limit(self.sms)
        return self

    def __exit__(self, *exc):
        set_sm_limit(self.prev)
        return False


def kv_append(k_new, v_new, k_cache, v_cache, pos, stream=None):
    _need(k_new, "k_new", torch.bfloat16, 3)
    _need(v_new, "v_new", torch.bfloat16, 3)
    B, H, D = k_new.shape
    L_max = k_cache.shape[2]
    check(_lib.load().nd_kv_append(_stream(stream), _ptr(k_new), _ptr(v_new), _ptr(k_cache),
                                   _ptr(v_cache), B, H, int(pos), L_max, D))


def linear(A, W, bias=None, residual=None, act="none", out=None, out_dtype=torch.bfloat16,
           stream=None):
    """Y = act(A·Wᵀ + bias) + residual with A [M][K], W [N][K] bf16.

    :linear (src/dispatch.jl:363-384) / fused_linear_gelu
    (notebook/compiler.ipynb cell 15) with the GELU variant `act`.
    """
    _need(A, "A", torch.bfloat16, 2)
    _need(W, "W", torch.bfloat16, 2)
    M, K = A.shape
    N = W.shape[0]
    if W.shape[1] != K:
        raise ValueError(f"A{tuple(A.shape)} and W{tuple(W.shape)} disagree on K")
    if bias is not None:
        _need(bias, "bias", torch.float32)
        if bias.numel() != N:
            raise ValueError("bias length != N")
    rdt = _lib.ND_F32
    if residual is not None:
        _need(residual, "residual", None, 2)
        if tuple(residual.shape) != (M, N):
            raise ValueError("residual shape != (M, N)")
        rdt = _DT[residual.dtype]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=A.device)
    _need(out, "out", None, 2)
    check(_lib.load().nd_gemm_bias_act(_stream(stream), _ptr(A), _ptr(W), _ptr(bias),
                                       _ptr(residual), rdt, _ptr(out), _DT[out.dtype], M, N, K,
                                       ACT[act] if isinstance(act, str) else int(act)))
    return out


def linear_qkv_cache(A, W, bias, out, k_cache, v_cache, B, S, pos0=0, stream=None):
    """The QKV projection out = A·Wᵀ + bias (A [B*S][K], W [3*H*64][K], bf16
    out) that also writes its K and V column blocks into the head-major
    caches [B][H][L_max][64] at positions pos0.. (nd_gemm_qkv_cache)."""
    _need(A, "A", torch.bfloat16, 2)
    _need(W, "W", torch.bfloat16, 2)
    _need(out, "out", torch.bfloat16, 2)
    _need(k_cache, "k_cache", torch.bfloat16, 4)
    _need(v_cache, "v_cache", torch.bfloat16, 4)
    M, K = A.shape
    _, H, L_max, D = k_cache.shape
    if D != 64 or W.shape != (3 * H * 64, K) or tuple(out.shape) != (M, 3 * H * 64):
        raise ValueError("QKV projection / cache shape mismatch")
    if v_cache.shape != k_cache.shape or k_cache.shape[0] != B:
        raise ValueError("cache shape mismatch")
    if bias is not None:
        _need(bias, "bias", torch.float32)
    check(_lib.load().nd_gemm_qkv_cache(_stream(stream), _ptr(A), _ptr(W), _ptr(bias), _ptr(out),
                                        M, K, _ptr(k_cache), _ptr(v_cache), int(B), int(S), H,
                                        L_max, int(pos0)))
    return out


def linear_qkv_cache_peers(A, W, bias, out, k_caches, v_caches, H, L_max, B, b0, S, pos0=0,
                           stream=None):
    """The full-head QKV projection of this rank's B prompts (sequences b0..)
    writing the K/V columns of head h into the cache of rank h // H
    (nd_gemm_qkv_cache_peers); k_caches / v_caches: every rank's cache base
    pointer (ints, [..][H][L_max][64] bf16), this rank's own included."""
    _need(A, "A", torch.bfloat16, 2)
    _need(W, "W", torch.bfloat16, 2)
    _need(out, "out", torch.bfloat16, 2)
    _need(bias, "bias", torch.float32, 1)
    tp = len(k_caches)
    M, K = A.shape
    if W.shape != (3 * tp * H * 64, K) or tuple(out.shape) != (M, 3 * tp * H * 64) or M != B * S:
        raise ValueError("QKV projection / cache shape mismatch")
    kc = (ctypes.c_void_p * tp)(*k_caches)
    vc = (ctypes.c_void_p * tp)(*v_caches)
    check(_lib.load().nd_gemm_qkv_cache_peers(_stream(stream), _ptr(A), _ptr(W), _ptr(bias),
                                              _ptr(out), M, K, kc, vc, tp, int(B), int(b0),
                                              int(S), int(H), int(L_max), int(pos0)))
    return out


def ln_linear(x, W, p=None, p_bias=None, gamma=None, beta=None, eps=1e-5, s_out=None, bias=None,
              act="none", out=None, out_dtype=torch.bfloat16, stream=None):
    """Y = act(LayerNorm(x + p + p_bias)·Wᵀ + bias) for at most 32 rows, with
    the residual sum s = bf16(x + p + p_bias) written to s_out if given
    (nd_ln_gemm: residual :add + :layernorm + :linear in one launch)."""
    _need(x, "x", torch.bfloat16, 2)
    _need(W, "W", torch.bfloat16, 2)
    M, K = x.shape
    N = W.shape[0]
    if W.shape[1] != K:
        raise ValueError(f"x{tuple(x.shape)} and W{tuple(W.shape)} disagree on K")
    for name, t in (("p", p), ("s_out", s_out)):
        if t is not None:
            _need(t, name, torch.bfloat16, 2)
            if tuple(t.shape) != (M, K):
                raise ValueError(f"{name} shape != x shape")
    for name, t, n in (("p_bias", p_bias, K), ("gamma", gamma, K), ("beta", beta, K),
                       ("bias", bias, N)):
        if t is not None:
            _need(t, name, torch.float32)
            if t.numel() != n:
                raise ValueError(f"{name} length != {n}")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    _need(out, "out", None, 2)
    check(_lib.load().nd_ln_gemm(_stream(stream), _ptr(x), _ptr(p), _ptr(p_bias), _ptr(gamma),
                                 _ptr(beta), float(eps), _ptr(s_out), _ptr(W), _ptr(bias),
                                 _ptr(out), _DT[out.dtype], M, N, K,
                                 ACT[act] if isinstance(act, str) else int(act)))
    return out


def gelu(x, act="sigmoid", out=None, stream=None):
    """Elementwise GELU of a float32 tensor (nd_gelu, the unfused :gelu op)."""
    _need(x, "x", torch.float32)
    if out is None:
        out = torch.empty_like(x)
    _need(out, "out", torch.float32)
    check(_lib.load().nd_gelu(_stream(stream), _ptr(x), _ptr(out), x.numel(),
                              ACT[act] if isinstance(act, str) else int(act)))
    return out


def scale_mask(scores, d_head, out=None, stream=None):
    """scores / sqrt(d_head) with the causal mask (-Inf above the diagonal) of
    one float32 [rows][cols] block (nd_scale_mask, the :scale_mask op)."""
    _need(scores, "scores", torch.float32, 2)
    if out is None:
        out = torch.empty_like(scores)
    _need(out, "out", torch.float32, 2)
    check(_lib.load().nd_scale_mask(_stream(stream), _ptr(scores), _ptr(out), scores.shape[0],
                                    scores.shape[1], int(d_head)))
    return out


def add(a, b, out=None, stream=None):
    """a + b for float32 tensors (nd_add, the :add op): b of a's shape; a
    vector of one value per column, else per row, of a 2-D a (the
    reference's vector cases, columns preferred); or, as its general
    broadcast does, a (1, cols) row, a (rows, 1) column or a single value."""
    _need(a, "a", torch.float32)
    _need(b, "b", torch.float32)
    rows, cols = (a.shape[0], a.shape[1]) if a.dim() == 2 else (1, a.numel())
    if tuple(b.shape) == tuple(a.shape):
        mode = 0
    elif a.dim() == 2 and b.dim() == 1 and b.numel() == cols:
        mode = 1
    elif a.dim() == 2 and b.dim() == 1 and b.numel() == rows:
        mode = 2
    elif a.dim() == 2 and b.dim() == 2 and tuple(b.shape) == (1, cols):
        mode = 1
    elif a.dim() == 2 and b.dim() == 2 and tuple(b.shape) == (rows, 1):
        mode = 2
    elif b.numel() == 1 and b.dim() <= a.dim():
        mode = 3
    else:
        raise ValueError(f"add: shapes {tuple(a.shape)} and {tuple(b.shape)} do not broadcast")
    if out is None:
        out = torch.empty_like(a)
    _need(out, "out", torch.float32)
    check(_lib.load().nd_add(_stream(stream), _ptr(a), _ptr(b), _ptr(out), rows, cols, mode))
    return out


def softmax(x, out=None, stream=None):
    """Row softmax of a float32 [rows][cols] matrix (nd_softmax, the :softmax op)."""
    _need(x, "x", torch.float32, 2)
    if out is None:
        out = torch.empty_like(x)
    _need(out, "out", torch.float32, 2)
    check(_lib.load().nd_softmax(_stream(stream), _ptr(x), _ptr(out), x.shape[0], x.shape[1]))
    return out


def layernorm(x, gamma=None, beta=None, eps=1e-5, out=None, out_dtype=None, mean=None,
              rstd=None, stats=True, stream=None):
    """Row LayerNorm of x [rows][d]; returns (y, mean, rstd).  With
    stats=False and no mean/rstd buffers the statistics are not written
    (mean and rstd come back as None)."""
    _need(x, "x", None, 2)
    rows, d = x.shape
    if out is None:
        out = torch.empty((rows, d), dtype=out_dtype or x.dtype, device=x.device)
    if mean is None and stats:
        mean = torch.empty(rows, dtype=torch.float32, device=x.device)
    if rstd is None and stats:
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    for n, t in (("gamma", gamma), ("beta", beta)):
        if t is not None:
            _need(t, n, torch.float32)
    check(_lib.load().nd_layernorm(_stream(stream), _ptr(x), _DT[x.dtype], _ptr(gamma),
                                   _ptr(beta), _ptr(out), _DT[out.dtype], _ptr(mean), _ptr(rstd),
                                   rows, d, float(eps)))
    return out, mean, rstd


def convert_2d(src, rows, cols, src_col_major, dst_dtype, out=None, stream=None):
    """Column-major (Julia) or row-major 2-D matrix -> row-major [rows][cols]."""
    _need(src, "src")
    if src.numel() != rows * cols:
        raise ValueError("src size != rows*cols")
    if out is None:
        out = torch.empty((rows, cols), dtype=dst_dtype, device=src.device)
    check(_lib.load().nd_convert_2d(_stream(stream), _ptr(src), _DT[src.dtype],
                                    int(bool(src_col_major)), _ptr(out), _DT[out.dtype], rows,
                                    cols))
    return out


def convert_2d_padded(src, rows, cols, src_col_major, dst_dtype, ld_dst, out=None, stream=None):
    """convert_2d into rows of ld_dst >= cols elements, the columns past cols
    zero (nd_convert_2d_padded): [rows][ld_dst]."""
    _need(src, "src")
    if src.numel() != rows * cols:
        raise ValueError("src size != rows*cols")
    if out is None:
        out = torch.empty((rows, ld_dst), dtype=dst_dtype, device=src.device)
    if tuple(out.shape) != (rows, ld_dst) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [rows][ld_dst] matrix")
    check(_lib.load().nd_convert_2d_padded(_stream(stream), _ptr(src), _DT[src.dtype],
                                           int(bool(src_col_major)), _ptr(out), _DT[out.dtype],
                                           rows, cols, ld_dst))
    return out


_IDX_DT = {torch.float32: _lib.ND_F32, torch.int32: _lib.ND_I32, torch.int64: _lib.ND_I64}


def gather_rows(table, idx, index_base=1, out=None, stream=None):
    """out[i] = table[idx[i] - index_base] on the device (nd_gather_rows: the
    :embedding op).  table [vocab][d] fp32 or bf16 with unit column stride;
    idx any shape of float32 / int32 / int64 indices on the device.  A bad
    index gives a zero row and sets the device error word (device_error()),
    without a host synchronisation."""
    if table.dim() != 2 or table.stride(1) != 1:
        raise ValueError("table must be 2-D with contiguous rows")
    if table.dtype not in _DT:
        raise ValueError(f"table dtype {table.dtype} not supported")
    if idx.dtype not in _IDX_DT:
        raise ValueError(f"index dtype {idx.dtype} not supported")
    if idx.device != table.device:
        raise ValueError("indices and table must be on the same device")
    idx = idx.reshape(-1).contiguous()
    n = idx.numel()
    vocab, d = table.shape
    if out is None:
        out = torch.empty((n, d), dtype=table.dtype, device=table.device)
    if out.dim() != 2 or tuple(out.shape) != (n, d) or out.stride(1) != 1 or out.dtype != table.dtype:
        raise ValueError("out must be an [n][d] matrix of the table's dtype with contiguous rows")
    check(_lib.load().nd_gather_rows(_stream(stream), _ptr(table), _DT[table.dtype],
                                     table.stride(0), vocab, _ptr(idx), _IDX_DT[idx.dtype],
                                     int(index_base), n, d, _ptr(out), out.stride(0)))
    return out


def copy_2d(src, dst, stream=None):
    """dst[:, :] = src[:, :] for 2-D views with unit column strides
    (nd_copy_2d: the :slice_cols, :hcat_heads and :identity copies)."""
    for name, t in (("src", src), ("dst", dst)):
        if t.dim() != 2 or (t.shape[1] > 1 and t.stride(1) != 1):
            raise ValueError(f"{name} must be 2-D with contiguous rows")
    if tuple(src.shape) != tuple(dst.shape) or src.dtype != dst.dtype:
        raise ValueError("src and dst differ in shape or dtype")
    rows, cols = src.shape
    ld = lambda t: t.stride(0) if rows > 1 else cols
    check(_lib.load().nd_copy_2d(_stream(stream), _ptr(src), ld(src), _ptr(dst), ld(dst), rows,
                                 cols, src.element_size()))
    return dst


def copy_2d_batched(src, dst, stream=None):
    """dst[b, :, :] = src[b, :, :] for 3-D views whose rows are contiguous
    (nd_copy_2d_batched: any batch and row strides)."""
    for name, t in (("src", src), ("dst", dst)):
        if not t.is_cuda or t.dim() != 3 or (t.shape[2] > 1 and t.stride(2) != 1):
            raise ValueError(f"{name} must be a 3-D CUDA view with contiguous rows")
    if tuple(src.shape) != tuple(dst.shape) or src.dtype != dst.dtype:
        raise ValueError("src and dst differ in shape or dtype")
    batch, rows, cols = src.shape
    check(_lib.load().nd_copy_2d_batched(_stream(stream), _ptr(src), src.stride(1), src.stride(0),
                                         _ptr(dst), dst.stride(1), dst.stride(0), batch, rows,
                                         cols, src.element_size()))
    return dst


def device_error():
    """Read and clear the device error word (non-zero after a timed-out wait)."""
    c = ctypes.c_int(0)
    check(_lib.load().nd_device_error(ctypes.byref(c)))
    return c.value


def embed(ids, wte, wpe=None, pos=None, out=None, stream=None):
    """y[t] = wte[ids[t]] + wpe[pos[t]] (bf16 [T][d]); ids/pos int32 [T]."""
    _need(ids, "ids", torch.int32, 1)
    _need(wte, "wte", torch.bfloat16, 2)
    T = ids.numel()
    vocab, d = wte.shape
    n_pos = 0
    if pos is not None:
        _need(pos, "pos", torch.int32, 1)
        _need(wpe, "wpe", torch.bfloat16, 2)
        n_pos = wpe.shape[0]
    if out is None:
        out = torch.empty((T, d), dtype=torch.bfloat16, device=wte.device)
    _need(out, "out", torch.bfloat16, 2)
    check(_lib.load().nd_embed(_stream(stream), _ptr(ids), _ptr(pos), _ptr(wte), _ptr(wpe),
                               _ptr(out), T, d, vocab, n_pos))
    return out


def argmax(logits, idx=None, val=None, stream=None):
    """First index of the largest value of each row of logits [rows][V]."""
    _need(logits, "logits", None, 2, contiguous=False)
    if logits.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    rows, V = logits.shape
    if idx is None:
        idx = torch.empty(rows, dtype=torch.int32, device=logits.device)
    check(_lib.load().nd_argmax(_stream(stream), _ptr(logits), _DT[logits.dtype],
                                logits.stride(0), rows, V, _ptr(idx), _ptr(val)))
    return idx


def kv_store(src, k_col, v_col, k_cache, v_cache, B, S, pos0=0, stream=None):
    """K/V rows of a [B·S][ld] bf16 projection into [B][H][L_max][64] caches."""
    _need(src, "src", torch.bfloat16, 2, contiguous=False)
    if src.stride(1) != 1:
        raise ValueError("src rows must be contiguous")
    _need(k_cache, "k_cache", torch.bfloat16, 4)
    _need(v_cache, "v_cache", torch.bfloat16, 4)
    _, H, L_max, D = k_cache.shape
    check(_lib.load().nd_kv_store(_stream(stream), _ptr(src), src.stride(0), k_col, v_col,
                                  _ptr(k_cache), _ptr(v_cache), B, S, H, L_max, pos0, D))


def add_layernorm(x, p, bias=None, gamma=None, beta=None, eps=1e-5, s_out=None, out=None,
                  stream=None):
    """s = x + p (+ bias) (bf16, s_out may be x), y = LayerNorm(s); returns (s, y)."""
    _need(x, "x", torch.bfloat16, 2)
    _need(p, "p", None, 2)
    rows, d = x.shape
    if s_out is None:
        s_out = torch.empty_like(x)
    if out is None:
        out = torch.empty_like(x)
    check(_lib.load().nd_add_layernorm(_stream(stream), _ptr(x), _ptr(p), _DT[p.dtype],
                                       _ptr(bias), _ptr(gamma), _ptr(beta), _ptr(s_out),
                                       _ptr(out), rows, d, float(eps)))
    return s_out, out


# ---- tensor-parallel reduction over NVLink peer memory ----------------------
def comm_region_bytes(rows_max, d):
    n = ctypes.c_size_t(0)
    check(_lib.load().nd_comm_region_bytes(rows_max, d, ctypes.byref(n)))
    return n.value


def comm_slot_offset(slot, rows_max, d):
    n = ctypes.c_size_t(0)
    check(_lib.load().nd_comm_slot_offset(slot, rows_max, d, ctypes.byref(n)))
    return n.value


def comm_alloc(nbytes):
    """A zero-filled region on the current device; returns (pointer, 64-byte IPC handle)."""
    p = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    check(_lib.load().nd_comm_alloc(nbytes, ctypes.byref(p), h))
    return p.value, h.raw


def comm_open(handle):
    p = ctypes.c_void_p()
    check(_lib.load().nd_comm_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(p)))
    return p.value


def comm_close(ptr):
    check(_lib.load().nd_comm_close(ctypes.c_void_p(ptr)))


def comm_free(ptr):
    check(_lib.load().nd_comm_free(ctypes.c_void_p(ptr)))


def allreduce_add_layernorm(regions, rank, region_bytes, rows_max, slot, x, bias, gamma, beta,
                            s_out, out, eps=1e-5, stream=None):
    """s_out = x + Σ_r (rank r's partial in `slot`) + bias, out = LayerNorm(s_out)."""
    _need(x, "x", torch.bfloat16, 2)
    rows, d = x.shape
    arr = (ctypes.c_void_p * len(regions))(*regions)
    check(_lib.load().nd_allreduce_add_layernorm(
        _stream(stream), arr, len(regions), rank, region_bytes, rows_max, slot, _ptr(x),
        _ptr(bias), _ptr(gamma), _ptr(beta), _ptr(s_out), _ptr(out), rows, d, float(eps)))
    return s_out, out


def gemm_allreduce_add_layernorm(a, w, regions, rank, region_bytes, rows_max, slot, x, bias, gamma,
                                 beta, s_out, out, eps=1e-5, stream=None):
    """s_out = x + Σ_r bf16(a_r · w_rᵀ) + bias, out = LayerNorm(s_out): this rank's projection
    tile and the cross-rank reduction in one launch (a [rows, K], w [d, K], both bf16)."""
    _need(a, "a", torch.bfloat16, 2)
    _need(w, "w", torch.bfloat16, 2)
    _need(x, "x", torch.bfloat16, 2)
    rows, d = x.shape
    if a.shape[0] != rows or w.shape[0] != d or a.shape[1] != w.shape[1]:
        raise ValueError(f"gemm_allreduce_add_layernorm: a {tuple(a.shape)} w {tuple(w.shape)} "
                         f"x {tuple(x.shape)}")
    arr = (ctypes.c_void_p * len(regions))(*regions)
    check(_lib.load().nd_gemm_allreduce_add_layernorm(
        _stream(stream), _ptr(a), _ptr(w), a.shape[1], arr, len(regions), rank, region_bytes,
        rows_max, slot, _ptr(x), _ptr(bias), _ptr(gamma), _ptr(beta), _ptr(s_out), _ptr(out),
        rows, d, float(eps)))
    return s_out, out
