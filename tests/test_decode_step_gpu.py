"""GPU checks of the decode-step entry points added for few-row decoding:

* nd_kv_decode_attn_qkv (decode attention read straight from a fused QKV
  projection row, padded or not) gives bit-for-bit the outputs and cache
  writes of nd_kv_decode_attn on the same q / k_new / v_new, and matches the
  oracle within the decode tolerance (max-abs 2e-2, rel-L2 1e-2);
* nd_argmax over a cluster of CTAs per row keeps the first maximum when equal
  maxima sit in different CTAs' ranges;
* programmatic dependent launch (nd_set_pdl) changes no result: a chain of
  decode-step ops, eager and captured in a CUDA graph, and a model's greedy
  decode give identical bits with it on and off.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu


def _ops():
    from neurodsl_b200 import ops
    return ops


def _t(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dtype)


@pytest.mark.parametrize("pad", [0, 24])
@pytest.mark.parametrize("L", [1, 130, 513])
def test_qkv_entry_matches_separate_inputs(L, pad):
    ops = _ops()
    rng = np.random.default_rng(L + pad)
    B, H, D, L_max = 5, 6, 64, 520
    qkv = oracle.bf16_round(rng.standard_normal((B, 3 * H * D + pad), dtype=np.float32))
    kc = oracle.bf16_round(rng.standard_normal((B, H, L_max, D), dtype=np.float32))
    vc = oracle.bf16_round(rng.standard_normal((B, H, L_max, D), dtype=np.float32))
    q = qkv[:, :H * D].reshape(B, H, D)
    kn = qkv[:, H * D:2 * H * D].reshape(B, H, D)
    vn = qkv[:, 2 * H * D:3 * H * D].reshape(B, H, D)

    k1, v1 = _t(kc), _t(vc)
    ref_out, _ = ops.kv_decode_attn(_t(q), k1, v1, L, k_new=_t(kn), v_new=_t(vn), want_lse=False)
    k2, v2 = _t(kc), _t(vc)
    qkv_t = _t(qkv)[:, :3 * H * D]
    if pad:
        assert qkv_t.stride(0) == 3 * H * D + pad
    out, _ = ops.kv_decode_attn_qkv(qkv_t, k2, v2, L)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    assert torch.equal(k2, k1) and torch.equal(v2, v1)

    kc2, vc2 = kc.copy(), vc.copy()
    kc2[:, :, L - 1] = kn
    vc2[:, :, L - 1] = vn
    ref, _ = oracle.kv_decode(q, kc2, vc2, L)
    o = out.float().cpu().numpy()
    assert float(np.abs(o - ref).max()) <= 2e-2
    assert float(np.linalg.norm(o - ref) / np.linalg.norm(ref)) <= 1e-2
    np.testing.assert_array_equal(k2[:, :, L - 1].float().cpu().numpy(), kn)


def test_qkv_entry_rejects_bad_stride():
    ops = _ops()
    from neurodsl_b200._lib import load
    B, H, D, L_max = 2, 2, 64, 16
    kc = torch.zeros(B, H, L_max, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    out = torch.empty(B, H, D, device="cuda", dtype=torch.bfloat16)
    qkv = torch.zeros(B, 3 * H * D + 8, device="cuda", dtype=torch.bfloat16)
    lib = load()
    for ld in (3 * H * D - 8, 3 * H * D + 4):   # too short; not a multiple of 8
        rc = lib.nd_kv_decode_attn_qkv(None, qkv.data_ptr(), ld, kc.data_ptr(), vc.data_ptr(),
                                       out.data_ptr(), 1, None, B, H, 4, L_max, D, 0.125, None, 0)
        assert rc != 0
    with pytest.raises(ValueError):             # column count is not 3*H*D
        ops.kv_decode_attn_qkv(qkv, kc, vc, 4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_argmax_ties_across_cluster_ranks(dtype):
    ops = _ops()
    rng = np.random.default_rng(9)
    rows, V = 6, 50257
    per = (V + 7) // 8                      # columns per CTA of an 8-CTA cluster
    x = rng.standard_normal((rows, V), dtype=np.float32)
    x[0, per - 1] = x[0, per] = 40.0        # tie across ranks 0 and 1
    x[1, 5 * per + 3] = x[1, 7 * per + 1] = 40.0
    x[2, V - 1] = 40.0                      # last column, last rank
    x[3, :per] = np.nan                     # a rank that sees only NaN
    x[3, 6 * per] = 40.0
    x[4, :] = 7.0                           # all equal: index 0
    t = torch.from_numpy(x).cuda().to(dtype)
    idx = ops.argmax(t).cpu().numpy()
    xr = t.float().cpu().numpy()
    ref = np.array([np.nanargmax(r) for r in xr])
    np.testing.assert_array_equal(idx, ref)
    assert list(idx[:5]) == [per - 1, 5 * per + 3, V - 1, 6 * per, 0]


def _step_chain(ops, w, B, H, L, bufs):
    """One decoder layer's decode launches plus the head: embed, LayerNorm,
    fused QKV, attention, out-projection, residual + LayerNorm, MLP, residual
    + LayerNorm, LM head, argmax."""
    xd, hd, qkv, ad, pd, ud, logits, ids, pos, ws = bufs
    ops.embed(ids, w["wte"], w["wpe"], pos, out=xd)
    ops.layernorm(xd, w["g"], w["b"], out=hd, stats=False)
    ops.linear(hd, w["w_qkv"], w["b_qkv"], out=qkv)
    ops.kv_decode_attn_qkv(qkv, w["kc"], w["vc"], L, out=ad.view(B, H, 64), workspace=ws)
    ops.linear(ad, w["w_o"], out=pd)
    ops.add_layernorm(xd, pd, w["b_o"], w["g"], w["b"], s_out=xd, out=hd)
    ops.linear(hd, w["w_1"], w["b_1"], act="tanh", out=ud)
    ops.linear(ud, w["w_2"], out=pd)
    ops.add_layernorm(xd, pd, w["b_2"], w["g"], w["b"], s_out=xd, out=hd)
    ops.linear(hd, w["wte"], out=logits)
    ops.argmax(logits, idx=ids)


def _chain_setup(seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    B, H, d, F, V, L_max = 16, 12, 768, 3072, 50257, 600
    bf = torch.bfloat16

    def r(*shape, s=0.02, dtype=bf):
        return (s * torch.randn(*shape, device="cuda", generator=gen)).to(dtype)
    w = {"wte": r(V, d), "wpe": r(L_max, d), "g": 1 + r(d, dtype=torch.float32),
         "b": r(d, dtype=torch.float32), "w_qkv": r(3 * d, d), "b_qkv": r(3 * d, dtype=torch.float32),
         "w_o": r(d, d), "b_o": r(d, dtype=torch.float32), "w_1": r(F, d),
         "b_1": r(F, dtype=torch.float32), "w_2": r(d, F), "b_2": r(d, dtype=torch.float32),
         "kc": r(B, H, L_max, 64, s=1.0), "vc": r(B, H, L_max, 64, s=1.0)}
    bufs = (torch.empty(B, d, device="cuda", dtype=bf), torch.empty(B, d, device="cuda", dtype=bf),
            torch.empty(B, 3 * d, device="cuda", dtype=bf), torch.empty(B, d, device="cuda", dtype=bf),
            torch.empty(B, d, device="cuda", dtype=bf), torch.empty(B, F, device="cuda", dtype=bf),
            torch.empty(B, V, device="cuda", dtype=torch.float32),
            torch.randint(0, V, (B,), device="cuda", generator=gen, dtype=torch.int32),
            torch.full((B,), 512, device="cuda", dtype=torch.int32),
            torch.zeros(1 << 20, device="cuda", dtype=torch.uint8))
    return w, bufs, B, H


@pytest.mark.parametrize("graph", [False, True])
def test_pdl_changes_no_result(graph):
    ops = _ops()
    results = []
    for pdl in (False, True):
        w, bufs, B, H = _chain_setup(3)
        torch.cuda.synchronize()
        with ops.pdl(pdl):
            if graph:
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for L in range(513, 521):
                        _step_chain(ops, w, B, H, L, bufs)
                torch.cuda.current_stream().wait_stream(s)
                g.replay()
            else:
                for L in range(513, 521):
                    _step_chain(ops, w, B, H, L, bufs)
        torch.cuda.synchronize()
        results.append([b.clone() for b in bufs[:8]] + [w["kc"].clone(), w["vc"].clone()])
    assert ops.set_pdl(False) is False
    for a, b in zip(*results):
        assert torch.equal(a, b)
    assert ops.device_error() == 0


def test_pdl_decode_reads_the_cache_row_the_projection_just_wrote():
    """With programmatic dependent launch on, a QKV projection of 64 rows (the
    tensor-core path) whose epilogue writes cache row L-1 (nd_gemm_qkv_cache,
    one token per sequence) is followed by decode attention without
    k_new / v_new, which must read that row only after the projection has
    finished: outputs and caches identical with PDL on and off, and the
    output within the decode tolerance of the oracle."""
    ops = _ops()
    B, H, K, L0, L_max = 64, 12, 768, 1000, 1024
    gen = torch.Generator(device="cuda").manual_seed(17)
    A = torch.randn(B, K, device="cuda", generator=gen).bfloat16()
    W = (0.05 * torch.randn(3 * H * 64, K, device="cuda", generator=gen)).bfloat16()
    bias = torch.zeros(3 * H * 64, device="cuda")
    q = torch.randn(B, H, 64, device="cuda", generator=gen).bfloat16()
    kc0 = torch.randn(B, H, L_max, 64, device="cuda", generator=gen).bfloat16()
    vc0 = torch.randn(B, H, L_max, 64, device="cuda", generator=gen).bfloat16()
    runs = []
    for pdl in (False, True):
        kc, vc = kc0.clone(), vc0.clone()
        qkv = torch.empty(B, 3 * H * 64, device="cuda", dtype=torch.bfloat16)
        outs = []
        torch.cuda.synchronize()
        with ops.pdl(pdl):
            for L in range(L0, L0 + 8):
                ops.linear_qkv_cache(A, W, bias, qkv, kc, vc, B, 1, pos0=L - 1)
                o, _ = ops.kv_decode_attn(q, kc, vc, L)
                outs.append(o.clone())
        torch.cuda.synchronize()
        runs.append((outs, kc, vc))
    assert ops.set_pdl(False) is False
    for a, b in zip(runs[0][0], runs[1][0]):
        assert torch.equal(a, b)
    assert torch.equal(runs[0][1], runs[1][1]) and torch.equal(runs[0][2], runs[1][2])
    L = L0 + 7
    ref, _ = oracle.kv_decode(q.float().cpu().numpy(), runs[1][1].float().cpu().numpy(),
                              runs[1][2].float().cpu().numpy(), L)
    got = runs[1][0][-1].float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-2
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-2
    assert ops.device_error() == 0


def test_model_decode_same_with_and_without_pdl():
    from neurodsl_b200.model import GPT, GPTConfig
    cfg = GPTConfig(n_layer=3, d_model=256, n_head=4, d_ff=1024, vocab=3001, n_pos=256)
    ids = torch.randint(0, cfg.vocab, (4, 40), device="cuda", dtype=torch.int32,
                        generator=torch.Generator(device="cuda").manual_seed(5))
    out = []
    for pdl in (False, True):
        m = GPT(cfg, seed=1, pdl=pdl)
        toks = m.generate(ids, 12, graph_chunk=4).clone()
        out.append((toks, m.buf["logits"].clone(), [c.clone() for c in m.k_cache]))
    assert torch.equal(out[0][0], out[1][0])
    assert torch.equal(out[0][1], out[1][1])
    for a, b in zip(out[0][2], out[1][2]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("M,N,K", [(16, 2304, 768), (1, 96, 64), (17, 3000, 1024), (32, 40, 1024), (3, 8, 32),
                                   (5, 50257, 768)])
@pytest.mark.parametrize("with_p", [False, True])
def test_ln_linear_matches_unfused_ops(M, N, K, with_p):
    """nd_ln_gemm gives the bits of nd_add_layernorm (or nd_layernorm) followed
    by nd_gemm_bias_act on its output, and the oracle's LayerNorm + linear
    within the GEMM tolerance."""
    ops = _ops()
    gen = torch.Generator(device="cuda").manual_seed(M + N + K)
    bf = torch.bfloat16
    x = torch.randn(M, K, device="cuda", generator=gen).to(bf)
    p = torch.randn(M, K, device="cuda", generator=gen).to(bf) if with_p else None
    pb = 0.1 * torch.randn(K, device="cuda", generator=gen) if with_p else None
    g = 1 + 0.1 * torch.randn(K, device="cuda", generator=gen)
    be = 0.1 * torch.randn(K, device="cuda", generator=gen)
    W = (torch.randn(N, K, device="cuda", generator=gen) / K ** 0.5).to(bf)
    bias = 0.1 * torch.randn(N, device="cuda", generator=gen)
    for act, odt in (("none", torch.float32), ("tanh", bf)):
        s_out = torch.empty_like(x) if with_p else None
        y = ops.ln_linear(x, W, p=p, p_bias=pb, gamma=g, beta=be, eps=1e-5, s_out=s_out,
                          bias=bias, act=act, out_dtype=odt)
        if with_p:
            s_ref, h = torch.empty_like(x), torch.empty_like(x)
            ops.add_layernorm(x, p, pb, g, be, 1e-5, s_out=s_ref, out=h)
        else:
            h, _, _ = ops.layernorm(x, g, be, eps=1e-5, out=torch.empty_like(x), stats=False)
        y_ref = ops.linear(h, W, bias, act=act, out_dtype=odt)
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref)
        if with_p:
            assert torch.equal(s_out, s_ref)
        hn = h.float().cpu().numpy()
        xs = x.float().cpu().numpy() + (p.float().cpu().numpy() + pb.cpu().numpy() if with_p else 0)
        ln_ref, _, _ = oracle.layernorm(oracle.bf16_round(xs), g.cpu().numpy(), be.cpu().numpy(), 1e-5)
        assert float(np.abs(hn - ln_ref).max()) <= 3e-2
        ref = oracle.linear(hn, W.float().cpu().numpy(), bias.cpu().numpy(), act=act)
        yn = y.float().cpu().numpy()
        assert float(np.abs(yn - ref).max()) <= 2e-2
        assert float(np.linalg.norm(yn - ref) / np.linalg.norm(ref)) <= 1e-2


def test_ln_linear_rejects_bad_arguments():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    bf = torch.bfloat16
    x = torch.zeros(4, 80, device="cuda", dtype=bf)
    W = torch.zeros(8, 80, device="cuda", dtype=bf)
    with pytest.raises(NeuroDSLError):                  # K % 32 != 0
        ops.ln_linear(x, W)
    x = torch.zeros(33, 64, device="cuda", dtype=bf)
    W = torch.zeros(8, 64, device="cuda", dtype=bf)
    with pytest.raises(NeuroDSLError):                  # more than 32 rows
        ops.ln_linear(x, W)
    x = torch.zeros(4, 64, device="cuda", dtype=bf)
    with pytest.raises(NeuroDSLError):                  # s_out aliases x
        ops.ln_linear(x, W, p=torch.zeros_like(x), s_out=x)
    x = torch.zeros(4, 2048, device="cuda", dtype=bf)
    with pytest.raises(NeuroDSLError):                  # K beyond the staged-row limit
        ops.ln_linear(x, torch.zeros(8, 2048, device="cuda", dtype=bf))
    assert ops.device_error() == 0
