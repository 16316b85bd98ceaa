"""GPU checks of the decoder's auxiliary ops through the C ABI: token +
position embedding, greedy argmax, prefill KV-cache fill and the residual add
fused with LayerNorm.  Integer and copy work is compared bit-exactly; the
LayerNorm output (bf16) within max-abs 2e-2 of the fp32 oracle.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu


def _ops():
    from neurodsl_b200 import ops
    return ops


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(torch.bfloat16)


def test_embed_tokens_and_positions_exact():
    ops = _ops()
    rng = np.random.default_rng(0)
    V, P, d, T = 1000, 64, 256, 77
    wte = oracle.bf16_round(rng.standard_normal((V, d), dtype=np.float32) * 0.02)
    wpe = oracle.bf16_round(rng.standard_normal((P, d), dtype=np.float32) * 0.02)
    ids = rng.integers(0, V, T).astype(np.int32)
    pos = (np.arange(T) % P).astype(np.int32)
    y = ops.embed(torch.from_numpy(ids).cuda(), _bf16(wte), _bf16(wpe), torch.from_numpy(pos).cuda())
    ref = oracle.bf16_round(wte[ids] + wpe[pos])
    np.testing.assert_array_equal(y.float().cpu().numpy(), ref)
    y2 = ops.embed(torch.from_numpy(ids).cuda(), _bf16(wte))
    np.testing.assert_array_equal(y2.float().cpu().numpy(), wte[ids])


def test_embed_out_of_range_id_sets_error_and_zero_row():
    ops = _ops()
    wte = torch.ones((10, 64), device="cuda", dtype=torch.bfloat16)
    ids = torch.tensor([3, 10, -1, 2], device="cuda", dtype=torch.int32)
    assert ops.device_error() == 0
    y = ops.embed(ids, wte)
    assert ops.device_error() == 16
    yn = y.float().cpu().numpy()
    assert (yn[0] == 1).all() and (yn[3] == 1).all()
    assert (yn[1] == 0).all() and (yn[2] == 0).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_argmax_first_maximum(dtype):
    ops = _ops()
    rng = np.random.default_rng(1)
    rows, V = 16, 50257
    x = rng.standard_normal((rows, V), dtype=np.float32)
    x[3, 100] = x[3, 200] = 50.0          # tie: the first index wins
    x[5, :] = -np.inf
    x[5, 7] = 0.0
    x[6, 0] = np.nan                      # NaN never wins over numbers
    t = torch.from_numpy(x).cuda().to(dtype)
    idx = ops.argmax(t).cpu().numpy()
    xr = t.float().cpu().numpy()
    ref = np.array([np.nanargmax(r) for r in xr])
    np.testing.assert_array_equal(idx, ref)
    assert idx[3] == 100 and idx[5] == 7
    # strided rows (a column window of a wider matrix)
    wide = torch.zeros((rows, V + 40), device="cuda", dtype=dtype)
    wide[:, 8:8 + V] = t
    idx2 = ops.argmax(wide[:, 8:8 + V]).cpu().numpy()
    np.testing.assert_array_equal(idx2, ref)


def test_kv_store_from_qkv_projection_exact():
    ops = _ops()
    rng = np.random.default_rng(2)
    B, S, H, L_max, pos0 = 2, 37, 3, 64, 5
    d = H * 64
    qkv = oracle.bf16_round(rng.standard_normal((B * S, 3 * d), dtype=np.float32))
    kc = torch.zeros((B, H, L_max, 64), device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ops.kv_store(_bf16(qkv), d, 2 * d, kc, vc, B, S, pos0)
    x = qkv.reshape(B, S, 3, H, 64)
    k_ref = np.zeros((B, H, L_max, 64), np.float32)
    v_ref = np.zeros_like(k_ref)
    k_ref[:, :, pos0:pos0 + S] = x[:, :, 1].transpose(0, 2, 1, 3)
    v_ref[:, :, pos0:pos0 + S] = x[:, :, 2].transpose(0, 2, 1, 3)
    np.testing.assert_array_equal(kc.float().cpu().numpy(), k_ref)
    np.testing.assert_array_equal(vc.float().cpu().numpy(), v_ref)


@pytest.mark.parametrize("d,p_f32", [(768, False), (1024, True), (2048, False), (200, True)])
def test_add_layernorm(d, p_f32):
    ops = _ops()
    rng = np.random.default_rng(3)
    rows = 300
    x = oracle.bf16_round(rng.standard_normal((rows, d), dtype=np.float32))
    p = rng.standard_normal((rows, d), dtype=np.float32)
    if not p_f32:
        p = oracle.bf16_round(p)
    bias = rng.standard_normal(d, dtype=np.float32) * 0.1
    g = 1 + 0.1 * rng.standard_normal(d, dtype=np.float32)
    b = 0.1 * rng.standard_normal(d, dtype=np.float32)
    xt = _bf16(x)
    pt = torch.from_numpy(p).cuda() if p_f32 else _bf16(p)
    cuda = lambda a: torch.from_numpy(a).cuda()
    s, y = ops.add_layernorm(xt, pt, cuda(bias), cuda(g), cuda(b), eps=1e-5, s_out=xt)
    s_ref = oracle.bf16_round(x + (p + bias))
    np.testing.assert_array_equal(s.float().cpu().numpy(), s_ref)   # in place: s is x
    y_ref, _, _ = oracle.layernorm(s_ref, g, b, 1e-5)
    err = np.abs(y.float().cpu().numpy() - y_ref).max()
    assert err <= 2e-2, err


def test_add_layernorm_rejects_bad_width():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    x = torch.zeros((4, 12), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(NeuroDSLError):
        ops.add_layernorm(x, x)


@pytest.mark.parametrize("B,S,H,K,pos0,bias_off", [(2, 100, 3, 192, 0, 0), (3, 77, 2, 128, 5, 0),
                                                    (2, 9, 3, 192, 0, 0), (2, 100, 3, 192, 0, 1)])
def test_qkv_projection_fills_the_caches(B, S, H, K, pos0, bias_off):
    """nd_gemm_qkv_cache gives the projection and cache rows of
    nd_gemm_bias_act followed by nd_kv_store, bit for bit: the tensor-core
    epilogue path (M > 32), the few-row path (M = 18) and an unaligned bias
    (which takes the two-launch form)."""
    ops = _ops()
    gen = torch.Generator(device="cuda").manual_seed(B * S + K)
    bf = torch.bfloat16
    M, N, L_max = B * S, 3 * H * 64, S + pos0 + 3
    A = torch.randn(M, K, device="cuda", generator=gen).to(bf)
    W = (0.05 * torch.randn(N, K, device="cuda", generator=gen)).to(bf)
    bias = torch.randn(N + bias_off, device="cuda", generator=gen)[bias_off:]
    kc0 = torch.randn(B, H, L_max, 64, device="cuda", generator=gen).to(bf)
    vc0 = torch.randn(B, H, L_max, 64, device="cuda", generator=gen).to(bf)
    y_ref = ops.linear(A, W, bias)
    kc_ref, vc_ref = kc0.clone(), vc0.clone()
    ops.kv_store(y_ref, H * 64, 2 * H * 64, kc_ref, vc_ref, B, S, pos0)
    y = torch.empty_like(y_ref)
    kc, vc = kc0.clone(), vc0.clone()
    ops.linear_qkv_cache(A, W, bias, y, kc, vc, B, S, pos0)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    assert torch.equal(kc, kc_ref) and torch.equal(vc, vc_ref)


@pytest.mark.parametrize("tp,Bl,rank,S,Hl,K", [(2, 2, 1, 40, 2, 128), (4, 1, 2, 50, 3, 192),
                                                (8, 3, 0, 17, 1, 64)])
def test_qkv_projection_into_the_owners_caches(tp, Bl, rank, S, Hl, K):
    """nd_gemm_qkv_cache_peers (the prompt-sharded prefill of a tensor-parallel
    model) on one GPU, the tp ranks' caches being separate local buffers: the
    projection is nd_gemm_bias_act's, and head h's keys/values land in cache
    h // Hl as head h % Hl of sequences rank·Bl .. — the full-head
    nd_gemm_qkv_cache rows, bit for bit; nothing else of any cache changes."""
    ops = _ops()
    gen = torch.Generator(device="cuda").manual_seed(tp * 100 + S)
    bf = torch.bfloat16
    H = tp * Hl
    B, M, N, L_max = tp * Bl, Bl * S, 3 * H * 64, S + 4
    A = torch.randn(M, K, device="cuda", generator=gen).to(bf)
    W = (0.05 * torch.randn(N, K, device="cuda", generator=gen)).to(bf)
    bias = torch.randn(N, device="cuda", generator=gen)
    # the full-head caches of this rank's prompts, as one GPU fills them
    kf = torch.zeros(Bl, H, L_max, 64, device="cuda", dtype=bf)
    vf = torch.zeros_like(kf)
    y_ref = torch.empty(M, N, device="cuda", dtype=bf)
    ops.linear_qkv_cache(A, W, bias, y_ref, kf, vf, Bl, S)
    kc0 = [torch.randn(B, Hl, L_max, 64, device="cuda", generator=gen).to(bf) for _ in range(tp)]
    vc0 = [torch.randn(B, Hl, L_max, 64, device="cuda", generator=gen).to(bf) for _ in range(tp)]
    kc, vc = [c.clone() for c in kc0], [c.clone() for c in vc0]
    y = torch.empty_like(y_ref)
    ops.linear_qkv_cache_peers(A, W, bias, y, [c.data_ptr() for c in kc], [c.data_ptr() for c in vc],
                               Hl, L_max, Bl, rank * Bl, S)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    b0 = rank * Bl
    for q in range(tp):
        for got, ref, base in ((kc[q], kf, kc0[q]), (vc[q], vf, vc0[q])):
            want = base.clone()
            want[b0:b0 + Bl, :, :S] = ref[:, q * Hl:(q + 1) * Hl, :S]
            assert torch.equal(got, want), q


def test_qkv_projection_into_the_owners_caches_rejects():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    bf = torch.bfloat16
    A = torch.zeros(16, 64, device="cuda", dtype=bf)     # 16 rows: the epilogue path needs > 32
    W = torch.zeros(3 * 2 * 64, 64, device="cuda", dtype=bf)
    bias = torch.zeros(3 * 2 * 64, device="cuda")
    y = torch.empty(16, 3 * 2 * 64, device="cuda", dtype=bf)
    c = [torch.zeros(2, 1, 20, 64, device="cuda", dtype=bf) for _ in range(2)]
    ptrs = [t.data_ptr() for t in c]
    with pytest.raises(NeuroDSLError):
        ops.linear_qkv_cache_peers(A, W, bias, y, ptrs, ptrs, 1, 20, 1, 0, 16)


def test_copy_2d_batched_matches_views():
    """nd_copy_2d_batched over strided 3-D views (the key/value packing of the
    prompt-sharded prefill: column blocks of a projection into per-rank
    chunks), element sizes 2 and 4, and a 2-byte-aligned case."""
    ops = _ops()
    gen = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(40, 3 * 256, device="cuda", generator=gen).bfloat16()
    src = qkv[:, 256:512].view(40, 4, 64).permute(1, 0, 2)       # [4][40][64], strides (64, 768, 1)
    dst = torch.zeros(4, 40, 2, 64, device="cuda", dtype=torch.bfloat16)[:, :, 1, :]
    ops.copy_2d_batched(src, dst)
    f = torch.randn(3, 17, 33, device="cuda", generator=gen)[:, :, 1:30]   # fp32, odd strides
    g = torch.zeros(3, 20, 40, device="cuda")[:, 2:19, 5:34]
    ops.copy_2d_batched(f, g)
    h = torch.randn(5, 7, 13, device="cuda", generator=gen).bfloat16()[:, :, 1:12]  # 2-byte aligned
    k = torch.zeros(5, 7, 11, device="cuda", dtype=torch.bfloat16)
    ops.copy_2d_batched(h, k)
    torch.cuda.synchronize()
    assert torch.equal(dst, src) and torch.equal(g, f) and torch.equal(k, h)
    from neurodsl_b200._lib import NeuroDSLError
    with pytest.raises(NeuroDSLError):        # more than 65535 views
        ops.copy_2d_batched(torch.zeros(70000, 1, 8, device="cuda"),
                            torch.zeros(70000, 1, 8, device="cuda"))


def test_sm_limit_leaves_results_unchanged():
    """nd_set_sm_limit caps the persistent GEMM and prefill-attention grids
    (the SMs left over run a collective beside them); the outputs keep their
    bits, and a negative cap is refused."""
    ops = _ops()
    gen = torch.Generator(device="cuda").manual_seed(12)
    A = torch.randn(4096, 1024, device="cuda", generator=gen).bfloat16()
    W = (0.03 * torch.randn(3072, 1024, device="cuda", generator=gen)).bfloat16()
    b = torch.randn(3072, device="cuda", generator=gen)
    q, k, v = (torch.randn(2, 4, 700, 64, device="cuda", generator=gen).bfloat16() for _ in range(3))
    y0 = ops.linear(A, W, b, act="tanh")
    o0 = ops.flash_attn_fwd(q, k, v, causal=True)[0].clone()
    for cap in (100, 37, 1):
        with ops.sm_limit(cap):
            y = ops.linear(A, W, b, act="tanh")
            o = ops.flash_attn_fwd(q, k, v, causal=True)[0]
        torch.cuda.synchronize()
        assert torch.equal(y, y0) and torch.equal(o, o0), cap
    assert ops.set_sm_limit(0) == 0
    from neurodsl_b200._lib import NeuroDSLError
    with pytest.raises(NeuroDSLError):
        ops.set_sm_limit(-1)
