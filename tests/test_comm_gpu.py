"""One-GPU checks of the NVLink tensor-parallel reduction
(nd_allreduce_add_layernorm) through the C ABI:

* with one rank the call is x + partial + bias followed by LayerNorm:
  compared with the oracle (s within one bf16 ulp: max-abs 2e-2 relative to
  |s| ≤ 4; y max-abs 2e-2);
* a peer that never arrives: two regions on this GPU, rank 1's flag is never
  set, so the bounded wait runs out (2 s) and the call leaves the device error
  word at 5 (kDevErrTimeoutComm) instead of hanging;
* bad arguments are refused before any launch;
* the projection fused with the reduction (nd_gemm_allreduce_add_layernorm)
  with one rank gives the same bits as the projection into the own slot
  (nd_gemm_bias_act) followed by nd_allreduce_add_layernorm, for row counts on
  both sides of 16, K from 32 to 4096 and d from 64 to 1024, with fused and
  separate calls interleaved over the two slots (their sequence numbers come
  from disjoint ranges), and matches the oracle; with a peer that never
  arrives it times out with the error code, and it refuses unsupported shapes.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu


def _ops():
    from neurodsl_b200 import ops
    return ops


def _slot(ops, region, k, rows_max, d):
    from neurodsl_b200.comm import _DeviceArray
    ptr = region + ops.comm_slot_offset(k, rows_max, d)
    return torch.as_tensor(_DeviceArray(ptr, (rows_max, d), "<i2"), device="cuda").view(
        torch.bfloat16)


def test_single_rank_matches_oracle():
    ops = _ops()
    rows_max, d, rows = 32, 768, 20
    nbytes = ops.comm_region_bytes(rows_max, d)
    region, _ = ops.comm_alloc(nbytes)
    try:
        rng = np.random.default_rng(0)
        x = oracle.bf16_round(rng.standard_normal((rows, d), dtype=np.float32))
        p = oracle.bf16_round(rng.standard_normal((rows, d), dtype=np.float32))
        bias = (0.1 * rng.standard_normal(d)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        b = (0.1 * rng.standard_normal(d)).astype(np.float32)
        cuda = lambda a: torch.from_numpy(a).cuda()
        for k in (0, 1, 0):
            _slot(ops, region, k, rows_max, d)[:rows].copy_(cuda(p).to(torch.bfloat16))
            xt = cuda(x).to(torch.bfloat16)
            s = torch.empty_like(xt)
            y = torch.empty_like(xt)
            ops.allreduce_add_layernorm([region], 0, nbytes, rows_max, k, xt, cuda(bias), cuda(g),
                                        cuda(b), s, y, eps=1e-5)
            torch.cuda.synchronize()
            s_ref = x + p + bias
            assert float(np.abs(s.float().cpu().numpy() - s_ref).max()) <= 2e-2
            y_ref, _, _ = oracle.layernorm(oracle.bf16_round(s_ref), g, b, 1e-5)
            assert float(np.abs(y.float().cpu().numpy() - y_ref).max()) <= 2e-2
        assert ops.device_error() == 0
    finally:
        ops.comm_free(region)


def test_missing_peer_times_out_with_error_code():
    ops = _ops()
    rows_max, d = 8, 256
    nbytes = ops.comm_region_bytes(rows_max, d)
    r0, _ = ops.comm_alloc(nbytes)
    r1, _ = ops.comm_alloc(nbytes)      # stands for a peer that never arrives
    try:
        x = torch.zeros((4, d), device="cuda", dtype=torch.bfloat16)
        s, y = torch.empty_like(x), torch.empty_like(x)
        assert ops.device_error() == 0
        ops.allreduce_add_layernorm([r0, r1], 0, nbytes, rows_max, 0, x, None, None, None, s, y)
        assert ops.device_error() == 5
    finally:
        ops.comm_free(r0)
        ops.comm_free(r1)


def test_rejects_bad_arguments():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    rows_max, d = 8, 256
    nbytes = ops.comm_region_bytes(rows_max, d)
    region, _ = ops.comm_alloc(nbytes)
    try:
        x = torch.zeros((4, d), device="cuda", dtype=torch.bfloat16)
        s, y = torch.empty_like(x), torch.empty_like(x)
        with pytest.raises(NeuroDSLError):       # slot must be 0 or 1
            ops.allreduce_add_layernorm([region], 0, nbytes, rows_max, 2, x, None, None, None, s, y)
        big = torch.zeros((9, d), device="cuda", dtype=torch.bfloat16)
        with pytest.raises(NeuroDSLError):       # more rows than the slots hold
            ops.allreduce_add_layernorm([region], 0, nbytes, rows_max, 0, big, None, None, None,
                                        torch.empty_like(big), torch.empty_like(big))
        with pytest.raises(NeuroDSLError):       # region too small for the shape
            ops.allreduce_add_layernorm([region], 0, nbytes // 2, rows_max, 0, x, None, None, None,
                                        s, y)
        with pytest.raises(NeuroDSLError):       # rank outside [0, tp)
            ops.allreduce_add_layernorm([region], 1, nbytes, rows_max, 0, x, None, None, None, s, y)
        assert ops.device_error() == 0
    finally:
        ops.comm_free(region)


def _fused_case(ops, rng, rows, d, K):
    cuda = lambda a: torch.from_numpy(a).cuda()
    a = oracle.bf16_round((0.5 * rng.standard_normal((rows, K))).astype(np.float32))
    w = oracle.bf16_round((rng.standard_normal((d, K)) / np.sqrt(K)).astype(np.float32))
    x = oracle.bf16_round(rng.standard_normal((rows, d), dtype=np.float32))
    bias = (0.1 * rng.standard_normal(d)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    b = (0.1 * rng.standard_normal(d)).astype(np.float32)
    t = {"a": cuda(a).to(torch.bfloat16), "w": cuda(w).to(torch.bfloat16),
         "x": cuda(x).to(torch.bfloat16), "bias": cuda(bias), "g": cuda(g), "b": cuda(b)}
    return (a, w, x, bias, g, b), t


@pytest.mark.parametrize("rows,d,K", [(1, 768, 384), (8, 768, 1536), (16, 1024, 4096),
                                      (17, 1024, 1024), (32, 256, 32), (5, 64, 96)])
def test_fused_projection_single_rank_bit_identical(rows, d, K):
    ops = _ops()
    rows_max = 32
    nbytes = ops.comm_region_bytes(rows_max, d)
    region, _ = ops.comm_alloc(nbytes)
    try:
        rng = np.random.default_rng(rows * 1000 + K)
        (a, w, x, bias, g, b), t = _fused_case(ops, rng, rows, d, K)
        # fused and separate calls interleaved: slots 0, 1, 0, 1
        outs = []
        for k, fused in ((0, True), (1, False), (0, False), (1, True)):
            s = torch.empty_like(t["x"])
            y = torch.empty_like(t["x"])
            if fused:
                ops.gemm_allreduce_add_layernorm(t["a"], t["w"], [region], 0, nbytes, rows_max, k,
                                                 t["x"], t["bias"], t["g"], t["b"], s, y)
            else:
                ops.linear(t["a"], t["w"], out=_slot(ops, region, k, rows_max, d)[:rows])
                ops.allreduce_add_layernorm([region], 0, nbytes, rows_max, k, t["x"], t["bias"],
                                            t["g"], t["b"], s, y)
            outs.append((s, y))
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        for s, y in outs[1:]:
            assert torch.equal(s, outs[0][0]) and torch.equal(y, outs[0][1])
        # against the oracle: the bf16 partial, then the residual + LayerNorm
        p = oracle.bf16_round(a.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
        s_ref = x + p + bias
        s_got = outs[0][0].float().cpu().numpy()
        # one bf16 ulp at the top binade of s: a flipped rounding of the
        # partial (fp32 vs exact accumulation) plus the rounding of s
        tol_s = 2.0 ** (np.ceil(np.log2(float(np.abs(s_ref).max()))) - 7)
        assert float(np.abs(s_got - s_ref).max()) <= tol_s
        y_ref, _, _ = oracle.layernorm(s_got, g, b, 1e-5)
        assert float(np.abs(outs[0][1].float().cpu().numpy() - y_ref).max()) <= 3e-2
    finally:
        ops.comm_free(region)


def test_fused_projection_in_place_residual():
    """s_out may be x itself (the residual stream updated in place)."""
    ops = _ops()
    rows, d, K, rows_max = 8, 512, 256, 8
    nbytes = ops.comm_region_bytes(rows_max, d)
    region, _ = ops.comm_alloc(nbytes)
    try:
        _, t = _fused_case(ops, np.random.default_rng(7), rows, d, K)
        s_ref, y_ref = torch.empty_like(t["x"]), torch.empty_like(t["x"])
        ops.gemm_allreduce_add_layernorm(t["a"], t["w"], [region], 0, nbytes, rows_max, 0, t["x"],
                                         t["bias"], t["g"], t["b"], s_ref, y_ref)
        xi, yi = t["x"].clone(), torch.empty_like(t["x"])
        ops.gemm_allreduce_add_layernorm(t["a"], t["w"], [region], 0, nbytes, rows_max, 1, xi,
                                         t["bias"], t["g"], t["b"], xi, yi)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        assert torch.equal(xi, s_ref) and torch.equal(yi, y_ref)
    finally:
        ops.comm_free(region)


def test_fused_projection_missing_peer_times_out():
    ops = _ops()
    rows_max, d, K = 8, 256, 128
    nbytes = ops.comm_region_bytes(rows_max, d)
    r0, _ = ops.comm_alloc(nbytes)
    r1, _ = ops.comm_alloc(nbytes)      # stands for a peer that never arrives
    try:
        _, t = _fused_case(ops, np.random.default_rng(3), 4, d, K)
        s, y = torch.empty_like(t["x"]), torch.empty_like(t["x"])
        assert ops.device_error() == 0
        ops.gemm_allreduce_add_layernorm(t["a"], t["w"], [r0, r1], 0, nbytes, rows_max, 0, t["x"],
                                         None, None, None, s, y)
        assert ops.device_error() == 5
    finally:
        ops.comm_free(r0)
        ops.comm_free(r1)


def test_fused_projection_rejects_unsupported_shapes():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    rows_max, d = 8, 256
    nbytes = ops.comm_region_bytes(rows_max, d)
    region, _ = ops.comm_alloc(nbytes)
    try:
        x = torch.zeros((4, d), device="cuda", dtype=torch.bfloat16)
        s, y = torch.empty_like(x), torch.empty_like(x)
        w = torch.zeros((d, 48), device="cuda", dtype=torch.bfloat16)
        with pytest.raises(NeuroDSLError):       # K not a multiple of 32
            ops.gemm_allreduce_add_layernorm(torch.zeros((4, 48), device="cuda",
                                                         dtype=torch.bfloat16), w, [region], 0,
                                             nbytes, rows_max, 0, x, None, None, None, s, y)
        w = torch.zeros((d, 64), device="cuda", dtype=torch.bfloat16)
        a = torch.zeros((4, 64), device="cuda", dtype=torch.bfloat16)
        with pytest.raises(NeuroDSLError):       # tp 3 is not taken by the fused kernel
            ops.gemm_allreduce_add_layernorm(a, w, [region] * 3, 0, nbytes, rows_max, 0, x, None,
                                             None, None, s, y)
        with pytest.raises(NeuroDSLError):       # slot must be 0 or 1
            ops.gemm_allreduce_add_layernorm(a, w, [region], 0, nbytes, rows_max, 2, x, None, None,
                                             None, s, y)
        with pytest.raises(ValueError):          # a and w disagree on K
            ops.gemm_allreduce_add_layernorm(a, torch.zeros((d, 32), device="cuda",
                                                            dtype=torch.bfloat16), [region], 0,
                                             nbytes, rows_max, 0, x, None, None, None, s, y)
        assert ops.device_error() == 0
    finally:
        ops.comm_free(region)
