"""One-GPU checks of the NVLink tensor-parallel reduction
(nd_allreduce_add_layernorm) through the C ABI:

* with one rank the call is x + partial + bias followed by LayerNorm:
  compared with the oracle (s within one bf16 ulp: max-abs 2e-2 relative to
  |s| ≤ 4; y max-abs 2e-2);
* a peer that never arrives: two regions on this GPU, rank 1's flag is never
  set, so the bounded wait runs out (2 s) and the call leaves the device error
  word at 5 (kDevErrTimeoutComm) instead of hanging;
* bad arguments are refused before any launch.
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
