"""GPU parity of nd_gemm_bias_act (the :linear / fused_linear_gelu rules)
against the oracle and a torch fp32 reference, through the C ABI."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _ops():
    from neurodsl_b200 import ops
    return ops


def _t(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dtype)


def check(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    err = float(np.abs(y - ref).max())
    rel = float(np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30))
    assert err <= MAX_ABS and rel <= REL_L2, (err, rel)


def test_golden_fixture(golden):
    g = golden("linear_gelu")
    ops = _ops()
    A, W, b = _t(g["A"]), _t(g["W"]), _t(g["bias"], torch.float32)
    for act in ("sigmoid", "tanh", "erf"):
        y = ops.linear(A, W, b, act=act, out_dtype=torch.float32)
        torch.cuda.synchronize()
        check(y.cpu().numpy(), g["Y_" + act])
    y = ops.linear(A, W, b, residual=_t(g["residual"], torch.float32), out_dtype=torch.float32)
    check(y.cpu().numpy(), g["Y_residual"])


@pytest.mark.parametrize("M,N,K", [(128, 4096, 1024), (128, 1024, 4096), (200, 300, 136),
                                   (1, 64, 64), (513, 768, 768), (4096, 4096, 1024)])
@pytest.mark.parametrize("act", ["none", "sigmoid"])
def test_shapes_vs_torch(M, N, K, act):
    ops = _ops()
    gen = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=gen).bfloat16()
    W = (0.02 * torch.randn(N, K, device="cuda", generator=gen)).bfloat16()
    b = torch.randn(N, device="cuda", generator=gen) * 0.1
    y = ops.linear(A, W, b, act=act, out_dtype=torch.float32)
    z = A.float() @ W.float().T + b
    if act == "sigmoid":
        z = z * torch.sigmoid(1.702 * z)
    torch.cuda.synchronize()
    check(y.cpu().numpy(), z.cpu().numpy())


@pytest.mark.parametrize("M,N,K", [(1, 768, 768), (7, 300, 96), (16, 2304, 768),
                                   (17, 50257, 768), (32, 1024, 4096), (30, 8, 32),
                                   (16, 768, 3072), (3, 40, 1056), (9, 96, 16384)])
@pytest.mark.parametrize("act,res", [("none", False), ("tanh", True), ("sigmoid", False)])
def test_few_rows_vs_oracle(M, N, K, act, res):
    """M <= 32 takes the weight-streaming path; compared with the oracle on
    bf16-rounded inputs, bf16 and fp32 outputs, with and without residual.
    The shapes cover K split over clusters of 1, 2, 3, 4 and 8 CTAs (K/32
    chunks of 32 per CTA batch, uneven last share at K = 1056) and warps that
    loop over more than one batch (K = 16384)."""
    ops = _ops()
    rng = np.random.default_rng(M * 7 + N + K)
    A = oracle.bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    # outputs of order one at every K, so the absolute tolerance stays above
    # half a bf16 ulp of the output
    w_std = min(0.03, 2.0 / np.sqrt(K))
    W = oracle.bf16_round((w_std * rng.standard_normal((N, K))).astype(np.float32))
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    R = oracle.bf16_round(rng.standard_normal((M, N), dtype=np.float32)) if res else None
    ref = oracle.linear(A, W, b, residual=R, act=act)
    for out_dtype in (torch.float32, torch.bfloat16):
        y = ops.linear(_t(A), _t(W), _t(b, torch.float32), residual=None if R is None else _t(R),
                       act=act, out_dtype=out_dtype)
        torch.cuda.synchronize()
        check(y.float().cpu().numpy(), ref)


def test_residual_bf16_and_bf16_out():
    ops = _ops()
    rng = np.random.default_rng(4)
    M, N, K = 130, 256, 192
    A = oracle.bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    W = oracle.bf16_round((0.05 * rng.standard_normal((N, K))).astype(np.float32))
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    R = oracle.bf16_round(rng.standard_normal((M, N), dtype=np.float32))
    y = ops.linear(_t(A), _t(W), _t(b, torch.float32), residual=_t(R), act="tanh")
    torch.cuda.synchronize()
    ref = oracle.linear(A, W, b, residual=R, act="tanh")
    check(y.float().cpu().numpy(), ref)


def test_rejects_bad_arguments():
    ops = _ops()
    from neurodsl_b200._lib import NeuroDSLError
    A = torch.zeros(4, 12, device="cuda", dtype=torch.bfloat16)  # K % 8 != 0
    W = torch.zeros(8, 12, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(NeuroDSLError):
        ops.linear(A, W)
