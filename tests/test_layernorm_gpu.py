"""GPU parity of nd_layernorm against the oracle (fp32 statistics; 1e-4
relative tolerance for fp32 in/out), through the C ABI."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402

pytestmark = pytest.mark.gpu


def _ops():
    from neurodsl_b200 import ops
    return ops


def test_golden_fixture(golden):
    g = golden("layernorm")
    ops = _ops()
    for d in (1024, 100):
        x = torch.from_numpy(g[f"x{d}"]).cuda()
        y, mu, rs = ops.layernorm(x, torch.from_numpy(g[f"gamma{d}"]).cuda(),
                                  torch.from_numpy(g[f"beta{d}"]).cuda(), eps=1e-5)
        torch.cuda.synchronize()
        np.testing.assert_allclose(y.cpu().numpy(), g[f"y{d}"], rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(mu.cpu().numpy(), g[f"mean{d}"], rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(rs.cpu().numpy(), g[f"rstd{d}"], rtol=1e-4)


@pytest.mark.parametrize("rows,d", [(1, 8), (128, 1024), (37, 768), (5, 4096), (3, 100),
                                    (1000, 1024), (2, 20000)])
def test_fp32_shapes(rows, d):
    ops = _ops()
    rng = np.random.default_rng(rows + d)
    x = (rng.standard_normal((rows, d)) * 2 + 0.3).astype(np.float32)
    g = rng.standard_normal(d).astype(np.float32)
    b = rng.standard_normal(d).astype(np.float32)
    y, mu, rs = ops.layernorm(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(),
                              torch.from_numpy(b).cuda(), eps=1e-5)
    torch.cuda.synchronize()
    y_ref, mu_ref, rs_ref = oracle.layernorm(x, g, b, eps=1e-5)
    np.testing.assert_allclose(y.cpu().numpy(), y_ref, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(rs.cpu().numpy(), rs_ref, rtol=1e-4)


def test_bf16_out_and_in():
    ops = _ops()
    rng = np.random.default_rng(9)
    x = oracle.bf16_round(rng.standard_normal((64, 1024)).astype(np.float32))
    xb = torch.from_numpy(x).cuda().bfloat16()
    y, _, _ = ops.layernorm(xb, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    y_ref, _, _ = oracle.layernorm(x)
    np.testing.assert_allclose(y.float().cpu().numpy(), y_ref, rtol=1e-2, atol=2e-2)
    y32, _, _ = ops.layernorm(xb, out_dtype=torch.float32)
    np.testing.assert_allclose(y32.cpu().numpy(), y_ref, rtol=1e-4, atol=1e-4)


def test_convert_2d_col_major():
    ops = _ops()
    rng = np.random.default_rng(2)
    rows, cols = 70, 45
    a = rng.standard_normal((rows, cols)).astype(np.float32)
    col_major = torch.from_numpy(np.asfortranarray(a).ravel(order="K")).cuda()
    out = ops.convert_2d(col_major, rows, cols, True, torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), a)
    outb = ops.convert_2d(col_major, rows, cols, True, torch.bfloat16)
    np.testing.assert_array_equal(outb.float().cpu().numpy(), oracle.bf16_round(a))
