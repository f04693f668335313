"""GPU parity of the gated dual projection (cfk_gdp_fwd / cfk_gdp_bwd) against the CPU oracle.

Tolerances: out, dx (16-bit) rtol = atol = 2e-2; dwp, dwg, dbp, dbg (f32) 1e-4 of max|.| plus
1e-4 relative, against float64 on the same 16-bit inputs.
"""

import pytest
import torch

import oracle
from conftest import assert_close_bf16, assert_close_f32

pytestmark = pytest.mark.gpu


def _inputs(m, k, n, dtype, seed, zero_bias=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    wp = (torch.randn(k, n, generator=g) / k ** 0.5).to(dtype)
    wg = (torch.randn(k, n, generator=g) / k ** 0.5).to(dtype)
    bp = (0 * torch.randn(n, generator=g) if zero_bias else 0.5 * torch.randn(n, generator=g)).to(dtype)
    bg = (0 * torch.randn(n, generator=g) if zero_bias else 0.5 * torch.randn(n, generator=g)).to(dtype)
    mask = (torch.rand(m, generator=g) > 0.1).to(dtype)
    dout = torch.randn(m, n, generator=g).to(dtype)
    return [t.cuda() for t in (x, wp, bp, wg, bg, mask, dout)]


SHAPES = [(1000, 128, 256), (300, 64, 64), (257, 48, 200), (130, 128, 512), (77, 40, 24),
          (64, 16, 8)]


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gdp_fwd(cuda_device, m, k, n, dtype):
    from colabfold_legacy_kernels import torch_ops
    x, wp, bp, wg, bg, mask, _ = _inputs(m, k, n, dtype, seed=m + k + n)
    out = torch_ops.gdp_fwd(x, wp, bp, wg, bg, mask)
    torch.cuda.synchronize()
    ref = oracle.gdp_fwd(*(t.cpu() for t in (x, wp, bp, wg, bg, mask)))
    assert_close_bf16(out, ref, "out")


@pytest.mark.parametrize("m,k,n", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gdp_bwd(cuda_device, m, k, n, dtype):
    from colabfold_legacy_kernels import torch_ops
    x, wp, bp, wg, bg, mask, dout = _inputs(m, k, n, dtype, seed=7 * m + k + n)
    dx, dwp, dbp, dwg, dbg = torch_ops.gdp_bwd(x, wp, bp, wg, bg, mask, dout)
    torch.cuda.synchronize()
    r = oracle.gdp_bwd(*(t.cpu() for t in (x, wp, bp, wg, bg, mask, dout)))
    assert_close_bf16(dx, r[0], "dx")
    assert_close_f32(dwp, r[1], "dwp")
    assert_close_f32(dbp, r[2], "dbp")
    assert_close_f32(dwg, r[3], "dwg")
    assert_close_f32(dbg, r[4], "dbg")


def test_gdp_triangle_multiplication_shape(cuda_device):
    """Config C4 shape class: packed a|b projections, zero biases, all-ones mask."""
    from colabfold_legacy_kernels import torch_ops
    cfg = oracle.configs.LnGdpConfig("c4_small", 1 << 15, 128, 256, 3)
    t = oracle.configs.make_ln_gdp_inputs(cfg)
    args = [t[n].cuda() for n in ("x", "wp", "bp", "wg", "bg", "mask")]
    out = torch_ops.gdp_fwd(*args)
    dx, dwp, dbp, dwg, dbg = torch_ops.gdp_bwd(*args, t["dout"].cuda())
    torch.cuda.synchronize()
    cpu = [a.cpu() for a in args]
    assert_close_bf16(out, oracle.gdp_fwd(*cpu), "out")
    r = oracle.gdp_bwd(*cpu, t["dout"])
    assert_close_bf16(dx, r[0], "dx")
    for a, b, name in ((dwp, r[1], "dwp"), (dbp, r[2], "dbp"), (dwg, r[3], "dwg"),
                       (dbg, r[4], "dbg")):
        assert_close_f32(a, b, name)


LN_GDP_SHAPES = [(1000, 128, 256), (300, 64, 64), (257, 48, 200), (130, 128, 512), (77, 40, 24),
                 (64, 16, 8)]


@pytest.mark.parametrize("m,k,n", LN_GDP_SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ln_gdp_fwd(cuda_device, m, k, n, dtype):
    """cfk_ln_gdp_fwd = gdp_fwd(LayerNorm(z)): fused kernel for the tcgen05 shapes, LayerNorm
    staged in the workspace for the others (K = 40, N = 512 here)."""
    from colabfold_legacy_kernels import torch_ops
    g = torch.Generator().manual_seed(3 * m + k + n)
    z = (2.0 * torch.randn(m, k, generator=g) + 0.5).to(dtype)
    gamma = 1.0 + 0.1 * torch.randn(k, generator=g)
    beta = 0.1 * torch.randn(k, generator=g)
    _, wp, bp, wg, bg, mask, _ = _inputs(m, k, n, dtype, seed=m + 2 * k + n)
    out, mean, rstd = torch_ops.ln_gdp_fwd(z.cuda(), gamma.cuda(), beta.cuda(), 1e-5, wp, bp, wg,
                                           bg, mask, return_stats=True)
    torch.cuda.synchronize()
    x, rmean, rrstd = oracle.layer_norm_fwd(z, gamma, beta, 1e-5)
    ref = oracle.gdp_fwd(x.to(dtype), *(t.cpu() for t in (wp, bp, wg, bg, mask)))
    assert_close_bf16(out, ref, "out")
    assert_close_f32(mean, rmean, "mean")
    assert_close_f32(rstd, rrstd, "rstd")
    # the same result as the two separate kernels, up to the 16-bit rounding of x
    y = torch_ops.layer_norm_fwd(z.cuda(), gamma.cuda(), beta.cuda(), 1e-5)
    two = torch_ops.gdp_fwd(y, wp, bp, wg, bg, mask)
    torch.cuda.synchronize()
    assert_close_bf16(out, two, "out vs LayerNorm then GDP", rtol=1e-2, atol=1e-2)
