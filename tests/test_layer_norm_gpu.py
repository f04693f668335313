"""GPU parity of LayerNorm forward/backward (cfk_ln_fwd / cfk_ln_bwd) against the CPU oracle.

Tolerances: y, dx (16-bit) rtol = atol = 2e-2; mean, rstd, dgamma, dbeta (f32) 1e-4 of the
tensor's max magnitude plus 1e-4 relative, against float64 on the same 16-bit inputs.
"""

import pytest
import torch

import oracle
from conftest import assert_close_bf16, assert_close_f32

pytestmark = pytest.mark.gpu


def _inputs(m, c, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, c, generator=g) * 2 + 0.5).to(dtype)
    gamma = 1 + 0.1 * torch.randn(c, generator=g)
    beta = 0.1 * torch.randn(c, generator=g)
    dy = torch.randn(m, c, generator=g).to(dtype)
    return [t.cuda() for t in (x, gamma, beta, dy)]


@pytest.mark.parametrize("c", [64, 128, 256, 384, 512, 768, 1024, 100, 1000, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ln_fwd_bwd(cuda_device, c, dtype):
    from colabfold_legacy_kernels import torch_ops
    m = 1037
    x, gamma, beta, dy = _inputs(m, c, dtype, seed=c)
    eps = 1e-5
    y, mean, rstd = torch_ops.layer_norm_fwd(x, gamma, beta, eps, return_stats=True)
    ry, rmean, rrstd = oracle.layer_norm_fwd(x.cpu(), gamma.cpu(), beta.cpu(), eps)
    assert_close_bf16(y, ry, "y")
    assert_close_f32(mean, rmean, "mean")
    assert_close_f32(rstd, rrstd, "rstd")
    rdx, rdg, rdb = oracle.layer_norm_bwd(x.cpu(), gamma.cpu(), dy.cpu(), eps)
    for stats in (True, False):
        dx, dg, db = torch_ops.layer_norm_bwd(x, gamma, dy, eps, mean=mean if stats else None,
                                              rstd=rstd if stats else None)
        torch.cuda.synchronize()
        assert_close_bf16(dx, rdx, "dx")
        assert_close_f32(dg, rdg, "dgamma")
        assert_close_f32(db, rdb, "dbeta")


def test_ln_large_rows(cuda_device):
    from colabfold_legacy_kernels import torch_ops
    m, c = 1 << 18, 128
    x, gamma, beta, dy = _inputs(m, c, torch.bfloat16, seed=3)
    y = torch_ops.layer_norm_fwd(x, gamma, beta, 1e-5)
    ry, _, _ = oracle.layer_norm_fwd(x.cpu(), gamma.cpu(), beta.cpu(), 1e-5)
    assert_close_bf16(y, ry, "y")
    dx, dg, db = torch_ops.layer_norm_bwd(x, gamma, dy, 1e-5)
    rdx, rdg, rdb = oracle.layer_norm_bwd(x.cpu(), gamma.cpu(), dy.cpu(), 1e-5)
    assert_close_bf16(dx, rdx, "dx")
    assert_close_f32(dg, rdg, "dgamma")
    assert_close_f32(db, rdb, "dbeta")


def test_ln_empty(cuda_device):
    from colabfold_legacy_kernels import torch_ops
    x = torch.empty(0, 128, dtype=torch.bfloat16, device="cuda")
    gamma = torch.ones(128, device="cuda")
    y = torch_ops.layer_norm_fwd(x, gamma, torch.zeros_like(gamma), 1e-5)
    assert y.shape == (0, 128)
    dx, dg, db = torch_ops.layer_norm_bwd(x, gamma, x, 1e-5)
    torch.cuda.synchronize()
    assert dg.abs().sum().item() == 0 and db.abs().sum().item() == 0
