"""cfk_ln_bwd_noalloc: the LayerNorm backward for callers that cannot provide device memory.

An XLA FFI handler receives only the buffers its binding declares and may not allocate, and
some hosts plan every device allocation in advance; such callers cannot pass cfk_ln_bwd a
workspace.  cfk_ln_bwd_noalloc keeps its scratch in a static device array instead.  This test
calls it through the C ABI and compares it with cfk_ln_bwd (the entry point that takes a
workspace) on two calls in a row, so stale contents of the shared array would show up.

Tolerances as in the other tests: dx (16-bit) rtol = atol = 2e-2; dgamma, dbeta (f32) 1e-4 of
max|.| plus 1e-4 relative.
"""

import pytest
import torch

import oracle
from conftest import assert_close_bf16, assert_close_f32

pytestmark = pytest.mark.gpu


def _noalloc(x, gamma, dy, eps, mean=None, rstd=None):
    from colabfold_legacy_kernels import cabi
    m, c = x.shape
    dx = torch.empty_like(x)
    dgamma = torch.empty(c, dtype=torch.float32, device=x.device)
    dbeta = torch.empty(c, dtype=torch.float32, device=x.device)
    code = cabi.CFK_BF16 if x.dtype == torch.bfloat16 else cabi.CFK_F16
    ptr = lambda t: None if t is None else t.data_ptr()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    cabi.call("cfk_ln_bwd_noalloc", stream, code, ptr(x), ptr(gamma), ptr(mean), ptr(rstd),
              ptr(dy), ptr(dx), ptr(dgamma), ptr(dbeta), m, c, float(eps))
    return dx, dgamma, dbeta


# C = 1024 with 70k rows fills the static scratch exactly (320 partials x 2 x 1024 floats)
@pytest.mark.parametrize("c,dtype", [(128, torch.bfloat16), (1000, torch.float16),
                                     (1024, torch.bfloat16)])
def test_noalloc_matches_workspace_entry_point(cuda_device, c, dtype):
    from colabfold_legacy_kernels import torch_ops
    g = torch.Generator().manual_seed(c)
    eps = 1e-5
    for call in range(2):  # two calls in a row: the shared scratch must not leak between them
        m = 70000 + 1000 * call
        x = (torch.randn(m, c, generator=g) * 1.5 + 0.3).to(dtype).cuda()
        gamma = (1 + 0.1 * torch.randn(c, generator=g)).cuda()
        beta = (0.1 * torch.randn(c, generator=g)).cuda()
        dy = torch.randn(m, c, generator=g).to(dtype).cuda()
        _, mean, rstd = torch_ops.layer_norm_fwd(x, gamma, beta, eps, return_stats=True)
        stats = (mean, rstd) if call == 0 else (None, None)
        ref = torch_ops.layer_norm_bwd(x, gamma, dy, eps, mean=stats[0], rstd=stats[1])
        got = _noalloc(x, gamma, dy, eps, mean=stats[0], rstd=stats[1])
        torch.cuda.synchronize()
        assert_close_bf16(got[0], ref[0], "dx (call %d)" % call)
        assert_close_f32(got[1], ref[1], "dgamma (call %d)" % call)
        assert_close_f32(got[2], ref[2], "dbeta (call %d)" % call)
        if call == 0:
            # and against the CPU oracle (float64) on the same 16-bit inputs
            rdx, rdg, rdb = oracle.layer_norm_bwd(x.cpu(), gamma.cpu(), dy.cpu(), eps)
            assert_close_bf16(got[0], rdx, "dx vs oracle")
            assert_close_f32(got[1], rdg, "dgamma vs oracle")
            assert_close_f32(got[2], rdb, "dbeta vs oracle")


def test_noalloc_empty_rows_give_zero_parameter_gradients(cuda_device):
    """M = 0: no row kernel runs; dgamma and dbeta are written as zeros (after a call that left
    nonzero partials in the shared array)."""
    c = 256
    x = torch.randn(5000, c, device="cuda").to(torch.bfloat16)
    gamma = torch.ones(c, device="cuda")
    _noalloc(x, gamma, x, 1e-5)
    empty = torch.empty(0, c, dtype=torch.bfloat16, device="cuda")
    dx, dg, db = _noalloc(empty, gamma, empty, 1e-5)
    torch.cuda.synchronize()
    assert dx.shape == (0, c)
    assert dg.abs().sum().item() == 0 and db.abs().sum().item() == 0


def test_noalloc_rejects_rows_wider_than_its_scratch(cuda_device):
    from colabfold_legacy_kernels import cabi
    x = torch.zeros(4, 2048, dtype=torch.bfloat16, device="cuda")
    gamma = torch.ones(2048, device="cuda")
    with pytest.raises(cabi.CfkError) as e:
        _noalloc(x, gamma, x, 1e-5)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT and "1024" in e.value.message
