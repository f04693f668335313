"""GPU parity of the plain projections (cfk_linear_fwd / cfk_linear_bwd_dx / cfk_linear_bwd_dw)
against float64 on the CPU, on the same 16-bit inputs.

The reference has no such entry points (its modules' projections are host-framework GEMMs);
these are the GEMMs of the attention modules on this build's own kernels.  Tolerances: y, dx
(16-bit) rtol = atol = 2e-2; dw, db (f32) 1e-4 of max|.| plus 1e-4 relative.
"""

import pytest
import torch

from conftest import assert_close_bf16, assert_close_f32

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, g, scale=1.0):
    return (scale * torch.randn(*shape, generator=g)).to(dtype)


# (M, K, N): tcgen05 shapes (K % 16 == 0, N up to 512 at K = 128, N = 8), ragged M, and
# CUDA-core shapes (K = 40; N = 1024 beyond the resident-weight budget)
FWD_SHAPES = [(1000, 128, 512), (300, 64, 136), (129, 128, 8), (257, 40, 24), (70, 128, 1024)]


@pytest.mark.parametrize("m,k,n", FWD_SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bias", [True, False])
def test_linear_fwd(cuda_device, m, k, n, dtype, bias):
    from colabfold_legacy_kernels import torch_ops
    g = torch.Generator().manual_seed(m + k + n + bias)
    x, w = _rand((m, k), dtype, g), _rand((k, n), dtype, g, k ** -0.5)
    b = _rand((n,), dtype, g, 0.5) if bias else None
    y = torch_ops.linear_fwd(x.cuda(), w.cuda(), b.cuda() if bias else None)
    ref = x.double() @ w.double() + (b.double() if bias else 0)
    assert_close_bf16(y, ref, "y")


def test_linear_fwd_split_and_strided(cuda_device):
    """Columns [0, 384) into a [M, 3, 128] buffer's view, [384, 512) into a column block of a
    wider buffer: the same values as one contiguous output."""
    from colabfold_legacy_kernels import torch_ops
    g = torch.Generator().manual_seed(7)
    m, k, n = 777, 128, 512
    x, w, b = _rand((m, k), torch.bfloat16, g), _rand((k, n), torch.bfloat16, g, 0.1), \
        _rand((n,), torch.bfloat16, g)
    x, w, b = x.cuda(), w.cuda(), b.cuda()
    whole = torch_ops.linear_fwd(x, w, b)
    y0 = torch.zeros(m, 384, dtype=torch.bfloat16, device="cuda")
    wide = torch.zeros(m, 200, dtype=torch.bfloat16, device="cuda")
    y1 = wide[:, 40:168]
    torch_ops.linear_fwd(x, w, b, out=(y0, y1))
    assert torch.equal(y0, whole[:, :384])
    assert torch.equal(y1, whole[:, 384:])
    assert not wide[:, :40].any() and not wide[:, 168:].any()


def _blocks(m, k, ns, dtype, seed, stride_pad=24):
    """Output-gradient blocks dy_s [M, n_s], the first a column block of a wider buffer (row
    stride n_0 + stride_pad), and weights w_s [K, n_s]."""
    g = torch.Generator().manual_seed(seed)
    dys, ws = [], []
    for i, n in enumerate(ns):
        if i == 0:
            buf = _rand((m, n + stride_pad), dtype, g).cuda()
            dys.append(buf[:, 8:8 + n])
        else:
            dys.append(_rand((m, n), dtype, g).cuda())
        ws.append(_rand((k, n), dtype, g, k ** -0.5).cuda())
    return dys, ws


DX_CASES = [(1000, 128, (384, 128, 16)), (333, 64, (64,)), (129, 128, (512, 128, 16, 64)),
            (100, 40, (24, 8))]


@pytest.mark.parametrize("m,k,ns", DX_CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_bwd_dx(cuda_device, m, k, ns, dtype):
    from colabfold_legacy_kernels import torch_ops
    dys, ws = _blocks(m, k, ns, dtype, seed=m + k + len(ns))
    dx = torch_ops.linear_bwd_dx(dys, ws)
    ref = sum(dy.cpu().double() @ w.cpu().double().t() for dy, w in zip(dys, ws))
    assert_close_bf16(dx, ref, "dx")


DW_CASES = [(1000, 128, (384, 128, 16), (False, True, False)), (5000, 64, (136,), (True,)),
            (129, 128, (512, 8), (True, True)), (100, 40, (24, 8), (True, False)),
            (3, 128, (128,), (True,))]


@pytest.mark.parametrize("m,k,ns,bias", DW_CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_bwd_dw(cuda_device, m, k, ns, bias, dtype):
    from colabfold_legacy_kernels import torch_ops
    dys, _ = _blocks(m, k, ns, dtype, seed=2 * m + k)
    g = torch.Generator().manual_seed(m)
    x = _rand((m, k), dtype, g).cuda()
    grads = torch_ops.linear_bwd_dw(x, dys, bias)
    again = torch_ops.linear_bwd_dw(x, dys, bias)
    xd = x.cpu().double()
    for (dw, db), (dw2, db2), dy, wb in zip(grads, again, dys, bias):
        assert_close_f32(dw, xd.t() @ dy.cpu().double(), "dw")
        assert torch.equal(dw, dw2), "dw is not reproducible"
        if wb:
            assert_close_f32(db, dy.cpu().double().sum(0), "db")
            assert torch.equal(db, db2)
        else:
            assert db is None


def test_linear_empty_rows(cuda_device):
    from colabfold_legacy_kernels import torch_ops
    k = 128
    x = torch.empty(0, k, dtype=torch.bfloat16, device="cuda")
    w = torch.randn(k, 256, device="cuda").to(torch.bfloat16)
    assert torch_ops.linear_fwd(x, w).shape == (0, 256)
    dy = torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")
    assert torch_ops.linear_bwd_dx([dy], [w]).shape == (0, k)
    (dw, db), = torch_ops.linear_bwd_dw(x, [dy], [True])
    assert not dw.any() and not db.any()


def test_linear_rejects_bad_arguments(cuda_device):
    from colabfold_legacy_kernels import cabi, torch_ops
    x = torch.randn(10, 64, device="cuda").to(torch.bfloat16)
    w = torch.randn(64, 12, device="cuda").to(torch.bfloat16)   # N % 8 != 0
    with pytest.raises(cabi.CfkError) as e:
        torch_ops.linear_fwd(x, w)
    assert e.value.code == cabi.CFK_ERR_INVALID_ARGUMENT
    w = torch.randn(64, 256, device="cuda").to(torch.bfloat16)
    y0 = torch.empty(10, 100, dtype=torch.bfloat16, device="cuda")  # split not at 128 columns
    y1 = torch.empty(10, 156, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(cabi.CfkError):
        torch_ops.linear_fwd(x, w, out=(y0, y1))
