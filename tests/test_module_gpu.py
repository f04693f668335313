"""The triangle-attention module on the GPU (colabfold_legacy_kernels.modules.TriangleAttention:
LayerNorm, attention through strided views, cuBLAS projections) against the float64 oracle of
config C1's module (oracle/module.py), forward and backward, around both nodes.

Tolerances: the output, elementwise atol = rtol = 2e-2 (bf16).  Gradients of z and of every
parameter are sums over all 16384 pair rows of products of bf16 values, so they are held to a
normwise bound: ||got - want|| <= 2e-2 ||want|| per tensor.
"""

import pytest
import torch

import oracle
from conftest import assert_close_bf16

pytestmark = pytest.mark.gpu

NAMES = ["gamma", "beta", "w_q", "w_k", "w_v", "w_b", "w_g", "b_g", "w_o", "b_o"]


def _case(seed=0, n=128, padded=True):
    p = oracle.module.make_params(128, 4, 32, seed=seed)
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(n, n, 128, generator=g)
    res = torch.ones(n)
    if padded:
        res[torch.rand(n, generator=g) < 0.05] = 0.0   # padded residues, as in C3
        res[-3:] = 0.0
    mask = res[:, None] * res[None, :]
    return z, mask, p


def _module(p):
    from colabfold_legacy_kernels.modules import TriangleAttention
    m = TriangleAttention(128, 4, 32, device="cuda")
    with torch.no_grad():
        for name, t in zip(NAMES, p.tensors()):
            getattr(m, name).copy_(t)
    return m


def _normwise(got, want, what, tol=2e-2):
    got, want = got.double().cpu(), want.double().cpu()
    err = float((got - want).norm())
    ref = float(want.norm())
    assert err <= tol * ref, "%s: ||err|| = %.4g > %g * ||want|| = %.4g" % (what, err, tol, ref)


@pytest.mark.parametrize("ending", [False, True])
def test_module_forward_backward_c1(cuda_device, ending):
    z, mask, p = _case(seed=0 if not ending else 1)
    m = _module(p)
    zg = z.cuda().requires_grad_(True)
    out = m(zg, mask.cuda(), ending=ending)
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(7))
    out.backward(dout.cuda().to(out.dtype))
    torch.cuda.synchronize()
    want = oracle.module.triangle_attention(z, mask, p, ending=ending)
    assert_close_bf16(out, want, "module out (ending=%s)" % ending)
    dz, grads = oracle.module.triangle_attention_bwd(z, mask, p, dout, ending=ending)
    _normwise(zg.grad, dz, "dz")
    for name in NAMES:
        _normwise(getattr(m, name).grad, grads[name], "d" + name)


def test_module_makes_no_transposed_copies(cuda_device):
    """q, k, v reach the kernels as views of the projection buffer: the module runs the strided
    entry points, and the attention output is a plain [Ni, Nj, H, D] tensor in both node types."""
    from colabfold_legacy_kernels import cabi
    z, mask, p = _case(seed=2, n=64, padded=False)
    m = _module(p)
    calls = []
    real = cabi.call

    def spy(name, *args):
        calls.append(name)
        return real(name, *args)

    cabi.call = spy
    try:
        for ending in (False, True):
            m(z.cuda(), mask.cuda(), ending=ending).float().sum().backward()
    finally:
        cabi.call = real
    torch.cuda.synchronize()
    assert calls.count("cfk_attn_fwd_strided") == 2 and calls.count("cfk_attn_bwd_strided") == 2
    assert "cfk_attn_fwd" not in calls and "cfk_attn_bwd" not in calls
