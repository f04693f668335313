"""The triangle-attention module on the GPU (colabfold_legacy_kernels.modules.TriangleAttention:
LayerNorm, attention through strided views, projections on the cfk_linear_* kernels) against
the float64 oracle of config C1's module (oracle/module.py), forward and backward, around both
nodes; and that a module step launches no library GEMM.

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


def test_module_step_launches_no_library_gemm(cuda_device):
    """Forward and backward of the triangle module (both nodes) run their projections on this
    build's kernels: the profiler's CUDA kernel list holds no cuBLAS / CUTLASS GEMM or GEMV,
    and the C ABI saw the projection entry points."""
    import re
    from colabfold_legacy_kernels import cabi
    z, mask, p = _case(seed=3, n=64, padded=True)
    m = _module(p)
    calls = []
    real = cabi.call

    def spy(name, *args):
        calls.append(name)
        return real(name, *args)

    cabi.call = spy
    try:
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            for ending in (False, True):
                zg = z.cuda().requires_grad_(True)
                m(zg, mask.cuda(), ending=ending).float().sum().backward()
            torch.cuda.synchronize()
    finally:
        cabi.call = real
    names = {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}
    library = sorted(n for n in names
                     if re.search(r"gemm|gemv|nvjet|xmma|cublas|cutlass", n, re.IGNORECASE))
    assert not library, "library GEMM kernels in a module step: %s" % library[:5]
    assert any("gdp_fwd_kernel" in n for n in names)
    assert any("linear_dx_kernel" in n for n in names)
    assert any("linear_dw_kernel" in n for n in names)
    for fn in ("cfk_linear_fwd", "cfk_linear_bwd_dx", "cfk_linear_bwd_dw"):
        assert fn in calls, fn


def _msa_case(column, seed):
    g = torch.Generator().manual_seed(seed)
    s, r, c_m, c_z = 64, 96, 64, 32
    heads, d = (4, 8) if column else (4, 16)
    p = oracle.module.make_msa_params(c_m, heads, d, c_z=None if column else c_z, seed=seed)
    m = torch.randn(s, r, c_m, generator=g)
    z = None if column else torch.randn(r, r, c_z, generator=g)
    mask = (torch.rand(s, r, generator=g) > 0.1).float()
    mask[:, -5:] = 0.0     # padded residues
    mask[-3:] = 0.0        # padded sequences
    return p, m, z, mask


@pytest.mark.parametrize("column", [False, True])
def test_msa_attention_modules(cuda_device, column):
    """MSA row attention with pair bias (D = 16) and MSA column attention (D = 8, batch = the
    residue axis through strides, zero bias) forward and backward against float64 autograd of
    the oracle modules."""
    from colabfold_legacy_kernels import modules
    p, m, z, mask = _msa_case(column, seed=30 + column)
    c_m = m.shape[2]
    if column:
        mod = modules.MSAColumnAttention(c_m, p.heads, p.w_q.shape[1] // p.heads, device="cuda")
    else:
        mod = modules.MSARowAttentionWithPairBias(c_m, z.shape[2], p.heads,
                                                  p.w_q.shape[1] // p.heads, device="cuda")
    with torch.no_grad():
        for name, t in p.named():
            getattr(mod, name).copy_(t)
    mg = m.cuda().requires_grad_(True)
    zg = None if column else z.cuda().requires_grad_(True)
    out = mod(mg, mask.cuda()) if column else mod(mg, zg, mask.cuda())
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(3))
    out.backward(dout.cuda().to(out.dtype))
    torch.cuda.synchronize()

    p64 = oracle.module.make_msa_params(c_m, p.heads, p.w_q.shape[1] // p.heads,
                                        c_z=None if column else z.shape[2], seed=30 + column,
                                        dtype=torch.float64)
    leaves = [t.requires_grad_(True) for _, t in p64.named()]
    m64 = m.double().requires_grad_(True)
    if column:
        ref = oracle.module.msa_column_attention(m64, mask, p64)
        ins = [m64]
    else:
        z64 = z.double().requires_grad_(True)
        ref = oracle.module.msa_row_attention(m64, z64, mask, p64)
        ins = [m64, z64]
    grads = torch.autograd.grad(ref, ins + leaves, dout.double())
    what = "column" if column else "row"
    assert_close_bf16(out, ref.detach(), "msa %s out" % what)
    _normwise(mg.grad, grads[0], "msa %s dm" % what)
    if not column:
        _normwise(zg.grad, grads[1], "msa row dz")
    ref_grads = {name: gref for (name, _), gref in zip(p64.named(), grads[len(ins):])}
    if not column:
        # d beta_z vanishes exactly (the bias gradient of every query row sums to zero over the
        # keys), so on its own it is pure rounding noise: check it with d gamma_z as one vector
        _normwise(torch.cat([mod.gamma_z.grad, mod.beta_z.grad]),
                  torch.cat([ref_grads.pop("gamma_z"), ref_grads.pop("beta_z")]),
                  "msa row d(gamma_z, beta_z)")
    for name, gref in ref_grads.items():
        _normwise(getattr(mod, name).grad, gref, "msa %s d%s" % (what, name))


@pytest.mark.parametrize("dtype,n", [(torch.bfloat16, 590_000 * 8 + 5), (torch.float16, 1003)])
def test_gate_kernels_against_torch_fp32(cuda_device, dtype, n):
    """cfk_gate_fwd / cfk_gate_bwd against a plain PyTorch fp32 evaluation of
    y = sigmoid(g) * o and its gradients, rtol = atol = 2e-2 (16-bit outputs), including a
    tail that is not a whole 16-byte vector."""
    from colabfold_legacy_kernels import torch_ops
    gen = torch.Generator(device="cuda").manual_seed(5)
    g = (torch.randn(n, device="cuda", generator=gen) * 3).to(dtype)
    o = torch.randn(n, device="cuda", generator=gen).to(dtype)
    dy = torch.randn(n, device="cuda", generator=gen).to(dtype)
    y = torch_ops.gate_fwd(g, o)
    d_o, dg = torch_ops.gate_bwd(g, o, dy)
    torch.cuda.synchronize()
    s = torch.sigmoid(g.float())
    assert_close_bf16(y, s * o.float(), "gate y")
    assert_close_bf16(d_o, dy.float() * s, "gate d_o")
    assert_close_bf16(dg, dy.float() * o.float() * s * (1 - s), "gate dg")
