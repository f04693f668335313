"""The CPU oracle against torch.autograd and against its own invariants (no GPU).

The backward restatements must equal autograd of the forward restatements; the forward must
follow the reference's replacement semantics (cuda/volta_mma_attn.cu:186-191).
"""

import math

import pytest
import torch

import oracle


def _attn_inputs(n=3, h=2, sq=9, sk=11, d=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, h, sq, d, generator=g, dtype=torch.float64)
    k = torch.randn(n, h, sk, d, generator=g, dtype=torch.float64)
    v = torch.randn(n, h, sk, d, generator=g, dtype=torch.float64)
    bias = torch.randn(h, sq, sk, generator=g, dtype=torch.float64)
    kmask = (torch.rand(n, sk, generator=g) > 0.3).to(torch.uint8)
    kmask[1] = 0
    return q, k, v, bias, kmask


def test_attention_masked_logits_are_replaced():
    q, k, v, bias, kmask = _attn_inputs()
    logits, keep = oracle.attention_logits(q, k, bias, kmask, 0.3)
    assert torch.all(logits[~keep.expand_as(logits)] == -1e4)


def test_attention_fully_masked_row_is_uniform():
    q, k, v, bias, kmask = _attn_inputs()
    out, lse = oracle.attention_fwd(q, k, v, bias, kmask, 0.3)
    assert torch.allclose(out[1], v[1].mean(dim=1, keepdim=True).expand_as(out[1]))
    assert torch.allclose(lse[1], torch.full_like(lse[1], -1e4 + math.log(11)))


def test_attention_ref_block_k_quirk():
    # The reference's padded key columns enter the softmax of fully masked rows with V = 0.
    q, k, v, bias, kmask = _attn_inputs(sk=11)
    out, _ = oracle.attention_fwd(q, k, v, bias, kmask, 0.3, ref_block_k=16)
    assert torch.allclose(out[1], v[1].sum(dim=1, keepdim=True).expand_as(out[1]) / 16)
    out0, _ = oracle.attention_fwd(q, k, v, bias, kmask, 0.3)
    assert torch.allclose(out[0], out0[0])


def test_attention_bwd_matches_autograd():
    q, k, v, bias, kmask = _attn_inputs()
    scale = 0.37
    qs, ks, vs, bs = (t.clone().requires_grad_() for t in (q, k, v, bias))
    out, lse = oracle.attention_fwd(qs, ks, vs, bs, kmask, scale)
    dout = torch.randn_like(out)
    out.backward(dout)
    dq, dk, dv, dbias = oracle.attention_bwd(q, k, v, bias, kmask, out.detach(), lse.detach(),
                                             dout, scale)
    for a, b, name in ((dq, qs.grad, "dq"), (dk, ks.grad, "dk"), (dv, vs.grad, "dv"),
                       (dbias, bs.grad, "dbias")):
        assert torch.allclose(a, b, atol=1e-10, rtol=1e-9), name


def test_layer_norm_matches_autograd_and_reference_variance():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(7, 24, generator=g, dtype=torch.float64) * 3 + 1
    gamma = 1 + 0.1 * torch.randn(24, generator=g, dtype=torch.float64)
    beta = 0.1 * torch.randn(24, generator=g, dtype=torch.float64)
    y, mean, rstd = oracle.layer_norm_fwd(x, gamma, beta, 1e-5)
    y2, _, _ = oracle.layer_norm_fwd(x, gamma, beta, 1e-5, two_pass=False)
    assert torch.allclose(y, y2, atol=1e-12)
    ref = torch.nn.functional.layer_norm(x, (24,), gamma, beta, 1e-5)
    assert torch.allclose(y, ref, atol=1e-12)
    xs, gs, bs = (t.clone().requires_grad_() for t in (x, gamma, beta))
    yy = torch.nn.functional.layer_norm(xs, (24,), gs, bs, 1e-5)
    dy = torch.randn_like(yy)
    yy.backward(dy)
    dx, dg, db = oracle.layer_norm_bwd(x, gamma, dy, 1e-5)
    assert torch.allclose(dx, xs.grad, atol=1e-10)
    assert torch.allclose(dg, gs.grad, atol=1e-10)
    assert torch.allclose(db, bs.grad, atol=1e-10)
    dx2, _, _ = oracle.layer_norm_bwd(x, gamma, dy, 1e-5, mean=mean, rstd=rstd)
    assert torch.allclose(dx, dx2)


def test_gdp_matches_autograd():
    g = torch.Generator().manual_seed(2)
    m, k, n = 13, 16, 24
    x, wp, wg = (torch.randn(*s, generator=g, dtype=torch.float64) for s in ((m, k), (k, n), (k, n)))
    bp, bg = torch.randn(n, generator=g, dtype=torch.float64), torch.randn(n, generator=g, dtype=torch.float64)
    mask = (torch.rand(m, generator=g) > 0.2).double()
    ts = [t.clone().requires_grad_() for t in (x, wp, bp, wg, bg)]
    out = oracle.gdp_fwd(*ts, mask)
    dout = torch.randn_like(out)
    out.backward(dout)
    grads = oracle.gdp_bwd(x, wp, bp, wg, bg, mask, dout)
    for a, t in zip(grads, ts):
        assert torch.allclose(a, t.grad, atol=1e-10)
    # the fused form equals the two-projection definition
    assert torch.allclose(out, mask[:, None] * (x @ wp + bp) * torch.sigmoid(x @ wg + bg))


def test_config_generators_shapes():
    cfg = oracle.configs.scaled(oracle.configs.C3, n=4, s=16)
    t = oracle.configs.make_attention_inputs(cfg)
    assert t["q"].shape == (4, 4, 16, 32) and t["bias"].shape == (4, 16, 16)
    assert t["kmask"].dtype == torch.uint8 and t["dout"].shape == t["q"].shape
    cfg2 = oracle.configs.scaled(oracle.configs.C2, n=8)
    t2 = oracle.configs.make_attention_inputs(cfg2)
    assert t2["q"].shape == (8, 8, 256, 32)
    # same seed, same tensors
    t3 = oracle.configs.make_attention_inputs(cfg2)
    assert torch.equal(t2["q"], t3["q"]) and torch.equal(t2["kmask"], t3["kmask"])


def _module_case(n=12, c=16, heads=2, head_dim=4, seed=3):
    p = oracle.module.make_params(c, heads, head_dim, seed=seed, dtype=torch.float64)
    g = torch.Generator().manual_seed(seed + 1)
    z = torch.randn(n, n, c, generator=g, dtype=torch.float64)
    res = (torch.rand(n, generator=g) > 0.2).double()
    res[0] = 0.0                                  # one padded residue: its row is fully masked
    mask = res[:, None] * res[None, :]
    return z, mask, p


@pytest.mark.parametrize("ending", [False, True])
def test_module_matches_the_literal_algorithms(ending):
    """The triangle-attention module (config C1's composition of LayerNorm, projections, the
    attention op and the gated output projection) equals an index-by-index evaluation of the
    starting-node / ending-node algorithms, including the axis swap of the ending node."""
    z, mask, p = _module_case()
    got = oracle.module.triangle_attention(z, mask, p, ending=ending)
    want = oracle.module.triangle_attention_literal(z, mask, p, ending=ending)
    assert torch.allclose(got, want, rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("ending", [False, True])
def test_module_backward_composition_equals_autograd(ending):
    """The module's gradients composed from the per-op backward restatements (the composition
    the GPU module performs) equal torch.autograd of the float64 forward."""
    z, mask, p = _module_case(seed=5)
    z = z.clone().requires_grad_(True)
    params = p.tensors()
    for t in params:
        t.requires_grad_(True)
    out = oracle.module.triangle_attention(z, mask, p, ending=ending)
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(9), dtype=torch.float64)
    auto = torch.autograd.grad(out, [z] + params, dout)
    dz, grads = oracle.module.triangle_attention_bwd(z.detach(), mask, p, dout, ending=ending)
    names = ["gamma", "beta", "w_q", "w_k", "w_v", "w_b", "w_g", "b_g", "w_o", "b_o"]
    assert torch.allclose(dz, auto[0], rtol=1e-9, atol=1e-10)
    for name, a in zip(names, auto[1:]):
        assert torch.allclose(grads[name], a, rtol=1e-9, atol=1e-10), name


def test_module_c1_fp32_close_to_fp64():
    """Config C1 (z [128,128,128], H = 4, D = 32, seed 0) end to end: the fp32 evaluation of the
    module stays within 1e-4 of the float64 one (relative to the output's scale)."""
    p = oracle.module.make_params(128, 4, 32, seed=0)
    g = torch.Generator().manual_seed(0)
    z = torch.randn(128, 128, 128, generator=g)
    mask = torch.ones(128, 128)
    out64 = oracle.module.triangle_attention(z, mask, p, dtype=torch.float64)
    out32 = oracle.module.triangle_attention(z, mask, p, dtype=torch.float32)
    scale = float(out64.abs().max())
    assert float((out32.double() - out64).abs().max()) <= 1e-4 * scale


@pytest.mark.parametrize("column", [False, True])
def test_msa_attention_modules_match_the_literal_algorithms(column):
    """MSA row attention with pair bias and MSA column attention, composed from the oracle's
    LayerNorm and attention, equal index-by-index evaluations of their algorithms."""
    g = torch.Generator().manual_seed(21)
    s, r = 7, 10
    p = oracle.module.make_msa_params(12, 3, 4, c_z=None if column else 6, seed=4,
                                      dtype=torch.float64)
    m = torch.randn(s, r, 12, generator=g, dtype=torch.float64)
    mask = (torch.rand(s, r, generator=g) > 0.25).double()
    mask[2] = 0.0
    if column:
        got = oracle.module.msa_column_attention(m, mask, p)
        want = oracle.module.msa_attention_literal(m, mask, p, column=True)
    else:
        z = torch.randn(r, r, 6, generator=g, dtype=torch.float64)
        got = oracle.module.msa_row_attention(m, z, mask, p)
        want = oracle.module.msa_attention_literal(m, mask, p, z=z)
    assert torch.allclose(got, want, rtol=1e-10, atol=1e-10)
