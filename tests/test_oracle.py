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
