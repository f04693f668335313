"""Triangle attention (around the starting or the ending node) built on the sm_100a kernels.

The reference ships the three kernels; ColabFold composes them into the Evoformer's triangle
attention (AlphaFold 2 supplement, Algorithms 13 and 14):

  x = LayerNorm(z);  q, k, v = x Wq, x Wk, x Wv;  bias = x Wb;  g = sigmoid(x Wg + bg)
  o = attention(q, k, v, bias, key mask);  out = (g * o) Wo + bo

This module runs that composition forward and backward on a B200:

* LayerNorm forward/backward: cfk_ln_fwd / cfk_ln_bwd.
* The projections: one GEMM x [Wq|Wk|Wv] into a [Ni, Nj, 3, H, D] buffer, one for the bias and
  one for the gate (cuBLAS through torch, bf16 with f32 accumulation).
* Attention forward/backward: cfk_attn_fwd_strided / cfk_attn_bwd_strided.  q, k, v are views
  of the projection buffer and the output is written straight into [Ni, Nj, H, D] storage, for
  both node types (around the ending node the batch axis is the second residue axis, which is
  just other strides), so no transposed copy of q, k, v, o or of their gradients is made; dq, dk
  and dv land in views of one [Ni, Nj, 3, H, D] gradient buffer that feeds the projection's
  weight gradient directly.
* The gate and the output projection: torch elementwise ops and a cuBLAS GEMM.

Activations are bf16; LayerNorm's gamma and beta are f32 (the kernels' contract); the weights are
kept in f32 and cast to bf16 for the GEMMs, so their gradients arrive in f32.
"""

import math

import torch

from . import torch_ops


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, beta, eps):
        y, mean, rstd = torch_ops.layer_norm_fwd(x, gamma, beta, eps, return_stats=True)
        ctx.save_for_backward(x, gamma, mean, rstd)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gamma, mean, rstd = ctx.saved_tensors
        dx, dgamma, dbeta = torch_ops.layer_norm_bwd(x, gamma, dy.contiguous(), ctx.eps,
                                                     mean=mean, rstd=rstd)
        return dx, dgamma, dbeta, None


class _Linear(torch.autograd.Function):
    """y = x W (+ b) whose bias gradient is a GEMV (dy^T 1) rather than a column reduction of
    dy, which for [590k, 128] bf16 gradients is several times slower."""

    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.has_bias = b is not None
        return torch.addmm(b, x, w) if b is not None else x @ w

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx = dy @ w.t() if ctx.needs_input_grad[0] else None
        dw = x.t() @ dy if ctx.needs_input_grad[1] else None
        db = None
        if ctx.has_bias and ctx.needs_input_grad[2]:
            ones = torch.ones(dy.shape[0], 1, dtype=dy.dtype, device=dy.device)
            db = (dy.t() @ ones).view(-1)
        return dx, dw, db


def _batch_first(ending):
    """Permutation of [Ni, Nj, H, D] storage into the kernels' [N, H, S, D] order."""
    return (1, 2, 0, 3) if ending else (0, 2, 1, 3)


class _Attention(torch.autograd.Function):
    """o [Ni, Nj, H, D] from qkv [Ni, Nj, 3, H, D] (all strided views, no copies)."""

    @staticmethod
    def forward(ctx, qkv, bias, kmask, scale, ending):
        perm = _batch_first(ending)
        q, k, v = (qkv[:, :, t].permute(*perm) for t in range(3))
        ni, nj, _, h, d = qkv.shape
        o = torch.empty((ni, nj, h, d), dtype=qkv.dtype, device=qkv.device)
        bias = bias.contiguous()
        _, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, scale, out=o.permute(*perm))
        ctx.save_for_backward(qkv, bias, kmask, o, lse)
        ctx.scale, ctx.ending = scale, ending
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, bias, kmask, o, lse = ctx.saved_tensors
        perm = _batch_first(ctx.ending)
        q, k, v = (qkv[:, :, t].permute(*perm) for t in range(3))
        dqkv = torch.empty_like(qkv)
        dq, dk, dv = (dqkv[:, :, t].permute(*perm) for t in range(3))
        dbias = torch.empty(bias.shape, dtype=torch.float32, device=bias.device)
        torch_ops.attention_bwd(q, k, v, bias, kmask, o.permute(*perm), lse,
                                do.contiguous().permute(*perm), ctx.scale,
                                grads=(dq, dk, dv, dbias))
        return dqkv, dbias.to(bias.dtype), None, None, None


class TriangleAttention(torch.nn.Module):
    """Gated triangle self-attention over a pair representation z [Ni, Nj, C].

    forward(z, mask, ending=False): mask [Ni, Nj] (nonzero = keep) masks the keys of each
    attention row; ending=False attends along j for every i (starting node), ending=True along
    i for every j (ending node).  Returns [Ni, Nj, C] in bf16.
    """

    def __init__(self, c=128, heads=4, head_dim=32, eps=1e-5, device=None):
        super().__init__()
        hd = heads * head_dim
        f32 = dict(dtype=torch.float32, device=device)
        self.heads, self.head_dim, self.eps = heads, head_dim, eps
        self.gamma = torch.nn.Parameter(torch.ones(c, **f32))
        self.beta = torch.nn.Parameter(torch.zeros(c, **f32))
        self.w_q = torch.nn.Parameter(torch.randn(c, hd, **f32) * c ** -0.5)
        self.w_k = torch.nn.Parameter(torch.randn(c, hd, **f32) * c ** -0.5)
        self.w_v = torch.nn.Parameter(torch.randn(c, hd, **f32) * c ** -0.5)
        self.w_b = torch.nn.Parameter(torch.randn(c, heads, **f32) * c ** -0.5)
        self.w_g = torch.nn.Parameter(torch.zeros(c, hd, **f32))
        self.b_g = torch.nn.Parameter(torch.ones(hd, **f32))
        self.w_o = torch.nn.Parameter(torch.zeros(hd, c, **f32))
        self.b_o = torch.nn.Parameter(torch.zeros(c, **f32))

    def forward(self, z, mask, ending=False):
        ni, nj, c = z.shape
        if ni != nj or mask.shape != (ni, nj):
            raise ValueError("triangle attention needs a square pair representation and mask")
        h, d = self.heads, self.head_dim
        bf = torch.bfloat16
        x = _LayerNorm.apply(z.to(bf).reshape(ni * nj, c), self.gamma, self.beta, self.eps)
        w_qkv = torch.cat([self.w_q, self.w_k, self.w_v], dim=1).to(bf)
        qkv = _Linear.apply(x, w_qkv, None).view(ni, nj, 3, h, d)
        b = _Linear.apply(x, self.w_b.to(bf), None).view(ni, nj, h)
        # bias[h, query, key]: (x Wb)[query, key] around the starting node, [key, query] around
        # the ending node (the pair swapped with the residue axes)
        bias = b.permute(2, 1, 0) if ending else b.permute(2, 0, 1)
        keep = (mask != 0).to(torch.uint8)
        kmask = (keep.t() if ending else keep).contiguous()
        o = _Attention.apply(qkv, bias, kmask, 1.0 / math.sqrt(d), ending)
        gate = torch.sigmoid(_Linear.apply(x, self.w_g.to(bf), self.b_g.to(bf)))
        out = _Linear.apply(gate * o.view(ni * nj, h * d), self.w_o.to(bf), self.b_o.to(bf))
        return out.view(ni, nj, c)
