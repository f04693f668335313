"""The Evoformer's attention modules built on the sm_100a kernels: triangle attention (around
the starting or the ending node), MSA row attention with pair bias, MSA column attention.

The reference ships the three kernels; ColabFold composes them into the Evoformer's triangle
attention (AlphaFold 2 supplement, Algorithms 13 and 14):

  x = LayerNorm(z);  q, k, v = x Wq, x Wk, x Wv;  bias = x Wb;  g = sigmoid(x Wg + bg)
  o = attention(q, k, v, bias, key mask);  out = (g * o) Wo + bo

This module runs that composition forward and backward on a B200:

* LayerNorm forward/backward: cfk_ln_fwd / cfk_ln_bwd.
* The projections on this build's tcgen05 kernels (cfk_linear_*): one launch x [Wq|Wk|Wv|Wg]
  + [0|0|0|bg] writes q|k|v into a [Ni, Nj, 3, H, D] buffer and the gate pre-activation into
  its own; the pair bias x Wb (Wb zero-padded to 16 columns) is a second small launch.  Their
  backward is one cfk_linear_bwd_dx over the blocks (dq|dk|dv, dg, the bias rows) and one
  cfk_linear_bwd_dw that reads x once (f32 weight and bias gradients, fixed summation order).
* Attention forward/backward: cfk_attn_fwd_strided / cfk_attn_bwd_strided.  q, k, v are views
  of the projection buffer and the output is written straight into [Ni, Nj, H, D] storage, for
  attention along either axis (around the ending node, or along an MSA column, the batch axis
  is the second axis, which is just other strides), so no transposed copy of q, k, v, o or of
  their gradients is made; dq, dk and dv land in views of one [Ni, Nj, 3, H, D] gradient
  buffer that feeds the projection's weight gradient directly.
* The gate: cfk_gate_fwd / cfk_gate_bwd, one fused pass each way; the output projection:
  cfk_linear_fwd, cfk_linear_bwd_dx and cfk_linear_bwd_dw.

No cuBLAS GEMM runs in a module step.  Activations are bf16; LayerNorm's gamma and beta are f32
(the kernels' contract); the weights are f32 master copies cast to bf16 for the kernels, and
their gradients come back in f32 straight from the f32 tensor-memory accumulators.
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
    """y = x W + b on this build's kernels (cfk_linear_fwd / cfk_linear_bwd_dx /
    cfk_linear_bwd_dw); W [K, N] and b [N] are f32 master weights cast to x's dtype for the
    kernels, and their gradients are returned in f32."""

    @staticmethod
    def forward(ctx, x, w, b):
        w16 = w.to(x.dtype).contiguous()
        y = torch_ops.linear_fwd(x, w16, b.to(x.dtype) if b is not None else None)
        ctx.save_for_backward(x, w16)
        ctx.has_bias = b is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w16 = ctx.saved_tensors
        dy = dy.contiguous()
        dx = torch_ops.linear_bwd_dx([dy], [w16]) if ctx.needs_input_grad[0] else None
        (dw, db), = torch_ops.linear_bwd_dw(x, [dy], [ctx.has_bias])
        return dx, dw, db


def _pad16(w, dtype):
    """w [C, n] (n <= 16) zero-padded to [C, 16] in dtype: the kernels take column blocks that
    are multiples of 8 (16 for the dx pass), and a pair bias has H = 4 or 8 columns."""
    out = torch.zeros((w.shape[0], 16), dtype=dtype, device=w.device)
    out[:, :w.shape[1]] = w.to(dtype)
    return out


class _PairBias(torch.autograd.Function):
    """x W_b [M, H] (no bias term), through a 16-column padded weight."""

    @staticmethod
    def forward(ctx, x, w_b):
        wb16 = _pad16(w_b, x.dtype)
        y = torch_ops.linear_fwd(x, wb16)
        ctx.save_for_backward(x, wb16)
        ctx.h = w_b.shape[1]
        return y[:, :ctx.h]

    @staticmethod
    def backward(ctx, dy):
        x, wb16 = ctx.saved_tensors
        d16 = torch.zeros((x.shape[0], 16), dtype=x.dtype, device=x.device)
        d16[:, :ctx.h] = dy
        dx = torch_ops.linear_bwd_dx([d16], [wb16]) if ctx.needs_input_grad[0] else None
        (dw, _), = torch_ops.linear_bwd_dw(x, [d16], [False])
        return dx, dw[:, :ctx.h]


class _InProj(torch.autograd.Function):
    """The input projections of a gated attention from x [M, C]: qkv [M, 3HD] = x [Wq|Wk|Wv],
    g [M, HD] = x Wg + bg, and, when w_b is given (triangle attention), the pair-bias rows
    [M, 16] = x Wb (zero-padded; columns [0, H) are the bias).  The forward writes q|k|v and g
    into their own buffers from one cfk_linear_fwd (two where 3HD is not a multiple of 128);
    the backward is one cfk_linear_bwd_dx over the blocks dq|dk|dv, dg (and the bias rows) and
    one cfk_linear_bwd_dw, which reads x once."""

    @staticmethod
    def forward(ctx, x, w_qkv, w_g, b_g, w_b):
        dt, m = x.dtype, x.shape[0]
        hd3, hd = w_qkv.shape[1], w_g.shape[1]
        w_all = torch.cat([w_qkv, w_g], 1).to(dt).contiguous()
        qkv = torch.empty((m, hd3), dtype=dt, device=x.device)
        g = torch.empty((m, hd), dtype=dt, device=x.device)
        if hd3 % 128 == 0:
            b_all = torch.cat([torch.zeros(hd3, device=x.device), b_g]).to(dt)
            torch_ops.linear_fwd(x, w_all, b_all, out=(qkv, g))
        else:
            torch_ops.linear_fwd(x, w_all[:, :hd3].contiguous(), None, out=qkv)
            torch_ops.linear_fwd(x, w_all[:, hd3:].contiguous(), b_g.to(dt), out=g)
        if w_b is not None:
            wb16 = _pad16(w_b, dt)
            b16 = torch_ops.linear_fwd(x, wb16)
        else:
            wb16 = b16 = x.new_empty(0)
        ctx.save_for_backward(x, w_all, wb16)
        ctx.hd3 = hd3
        ctx.nb = w_b.shape[1] if w_b is not None else 0
        return qkv, g, b16

    @staticmethod
    def backward(ctx, d_qkv, d_g, d_b16):
        x, w_all, wb16 = ctx.saved_tensors
        hd3 = ctx.hd3
        dys = [d_qkv.contiguous(), d_g.contiguous()]
        ws = [w_all[:, :hd3].contiguous(), w_all[:, hd3:].contiguous()]
        with_bias = [False, True]
        if ctx.nb:
            dys.append(d_b16.contiguous())
            ws.append(wb16)
            with_bias.append(False)
        dx = torch_ops.linear_bwd_dx(dys, ws) if ctx.needs_input_grad[0] else None
        grads = torch_ops.linear_bwd_dw(x, dys, with_bias)
        d_wb = grads[2][0][:, :ctx.nb] if ctx.nb else None
        return dx, grads[0][0], grads[1][0], grads[1][1], d_wb


class _Gate(torch.autograd.Function):
    """sigmoid(g) * o with the forward and the backward each one fused pass (cfk_gate_*)."""

    @staticmethod
    def forward(ctx, g, o):
        g, o = g.contiguous(), o.contiguous()
        ctx.save_for_backward(g, o)
        return torch_ops.gate_fwd(g, o)

    @staticmethod
    def backward(ctx, dy):
        g, o = ctx.saved_tensors
        d_o, dg = torch_ops.gate_bwd(g, o, dy.contiguous())
        return dg, d_o


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


def _gated_attention(x, a, b, heads, head_dim, w_qkv, w_g, b_g, w_o, b_o, bias, kmask,
                     over_first, w_b=None, bias_view=None):
    """Gated attention over one axis of normalised rows x [a*b, C] (bf16) laid out [a, b, C]:
    over the second axis (batch = first axis) or, with over_first, over the first (batch =
    second axis).  bias [H, S, S] bf16 (S = the attended axis' length), or, with w_b, the pair
    bias x Wb reshaped by bias_view(rows [a*b, H]) -> [H, S, S].  kmask u8 [batch, S].
    Returns [a*b, C_out]."""
    qkv, g, b16 = _InProj.apply(x, w_qkv, w_g, b_g, w_b)
    if w_b is not None:
        bias = bias_view(b16[:, :w_b.shape[1]])
    o = _Attention.apply(qkv.view(a, b, 3, heads, head_dim), bias, kmask,
                         1.0 / math.sqrt(head_dim), over_first)
    gated = _Gate.apply(g, o.view(a * b, heads * head_dim))
    return _Linear.apply(gated, w_o, b_o)


class _GatedAttentionParams(torch.nn.Module):
    """LayerNorm and gated-attention parameters (f32 master copies): gamma, beta, w_q, w_k,
    w_v, w_g, b_g, w_o, b_o.  The gate starts open (b_g = 1) and the output at zero (w_o = 0),
    as in AlphaFold."""

    def __init__(self, c, heads, head_dim, eps, device):
        super().__init__()
        hd = heads * head_dim
        f32 = dict(dtype=torch.float32, device=device)
        self.heads, self.head_dim, self.eps = heads, head_dim, eps
        self.gamma = torch.nn.Parameter(torch.ones(c, **f32))
        self.beta = torch.nn.Parameter(torch.zeros(c, **f32))
        self.w_q = torch.nn.Parameter(torch.randn(c, hd, **f32) * c ** -0.5)
        self.w_k = torch.nn.Parameter(torch.randn(c, hd, **f32) * c ** -0.5)
        self.w_v = torch.nn.Parameter(torch.randn(c, hd, **f32) * c ** -0.5)
        self.w_g = torch.nn.Parameter(torch.zeros(c, hd, **f32))
        self.b_g = torch.nn.Parameter(torch.ones(hd, **f32))
        self.w_o = torch.nn.Parameter(torch.zeros(hd, c, **f32))
        self.b_o = torch.nn.Parameter(torch.zeros(c, **f32))

    def _norm(self, t):
        a, b, c = t.shape
        return _LayerNorm.apply(t.to(torch.bfloat16).reshape(a * b, c), self.gamma, self.beta,
                                self.eps)

    def _attend(self, x, a, b, bias, kmask, over_first, w_b=None, bias_view=None):
        w_qkv = torch.cat([self.w_q, self.w_k, self.w_v], dim=1)
        return _gated_attention(x, a, b, self.heads, self.head_dim, w_qkv, self.w_g, self.b_g,
                                self.w_o, self.b_o, bias, kmask, over_first, w_b, bias_view)


class TriangleAttention(_GatedAttentionParams):
    """Gated triangle self-attention over a pair representation z [Ni, Nj, C].

    forward(z, mask, ending=False): mask [Ni, Nj] (nonzero = keep) masks the keys of each
    attention row; ending=False attends along j for every i (starting node), ending=True along
    i for every j (ending node).  Returns [Ni, Nj, C] in bf16.
    """

    def __init__(self, c=128, heads=4, head_dim=32, eps=1e-5, device=None):
        super().__init__(c, heads, head_dim, eps, device)
        self.w_b = torch.nn.Parameter(
            torch.randn(c, heads, dtype=torch.float32, device=device) * c ** -0.5)

    def forward(self, z, mask, ending=False):
        ni, nj, c = z.shape
        if ni != nj or mask.shape != (ni, nj):
            raise ValueError("triangle attention needs a square pair representation and mask")
        x = self._norm(z)

        def bias_view(rows):
            # bias[h, query, key]: (x Wb)[query, key] around the starting node, [key, query]
            # around the ending node (the pair swapped with the residue axes)
            b = rows.view(ni, nj, self.heads)
            return b.permute(2, 1, 0) if ending else b.permute(2, 0, 1)

        keep = (mask != 0).to(torch.uint8)
        kmask = (keep.t() if ending else keep).contiguous()
        return self._attend(x, ni, nj, None, kmask, ending, self.w_b, bias_view).view(ni, nj, c)


class MSARowAttentionWithPairBias(_GatedAttentionParams):
    """Gated self-attention along the residues of each MSA row, biased by the pair
    representation (AlphaFold 2 supplement, Algorithm 7).

    forward(m, z, msa_mask): m [S, R, C_m], z [R, R, C_z], msa_mask [S, R].  The bias is
    LayerNorm(z) W_b, [H, R, R], shared by all S rows.  Returns [S, R, C_m] in bf16.
    """

    def __init__(self, c_m=64, c_z=128, heads=8, head_dim=8, eps=1e-5, device=None):
        super().__init__(c_m, heads, head_dim, eps, device)
        f32 = dict(dtype=torch.float32, device=device)
        self.gamma_z = torch.nn.Parameter(torch.ones(c_z, **f32))
        self.beta_z = torch.nn.Parameter(torch.zeros(c_z, **f32))
        self.w_b = torch.nn.Parameter(torch.randn(c_z, heads, **f32) * c_z ** -0.5)

    def forward(self, m, z, msa_mask):
        s, r, c = m.shape
        if z.shape[:2] != (r, r) or msa_mask.shape != (s, r):
            raise ValueError("m [S,R,C], z [R,R,Cz] and msa_mask [S,R] disagree")
        x = self._norm(m)
        zn = _LayerNorm.apply(z.to(torch.bfloat16).reshape(r * r, z.shape[2]), self.gamma_z,
                              self.beta_z, self.eps)
        bias = _PairBias.apply(zn, self.w_b).view(r, r, self.heads)
        kmask = (msa_mask != 0).to(torch.uint8).contiguous()
        return self._attend(x, s, r, bias.permute(2, 0, 1), kmask, False).view(s, r, c)


class MSAColumnAttention(_GatedAttentionParams):
    """Gated self-attention along the sequences of each MSA column (AlphaFold 2 supplement,
    Algorithm 8): the batch is the residue axis, read through strides, and there is no pair
    bias (the kernel gets a zero bias).

    forward(m, msa_mask): m [S, R, C_m], msa_mask [S, R].  Returns [S, R, C_m] in bf16.
    """

    def __init__(self, c_m=64, heads=8, head_dim=8, eps=1e-5, device=None):
        super().__init__(c_m, heads, head_dim, eps, device)

    def forward(self, m, msa_mask):
        s, r, c = m.shape
        if msa_mask.shape != (s, r):
            raise ValueError("m [S,R,C] and msa_mask [S,R] disagree")
        x = self._norm(m)
        bias = torch.zeros((self.heads, s, s), dtype=torch.bfloat16, device=m.device)
        kmask = (msa_mask != 0).to(torch.uint8).t().contiguous()
        return self._attend(x, s, r, bias, kmask, True).view(s, r, c)
