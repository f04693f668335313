"""Triangle-attention module around the attention kernel (config C1) -- CPU restatement, TEST
ORACLE ONLY.

The reference ships the kernels, not the module that calls them; its caller (ColabFold's
triangle attention, the AlphaFold 2 supplement's Algorithms 13 and 14) composes them as

  x        = LayerNorm(z)                         z [Ni, Nj, C]   (VoltaLayerNorm,
                                                                   cuda/volta_ops.cu:40-58)
  q, k, v  = x Wq, x Wk, x Wv  as [Ni, H, Nj, D]  (batch = the first residue axis)
  bias     = x Wb              as [H, Nj, Nj]     (bias[h, j, k] = (x Wb)[j, k, h], shared by
                                                   every batch row i)
  o        = attention(q, k, v, bias, kmask = mask, scale = 1/sqrt(D))
                                                  (VoltaMma, cuda/volta_mma_attn.cu:139-271)
  g        = sigmoid(x Wg + bg)
  out      = (g * o) Wo + bo                      [Ni, Nj, C]

around the starting node.  Around the ending node attention runs over i for every j with
logit = q_ij . k_kj + b_ki: the same module applied to z with its two residue axes swapped (the
mask swapped likewise), its output swapped back.

Everything is float64 torch by default and differentiable, so the module's gradients are
torch.autograd of this forward (tests/test_oracle.py checks the composition against a literal
index-by-index evaluation of both algorithms).
"""

import math
from dataclasses import dataclass

import torch

from .attention import attention_fwd
from .layer_norm import layer_norm_fwd


@dataclass
class TriAttnParams:
    gamma: torch.Tensor  # [C]
    beta: torch.Tensor   # [C]
    w_q: torch.Tensor    # [C, H*D]
    w_k: torch.Tensor
    w_v: torch.Tensor
    w_b: torch.Tensor    # [C, H]
    w_g: torch.Tensor    # [C, H*D]
    b_g: torch.Tensor    # [H*D]
    w_o: torch.Tensor    # [H*D, C]
    b_o: torch.Tensor    # [C]
    heads: int
    eps: float = 1e-5

    def tensors(self):
        return [self.gamma, self.beta, self.w_q, self.w_k, self.w_v, self.w_b, self.w_g,
                self.b_g, self.w_o, self.b_o]


def make_params(c=128, heads=4, head_dim=32, seed=0, dtype=torch.float32, device="cpu"):
    """C1's parameters: gamma = 1 + 0.1 N, beta = 0.1 N, weights N(0, 1/C); the gate bias 1
    and the output bias 0 (AlphaFold's initialisation of those two)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    hd = heads * head_dim

    def rn(*shape, std=1.0):
        return (torch.randn(*shape, generator=g) * std).to(dtype=dtype, device=device)

    return TriAttnParams(
        gamma=1.0 + rn(c, std=0.1), beta=rn(c, std=0.1),
        w_q=rn(c, hd, std=c ** -0.5), w_k=rn(c, hd, std=c ** -0.5), w_v=rn(c, hd, std=c ** -0.5),
        w_b=rn(c, heads, std=c ** -0.5), w_g=rn(c, hd, std=c ** -0.5),
        b_g=torch.ones(hd, dtype=dtype, device=device), w_o=rn(hd, c, std=hd ** -0.5),
        b_o=torch.zeros(c, dtype=dtype, device=device), heads=heads)


def triangle_attention(z, mask, p, ending=False, dtype=torch.float64):
    """The module's output [Ni, Nj, C] in `dtype`.  z [Ni, Nj, C]; mask [Ni, Nj] (0 = padded
    residue pair, used as the attention key mask of each batch row)."""
    if ending:
        return triangle_attention(z.transpose(0, 1), mask.transpose(0, 1), p, False,
                                  dtype).transpose(0, 1)
    ni, nj, c = z.shape
    h = p.heads
    cast = [t.to(dtype) for t in p.tensors()]
    gamma, beta, w_q, w_k, w_v, w_b, w_g, b_g, w_o, b_o = cast
    x = layer_norm_fwd(z.reshape(ni * nj, c), gamma, beta, p.eps, dtype)[0].view(ni, nj, c)
    hd = w_q.shape[1]
    d = hd // h

    def heads_first(t):  # [Ni, Nj, H*D] -> [Ni, H, Nj, D]
        return t.view(ni, nj, h, d).permute(0, 2, 1, 3)

    q, k, v = heads_first(x @ w_q), heads_first(x @ w_k), heads_first(x @ w_v)
    bias = (x @ w_b).permute(2, 0, 1)                      # [H, Nj(query), Nj(key)]
    o, _ = attention_fwd(q, k, v, bias, mask.to(torch.uint8), 1.0 / math.sqrt(d), dtype)
    o = o.permute(0, 2, 1, 3).reshape(ni, nj, hd)
    gate = torch.sigmoid(x @ w_g + b_g)
    return (gate * o) @ w_o + b_o


def triangle_attention_literal(z, mask, p, ending=False):
    """Index-by-index float64 evaluation of Algorithm 13 (starting node) or 14 (ending node),
    written independently of triangle_attention() to check its axis bookkeeping."""
    z = z.double()
    gamma, beta, w_q, w_k, w_v, w_b, w_g, b_g, w_o, b_o = [t.double() for t in p.tensors()]
    ni, nj, c = z.shape
    h = p.heads
    d = w_q.shape[1] // h
    mu = z.mean(-1, keepdim=True)
    x = (z - mu) / torch.sqrt(((z - mu) ** 2).mean(-1, keepdim=True) + p.eps) * gamma + beta
    q = (x @ w_q).view(ni, nj, h, d)
    k = (x @ w_k).view(ni, nj, h, d)
    v = (x @ w_v).view(ni, nj, h, d)
    b = x @ w_b                                            # [Ni, Nj, H]
    keep = mask != 0
    if not ending:
        # a_ijk = q_ij . k_ik / sqrt(d) + b_jk, over keys k of row i
        logit = torch.einsum("ijhd,ikhd->ijkh", q, k) / math.sqrt(d) + b[None, :, :, :]
        logit = torch.where(keep[:, None, :, None], logit, torch.full_like(logit, -1e4))
        a = torch.softmax(logit, dim=2)
        o = torch.einsum("ijkh,ikhd->ijhd", a, v)
    else:
        # a_ijk = q_ij . k_kj / sqrt(d) + b_ki, over keys k of column j
        logit = torch.einsum("ijhd,kjhd->ijkh", q, k) / math.sqrt(d) + \
            b.permute(1, 0, 2)[:, None, :, :]
        logit = torch.where(keep.t()[None, :, :, None], logit, torch.full_like(logit, -1e4))
        a = torch.softmax(logit, dim=2)
        o = torch.einsum("ijkh,kjhd->ijhd", a, v)
    gate = torch.sigmoid(x @ w_g + b_g)
    return (gate * o.reshape(ni, nj, h * d)) @ w_o + b_o


def triangle_attention_bwd(z, mask, p, dout, ending=False, dtype=torch.float64):
    """(dz, {name: dparam}) of triangle_attention composed from the per-op backward
    restatements (layer_norm_bwd, attention_bwd) and the transposes of the linear maps -- the
    composition the GPU module performs with the sm_100a kernels.  tests/test_oracle.py checks
    it against torch.autograd of triangle_attention."""
    from .attention import attention_bwd
    from .layer_norm import layer_norm_bwd
    if ending:
        dz, grads = triangle_attention_bwd(z.transpose(0, 1), mask.transpose(0, 1), p,
                                           dout.transpose(0, 1), False, dtype)
        return dz.transpose(0, 1), grads
    ni, nj, c = z.shape
    h = p.heads
    gamma, beta, w_q, w_k, w_v, w_b, w_g, b_g, w_o, b_o = [t.to(dtype) for t in p.tensors()]
    hd = w_q.shape[1]
    d = hd // h
    scale = 1.0 / math.sqrt(d)
    z2 = z.reshape(ni * nj, c).to(dtype)
    x2, mean, rstd = layer_norm_fwd(z2, gamma, beta, p.eps, dtype)
    x = x2.view(ni, nj, c)

    def heads_first(t):
        return t.reshape(ni, nj, h, d).permute(0, 2, 1, 3)

    def heads_last(t):
        return t.permute(0, 2, 1, 3).reshape(ni, nj, hd)

    q, k, v = heads_first(x @ w_q), heads_first(x @ w_k), heads_first(x @ w_v)
    bias = (x @ w_b).permute(2, 0, 1)
    kmask = mask.to(torch.uint8)
    o4, lse = attention_fwd(q, k, v, bias, kmask, scale, dtype)
    o = heads_last(o4)
    gate = torch.sigmoid(x @ w_g + b_g)
    dout = dout.to(dtype)
    # out = (gate * o) Wo + bo
    go = gate * o
    d_go = dout @ w_o.t()
    grads = {"w_o": go.reshape(-1, hd).t() @ dout.reshape(-1, c),
             "b_o": dout.reshape(-1, c).sum(0)}
    d_o = d_go * gate
    d_pre = d_go * o * gate * (1.0 - gate)               # through the sigmoid
    grads["w_g"] = x2.t() @ d_pre.reshape(-1, hd)
    grads["b_g"] = d_pre.reshape(-1, hd).sum(0)
    dx = d_pre @ w_g.t()
    dq, dk, dv, dbias = attention_bwd(q, k, v, bias, kmask, o4, lse, heads_first(d_o), scale,
                                      dtype)
    for name, dt, w in (("w_q", dq, w_q), ("w_k", dk, w_k), ("w_v", dv, w_v)):
        dt = heads_last(dt)
        grads[name] = x2.t() @ dt.reshape(-1, hd)
        dx = dx + dt @ w.t()
    db = dbias.permute(1, 2, 0)                            # [Nj(query), Nj(key), H]
    grads["w_b"] = x2.t() @ db.reshape(-1, h)
    dx = dx + db @ w_b.t()
    dz, grads["gamma"], grads["beta"] = layer_norm_bwd(z2, gamma, dx.reshape(-1, c), p.eps, mean,
                                                       rstd, dtype)
    return dz.view(ni, nj, c), grads


# ------------------------------------------------------------------------------------------
# MSA row attention with pair bias and MSA column attention (AlphaFold 2 supplement,
# Algorithms 7 and 8): the same gated attention over one axis of m [S, R, C_m].
# ------------------------------------------------------------------------------------------

@dataclass
class MsaAttnParams:
    gamma: torch.Tensor  # [C_m]
    beta: torch.Tensor
    w_q: torch.Tensor    # [C_m, H*D]
    w_k: torch.Tensor
    w_v: torch.Tensor
    w_g: torch.Tensor
    b_g: torch.Tensor    # [H*D]
    w_o: torch.Tensor    # [H*D, C_m]
    b_o: torch.Tensor    # [C_m]
    heads: int
    gamma_z: torch.Tensor = None  # row attention only: LayerNorm of z and the bias weights
    beta_z: torch.Tensor = None
    w_b: torch.Tensor = None      # [C_z, H]
    eps: float = 1e-5

    NAMES = ("gamma", "beta", "w_q", "w_k", "w_v", "w_g", "b_g", "w_o", "b_o")
    PAIR_NAMES = ("gamma_z", "beta_z", "w_b")

    def named(self):
        names = self.NAMES + (self.PAIR_NAMES if self.w_b is not None else ())
        return [(n, getattr(self, n)) for n in names]


def make_msa_params(c_m=64, heads=8, head_dim=8, c_z=None, seed=0, dtype=torch.float32):
    """Random parameters (LayerNorm gamma = 1 + 0.1 N, beta = 0.1 N; weights N(0, 1/fan-in);
    gate bias 1 + 0.1 N, output bias 0.1 N); c_z given = with the pair-bias branch."""
    g = torch.Generator().manual_seed(seed)
    hd = heads * head_dim

    def rn(*shape, std=1.0):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    p = MsaAttnParams(gamma=1.0 + rn(c_m, std=0.1), beta=rn(c_m, std=0.1),
                      w_q=rn(c_m, hd, std=c_m ** -0.5), w_k=rn(c_m, hd, std=c_m ** -0.5),
                      w_v=rn(c_m, hd, std=c_m ** -0.5), w_g=rn(c_m, hd, std=c_m ** -0.5),
                      b_g=1.0 + rn(hd, std=0.1), w_o=rn(hd, c_m, std=hd ** -0.5),
                      b_o=rn(c_m, std=0.1), heads=heads)
    if c_z is not None:
        p.gamma_z, p.beta_z = 1.0 + rn(c_z, std=0.1), rn(c_z, std=0.1)
        p.w_b = rn(c_z, heads, std=c_z ** -0.5)
    return p


def _gated_over_second_axis(x, p, bias, kmask, dtype):
    """Gated attention along the second axis of x [A, B, C] (batch = first axis)."""
    a, b, c = x.shape
    w = {n: t.to(dtype) for n, t in p.named()}
    hd = w["w_q"].shape[1]
    d = hd // p.heads

    def heads_first(t):
        return t.view(a, b, p.heads, d).permute(0, 2, 1, 3)

    q, k, v = (heads_first(x @ w[n]) for n in ("w_q", "w_k", "w_v"))
    o, _ = attention_fwd(q, k, v, bias, kmask, 1.0 / math.sqrt(d), dtype)
    o = o.permute(0, 2, 1, 3).reshape(a, b, hd)
    gate = torch.sigmoid(x @ w["w_g"] + w["b_g"])
    return (gate * o) @ w["w_o"] + w["b_o"]


def _ln3(t, gamma, beta, eps, dtype):
    a, b, c = t.shape
    return layer_norm_fwd(t.reshape(a * b, c), gamma.to(dtype), beta.to(dtype), eps,
                          dtype)[0].view(a, b, c)


def msa_row_attention(m, z, mask, p, dtype=torch.float64):
    """Algorithm 7: attention along the residues of each MSA row s, bias from LayerNorm(z).
    m [S, R, C_m], z [R, R, C_z], mask [S, R]."""
    x = _ln3(m, p.gamma, p.beta, p.eps, dtype)
    zn = _ln3(z, p.gamma_z, p.beta_z, p.eps, dtype)
    bias = (zn @ p.w_b.to(dtype)).permute(2, 0, 1)        # [H, R(query), R(key)]
    return _gated_over_second_axis(x, p, bias, mask.to(torch.uint8), dtype)


def msa_column_attention(m, mask, p, dtype=torch.float64):
    """Algorithm 8: attention along the sequences of each MSA column r, no pair bias."""
    s = m.shape[0]
    x = _ln3(m, p.gamma, p.beta, p.eps, dtype).transpose(0, 1)      # [R, S, C]
    bias = torch.zeros(p.heads, s, s, dtype=dtype)
    out = _gated_over_second_axis(x.contiguous(), p, bias, mask.t().to(torch.uint8), dtype)
    return out.transpose(0, 1)


def msa_attention_literal(m, mask, p, z=None, column=False):
    """Index-by-index float64 evaluation of Algorithm 7 (z given) or 8 (column=True)."""
    m = m.double()
    w = {n: t.double() for n, t in p.named()}

    def ln(t, gamma, beta):
        mu = t.mean(-1, keepdim=True)
        return (t - mu) / torch.sqrt(((t - mu) ** 2).mean(-1, keepdim=True) + p.eps) * gamma + beta

    x = ln(m, w["gamma"], w["beta"])
    s, r, _ = x.shape
    h = p.heads
    d = w["w_q"].shape[1] // h
    q, k, v = ((x @ w[n]).view(s, r, h, d) for n in ("w_q", "w_k", "w_v"))
    keep = mask != 0
    if not column:
        b = ln(z.double(), w["gamma_z"], w["beta_z"]) @ w["w_b"]        # [R, R, H]
        # a_sij = q_si . k_sj / sqrt(d) + b_ij over residues j of row s
        logit = torch.einsum("sihd,sjhd->sijh", q, k) / math.sqrt(d) + b[None]
        logit = torch.where(keep[:, None, :, None], logit, torch.full_like(logit, -1e4))
        o = torch.einsum("sijh,sjhd->sihd", torch.softmax(logit, dim=2), v)
    else:
        # a_sti = q_si . k_ti / sqrt(d) over sequences t of column i
        logit = torch.einsum("sihd,tihd->sith", q, k) / math.sqrt(d)
        logit = torch.where(keep.t()[None, :, :, None], logit, torch.full_like(logit, -1e4))
        o = torch.einsum("sith,tihd->sihd", torch.softmax(logit, dim=2), v)
    gate = torch.sigmoid(x @ w["w_g"] + w["b_g"])
    return (gate * o.reshape(s, r, h * d)) @ w["w_o"] + w["b_o"]
