"""Attention with an additive pair bias and a key mask -- CPU restatement (test oracle).

Forward, after cuda/volta_mma_attn.cu (VoltaMma), lines cited per step:

  logit[n,h,i,j] = scale * <q[n,h,i], k[n,h,j]> + bias[h,i,j]      (:189-190; the scale applies
                                                                   to q.k only, bias unscaled)
                 = -1e4                      if kmask[n,j] == 0    (:186-188; the masked logit
                                                                   is REPLACED, bias dropped)
  out[n,h,i]     = sum_j softmax_j(logit[n,h,i,:]) v[n,h,j]        (:198-253, online base-2
                                                                   softmax; normalised by
                                                                   1/max(l, 1e-30) at :265)

The reference also gives -1e4 to the padding columns of its last key tile, j in
[Sk, ceil(Sk/block_k)*block_k), with zero V rows (:144-146,186).  This only changes rows whose
keys are all masked (they then average over more "keys" than exist).  The default here is the
mathematical definition (softmax over the Sk real keys), which the B200 kernels implement;
`ref_block_k=` reproduces the reference quirk for pinning against its own outputs.

Backward (the reference has none): the exact derivative of the forward.  Masked logits are
constants, so their dlogit is zero; the softmax weights of masked keys (nonzero only in rows
whose keys are all masked) still carry gradient to v.

  P = exp(logit - lse),  dV = P^T dO,  dP = dO V^T,  delta_i = sum_d dO[i,d] O[i,d],
  dS = P * (dP - delta) (0 where masked),  dQ = scale dS K,  dK = scale dS^T Q,
  dbias[h,i,j] = sum_n dS[n,h,i,j].
"""

import math

import torch

MASKED_LOGIT = -1.0e4  # cuda/volta_mma_attn.cu:25


def _as(t, dtype):
    return t.to(dtype) if t.dtype != dtype else t


def attention_logits(q, k, bias, kmask, scale, dtype=torch.float64):
    """Logits [N,H,Sq,Sk] with the reference's replacement of masked keys."""
    q, k, bias = _as(q, dtype), _as(k, dtype), _as(bias, dtype)
    s = torch.einsum("nhid,nhjd->nhij", q, k) * scale + bias.unsqueeze(0)
    keep = (kmask != 0)[:, None, None, :]
    return torch.where(keep, s, torch.full_like(s, MASKED_LOGIT)), keep


def attention_fwd(q, k, v, bias, kmask, scale, dtype=torch.float64, ref_block_k=None):
    """Returns (out [N,H,Sq,D], lse [N,H,Sq]) in `dtype` (lse in natural-log units).

    q,k,v: [N,H,S,D]; bias: [H,Sq,Sk]; kmask: uint8 [N,Sk].
    """
    logits, _ = attention_logits(q, k, bias, kmask, scale, dtype)
    v = _as(v, dtype)
    if ref_block_k:
        sk = logits.shape[-1]
        pad = (-sk) % int(ref_block_k)
        if pad:
            logits = torch.cat([logits, torch.full(logits.shape[:-1] + (pad,), MASKED_LOGIT,
                                                   dtype=dtype)], dim=-1)
            v = torch.cat([v, torch.zeros(v.shape[:2] + (pad,) + v.shape[3:], dtype=dtype)],
                          dim=2)
    m = logits.amax(dim=-1, keepdim=True)
    p = torch.exp(logits - m)
    l = p.sum(dim=-1, keepdim=True)
    out = torch.einsum("nhij,nhjd->nhid", p, v) / l.clamp_min(1e-30)
    lse = (m + torch.log(l)).squeeze(-1)
    return out, lse


def attention_fwd_chunked(q, k, v, bias, kmask, scale, dtype=torch.float32, chunk=16):
    """attention_fwd over batch rows in chunks (bounds the [chunk,H,Sq,Sk] score memory)."""
    outs, lses = [], []
    for n0 in range(0, q.shape[0], chunk):
        sl = slice(n0, n0 + chunk)
        o, l = attention_fwd(q[sl], k[sl], v[sl], bias, kmask[sl], scale, dtype=dtype)
        outs.append(o)
        lses.append(l)
    return torch.cat(outs), torch.cat(lses)


def attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale, dtype=torch.float64):
    """Returns (dq, dk, dv, dbias) in `dtype`.

    `out` and `lse` are the forward's outputs as the kernel produced them (the backward is a
    function of them, so the oracle takes them as inputs just as the kernel does).
    """
    q, k, v = _as(q, dtype), _as(k, dtype), _as(v, dtype)
    out, lse, dout = _as(out, dtype), _as(lse, dtype), _as(dout, dtype)
    logits, keep = attention_logits(q, k, bias, kmask, scale, dtype)
    p = torch.exp(logits - lse.unsqueeze(-1))
    dv = torch.einsum("nhij,nhid->nhjd", p, dout)
    dp = torch.einsum("nhid,nhjd->nhij", dout, v)
    delta = (dout * out).sum(dim=-1, keepdim=True)
    ds = p * (dp - delta)
    ds = torch.where(keep, ds, torch.zeros_like(ds))
    dq = torch.einsum("nhij,nhjd->nhid", ds, k) * scale
    dk = torch.einsum("nhij,nhid->nhjd", ds, q) * scale
    dbias = ds.sum(dim=0)
    return dq, dk, dv, dbias


def flops_fwd(n, h, sq, sk, d):
    """Algorithmic forward FLOPs: QK^T and PV, 2 flops per multiply-add."""
    return 4 * n * h * sq * sk * d


def flops_bwd(n, h, sq, sk, d):
    """Algorithmic backward FLOPs: dV, dP, dQ, dK (the recomputation of S is not counted)."""
    return 8 * n * h * sq * sk * d


def default_scale(d):
    return 1.0 / math.sqrt(d)
