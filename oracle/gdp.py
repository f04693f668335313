"""Gated dual projection -- CPU restatement (test oracle).

Forward after volta_gdp_kernel (cuda/volta_ops.cu:185-207, twin cuda/volta_gdp_wmma.cu:84-94):
  p = x @ wp + bp,  g = x @ wg + bg,  out = mask[:, None] * p * sigmoid(g).
Both products contract over K with f32 accumulation in the reference (:143-183).

Backward (the reference has none), mask treated as a constant:
  s = sigmoid(g), dp = dout * mask * s, dg = dout * mask * p * s * (1 - s),
  dx = dp @ wp^T + dg @ wg^T, dwp = x^T @ dp, dwg = x^T @ dg, dbp = sum_m dp, dbg = sum_m dg.
"""

import torch


def gdp_fwd(x, wp, bp, wg, bg, mask, dtype=torch.float64):
    x, wp, bp, wg, bg, mask = (t.to(dtype) for t in (x, wp, bp, wg, bg, mask))
    p = x @ wp + bp
    g = x @ wg + bg
    return mask[:, None] * p * torch.sigmoid(g)


def gdp_bwd(x, wp, bp, wg, bg, mask, dout, dtype=torch.float64):
    """Returns (dx, dwp, dbp, dwg, dbg) in `dtype`."""
    x, wp, bp, wg, bg, mask, dout = (t.to(dtype) for t in (x, wp, bp, wg, bg, mask, dout))
    p = x @ wp + bp
    s = torch.sigmoid(x @ wg + bg)
    dm = dout * mask[:, None]
    dp = dm * s
    dg = dm * p * s * (1 - s)
    dx = dp @ wp.T + dg @ wg.T
    return dx, x.T @ dp, dp.sum(dim=0), x.T @ dg, dg.sum(dim=0)


def flops_fwd(m, k, n):
    return 2 * 2 * m * k * n


def flops_bwd(m, k, n):
    """dx (two products) and dwp, dwg; the recomputation of p and g is not counted."""
    return 4 * 2 * m * k * n


def bytes_fwd(m, k, n, elem=2):
    return (m * k + m * n + 2 * k * n) * elem


def bytes_bwd(m, k, n, elem=2):
    return (2 * m * k + m * n + 2 * k * n) * elem
