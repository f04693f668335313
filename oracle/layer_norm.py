"""LayerNorm over the last axis -- CPU restatement (test oracle).

Forward after volta_layer_norm_kernel (cuda/volta_ops.cu:40-58):
  mean = sum(x)/C, var = max(E[x^2] - mean^2, 0) (:51-53), rstd = 1/sqrt(var + eps) (:54),
  y = (x - mean) * rstd * gamma + beta (:55-57).
In float64 the reference's E[x^2] - mean^2 and the two-pass mean((x-mean)^2) agree to ~1e-15,
so one formula (`two_pass`) serves both; `two_pass=False` evaluates the reference's literally.

Backward (the reference has none): with xhat = (x - mean) * rstd and g = dy * gamma,
  dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  dgamma = sum_rows dy * xhat,
  dbeta = sum_rows dy.
"""

import torch


def layer_norm_fwd(x, gamma, beta, eps, dtype=torch.float64, two_pass=True):
    """Returns (y, mean, rstd) in `dtype`; x [M,C], gamma/beta [C]."""
    x = x.to(dtype)
    mean = x.mean(dim=-1)
    if two_pass:
        var = ((x - mean[:, None]) ** 2).mean(dim=-1)
    else:
        var = ((x * x).mean(dim=-1) - mean * mean).clamp_min(0.0)
    rstd = torch.rsqrt(var + eps)
    y = (x - mean[:, None]) * rstd[:, None] * gamma.to(dtype) + beta.to(dtype)
    return y, mean, rstd


def layer_norm_bwd(x, gamma, dy, eps, mean=None, rstd=None, dtype=torch.float64):
    """Returns (dx, dgamma, dbeta) in `dtype`."""
    x, dy, gamma = x.to(dtype), dy.to(dtype), gamma.to(dtype)
    if mean is None or rstd is None:
        _, mean, rstd = layer_norm_fwd(x, gamma, torch.zeros_like(gamma), eps, dtype)
    mean, rstd = mean.to(dtype), rstd.to(dtype)
    xhat = (x - mean[:, None]) * rstd[:, None]
    g = dy * gamma
    dx = rstd[:, None] * (g - g.mean(dim=-1, keepdim=True)
                          - xhat * (g * xhat).mean(dim=-1, keepdim=True))
    return dx, (dy * xhat).sum(dim=0), dy.sum(dim=0)


def bytes_fwd(m, c, elem=2):
    """Algorithmic HBM bytes of the forward: read x, write y."""
    return 2 * m * c * elem


def bytes_bwd(m, c, elem=2):
    """Algorithmic HBM bytes of the backward: read x and dy, write dx, read mean and rstd."""
    return 3 * m * c * elem + 2 * m * 4
