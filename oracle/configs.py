"""Seeded synthetic inputs for the benchmark configurations (BASELINE.json "configs").

No protein data is needed or used: every tensor is drawn from a seeded generator with the shapes
and distributions the configurations name.  Generation runs on any torch device (the bench draws
its full-size inputs on the GPU; the tests draw small ones on the CPU); fp32 draws are rounded
once to the 16-bit storage type.

C1  CPU triangle-attention module check, N_res=128            (seed 0)
C2  MSA row attention fwd+bwd [512 x 256], H=8, d=32           (seed 1)
C3  triangle attention (starting node) fwd+bwd, N_res=768      (seed 2)
C4  LayerNorm + gated dual projection fwd+bwd, z [1024,1024,128] (seed 3)
C5  triangle attention fwd only, N_res=2048                    (seed 4)
"""

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class AttnConfig:
    name: str
    n: int          # attention batch (MSA sequences, or pair rows for triangle attention)
    h: int
    s: int          # Sq == Sk
    d: int
    seed: int
    backward: bool
    mask: str       # "msa": 25% of rows lose their last ~10% keys; "tri": 5% residues padded;
                    # "none": all ones
    from_pair: bool  # q/k/v/bias are projections of LN(z) (triangle attention); else N(0,1)


C2 = AttnConfig("msa_row_512x256", 512, 8, 256, 32, 1, True, "msa", False)
C3 = AttnConfig("tri_start_768", 768, 4, 768, 32, 2, True, "tri", True)
C5 = AttnConfig("tri_start_2048_fwd", 2048, 4, 2048, 32, 4, False, "none", True)
ATTN_CONFIGS = {c.name: c for c in (C2, C3, C5)}


def scaled(cfg, n=None, s=None):
    """The same configuration with a smaller batch and/or sequence (for tests and CPU samples)."""
    return AttnConfig(cfg.name + "_small", n or cfg.n, cfg.h, s or cfg.s, cfg.d, cfg.seed,
                      cfg.backward, cfg.mask, cfg.from_pair)


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, g, device, std=1.0):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


def _ln(z, gamma, beta, eps=1e-5):
    mean = z.mean(dim=-1, keepdim=True)
    var = ((z - mean) ** 2).mean(dim=-1, keepdim=True)
    return (z - mean) * torch.rsqrt(var + eps) * gamma + beta


def make_kmask(cfg, g, device):
    n, s = cfg.n, cfg.s
    kmask = torch.ones(n, s, dtype=torch.uint8, device=device)
    if cfg.mask == "msa":
        rows = torch.rand(n, generator=g, device=device) < 0.25
        cut = s - max(1, int(round(0.1 * s)))
        kmask[rows, cut:] = 0
    elif cfg.mask == "tri":
        padded = torch.rand(s, generator=g, device=device) < 0.05
        kmask[:, padded] = 0
        rows = padded if n == s else torch.rand(n, generator=g, device=device) < 0.05
        kmask[rows, :] = 0
    return kmask


def make_attention_inputs(cfg, device="cpu", dtype=torch.bfloat16, chunk=64):
    """Returns dict q,k,v,bias,kmask,dout,scale for an AttnConfig.

    Layout is the FFI layout [N,H,S,D] for q/k/v/dout, bias [H,S,S], kmask uint8 [N,S].
    For `from_pair` configs the tensors are projections of LN(z), z ~ N(0,1) [n, s, 128], with
    N(0, 1/128) weights and gamma ~ 1 + 0.1 N(0,1), beta ~ 0.1 N(0,1), eps 1e-5, as in the
    triangle attention module; z is generated in row chunks to bound memory.
    """
    g = _gen(cfg.seed, device)
    n, h, s, d = cfg.n, cfg.h, cfg.s, cfg.d
    c_z = 128
    if cfg.from_pair:
        gamma = 1.0 + 0.1 * _randn((c_z,), g, device)
        beta = 0.1 * _randn((c_z,), g, device)
        w_qkv = _randn((c_z, 3 * h * d), g, device, 1.0 / math.sqrt(c_z))
        w_b = _randn((c_z, h), g, device, 1.0 / math.sqrt(c_z))
        q = torch.empty((n, h, s, d), dtype=dtype, device=device)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        bias32 = torch.empty((s, s, h), dtype=torch.float32, device=device) if n == s else None
        for r0 in range(0, n, chunk):
            r1 = min(n, r0 + chunk)
            z = _randn((r1 - r0, s, c_z), g, device)
            x = _ln(z, gamma, beta)
            qkv = (x @ w_qkv).view(r1 - r0, s, 3, h, d).permute(2, 0, 3, 1, 4)
            q[r0:r1], k[r0:r1], v[r0:r1] = qkv[0].to(dtype), qkv[1].to(dtype), qkv[2].to(dtype)
            if bias32 is not None:
                bias32[r0:r1] = x @ w_b
        if bias32 is None:
            zb = _randn((s, s, c_z), g, device)
            bias32 = _ln(zb, gamma, beta) @ w_b
        bias = bias32.permute(2, 0, 1).contiguous().to(dtype)
    else:
        q = _randn((n, h, s, d), g, device).to(dtype)
        k = _randn((n, h, s, d), g, device).to(dtype)
        v = _randn((n, h, s, d), g, device).to(dtype)
        bias = _randn((h, s, s), g, device).to(dtype)
    kmask = make_kmask(cfg, g, device)
    dout = _randn((n, h, s, d), g, device).to(dtype) if cfg.backward else None
    return dict(q=q, k=k, v=v, bias=bias, kmask=kmask, dout=dout, scale=1.0 / math.sqrt(d))


@dataclass(frozen=True)
class LnGdpConfig:
    name: str
    m: int
    c: int
    n_out: int
    seed: int


C4 = LnGdpConfig("ln_gdp_1024x1024x128", 1024 * 1024, 128, 256, 3)


def make_ln_gdp_inputs(cfg, device="cpu", dtype=torch.bfloat16):
    """z [M,C] ~ N(0,1); gamma/beta; four N(0,1/C) [C,C] weights packed as wp=[Wp_a|Wp_b],
    wg=[Wg_a|Wg_b] ([C, 2C]); bp=bg=0; mask=1; dA,dB ~ N(0,1) packed as dout [M, 2C];
    dy ~ N(0,1) [M,C] for the LayerNorm backward."""
    g = _gen(cfg.seed, device)
    m, c, n = cfg.m, cfg.c, cfg.n_out
    x = _randn((m, c), g, device).to(dtype)
    gamma = 1.0 + 0.1 * _randn((c,), g, device)
    beta = 0.1 * _randn((c,), g, device)
    wp = _randn((c, n), g, device, 1.0 / math.sqrt(c)).to(dtype)
    wg = _randn((c, n), g, device, 1.0 / math.sqrt(c)).to(dtype)
    bp = torch.zeros(n, device=device, dtype=dtype)
    bg = torch.zeros(n, device=device, dtype=dtype)
    mask = torch.ones(m, device=device, dtype=dtype)
    dout = _randn((m, n), g, device).to(dtype)
    dy = _randn((m, c), g, device).to(dtype)
    return dict(x=x, gamma=gamma, beta=beta, eps=1e-5, wp=wp, wg=wg, bp=bp, bg=bg, mask=mask,
                dout=dout, dy=dy)
