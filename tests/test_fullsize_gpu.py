"""GPU parity at the benchmark configurations' full sizes (C2, C3, C4) against the CPU oracle.

The kernels run on the whole workload, exactly as bench.py runs it (same seeded generators, on
the device).  The oracle then checks:

* per-row outputs (out, lse, dq, dk, dv; LayerNorm y and dx; GDP out and dx) on a sample of
  rows that includes the edge rows (the first and last tiles, fully masked attention rows, rows
  with masked keys) in float64;
* every reduction over the batch/row axis on ALL rows: attention dbias (sums of dS over all 768
  or 512 attention rows; float32 oracle chunks added in float64), LayerNorm dgamma/dbeta and
  the GDP weight and bias gradients over all 1,048,576 rows (float64).

Tolerances (north_star): 16-bit outputs rtol = atol = 2e-2; f32 outputs 1e-4 of the tensor's
max magnitude plus 1e-4 relative.
"""

import pytest
import torch

import oracle
from conftest import assert_close_bf16, assert_close_f32

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _sample_rows(kmask, count=16, seed=0):
    """Row indices to check: first and last rows, up to 4 fully masked rows, up to 4 rows with
    some masked keys, the rest random."""
    n = kmask.shape[0]
    km = kmask.cpu()
    full = (km == 0).all(dim=1).nonzero().flatten().tolist()
    part = ((km == 0).any(dim=1) & (km != 0).any(dim=1)).nonzero().flatten().tolist()
    rows = {0, 1, n - 2, n - 1}
    rows.update(full[:4])
    rows.update(part[:4])
    g = torch.Generator().manual_seed(seed)
    for r in torch.randperm(n, generator=g).tolist():
        if len(rows) >= count:
            break
        rows.add(r)
    return sorted(rows)


def _attention_full(cfg, what):
    from colabfold_legacy_kernels import torch_ops, cabi
    dev = torch.device("cuda", 0)
    inp = oracle.configs.make_attention_inputs(cfg, device=dev)
    q, k, v, bias, kmask, dout = (inp[x] for x in ("q", "k", "v", "bias", "kmask", "dout"))
    scale = inp["scale"]
    cabi.clear_device_status()
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, scale)
    dq, dk, dv, dbias = torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale)
    torch.cuda.synchronize()
    assert cabi.device_status() == 0

    c = {x: t.cpu() for x, t in (("q", q), ("k", k), ("v", v), ("bias", bias), ("kmask", kmask),
                                 ("dout", dout), ("out", out), ("lse", lse))}
    rows = _sample_rows(c["kmask"])
    sel = torch.tensor(rows)
    r_out, r_lse = oracle.attention_fwd(c["q"][sel], c["k"][sel], c["v"][sel], c["bias"],
                                        c["kmask"][sel], scale)
    assert_close_bf16(out.cpu()[sel], r_out, what + " out (sampled rows)")
    assert_close_f32(lse.cpu()[sel], r_lse, what + " lse (sampled rows)")
    r = oracle.attention_bwd(c["q"][sel], c["k"][sel], c["v"][sel], c["bias"], c["kmask"][sel],
                             c["out"][sel], c["lse"][sel], c["dout"][sel], scale)
    assert_close_bf16(dq.cpu()[sel], r[0], what + " dq (sampled rows)")
    assert_close_bf16(dk.cpu()[sel], r[1], what + " dk (sampled rows)")
    assert_close_bf16(dv.cpu()[sel], r[2], what + " dv (sampled rows)")

    # dbias sums dS over every attention row: all rows through the oracle, in chunks
    n = q.shape[0]
    acc = torch.zeros(dbias.shape, dtype=torch.float64)
    chunk = 8
    for r0 in range(0, n, chunk):
        s = slice(r0, r0 + chunk)
        part = oracle.attention_bwd(c["q"][s], c["k"][s], c["v"][s], c["bias"], c["kmask"][s],
                                    c["out"][s], c["lse"][s], c["dout"][s], scale,
                                    dtype=torch.float32)[3]
        acc += part.double()
    assert_close_f32(dbias, acc, what + " dbias (all %d rows)" % n)


def test_c3_triangle_768_full(cuda_device):
    """C3: 768 rows x H=4 x S=768 x d=32 with 5 % padded residues (fully masked rows included);
    the forward takes its three-rows-per-item path and the backward one item per (head, query
    tile, key tile) walking all 768 rows (dbias in registers, written once)."""
    _attention_full(oracle.configs.C3, "C3")


def test_c2_msa_row_512_full(cuda_device):
    """C2: 512 rows x H=8 x S=256 x d=32, a quarter of the rows with their last 10 % of keys
    masked; the backward splits the rows into batch chunks whose dbias are added."""
    _attention_full(oracle.configs.C2, "C2")


def test_c4_layer_norm_full(cuda_device):
    """C4: LayerNorm forward and backward on 1,048,576 x 128 rows."""
    from colabfold_legacy_kernels import torch_ops
    dev = torch.device("cuda", 0)
    inp = oracle.configs.make_ln_gdp_inputs(oracle.configs.C4, device=dev)
    x, gamma, beta, dy, eps = inp["x"], inp["gamma"], inp["beta"], inp["dy"], inp["eps"]
    y, mean, rstd = torch_ops.layer_norm_fwd(x, gamma, beta, eps, return_stats=True)
    dx, dg, db = torch_ops.layer_norm_bwd(x, gamma, dy, eps, mean=mean, rstd=rstd)
    torch.cuda.synchronize()
    m = x.shape[0]
    xc, dyc, gc, bc = x.cpu(), dy.cpu(), gamma.cpu(), beta.cpu()
    sel = torch.cat([torch.arange(0, 256), torch.arange(m - 256, m),
                     torch.randperm(m, generator=torch.Generator().manual_seed(1))[:3584]])
    ry, _, _ = oracle.layer_norm_fwd(xc[sel], gc, bc, eps)
    assert_close_bf16(y.cpu()[sel], ry, "C4 LayerNorm y (sampled rows)")
    rdx, _, _ = oracle.layer_norm_bwd(xc[sel], gc, dyc[sel], eps)
    assert_close_bf16(dx.cpu()[sel], rdx, "C4 LayerNorm dx (sampled rows)")
    # statistics of every row, and dgamma / dbeta summed over every row
    rmean = torch.empty(m, dtype=torch.float64)
    rrstd = torch.empty(m, dtype=torch.float64)
    rdg = torch.zeros(x.shape[1], dtype=torch.float64)
    rdb = torch.zeros(x.shape[1], dtype=torch.float64)
    for r0 in range(0, m, 1 << 16):
        s = slice(r0, r0 + (1 << 16))
        _, mu, rs = oracle.layer_norm_fwd(xc[s], gc, bc, eps)
        rmean[s], rrstd[s] = mu, rs
        _, a, b = oracle.layer_norm_bwd(xc[s], gc, dyc[s], eps, mean=mu, rstd=rs)
        rdg += a
        rdb += b
    assert_close_f32(mean, rmean, "C4 LayerNorm mean (all rows)")
    assert_close_f32(rstd, rrstd, "C4 LayerNorm rstd (all rows)")
    assert_close_f32(dg, rdg, "C4 LayerNorm dgamma (all rows)")
    assert_close_f32(db, rdb, "C4 LayerNorm dbeta (all rows)")


def test_c4_gdp_full(cuda_device):
    """C4: gated dual projection forward and backward on 1,048,576 rows, K = 128, N = 256."""
    from colabfold_legacy_kernels import torch_ops
    dev = torch.device("cuda", 0)
    inp = oracle.configs.make_ln_gdp_inputs(oracle.configs.C4, device=dev)
    names = ("x", "wp", "bp", "wg", "bg", "mask")
    args = [inp[k] for k in names]
    out = torch_ops.gdp_fwd(*args)
    dx, dwp, dbp, dwg, dbg = torch_ops.gdp_bwd(*args, inp["dout"])
    torch.cuda.synchronize()
    cpu = [a.cpu() for a in args]
    doc = inp["dout"].cpu()
    m = cpu[0].shape[0]
    sel = torch.cat([torch.arange(0, 256), torch.arange(m - 256, m),
                     torch.randperm(m, generator=torch.Generator().manual_seed(2))[:3584]])
    rows = [cpu[0][sel]] + cpu[1:5] + [cpu[5][sel]]
    assert_close_bf16(out.cpu()[sel], oracle.gdp_fwd(*rows), "C4 GDP out (sampled rows)")
    assert_close_bf16(dx.cpu()[sel], oracle.gdp_bwd(*rows, doc[sel])[0],
                      "C4 GDP dx (sampled rows)")
    acc = [torch.zeros(t.shape, dtype=torch.float64) for t in (dwp, dbp, dwg, dbg)]
    for r0 in range(0, m, 1 << 16):
        s = slice(r0, r0 + (1 << 16))
        r = oracle.gdp_bwd(cpu[0][s], *cpu[1:5], cpu[5][s], doc[s])
        for a, b in zip(acc, r[1:]):
            a += b
    for got, exp, name in zip((dwp, dbp, dwg, dbg), acc, ("dwp", "dbp", "dwg", "dbg")):
        assert_close_f32(got, exp, "C4 GDP %s (all rows)" % name)


def test_c4_ln_gdp_fused_full(cuda_device):
    """C4: the LayerNorm-fused GDP forward (cfk_ln_gdp_fwd) on 1,048,576 rows against the
    oracle's LayerNorm then GDP (sampled rows) and its row statistics (every row)."""
    from colabfold_legacy_kernels import torch_ops
    dev = torch.device("cuda", 0)
    inp = oracle.configs.make_ln_gdp_inputs(oracle.configs.C4, device=dev)
    z, gamma, beta, eps = inp["x"], inp["gamma"], inp["beta"], inp["eps"]
    w = [inp[k] for k in ("wp", "bp", "wg", "bg", "mask")]
    out, mean, rstd = torch_ops.ln_gdp_fwd(z, gamma, beta, eps, *w, return_stats=True)
    torch.cuda.synchronize()
    m = z.shape[0]
    zc, gc, bc = z.cpu(), gamma.cpu(), beta.cpu()
    wc = [t.cpu() for t in w]
    sel = torch.cat([torch.arange(0, 256), torch.arange(m - 256, m),
                     torch.randperm(m, generator=torch.Generator().manual_seed(4))[:3584]])
    x, _, _ = oracle.layer_norm_fwd(zc[sel], gc, bc, eps)
    ref = oracle.gdp_fwd(x.to(z.dtype), *wc[:4], wc[4][sel])
    assert_close_bf16(out.cpu()[sel], ref, "C4 LN+GDP out (sampled rows)")
    rmean = torch.empty(m, dtype=torch.float64)
    rrstd = torch.empty(m, dtype=torch.float64)
    for r0 in range(0, m, 1 << 16):
        s = slice(r0, r0 + (1 << 16))
        _, rmean[s], rrstd[s] = oracle.layer_norm_fwd(zc[s], gc, bc, eps)
    assert_close_f32(mean, rmean, "C4 LN+GDP mean (all rows)")
    assert_close_f32(rstd, rrstd, "C4 LN+GDP rstd (all rows)")


def test_module_scale_projections_full(cuda_device):
    """The triangle module's projections at C3 size (589,824 rows of C = 128): q|k|v and the
    gate from one cfk_linear_fwd, dx over the three gradient blocks (dq|dk|dv, dg, the padded
    bias rows) and their weight/bias gradients, against a plain PyTorch fp32 reference of the
    same products (sampled rows for y and dx, every row for dw and db)."""
    from colabfold_legacy_kernels import torch_ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(6)
    m, c = 768 * 768, 128
    bf = torch.bfloat16
    x = torch.randn(m, c, device=dev, generator=g).to(bf)
    w = (torch.randn(c, 512, device=dev, generator=g) * c ** -0.5).to(bf)
    b = torch.cat([torch.zeros(384, device=dev), torch.randn(128, device=dev, generator=g)]).to(bf)
    qkv = torch.empty(m, 384, dtype=bf, device=dev)
    gate = torch.empty(m, 128, dtype=bf, device=dev)
    torch_ops.linear_fwd(x, w, b, out=(qkv, gate))
    dys = [torch.randn(m, n, device=dev, generator=g).to(bf) for n in (384, 128, 16)]
    ws = [w[:, :384].contiguous(), w[:, 384:].contiguous(),
          (torch.randn(c, 16, device=dev, generator=g) * c ** -0.5).to(bf)]
    dx = torch_ops.linear_bwd_dx(dys, ws)
    grads = torch_ops.linear_bwd_dw(x, dys, [False, True, False])
    torch.cuda.synchronize()
    sel = torch.cat([torch.arange(0, 256), torch.arange(m - 256, m),
                     torch.randperm(m, generator=torch.Generator().manual_seed(5))[:3584]]).to(dev)
    xf = x.float()
    ref_y = xf[sel] @ w.float() + b.float()
    assert_close_bf16(torch.cat([qkv[sel], gate[sel]], 1), ref_y, "projection y (sampled rows)")
    ref_dx = sum(dy[sel].float() @ wt.float().t() for dy, wt in zip(dys, ws))
    assert_close_bf16(dx[sel], ref_dx, "projection dx (sampled rows)")
    for (dw, db), dy, name in zip(grads, dys, ("qkv", "g", "bias")):
        assert_close_f32(dw, xf.t() @ dy.float(), "dw %s (all rows)" % name)
        if db is not None:
            assert_close_f32(db, dy.float().sum(0), "db %s (all rows)" % name)
