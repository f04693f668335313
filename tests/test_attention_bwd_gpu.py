"""GPU parity of the attention backward (cfk_attn_bwd through the C ABI) against the CPU oracle.

The backward is a function of the forward's out and lse, so the oracle receives the kernel's
own out and lse and evaluates the exact derivative in float64.
Tolerances: dq, dk, dv (16-bit) rtol = atol = 2e-2; dbias (f32) 1e-4 of max|dbias| plus 1e-4
relative.
"""

import math

import pytest
import torch

import oracle
from conftest import assert_close_bf16, assert_close_f32

pytestmark = pytest.mark.gpu


def _inputs(n, h, sq, sk, d, dtype, seed, mask_mode="random"):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, h, sq, d, generator=g).to(dtype)
    k = torch.randn(n, h, sk, d, generator=g).to(dtype)
    v = torch.randn(n, h, sk, d, generator=g).to(dtype)
    bias = torch.randn(h, sq, sk, generator=g).to(dtype)
    dout = torch.randn(n, h, sq, d, generator=g).to(dtype)
    kmask = torch.ones(n, sk, dtype=torch.uint8)
    if mask_mode == "random":
        kmask = (torch.rand(n, sk, generator=g) > 0.2).to(torch.uint8)
        if n > 1:
            kmask[1] = 0
    return [t.cuda() for t in (q, k, v, bias, kmask, dout)]


def _check(q, k, v, bias, kmask, dout, scale, what):
    from colabfold_legacy_kernels import torch_ops
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, scale)
    dq, dk, dv, dbias = torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale)
    torch.cuda.synchronize()
    r = oracle.attention_bwd(q.cpu(), k.cpu(), v.cpu(), bias.cpu(), kmask.cpu(), out.cpu(),
                             lse.cpu(), dout.cpu(), scale)
    assert_close_bf16(dq, r[0], what + " dq")
    assert_close_bf16(dk, r[1], what + " dk")
    assert_close_bf16(dv, r[2], what + " dv")
    assert_close_f32(dbias, r[3], what + " dbias")
    return dq, dk, dv, dbias


@pytest.mark.parametrize("d", [8, 16, 32, 64])
def test_bwd_head_dims_ragged(cuda_device, d):
    t = _inputs(3, 2, 130, 200, d, torch.bfloat16, seed=100 + d)
    _check(*t, 1.0 / math.sqrt(d), "d=%d" % d)


def test_bwd_fp16(cuda_device):
    t = _inputs(4, 2, 256, 128, 32, torch.float16, seed=7)
    _check(*t, 1.0 / math.sqrt(32), "fp16")


def test_bwd_unaligned_key_count(cuda_device):
    t = _inputs(2, 3, 70, 77, 32, torch.bfloat16, seed=8)
    _check(*t, 0.2, "Sk=77")


def test_bwd_msa_shape_batch_chunks(cuda_device):
    # few (query, key) tiles: the batch rows are split into chunks whose dbias add up
    cfg = oracle.configs.scaled(oracle.configs.C2, n=24)
    inp = oracle.configs.make_attention_inputs(cfg)
    t = [inp[k].cuda() for k in ("q", "k", "v", "bias", "kmask", "dout")]
    _check(*t, inp["scale"], "msa")


def test_bwd_triangle_shape_deterministic_dbias(cuda_device):
    from colabfold_legacy_kernels import torch_ops, cabi
    cfg = oracle.configs.scaled(oracle.configs.C3, n=12, s=384)
    inp = oracle.configs.make_attention_inputs(cfg)
    t = [inp[k].cuda() for k in ("q", "k", "v", "bias", "kmask", "dout")]
    cabi.clear_device_status()
    _, _, _, db1 = _check(*t, inp["scale"], "triangle")
    q, k, v, bias, kmask, dout = t
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, inp["scale"])
    _, _, _, db2 = torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, inp["scale"])
    torch.cuda.synchronize()
    # 4 heads x 3 x 3 tiles = 36 items < SM count -> batch chunks; their partial dbias tiles
    # are added in a fixed order, so two runs agree bit for bit
    assert torch.equal(db1, db2)
    assert cabi.device_status() == 0


def test_bwd_select_path(cuda_device):
    t = _inputs(2, 1, 40, 130, 16, torch.bfloat16, seed=12, mask_mode="none")
    t[3] = torch.full_like(t[3], -30000.0)
    t[4][:, 5] = 0
    t[4][:, 129] = 0
    _check(*t, 0.25, "select path")


@pytest.mark.parametrize("shape", [(24, 2, 200, 200, 32), (40, 4, 256, 256, 16), (6, 2, 130, 70, 8)])
def test_bwd_overwrites_prefilled_outputs(cuda_device, shape):
    """Head dims 8-32 add their 16-bit partial sums straight into dq, dk and dv, which the call
    zeroes first: gradient buffers holding old values (here 7.0, and NaN in dbias) give the same
    results as fresh ones, and the oracle's."""
    from colabfold_legacy_kernels import torch_ops
    n, h, sq, sk, d = shape
    q, k, v, bias, kmask, dout = _inputs(n, h, sq, sk, d, torch.bfloat16, seed=31 + n)
    scale = 1.0 / math.sqrt(d)
    fresh = _check(q, k, v, bias, kmask, dout, scale, "fresh")
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, scale)
    grads = (torch.full_like(q, 7.0), torch.full_like(k, 7.0), torch.full_like(v, 7.0),
             torch.full((h, sq, sk), float("nan"), dtype=torch.float32, device=q.device))
    again = torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale, grads=grads)
    torch.cuda.synchronize()
    for a, b, name in zip(again, fresh, ("dq", "dk", "dv")):
        # partials reduced in a timing-dependent order: equal up to 16-bit rounding
        assert_close_bf16(a, b, name + " prefilled vs fresh", rtol=1e-2, atol=1e-2)
    assert torch.equal(again[3], fresh[3]), "dbias"
