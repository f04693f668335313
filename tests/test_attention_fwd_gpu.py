"""GPU parity of the attention forward (cfk_attn_fwd through the C ABI) against the CPU oracle.

Tolerances: out (bf16/fp16) rtol = atol = 2e-2; lse (f32) 1e-4 of max|lse| plus 1e-4 relative,
both against the float64 oracle on the same 16-bit inputs.
"""

import math

import pytest
import torch

import oracle
from conftest import assert_close_bf16, assert_close_f32

pytestmark = pytest.mark.gpu


def _inputs(n, h, sq, sk, d, dtype, seed, mask_mode="random", device="cuda"):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, h, sq, d, generator=g).to(dtype)
    k = torch.randn(n, h, sk, d, generator=g).to(dtype)
    v = torch.randn(n, h, sk, d, generator=g).to(dtype)
    bias = torch.randn(h, sq, sk, generator=g).to(dtype)
    kmask = torch.ones(n, sk, dtype=torch.uint8)
    if mask_mode == "random":
        kmask = (torch.rand(n, sk, generator=g) > 0.2).to(torch.uint8)
        if n > 1:
            kmask[1] = 0          # one batch row with every key masked
    elif mask_mode == "tail":
        kmask[:, sk - max(1, sk // 10):] = 0
    return [t.to(device) for t in (q, k, v, bias, kmask)]


def _run(q, k, v, bias, kmask, scale):
    from colabfold_legacy_kernels import torch_ops
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, scale)
    torch.cuda.synchronize()
    return out, lse


def _check(q, k, v, bias, kmask, scale, what):
    out, lse = _run(q, k, v, bias, kmask, scale)
    ref_out, ref_lse = oracle.attention_fwd(q.cpu(), k.cpu(), v.cpu(), bias.cpu(), kmask.cpu(),
                                            scale)
    assert_close_bf16(out, ref_out, what + " out")
    assert_close_f32(lse, ref_lse, what + " lse")
    return out, lse


@pytest.mark.parametrize("d", [8, 16, 32, 64])
def test_fwd_head_dims_ragged(cuda_device, d):
    # odd batch (a group with one missing row), Sq and Sk not multiples of the 128 tile
    q, k, v, bias, kmask = _inputs(3, 2, 130, 200, d, torch.bfloat16, seed=d)
    _check(q, k, v, bias, kmask, 1.0 / math.sqrt(d), "d=%d" % d)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fwd_dtypes(cuda_device, dtype):
    q, k, v, bias, kmask = _inputs(4, 2, 256, 256, 32, dtype, seed=11, mask_mode="tail")
    _check(q, k, v, bias, kmask, 1.0 / math.sqrt(32), str(dtype))


def test_fwd_unaligned_key_count(cuda_device):
    # Sk % 8 != 0: the bias rows are not 16-byte aligned, so the bias is read without TMA
    q, k, v, bias, kmask = _inputs(2, 3, 70, 77, 32, torch.bfloat16, seed=5)
    _check(q, k, v, bias, kmask, 0.2, "Sk=77")


def test_fwd_single_row_single_key(cuda_device):
    q, k, v, bias, kmask = _inputs(1, 1, 1, 1, 16, torch.bfloat16, seed=6, mask_mode="none")
    _check(q, k, v, bias, kmask, 0.25, "1x1")


def test_fwd_fully_masked_batch_row_is_uniform_average(cuda_device):
    q, k, v, bias, kmask = _inputs(2, 2, 64, 150, 32, torch.bfloat16, seed=7, mask_mode="none")
    kmask[0] = 0
    out, lse = _check(q, k, v, bias, kmask, 1.0 / math.sqrt(32), "fully masked")
    mean_v = v[0].double().mean(dim=1, keepdim=True).expand(-1, 64, -1)
    assert_close_bf16(out[0], mean_v, "uniform average")
    expect_lse = torch.full_like(lse[0], -1e4 + math.log(150), dtype=torch.float64)
    assert_close_f32(lse[0], expect_lse, "lse of fully masked row")


def test_fwd_msa_shape(cuda_device):
    cfg = oracle.configs.scaled(oracle.configs.C2, n=6)
    inp = oracle.configs.make_attention_inputs(cfg, device="cpu")
    t = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    _check(t["q"], t["k"], t["v"], t["bias"], t["kmask"], t["scale"], "msa")


def test_fwd_triangle_shape(cuda_device):
    cfg = oracle.configs.scaled(oracle.configs.C3, n=8, s=384)
    inp = oracle.configs.make_attention_inputs(cfg, device="cpu")
    t = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    _check(t["q"], t["k"], t["v"], t["bias"], t["kmask"], t["scale"], "triangle")


def test_fwd_large_complex_shape(cuda_device):
    """Config C5's shape class (N_res = 2048: 16 key tiles per row, all-ones mask), two rows."""
    cfg = oracle.configs.scaled(oracle.configs.C5, n=2)
    inp = oracle.configs.make_attention_inputs(cfg, device="cpu")
    t = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    _check(t["q"], t["k"], t["v"], t["bias"], t["kmask"], t["scale"], "tri-2048")


def test_fwd_deterministic_and_no_timeouts(cuda_device):
    from colabfold_legacy_kernels import cabi
    cabi.clear_device_status()
    q, k, v, bias, kmask = _inputs(5, 4, 300, 260, 32, torch.bfloat16, seed=9)
    a, la = _run(q, k, v, bias, kmask, 0.17)
    b, lb = _run(q, k, v, bias, kmask, 0.17)
    assert torch.equal(a, b) and torch.equal(la, lb)
    assert cabi.device_status() == 0


def test_fwd_large_bias_rows_select_path(cuda_device):
    # All kept logits far below -1e4: the replaced masked keys (-1e4) must win, exactly as in the
    # reference (volta_mma_attn.cu:186-188).
    q, k, v, bias, kmask = _inputs(2, 1, 40, 130, 16, torch.bfloat16, seed=12, mask_mode="none")
    bias = torch.full_like(bias, -30000.0)
    kmask[:, 5] = 0
    kmask[:, 129] = 0
    _check(q, k, v, bias, kmask, 0.25, "select path")


def _rows_per_item(n, h, sq, sms):
    """The forward's choice of batch rows per work item for D <= 32 (rows_per_item in
    attention_fwd.cu): three when their estimated waves x rows x cost is lower, else two."""
    def cost(nw, per_row):
        items = (n + nw - 1) // nw * h * ((sq + 127) // 128)
        grid = max(1, min(items, sms))
        return (items + grid - 1) // grid * nw * per_row
    return 3 if cost(3, 0.982) < cost(2, 1.0) else 2


@pytest.mark.parametrize("d", [8, 16, 32])
def test_fwd_three_rows_per_item(cuda_device, d):
    """Enough batch rows that the kernel runs three per work item (P written over S in tensor
    memory), including an odd last group (602 = 3 * 200 + 2) and ragged keys."""
    n, h, sq, sk = 602, 4, 128, 136
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert _rows_per_item(n, h, sq, sms) == 3
    q, k, v, bias, kmask = _inputs(n, h, sq, sk, d, torch.bfloat16, seed=40 + d)
    _check(q, k, v, bias, kmask, 1.0 / math.sqrt(d), "three rows per item, d=%d" % d)
