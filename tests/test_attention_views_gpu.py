"""Attention over strided views (cfk_attn_fwd_strided, cfk_attn_bwd_strided through the C ABI).

Triangle attention around the ending node and MSA column attention attend over the other
residue axis of the same activations: with q, k, v stored [S, N, H, D] (the batch axis second),
q.permute(1, 2, 0, 3) is the [N, H, S, D] operand.  The kernels take such views as strides of
their TMA descriptors and row addressing, so no transposed copy is made.

The forward through views runs the same tiles and arithmetic as the packed call and must
match it bit for bit.  The backward's dq, dk, dv add f32 partials with bulk reductions whose
order can vary between launches, so they are compared with the packed call at bf16 tolerance
(rtol = atol = 2e-2) and with the float64 oracle; dbias with the f32 tolerance.
"""

import math

import pytest
import torch

import oracle
from conftest import assert_close_bf16, assert_close_f32

pytestmark = pytest.mark.gpu


def _rows(storage_shape, perm, dtype, g):
    """A [N,H,S,D] view of a freshly drawn tensor stored as `storage_shape`."""
    return torch.randn(*storage_shape, generator=g).to(dtype).cuda().permute(*perm)


def _ending_node(n, h, sq, sk, d, dtype, seed):
    """q, k, v, dout as views of [S, N, H, D] storage; bias, kmask packed."""
    g = torch.Generator().manual_seed(seed)
    q = _rows((sq, n, h, d), (1, 2, 0, 3), dtype, g)
    k = _rows((sk, n, h, d), (1, 2, 0, 3), dtype, g)
    v = _rows((sk, n, h, d), (1, 2, 0, 3), dtype, g)
    dout = _rows((sq, n, h, d), (1, 2, 0, 3), dtype, g)
    bias = torch.randn(h, sq, sk, generator=g).to(dtype).cuda()
    kmask = (torch.rand(n, sk, generator=g) > 0.2).to(torch.uint8).cuda()
    return q, k, v, bias, kmask, dout


def _sndh_like(t):
    """An empty tensor with t's [N,H,S,D] shape, stored [S, N, H, D] and viewed [N,H,S,D]."""
    n, h, s, d = t.shape
    return torch.empty((s, n, h, d), dtype=t.dtype, device=t.device).permute(1, 2, 0, 3)


@pytest.mark.parametrize("d", [8, 16, 32, 64])
def test_fwd_ending_node_views_match_packed(cuda_device, d):
    from colabfold_legacy_kernels import torch_ops
    q, k, v, bias, kmask, _ = _ending_node(5, 2, 200, 136, d, torch.bfloat16, seed=300 + d)
    assert not q.is_contiguous()
    scale = 1.0 / math.sqrt(d)
    out_view = _sndh_like(q)  # out through a view as well
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, scale, out=out_view)
    ref, ref_lse = torch_ops.attention_fwd(q.contiguous(), k.contiguous(), v.contiguous(), bias,
                                           kmask, scale)
    torch.cuda.synchronize()
    assert out.data_ptr() == out_view.data_ptr()
    assert torch.equal(out, ref), "strided forward differs from the packed call"
    assert torch.equal(lse, ref_lse)
    r = oracle.attention_fwd(q.cpu(), k.cpu(), v.cpu(), bias.cpu(), kmask.cpu(), scale)
    assert_close_bf16(out, r[0], "ending-node out")


def test_fwd_nshd_layout_fp16(cuda_device):
    """q, k, v stored [N, S, H, D], out packed."""
    from colabfold_legacy_kernels import torch_ops
    g = torch.Generator().manual_seed(11)
    n, h, s, d = 3, 4, 160, 32
    q, k, v = (_rows((n, s, h, d), (0, 2, 1, 3), torch.float16, g) for _ in range(3))
    bias = torch.randn(h, s, s, generator=g).half().cuda()
    kmask = torch.ones(n, s, dtype=torch.uint8).cuda()
    kmask[0, 150:] = 0
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, 0.2)
    ref, ref_lse = torch_ops.attention_fwd(q.contiguous(), k.contiguous(), v.contiguous(), bias,
                                           kmask, 0.2)
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(lse, ref_lse)


@pytest.mark.parametrize("d,dtype", [(8, torch.bfloat16), (16, torch.bfloat16),
                                     (32, torch.bfloat16), (64, torch.bfloat16),
                                     (32, torch.float16)])
def test_bwd_ending_node_views(cuda_device, d, dtype):
    """Every [N,H,S,D] operand and gradient a view of [S, N, H, D] storage (the backward adds
    its 16-bit partial sums into the dq/dk/dv views through strided TMA maps)."""
    from colabfold_legacy_kernels import torch_ops
    q, k, v, bias, kmask, dout = _ending_node(4, 2, 190, 250, d, dtype, seed=400 + d)
    scale = 1.0 / math.sqrt(d)
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, scale, out=_sndh_like(q))
    grads = (_sndh_like(q), _sndh_like(k), _sndh_like(v),
             torch.empty(bias.shape, dtype=torch.float32, device=q.device))
    dq, dk, dv, dbias = torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale,
                                                grads=grads)
    packed = [t.contiguous() for t in (q, k, v)]
    rq, rk, rv, rb = torch_ops.attention_bwd(*packed, bias, kmask, out.contiguous(), lse,
                                             dout.contiguous(), scale)
    torch.cuda.synchronize()
    assert not dq.is_contiguous() and dq.data_ptr() == grads[0].data_ptr()
    assert_close_bf16(dq, rq, "view dq vs packed")
    assert_close_bf16(dk, rk, "view dk vs packed")
    assert_close_bf16(dv, rv, "view dv vs packed")
    assert_close_f32(dbias, rb, "view dbias vs packed")
    r = oracle.attention_bwd(q.cpu(), k.cpu(), v.cpu(), bias.cpu(), kmask.cpu(), out.cpu(),
                             lse.cpu(), dout.cpu(), scale)
    assert_close_bf16(dq, r[0], "ending-node dq")
    assert_close_bf16(dk, r[1], "ending-node dk")
    assert_close_bf16(dv, r[2], "ending-node dv")
    assert_close_f32(dbias, r[3], "ending-node dbias")


def test_bwd_phases_with_views(cuda_device):
    """cfk_attn_bwd_phase_strided issued 0, 1, 2 equals the one-call strided backward."""
    from colabfold_legacy_kernels import torch_ops
    q, k, v, bias, kmask, dout = _ending_node(3, 2, 130, 130, 32, torch.bfloat16, seed=5)
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, 0.25)
    n, h, sq, d = q.shape
    ws = torch_ops.attention_bwd_workspace(n, h, sq, k.shape[2], d, q.device)
    grads = (_sndh_like(q), _sndh_like(k), _sndh_like(v),
             torch.empty(bias.shape, dtype=torch.float32, device=q.device))
    for ph in range(3):
        torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, 0.25, workspace=ws,
                                grads=grads, phase=ph)
    one = torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, 0.25)
    torch.cuda.synchronize()
    for a, b, name in zip(grads[:3], one[:3], ("dq", "dk", "dv")):
        assert_close_bf16(a, b, "phases " + name)
    assert_close_f32(grads[3], one[3], "phases dbias")


def test_empty_keys_and_queries_through_views(cuda_device):
    """Sk = 0: the strided out is zeroed and nothing else in its storage is touched; Sq = 0:
    dk and dv are zeroed through their views."""
    from colabfold_legacy_kernels import cabi, torch_ops
    n, h, sq, d = 3, 2, 40, 16
    store = torch.full((sq, n, 2 * h, d), 7.0, dtype=torch.bfloat16, device="cuda")
    out = store[:, :, :h].permute(1, 2, 0, 3)  # the first h of every 2h head slots
    q = torch.randn(n, h, sq, d, device="cuda").bfloat16()
    k = torch.empty(n, h, 0, d, device="cuda", dtype=torch.bfloat16)
    bias = torch.empty(h, sq, 0, device="cuda", dtype=torch.bfloat16)
    kmask = torch.empty(n, 0, dtype=torch.uint8, device="cuda")
    torch_ops.attention_fwd(q, k, k, bias, kmask, 1.0, out=out)
    torch.cuda.synchronize()
    assert torch.all(store[:, :, :h] == 0) and torch.all(store[:, :, h:] == 7)

    sk = 24
    gstore = torch.full((sk, n, 2 * h, d), 7.0, dtype=torch.bfloat16, device="cuda")
    dk = gstore[:, :, :h].permute(1, 2, 0, 3)
    dv = gstore[:, :, h:].permute(1, 2, 0, 3)
    q0 = torch.empty(n, h, 0, d, device="cuda", dtype=torch.bfloat16)
    kk = torch.randn(n, h, sk, d, device="cuda").bfloat16()
    dbias = torch.full((h, 0, sk), 1.0, device="cuda")
    lse0 = torch.empty(n, h, 0, device="cuda")
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    torch_ops.attention_bwd(q0, kk, kk, torch.empty(h, 0, sk, device="cuda").bfloat16(),
                            torch.ones(n, sk, dtype=torch.uint8, device="cuda"), q0, lse0, q0,
                            1.0, workspace=ws, grads=(q0.clone(), dk, dv, dbias))
    torch.cuda.synchronize()
    assert torch.all(gstore == 0)
    assert cabi.device_status() == 0


def test_fwd_bwd_views_three_rows_per_item(cuda_device):
    """Enough batch rows that the forward runs three per work item (602 rows, H = 4, one query
    tile), through ending-node views: forward bit for bit as the packed call, backward against
    the packed call."""
    from colabfold_legacy_kernels import torch_ops
    q, k, v, bias, kmask, dout = _ending_node(602, 4, 128, 136, 32, torch.bfloat16, seed=610)
    out, lse = torch_ops.attention_fwd(q, k, v, bias, kmask, 0.2, out=_sndh_like(q))
    ref, ref_lse = torch_ops.attention_fwd(q.contiguous(), k.contiguous(), v.contiguous(), bias,
                                           kmask, 0.2)
    grads = (_sndh_like(q), _sndh_like(k), _sndh_like(v),
             torch.empty(bias.shape, dtype=torch.float32, device=q.device))
    dq, dk, dv, dbias = torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, 0.2,
                                                grads=grads)
    rq, rk, rv, rb = torch_ops.attention_bwd(q.contiguous(), k.contiguous(), v.contiguous(), bias,
                                             kmask, ref, ref_lse, dout.contiguous(), 0.2)
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
    assert_close_bf16(dq, rq, "602-row view dq")
    assert_close_bf16(dk, rk, "602-row view dk")
    assert_close_bf16(dv, rv, "602-row view dv")
    assert_close_f32(dbias, rb, "602-row view dbias")
