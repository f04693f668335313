"""Attention, LayerNorm and gated-dual-projection rows sharded across the GPUs of one node (one
process per GPU).

The attention batch axis (MSA sequences for row attention, pair rows for triangle attention) is
independent: every rank takes a contiguous block of rows with the full bias, runs the forward
and backward on it, and the per-rank dbias partials (dbias sums over rows) are added with one
all-reduce.  dq, dk and dv stay row-local.  On GPUs the all-reduce runs on a side stream as soon
as the backward's main kernel has finished dbias, overlapping the conversion of the dq/dk/dv
accumulators (the third backward launch).

LayerNorm and the gated dual projection are row-wise too (ShardedLnGdp): x, y, dx, out stay
row-local, and the parameter gradients (dgamma, dbeta; dwp, dbp, dwg, dbg), which sum over rows,
are written by the kernels into one flat f32 buffer and added with a single all-reduce.

The reference is single-device (grid-level parallelism only, cuda/volta_mma_attn.cu:295); this
module is new capability.
"""

from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_rows(n_rows, world, rank):
    """[start, stop) of the rows rank `rank` of `world` owns: contiguous, sizes differ by <= 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank %r/%r" % (world, rank))
    return rank * n_rows // world, (rank + 1) * n_rows // world


@dataclass
class ShardResult:
    out: torch.Tensor
    lse: torch.Tensor
    dq: torch.Tensor
    dk: torch.Tensor
    dv: torch.Tensor
    dbias: torch.Tensor   # summed over all ranks


def _default_fwd(q, k, v, bias, kmask, scale):
    from . import torch_ops
    return torch_ops.attention_fwd(q, k, v, bias, kmask, scale)


class ShardedAttention:
    """Forward + backward of attention on this rank's rows, dbias all-reduced over `group`.

    `fwd(q, k, v, bias, kmask, scale) -> (out, lse)` and `bwd(...)` default to the sm_100a
    kernels; tests pass CPU implementations to check the sharding and the reduction alone.
    """

    def __init__(self, group=None, fwd=None, bwd=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.fwd = fwd or _default_fwd
        self.bwd = bwd
        self._ws = None
        self._comm = None

    def rows(self, n_rows):
        return shard_rows(n_rows, self.world, self.rank)

    def step(self, q, k, v, bias, kmask, dout, scale):
        """q, k, v, dout, kmask: this rank's rows; bias: full.  Returns a ShardResult."""
        out, lse = self.fwd(q, k, v, bias, kmask, scale)
        if self.bwd is not None:
            dq, dk, dv, dbias = self.bwd(q, k, v, bias, kmask, out, lse, dout, scale)
            if self.world > 1:
                dist.all_reduce(dbias, group=self.group)
        else:
            dq, dk, dv, dbias = self._bwd_overlapped(q, k, v, bias, kmask, out, lse, dout, scale)
        return ShardResult(out, lse, dq, dk, dv, dbias)

    def _bwd_overlapped(self, q, k, v, bias, kmask, out, lse, dout, scale):
        from . import torch_ops
        n, h, sq, d = q.shape
        sk = k.shape[2]
        if self._ws is None or self._ws.numel() < torch_ops.cabi.workspace_size(
                "cfk_attn_bwd_workspace_size", n, h, sq, sk, d):
            self._ws = torch_ops.attention_bwd_workspace(n, h, sq, sk, d, q.device)
        grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
                 torch.empty((h, sq, sk), dtype=torch.float32, device=q.device))
        args = (q, k, v, bias, kmask, out, lse, dout, scale)
        torch_ops.attention_bwd(*args, workspace=self._ws, grads=grads, phase=0)
        torch_ops.attention_bwd(*args, workspace=self._ws, grads=grads, phase=1)
        if self.world > 1:
            stream = torch.cuda.current_stream(q.device)
            if self._comm is None:
                self._comm = torch.cuda.Stream(q.device)
            self._comm.wait_stream(stream)
            with torch.cuda.stream(self._comm):
                dist.all_reduce(grads[3], group=self.group)
            grads[3].record_stream(self._comm)
        torch_ops.attention_bwd(*args, workspace=self._ws, grads=grads, phase=2)
        if self.world > 1:
            torch.cuda.current_stream(q.device).wait_stream(self._comm)
        return grads


def _flat_views(buf, shapes):
    """Consecutive views of the flat tensor `buf` with the given shapes."""
    out, off = [], 0
    for shape in shapes:
        n = 1
        for d in shape:
            n *= d
        out.append(buf[off:off + n].view(shape))
        off += n
    return out


class ShardedLnGdp:
    """LayerNorm and GDP backward on this rank's rows; the parameter gradients are all-reduced
    over `group` in one collective per backward.  The forwards are row-local: call them on the
    rank's rows directly (torch_ops.layer_norm_fwd, gdp_fwd, ln_gdp_fwd).

    `ln_bwd(x, gamma, dy, eps, mean, rstd, grads)` and `gdp_bwd(x, wp, bp, wg, bg, mask, dout,
    grads)` fill the given gradient tensors; they default to the sm_100a kernels, and tests pass
    CPU implementations to check the sharding and the reduction alone.
    """

    def __init__(self, group=None, ln_bwd=None, gdp_bwd=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.ln_bwd_fn = ln_bwd or _default_ln_bwd
        self.gdp_bwd_fn = gdp_bwd or _default_gdp_bwd

    def rows(self, n_rows):
        return shard_rows(n_rows, self.world, self.rank)

    def _reduce(self, flat):
        if self.world > 1:
            dist.all_reduce(flat, group=self.group)

    def layer_norm_bwd(self, x, gamma, dy, eps, mean=None, rstd=None):
        """x, dy, mean, rstd: this rank's rows.  Returns (dx, dgamma, dbeta), the last two summed
        over all ranks' rows."""
        c = x.shape[1]
        flat = torch.empty(2 * c, dtype=torch.float32, device=x.device)
        dgamma, dbeta = _flat_views(flat, [(c,), (c,)])
        dx = torch.empty_like(x)
        self.ln_bwd_fn(x, gamma, dy, eps, mean, rstd, (dx, dgamma, dbeta))
        self._reduce(flat)
        return dx, dgamma, dbeta

    def gdp_bwd(self, x, wp, bp, wg, bg, mask, dout):
        """x, mask, dout: this rank's rows.  Returns (dx, dwp, dbp, dwg, dbg), the last four
        summed over all ranks' rows."""
        k, n = wp.shape
        flat = torch.empty(2 * k * n + 2 * n, dtype=torch.float32, device=x.device)
        dwp, dwg, dbp, dbg = _flat_views(flat, [(k, n), (k, n), (n,), (n,)])
        dx = torch.empty_like(x)
        self.gdp_bwd_fn(x, wp, bp, wg, bg, mask, dout, (dx, dwp, dbp, dwg, dbg))
        self._reduce(flat)
        return dx, dwp, dbp, dwg, dbg


def _default_ln_bwd(x, gamma, dy, eps, mean, rstd, grads):
    from . import torch_ops
    torch_ops.layer_norm_bwd(x, gamma, dy, eps, mean=mean, rstd=rstd, grads=grads)


def _default_gdp_bwd(x, wp, bp, wg, bg, mask, dout, grads):
    from . import torch_ops
    torch_ops.gdp_bwd(x, wp, bp, wg, bg, mask, dout, grads=grads)
