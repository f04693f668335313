"""Attention rows sharded across the GPUs of one node (one process per GPU).

The attention batch axis (MSA sequences for row attention, pair rows for triangle attention) is
independent: every rank takes a contiguous block of rows with the full bias, runs the forward
and backward on it, and the per-rank dbias partials (dbias sums over rows) are added with one
all-reduce.  dq, dk and dv stay row-local.  On GPUs the all-reduce runs on a side stream as soon
as the backward's main kernel has finished dbias, overlapping the conversion of the dq/dk/dv
accumulators (the third backward launch).

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
