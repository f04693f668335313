"""Attention, LayerNorm and gated-dual-projection rows sharded across the GPUs of one node (one
process per GPU).

The attention batch axis (MSA sequences for row attention, pair rows for triangle attention) is
independent: every rank takes a contiguous block of rows with the full bias, runs the forward
and backward on it, and the per-rank dbias partials (dbias sums over rows) are added with one
collective.  dq, dk and dv stay row-local.  On GPUs the collective runs on a side stream as soon
as the backward's main kernel has finished dbias, beside the backward's third launch (head
dim 64's accumulator conversion; empty for head dims up to 32).

The collective is an all-reduce (every rank receives all of dbias) or, with
dbias_reduce="scatter", a reduce-scatter by query rows: rank r receives the summed dbias rows
shard_rows(Sq, world, r) of every head.  The pair bias of a triangle or MSA-row attention is a
projection of the pair representation, bias[h, i, j] from z[i, j], so in a module whose pair
rows are sharded the same way as the attention rows, rank r needs exactly those dbias rows to
back-propagate into its own z rows; the reduce-scatter moves half the bytes of the all-reduce.
With dbias_reduce="peer" the same reduce-scatter runs as this library's own kernel over peer
memory (PeerDbiasExchange: every rank's dbias in CUDA-IPC memory, one launch that reads its
rows from every rank over NVLink and adds them in rank order) instead of an NCCL collective.

LayerNorm and the gated dual projection are row-wise too (ShardedLnGdp): x, y, dx, out stay
row-local, and the parameter gradients (dgamma, dbeta; dwp, dbp, dwg, dbg), which sum over rows,
are written by the kernels into one flat f32 buffer and added with a single all-reduce.

The reference is single-device (grid-level parallelism only, cuda/volta_mma_attn.cu:295); this
module is new capability.
"""

import ctypes
import warnings
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
    dbias: torch.Tensor   # summed over all ranks: [H, Sq, Sk], or with dbias_reduce="scatter"
                          # this rank's query rows [H, Sq / world, Sk]


def _default_fwd(q, k, v, bias, kmask, scale):
    from . import torch_ops
    return torch_ops.attention_fwd(q, k, v, bias, kmask, scale)


def scatter_dbias(dbias, world, rank, group=None):
    """Reduce-scatter of dbias [H, Sq, Sk] by query rows over `group`: returns this rank's rows
    shard_rows(Sq, world, rank) of the sum over ranks, [H, Sq / world, Sk].  Sq must be a
    multiple of `world` (equal chunks).  The rows are first gathered rank-major, [world, H,
    Sq / world, Sk], one copy, so that one collective covers every head."""
    h, sq, sk = dbias.shape
    if sq % world:
        raise ValueError("dbias reduce-scatter needs Sq (%d) to be a multiple of the world "
                         "size (%d)" % (sq, world))
    part = sq // world
    src = dbias.view(h, world, part, sk).transpose(0, 1).contiguous()
    out = torch.empty((h, part, sk), dtype=dbias.dtype, device=dbias.device)
    dist.reduce_scatter_tensor(out.view(-1), src.view(-1), group=group)
    return out


class _DeviceBuffer:
    """A device allocation made outside torch, seen by torch through __cuda_array_interface__
    (torch.as_tensor wraps it without a copy; the allocation's owner frees it)."""

    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": tuple(int(x) for x in shape), "typestr": "<f4",
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


class PeerDbiasExchange:
    """dbias [H, Sq, Sk] of every rank of `group` in CUDA-IPC memory, and its reduce-scatter by
    query rows as one kernel over peer memory (cfk_dbias_reduce_scatter).

    `dbias` is this rank's buffer: pass it to the backward as its dbias output.  After the
    backward, reduce_scatter() (enqueued on `stream`) writes into `out` [H, Sq / world, Sk] the
    sum over ranks, in rank order, of this rank's query rows; when it completes no peer reads
    `dbias` any more.  Every rank must create the exchange, call reduce_scatter and close() in
    the same order (creation and close() are collective on `group`).  One process per GPU;
    2 <= world <= 8, Sq % world == 0, Sk % 4 == 0."""

    def __init__(self, shape, device, group=None):
        from . import cabi
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shape = tuple(int(x) for x in shape)
        self.device = torch.device(device)
        h, sq, sk = self.shape
        if not 2 <= self.world <= 8 or sq % self.world or sk % 4:
            raise ValueError("PeerDbiasExchange: world %d, dbias %r (2 <= world <= 8, Sq a "
                             "multiple of the world size, Sk of 4)" % (self.world, self.shape))
        nbytes = cabi.function("cfk_dbias_exchange_bytes")(h, sq, sk)
        if nbytes == 0:
            raise ValueError("PeerDbiasExchange: dbias %r too large" % (self.shape,))
        self._cabi = cabi
        # every rank takes part in the one gather below, also when its allocation failed, so
        # that the ranks' collectives stay matched; then all of them raise or none does
        own = ctypes.c_void_p()
        raw = None
        try:
            with torch.cuda.device(self.device):
                handle = ctypes.create_string_buffer(cabi.CFK_IPC_HANDLE_BYTES)
                cabi.call("cfk_ipc_alloc", nbytes, ctypes.byref(own), handle)
                raw = handle.raw
        except Exception:
            raw = None
        handles = [None] * self.world
        dist.all_gather_object(handles, raw, group=group)
        failed = [r for r, raw_r in enumerate(handles) if raw_r is None]
        ptrs = []
        try:
            if failed:
                raise RuntimeError("PeerDbiasExchange: rank(s) %s could not allocate" % failed)
            with torch.cuda.device(self.device):
                for r, raw_r in enumerate(handles):
                    if r == self.rank:
                        ptrs.append(own.value)
                        continue
                    peer = ctypes.c_void_p()
                    cabi.call("cfk_ipc_open", ctypes.create_string_buffer(raw_r, len(raw_r)),
                              ctypes.byref(peer))
                    ptrs.append(peer.value)
        except Exception:
            # undo this rank's part (no collective: the other ranks may have succeeded)
            for r, ptr in enumerate(ptrs):
                if r != self.rank:
                    cabi.call("cfk_ipc_close", ptr)
            if own.value:
                cabi.call("cfk_ipc_free", own.value)
            raise
        self._own = own.value
        self._ptrs = ptrs
        self._buffers = (ctypes.c_void_p * self.world)(*ptrs)
        self.dbias = torch.as_tensor(_DeviceBuffer(self._own, self.shape), device=self.device)
        self.out = torch.empty((h, sq // self.world, sk), dtype=torch.float32,
                               device=self.device)

    @classmethod
    def create_or_none(cls, shape, device, group=None):
        """An exchange on every rank, or None on every rank when any rank could not set its
        part up (CUDA IPC unavailable, a mapping refused, ...), so that the ranks agree on
        which reduction they run.  Collective on `group`."""
        ex = None
        try:
            ex = cls(shape, device, group)
        except Exception as e:  # reported here and agreed on below
            warnings.warn("PeerDbiasExchange: set-up failed on this rank (%s: %s); every rank "
                          "falls back" % (type(e).__name__, e))
            ex = None
        ok = torch.tensor([1 if ex is not None else 0], dtype=torch.int32,
                          device=torch.device(device))
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 1:
            return ex
        if ex is not None:
            ex._release()
        dist.barrier(group=group)  # every rank has unmapped its peers' buffers
        if ex is not None:
            ex._free_own()
        return None

    def reduce_scatter(self, out=None, stream=None):
        """Enqueues the reduce-scatter of `dbias` into `out` (default: self.out) on `stream`
        (default: the current stream); returns `out`."""
        out = self.out if out is None else out
        if (out.dtype != torch.float32 or not out.is_contiguous() or out.device != self.device
                or tuple(out.shape) != tuple(self.out.shape)):
            raise ValueError("reduce_scatter: out must be a contiguous f32 %r tensor on %s"
                             % (tuple(self.out.shape), self.device))
        stream = torch.cuda.current_stream(self.device) if stream is None else stream
        h, sq, sk = self.shape
        self._cabi.call("cfk_dbias_reduce_scatter", stream.cuda_stream, self._buffers,
                        self.world, self.rank, h, sq, sk, out.data_ptr())
        return out

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (collective: every rank calls it
        after its last reduce_scatter)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._release()
        dist.barrier(group=self.group)  # every peer has unmapped this rank's buffer
        self._free_own()

    def _release(self):
        """Unmaps the peers' buffers (this rank only)."""
        with torch.cuda.device(self.device):
            for r, ptr in enumerate(self._ptrs):
                if r != self.rank and ptr is not None:
                    self._cabi.call("cfk_ipc_close", ptr)
        self._ptrs = [p if r == self.rank else None for r, p in enumerate(self._ptrs)]

    def _free_own(self):
        if self._own is None:
            return
        with torch.cuda.device(self.device):
            self.dbias = None
            self._cabi.call("cfk_ipc_free", self._own)
        self._own = None


class ShardedAttention:
    """Forward + backward of attention on this rank's rows, dbias reduced over `group`.

    `fwd(q, k, v, bias, kmask, scale) -> (out, lse)` and `bwd(...)` default to the sm_100a
    kernels; tests pass CPU implementations to check the sharding and the reduction alone.
    `dbias_reduce`: "all" (all-reduce, every rank gets the whole sum), "scatter" (each rank
    gets the summed rows of its own query-row shard; see the module docstring) or "peer" (the
    same rows by this library's peer-memory kernel, PeerDbiasExchange; sm_100a kernels only;
    call close() on every rank when done).
    """

    def __init__(self, group=None, fwd=None, bwd=None, dbias_reduce="all"):
        if dbias_reduce not in ("all", "scatter", "peer"):
            raise ValueError("dbias_reduce must be 'all', 'scatter' or 'peer', not %r"
                             % (dbias_reduce,))
        if dbias_reduce == "peer" and (fwd is not None or bwd is not None):
            raise ValueError("dbias_reduce='peer' runs the sm_100a kernels only")
        self._exchange = None
        self.dbias_reduce = dbias_reduce
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.fwd = fwd or _default_fwd
        self.bwd = bwd
        self._ws = None
        self._comm = None

    def rows(self, n_rows):
        return shard_rows(n_rows, self.world, self.rank)

    def close(self):
        """Releases the peer-memory exchange (collective with dbias_reduce='peer')."""
        if self._exchange is not None:
            self._exchange.close()
            self._exchange = None

    def _reduce(self, dbias):
        """The cross-rank sum of dbias, whole or this rank's query rows."""
        if self.dbias_reduce == "peer":
            out = torch.empty((dbias.shape[0], dbias.shape[1] // self.world, dbias.shape[2]),
                              dtype=torch.float32, device=dbias.device)
            return self._exchange.reduce_scatter(out)
        if self.dbias_reduce == "scatter":
            return scatter_dbias(dbias, self.world, self.rank, self.group)
        dist.all_reduce(dbias, group=self.group)
        return dbias

    def step(self, q, k, v, bias, kmask, dout, scale):
        """q, k, v, dout, kmask: this rank's rows; bias: full.  Returns a ShardResult."""
        out, lse = self.fwd(q, k, v, bias, kmask, scale)
        if self.bwd is not None:
            dq, dk, dv, dbias = self.bwd(q, k, v, bias, kmask, out, lse, dout, scale)
            if self.world > 1:
                dbias = self._reduce(dbias)
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
        if self.dbias_reduce == "peer" and self.world > 1:
            if self._exchange is not None and self._exchange.shape != (h, sq, sk):
                self.close()
            if self._exchange is None:
                self._exchange = PeerDbiasExchange.create_or_none((h, sq, sk), q.device,
                                                                  self.group)
                if self._exchange is None:  # every rank falls back together
                    self.dbias_reduce = "scatter"
        if self._exchange is not None:
            # the backward writes dbias straight into this rank's exchange buffer
            dbias_out = self._exchange.dbias
        else:
            dbias_out = torch.empty((h, sq, sk), dtype=torch.float32, device=q.device)
        grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), dbias_out)
        args = (q, k, v, bias, kmask, out, lse, dout, scale)
        torch_ops.attention_bwd(*args, workspace=self._ws, grads=grads, phase=0)
        torch_ops.attention_bwd(*args, workspace=self._ws, grads=grads, phase=1)
        dbias = grads[3]
        if self.world > 1:
            stream = torch.cuda.current_stream(q.device)
            if self._comm is None:
                self._comm = torch.cuda.Stream(q.device)
            self._comm.wait_stream(stream)
            with torch.cuda.stream(self._comm):
                dbias = self._reduce(grads[3])
            grads[3].record_stream(self._comm)
            dbias.record_stream(stream)  # allocated on the comm stream, used on this one
        torch_ops.attention_bwd(*args, workspace=self._ws, grads=grads, phase=2)
        if self.world > 1:
            torch.cuda.current_stream(q.device).wait_stream(self._comm)
        return grads[0], grads[1], grads[2], dbias


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
