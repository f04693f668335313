"""Row-sharded attention with the dbias all-reduce or reduce-scatter, on CPU ranks (gloo, world
size 2).

The sharding and the reduction are host logic; the per-rank compute is the CPU oracle here (the
GPU path passes the sm_100a kernels instead).  A second test makes one rank fail before the
collective and checks that the other rank gets an error instead of hanging.
"""

import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(3)
    n, h, s, d = 6, 2, 10, 8
    q, k, v, dout = (torch.randn(n, h, s, d, generator=g, dtype=torch.float64) for _ in range(4))
    bias = torch.randn(h, s, s, generator=g, dtype=torch.float64)
    kmask = (torch.rand(n, s, generator=g) > 0.3).to(torch.uint8)
    kmask[2] = 0
    return q, k, v, bias, kmask, dout, 0.35


def _worker(rank, world, port, queue, fail_rank, reduce="all"):
    try:
        sys.path[:0] = [REPO, os.path.join(REPO, "colabfold-legacy-kernels_b200", "src")]
        import torch.distributed as dist
        import oracle
        from colabfold_legacy_kernels.parallel import ShardedAttention, shard_rows
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=timedelta(seconds=15))
        q, k, v, bias, kmask, dout, scale = _inputs()
        r0, r1 = shard_rows(q.shape[0], world, rank)

        def fwd(q, k, v, bias, kmask, scale):
            return oracle.attention_fwd(q, k, v, bias, kmask, scale)

        def bwd(q, k, v, bias, kmask, out, lse, dout, scale):
            if rank == fail_rank:
                raise RuntimeError("injected failure on rank %d" % rank)
            return list(oracle.attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale))

        sa = ShardedAttention(fwd=fwd, bwd=bwd, dbias_reduce=reduce)
        res = sa.step(q[r0:r1], k[r0:r1], v[r0:r1], bias, kmask[r0:r1], dout[r0:r1], scale)
        out, lse = oracle.attention_fwd(q, k, v, bias, kmask, scale)
        ref = oracle.attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale)
        dbias_ref = ref[3]
        if reduce == "scatter":  # this rank's query rows of the summed dbias
            s0, s1 = shard_rows(q.shape[2], world, rank)
            dbias_ref = ref[3][:, s0:s1]
            assert tuple(res.dbias.shape) == tuple(dbias_ref.shape), res.dbias.shape
        errs = {
            "dq": float((res.dq - ref[0][r0:r1]).abs().max()),
            "dk": float((res.dk - ref[1][r0:r1]).abs().max()),
            "dv": float((res.dv - ref[2][r0:r1]).abs().max()),
            "dbias": float((res.dbias - dbias_ref).abs().max()),
            "out": float((res.out - out[r0:r1]).abs().max()),
        }
        queue.put((rank, "ok", errs))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent; the failing rank exits
        queue.put((rank, "error", "%s: %s" % (type(e).__name__, e)))


def _run(world, fail_rank=None, timeout=120, reduce="all"):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue, fail_rank, reduce))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=timeout)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


def test_row_sharding_covers_all_rows():
    from colabfold_legacy_kernels.parallel import shard_rows
    for n in (1, 7, 768):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("reduce", ["all", "scatter"])
def test_sharded_step_matches_single_process(reduce):
    results = _run(2, reduce=reduce)
    for rank in (0, 1):
        status, errs = results[rank]
        assert status == "ok", errs
        for name, err in errs.items():
            assert err < 1e-12, (rank, name, err)


def test_failed_rank_gives_error_not_hang():
    results = _run(2, fail_rank=1)
    assert results[1][0] == "error" and "injected" in results[1][1]
    # the surviving rank's all-reduce ends with an error (peer gone), within the timeout
    assert results[0][0] == "error", results[0]


# --------------------------------------------------------------------------------------------
# LayerNorm and GDP rows sharded, parameter gradients all-reduced (ShardedLnGdp)
# --------------------------------------------------------------------------------------------
def _ln_gdp_inputs():
    g = torch.Generator().manual_seed(5)
    m, c, n = 11, 16, 24
    x = torch.randn(m, c, generator=g, dtype=torch.float64)
    gamma = 1 + 0.1 * torch.randn(c, generator=g, dtype=torch.float64)
    dy = torch.randn(m, c, generator=g, dtype=torch.float64)
    wp, wg = (torch.randn(c, n, generator=g, dtype=torch.float64) / 4 for _ in range(2))
    bp, bg = (0.3 * torch.randn(n, generator=g, dtype=torch.float64) for _ in range(2))
    mask = (torch.rand(m, generator=g) > 0.2).to(torch.float64)
    dout = torch.randn(m, n, generator=g, dtype=torch.float64)
    return x, gamma, dy, wp, bp, wg, bg, mask, dout


def _ln_gdp_worker(rank, world, port, queue):
    try:
        sys.path[:0] = [REPO, os.path.join(REPO, "colabfold-legacy-kernels_b200", "src")]
        import torch.distributed as dist
        import oracle
        from colabfold_legacy_kernels.parallel import ShardedLnGdp
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=timedelta(seconds=15))
        x, gamma, dy, wp, bp, wg, bg, mask, dout = _ln_gdp_inputs()

        def ln_bwd(x, gamma, dy, eps, mean, rstd, grads):
            for t, v in zip(grads, oracle.layer_norm_bwd(x, gamma, dy, eps)):
                t.copy_(v)

        def gdp_bwd(x, wp, bp, wg, bg, mask, dout, grads):
            for t, v in zip(grads, oracle.gdp_bwd(x, wp, bp, wg, bg, mask, dout)):
                t.copy_(v)

        sh = ShardedLnGdp(ln_bwd=ln_bwd, gdp_bwd=gdp_bwd)
        r0, r1 = sh.rows(x.shape[0])
        ln = sh.layer_norm_bwd(x[r0:r1], gamma, dy[r0:r1], 1e-5)
        gd = sh.gdp_bwd(x[r0:r1], wp, bp, wg, bg, mask[r0:r1], dout[r0:r1])
        ln_ref = oracle.layer_norm_bwd(x, gamma, dy, 1e-5)
        gd_ref = oracle.gdp_bwd(x, wp, bp, wg, bg, mask, dout)
        errs = {"ln_dx": float((ln[0].double() - ln_ref[0][r0:r1]).abs().max())}
        for name, a, b in (("dgamma", ln[1], ln_ref[1]), ("dbeta", ln[2], ln_ref[2])):
            errs[name] = float((a.double() - b).abs().max() / b.abs().max())
        errs["gdp_dx"] = float((gd[0].double() - gd_ref[0][r0:r1]).abs().max())
        for name, a, b in zip(("dwp", "dbp", "dwg", "dbg"), gd[1:], gd_ref[1:]):
            errs[name] = float((a.double() - b).abs().max() / b.abs().max())
        queue.put((rank, "ok", errs))
        dist.destroy_process_group()
    except Exception as e:
        queue.put((rank, "error", "%s: %s\n%s" % (type(e).__name__, e, traceback.format_exc())))


def test_sharded_ln_gdp_matches_single_process():
    """Row shards of 11 rows over 2 ranks: dx row-local, parameter gradients (reduced in f32 via
    one all-reduce of a flat buffer) equal the full-batch oracle's to f32 rounding."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ln_gdp_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (s, e)) for r, s, e in (queue.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    for rank in (0, 1):
        status, errs = results[rank]
        assert status == "ok", errs
        for name, err in errs.items():
            assert err < (1e-12 if name.endswith("dx") else 1e-6), (rank, name, err)


def test_scatter_rejects_uneven_rows():
    from colabfold_legacy_kernels.parallel import ShardedAttention, scatter_dbias
    with pytest.raises(ValueError):
        ShardedAttention(dbias_reduce="sum")
    with pytest.raises(ValueError, match="multiple of the world size"):
        scatter_dbias(torch.zeros(2, 9, 4), 2, 0)


def _exchange_worker(rank, world, port, queue):
    try:
        sys.path[:0] = [REPO, os.path.join(REPO, "colabfold-legacy-kernels_b200", "src")]
        import torch.distributed as dist
        from colabfold_legacy_kernels.parallel import PeerDbiasExchange
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=timedelta(seconds=15))
        # no GPU here: every rank's buffer allocation fails, and the ranks agree on "none"
        # through the collectives instead of some of them waiting for the others
        ex = PeerDbiasExchange.create_or_none((2, 8, 8), "cpu")
        try:
            PeerDbiasExchange((2, 8, 8), "cpu")
            direct = "no error"
        except RuntimeError as e:
            direct = str(e)
        queue.put((rank, "ok", (ex is None, direct)))
        dist.destroy_process_group()
    except Exception as e:
        queue.put((rank, "error", "%s: %s" % (type(e).__name__, e)))


def test_peer_exchange_setup_failure_is_collective():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (s, e)) for r, s, e in (queue.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    for rank in (0, 1):
        status, payload = results[rank]
        assert status == "ok", payload
        none, direct = payload
        assert none, rank
        assert "could not allocate" in direct and "[0, 1]" in direct, direct
