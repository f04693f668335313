"""Row sharding on two GPUs with NCCL (skipped with fewer than two GPUs).

Attention (ShardedAttention: dbias all-reduced, or reduce-scattered by query rows by NCCL or by
the library's peer-memory kernel, on a side stream) and LayerNorm / GDP
(ShardedLnGdp: one all-reduce of the flat parameter-gradient buffer), each rank on its own GPU,
against the same kernels run on the full batch on one GPU, and against the CPU oracle
(float64; the all-reduced dbias over both ranks' rows).  Row-local outputs computed
without reductions across CTAs match exactly (a row's result does not depend on the other
rows); dq/dv to their last bit, and the reduced gradients to f32 summation-order rounding.  NVLS is off (NCCL_NVLS_ENABLE=0) as for every multi-rank test here.
"""

import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _excess_bf16(a, e, rtol=2e-2, atol=2e-2):
    """max(|a - e| - (atol + rtol |e|)) over the elements: <= 0 when every element is within the
    16-bit tolerance."""
    a, e = a.double().cpu(), e.double().cpu()
    return float(((a - e).abs() - (atol + rtol * e.abs())).max())


def _excess_f32(a, e, rel=1e-4):
    """max(|a - e| - rel (|e| + max|e|)): <= 0 when every element is within the f32 tolerance."""
    a, e = a.double().cpu(), e.double().cpu()
    return float(((a - e).abs() - rel * (e.abs() + e.abs().max())).max())


def _worker(rank, world, port, queue):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        sys.path[:0] = [REPO, os.path.join(REPO, "colabfold-legacy-kernels_b200", "src")]
        import torch.distributed as dist
        import oracle
        from colabfold_legacy_kernels import torch_ops
        from colabfold_legacy_kernels.parallel import ShardedAttention, ShardedLnGdp, shard_rows
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method="tcp://127.0.0.1:%d" % port, rank=rank,
                                world_size=world, timeout=timedelta(seconds=60))
        errs = {}
        # attention, config C3's shape class at 24 rows x 256
        cfg = oracle.configs.scaled(oracle.configs.C3, n=24, s=256)
        inp = oracle.configs.make_attention_inputs(cfg, device="cpu")
        t = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in inp.items()}
        sa = ShardedAttention()
        r0, r1 = sa.rows(t["q"].shape[0])
        res = sa.step(*(t[x][r0:r1] for x in ("q", "k", "v")), t["bias"], t["kmask"][r0:r1],
                      t["dout"][r0:r1], t["scale"])
        out, lse = torch_ops.attention_fwd(t["q"], t["k"], t["v"], t["bias"], t["kmask"],
                                           t["scale"])
        dq, dk, dv, db = torch_ops.attention_bwd(t["q"], t["k"], t["v"], t["bias"], t["kmask"],
                                                 out, lse, t["dout"], t["scale"])
        torch.cuda.synchronize()
        errs["attn_out"] = float((res.out.float() - out[r0:r1].float()).abs().max())
        # dq, dv: sums of partials reduced in f32 in a timing-dependent order, then rounded to
        # 16 bits, so they may differ in the last bit
        errs["attn_dq_bf"] = float((res.dq.float() - dq[r0:r1].float()).abs().max()
                                   / dq.float().abs().max())
        errs["attn_dv_bf"] = float((res.dv.float() - dv[r0:r1].float()).abs().max()
                                   / dv.float().abs().max())
        errs["attn_dbias_rel"] = float((res.dbias - db).abs().max() / db.abs().max())
        # the same step with dbias reduce-scattered by query rows: this rank's rows of the sum
        res_rs = ShardedAttention(dbias_reduce="scatter").step(
            *(t[x][r0:r1] for x in ("q", "k", "v")), t["bias"], t["kmask"][r0:r1],
            t["dout"][r0:r1], t["scale"])
        s0, s1 = shard_rows(t["q"].shape[2], world, rank)
        torch.cuda.synchronize()
        assert tuple(res_rs.dbias.shape) == (db.shape[0], s1 - s0, db.shape[2])
        errs["attn_dbias_scatter_rel"] = float((res_rs.dbias - db[:, s0:s1]).abs().max()
                                               / db.abs().max())
        # ... and by this library's peer-memory kernel (CUDA-IPC buffers, rows read over
        # NVLink, added in rank order): two steps in a row, then the exchange alone replayed
        # twice from a CUDA graph; each must equal the NCCL reduce-scatter (two ranks: one
        # addition, the same in either order)
        from colabfold_legacy_kernels import cabi
        sa_peer = ShardedAttention(dbias_reduce="peer")
        for call in (1, 2):
            res_peer = sa_peer.step(*(t[x][r0:r1] for x in ("q", "k", "v")), t["bias"],
                                    t["kmask"][r0:r1], t["dout"][r0:r1], t["scale"])
            torch.cuda.synchronize()
            errs["attn_dbias_peer%d_rel" % call] = float(
                (res_peer.dbias - res_rs.dbias).abs().max() / db.abs().max())
        ex = sa_peer._exchange
        replay_out = torch.full_like(ex.out, float("nan"))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ex.reduce_scatter(out=replay_out)
        for call in (1, 2):
            graph.replay()
            torch.cuda.synchronize()
            errs["attn_dbias_peer_graph%d_rel" % call] = float(
                (replay_out - res_rs.dbias).abs().max() / db.abs().max())
        del graph
        errs["peer_status_rel"] = float(cabi.device_status())
        sa_peer.close()
        # the sharded results against the CPU oracle (float64): this rank's rows, and dbias
        # summed over both ranks' rows by the all-reduce
        c = {x: t[x].cpu() for x in ("q", "k", "v", "bias", "kmask", "dout")}
        r_out, r_lse = oracle.attention_fwd(c["q"], c["k"], c["v"], c["bias"], c["kmask"],
                                            t["scale"])
        r = oracle.attention_bwd(c["q"], c["k"], c["v"], c["bias"], c["kmask"], out.cpu(),
                                 lse.cpu(), c["dout"], t["scale"])
        errs["oracle_out_excess"] = _excess_bf16(res.out, r_out[r0:r1])
        errs["oracle_dq_excess"] = _excess_bf16(res.dq, r[0][r0:r1])
        errs["oracle_dk_excess"] = _excess_bf16(res.dk, r[1][r0:r1])
        errs["oracle_dv_excess"] = _excess_bf16(res.dv, r[2][r0:r1])
        errs["oracle_dbias_excess"] = _excess_f32(res.dbias, r[3])
        # LayerNorm + GDP, config C4's shape class at 3000 rows
        ci = oracle.configs.make_ln_gdp_inputs(oracle.configs.LnGdpConfig("c4_small", 3000, 128,
                                                                          256, 3), device=dev)
        sh = ShardedLnGdp()
        m0, m1 = sh.rows(3000)
        x, g, dy = ci["x"], ci["gamma"], ci["dy"]
        ln = sh.layer_norm_bwd(x[m0:m1], g, dy[m0:m1], 1e-5)
        gd = sh.gdp_bwd(x[m0:m1], ci["wp"], ci["bp"], ci["wg"], ci["bg"], ci["mask"][m0:m1],
                        ci["dout"][m0:m1])
        ln_ref = torch_ops.layer_norm_bwd(x, g, dy, 1e-5)
        gd_ref = torch_ops.gdp_bwd(x, ci["wp"], ci["bp"], ci["wg"], ci["bg"], ci["mask"],
                                   ci["dout"])
        torch.cuda.synchronize()
        errs["ln_dx"] = float((ln[0].float() - ln_ref[0][m0:m1].float()).abs().max())
        errs["gdp_dx"] = float((gd[0].float() - gd_ref[0][m0:m1].float()).abs().max())
        for name, a, b in (("dgamma_rel", ln[1], ln_ref[1]), ("dbeta_rel", ln[2], ln_ref[2]),
                           ("dwp_rel", gd[1], gd_ref[1]), ("dbp_rel", gd[2], gd_ref[2]),
                           ("dwg_rel", gd[3], gd_ref[3]), ("dbg_rel", gd[4], gd_ref[4])):
            errs[name] = float((a - b).abs().max() / b.abs().max())
        queue.put((rank, "ok", errs))
        dist.destroy_process_group()
    except Exception as e:
        queue.put((rank, "error", "%s: %s\n%s" % (type(e).__name__, e, traceback.format_exc())))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sharding_matches_one_gpu():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (s, e)) for r, s, e in (queue.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank in (0, 1):
        status, errs = results[rank]
        assert status == "ok", errs
        for name, err in errs.items():
            bound = 1e-5 if name.endswith("_rel") else (1e-2 if name.endswith("_bf") else 0.0)
            # *_excess: the oracle tolerance minus the error, <= 0 when within tolerance
            assert err <= bound, (rank, name, err)
