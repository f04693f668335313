"""Benchmark of the B200 Evoformer kernels -- prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json metric "tri-attn fwd+bwd TFLOP/s @N_res=768 ..."): one step is the
triangle-attention (starting node) forward + backward with pair bias and key mask at
N_res = 768, H = 4, d = 32, bf16 (config C3): out, lse = attn_fwd(q, k, v, bias, kmask);
dq, dk, dv, dbias = attn_bwd(...).  The 768 attention rows are sharded across the N GPUs
(strong scaling); every GPU holds the full bias and the per-GPU dbias partials are summed once
per step, by default reduce-scattered by query rows with the library's peer-memory kernel
(cfk_dbias_reduce_scatter; --dbias-reduce scatter|all for NCCL's reduce-scatter or
all-reduce).  Inputs are synthetic, drawn from seeded generators with the
configuration's shapes and distributions (oracle/configs.py), and resident in HBM.

value      = 695.8 GFLOP (algorithmic fwd+bwd flops of the whole job) / ms_per_step
e2e        = the same metric through the C ABI with pinned host buffers: every step copies
             q, k, v, bias, kmask, dout host->device and out, dq, dk, dv, dbias device->host
roofline   = the dominant kernel (the backward main kernel), achieved TFLOP/s from CUDA events
             around its launches against the measured burst bf16 peak (it runs inside a step of
             a few ms, not a seconds-long loop)
cpu_baseline = the CPU oracle (torch, fp32, all host threads) on a bounded sample of rows
Also reported: LayerNorm forward HBM GB/s and the gated dual projection on config C4.

--impl reference times the reference's CPU path for this workload: the reference ships GPU
kernels for sm_70/sm_75 only and no CPU implementation, so its semantics restated on the CPU
(oracle/, torch fp32, all host threads) stand in; every step is the whole 768-row workload.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "colabfold-legacy-kernels_b200" / "src"))
sys.path.insert(0, str(REPO))

METRIC = "tri-attn fwd+bwd TFLOP/s @N_res=768"
UNIT = "TFLOP/s"
N_RES, HEADS, HEAD_DIM = 768, 4, 32


def attn_flops(n, h, s, d):
    return 12 * n * h * s * s * d  # 4 n h s^2 d forward + 8 n h s^2 d backward


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        j = json.loads(p.read_text())
        return {"hbm_gbs": j["hbm_gbs"], "bf16": j["bf16_tflops"],
                "bf16_sustained": j.get("bf16_tflops_sustained", j["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def traffic_from_profiles(key):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary, if one exists."""
    p = REPO / "profiles" / "traffic.json"
    if p.is_file():
        try:
            return json.loads(p.read_text()).get(key)
        except (ValueError, OSError):
            return None
    return None


class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons of one GPU in a background
    thread while the timed region runs: NVML every ~2 ms (timed regions can be a few tens of
    ms), or nvidia-smi every 50 ms when NVML is unavailable.  Read-only."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, index, device=None):
        self.index = index
        self.device = device
        self.proc = None
        self.nvml = None
        self.lines = []
        self.samples = []  # (sm_mhz, reason bits)
        self.max_mhz = None
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        handle = None
        try:
            import torch
            p = torch.cuda.get_device_properties(self.device if self.device is not None
                                                 else self.index)
            bus = "%08X:%02X:%02X.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        return pynvml, handle

    def __enter__(self):
        try:
            pynvml, h = self._nvml_handle()
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.nvml = (pynvml, h, reasons)
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _poll_nvml(self):
        pynvml, h, reasons = self.nvml
        while not self.stop.is_set():
            try:
                self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                     int(reasons(h))))
            except Exception:
                return
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml:
            self.thread.join(timeout=2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], self.max_mhz, set()
        for mhz, bits in self.samples:
            sm.append(mhz)
            for name, bit in self.REASON_BITS.items():
                if bits & bit:
                    reasons.add(name)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml" if self.samples else "nvidia-smi"}


# ------------------------------------------------------------------------------------------
# CPU legs (oracle): the reference arm and the cpu_baseline field
# ------------------------------------------------------------------------------------------
def cpu_attention_sample(inputs_cpu, rows, reps=1):
    """Times the oracle's fp32 forward + backward on `rows` attention rows; returns
    (seconds per rep, flops per rep, threads)."""
    import torch
    import oracle
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    q, k, v, bias, kmask, dout = (inputs_cpu[x][:rows] if x not in ("bias",) else inputs_cpu[x]
                                  for x in ("q", "k", "v", "bias", "kmask", "dout"))
    scale = inputs_cpu["scale"]
    f32 = torch.float32
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        out, lse = oracle.attention_fwd_chunked(q, k, v, bias, kmask, scale, dtype=f32, chunk=4)
        for r0 in range(0, rows, 4):
            sl = slice(r0, r0 + 4)
            oracle.attention_bwd(q[sl], k[sl], v[sl], bias, kmask[sl], out[sl], lse[sl],
                                 dout[sl], scale, dtype=f32)
        times.append(time.perf_counter() - t0)
    n, h, s, d = q.shape
    return statistics.median(times), attn_flops(n, h, s, d), torch.get_num_threads()


def cpu_sample_inputs(rows):
    import oracle
    cfg = oracle.configs.C3
    # the same generator as the GPU run, on the CPU, for the first `rows` rows
    small = oracle.configs.AttnConfig(cfg.name, rows, cfg.h, cfg.s, cfg.d, cfg.seed, True,
                                      cfg.mask, cfg.from_pair)
    return oracle.configs.make_attention_inputs(small, device="cpu")


def run_reference(args, rank):
    """--impl reference: the CPU restatement, rank 0 only.  Every step is the whole C3 workload
    (all 768 attention rows, forward + backward), so the step time is measured, not scaled."""
    if rank != 0:
        return None
    rows = args.ref_rows or N_RES
    inputs = cpu_sample_inputs(rows)
    # warm-up: one small slice (thread pools, allocator), not a whole step
    cpu_attention_sample(cpu_sample_inputs(8), 8)
    secs = []
    flops = None
    threads = None
    t_all = time.perf_counter()
    for _ in range(args.steps):
        t, flops, threads = cpu_attention_sample(inputs, rows)
        secs.append(t)
    wall = time.perf_counter() - t_all
    sec = statistics.median(secs)
    value = flops / sec / 1e12
    sample = "all %d of %d attention rows of config C3 per step (fwd+bwd, fp32 torch on %d " \
             "threads)" % (rows, N_RES, threads)
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "wall_s_timed": wall,
        "config": {"workload": "tri_start_768 fwd+bwd (C3)", "n_res": N_RES, "heads": HEADS,
                   "head_dim": HEAD_DIM, "rows_per_step": rows,
                   "warmup_note": "one 8-row slice warms the thread pool; the W warm-up steps "
                                  "of a whole workload each are not repeated on the CPU"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU implementation and its GPU kernels are sm_70/sm_75 "
                "only; its semantics restated in oracle/ (torch CPU) are timed instead",
    }


# ------------------------------------------------------------------------------------------
# GPU leg
# ------------------------------------------------------------------------------------------
def device_status_max(dev, world):
    """The status word of this device, the largest over the ranks."""
    import torch
    import torch.distributed as dist
    from colabfold_legacy_kernels import cabi
    torch.cuda.synchronize(dev)
    code = cabi.device_status()
    if world > 1:
        t = torch.tensor([code], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        code = int(t.item())
    return code


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import oracle
    from colabfold_legacy_kernels import torch_ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = oracle.configs.C3
    full = oracle.configs.make_attention_inputs(cfg, device=dev)
    r0 = rank * N_RES // world
    r1 = (rank + 1) * N_RES // world
    if args.rows:
        r1 = r0 + args.rows  # profiling: a subset of the rows
    q, k, v, dout, kmask = (full[x][r0:r1].contiguous() for x in ("q", "k", "v", "dout", "kmask"))
    bias, scale = full["bias"], full["scale"]
    del full
    n = r1 - r0
    out = torch.empty_like(q)
    lse = torch.empty((n, HEADS, N_RES), dtype=torch.float32, device=dev)
    grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
             torch.empty((HEADS, N_RES, N_RES), dtype=torch.float32, device=dev))
    ws = torch_ops.attention_bwd_workspace(n, HEADS, N_RES, N_RES, HEAD_DIM, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    comm = torch.cuda.Stream(dev) if world > 1 else None

    # marks of one eager step: main stream t0 | fwd | prep | main | phase2 | t1, and the
    # dbias reduction on the comm stream ar0 | ar1 (all timed from t0)
    ev = {name: torch.cuda.Event(enable_timing=True)
          for name in ("t0", "fwd", "prep", "main", "phase2", "t1", "ar0", "ar1")}

    main_set = {"q": q, "k": k, "v": v, "dout": dout, "kmask": kmask, "bias": bias, "out": out,
                "lse": lse, "grads": grads}
    # dbias across ranks: reduce-scatter by query rows (each rank receives the summed rows of its
    # own residue rows, which is what a row-sharded module back-propagates into its pair rows),
    # or all-reduce
    reduce_mode = args.dbias_reduce if world > 1 and N_RES % world == 0 else "all"
    exchanges = []  # peer-memory exchanges (reduce_mode "peer"), closed at the end
    if world > 1 and reduce_mode == "peer":
        from colabfold_legacy_kernels.parallel import PeerDbiasExchange
        ex = PeerDbiasExchange.create_or_none((HEADS, N_RES, N_RES), dev)
        if ex is None:  # CUDA IPC unavailable on some rank: every rank uses NCCL instead
            reduce_mode = "scatter"
        else:
            exchanges.append(ex)
            # the backward writes dbias straight into this rank's exchange buffer
            grads = (grads[0], grads[1], grads[2], ex.dbias)
            main_set.update(grads=grads, dbias_red=ex.out, exchange=ex)
    if world > 1 and reduce_mode == "scatter":
        part = N_RES // world
        main_set["rs_src"] = torch.empty((world, HEADS, part, N_RES), dtype=torch.float32,
                                         device=dev)
        main_set["dbias_red"] = torch.empty((HEADS, part, N_RES), dtype=torch.float32,
                                            device=dev)

    def reduce_dbias(b):
        """The cross-rank sum of this step's dbias (comm stream): the rank's query rows into
        b["dbias_red"], or the whole of it in place."""
        if reduce_mode == "peer":
            b["exchange"].reduce_scatter(stream=torch.cuda.current_stream(dev))
        elif reduce_mode == "scatter":
            b["rs_src"].copy_(b["grads"][3].view(HEADS, world, part, N_RES).transpose(0, 1))
            dist.reduce_scatter_tensor(b["dbias_red"].view(-1), b["rs_src"].view(-1))
        else:
            dist.all_reduce(b["grads"][3])

    def step(record=False, b=main_set):
        stream = torch.cuda.current_stream(dev)
        bq, bk, bv, bb, bm, bo, bl, bd, bg = (b[x] for x in ("q", "k", "v", "bias", "kmask", "out",
                                                            "lse", "dout", "grads"))
        if record:
            ev["t0"].record(stream)
        torch_ops.attention_fwd(bq, bk, bv, bb, bm, scale, out=bo, lse=bl)
        if record:
            ev["fwd"].record(stream)
        torch_ops.attention_bwd(bq, bk, bv, bb, bm, bo, bl, bd, scale, workspace=ws,
                                grads=bg, phase=0)
        if record:
            ev["prep"].record(stream)
        torch_ops.attention_bwd(bq, bk, bv, bb, bm, bo, bl, bd, scale, workspace=ws,
                                grads=bg, phase=1)
        if record:
            ev["main"].record(stream)
        if world > 1:
            # dbias is final after the main kernel: reduce it while phase 2 runs (head dim 64's
            # conversion; empty for the head dims <= 32, whose main kernel completes dq, dk, dv)
            comm.wait_stream(stream)
            with torch.cuda.stream(comm):
                if record:
                    ev["ar0"].record(comm)
                reduce_dbias(b)
                if record:
                    ev["ar1"].record(comm)
        torch_ops.attention_bwd(bq, bk, bv, bb, bm, bo, bl, bd, scale, workspace=ws,
                                grads=bg, phase=2)
        if record:
            ev["phase2"].record(stream)
        if world > 1:
            stream.wait_stream(comm)
        if record:
            ev["t1"].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    marks = {name: [] for name in ev if name != "t0"}
    with ClockSampler(local_rank, dev) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        wall0 = time.perf_counter()
        for _ in range(args.steps):
            flush.zero_()  # untimed: evicts L2 between steps
            step(record=True)
            torch.cuda.synchronize()
            for name in marks:
                if world > 1 or name not in ("ar0", "ar1"):
                    marks[name].append(ev["t0"].elapsed_time(ev[name]))
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        wall = time.perf_counter() - wall0
        graph_ms = []
        if not args.no_graph:
            # The same step captured once in a CUDA graph (the dbias reduction included) and
            # replayed: the host's per-launch work leaves the timed region, which matters when
            # a step is short (many GPUs).  W warm-up replays, then K timed ones, L2 flushed
            # between them as above.
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                step()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph):
                step()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            for _ in range(args.warmup):
                graph.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            for _ in range(args.steps):
                flush.zero_()  # untimed: evicts L2 between steps
                g0.record()
                graph.replay()
                g1.record()
                torch.cuda.synchronize()
                graph_ms.append(g0.elapsed_time(g1))
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            del graph  # holds NCCL work: released before the process group goes away
    mean = lambda xs: sum(xs) / len(xs) if xs else 0.0
    # per-step phase durations from the marks (eager loop)
    pairs = {"fwd": (None, "fwd"), "bwd_prep": ("fwd", "prep"),
             "bwd_main": ("prep", "main"), "bwd_phase2": ("main", "phase2")}
    parts = {}
    for name, (a, b) in pairs.items():
        parts[name] = mean([mb - (marks[a][i] if a else 0.0) for i, mb in enumerate(marks[b])])
    if world > 1:
        parts["dbias_reduce"] = mean([e - b for b, e in zip(marks["ar0"], marks["ar1"])])
        # the part of the reduction that phase 2 does not hide: it ends after phase 2
        parts["dbias_reduce_exposed"] = mean([max(0.0, e - c) for e, c in
                                              zip(marks["ar1"], marks["phase2"])])
    ms = mean(marks["t1"])
    ms_graph = mean(graph_ms)
    names = sorted(parts)
    if world > 1:
        t = torch.tensor([ms, ms_graph] + [parts[k] for k in names], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = t.tolist()
        ms, ms_graph = vals[:2]
        parts = dict(zip(names, vals[2:]))
    ms_fwd, ms_bwd = parts["fwd"], parts["bwd_main"]
    ms_eager = ms
    if graph_ms:
        ms = ms_graph
    total_flops = attn_flops(N_RES, HEADS, N_RES, HEAD_DIM)
    value = total_flops / (ms * 1e-3) / 1e12

    if args.profile:
        return {"profile": True, "rows": n, "ms_per_step": ms, "ms_fwd": ms_fwd, "ms_bwd": ms_bwd}

    # ---------------- end to end through the C ABI with host buffers ----------------
    host = {x: torch.empty_like(t, device="cpu").pin_memory()
            for x, t in (("q", q), ("k", k), ("v", v), ("dout", dout), ("kmask", kmask),
                         ("bias", bias))}
    for x, t in (("q", q), ("k", k), ("v", v), ("dout", dout), ("kmask", kmask), ("bias", bias)):
        host[x].copy_(t)
    # dbias comes back as this rank's reduced result (its rows with the reduce-scatter)
    host_out = {x: torch.empty_like(t, device="cpu").pin_memory()
                for x, t in (("out", out), ("dq", grads[0]), ("dk", grads[1]), ("dv", grads[2]),
                             ("dbias", main_set.get("dbias_red", grads[3])))}
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out.values())
    # Steps are pipelined over two device buffer sets: step i's host->device copies (one
    # stream) overlap step i-1's compute and step i-2's device->host copies (two more streams);
    # every step still copies all its inputs in and all its results out inside the timed region.
    sets = [main_set, {x: (tuple(torch.empty_like(g) for g in t) if x == "grads"
                           else torch.empty_like(t)) for x, t in main_set.items()
                       if x != "exchange"}]
    if reduce_mode == "peer":
        ex = PeerDbiasExchange.create_or_none((HEADS, N_RES, N_RES), dev)
        if ex is None:
            raise RuntimeError("the second peer-memory exchange could not be set up")
        exchanges.append(ex)
        sets[1].update(grads=sets[1]["grads"][:3] + (ex.dbias,), dbias_red=ex.out, exchange=ex)
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_comp = torch.cuda.current_stream(dev)
    in_ev = [torch.cuda.Event() for _ in range(2)]
    comp_ev = [torch.cuda.Event() for _ in range(2)]
    out_ev = [torch.cuda.Event() for _ in range(2)]

    def pipelined(nsteps):
        for i in range(nsteps):
            b = sets[i % 2]
            with torch.cuda.stream(s_h2d):
                if i >= 2:
                    s_h2d.wait_event(comp_ev[i % 2])  # step i-2 is done reading this set
                for x in ("q", "k", "v", "dout", "kmask", "bias"):
                    b[x].copy_(host[x], non_blocking=True)
                in_ev[i % 2].record(s_h2d)
            s_comp.wait_event(in_ev[i % 2])
            if i >= 2:
                s_comp.wait_event(out_ev[i % 2])  # step i-2's results are copied out
            step(b=b)
            comp_ev[i % 2].record(s_comp)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(comp_ev[i % 2])
                for x, t in (("out", b["out"]), ("dq", b["grads"][0]), ("dk", b["grads"][1]),
                             ("dv", b["grads"][2]),
                             ("dbias", b.get("dbias_red", b["grads"][3]))):
                    host_out[x].copy_(t, non_blocking=True)
                out_ev[i % 2].record(s_d2h)
        s_comp.wait_stream(s_d2h)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pipelined(2)  # warm-up
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(s_comp)
    s_h2d.wait_stream(s_comp)
    s_d2h.wait_stream(s_comp)
    # as many steps as the device-timed loop (at least e2e_steps): the pipeline's fill (the
    # first step's inputs) and drain (the last step's results) are amortised like any step's
    e2e_n = max(args.steps, args.e2e_steps)
    pipelined(e2e_n)
    e1.record(s_comp)
    torch.cuda.synchronize()
    me2e = e0.elapsed_time(e1) / e2e_n
    if world > 1:
        t = torch.tensor([me2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        me2e = t.item()
        h2d_t = torch.tensor([h2d, d2h], device=dev, dtype=torch.float64)
        dist.all_reduce(h2d_t)
        h2d, d2h = (int(x) for x in h2d_t.tolist())
    e2e_value = total_flops / (me2e * 1e-3) / 1e12

    for ex in exchanges:  # collective: every rank closes them in the same order
        ex.close()
    pk = peaks()
    bwd_flops_launch = 8 * n * HEADS * N_RES * N_RES * HEAD_DIM
    achieved = bwd_flops_launch / (ms_bwd * 1e-3) / 1e12
    roofline = {
        "kernel": "attn_bwd_kernel<bf16, D=32> (cfk_attn_bwd phase 1)",
        "bound": "tensor", "achieved": achieved, "peak": pk["bf16"],
        "unit": "TFLOP/s", "frac": achieved / pk["bf16"],
        "peak_source": pk["source"] + " bf16_tflops (burst: the kernel runs inside a step of a "
                       "few ms)",
        "traffic": traffic_from_profiles("attn_bwd_tri768"),
        "flops_per_launch": bwd_flops_launch,
        "ms_per_launch": ms_bwd,
        "fwd_kernel": {"achieved": 4 * n * HEADS * N_RES * N_RES * HEAD_DIM / (ms_fwd * 1e-3) / 1e12,
                       "ms_per_launch": ms_fwd, "unit": "TFLOP/s",
                       "traffic": traffic_from_profiles("attn_fwd_tri768")},
    }
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "tri_start_768 fwd+bwd (C3)", "n_res": N_RES, "heads": HEADS,
                   "head_dim": HEAD_DIM, "rows_per_gpu": n, "parallelism": "rows%d" % world,
                   "l2": "flushed between steps (256 MB write, outside the timed events)",
                   "launch": ("one CUDA graph replay per step (the step captured once, the dbias "
                              "reduction included)" if ms_graph else "eager launches"),
                   "dbias_reduction": None if world == 1 else (
                       "reduce-scatter by query rows (each rank receives the summed dbias rows "
                       "of its own residue rows) by this library's peer-memory kernel "
                       "(cfk_dbias_reduce_scatter: CUDA-IPC buffers, one launch reading every "
                       "rank's rows over NVLink), side stream after the main kernel"
                       if reduce_mode == "peer" else
                       "NCCL reduce-scatter by query rows (each rank receives the summed dbias "
                       "rows of its own residue rows), side stream after the main kernel"
                       if reduce_mode == "scatter" else
                       "NCCL all-reduce, side stream after the main kernel"),
                   "eager_ms_per_step": ms_eager},
        "breakdown_ms": dict({k: round(v, 4) for k, v in parts.items()},
                             note="eager step, mean per step, max over ranks; dbias_reduce = the "
                                  "dbias collective on the comm stream (the reduce-scatter "
                                  "includes its rank-major gather copy), dbias_reduce_exposed = "
                                  "the time it runs past the end of phase 2 (empty at head dim "
                                  "32); bwd_prep = row statistics and the zeroing of dq, dk, dv"),
        # per step: attn_fwd, attn_bwd_prep, the dq/dk/dv zeroing, attn_bwd
        "gpu_launches": 4 * args.steps,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": me2e, "steps": e2e_n,
                "overlap": "double-buffered: host->device copies of step i+1 and device->host "
                           "copies of step i-1 run on two streams beside step i"},
        "roofline": roofline,
        "clocks": clocks.summary(),
        "wall_s_timed": wall,
        # the per-device status word after the timed work: nonzero if any kernel wait (a barrier
        # inside a kernel, or a wait for another GPU in the dbias exchange) ran past its limit
        "device_status": device_status_max(dev, world),
    }
    if world == 1 and not args.skip_extras:
        result["attention_views"] = bench_attention_views(dev, ms_eager)
        result["module"] = bench_module(dev, ms_eager)
        result["other_attention_configs"] = bench_other_attention(dev)
        result["layernorm"] = bench_layernorm(dev, pk)
        result["gdp"] = bench_gdp(dev, pk)
    elif not args.skip_extras:
        result["other_attention_configs"] = bench_other_attention(dev, world=world, rank=rank,
                                                                  reduce_mode=args.dbias_reduce)
        result.update(bench_ln_gdp_sharded(dev, pk, world))
    return result


def bench_attention_views(dev, packed_ms, steps=10):
    """The C3 step (fwd + the three backward launches) with q, k, v, dout, out, dq, dk, dv as
    [N,H,S,D] views of [S,N,H,D] storage: the layout of triangle attention around the ending
    node (attention over the first residue axis), passed to the kernels as strides
    (cfk_attn_*_strided) instead of transposed copies.  Eager launches, L2 flushed between
    steps; compared with the packed eager step of the same run."""
    import torch
    import oracle
    from colabfold_legacy_kernels import torch_ops

    full = oracle.configs.make_attention_inputs(oracle.configs.C3, device=dev)

    def as_view(t):  # same values, stored [S, N, H, D], viewed [N, H, S, D]
        return t.permute(2, 0, 1, 3).contiguous().permute(1, 2, 0, 3)

    def empty_view(t):
        return torch.empty_like(t.permute(2, 0, 1, 3)).permute(1, 2, 0, 3)

    q, k, v, dout = (as_view(full[x]) for x in ("q", "k", "v", "dout"))
    bias, kmask, scale = full["bias"], full["kmask"], full["scale"]
    del full
    n = q.shape[0]
    out = empty_view(q)
    lse = torch.empty((n, HEADS, N_RES), dtype=torch.float32, device=dev)
    grads = (empty_view(q), empty_view(k), empty_view(v),
             torch.empty((HEADS, N_RES, N_RES), dtype=torch.float32, device=dev))
    ws = torch_ops.attention_bwd_workspace(n, HEADS, N_RES, N_RES, HEAD_DIM, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]

    def step():
        evs[0].record()
        torch_ops.attention_fwd(q, k, v, bias, kmask, scale, out=out, lse=lse)
        evs[1].record()
        for ph in range(3):
            torch_ops.attention_bwd(q, k, v, bias, kmask, out, lse, dout, scale, workspace=ws,
                                    grads=grads, phase=ph)
            evs[2 + ph].record()

    for _ in range(3):
        step()
    names = ("fwd", "bwd_prep", "bwd_main", "bwd_phase2")
    ts, parts = [], {k: [] for k in names}
    for _ in range(steps):
        flush.zero_()
        step()
        torch.cuda.synchronize()
        ts.append(evs[0].elapsed_time(evs[4]))
        for i, name in enumerate(names):
            parts[name].append(evs[i].elapsed_time(evs[i + 1]))
    med = lambda xs: sorted(xs)[len(xs) // 2]
    ms = med(ts)
    return {"workload": "tri_end_768 fwd+bwd: [S,N,H,D] storage viewed as [N,H,S,D]",
            "metric": METRIC, "unit": UNIT,
            "value": round(attn_flops(n, HEADS, N_RES, HEAD_DIM) / (ms * 1e-3) / 1e12, 1),
            "ms_per_step": round(ms, 4), "packed_eager_ms_per_step": round(packed_ms, 4),
            "ms_per_launch": {name: round(med(t), 4) for name, t in parts.items()},
            "launch": "eager", "steps": steps,
            "l2": "flushed between steps (256 MB write, outside the timed events)"}


def bench_other_attention(dev, steps=10, world=1, rank=0, reduce_mode="all"):
    """BASELINE's other attention configurations, full size: C2 (MSA row attention with pair
    bias, [512, 8, 256, 32], fwd + the three backward launches) and C5 (triangle attention at
    N_res = 2048, forward only).  With N ranks the attention rows are sharded as in the
    headline step (every GPU holds the full bias); C2's per-rank dbias partials are summed by an
    NCCL reduce-scatter by query rows (reduce_mode "scatter") or all-reduce on a side stream
    after the main kernel.  Eager launches,
    L2 flushed between steps (untimed); whole-job TFLOP/s over the slowest rank's mean step."""
    import torch
    import torch.distributed as dist
    import oracle
    from colabfold_legacy_kernels import torch_ops
    from colabfold_legacy_kernels.parallel import scatter_dbias, shard_rows

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    comm = torch.cuda.Stream(dev) if world > 1 else None

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ts = []
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        ms = sum(ts) / len(ts)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms

    out = {}
    for cfg, backward in ((oracle.configs.C2, True), (oracle.configs.C5, False)):
        t = oracle.configs.make_attention_inputs(cfg, device=dev)
        n_all, h, s, d = t["q"].shape
        r0, r1 = shard_rows(n_all, world, rank)
        q, k, v, kmask = (t[x][r0:r1].contiguous() for x in ("q", "k", "v", "kmask"))
        bias, scale = t["bias"], t["scale"]
        dout = t["dout"][r0:r1].contiguous() if backward else None
        del t
        n = r1 - r0
        o = torch.empty_like(q)
        lse = torch.empty((n, h, s), dtype=torch.float32, device=dev)
        if backward:
            ws = torch_ops.attention_bwd_workspace(n, h, s, s, d, dev)
            grads = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
                     torch.empty((h, s, s), dtype=torch.float32, device=dev))
            scatter = world > 1 and reduce_mode == "scatter" and s % world == 0
            ex = None
            if world > 1 and reduce_mode == "peer" and s % world == 0:
                from colabfold_legacy_kernels.parallel import PeerDbiasExchange
                ex = PeerDbiasExchange.create_or_none((h, s, s), dev)
                if ex is None:  # every rank falls back to NCCL together
                    scatter = True
                else:
                    grads = grads[:3] + (ex.dbias,)

            def fn():
                stream = torch.cuda.current_stream(dev)
                torch_ops.attention_fwd(q, k, v, bias, kmask, scale, out=o, lse=lse)
                args = (q, k, v, bias, kmask, o, lse, dout, scale)
                torch_ops.attention_bwd(*args, workspace=ws, grads=grads, phase=0)
                torch_ops.attention_bwd(*args, workspace=ws, grads=grads, phase=1)
                if world > 1:
                    comm.wait_stream(stream)
                    with torch.cuda.stream(comm):
                        if ex is not None:
                            ex.reduce_scatter(stream=comm)
                        elif scatter:
                            scatter_dbias(grads[3], world, rank)
                        else:
                            dist.all_reduce(grads[3])
                torch_ops.attention_bwd(*args, workspace=ws, grads=grads, phase=2)
                if world > 1:
                    stream.wait_stream(comm)
            flops = attn_flops(n_all, h, s, d)
        else:
            def fn():
                torch_ops.attention_fwd(q, k, v, bias, kmask, scale, out=o, lse=lse)
            flops = 4 * n_all * h * s * s * d
        ms = timed(fn)
        out[cfg.name] = {"shape": [n_all, h, s, d], "rows_per_gpu": n,
                         "pass": "fwd+bwd" if backward else "fwd",
                         "ms": round(ms, 4), "tflops": round(flops / (ms * 1e9), 1),
                         "gflop": round(flops / 1e9, 1)}
        if backward and world > 1:
            out[cfg.name]["dbias_reduction"] = "%s, %d MB f32, side stream after the main " \
                "kernel" % ("peer-memory reduce-scatter by query rows (cfk_dbias_reduce_scatter)"
                            if ex is not None else "NCCL reduce-scatter by query rows" if scatter
                            else "NCCL all-reduce", round(h * s * s * 4 / 1e6, 1))
            if ex is not None:
                ex.close()
        del q, k, v, o, lse, fn
        if backward:
            del ws, grads, dout
    out["n_gpus"] = world
    out["scaling"] = "strong (the configuration's rows sharded over the GPUs)"
    out["launch"] = "eager"
    out["l2"] = "flushed between steps (256 MB write, outside the timed events)"
    return out


def bench_module(dev, attn_ms, steps=10):
    """The triangle-attention module (modules.TriangleAttention: LayerNorm, projections, gated
    attention, output projection) forward + backward on a C3-sized pair representation
    z [768, 768, 128] with 5 % padded residues, around the starting and the ending node.  Eager,
    L2 flushed between steps; `attention_kernels_ms` is the packed attention step of the same
    run, so the rest is the module's LayerNorm, GEMMs and elementwise work."""
    import torch
    from colabfold_legacy_kernels.modules import TriangleAttention

    g = torch.Generator(device=dev).manual_seed(2)
    z = torch.randn(N_RES, N_RES, 128, device=dev, generator=g).bfloat16().requires_grad_(True)
    res = (torch.rand(N_RES, device=dev, generator=g) >= 0.05).float()
    mask = res[:, None] * res[None, :]
    m = TriangleAttention(128, HEADS, HEAD_DIM, device=dev)
    dout = torch.randn(N_RES, N_RES, 128, device=dev, generator=g).bfloat16()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    for ending in (False, True):
        def step():
            # fresh gradients every step, as a training step with zero_grad(set_to_none=True)
            # takes them (no accumulation into earlier steps' .grad)
            m.zero_grad(set_to_none=True)
            z.grad = None
            m(z, mask, ending=ending).backward(dout)

        for _ in range(3):
            step()
        ts = []
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        out["ending" if ending else "starting"] = round(sorted(ts)[len(ts) // 2], 4)
    m2 = N_RES * N_RES
    gemm = 3 * 2 * m2 * 128 * (3 * HEADS * HEAD_DIM + HEADS + 2 * HEADS * HEAD_DIM)
    return {"workload": "triangle-attention module fwd+bwd, z [768,768,128] bf16, 5 % padded",
            "ms_per_step": out, "attention_kernels_ms": round(attn_ms, 4),
            "flops_per_step": attn_flops(N_RES, HEADS, N_RES, HEAD_DIM) + gemm,
            "tflops": {k: round((attn_flops(N_RES, HEADS, N_RES, HEAD_DIM) + gemm) / (v * 1e9), 1)
                       for k, v in out.items()},
            "launch": "eager", "steps": steps,
            "l2": "flushed between steps (256 MB write, outside the timed events)"}


def bench_ln_gdp_sharded(dev, pk, world, steps=20):
    """LayerNorm and GDP on config C4 with its rows sharded over the N ranks (ShardedLnGdp: the
    forwards are row-local, each backward ends with one all-reduce of the parameter gradients).
    Whole-job rates: C4's algorithmic bytes / flops over the slowest rank's time."""
    import torch
    import torch.distributed as dist
    import oracle
    from colabfold_legacy_kernels import torch_ops
    from colabfold_legacy_kernels.parallel import ShardedLnGdp
    inp = oracle.configs.make_ln_gdp_inputs(oracle.configs.C4, device=dev)
    m, c = inp["x"].shape
    n = inp["wp"].shape[1]
    sh = ShardedLnGdp()
    m0, m1 = sh.rows(m)
    x, dy, mask, dout = (inp[k][m0:m1].contiguous() for k in ("x", "dy", "mask", "dout"))
    gamma, beta, wp, bp, wg, bg = (inp[k] for k in ("gamma", "beta", "wp", "bp", "wg", "bg"))
    del inp

    def slowest(ms):
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    # Consecutive launches rotate over K copies of this rank's shard, K x (x bytes) >= 3 x L2,
    # so every launch streams its inputs from HBM although one shard may fit in L2 at N >= 4.
    xbytes = x.numel() * x.element_size()
    nsets = max(1, min(16, -(-3 * L2_BYTES // xbytes)))
    sets = [(x, dy, mask, dout)] + [tuple(t.clone() for t in (x, dy, mask, dout))
                                    for _ in range(nsets - 1)]
    stats = [torch_ops.layer_norm_fwd(st[0], gamma, beta, 1e-5, return_stats=True) for st in sets]
    outs = [torch.empty((m1 - m0, n), dtype=x.dtype, device=dev) for _ in sets]
    ms = {"ln_fwd": slowest(_stream_ms_sets(
              [lambda i=i: torch_ops.layer_norm_fwd(sets[i][0], gamma, beta, 1e-5,
                                                    out=stats[i][0]) for i in range(nsets)],
              steps)),
          "ln_bwd": slowest(_stream_ms_sets(
              [lambda i=i: sh.layer_norm_bwd(sets[i][0], gamma, sets[i][1], 1e-5, stats[i][1],
                                             stats[i][2]) for i in range(nsets)], steps)),
          "gdp_fwd": slowest(_stream_ms_sets(
              [lambda i=i: torch_ops.gdp_fwd(sets[i][0], wp, bp, wg, bg, sets[i][2],
                                             out=outs[i]) for i in range(nsets)], steps)),
          "gdp_bwd": slowest(_stream_ms_sets(
              [lambda i=i: sh.gdp_bwd(sets[i][0], wp, bp, wg, bg, sets[i][2], sets[i][3])
               for i in range(nsets)], steps))}
    note = ("rows sharded over %d GPUs; backward parameter gradients all-reduced once (NCCL); "
            "launches back to back rotating over %d copies of the %d MB per-GPU x shard (and its "
            "dy/dout/mask), %d MB >= 3 x L2, so inputs stream from HBM"
            % (world, nsets, xbytes >> 20, (nsets * xbytes) >> 20))

    def gbs(nbytes, t):
        return nbytes / (t * 1e-3) / 1e9

    def tfs(flops, t):
        return flops / (t * 1e-3) / 1e12

    return {
        "layernorm": {"sharding": note, "n_gpus": world,
                      "fwd": {"metric": "LayerNorm fwd HBM GB/s [1M x 128] bf16", "unit": "GB/s",
                              "value": gbs(oracle.layer_norm.bytes_fwd(m, c), ms["ln_fwd"]),
                              "ms": ms["ln_fwd"]},
                      "bwd": {"metric": "LayerNorm bwd HBM GB/s [1M x 128] bf16", "unit": "GB/s",
                              "value": gbs(oracle.layer_norm.bytes_bwd(m, c), ms["ln_bwd"]),
                              "ms": ms["ln_bwd"]}},
        "gdp": {"sharding": note, "n_gpus": world,
                "fwd": {"metric": "GDP fwd TFLOP/s [1M x 128 -> 256] bf16", "unit": "TFLOP/s",
                        "value": tfs(oracle.gdp.flops_fwd(m, c, n), ms["gdp_fwd"]),
                        "ms": ms["gdp_fwd"]},
                "bwd": {"metric": "GDP bwd TFLOP/s [1M x 128 -> 256] bf16", "unit": "TFLOP/s",
                        "value": tfs(oracle.gdp.flops_bwd(m, c, n), ms["gdp_bwd"]),
                        "ms": ms["gdp_bwd"]}},
    }


L2_NOTE = "inputs larger than L2 (x 268 MB), launches back to back, no flush"
L2_BYTES = 126 * 1000 * 1000


def _stream_ms_sets(fns, steps):
    """Mean device time per call of `steps` calls enqueued back to back between two events,
    call i running fns[i % len(fns)] (each on its own copy of the inputs)."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(max(3, len(fns))):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    e0.record()
    for i in range(steps):
        fns[i % len(fns)]()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _stream_ms(fn, steps):
    """Mean device time per call of `steps` calls enqueued back to back between two events.

    The C4 inputs are larger than the 126 MB L2, so consecutive calls stream from HBM without a
    flush; enqueueing them back to back keeps the host's per-call launch latency out of the
    device time (an isolated call would include it)."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def bench_gdp(dev, pk, steps=20):
    """Gated dual projection forward and backward on config C4 (M = 1024*1024, K = 128, the
    a/b pair as one call with N = 256, bf16).  Roofline: the larger of bytes / measured HBM
    bandwidth and flops / measured dense bf16 peak (burst), divided by the measured time."""
    import torch
    import oracle
    from colabfold_legacy_kernels import torch_ops
    inp = oracle.configs.make_ln_gdp_inputs(oracle.configs.C4, device=dev)
    x, wp, bp, wg, bg, mask, dout = (inp[k] for k in ("x", "wp", "bp", "wg", "bg", "mask", "dout"))
    m, kk = x.shape
    n = wp.shape[1]
    out = torch.empty((m, n), dtype=x.dtype, device=dev)
    res = {"l2": L2_NOTE}

    def line(name, ms, flops, nbytes, traffic):
        t_bound = max(nbytes / (pk["hbm_gbs"] * 1e9), flops / (pk["bf16"] * 1e12))
        return {"metric": "GDP %s TFLOP/s [1M x 128 -> 256] bf16" % name,
                "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms,
                "hbm_gbs": nbytes / (ms * 1e-3) / 1e9,
                "roofline": {"bound": "hbm" if nbytes / pk["hbm_gbs"] / 1e9 >= flops / pk["bf16"] / 1e12
                             else "tensor", "algorithmic_bytes": nbytes, "flops": flops,
                             "bound_ms": t_bound * 1e3, "frac": t_bound * 1e3 / ms,
                             "traffic": traffic,
                             "peaks": {"hbm_gbs": pk["hbm_gbs"], "bf16_tflops": pk["bf16"]}}}

    ms = _stream_ms(lambda: torch_ops.gdp_fwd(x, wp, bp, wg, bg, mask, out=out), steps)
    fwd_bytes = 2 * (m * kk + m * n + m + 2 * kk * n + 2 * n)
    res["fwd"] = line("fwd", ms, oracle.gdp.flops_fwd(m, kk, n), fwd_bytes,
                      traffic_from_profiles("gdp_fwd_c4"))
    nbytes = cabi_gdp_workspace(m, kk, n)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    ms = _stream_ms(lambda: torch_ops.gdp_bwd(x, wp, bp, wg, bg, mask, dout, workspace=ws),
                    steps)
    # LayerNorm fused into the forward (cfk_ln_gdp_fwd) against LayerNorm then GDP
    z, gamma, beta = inp["x"], inp["gamma"], inp["beta"]
    y = torch.empty_like(z)
    ms_fused = _stream_ms(lambda: torch_ops.ln_gdp_fwd(z, gamma, beta, 1e-5, wp, bp, wg, bg, mask,
                                                       out=out), steps)
    ms_two = _stream_ms(lambda: (torch_ops.layer_norm_fwd(z, gamma, beta, 1e-5, out=y),
                                 torch_ops.gdp_fwd(y, wp, bp, wg, bg, mask, out=out)), steps)
    fused_bytes = 2 * (m * kk + m * n + m + 2 * kk * n + 2 * n) + 8 * kk
    t_fused = max(fused_bytes / (pk["hbm_gbs"] * 1e9),
                  oracle.gdp.flops_fwd(m, kk, n) / (pk["bf16"] * 1e12))
    res["ln_fwd_fused"] = {
        "metric": "LayerNorm + GDP fwd [1M x 128 -> 256] bf16, one kernel", "ms": ms_fused,
        "unit": "ms", "separate_ms": ms_two,
        "roofline": {"bound": "hbm", "algorithmic_bytes": fused_bytes, "bound_ms": t_fused * 1e3,
                     "frac": t_fused * 1e3 / ms_fused}}
    bwd_bytes = 2 * (m * kk + m * n + m * kk + m) + 4 * (2 * kk * n + 2 * n)
    dx_t, dw_t = traffic_from_profiles("gdp_bwd_dx_c4"), traffic_from_profiles("gdp_bwd_dw_c4")
    res["bwd"] = line("bwd", ms, oracle.gdp.flops_bwd(m, kk, n), bwd_bytes,
                      dx_t + dw_t if dx_t and dw_t else None)
    return res


def cabi_gdp_workspace(m, k, n):
    from colabfold_legacy_kernels import cabi
    return cabi.workspace_size("cfk_gdp_bwd_workspace_size", m, k, n)


def bench_layernorm(dev, pk, steps=20):
    """LayerNorm forward and backward on config C4 (M = 1024*1024, C = 128, bf16)."""
    import torch
    import oracle
    from colabfold_legacy_kernels import torch_ops
    inp = oracle.configs.make_ln_gdp_inputs(oracle.configs.C4, device=dev)
    x, gamma, beta, dy = inp["x"], inp["gamma"], inp["beta"], inp["dy"]
    m, c = x.shape
    y = torch.empty_like(x)
    mean = torch.empty(m, device=dev)
    rstd = torch.empty(m, device=dev)
    res = {"l2": L2_NOTE}
    ms = _stream_ms(lambda: torch_ops.layer_norm_fwd(x, gamma, beta, 1e-5, out=y), steps)
    gbs = oracle.layer_norm.bytes_fwd(m, c) / (ms * 1e-3) / 1e9
    res["fwd"] = {"metric": "LayerNorm fwd HBM GB/s [1M x 128] bf16", "value": gbs, "unit": "GB/s",
                  "ms": ms, "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"],
                                         "unit": "GB/s", "frac": gbs / pk["hbm_gbs"],
                                         "traffic": traffic_from_profiles("ln_fwd_c4")}}
    y, mean, rstd = torch_ops.layer_norm_fwd(x, gamma, beta, 1e-5, return_stats=True)
    ws = torch.empty(1 << 22, dtype=torch.uint8, device=dev)
    ms = _stream_ms(lambda: torch_ops.layer_norm_bwd(x, gamma, dy, 1e-5, mean=mean, rstd=rstd,
                                                     workspace=ws), steps)
    gbs = oracle.layer_norm.bytes_bwd(m, c) / (ms * 1e-3) / 1e9
    res["bwd"] = {"metric": "LayerNorm bwd HBM GB/s [1M x 128] bf16", "value": gbs,
                  "unit": "GB/s", "ms": ms, "roofline": {"bound": "hbm", "achieved": gbs,
                                                         "peak": pk["hbm_gbs"], "unit": "GB/s",
                                                         "frac": gbs / pk["hbm_gbs"],
                                                         "traffic": traffic_from_profiles("ln_bwd_c4")}}
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="reference arm: attention rows per step (default: all 768)")
    ap.add_argument("--skip-extras", action="store_true", help="skip LayerNorm/GDP lines")
    ap.add_argument("--dbias-reduce", choices=("peer", "scatter", "all"), default="peer",
                    help="N > 1: dbias reduce-scatter by query rows through this library's "
                         "peer-memory kernel (default) or NCCL, or an NCCL all-reduce")
    ap.add_argument("--no-graph", action="store_true",
                    help="time the eager step only (no CUDA-graph replay)")
    ap.add_argument("--skip-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--rows", type=int, default=0,
                    help="profiling only: attention rows on this GPU instead of 768/N")
    ap.add_argument("--profile", action="store_true",
                    help="profiling only: time the attention steps and stop (no e2e/extras/cpu)")
    ap.add_argument("--profile-extras", action="store_true",
                    help="profiling only: run the LayerNorm and GDP lines (C4) alone, 2 steps")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile_extras:
        import torch
        dev = torch.device("cuda", 0)
        pk = peaks()
        print(json.dumps({"profile": True, "layernorm": bench_layernorm(dev, pk, steps=2),
                          "gdp": bench_gdp(dev, pk, steps=2)}), flush=True)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            sys.exit("bench.py: --gpus %d needs torchrun with %d processes" % (args.gpus, args.gpus))
    if args.impl == "reference":
        res = run_reference(args, rank)
        if rank == 0:
            print(json.dumps(res), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        res = run_ours(args, rank, world, local_rank)
        if rank == 0 and world == 1 and not args.skip_cpu and not args.profile:
            # size the sample to ~5 s per repetition (3 repetitions, ~15 s of CPU work)
            probe = cpu_sample_inputs(32)
            t32, _, _ = cpu_attention_sample(probe, 32)
            rows = int(max(8, min(N_RES, 32 * 5.0 / max(t32, 1e-3))))
            inputs = cpu_sample_inputs(rows)
            sec, flops, threads = cpu_attention_sample(inputs, rows, reps=3)
            res["cpu_baseline"] = {
                "value": flops / sec / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": "%d of %d rows of C3 fwd+bwd, oracle/ fp32 torch, median of 3 (%.2f s)"
                          % (rows, N_RES, sec)}
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
