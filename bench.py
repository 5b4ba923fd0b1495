"""Benchmark of the gated delta-rule hot path (driver contract: one JSON line).

Headline workload (BASELINE configs[1] at its largest batch, which is also
config 4 at N=1): GDN decode, B=1024, Hqk=16, Hv=32, d_k=d_v=128, fp32 state
(4.3 GB of algorithmic traffic per step: larger than L2, so no flush is
needed), one decode token per step, state updated in place.  With N GPUs the
32 value heads are sharded Hv/N per GPU (fixed total work: strong scaling)
and the outputs are all-gathered over NVLink (NCCL) once per step.

  value : algorithmic state GB/s of the whole job, device-timed (CUDA events,
          max over ranks), inputs resident in HBM.
  e2e   : the same metric through the public API with host buffers: every step
          copies its q/k/v/g/beta from pinned host memory, launches, and reads
          o back to pinned host memory inside the timed region.
``--impl reference`` times the reference's CPU recurrence (the oracle port,
all host threads) on the same metric.
"""
from __future__ import annotations

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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
# More hardware work queues than streams in use (main, gather side stream, one
# per destination rank, NCCL): with the default 8, a stream-memory wait on one
# queue can stall unrelated streams mapped onto it.  Set before CUDA starts.
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import __graft_entry__ as graft  # noqa: E402

METRIC = "GDN decode state GB/s"
UNIT = "GB/s"
B, HQK, HV, D = 1024, 16, 32, 128  # B is overridable with --batch (profiling runs)
HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return j["hbm_gbs"], j.get("bf16_tflops", BF16_FALLBACK_TFLOPS), "measured"
    return HBM_FALLBACK_GBS, BF16_FALLBACK_TFLOPS, "fallback"


# DRAM traffic of one headline decode launch (B=1024), from an ncu capture:
# dram__bytes_read.sum + dram__bytes_write.sum of decode_kernel at B=256
# (1,021.9 MB; the full B=1024 launch is too large to capture under the
# profiling size rule), scaled x4 by the sequences processed.  The capture
# command and its figures are in profiles/gdn_decode_B1024.md.
DECODE_TRAFFIC_BYTES_B1024 = 4_087_588_352


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.25)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo")
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------- CPU
def cpu_sample(seconds: float = 10.0):
    """The oracle port (C, all host threads) on a bounded sample of the
    headline workload: batches of 32 sequences x 32 value heads, one decode
    step each, repeated for about `seconds`.  Returns (GB/s, threads, text)."""
    orc = graft.oracle()
    inputs = graft.submodule("inputs")
    Bs = 32
    x = inputs.make_decode_inputs(1, Bs, HQK, HV, D, seed=0)
    args = [t.float().numpy() for t in (x.q, x.k, x.v, x.g, x.beta)]
    S = x.state.numpy()
    orc.gdn_decode_steps(*args, S)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        orc.gdn_decode_steps(*args, S)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = n * graft.submodule("inputs").gdn_decode_bytes(Bs, HQK, HV, D, D) / el / 1e9
    sample = (f"{n} one-step calls of B={Bs} (of {B}) x Hv={HV} heads, d=128, "
              f"{el:.1f} s of CPU work")
    return gbs, orc.num_threads(), sample


def run_reference(args, world, rank):
    if rank != 0:
        return
    inputs = graft.submodule("inputs")
    orc = graft.oracle()
    Bs = 32
    x = inputs.make_decode_inputs(1, Bs, HQK, HV, D, seed=0)
    a = [t.float().numpy() for t in (x.q, x.k, x.v, x.g, x.beta)]
    S = x.state.numpy()
    for _ in range(args.warmup):
        orc.gdn_decode_steps(*a, S)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.gdn_decode_steps(*a, S)
    el = time.perf_counter() - t0
    gbs = args.steps * inputs.gdn_decode_bytes(Bs, HQK, HV, D, D) / el / 1e9
    ms = el / args.steps * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (BASELINE distributions, seed 0)",
        "config": {"workload": "GDN decode B=1024 Hqk=16 Hv=32 d=128 (CPU: bounded sample of "
                               f"B={Bs} sequences per step)", "global_batch": B,
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": orc.num_threads(),
                         "kind": "port",
                         "sample": f"each step: one decode step of B={Bs} x Hv={HV} heads "
                                   "through the C restatement of gdn_decode_reference"},
        "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- GPU
def run_gpu(args, world, rank, local):
    pkg = graft.package()
    inputs = graft.submodule("inputs")
    sharded = graft.submodule("sharded")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shard = sharded.shard_heads(HV, HQK, world, rank)
    hv, hq = shard.h1 - shard.h0, shard.hq1 - shard.hq0
    pool = 4  # distinct token inputs cycled through the steps
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    state = torch.randn((B, hv, D, D), generator=gen, device=dev) * 0.02
    toks = []
    for i in range(pool):
        x = inputs.make_decode_inputs(1, B, hq, hv, D, seed=100 * rank + i, device=dev,
                                      state_std=0.0)
        toks.append([x.q[0], x.k[0], x.v[0], x.g[0], x.beta[0]])
    # two output buffers: the all-gather of step i (NCCL stream) overlaps the
    # decode of step i + 1; step i + 2 waits for it before reusing the buffer
    outs = [torch.empty((B, hv, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    out = outs[0]
    gmode = args.gather if args.gather != "auto" else "fused"
    ce = world > 1 and gmode == "ce"
    fused = world > 1 and gmode == "fused"
    res = args.sm_reserve if args.sm_reserve >= 0 else min(48, 8 * world if world > 2 else 16)
    res = res if (world > 1 and gmode == "nccl") else 0
    if fused:
        # the decode kernel writes every output row into every rank's
        # head-major buffer itself (NVLink stores) and signals arrival
        fg = sharded.FusedGather(B, HV, D, shard.h0, hv, torch.bfloat16, dev)
        fsteps = [[fg.decode_step(slot, *t, state) for slot in range(2)] for t in toks]
    else:
        steps = [pkg.DecodeStep(*t, state, out=outs[0], sm_reserve=res) for t in toks]
        steps2 = [pkg.DecodeStep(*t, state, out=outs[1], sm_reserve=res) for t in toks]
    gbufs = [torch.empty((world, B, hv, D), dtype=torch.bfloat16, device=dev) for _ in range(2)] \
        if world > 1 else None
    gather_buf = gbufs[0] if world > 1 else None
    works = [None, None]

    def launch(i):
        if fused:
            fg.launch(fsteps[i % pool])
        else:
            (steps if i % 2 == 0 else steps2)[i % pool]()

    if ce:
        # copy-engine all-gather (no SMs): push on a side stream after each
        # decode; the decode of step i + 2 waits for step i's copies to leave
        # its output buffer
        pg = sharded.PeerGather(B * hv * D, torch.bfloat16, dev)
        side = torch.cuda.Stream(dev)
        peer_streams = [torch.cuda.Stream(dev) for _ in range(world)]  # one copy engine each
        ev_dec = [torch.cuda.Event() for _ in range(2)]
        ev_out_free = [None, None]
        gstep = [0]

    def gather(i):
        if fused or gmode == "none":
            return  # done inside the decode kernel (or not at all)
        if world > 1 and ce:
            gstep[0] += 1
            ms_ = torch.cuda.current_stream(dev)
            ev_dec[i % 2].record(ms_)
            for ps in peer_streams:
                ps.wait_event(ev_dec[i % 2])
            pg.push(outs[i % 2], gstep[0], peer_streams=peer_streams)
            for ps in peer_streams:
                side.wait_stream(ps)
            ev = torch.cuda.Event()
            ev.record(side)
            ev_out_free[i % 2] = ev
            pg.wait(gstep[0], side)      # every rank's slice of this step has landed
            pg.release(gstep[0], side)   # (the bench consumes nothing further)
        elif world > 1:
            works[i % 2] = dist.all_gather_into_tensor(gbufs[i % 2].view(-1), outs[i % 2].view(-1),
                                                       async_op=True)

    def settle(i):
        if gmode == "none":
            return
        if ce:
            ev = ev_out_free[i % 2]
            if ev is not None:
                torch.cuda.current_stream(dev).wait_event(ev)
                ev_out_free[i % 2] = None
            return
        w = works[i % 2]
        if w is not None:
            w.wait()
            works[i % 2] = None

    def join():
        if ce:
            torch.cuda.current_stream(dev).wait_stream(side)

    def one_step(i):
        settle(i)
        launch(i)
        gather(i)
        if args.no_overlap:
            settle(i)

    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        one_step(i)
    settle(args.warmup)
    settle(args.warmup + 1)
    join()
    pkg.check_device_status(dev)
    use_graph = world > 1 and not args.no_graph and gmode == "nccl"
    n_kev = min(args.steps, 200) if use_graph else args.steps
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_kev)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def eager_steps(n, record):
        for i in range(n):
            settle(i)
            if record:
                kev[i][0].record(stream)
            launch(i)
            if record:
                kev[i][1].record(stream)
            gather(i)
            if args.no_overlap:
                settle(i)
        settle(n)
        settle(n + 1)
        join()

    graph = None
    if use_graph:
        # N > 1: steps are short (the state per GPU shrinks as 1/N), so the host
        # loop of one library launch + one NCCL call per step would bound the
        # rate.  Capture G steps (decode + overlapped all-gather) in a CUDA
        # graph and replay it; kernel durations come from an eager pass.
        barrier(world)
        torch.cuda.synchronize(dev)
        eager_steps(n_kev, True)
        torch.cuda.synchronize(dev)
        kern_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / n_kev, world, dev)
        G = 10
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                eager_steps(G, False)
        torch.cuda.current_stream(dev).wait_stream(cap)
        graph.replay()
        torch.cuda.synchronize(dev)
        replays = max(1, args.steps // G)
        timed_steps = replays * G
    else:
        timed_steps = args.steps
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        e0.record(stream)
        if graph is not None:
            for _ in range(replays):
                graph.replay()
        else:
            eager_steps(args.steps, True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    pkg.check_device_status(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / timed_steps, world, dev)
    if graph is None:
        kern_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in kev) / args.steps, world, dev)
    total_bytes = inputs.gdn_decode_bytes(B, HQK, HV, D, D)
    value = total_bytes / (ms * 1e-3) / 1e9
    local_bytes = inputs.gdn_decode_bytes(B, hq, hv, D, D)
    hbm, bf16, peak_kind = peaks()
    achieved = local_bytes / (kern_ms * 1e-3) / 1e9

    # ---- parity of one more step (and of its gather) against the C oracle
    def gathered(i):  # [N, B, hv, d] rank-major slot holding step i's gathered outputs
        if gmode == "none":
            return None
        if fused:
            return fg.wait(fg.step).view(B, world, hv, D).permute(1, 0, 2, 3)
        if ce:
            return pg.buf[gstep[0] % 2].view(world, B, hv, D)
        return gbufs[i % 2]

    last_out = (lambda: fg.local_out(fg.step % 2)) if fused else (lambda: outs[0])
    parity = decode_parity(graft.oracle(), toks, state, last_out, launch, gather, settle, join,
                           gathered, shard, world, rank, dev)

    # ---- e2e through the public API with pinned host buffers
    e2e_steps = min(args.steps, 200)
    e2e_ms, h2d, d2h = run_e2e(pkg, toks, state, hv, world, rank, dev, e2e_steps)
    e2e_val = total_bytes / (e2e_ms * 1e-3) / 1e9

    extras = {}
    cpu = None
    if not args.no_extras:
        if world == 1:
            extras = run_extras(pkg, inputs, dev, hbm, bf16, with_cpu=not args.no_cpu)
        else:
            extras = run_seqpar_extras(pkg, inputs, dev, world, rank, bf16)
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, cores, sample = cpu_sample(args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": sample}
    if rank != 0:
        return
    # per launch: a rank streams 1/N of the heads, so 1/N of the B=1024 traffic
    traffic = DECODE_TRAFFIC_BYTES_B1024 // world if B == 1024 else None
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": timed_steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (BASELINE distributions, seed 0)",
        "config": {"workload": "GDN decode (BASELINE configs[1], B=1024; config 4 at N>1)",
                   "global_batch": B, "Hqk": HQK, "Hv": HV, "d_k": D, "d_v": D,
                   "io_dtype": "bf16", "state": "fp32 in place",
                   "parallelism": f"value-head shard x{world}" + (
                       {"ce": " + copy-engine all-gather of o", "nccl": " + NCCL all-gather of o",
                        "fused": " + all-gather of o fused into the decode kernel (NVLink stores)",
                        "none": " (diagnostic: no all-gather)"}[gmode]
                       if world > 1 else ""),
                   "l2": "inputs larger than L2 (4.3 GB state), no flush"},
        "tokens_per_s": round(B / (ms * 1e-3), 1),
        "pct_of_8TBs_per_gpu": round(100 * value / world / 8000.0, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic,
                     "peak_kind": f"{peak_kind} (burst copy)",
                     "kernel": "decode_kernel<128,128,bf16,GDN>",
                     "algorithmic_bytes_per_launch": local_bytes},
        "e2e": {"value": round(e2e_val, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "copies": "pinned host <-> device every step, double-buffered on two copy "
                          "streams (H2D of step i+1 and D2H of step i overlap decode); "
                          "h2d counts all ranks, d2h is rank 0's gathered output"},
        "parity": parity,
        "gpu_launches": timed_steps,
        "cuda_graph": graph is not None,
        "allgather_overlapped": world > 1 and not args.no_overlap,
        "allgather": {"ce": "copy-engine push over NVLink (IPC)", "nccl": "NCCL",
                      "fused": "decode kernel stores into every rank's buffer over NVLink (IPC)",
                      "none": None}[gmode]
                     if world > 1 else None,
        "sm_reserve": res,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "extras": extras,
    }
    print(json.dumps(line), flush=True)


def decode_parity(orc, toks, state, last_out, launch, gather, settle, join, gathered, shard,
                  world, rank, dev, n_seq=8):
    """One more decode step after the timed region, through the same launch
    and gather path as the timed steps, checked against the C oracle (the
    restatement of gdn_decode_reference, pytorch_reference_gdn.py:38-91) on
    a fixed sample of ``n_seq`` sequences x every local value head: this
    rank's outputs and state rows, and on rank 0 the gathered [B, Hv, d]
    rows of every rank's heads.  Tolerances: outputs rtol 2e-2 / atol 1e-2,
    state max-abs 1e-3."""
    import numpy as np
    rtol, atol, s_atol = 2e-2, 1e-2, 1e-3
    torch.cuda.synchronize(dev)
    idx = torch.linspace(0, B - 1, n_seq).round().long().to(dev)
    q, k, v, g, beta = [t.index_select(0, idx).float().cpu() for t in toks[0]]
    S0 = state.index_select(0, idx).cpu().numpy()
    launch(0)          # bound to toks[0]
    gather(0)
    settle(0)
    join()
    torch.cuda.synchronize(dev)
    o_dev = last_out().index_select(0, idx).float().cpu().numpy()
    S1 = state.index_select(0, idx).cpu().numpy()
    o_ref, s_ref = orc.gdn_decode_steps(q[None], k[None], v[None], g[None], beta[None], S0)
    o_ref = o_ref[0]

    def excess(x, r):  # > 0 where |x - r| exceeds atol + rtol |r|
        return float((np.abs(x - r) - (atol + rtol * np.abs(r))).max())

    err_o = float(np.abs(o_dev - o_ref).max())
    err_s = float(np.abs(S1 - s_ref).max())
    bad = max(excess(o_dev, o_ref), err_s - s_atol)
    err_g = None
    if world > 1 and gathered(0) is not None:
        mine = torch.from_numpy(o_ref).to(dev)                       # [n, hv, d]
        allref = torch.empty((world,) + tuple(mine.shape), dtype=mine.dtype, device=dev)
        dist.all_gather_into_tensor(allref.view(-1), mine.reshape(-1))
        hv = mine.shape[1]
        ref_full = allref.permute(1, 0, 2, 3).reshape(n_seq, world * hv, -1).cpu().numpy()
        got = gathered(0).index_select(1, idx)                       # [N, n, hv, d]
        got_full = got.permute(1, 0, 2, 3).reshape(n_seq, world * hv, -1).float().cpu().numpy()
        err_g = float(np.abs(got_full - ref_full).max())
        bad = max(bad, excess(got_full, ref_full))
        t = torch.tensor([err_o, err_s, bad], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        err_o, err_s, bad = (float(x) for x in t.tolist())
    return {"checked": True, "oracle": "C restatement of gdn_decode_reference (fp32)",
            "sample": f"{n_seq} sequences x all {shard.h1 - shard.h0} local value heads per rank"
                      + (", gathered rows on rank 0" if world > 1 else ""),
            "max_abs_o": err_o, "max_abs_S": err_s, "max_abs_o_gathered": err_g,
            "tol": {"o_rtol": rtol, "o_atol": atol, "S_atol": s_atol}, "ok": bad <= 0.0}


def run_e2e(pkg, toks, state, hv, world, rank, dev, n_steps):
    """End-to-end decode through the public API (DecodeStep; with N > 1 the
    NCCL all-gather and head-major permute of ShardedGDNDecoder.gather) with
    host buffers.  Every step copies its q/k/v/g/beta from pinned host memory
    and reads its output back (rank 0 reads the gathered [B, Hv, d]).  The
    copies are double-buffered on two copy streams: step i+1's inputs travel
    while step i decodes, and step i's output travels while step i+1 decodes.
    Returns (ms per step, max over ranks; H2D bytes per step over all ranks;
    D2H bytes per step)."""
    pool = len(toks)
    host = [[t.cpu().pin_memory() for t in tk] for tk in toks]
    dev_in = [[torch.empty_like(t) for t in toks[0]] for _ in range(2)]
    outs = [torch.empty((B, hv, D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    steps = [pkg.DecodeStep(*dev_in[s], state, out=outs[s]) for s in range(2)]
    reads = world == 1 or rank == 0
    o_host = [torch.empty((B, HV if world > 1 else hv, D), dtype=torch.bfloat16).pin_memory()
              for _ in range(2)]
    full = [torch.empty((B, HV, D), dtype=torch.bfloat16, device=dev) for _ in range(2)] \
        if world > 1 else None
    gbuf = torch.empty((world, B, hv, D), dtype=torch.bfloat16, device=dev) if world > 1 else None
    comp = torch.cuda.current_stream(dev)
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [None, None]   # step i's decode (and gather) done with dev_in[s], outs[s]
    ev_read = [None, None]   # step i's output copied to the host

    def step(i):
        s = i % 2
        if ev_used[s] is not None:
            h2d_s.wait_event(ev_used[s])
        with torch.cuda.stream(h2d_s):
            for hsrc, ddst in zip(host[i % pool], dev_in[s]):
                ddst.copy_(hsrc, non_blocking=True)
        ev_in[s].record(h2d_s)
        comp.wait_event(ev_in[s])
        if ev_read[s] is not None:
            comp.wait_event(ev_read[s])
        res = steps[s]()
        if world > 1:
            dist.all_gather_into_tensor(gbuf.view(-1), res.view(-1))
            full[s].view(B, world, hv, D).copy_(gbuf.permute(1, 0, 2, 3))
            res = full[s]
        ev = torch.cuda.Event()
        ev.record(comp)
        ev_used[s] = ev
        if reads:
            d2h_s.wait_event(ev)
            with torch.cuda.stream(d2h_s):
                o_host[s].copy_(res, non_blocking=True)
            ev2 = torch.cuda.Event()
            ev2.record(d2h_s)
            ev_read[s] = ev2

    for i in range(3):
        step(i)
    torch.cuda.synchronize(dev)
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(comp)
    h2d_s.wait_event(f0)
    for i in range(n_steps):
        step(i)
    comp.wait_stream(d2h_s)
    comp.wait_stream(h2d_s)
    f1.record(comp)
    torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(f0.elapsed_time(f1) / n_steps, world, dev)
    h2d = sum(t.numel() * t.element_size() for t in host[0]) * world
    d2h = o_host[0].numel() * o_host[0].element_size()
    return ms, h2d, d2h


def _time_graph(fn, reps=20, warm=3):
    """Captures fn() in a CUDA graph and returns ms per replay."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    for _ in range(warm):
        g.replay()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def _cpu_timed(fn, min_seconds=1.0):
    """Runs fn() once to warm, then repeats it for at least ``min_seconds``;
    returns seconds per call."""
    fn()
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return el / n


def cpu_baselines(inputs):
    """The oracle port (C, all host threads) timed on bounded samples of the
    secondary configs; each entry becomes the ``cpu_baseline`` of the matching
    extras line.  Returns {name: cpu_baseline dict}."""
    orc = graft.oracle()
    cores = orc.num_threads()
    out = {}
    # config 0: all 64 steps at B=8 (the whole config)
    x = inputs.make_decode_inputs(64, 8, HQK, HV, D, seed=0)
    a = [t.float().numpy() for t in (x.q, x.k, x.v, x.g, x.beta)]
    el = _cpu_timed(lambda: orc.gdn_decode_steps(*a, x.state.numpy()))
    out["config0"] = {"value": round(8 * 64 / el, 1), "unit": "tokens/s", "cores": cores,
                      "kind": "port", "sample": "the whole config: 64 steps at B=8, 32 heads",
                      "seconds": round(el, 3)}
    # config 1: one step at B=64 (whole) and a B=64 sample of B=256
    x = inputs.make_decode_inputs(1, 64, HQK, HV, D, seed=1)
    a = [t.float().numpy() for t in (x.q, x.k, x.v, x.g, x.beta)]
    el = _cpu_timed(lambda: orc.gdn_decode_steps(*a, x.state.numpy()))
    gbs = inputs.gdn_decode_bytes(64, HQK, HV) / el / 1e9
    for b_ in (64, 256):
        out[f"config1_B{b_}"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores,
                                 "kind": "port",
                                 "sample": "one decode step at B=64" + (" (of 256)" if b_ > 64 else ""),
                                 "seconds": round(el, 3)}
    # config 2: the whole config, 64 float64 KDA steps at B=64
    x = inputs.make_decode_inputs(64, 64, 32, 32, D, kda=True, seed=2)
    a = [t.float().numpy() for t in (x.q, x.k, x.v, x.g, x.beta)]
    el = _cpu_timed(lambda: orc.kda_decode_steps(*a, x.state.numpy()))
    out["config2"] = {"value": round(64 * inputs.kda_decode_bytes(64, 32, 32) / el / 1e9, 3),
                      "unit": "GB/s", "cores": cores, "kind": "port",
                      "sample": "the whole config: 64 steps at B=64, 32 heads, float64",
                      "seconds": round(el, 3)}
    # config 3: the sequential T=4096 recurrence for 16 value heads of one sequence
    p = inputs.make_prefill_inputs(1, 4096, 8, 16, D, seed=3)
    el = _cpu_timed(lambda: orc.gdn_prefill(p.q, p.k, p.v, p.g, p.beta))
    fl = inputs.gdn_prefill_flops(1, 4096, 8, 16, D, 64)
    out["config3"] = {"value": round(fl / el / 1e12, 5), "unit": "TFLOP/s (chunked-form equivalent)",
                      "head_tokens_per_s": round(16 * 4096 / el, 1), "cores": cores, "kind": "port",
                      "sample": "sequential recurrence over T=4096 for b=0, 16 value heads "
                                "(8 q/k heads) of the 4 x 32", "seconds": round(el, 3)}
    # KDA prefill: float64 recurrence over T=4096 for 8 heads of one sequence
    p = inputs.make_kda_prefill_inputs(1, 4096, 8, 8, D, seed=3)
    el = _cpu_timed(lambda: orc.kda_prefill(p.q, p.k, p.v, p.g, p.beta))
    out["kda_prefill"] = {"value": round(8 * 4096 / el, 1), "unit": "head-tokens/s", "cores": cores,
                          "kind": "port", "sample": "float64 recurrence over T=4096 for b=0, "
                                                    "8 of the 4 x 32 heads", "seconds": round(el, 3)}
    return out


def run_extras(pkg, inputs, dev, hbm, bf16, with_cpu=True):
    """Secondary BASELINE configs, device-timed (not the headline), each with
    the CPU oracle port timed beside it on a stated sample."""
    ex = {}
    cpu = cpu_baselines(inputs) if with_cpu else {}
    # config 0: B=8, 64 sequential steps per CUDA-graph replay
    x = inputs.make_decode_inputs(64, 8, HQK, HV, D, seed=0, device=dev)
    st = x.state.clone()
    o = torch.empty((8, HV, D), dtype=torch.bfloat16, device=dev)
    s0 = [pkg.DecodeStep(x.q[t], x.k[t], x.v[t], x.g[t], x.beta[t], st, out=o) for t in range(64)]
    ms = _time_graph(lambda: [s() for s in s0])
    ex["config0_gdn_B8_64steps"] = {
        "tokens_per_s": round(8 * 64 / (ms * 1e-3), 1), "us_per_step": round(ms * 1e3 / 64, 3),
        "state_GBps_equiv": round(64 * inputs.gdn_decode_bytes(8, HQK, HV) / (ms * 1e-3) / 1e9, 1),
        "note": "16.8 MB state is L2-resident; GB/s-equivalent can exceed HBM peak",
        "cpu_baseline": cpu.get("config0")}
    del x, st, s0
    # config 1 sweep (B=64, 256): one decode step, state in place, 100
    # iterations; the graph holds 20 consecutive steps so that its own launch
    # is not counted against every step
    for b in (64, 256):
        x = inputs.make_decode_inputs(1, b, HQK, HV, D, seed=1, device=dev)
        st = x.state.clone()
        s1 = pkg.DecodeStep(x.q[0], x.k[0], x.v[0], x.g[0], x.beta[0], st)
        ms = _time_graph(lambda: [s1() for _ in range(20)], reps=5) / 20
        gbs = inputs.gdn_decode_bytes(b, HQK, HV) / (ms * 1e-3) / 1e9
        ex[f"config1_gdn_B{b}"] = {"GBps": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4),
                                   "us": round(ms * 1e3, 2), "steps_per_graph": 20,
                                   "cpu_baseline": cpu.get(f"config1_B{b}")}
        del x, st, s1
    # sustained headline decode: >= 1 s of back-to-back steps, clocks sampled
    x = inputs.make_decode_inputs(1, B, HQK, HV, D, seed=1, device=dev)
    st = x.state.clone()
    s1 = pkg.DecodeStep(x.q[0], x.k[0], x.v[0], x.g[0], x.beta[0], st)
    for _ in range(20):
        s1()
    n_sus = 1600
    a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(dev.index or 0) as clk:
        a_.record()
        for _ in range(n_sus):
            s1()
        b_.record()
        torch.cuda.synchronize()
    ms = a_.elapsed_time(b_) / n_sus
    gbs = inputs.gdn_decode_bytes(B, HQK, HV) / (ms * 1e-3) / 1e9
    ex[f"sustained_gdn_B{B}"] = {"GBps": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4),
                                 "steps": n_sus, "seconds": round(ms * n_sus / 1e3, 3),
                                 "clocks": clk.summary(),
                                 "note": "the headline kernel timed over >= 1 s back to back "
                                         "(burst peak as denominator)"}
    del x, st, s1
    # optional fp16 state (half the streamed state bytes) at the headline size
    x = inputs.make_decode_inputs(1, B, HQK, HV, D, seed=1, device=dev)
    st = x.state.to(torch.float16)
    s1 = pkg.DecodeStep(x.q[0], x.k[0], x.v[0], x.g[0], x.beta[0], st)
    ms = _time_graph(lambda: [s1() for _ in range(10)], reps=5) / 10
    byts = inputs.gdn_decode_bytes(B, HQK, HV) - B * HV * D * D * 4  # state at 2 bytes
    ex[f"fp16_state_gdn_B{B}"] = {"GBps": round(byts / (ms * 1e-3) / 1e9, 1),
                                  "frac_of_hbm": round(byts / (ms * 1e-3) / 1e9 / hbm, 4),
                                  "tokens_per_s": round(B / (ms * 1e-3), 1), "us": round(ms * 1e3, 2),
                                  "note": "option, not the BASELINE fp32 state",
                                  "cpu_baseline": cpu.get("config1_B256")}
    del x, st, s1
    # config 2: KDA B=64, H=32, 64 steps per replay
    x = inputs.make_decode_inputs(64, 64, 32, 32, D, kda=True, seed=2, device=dev)
    st = x.state.clone()
    o = torch.empty((64, 32, D), dtype=torch.bfloat16, device=dev)
    s2 = [pkg.DecodeStep(x.q[t], x.k[t], x.v[t], x.g[t], x.beta[t], st, out=o, kda=True)
          for t in range(64)]
    ms = _time_graph(lambda: [s() for s in s2], reps=10)
    gbs = 64 * inputs.kda_decode_bytes(64, 32, 32) / (ms * 1e-3) / 1e9
    ex["config2_kda_B64_64steps"] = {"GBps": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4),
                                     "us_per_step": round(ms * 1e3 / 64, 2),
                                     "note": "268 MB state; partly L2-resident across steps",
                                     "cpu_baseline": cpu.get("config2")}
    del x, st, s2
    # config 3: chunked prefill
    p = inputs.make_prefill_inputs(4, 4096, HQK, HV, D, seed=3, device=dev)
    fs = torch.empty((4, HV, D, D), dtype=torch.float32, device=dev)
    po = torch.empty((4, 4096, HV, D), dtype=torch.bfloat16, device=dev)
    fn = lambda: pkg.gdn_prefill(p.q, p.k, p.v, p.g, p.beta, out=po, final_state=fs)
    ms = _time_events(fn, reps=10)
    fl = inputs.gdn_prefill_flops(4, 4096, HQK, HV, D, 64)
    tf = fl / (ms * 1e-3) / 1e12
    ex["config3_prefill_B4_T4096"] = {"ms": round(ms, 4), "TFLOPs": round(tf, 1),
                                      "frac_of_bf16_peak": round(tf / bf16, 4),
                                      "chunked_form_GFLOP": round(fl / 1e9, 2),
                                      "cpu_baseline": cpu.get("config3")}
    del p, fs, po
    # KDA prefill at the config 3 length, H=32: the chunked tensor-core form
    # (the default at d = 128) and the recurrent form (state on chip)
    p = inputs.make_kda_prefill_inputs(4, 4096, 32, 32, D, seed=3, device=dev)
    fs = torch.empty((4, 32, D, D), dtype=torch.float32, device=dev)
    po = torch.empty((4, 4096, 32, D), dtype=torch.bfloat16, device=dev)
    fn = lambda: pkg.kda_prefill(p.q, p.k, p.v, p.g, p.beta, out=po, final_state=fs, form="chunked")
    ms = _time_events(fn, reps=10)
    fl = inputs.gdn_prefill_flops(4, 4096, 32, 32, D, 64)  # same chunked-form FLOPs, Hqk = Hv
    tf = fl / (ms * 1e-3) / 1e12
    ex["kda_prefill_B4_T4096_H32"] = {
        "ms": round(ms, 4), "tokens_per_s": round(4 * 4096 / (ms * 1e-3), 1),
        "TFLOPs": round(tf, 1), "frac_of_bf16_peak": round(tf / bf16, 4),
        "chunked_form_GFLOP": round(fl / 1e9, 2),
        "GBps_compulsory": round(inputs.kda_prefill_bytes(4, 4096, 32, 32, D) / (ms * 1e-3) / 1e9, 1),
        "note": "chunked form on tcgen05 (64-token chunks, per-channel decays in the operands)",
        "cpu_baseline": cpu.get("kda_prefill")}
    fn = lambda: pkg.kda_prefill(p.q, p.k, p.v, p.g, p.beta, out=po, final_state=fs, form="recurrent")
    ms = _time_events(fn, reps=5, warm=2)
    ex["kda_prefill_recurrent_B4_T4096_H32"] = {
        "ms": round(ms, 4), "tokens_per_s": round(4 * 4096 / (ms * 1e-3), 1),
        "fp32_TOPs_recurrent": round(inputs.kda_recurrent_ops(4, 4096, 32, D) / (ms * 1e-3) / 1e12, 2),
        "note": "recurrent form on CUDA cores (every d); no tensor cores",
        "cpu_baseline": cpu.get("kda_prefill")}
    del p, fs, po
    return ex


def _time_events(fn, reps=10, warm=3):
    """ms per call of fn(), CUDA events on the current stream after warm-up."""
    for _ in range(warm):
        fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_seqpar_extras(pkg, inputs, dev, world, rank, bf16):
    """N > 1: config 3 (B=4, T=4096) split by time over the N ranks with
    sharded.gdn_prefill_seqpar, timed (CUDA events, max over ranks) and checked
    on a sampled head against the sequential oracle over the full T."""
    import numpy as np
    sharded = graft.submodule("sharded")
    Bp, Tp = 4, 4096
    p = inputs.make_prefill_inputs(Bp, Tp, HQK, HV, D, seed=3, device=dev)
    seg = Tp // world
    t0 = rank * seg
    t1 = Tp if rank == world - 1 else t0 + seg
    x = [t[:, t0:t1].contiguous() for t in (p.q, p.k, p.v, p.g, p.beta)]
    fn = lambda: sharded.gdn_prefill_seqpar(*x)
    barrier(world)
    ms = max_over_ranks(_time_events(fn, reps=5, warm=2), world, dev)
    single = max_over_ranks(_time_events(lambda: pkg.gdn_prefill(p.q, p.k, p.v, p.g, p.beta), reps=5),
                            world, dev)
    fl = inputs.gdn_prefill_flops(Bp, Tp, HQK, HV, D, 64)
    # parity: sequence b=1, value head 5 (q/k head 2) over the full T
    bs, hs, hqs = 1, 5, 5 // (HV // HQK)
    o, S = fn()
    torch.cuda.synchronize(dev)
    cpu = [t.float().cpu() for t in (p.q, p.k, p.v, p.g, p.beta)]
    o_ref, s_ref = graft.oracle().gdn_prefill(cpu[0][bs:bs + 1, :, hqs:hqs + 1],
                                              cpu[1][bs:bs + 1, :, hqs:hqs + 1],
                                              cpu[2][bs:bs + 1, :, hs:hs + 1],
                                              cpu[3][bs:bs + 1, :, hs:hs + 1],
                                              cpu[4][bs:bs + 1, :, hs:hs + 1])
    got = o[bs, :, hs].float().cpu().numpy()
    ref = o_ref[0, t0:t1, 0]
    err_o = float(np.abs(got - ref).max())
    bad = float((np.abs(got - ref) - (1e-2 + 2e-2 * np.abs(ref))).max())
    err_s = float(np.abs(S[bs, hs].cpu().numpy() - s_ref[0, 0]).max()) if rank == world - 1 else 0.0
    t = torch.tensor([err_o, err_s, bad], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    err_o, err_s, bad = (float(v) for v in t.tolist())
    tf = fl / (ms * 1e-3) / 1e12
    return {"seqpar_prefill_B4_T4096": {
        "ms": round(ms, 4), "TFLOPs_chunked_form": round(tf, 1),
        "frac_of_bf16_peak_per_job": round(tf / bf16, 4),
        "single_gpu_prefill_ms": round(single, 4), "speedup_vs_one_gpu": round(single / ms, 3),
        "segments": f"{world} x T={seg}",
        "parity": {"checked": True, "sample": "b=1, value head 5, every token; final state on "
                                              "the last rank", "oracle": "sequential fp32 recurrence",
                   "max_abs_o": err_o, "max_abs_S": err_s, "ok": bad <= 0.0 and err_s < 1e-3}}}


def run_prefill(args, world, rank, local):
    """BASELINE config 3 (B=4, T=4096, Hqk=16, Hv=32, chunk 64) as its own
    line: chunked-form TFLOP/s, device-timed; used for profiling the prefill."""
    pkg = graft.package()
    inputs = graft.submodule("inputs")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    Bp, Tp = 4, 4096
    p = inputs.make_prefill_inputs(Bp, Tp, HQK, HV, D, seed=3, device=dev)
    fs = torch.empty((Bp, HV, D, D), dtype=torch.float32, device=dev)
    po = torch.empty((Bp, Tp, HV, D), dtype=torch.bfloat16, device=dev)
    fn = lambda: pkg.gdn_prefill(p.q, p.k, p.v, p.g, p.beta, out=po, final_state=fs)
    for _ in range(args.warmup):
        fn()
    pkg.check_device_status(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    a.record()
    for _ in range(args.steps):
        fn()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / args.steps
    hbm, bf16, kind = peaks()
    fl = inputs.gdn_prefill_flops(Bp, Tp, HQK, HV, D, 64)
    tf = fl / (ms * 1e-3) / 1e12
    if rank == 0:
        print(json.dumps({"metric": "GDN prefill chunked-form TFLOP/s", "value": round(tf, 2),
                          "unit": "TFLOP/s", "ms_per_step": round(ms, 4), "steps": args.steps,
                          "warmup": args.warmup, "n_gpus": world,
                          "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": bf16,
                                       "unit": "TFLOP/s", "frac": round(tf / bf16, 4),
                                       "peak_kind": f"{kind} (burst bf16 GEMM)"},
                          "config": {"workload": "GDN prefill B=4 T=4096 Hqk=16 Hv=32 d=128 C=64"}}),
              flush=True)


def run_kda_prefill(args, world, rank, local):
    """KDA prefill (per-channel gate) at B=4, H=32, T=--seq (default 4096, the
    config 3 length) as its own line, device-timed; used for profiling."""
    pkg = graft.package()
    inputs = graft.submodule("inputs")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    Bp, Tp, H = 4, args.seq, 32
    p = inputs.make_kda_prefill_inputs(Bp, Tp, H, H, D, seed=3, device=dev)
    fs = torch.empty((Bp, H, D, D), dtype=torch.float32, device=dev)
    po = torch.empty((Bp, Tp, H, D), dtype=torch.bfloat16, device=dev)
    fn = lambda: pkg.kda_prefill(p.q, p.k, p.v, p.g, p.beta, out=po, final_state=fs,
                                 form=args.kda_form)
    for _ in range(args.warmup):
        fn()
    pkg.check_device_status(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    a.record()
    for _ in range(args.steps):
        fn()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / args.steps
    if rank == 0:
        print(json.dumps({"metric": "KDA prefill tokens/s", "value": round(Bp * Tp / (ms * 1e-3), 1),
                          "unit": "tokens/s", "ms_per_step": round(ms, 4), "steps": args.steps,
                          "warmup": args.warmup, "n_gpus": world,
                          "form": args.kda_form,
                          "TFLOPs_chunked_form": round(
                              inputs.gdn_prefill_flops(Bp, Tp, H, H, D, 64) / (ms * 1e-3) / 1e12, 1),
                          "config": {"workload": f"KDA prefill B={Bp} T={Tp} H={H} d={D}"}}),
              flush=True)


def main():
    global B
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--sm-reserve", type=int, default=-1,
                    help="SMs the decode leaves to the overlapped all-gather (N>1); default "
                         "by N: 16 at 2, 32 at 4, 48 at 8 (measured best on B200 x8)")
    ap.add_argument("--gather", default="auto", choices=("auto", "fused", "ce", "nccl", "none"),
                    help="N>1 output all-gather: fused into the decode kernel (NVLink stores, the "
                         "default), copy engines over NVLink (ce) or NCCL; none (diagnostic: "
                         "outputs stay on their rank)")
    ap.add_argument("--no-graph", action="store_true",
                    help="N>1: launch every step from the host instead of replaying a CUDA graph")
    ap.add_argument("--no-overlap", action="store_true",
                    help="N>1: run each step's all-gather after its decode, not overlapped")
    ap.add_argument("--workload", default="decode", choices=("decode", "prefill", "kda_prefill"),
                    help="decode (headline, configs[1]/4), prefill (config 3) or kda_prefill "
                         "(B=4, H=32, T=--seq); the last two for profiling")
    ap.add_argument("--seq", type=int, default=4096, help="kda_prefill sequence length")
    ap.add_argument("--kda-form", default="chunked", choices=("chunked", "recurrent"),
                    help="kda_prefill workload: the chunked tensor-core form or the recurrent form")
    ap.add_argument("--batch", type=int, default=B,
                    help="decode batch (default 1024, the headline; smaller for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    B = args.batch
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "prefill":
            graft.build()
            run_prefill(args, world, rank, local)
        elif args.workload == "kda_prefill":
            graft.build()
            run_kda_prefill(args, world, rank, local)
        else:
            graft.build()
            run_gpu(args, world, rank, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
