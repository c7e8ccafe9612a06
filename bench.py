#!/usr/bin/env python
"""Benchmark of the decode-sampling path (BASELINE metric: sampled rows/s and logits GB/s
against HBM peak at V=262144, plus the p50 step latency at B=1).

Workload (one "step" = one gs_sample over the batch): configuration C4, the throughput
batch, B=4096 rows x V=262144 float32 logits (4 GiB, larger than L2), soft cap 30,
256-id penalty history at 1.1/0.5/0.3, a 4096-state constraint bitmask at 2% density,
temperature 0.8, topK 50, topP 0.95.  Rows are independent (one PRNG stream each), so each
of the N GPUs samples its own C4 batch of 4096 rows (weak scaling: the work per GPU is
fixed, the global batch is 4096·N; no collective on the data path).  Launched as one
process per GPU (torchrun).

Also reported on rank 0: the other configurations at their own batch sizes (C2 on the
histogram path, C3, C4 without its constraint mask in float32 and bfloat16, C4 bfloat16),
each with its dominant kernels' HBM roofline; the p50/p95 step latency of C1 (B=1, 256
sequential steps); the end-to-end rate through the host-buffer entry point
(gs_sample_host); the CPU oracle timed on the host cores as a baseline; the constraint
bitmask builder and the int2 LM head.  With N > 1 GPUs, every rank also runs C5 in the
vocabulary-sharded layout (each GPU one slice of every row, one all-gather of the
per-shard records per step).

`--impl reference` times the reference sampler's CPU restatement (oracle/oracle.cpp; the
reference is TypeScript and there is no Node runtime on the machine) on all host threads.

`--only NAME` runs one workload a few times and exits (the driver the profiles/ captures
run under ncu): C1..C5 (`--rows`, `--calls`, `--no-mask`, `--no-history`, `--topk`,
`--dtype`), `lm-head` / `lm-head-sample` (`--rows`, `--calls`) or `mask-builder`
(`--states`, `--calls`).
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
PKG = "gemma-webgpu-engine_b200"
VOCAB = 262144
GLOBAL_BATCH = 4096
WORKLOAD_DESC = ("C4: B=4096 x V=262144 logits, soft cap 30, 256-id penalty history (1.1/0.5/0.3), "
                 "4096-state constraint bitmask at 2%, temperature 0.8, topK 50, topP 0.95")
METRIC = "sampled rows/s at V=262144 (C4 full pipeline)"
UNIT = "rows/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--dtype", default="f32", choices=["f32", "bf16"])
    ap.add_argument("--no-extras", action="store_true", help="skip bf16 / latency / e2e / cpu legs")
    ap.add_argument("--rows", type=int, default=None,
                    help="rows per GPU (default: the configuration's batch, 4096 for C4); smaller values are for "
                         "profiler captures")
    ap.add_argument("--only", default=None,
                    choices=["C1", "C2", "C3", "C4", "C5", "lm-head", "lm-head-sample", "mask-builder"],
                    help="run one workload --calls times and exit (profiling driver)")
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--no-mask", action="store_true", help="--only: drop the configuration's constraint table")
    ap.add_argument("--no-history", action="store_true", help="--only: drop the configuration's penalty history")
    ap.add_argument("--topk", type=int, default=None, help="--only: override the configuration's topK")
    ap.add_argument("--states", type=int, default=512, help="--only mask-builder: DFA states")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_row(leg: str):
    """DRAM bytes per row of a leg's dominant kernel(s) from the committed ncu summary
    (profiles/dram_traffic.json: one capture per leg, scaled by rows)."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        e = d.get(leg)
        return None if e is None else float(e["dram_bytes"]) / float(e["rows"])
    except Exception:
        return None


def bench_config(world: int, per: int, dtype: str) -> dict:
    """The `config` of the headline line; the reference arm reports the same dict."""
    return {"workload": WORKLOAD_DESC, "global_batch": per * world, "rows_per_gpu": per, "vocab": VOCAB,
            "logits_dtype": dtype, "parallelism": f"rows across {world} GPU(s), {per} per GPU (no collective)",
            "l2": "inputs larger than L2 (rows x 1 MiB per GPU)"}


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 100 ms into a temp file."""

    FIELDS = ("uuid,timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-f", self.path], stdout=subprocess.DEVNULL,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 10 or parts[0] != self.uuid:
                        continue
                    try:
                        ts = datetime.datetime.strptime(parts[1], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    except ValueError:
                        continue
                    rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
        except FileNotFoundError:
            pass
        inside = [r for r in rows if t0 <= r[0] <= t1]
        if len(inside) < 3:
            inside = [r for r in rows if t0 - 2.0 <= r[0] <= t1 + 0.5] or rows
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[3]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": reasons, "samples": len(inside)}


# ------------------------------------------------------------------------ our arm

def run_ours(args, rank, world, local):
    import numpy as np
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    pkg = importlib.import_module(PKG)
    W = importlib.import_module(PKG + ".workloads")
    L = pkg._lib

    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    per = args.rows or GLOBAL_BATCH  # this GPU's own batch (rank 0's rows are C4's rows)
    wl = W.make("C4", device=dev, rows=per, shard=rank)
    logits = wl.logits.to(dtype).contiguous()
    hist = wl.history.contiguous()
    hlen = wl.history_len.contiguous()
    mstate = wl.mask_state.contiguous()
    table = wl.mask_table
    seeds = wl.seeds
    del wl
    torch.cuda.empty_cache()
    rng = torch.tensor([pkg.SeededRandom(s).state for s in seeds], dtype=torch.float64, device=dev)
    params = W.base_params(temperature=0.8, topK=50, topP=0.95, repetitionPenalty=1.1, presencePenalty=0.5,
                           frequencyPenalty=0.3, repetitionWindow=256)
    sampler = pkg.GpuSampler(local)
    sampler.reserve(per, VOCAB, 50, hist.shape[1])
    stream = torch.cuda.current_stream(dev)
    out = None

    def step():
        nonlocal out
        out = sampler.sample(logits, params, softcap=30.0, history=hist, history_len=hlen, mask_table=table,
                             mask_state=mstate, rng_state=rng, stream=stream.cuda_stream, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    flags = out.flags.cpu().numpy().view(np.uint32)
    assert not (flags & L.FLAG_ERRORS).any(), "row errors in the benchmark batch"

    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    # timed region
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    L.lib().gs_profile_enable(sampler.handle, 1)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    if world > 1:
        dist.barrier()
    elapsed_ms = ev0.elapsed_time(ev1)
    import ctypes
    s_ms, s_n, m_ms, m_n = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double(), ctypes.c_int64()
    L.lib().gs_profile_read(sampler.handle, ctypes.byref(s_ms), ctypes.byref(s_n), ctypes.byref(m_ms),
                            ctypes.byref(m_n))
    L.lib().gs_profile_enable(sampler.handle, 0)
    time.sleep(0.2)
    clocks.stop()
    clk = clocks.summary(t_wall0, t_wall1)
    stream_avg_s = s_ms.value / max(1, s_n.value) / 1e3
    merge_avg_s = m_ms.value / max(1, m_n.value) / 1e3
    # rows of the last timed step whose draw or cut fell within 1e-6 of a boundary
    lf = out.flags.cpu().numpy().view(np.uint32)
    nb = torch.tensor([int(((lf & L.FLAG_BOUNDARY) != 0).sum())], dtype=torch.int64, device=dev)
    if world > 1:
        dist.all_reduce(nb)
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())

    esz = 2 if args.dtype == "bf16" else 4
    bytes_per_row = VOCAB * esz + VOCAB // 8 + 4 * hist.shape[1]
    total_rows = per * world
    value = total_rows * args.steps / (elapsed_ms / 1e3)
    peak, peak_kind = measured_peak()
    achieved = per * bytes_per_row / stream_avg_s / 1e9
    tpr = traffic_per_row(f"c4_{args.dtype}")
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.dtype == "f32" else "bf16", "data": "synthetic (seeded torch Philox, C4 distributions)",
        "config": bench_config(world, per, args.dtype),
        "logits_gbps": total_rows * bytes_per_row * args.steps / (elapsed_ms / 1e3) / 1e9,
        "roofline": {"bound": "hbm", "kernel": "gs::stream2_kernel", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": None if tpr is None else tpr * per,
                     "algorithmic_bytes_per_launch": per * bytes_per_row,
                     "avg_launch_us": stream_avg_s * 1e6, "merge_avg_launch_us": merge_avg_s * 1e6},
        "gpu_launches": 2 * args.steps * world,
        "boundary_rows": {"count": int(nb.item()), "of": per * world,
                          "what": "rows of the last timed step flagged GS_FLAG_BOUNDARY_* (a top-p cut, min-p, "
                                  "typical-p or draw decision within 1e-6 of its boundary)"},
        "clocks": clk,
    }
    if not args.no_extras:
        # end to end on every rank (whole-job rows over the slowest rank's time)
        result["e2e"] = e2e_leg(args, pkg, sampler, dev, logits, hist, hlen, table, mstate, seeds, params, per,
                                world)
    if world > 1 and not args.no_extras:
        # every rank takes part: C4 as written (its 4096 rows split over the GPUs), then C5
        # with one all-gather of shard records per step
        result["c4_strong_split"] = strong_split_leg(pkg, sampler, dev, logits, hist, hlen, table, mstate, params,
                                                     world)
        result["c5_vocab_sharded"] = c5_sharded_leg(pkg, W, sampler, dev, rank, world)
    if rank == 0 and not args.no_extras:
        del logits
        torch.cuda.empty_cache()
        result.update(extras(args, pkg, W, sampler, dev, None, hist, hlen, table, mstate, seeds, params, per,
                             world))
    sampler.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def e2e_leg(args, pkg, sampler, dev, logits, hist, hlen, table, mstate, seeds, params, per, world):
    """gs_sample_host with pinned host buffers: host->device copies of the step's inputs and
    device->host copies of its outputs inside the timed region, on every rank."""
    import torch
    stream = torch.cuda.current_stream(dev)
    n_e2e = max(3, min(10, args.steps))
    hx = logits.cpu().pin_memory().numpy() if logits.dtype == torch.float32 else None
    if hx is None:
        hx = logits.view(torch.int16).cpu().pin_memory().numpy()
    hh = hist.cpu().pin_memory().numpy()
    hl = hlen.cpu().pin_memory().numpy()
    hs = mstate.cpu().pin_memory().numpy()
    hr = torch.tensor([pkg.SeededRandom(s).state for s in seeds], dtype=torch.float64).pin_memory().numpy()
    dt = pkg._lib.GS_DTYPE_F32 if logits.dtype == torch.float32 else pkg._lib.GS_DTYPE_BF16
    for _ in range(2):
        sampler.sample_host(hx, params, softcap=30.0, history=hh, history_len=hl, mask_table=table, mask_state=hs,
                            rng_state=hr, stream=stream.cuda_stream, dtype=dt)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n_e2e):
        sampler.sample_host(hx, params, softcap=30.0, history=hh, history_len=hl, mask_table=table, mask_state=hs,
                            rng_state=hr, stream=stream.cuda_stream, dtype=dt)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_s = e0.elapsed_time(e1) / 1e3
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    h2d = hx.nbytes + hh.nbytes + hl.nbytes + hs.nbytes + hr.nbytes
    d2h = per * (4 + 4 + 8)
    return {"value": per * world * n_e2e / e2e_s, "unit": UNIT, "h2d_bytes_per_step": int(h2d * world),
            "d2h_bytes_per_step": int(d2h * world), "steps": n_e2e,
            "api": "gs_sample_host (host logits/history/states in pinned memory, ids+flags+states back), "
                   "every rank, slowest rank's time"}


def extras(args, pkg, W, sampler, dev, logits, hist, hlen, table, mstate, seeds, params, per, world):
    """Rank 0's other legs (after the headline's logits are freed)."""
    import torch

    res = {}
    stream = torch.cuda.current_stream(dev)
    # ---- the other configurations at their own batch sizes, each with its roofline
    legs = {}
    legs["c4_bf16"] = config_leg(pkg, W, sampler, dev, "C4", per, dtype=torch.bfloat16, steps=100)
    legs["c4_f32_unmasked"] = config_leg(pkg, W, sampler, dev, "C4", per, mask=False, steps=100)
    legs["c4_bf16_unmasked"] = config_leg(pkg, W, sampler, dev, "C4", per, dtype=torch.bfloat16, mask=False,
                                          steps=100)
    legs["c3"] = config_leg(pkg, W, sampler, dev, "C3", 256, steps=200)
    legs["c2"] = config_leg(pkg, W, sampler, dev, "C2", 64, steps=200)
    legs["c2_typical"] = config_leg(pkg, W, sampler, dev, "C2", 64, steps=200, override={"typicalP": 0.9},
                                    label="c2_typical")
    res["configs"] = legs
    res["bf16"] = {k: legs["c4_bf16"][k] for k in ("value", "unit", "steps", "logits_gbps")}
    # ---- C1 latency: B=1, 256 sequential steps, fresh logits each step, one seeded stream
    steps = 256
    lg = torch.empty((steps, VOCAB), dtype=torch.float32, device=dev)
    for s in range(steps):
        lg[s] = W.make("C1", device=dev, step=s).logits[0]
    # (a decode loop converts its fixed config once, prepare_params, and binds its call,
    # GpuSampler.bind: the call's structures are built once, each step sets the logits)
    p1 = pkg.prepare_params(W.base_params(temperature=0.8, topK=40, topP=0.95, repetitionWindow=0))
    st = torch.tensor([pkg.SeededRandom(42).state], dtype=torch.float64, device=dev)
    step1 = sampler.bind(lg[0:1], p1, softcap=30.0, rng_state=st, stream=stream.cuda_stream)

    def time_loop(call):
        for s in range(16):
            call(s)
        st.fill_(pkg.SeededRandom(42).state)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        evs[0].record(stream)
        h0 = time.perf_counter()
        for s in range(steps):
            call(s)
            evs[s + 1].record(stream)
        host = (time.perf_counter() - h0) / steps * 1e6
        torch.cuda.synchronize()
        return sorted(evs[i].elapsed_time(evs[i + 1]) * 1e3 for i in range(steps)), host

    lat, host_us = time_loop(lambda s: step1(lg[s:s + 1]))
    o1 = None

    def via_sample(s):
        nonlocal o1
        o1 = sampler.sample(lg[s:s + 1], p1, softcap=30.0, rng_state=st, stream=stream.cuda_stream, out=o1)

    lat_s, host_s = time_loop(via_sample)
    # the kernels' own device time per step (the library's events around its launches)
    import ctypes
    Lb = pkg._lib.lib()
    Lb.gs_profile_enable(sampler.handle, 1)
    for s in range(steps):
        step1(lg[s:s + 1])
    torch.cuda.synchronize()
    s_ms, s_n, m_ms, m_n = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double(), ctypes.c_int64()
    Lb.gs_profile_read(sampler.handle, ctypes.byref(s_ms), ctypes.byref(s_n), ctypes.byref(m_ms), ctypes.byref(m_n))
    Lb.gs_profile_enable(sampler.handle, 0)
    kern_us = (s_ms.value + m_ms.value) / max(1, s_n.value) * 1e3
    # the same 256 steps captured in one CUDA graph: no host work between the steps
    graph_us = None
    try:
        gs = torch.cuda.Stream(dev)
        gs.wait_stream(stream)
        stepg = sampler.bind(lg[0:1], p1, softcap=30.0, rng_state=st, stream=gs.cuda_stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gs):
            for s in range(steps):
                stepg(lg[s:s + 1])
        with torch.cuda.stream(gs):
            for _ in range(3):
                graph.replay()
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        with torch.cuda.stream(gs):  # (replay launches on the current stream)
            g0.record(gs)
            for _ in range(reps):
                graph.replay()
            g1.record(gs)
        torch.cuda.synchronize()
        graph_us = g0.elapsed_time(g1) * 1e3 / (reps * steps)
        del graph
    except RuntimeError as e:  # a capture the runtime refuses: report the step times without it
        print(f"latency_b1: graph capture failed: {e}", file=sys.stderr)
        torch.cuda.synchronize()
    # the reference's default decode config (src/runtime/decoding.ts:16-29): C1's settings with
    # a 1.05 repetition penalty over a 64-id window (a fixed window here: the work per step
    # does not depend on which ids it holds)
    pw = pkg.prepare_params(W.base_params(temperature=0.8, topK=40, topP=0.95, repetitionPenalty=1.05,
                                          repetitionWindow=64))
    hw = torch.randint(0, VOCAB, (1, 64), dtype=torch.int32, device=dev,
                       generator=torch.Generator(device=dev).manual_seed(64))
    hwl = torch.full((1,), 64, dtype=torch.int32, device=dev)
    stepw = sampler.bind(lg[0:1], pw, softcap=30.0, history=hw, history_len=hwl, rng_state=st,
                         stream=stream.cuda_stream)
    latw, _ = time_loop(lambda s: stepw(lg[s:s + 1]))
    # the same under a constraint row (about half the vocabulary allowed; the JSON / tool-call
    # decoding of the reference's constrained generate)
    gm = torch.Generator(device=dev).manual_seed(65)
    mt = torch.randint(-2**31, 2**31 - 1, (1, VOCAB // 32), dtype=torch.int32, device=dev, generator=gm)
    ms = torch.zeros(1, dtype=torch.int32, device=dev)
    stepm = sampler.bind(lg[0:1], pw, softcap=30.0, history=hw, history_len=hwl, mask_table=mt, mask_state=ms,
                         rng_state=st, stream=stream.cuda_stream)
    latm, _ = time_loop(lambda s: stepm(lg[s:s + 1]))
    res["latency_b1"] = {"workload": "C1: B=1, V=262144, soft cap 30, T=0.8, topK 40, topP 0.95, seed 42, "
                                     "256 sequential steps",
                         "sample_api_p50_us": lat_s[len(lat_s) // 2], "sample_api_host_us_per_call": host_s,
                         "default_config_p50_us": latw[len(latw) // 2],
                         "default_config_p95_us": latw[int(len(latw) * 0.95)],
                         "constrained_p50_us": latm[len(latm) // 2],
                         "constrained_p95_us": latm[int(len(latm) * 0.95)],
                         "constrained": "the default config under a constraint row allowing about half the ids",
                         "default_config": "DEFAULT_DECODING_CONFIG: the same with repetitionPenalty 1.05 over a "
                                           "64-id window (fixed ids)",
                         "p50_us": lat[len(lat) // 2], "p95_us": lat[int(len(lat) * 0.95)],
                         "kernel_us": kern_us, "graph_us_per_step": graph_us, "host_us_per_call": host_us,
                         "timing": "p50/p95: CUDA events between consecutive decode-loop calls (GpuSampler.bind: "
                                   "gs_sample with the call's structures built once; device time, no graph; 256 "
                                   "distinct 1 MiB rows, 256 MiB > L2); sample_api_*: the same through "
                                   "GpuSampler.sample (structures rebuilt each call); kernel_us: the library's "
                                   "events around its launches, average per step; graph_us_per_step: the 256 calls "
                                   "captured in one CUDA graph, replayed (device time per step, no host work "
                                   "between steps); host_us_per_call: host time of one bound call from Python"}
    del lg
    # ---- CPU baseline (N = 1 only): the oracle on a bounded sample of the same rows
    if world == 1:
        res["cpu_baseline"] = cpu_baseline(W, dev, per)
        res["mask_builder"] = mask_builder_leg(pkg, W, sampler)
        res["lm_head"] = lm_head_leg(pkg, sampler, stream)
    return res


def config_leg(pkg, W, sampler, dev, name, rows, dtype=None, mask=True, history=True, steps=100, override=None,
               label=None):
    """One configuration at `rows` rows: rows/s, the path's kernel time split (streaming
    pass / merge or histogram path, CUDA events recorded by the library) and the HBM
    roofline of the dominant launches.  Inputs smaller than twice L2 are replicated and
    the copies used in turn, so that every step reads its logits from HBM.  `override`:
    sampling parameters replacing the configuration's (named by `label`)."""
    import torch
    import ctypes
    L = pkg._lib
    wl = W.make(name, device=dev, rows=rows, dtype=dtype)
    params = pkg.prepare_params([dict(p, **override) for p in wl.params] if override else wl.params)
    kw = dict(softcap=wl.softcap)
    if history and wl.history is not None:
        kw.update(history=wl.history, history_len=wl.history_len)
    if mask and wl.mask_table is not None:
        kw.update(mask_table=wl.mask_table, mask_state=wl.mask_state)
    esz = wl.logits.element_size()
    in_bytes = wl.logits.numel() * esz
    copies = min(8, max(1, -(-2 * 126 * 2**20 // in_bytes)))
    xs = [wl.logits] + [wl.logits.clone() for _ in range(copies - 1)]
    rng = wl.rng_state(dev)
    stream = torch.cuda.current_stream(dev)
    out = None
    for i in range(5):
        out = sampler.sample(xs[i % copies], params, rng_state=rng, stream=stream.cuda_stream, out=out, **kw)
    torch.cuda.synchronize()
    fl = out.flags.cpu().numpy().view("uint32")
    errors = int(((fl & L.FLAG_ERRORS) != 0).sum())
    L.lib().gs_profile_enable(sampler.handle, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        out = sampler.sample(xs[i % copies], params, rng_state=rng, stream=stream.cuda_stream, out=out, **kw)
    e1.record(stream)
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3
    s_ms, s_n, m_ms, m_n = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double(), ctypes.c_int64()
    L.lib().gs_profile_read(sampler.handle, ctypes.byref(s_ms), ctypes.byref(s_n), ctypes.byref(m_ms),
                            ctypes.byref(m_n))
    L.lib().gs_profile_enable(sampler.handle, 0)
    stream_us = s_ms.value / max(1, s_n.value) * 1e3
    merge_us = m_ms.value / max(1, m_n.value) * 1e3
    large = bool((fl & L.FLAG_LARGE_PATH).all())
    hl = wl.history.shape[1] if (history and wl.history is not None) else 0
    bpr = wl.vocab * esz + (wl.vocab // 8 if (mask and wl.mask_table is not None) else 0) + 4 * hl
    peak, peak_kind = measured_peak()
    tag = f"{name.lower()}" + ("" if name != "C4" else f"_{'bf16' if esz == 2 else 'f32'}") + \
        ("_unmasked" if (name == "C4" and not mask) else "")
    if large:
        kern, kern_us = "histogram path (large_hist, large_select, large_gather, large_resolve)", merge_us
    elif mask and wl.mask_table is not None:
        kern, kern_us = "gs::stream2_kernel (streaming pass)", stream_us
    else:
        kern, kern_us = "gs::dense_kernel (streaming pass)", stream_us
    achieved = rows * bpr / (kern_us / 1e6) / 1e9
    tpr = traffic_per_row(tag)
    if label:
        tag = label
    res = {
        "workload": f"{name} x {rows} rows" + ("" if mask or wl.mask_table is None else ", no constraint mask") +
                    (f", {label}: {override}" if override else ""),
        "value": rows * steps / dt, "unit": UNIT, "steps": steps, "us_per_step": dt / steps * 1e6,
        "logits_dtype": "bf16" if esz == 2 else "f32",
        "logits_gbps": rows * bpr * steps / dt / 1e9, "row_errors": errors,
        "l2": f"{copies} copies of the {in_bytes / 2**20:.0f} MiB input used in turn" if copies > 1
              else "input larger than L2",
        "kernel_split_us": {"streaming_pass": stream_us, "merge_or_histogram_path": merge_us},
        "roofline": {"bound": "hbm", "kernel": kern, "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                     "algorithmic_bytes_per_launch": rows * bpr, "avg_launch_us": kern_us,
                     "step_frac": rows * bpr / (dt / steps) / 1e9 / peak,
                     "traffic": None if tpr is None else tpr * rows},
    }
    del xs, wl
    torch.cuda.empty_cache()
    return res


def strong_split_leg(pkg, sampler, dev, logits, hist, hlen, table, mstate, params, world, steps=300):
    """C4 as BASELINE states it: one batch of 4096 rows split evenly over the N GPUs
    (4096/N rows per rank, each rank's first rows of its own batch), rows/s of the whole
    batch over the slowest rank's device time, and the kernel split of rank 0."""
    import ctypes
    import torch
    import torch.distributed as dist
    L = pkg._lib
    per = GLOBAL_BATCH // world
    x, h, hl, ms = logits[:per], hist[:per].contiguous(), hlen[:per].contiguous(), mstate[:per].contiguous()
    rng = torch.zeros(per, dtype=torch.float64, device=dev) + pkg.SeededRandom(3000).state
    stream = torch.cuda.current_stream(dev)
    out = None
    for _ in range(10):
        out = sampler.sample(x, params, softcap=30.0, history=h, history_len=hl, mask_table=table, mask_state=ms,
                             rng_state=rng, stream=stream.cuda_stream, out=out)
    torch.cuda.synchronize()
    dist.barrier()
    L.lib().gs_profile_enable(sampler.handle, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        out = sampler.sample(x, params, softcap=30.0, history=h, history_len=hl, mask_table=table, mask_state=ms,
                             rng_state=rng, stream=stream.cuda_stream, out=out)
    e1.record(stream)
    torch.cuda.synchronize()
    s_ms, s_n, m_ms, m_n = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double(), ctypes.c_int64()
    L.lib().gs_profile_read(sampler.handle, ctypes.byref(s_ms), ctypes.byref(s_n), ctypes.byref(m_ms),
                            ctypes.byref(m_n))
    L.lib().gs_profile_enable(sampler.handle, 0)
    t = torch.tensor([e0.elapsed_time(e1) / 1e3], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dt = float(t.item())
    return {"workload": f"C4: one batch of {GLOBAL_BATCH} rows split evenly, {per} rows per GPU", "n_gpus": world,
            "value": GLOBAL_BATCH * steps / dt, "unit": UNIT, "ms_per_step": dt / steps * 1e3, "steps": steps,
            "scaling": "strong", "rank0_kernel_split_us": {"streaming_pass": s_ms.value / max(1, s_n.value) * 1e3,
                                                           "merge": m_ms.value / max(1, m_n.value) * 1e3},
            "timing": "CUDA events, slowest rank; the driver's 1-GPU line is the N = 1 point"}


def c5_sharded_leg(pkg, W, sampler, dev, rank, world, steps=200):
    """C5 in the vocabulary-sharded layout on every rank: rank g holds ids
    [g·V/N, (g+1)·V/N) of the 8 rows; per step gs_shard_sample (the library's own NCCL
    exchange: partials, ncclAllGather of the records, merge).  Device time per step and of
    the torch all-gather of the same records alone (CUDA events, slowest rank), and whether
    every rank's ids equal whole-row sampling."""
    import torch
    import torch.distributed as dist
    SH = importlib.import_module(PKG + ".sharding")
    wl = W.make("C5", device=dev)
    rows = wl.rows
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(SH.NcclShardedSampler.unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    ns = SH.NcclShardedSampler(sampler, VOCAB, rank, world, bytes(uid.cpu().numpy().tobytes()), timeout_ms=30000)
    off, size = ns.plan.offset, ns.plan.size
    local = wl.logits[:, off:off + size].contiguous()
    params = pkg.prepare_params(wl.params)
    stream = torch.cuda.current_stream(dev)
    rng = wl.rng_state(dev)
    rng_w = wl.rng_state(dev)
    whole = sampler.sample(wl.logits, params, softcap=wl.softcap, rng_state=rng_w)
    res = ns.sample(local, params, softcap=wl.softcap, rng_state=rng)
    torch.cuda.synchronize()
    same = bool(torch.equal(res.ids, whole.ids)) and bool(torch.equal(rng, rng_w))
    ok = torch.tensor([1 if same else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    ns.timeout_ms = 0  # (asynchronous steps inside the timed loop)
    for _ in range(5):
        ns.sample(local, params, softcap=wl.softcap, rng_state=rng)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        ns.sample(local, params, softcap=wl.softcap, rng_state=rng)
    e1.record(stream)
    torch.cuda.synchronize()
    step_s = e0.elapsed_time(e1) / 1e3 / steps
    rec = sampler.shard_partials(local, params, vocab_offset=off, vocab_total=VOCAB, softcap=wl.softcap)
    rec_bytes = rec.numel()
    for _ in range(3):
        SH.exchange_records(rec)
    torch.cuda.synchronize()
    ga = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ga[0].record(stream)
    for _ in range(steps):
        SH.exchange_records(rec)
    ga[1].record(stream)
    torch.cuda.synchronize()
    ag_s = ga[0].elapsed_time(ga[1]) / 1e3 / steps
    t = torch.tensor([step_s, ag_s], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_s, ag_s = float(t[0]), float(t[1])
    ns.close()
    return {"workload": f"C5: B={rows}, V={VOCAB} split into {world} contiguous shards of {size} ids, Gumbel(0,2) "
                        "+ 30 planted ties, T 1.5, topK 1024, topP 0.99",
            "us_per_step": step_s * 1e6, "rows_per_s": rows / step_s, "allgather_us": ag_s * 1e6,
            "record_bytes_per_rank": rec_bytes, "nccl_ranks": world, "matches_whole_row_sampling": bool(ok.item()),
            "exchange": "gs_shard_sample (the library's own ncclAllGather; NCCL loaded at run time)",
            "timing": "CUDA events around steps of partials + NCCL all-gather + merge, slowest rank; allgather_us: "
                      "torch.distributed all-gather of the same records alone"}


def lm_head_leg(pkg, sampler, stream):
    """The int2 LM head (decode-lm-head.ts) at the reference's shape: V = 262144 rows of
    1536 2-bit codes (100.7 MB packed), per batch size the device time of one
    gs_lm_head_logits call, and activations -> token with gs_lm_head_sample at B = 1."""
    import numpy as np
    import torch
    from oracle import oracle as O
    LM = importlib.import_module(PKG + ".lm_head")
    V, H = VOCAB, 1536
    packed, scales, act, act_sum = LM.synthetic(V, H, 64, seed=91)
    head = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0)
    peak, peak_kind = measured_peak()
    out = {"shape": {"vocab": V, "hidden": H, "packed_mb": V * H / 4 / 1e6},
           "timing": "CUDA events around 20 back-to-back calls on one stream (device time per call, weights "
                     "100.7 MB > L2 so every call streams them from HBM)", "batches": {}}
    a_all, s_all = torch.from_numpy(act).cuda(), torch.from_numpy(act_sum).cuda()
    for B in (1, 4, 16, 64):
        a, sm = a_all[:B].contiguous(), s_all[:B].contiguous()
        lg = torch.empty((B, V), dtype=torch.float32, device=a.device)
        for _ in range(3):
            head.logits(a, sm, out=lg, stream=stream.cuda_stream)
        reps = 20
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            head.logits(a, sm, out=lg, stream=stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        head.check()
        us = e0.elapsed_time(e1) * 1e3 / reps
        alg = V * H // 4 + V * 4 + B * H * 4 + B * V * 4  # packed codes, row scales, activations, logits
        out["batches"][str(B)] = {
            "us_per_call": us, "rows_per_s": B / us * 1e6, "int_tops": 2.0 * B * H * V / us / 1e6,
            "kernel": "dp4a GEMV" if B <= 4 else "tcgen05 kind::i8 MMA (weights expanded into TMEM)",
            "roofline": {"bound": "hbm", "achieved": alg / us / 1e3, "peak": peak, "unit": "GB/s",
                         "frac": alg / us / 1e3 / peak, "algorithmic_bytes": alg,
                         "peak_source": f"{peak_kind} hbm_gbs"}}
    # activations -> token (C1's sampling parameters), B = 1
    p1 = [dict(temperature=0.8, topK=40, topP=0.95, minP=0.0, typicalP=1.0, repetitionPenalty=1.0,
               presencePenalty=0.0, frequencyPenalty=0.0)]
    st = torch.tensor([pkg.SeededRandom(42).state], dtype=torch.float64, device=a_all.device)
    a1, s1 = a_all[:1].contiguous(), s_all[:1].contiguous()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(65)]

    def route_p50(route):
        head.set_route(route)
        f0 = head.fused_calls
        for _ in range(3):
            head.sample(a1, s1, p1, softcap=30.0, rng_state=st, stream=stream.cuda_stream)
        evs[0].record(stream)
        for i in range(64):
            head.sample(a1, s1, p1, softcap=30.0, rng_state=st, stream=stream.cuda_stream)
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
        lat = sorted(evs[i].elapsed_time(evs[i + 1]) * 1e3 for i in range(64))
        return lat, head.fused_calls - f0

    lat, fused = route_p50("auto")
    lat_f, _ = route_p50("fused")
    head.set_route("auto")
    # the same step as two calls (logits to HBM, then gs_sample), for comparison
    lg1 = torch.empty((1, V), dtype=torch.float32, device=a_all.device)
    st2 = st.clone()
    for _ in range(3):
        head.logits(a1, s1, out=lg1, stream=stream.cuda_stream)
        sampler.sample(lg1, p1, softcap=30.0, rng_state=st2, stream=stream.cuda_stream)
    evs[0].record(stream)
    for i in range(64):
        head.logits(a1, s1, out=lg1, stream=stream.cuda_stream)
        sampler.sample(lg1, p1, softcap=30.0, rng_state=st2, stream=stream.cuda_stream)
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    lat2 = sorted(evs[i].elapsed_time(evs[i + 1]) * 1e3 for i in range(64))
    out["sample_b1"] = {"p50_us": lat[32], "p95_us": lat[int(64 * 0.95)],
                        "route": "fused (logits kept on chip, shard-record merge)" if fused >= 67
                                 else "two-step inside the call (GEMV, then the single-launch decode step)",
                        "fused_route_p50_us": lat_f[32], "two_step_p50_us": lat2[32],
                        "timing": "CUDA events between consecutive gs_lm_head_sample calls (LM head + sampling; "
                                  "default route, then the fused route forced); two_step: gs_lm_head_logits then "
                                  "gs_sample per step"}
    head.close()
    # the oracle's exact LM head on the host (one core), one row
    c0 = time.perf_counter()
    O.lm_head(packed[:16384], scales[:16384], act[:1], act_sum[:1], in_scale=0.02)
    cdt = (time.perf_counter() - c0) * (V / 16384)
    out["cpu_oracle"] = {"us_per_row": cdt * 1e6, "cores": 1,
                         "sample": "oracle_lm_head_exact over 16384 of the 262144 rows, one activation row, scaled"}
    out["data"] = "synthetic: seeded packed codes, row scales and int8-grid activations (lm_head.synthetic)"
    return out


def mask_builder_leg(pkg, W, sampler):
    """The constraint bitmask builder at the size of C3/C4's tables: 4096 states x V."""
    import numpy as np
    import torch
    from oracle import oracle as O
    C = importlib.import_module(PKG + ".constraints")
    off, b = W.synthetic_token_bytes(VOCAB)
    tr, fi = W.synthetic_dfa(4096)
    dfa = C.Dfa.from_transitions(tr, fi)
    g = C.GpuConstraint(sampler, dfa, (off, b))
    states = list(range(4096))
    table, dead = g.build_masks(states)
    torch.cuda.synchronize()
    reps = 5
    t0 = time.perf_counter()
    for _ in range(reps):
        table, dead = g.build_masks(states, table=table)
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / reps
    allowed = int(np.unpackbits(table.cpu().numpy().view(np.uint8)).sum())
    g.close()
    node, plen, pb = C.pack_states(states[:4])
    c0 = time.perf_counter()
    O.constraint_masks(dfa.arrays(), (off, b), node, plen, pb)
    cdt = time.perf_counter() - c0
    words = (VOCAB + 31) // 32
    return {"states": 4096, "vocab": VOCAB, "ms_per_table": dt * 1e3, "rows_per_s": 4096 / dt,
            "table_gbs": 4096 * words * 4 / dt / 1e9, "allowed_fraction": allowed / (4096 * VOCAB),
            "timing": "wall clock around gs_constraint_build_masks (state upload, walk and post kernels, sync)",
            "cpu_oracle": {"rows_per_s": 4 / cdt, "cores": 1, "sample": "4 states, oracle/oracle.cpp trie DFS "
                                                                          "restating legalTokenIds (trie build included)"},
            "data": "synthetic: seeded token bytes (workloads.synthetic_token_bytes) and a 4096-node code-point DFA "
                    "(workloads.synthetic_dfa); the Gemma tokenizer's bytes are not available"}


def cpu_baseline(W, dev, per):
    import numpy as np
    import torch
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    # about 10-30 s of host work: ~25 rows/s per core for C4 rows
    n = min(per, max(64, 25 * threads * 15))
    wl = W.make("C4", device=dev, rows=n)
    x = wl.logits.float().cpu().numpy()
    h = wl.history.cpu().numpy()
    hl = wl.history_len.cpu().numpy()
    ms = wl.mask_state.cpu().numpy()
    used = sorted(set(ms.tolist()))
    remap = {s: i for i, s in enumerate(used)}
    tb = wl.mask_table[torch.tensor(used, device=wl.mask_table.device)].cpu().numpy().view(np.uint32)
    ms2 = np.array([remap[s] for s in ms.tolist()], dtype=np.int32)
    st = np.array([O.seeded_init(s) for s in wl.seeds[:n]], dtype=np.float64)
    p = dict(wl.params[0], repetitionWindow=h.shape[1])
    del wl
    t0 = time.perf_counter()
    O.sample_rows(x, VOCAB, 30.0, h, hl, tb, ms2, [p], rng_state=st, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} rows of C4 (float32), oracle/oracle.cpp restating src/runtime/sampling.ts, "
                      f"{threads} host threads, {dt:.2f} s wall"}


# ------------------------------------------------------------------ reference arm

def run_reference(args, rank, world):
    if rank != 0:
        return
    import numpy as np
    import torch
    from oracle import oracle as O
    W = importlib.import_module(PKG + ".workloads")

    threads = os.cpu_count() or 1
    rows = threads  # one row per host thread per step
    g = torch.Generator().manual_seed(31)
    x = (torch.randn((rows, VOCAB), generator=g) * 2.0).numpy()
    hist = torch.randint(0, VOCAB, (rows, 256), generator=g).to(torch.int32).numpy()
    hlen = np.full(rows, 256, dtype=np.int32)
    allowed = torch.rand((rows, VOCAB), generator=g) < 0.02
    table = W.pack_bits(allowed).numpy().view(np.uint32)
    mstate = np.arange(rows, dtype=np.int32)
    p = W.base_params(temperature=0.8, topK=50, topP=0.95, repetitionPenalty=1.1, presencePenalty=0.5,
                      frequencyPenalty=0.3, repetitionWindow=256)
    st = np.array([O.seeded_init(3000 + i) for i in range(rows)], dtype=np.float64)

    def step():
        O.sample_rows(x, VOCAB, 30.0, hist, hlen, table, mstate, [p], rng_state=st, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = rows * args.steps / dt
    sample = (f"{rows} C4-distributed rows per step (one per host thread) of the {GLOBAL_BATCH}-row C4 batch, "
              f"rows/s extrapolated from them; oracle/oracle.cpp (C++ restatement of src/runtime/sampling.ts; the "
              f"TypeScript reference needs Node, which is not installed)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded torch CPU generator, C4 distributions)",
        "config": bench_config(world, GLOBAL_BATCH, "f32"),
        "sample_rows_per_step": rows,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_only(args):
    """Profiling driver: one workload `--calls` times on cuda:0, then a one-line summary."""
    import numpy as np
    import torch
    pkg = importlib.import_module(PKG)
    W = importlib.import_module(PKG + ".workloads")
    dev = torch.device("cuda", 0)
    sampler = pkg.GpuSampler(0)
    if args.only in ("C1", "C2", "C3", "C4", "C5"):
        dtype = torch.bfloat16 if args.dtype == "bf16" else None
        wl = W.make(args.only, device=dev, rows=args.rows, dtype=dtype)
        params = [dict(p, topK=args.topk) for p in wl.params] if args.topk is not None else wl.params
        params = pkg.prepare_params(params)
        kw = dict(softcap=wl.softcap, rng_state=wl.rng_state(dev))
        if wl.history is not None and not args.no_history:
            kw.update(history=wl.history, history_len=wl.history_len)
        if wl.mask_table is not None and not args.no_mask:
            kw.update(mask_table=wl.mask_table, mask_state=wl.mask_state)
        res = None
        for _ in range(args.calls):
            res = sampler.sample(wl.logits, params, **kw)
        torch.cuda.synchronize()
        fl = res.flags.cpu().numpy().view(np.uint32)
        print(args.only, "rows", wl.rows, "first ids", res.ids[:4].tolist(), "row errors",
              int(((fl & pkg._lib.FLAG_ERRORS) != 0).sum()))
    elif args.only in ("lm-head", "lm-head-sample"):
        LM = importlib.import_module(PKG + ".lm_head")
        rows = args.rows or 1
        packed, scales, act, act_sum = LM.synthetic(VOCAB, 1536, rows, seed=5)
        head = LM.GpuLmHead(sampler, packed, scales, 0.02, 0.0)
        x, s = torch.from_numpy(act).to(dev), torch.from_numpy(act_sum).to(dev)
        if args.only == "lm-head-sample":
            p = [dict(temperature=0.8, topK=40, topP=0.95, minP=0.0, typicalP=1.0, repetitionPenalty=1.0,
                      presencePenalty=0.0, frequencyPenalty=0.0)]
            st = torch.arange(rows, dtype=torch.float64, device=dev)
            for _ in range(args.calls):
                res = head.sample(x, s, p, softcap=30.0, rng_state=st)
            head.check()
            torch.cuda.synchronize()
            print("rows", rows, "ids", res.ids.tolist(), "fused calls", head.fused_calls)
        else:
            out = None
            for _ in range(args.calls):
                out = head.logits(x, s, out=out)
            head.check()
            torch.cuda.synchronize()
            print("rows", rows, "logits[0, :4]", out[0, :4].tolist())
        head.close()
    else:  # mask-builder
        C = importlib.import_module(PKG + ".constraints")
        tr, fi = W.synthetic_dfa(max(args.states, 1))
        con = C.GpuConstraint(sampler, C.Dfa.from_transitions(tr, fi), W.synthetic_token_bytes())
        table = None
        for _ in range(args.calls):
            table, dead = con.build_masks(list(range(args.states)), table=table)
        torch.cuda.synchronize()
        print("states", args.states, "rows with nothing allowed", int(dead.sum()))
        con.close()
    sampler.close()


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.only:
        run_only(args)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
