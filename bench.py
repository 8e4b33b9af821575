#!/usr/bin/env python
"""Benchmark: INT8/INT4 weight-quantized GEMM sweep on B200.

Workload (one step): the quantized-matmul sweep of A[M x 768] (f32,
U(-1,1), seed 1) times W[768 x 3072] (N(0,0.02), seed 2, quantized by the
reference's own routines: INT8 per output channel, INT4 group 32) plus an
f32 bias, for M in {1, 16, 128, 2048} and both weight types -- 8 quantized
matmuls, each = activation row quantization + exact-int32 tensor-core GEMM
+ dequantizing epilogue, all through libopencuda_cuda.so.

value   = algorithmic integer ops of the sweep (2*M*N*K summed) / device
          time, whole job (sum over ranks / max over ranks), in TOPS.
e2e     = the same ops through the host-slice C ABI (oc_blas_qgemm_*): every
          call copies A, the quantized weights, scales and bias from pinned
          host memory and copies Y back, timed on the host clock.
Inputs rotate over 8 device-resident sets (~300 MB > 126 MB L2) so every
step reads HBM, not L2.  `--impl reference` times the reference's CPU path
for the same sweep (dequantize + naive sgemm + bias, restated in C) on all
host cores.  N>1: every rank runs its own sweep (replicas, weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "open-cuda_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

K_DIM, N_DIM, GROUP4 = 768, 3072, 32
M_SWEEP = (1, 16, 128, 2048)
N_SETS = 8
METRIC = "INT8/INT4 weight-quantized GEMM TOPS (M in {1,16,128,2048}, K=768, N=3072)"


def sweep_ops() -> int:
    return 2 * sum(2 * m * K_DIM * N_DIM for m in M_SWEEP)  # two weight types


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-once", action="store_true",
                    help="run one warm sweep per set and exit (for ncu launch lists)")
    return ap.parse_args()


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# the CPU path of the reference (oracle restatement), bounded sample
# ----------------------------------------------------------------------------

def cpu_reference_sample(target_s: float = 6.0):
    """Times the reference's CPU composition for the sweep: dequantize the
    weights, naive sgemm (one task per 256 output elements, strided B, the
    per-call copies) and the host bias add, on all host cores.  Large M are
    sampled by rows and scaled linearly in M.  Returns (TOPS, desc, cores)."""
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    t_total = 0.0
    sample = []
    A_full, WT, bias = synth.qgemm_case(max(M_SWEEP), K_DIM, N_DIM)
    t8 = oracle.quantize_int8(WT.ravel(), K_DIM)
    t4 = oracle.quantize_int4(WT.ravel(), GROUP4)
    budget = target_s / (2 * len(M_SWEEP))

    def timed(bits, t, g, rows):
        t0 = time.perf_counter()
        oracle.qgemm_weight_only(bits, rows, K_DIM, N_DIM, g, A_full[:rows], t.data, t.scales, bias, faithful=True)
        return time.perf_counter() - t0

    for bits, t, g in ((8, t8, K_DIM), (4, t4, GROUP4)):
        # two-point model per call: t(rows) = fixed (dequantize, transpose,
        # copies of W) + rows * per_row (the naive GEMM rows)
        t1 = timed(bits, t, g, 1)
        r2 = 8
        t2 = timed(bits, t, g, r2)
        per_row = max((t2 - t1) / (r2 - 1), 1e-9)
        fixed = max(t1 - per_row, 0.0)
        for m in M_SWEEP:
            rows = max(1, min(m, int(max(budget - fixed, per_row) / per_row)))
            dt = timed(bits, t, g, rows)
            t_total += dt if rows == m else (dt - fixed) * (m / rows) + fixed
            sample.append(f"W{bits} M={m}: {rows} rows")
    tops = sweep_ops() / t_total / 1e12
    desc = ("reference CPU path restated in C (dequantize + naive sgemm with per-call copies + bias); "
            + "; ".join(sample) + "; sampled calls scaled as fixed + rows * per-row time")
    return tops, desc, cores, t_total


def run_reference(args, rank, world):
    if rank != 0:
        return
    vals = []
    for i in range(args.warmup + args.steps):
        tops, desc, cores, t = cpu_reference_sample(target_s=2.0)
        if i >= args.warmup:
            vals.append(tops)
    v = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sweep_ops() / (v * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (SplitMix64-seeded U(-1,1) activations, N(0,0.02) weights)",
        "config": {"workload": "config-2 quantized GEMM sweep on the reference CPU path", "K": K_DIM, "N": N_DIM,
                   "M": list(M_SWEEP), "weights": ["int8 per-channel", "int4 group 32"]},
        "cpu_baseline": {"value": v, "unit": "TOPS", "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------

class Sweep:
    """Device-resident inputs for N_SETS rotating copies of the sweep."""

    def __init__(self, torch, oc, device):
        import synth

        self.torch, self.oc = torch, oc
        A, WT, bias = synth.qgemm_case(max(M_SWEEP), K_DIM, N_DIM)
        self.host = (A, WT, bias)
        Wd = torch.from_numpy(WT).to(device)
        q8, s8 = oc.quantize_int8(Wd, K_DIM)       # per output channel
        q4, s4 = oc.quantize_int4(Wd, GROUP4)      # group 32, packed
        torch.cuda.synchronize()
        self.sets = []
        for _ in range(N_SETS):
            s = {
                "A": {m: torch.from_numpy(A[:m]).to(device) for m in M_SWEEP},
                "q8": q8.clone().view(N_DIM, K_DIM), "s8": s8.clone(),
                "q4": q4.clone(), "s4": s4.clone(),
                "bias": torch.from_numpy(bias).to(device),
                "Y": {m: torch.empty(m, N_DIM, dtype=torch.float32, device=device) for m in M_SWEEP},
                "qa": {m: torch.empty(m, K_DIM, dtype=torch.int8, device=device) for m in M_SWEEP},
                "sa": {m: torch.empty(m, dtype=torch.float32, device=device) for m in M_SWEEP},
            }
            self.sets.append(s)
        self.launches_per_step = 0

    def step(self, i):
        """One sweep on set i: 8 full quantized matmuls (oc_qgemm_*: row
        quantization of A + GEMM), 2 kernel launches each."""
        oc = self.oc
        s = self.sets[i % N_SETS]
        for m in M_SWEEP:
            oc.qgemm_w8a8(s["A"][m], s["q8"], s["s8"], s["bias"], out=s["Y"][m])
            oc.qgemm_w4a8(s["A"][m], s["q4"], s["s4"], GROUP4, s["bias"], out=s["Y"][m])
        return 4 * len(M_SWEEP)

    def prequantize(self):
        """qa/sa of every set, for timing the GEMM kernels alone."""
        for s in self.sets:
            for m in M_SWEEP:
                qa, sa = self.oc.quantize_rows_int8(s["A"][m])
                s["qa"][m].copy_(qa)
                s["sa"][m].copy_(sa)


def gemm_bytes(kind: str, m: int) -> int:
    """Algorithmic bytes of one GEMM launch: qa + sa + weights + scales + bias + Y."""
    w = N_DIM * K_DIM if kind == "w8" else N_DIM * K_DIM // 2
    sc = N_DIM * 4 if kind == "w8" else N_DIM * (K_DIM // GROUP4) * 4
    return m * K_DIM + m * 4 + w + sc + N_DIM * 4 + m * N_DIM * 4


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import opencuda_cuda as oc

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    sweep = Sweep(torch, oc, device)
    stream = torch.cuda.Stream(device)
    hbm_peak, peak_kind = load_peaks()

    # warm up eagerly (sets kernel attributes), then capture one graph per set
    oc.workspace(max(M_SWEEP), K_DIM, device)
    with torch.cuda.stream(stream):
        for i in range(N_SETS):
            sweep.step(i)
    stream.synchronize()
    graphs = []
    for i in range(N_SETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launches = sweep.step(i)
        graphs.append(g)
    torch.cuda.synchronize()

    if args.profile_once:
        for g in graphs:
            g.replay()
        torch.cuda.synchronize()
        return

    for i in range(args.warmup):
        graphs[i % N_SETS].replay()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.steps):
            graphs[i % N_SETS].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        dist.barrier()
    clk = clocks.stop()
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = sweep_ops() * world / (ms_step * 1e-3) / 1e12

    # per-kernel device times (each launch alone on the stream, rotating sets)
    # per-kernel device times: each GEMM kernel alone, REPS launches over the
    # rotating sets captured in one graph, events around the replay
    per = {}
    reps = 32
    with torch.cuda.stream(stream):
        sweep.prequantize()
    torch.cuda.synchronize()
    for kind in ("w8", "w4"):
        for m in M_SWEEP:
            def launch_all():
                for r in range(reps):
                    s = sweep.sets[r % N_SETS]
                    if kind == "w8":
                        oc.igemm_w8a8(s["qa"][m], s["sa"][m], s["q8"], s["s8"], s["bias"], out=s["Y"][m])
                    else:
                        oc.igemm_w4a8(s["qa"][m], s["sa"][m], s["q4"], s["s4"], GROUP4, s["bias"], out=s["Y"][m])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                launch_all()
            g.replay()
            torch.cuda.synchronize()
            samples = []
            for _ in range(3):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    a.record(stream)
                    g.replay()
                    b.record(stream)
                torch.cuda.synchronize()
                samples.append(a.elapsed_time(b) * 1e3 / reps)
            del g
            us = statistics.median(samples)
            ops = 2 * m * K_DIM * N_DIM
            by = gemm_bytes(kind, m)
            per[f"{kind}a8_M{m}"] = {"us": round(us, 3), "TOPS": round(ops / us / 1e6, 2),
                                     "GB/s": round(by / us / 1e3, 1)}
    dom = max(per, key=lambda k: per[k]["us"])
    dkind, dm = dom.split("a8_M")
    dm = int(dm)
    dbytes = gemm_bytes(dkind, dm)
    achieved = dbytes / (per[dom]["us"] * 1e-6) / 1e9
    roofline = {"bound": "hbm", "kernel": f"gemm_{dkind}a8 M={dm}", "achieved": round(achieved, 1),
                "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes": dbytes,
                "traffic": None}

    # e2e through the host-slice C ABI with pinned host buffers
    e2e = None
    if True:  # every rank runs its replica's e2e sweep; the max is reported
        A, WT, bias = sweep.host
        dev = oc.Device(local)
        s0 = sweep.sets[0]
        hA = {m: torch.from_numpy(A[:m]).pin_memory() for m in M_SWEEP}
        hq8, hs8 = s0["q8"].cpu().pin_memory(), s0["s8"].cpu().pin_memory()
        hq4, hs4 = s0["q4"].cpu().pin_memory(), s0["s4"].cpu().pin_memory()
        hb = torch.from_numpy(bias).pin_memory()
        hY = {m: torch.empty(m * N_DIM, dtype=torch.float32).pin_memory() for m in M_SWEEP}
        L = oc.lib()

        def e2e_step():
            for m in M_SWEEP:
                oc.check(L.oc_blas_qgemm_w8a8(dev.handle, m, N_DIM, K_DIM, hA[m].data_ptr(), hq8.data_ptr(),
                                              hs8.data_ptr(), hb.data_ptr(), hY[m].data_ptr()))
                oc.check(L.oc_blas_qgemm_w4a8(dev.handle, m, N_DIM, K_DIM, GROUP4, hA[m].data_ptr(),
                                              hq4.data_ptr(), hs4.data_ptr(), hb.data_ptr(), hY[m].data_ptr()))

        for _ in range(max(2, args.warmup)):
            e2e_step()
        e2e_steps = max(5, args.steps // 5)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step()
        t_e2e = (time.perf_counter() - t0) / e2e_steps
        if dist:
            t = torch.tensor([t_e2e], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        per_m_weights = hq8.numel() + hs8.numel() * 4 + hq4.numel() + hs4.numel() * 4 + 2 * hb.numel() * 4
        h2d = sum(2 * m * K_DIM * 4 + per_m_weights for m in M_SWEEP)
        d2h = sum(m * N_DIM * 4 for m in M_SWEEP) * 2
        e2e = {"value": sweep_ops() * world / t_e2e / 1e12, "unit": "TOPS", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(t_e2e * 1e3, 3)}
        dev.close()

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        tops, desc, cores, _ = cpu_reference_sample()
        cpu = {"value": tops, "unit": "TOPS", "cores": cores, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 x int8 -> int32 (f32 in/out)",
            "data": "synthetic (SplitMix64-seeded U(-1,1) activations, N(0,0.02) weights, no dataset)",
            "config": {"workload": "config-2 quantized GEMM sweep: M in {1,16,128,2048}, K=768, N=3072, "
                                   "W8A8 per-channel + W4A8 group-32, f32 bias and output",
                       "parallelism": f"replicas x{world}",
                       "l2": f"{N_SETS} rotating device input sets (~300 MB) > 126 MB L2",
                       "graph": "one CUDA graph per set (quantize + GEMM per matmul)"},
            "gpu_launches": launches * args.steps,
            "per_kernel": per,
            "roofline": roofline,
            "clocks": clk,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        del graphs
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
