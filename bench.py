#!/usr/bin/env python
"""Benchmarks of the open-cuda matmul hot path on B200.

Default workload (`--workload qgemm`, the headline metric): the INT8/INT4
weight-quantized GEMM sweep.  A[M x 768] (f32, U(-1,1), seed 1) times
W[768 x 3072] (N(0,0.02), seed 2, quantized by the reference's own
routines: INT8 per output channel, INT4 group 32) plus an f32 bias, for M in
{1, 16, 128, 2048} and both weight types -- 8 quantized matmuls per step,
each = activation row quantization + exact-int32 tensor-core GEMM (or the
skinny dp4a kernel for M <= 16) + dequantizing epilogue.

Other workloads (same JSON contract, one line each):
  sgemm     f32 A[512x768] . B[768x2304] + bias (GPT-2 c_attn shape), f16-term GEMM
  gpt2      GPT-2 124M random-init (load_random seed 3), 32-token prompts,
            128 greedy tokens, batch 32 (batch 1 reported beside it)
  int4      INT4 group-32 sweep K=3584, N in {3584, 18944, 152064},
            M in {1, 8, 64, 512, 4096}; N column-sharded over the ranks
            with an NCCL all-gather (strong scaling)
  moe       DeepSeek-style MoE: 8192 tokens x d 7168, 256 experts (d_ff 2048,
            INT8) + 1 shared, top-8; experts sharded over the ranks with NCCL
            all-to-all dispatch/combine (strong scaling)
  mla       MLA: KV[16384 x 7168] -> latent 512 -> K and V [16384 x 16384]
  flash     fused multi-head attention, 96 x 2048 x 64 and 32 x 4096 x 128,
            causal and full (tcgen05, f16 hi / lo operand terms)

value   = algorithmic work of one step / device time (CUDA events on the
          launching stream, max over ranks), whole job.
e2e     = the same metric through the reference-facing call with host
          buffers, host<->device copies inside the timed region.
`--impl reference` times the reference's CPU path for the workload (the C
restatement of its loops, all host cores) on a bounded sample.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "open-cuda_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

DATA = "synthetic (SplitMix64-seeded inputs as the reference's tests draw them; no dataset, no checkpoint)"

def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qgemm", choices=["qgemm", "qgemm_a8", "sgemm", "gpt2", "int4", "moe", "mla",
                                                           "flash"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-once", action="store_true",
                    help="run one warm pass of the workload's kernels and exit (for ncu launch lists)")
    ap.add_argument("--a8-k3584", action="store_true",
                    help="with --workload qgemm_a8 --profile-once: only the W8A8 GEMM at M=2048 K=3584 N=18944, "
                         "twice (for an ncu capture of the long-K kind::i8 kernel)")
    return ap.parse_args()


def load_peaks():
    """(hbm GB/s, int8 dense TOPS, tf32 dense TFLOP/s, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        bf16 = float(d["bf16_tflops"])
        return float(d["hbm_gbs"]), 2.0 * bf16, 0.5 * bf16, "measured"
    except Exception:
        return 6650.0, 2.0 * 1590.0, 0.5 * 1590.0, "fallback"


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


def roofline(kernel: str, ops: float, nbytes: float, us: float, peaks, ops_unit="TOPS"):
    """Roofline entry of one kernel: the bound is whichever of the tensor
    time (ops / dense peak) and the HBM time (algorithmic bytes / copy
    bandwidth) is longer; achieved and peak are in that bound's unit."""
    hbm, int8, tf32, src = peaks
    if ops_unit == "F16T3":  # f32 products as three f16-term MMAs at the bf16 rate
        tensor_peak = int8 / 2.0 / 3.0
    else:
        tensor_peak = int8 if ops_unit == "TOPS" else tf32 / 3.0  # 3xTF32: three MMAs per product
    t_tensor = ops / (tensor_peak * 1e12)
    t_hbm = nbytes / (hbm * 1e9)
    tr = None  # DRAM traffic comes from ncu captures, never from a timed run
    if t_hbm >= t_tensor:
        ach = nbytes / (us * 1e-6) / 1e9
        return {"bound": "hbm", "kernel": kernel, "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(ach / hbm, 4), "peak_source": f"{src} hbm_gbs (copy bandwidth)",
                "algorithmic_bytes": int(nbytes), "algorithmic_ops": int(ops), "us_per_launch": round(us, 3),
                "traffic": tr}
    ach = ops / (us * 1e-6) / 1e12
    unit = "TOPS" if ops_unit == "TOPS" else "TFLOP/s"
    how = {"TOPS": "int8 dense = 2 x measured bf16_tflops",
           "F16T3": "measured bf16_tflops / 3 (f16 MMAs at the bf16 rate, three per f32 product)"}.get(
        ops_unit, "3xTF32 effective = measured bf16_tflops / 2 (tf32 rate) / 3")
    return {"bound": "tensor", "kernel": kernel, "achieved": round(ach, 2), "peak": round(tensor_peak, 1),
            "unit": unit, "frac": round(ach / tensor_peak, 4), "peak_source": f"{src}: {how}",
            "algorithmic_bytes": int(nbytes), "algorithmic_ops": int(ops), "us_per_launch": round(us, 3),
            "traffic": tr}


# ----------------------------------------------------------------------------
# GPU context and timing
# ----------------------------------------------------------------------------

class Ctx:
    def __init__(self, args):
        import torch

        import opencuda_cuda as oc

        self.args = args
        self.torch, self.oc = torch, oc
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        self.dist = None
        if self.world > 1:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.device)
            self.dist = dist
        self.stream = torch.cuda.Stream(self.device)
        self.peaks = load_peaks()

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        if not self.dist:
            return v
        t = self.torch.tensor([v], device=self.device, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, run_step, steps: int, stream=None):
        """Device ms per step of `run_step(i)` for i in 0..steps-1 (CUDA
        events on the launching stream, barrier + synchronize on both sides,
        max over ranks) and the clock record of the timed region."""
        torch = self.torch
        s = stream if stream is not None else self.stream
        clocks = ClockSampler(self.local)
        clocks.start()
        time.sleep(0.3)
        self.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            for i in range(steps):
                run_step(i)
            e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        self.barrier()
        clk = clocks.stop()
        return self.max_over_ranks(ms) / steps, clk

    def kernel_us(self, launch, reps: int = 16, graph: bool = True) -> float:
        """Median device time of one `launch()` (events around `reps`
        back-to-back launches, from a CUDA graph when `graph`)."""
        torch = self.torch
        s = self.stream
        with torch.cuda.stream(s):
            launch()
        torch.cuda.synchronize()
        g = None
        if graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(reps):
                    launch()
        samples = []
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(s):
                a.record(s)
                if g is not None:
                    g.replay()
                else:
                    for _ in range(reps):
                        launch()
                b.record(s)
            torch.cuda.synchronize()
            samples.append(a.elapsed_time(b) * 1e3 / reps)
        del g
        return statistics.median(samples)

    def close(self, *graphs, finish=True):
        for g in graphs:
            del g
        if finish:
            self.finish()

    def finish(self):
        if self.dist:
            self.dist.barrier()
            self.dist.destroy_process_group()
            self.dist = None


def emit(ctx, metric, value, unit, ms_step, dtype, config, launches, roof, clk, e2e, cpu, extra=None,
         scaling="weak", higher=True):
    if ctx.rank != 0:
        return
    line = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": ctx.world, "steps": ctx.args.steps,
        "warmup": ctx.args.warmup, "ms_per_step": ms_step, "higher_is_better": higher, "scaling": scaling,
        "vs_baseline": None, "dtype": dtype, "data": DATA, "config": config, "gpu_launches": launches,
        "roofline": roof, "clocks": clk, "e2e": e2e, "cpu_baseline": cpu,
    }
    if extra:
        line.update(extra)
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# qgemm: INT8/INT4 weight-quantized GEMM sweep (headline)
# ----------------------------------------------------------------------------

Q_K, Q_N, Q_G = 768, 3072, 32
Q_M = (1, 16, 128, 2048)
Q_SETS = 48  # rotating input sets: 48 x 3.85 MB of quantized weights + scales (185 MB) > 126 MB L2
Q_METRIC = "INT8/INT4 weight-quantized GEMM TOPS (M in {1,16,128,2048}, K=768, N=3072)"
# config-4 cold-HBM decode GEMV: one activation row against the 7B-class vocabulary projection
V_K, V_N = 3584, 152064


def q_ops() -> int:
    return 2 * sum(2 * m * Q_K * Q_N for m in Q_M)  # two weight types


def wo_kernel_name(kind: str, m: int, k: int, n: int, group: int = Q_G) -> str:
    """The weight-only route the library takes for this call (oc_qgemm_wo.cu)."""
    if kind == "w4" and group == 32 and 1 <= m <= 64 and k % 128 == 0 and (n + 127) // 128 >= 148:
        return "wo4g_prep_kernel + gemm_wo4g_kernel"
    if m <= 16:
        return "wo_skinny_kernel"
    return "wo_prep_kernel + gemm_wo_kernel (one call)"


def wo_bytes(kind: str, m: int, k: int, n: int, group: int = Q_G) -> int:
    """Algorithmic bytes of one weight-only call: f32 A + quantized weights +
    f32 scales + bias + f32 Y."""
    w = n * k if kind == "w8" else n * k // 2
    sc = n * 4 if kind == "w8" else n * (k // group) * 4
    return m * k * 4 + w + sc + n * 4 + m * n * 4


def a8_bytes(kind: str, m: int) -> int:
    """Algorithmic bytes of one int8-activation GEMM launch: qa + sa + weights + scales + bias + Y."""
    w = Q_N * Q_K if kind == "w8" else Q_N * Q_K // 2
    sc = Q_N * 4 if kind == "w8" else Q_N * (Q_K // Q_G) * 4
    return m * Q_K + m * 4 + w + sc + Q_N * 4 + m * Q_N * 4


def wo_chunk_cols(k: int, wt: int = 2) -> int:
    """Columns per chunk of the weight-only GEMM (expanded terms <= 40 MB)."""
    return max(128, (40 << 20) // (k * 2 * wt + 4) // 128 * 128)


def wo_launches(m: int, k: int) -> int:
    """Kernels one weight-only call launches: the skinny kernel (m <= 16, one
    launch while the rows fit its shared memory) or preparation + GEMM."""
    if m <= 16:
        step = max(1, min(16, (200 << 10) // (k * 4)))
        return -(-m // step)
    return 2


def roofline_wo(kind: str, m: int, k: int, n: int, us: float, peaks, what: str):
    """Roofline of a weight-only call.  Its products run as f16 terms on the
    tensor cores: 2 kind::f16 MMAs per product step for INT8 weights, 3 for
    INT4, so the tensor ceiling is the measured bf16 dense rate / 2 or / 3 in
    f32-equivalent FLOP/s; the HBM ceiling is the algorithmic bytes at the
    measured copy bandwidth.  The bound is the longer of the two times."""
    hbm, _, _, src = peaks
    bf16 = 2.0 * peaks[2]
    terms = 2 if kind == "w8" else 3
    peak_t = bf16 / terms
    ops, nbytes = 2 * m * k * n, wo_bytes(kind, m, k, n)
    t_t, t_h = ops / (peak_t * 1e12), nbytes / (hbm * 1e9)
    common = {"kernel": what, "algorithmic_bytes": int(nbytes), "algorithmic_ops": int(ops),
              "us_per_launch": round(us, 3), "traffic": None}
    if t_h >= t_t:
        ach = nbytes / (us * 1e-6) / 1e9
        return dict(common, bound="hbm", achieved=round(ach, 1), peak=hbm, unit="GB/s", frac=round(ach / hbm, 4),
                    peak_source=f"{src} hbm_gbs (copy bandwidth)")
    ach = ops / (us * 1e-6) / 1e12
    return dict(common, bound="tensor", achieved=round(ach, 2), peak=round(peak_t, 1), unit="TFLOP/s",
                frac=round(ach / peak_t, 4),
                peak_source=f"{src} bf16_tflops / {terms} (f16 MMAs per f32 product step)")


def cpu_qgemm(target_s: float = 6.0):
    """The reference's CPU composition for the sweep: dequantize the weights,
    naive sgemm (one task per 256 output elements, strided B, the per-call
    copies) and the host bias add, on all host cores.  Large M are sampled
    by rows: t(rows) = fixed + rows * per_row, fitted from two calls."""
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    t_total = 0.0
    sample = []
    A_full, WT, bias = synth.qgemm_case(max(Q_M), Q_K, Q_N)
    t8 = oracle.quantize_int8(WT.ravel(), Q_K)
    t4 = oracle.quantize_int4(WT.ravel(), Q_G)
    budget = target_s / (2 * len(Q_M))

    def timed(bits, t, g, rows):
        t0 = time.perf_counter()
        oracle.qgemm_weight_only(bits, rows, Q_K, Q_N, g, A_full[:rows], t.data, t.scales, bias, faithful=True)
        return time.perf_counter() - t0

    for bits, t, g in ((8, t8, Q_K), (4, t4, Q_G)):
        t1 = timed(bits, t, g, 1)
        r2 = 8
        t2 = timed(bits, t, g, r2)
        per_row = max((t2 - t1) / (r2 - 1), 1e-9)
        fixed = max(t1 - per_row, 0.0)
        for m in Q_M:
            rows = max(1, min(m, int(max(budget - fixed, per_row) / per_row)))
            dt = timed(bits, t, g, rows)
            t_total += dt if rows == m else (dt - fixed) * (m / rows) + fixed
            sample.append(f"W{bits} M={m}: {rows} rows")
    v = q_ops() / t_total / 1e12
    desc = ("reference CPU path restated in C (dequantize + naive sgemm with per-call copies + bias); "
            + "; ".join(sample) + "; sampled calls scaled as fixed + rows * per-row time")
    return {"value": v, "unit": "TOPS", "cores": cores, "kind": "port", "sample": desc}


def _rotating_us(ctx, launch_of, nsets: int, reps: int = 32) -> float:
    """kernel_us of a launch that walks `nsets` input sets round robin."""
    ctr = [0]

    def launch():
        launch_of(ctr[0] % nsets)
        ctr[0] += 1

    return ctx.kernel_us(launch, reps=reps)


def qgemm_cold_gemv(ctx, once: bool = False):
    """Config-4 decode GEMV from cold HBM: M=1, K=3584, N=152064, weight-only
    INT8 (545 MB of weights) and INT4 g32 (272 MB packed + 68 MB scales)."""
    torch, oc = ctx.torch, ctx.oc
    g = torch.Generator(device=ctx.device).manual_seed(5)
    W = torch.randn(V_N, V_K, generator=g, device=ctx.device) * 0.02
    q8, s8 = oc.quantize_int8(W.view(-1), V_K)
    q4, s4 = oc.quantize_int4(W.view(-1), Q_G)
    del W
    A = torch.rand(1, V_K, generator=g, device=ctx.device) * 2 - 1
    b = torch.zeros(V_N, device=ctx.device)
    Y = torch.empty(1, V_N, device=ctx.device)
    out = {}
    for kind in ("w8", "w4"):
        def launch():
            if kind == "w8":
                oc.qgemm_w8(A, q8, s8, bias=b, out=Y)
            else:
                oc.qgemm_w4(A, q4, s4, Q_G, bias=b, out=Y)

        if once:
            launch()
            torch.cuda.synchronize()
            continue
        us = ctx.kernel_us(launch, reps=8)
        nb = wo_bytes(kind, 1, V_K, V_N)
        out[f"{kind}_M1_K{V_K}_N{V_N}"] = {"us": round(us, 2), "GB/s": round(nb / us / 1e3, 1),
                                           "frac_hbm": round(nb / us / 1e3 / ctx.peaks[0], 4),
                                           "bytes": nb, "kernel": wo_kernel_name(kind, 1, V_K, V_N)}
    del q8, s8, q4, s4
    torch.cuda.empty_cache()
    return out


def qgemm_gpt2_batch1(ctx):
    """GPT-2 124M greedy decode at batch 1 (load_random seed 3, 32-token
    prompt, 128 new tokens): tok/s and the decode step's weight bytes per
    second against HBM."""
    import gpt
    import synth

    torch = ctx.torch
    m = gpt.GptModel.load_random(gpt.GptConfig.gpt2_124m(), 3, device=ctx.local, max_batch=1,
                                 max_prompt_len=G_PROMPT)
    p = synth.gpt_prompts(1, G_PROMPT)[0]
    ext = torch.cuda.ExternalStream(m.stream(), device=ctx.device)
    for _ in range(3):
        m.generate(p, G_NEW)
    torch.cuda.synchronize()
    n0 = m.kernel_launches()
    steps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(steps):
        m.generate(p, G_NEW)
    e1.record(ext)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    launches = (m.kernel_launches() - n0) // steps
    m.close()
    H, V, I = 768, 50257, 3072
    step_bytes = 12 * 4 * (H * 3 * H + H * H + H * I + I * H) + 4 * H * V
    per_tok_us = ms * 1e3 / G_NEW
    gbs = step_bytes / (per_tok_us * 1e-6) / 1e9
    return {"tok_s": round(G_NEW / (ms * 1e-3), 1), "us_per_token": round(per_tok_us, 2),
            "weight_bytes_per_token": step_bytes, "GB/s": round(gbs, 1), "frac_hbm": round(gbs / ctx.peaks[0], 4),
            "gpu_launches_per_generate": launches,
            "note": "per-token time includes the amortised 32-token prefill"}


def other_configs(ctx):
    """Compact device-timed figures of the other configs, so that the default
    line carries one of each (the per-workload lines hold the full sweeps):
    config 1 sgemm, config 4's vocabulary-shaped INT4 GEMM at M = 64 and
    4096, config 5's MLA projections and MoE block.  CUDA events, inputs
    resident in HBM, rotating sets or operands larger than L2."""
    import moe
    import synth

    torch, oc = ctx.torch, ctx.oc
    d = ctx.device
    out = {}
    # config 1: sgemm 512x768x2304 + bias (16 rotating sets, 213 MB)
    A, B, bias = s_case()
    sets = [(torch.from_numpy(A).to(d), torch.from_numpy(B).to(d), torch.from_numpy(bias).to(d),
             torch.empty(S_M, S_N, device=d)) for _ in range(S_SETS)]
    us = _rotating_us(ctx, lambda j: oc.sgemm(sets[j][0], sets[j][1], C=sets[j][3], bias=sets[j][2]), S_SETS)
    out["sgemm_512x768x2304"] = {"us": round(us, 2), "TFLOP/s": round(2 * S_M * S_K * S_N / us / 1e6, 1)}
    del sets
    # config 4: INT4 g32 weight-only at K=3584, N=152064 (340 MB of weights and scales)
    g = torch.Generator(device=d).manual_seed(5)
    W = torch.randn(V_N, V_K, generator=g, device=d) * 0.02
    q4, s4 = oc.quantize_int4(W.view(-1), Q_G)
    del W
    for m in (64, 4096):
        Am = torch.rand(m, V_K, generator=g, device=d) * 2 - 1
        Y = torch.empty(m, V_N, device=d)
        us = ctx.kernel_us(lambda: oc.qgemm_w4(Am, q4, s4, Q_G, out=Y), reps=3, graph=False)
        out[f"int4_M{m}_K{V_K}_N{V_N}"] = {"us": round(us, 1), "TFLOP/s": round(2 * m * V_K * V_N / us / 1e6, 1)}
        del Am, Y
    del q4, s4
    torch.cuda.empty_cache()
    # config 5: MLA compress 16384x7168 -> 512 and one decompress 512 -> 16384
    kv = torch.randn(L_SEQ, L_DH, generator=g, device=d) * 0.02
    down = torch.randn(L_DH, L_DC, generator=g, device=d) * 0.02
    up = torch.randn(L_DC, L_UP, generator=g, device=d) * 0.02
    lat = oc.mla_compress_kv(kv, down)
    us_c = ctx.kernel_us(lambda: oc.mla_compress_kv(kv, down), reps=3, graph=False)
    us_d = ctx.kernel_us(lambda: oc.mla_decompress_kv(lat, up), reps=3, graph=False)
    out["mla"] = {"compress_us": round(us_c, 1), "compress_TFLOP/s": round(2 * L_SEQ * L_DH * L_DC / us_c / 1e6, 1),
                  "decompress_us": round(us_d, 1), "decompress_TFLOP/s": round(2 * L_SEQ * L_DC * L_UP / us_d / 1e6, 1)}
    del kv, down, up, lat
    torch.cuda.empty_cache()
    # config 5: MoE block, 8192 tokens, 256 INT8 experts top-8 + the shared expert (one GPU)
    w = moe.random_weights(E_E, E_D, E_F, 5, d)
    x = torch.from_numpy(synth.uniform(70, E_T * E_D).reshape(E_T, E_D)).to(d)
    lg = torch.from_numpy(synth.normal(71, E_T * E_E).reshape(E_T, E_E)).to(d)
    with torch.cuda.stream(ctx.stream):
        moe.moe_forward(x, lg, w, E_K)
    torch.cuda.synchronize()
    us = ctx.kernel_us(lambda: moe.moe_forward(x, lg, w, E_K), reps=3, graph=False)
    out["moe_block"] = {"us": round(us, 1), "TOPS": round(e_ops() / us / 1e6, 1)}
    del w, x, lg
    torch.cuda.empty_cache()
    return out


def qgemm_sharded(ctx):
    """N > 1: the config-4 column-sharded INT4 g32 weight-only GEMM (K=3584,
    N=152064): each rank computes its N/g columns, one NCCL all-gather plus
    oc_gather_columns lay them out as [M][N] on every rank.  Timed per M with
    the exchange inside (max over ranks), the all-gather alone beside it;
    rank 0 checks the gathered result bit for bit against every shard's
    product computed on its own GPU."""
    import shard

    torch, oc = ctx.torch, ctx.oc
    plan = shard.ColumnShard(V_N, ctx.world)
    g = torch.Generator(device=ctx.device).manual_seed(5)
    W = torch.randn(V_N, V_K, generator=g, device=ctx.device) * 0.02  # the same matrix on every rank
    q4, s4 = oc.quantize_int4(W.view(-1), Q_G)
    del W
    bias = torch.randn(V_N, generator=g, device=ctx.device) * 0.02
    (b0, b1), (c0, c1) = plan.w4_slices(ctx.rank, V_K, Q_G)
    r0, r1 = plan.rows(ctx.rank)
    wl, sl, bl = q4[b0:b1].clone(), s4[c0:c1].clone(), bias[r0:r1].clone()
    out = {"ranks": ctx.world, "columns_per_rank": plan.cols, "collective": "NCCL all_gather_into_tensor",
           "per_M": {}}
    identical = True
    for m in (1, 512, 4096):
        A = torch.rand(m, V_K, generator=g, device=ctx.device) * 2 - 1

        def step(_i):
            local = oc.qgemm_w4(A, wl, sl, Q_G, bias=bl)
            return shard.gather_columns(local, plan)

        local = oc.qgemm_w4(A, wl, sl, Q_G, bias=bl)
        flat = torch.empty(ctx.world * local.numel(), device=ctx.device)
        with torch.cuda.stream(ctx.stream):
            for i in range(3):
                y = step(i)
                ctx.dist.all_gather_into_tensor(flat, local.view(-1))
        torch.cuda.synchronize()
        reps = 10 if m < 4096 else 5
        ms, _ = ctx.timed(step, reps)
        ms_ag, _ = ctx.timed(lambda _i: ctx.dist.all_gather_into_tensor(flat, local.view(-1)), reps)
        with torch.cuda.stream(ctx.stream):
            y = step(0)
        torch.cuda.synchronize()
        if ctx.rank == 0:  # every shard's product on this GPU, laid side by side
            ref = torch.empty(m, V_N, device=ctx.device)
            for r in range(ctx.world):
                (x0, x1), (y0, y1) = plan.w4_slices(r, V_K, Q_G)
                s0_, s1_ = plan.rows(r)
                ref[:, s0_:s1_] = oc.qgemm_w4(A, q4[x0:x1], s4[y0:y1], Q_G, bias=bias[s0_:s1_])
            torch.cuda.synchronize()
            identical = identical and bool(torch.equal(ref.view(torch.int32), y.view(torch.int32)))
            del ref
        ops = 2 * m * V_K * V_N
        out["per_M"][f"M{m}"] = {"ms": round(ms, 4), "allgather_ms": round(ms_ag, 4),
                                 "allgather_share": round(ms_ag / ms, 3), "TOPS": round(ops / (ms * 1e-3) / 1e12, 2),
                                 "gathered_MB": round(m * V_N * 4 / 2 ** 20, 1)}
    out["bit_identical_to_shards_on_one_gpu"] = identical
    return out


def moe_ep_extra(ctx):
    """N > 1: the config-5 MoE block run expert-parallel (E/g experts and T/g
    tokens per rank, the shared expert on every rank): count all-to-all, row
    all-to-all, output all-to-all (NCCL).  Timed with the exchanges inside
    (max over ranks), and the three all-to-alls alone with the same splits
    beside it."""
    import moe
    import synth

    torch = ctx.torch
    import torch.distributed as dist

    g = ctx.world
    w = moe.random_weights(E_E // g, E_D, E_F, 5 + ctx.rank, ctx.device)
    T = E_T // g
    x = torch.from_numpy(synth.uniform(70 + ctx.rank, T * E_D).reshape(T, E_D)).to(ctx.device)
    lg = torch.from_numpy(synth.normal(71 + ctx.rank, T * E_E).reshape(T, E_E)).to(ctx.device)
    torch.cuda.synchronize()

    def step(_i):
        return moe.moe_forward_ep(x, lg, w, E_E, E_K)

    with torch.cuda.stream(ctx.stream):
        for _ in range(2):
            step(0)
    torch.cuda.synchronize()
    ms, _ = ctx.timed(step, 5)
    # the exchanges alone, with this block's splits
    idx, _tw = moe.route(lg, E_K)
    dest = torch.div(idx, E_E // g, rounding_mode="floor").reshape(-1)
    cnt_send = torch.bincount(dest, minlength=g).to(torch.int32)
    cnt_recv = torch.empty_like(cnt_send)
    dist.all_to_all_single(cnt_recv, cnt_send)
    send, recv = [int(v) for v in cnt_send.tolist()], [int(v) for v in cnt_recv.tolist()]
    row_bytes = E_D + 8  # int8 row, f32 scale, int32 local expert id
    sb = torch.empty(sum(send), row_bytes, dtype=torch.uint8, device=ctx.device)
    rb = torch.empty(sum(recv), row_bytes, dtype=torch.uint8, device=ctx.device)
    ob = torch.empty(sum(recv), E_D, device=ctx.device)
    bb = torch.empty(sum(send), E_D, device=ctx.device)

    def exchange(_i):
        dist.all_to_all_single(cnt_recv, cnt_send)
        dist.all_to_all_single(rb, sb, recv, send)
        dist.all_to_all_single(bb, ob, send, recv)

    ms_x, _ = ctx.timed(exchange, 5)
    ops = e_ops() / g  # this rank's share of the block's work
    return {"ranks": g, "experts_per_rank": E_E // g, "tokens_per_rank": T, "collective": "NCCL all_to_all_single x3",
            "ms": round(ms, 3), "all_to_all_ms": round(ms_x, 3), "all_to_all_share": round(ms_x / ms, 3),
            "TOPS": round(ops * g / (ms * 1e-3) / 1e12, 1),
            "rows_sent": sum(send), "MB_exchanged_per_rank": round((sum(send) * row_bytes + sum(recv) * E_D * 4) / 2 ** 20, 1)}


def run_qgemm(ctx):
    torch, oc, args = ctx.torch, ctx.oc, ctx.args
    import synth

    if args.profile_once and args.a8_k3584:
        m, n, K = A8_BIG[0][0], A8_BIG[0][1], 3584
        g = torch.Generator(device=ctx.device).manual_seed(9)
        qw, sw = oc.quantize_int8((torch.randn(n, K, generator=g, device=ctx.device) * 0.02).view(-1), K)
        qa, sa = oc.quantize_rows_int8(torch.rand(m, K, generator=g, device=ctx.device) * 2 - 1)
        Y = torch.empty(m, n, device=ctx.device)
        for _ in range(2):
            oc.igemm_w8a8(qa, sa, qw.view(n, K), sw, None, out=Y)
        torch.cuda.synchronize()
        return
    A, WT, bias = synth.qgemm_case(max(Q_M), Q_K, Q_N)
    Wd = torch.from_numpy(WT).to(ctx.device)
    q8, s8 = oc.quantize_int8(Wd, Q_K)       # per output channel
    q4, s4 = oc.quantize_int4(Wd, Q_G)      # group 32, packed
    Ad = torch.from_numpy(A).to(ctx.device)
    bd = torch.from_numpy(bias).to(ctx.device)
    torch.cuda.synchronize()
    sets = []
    for _ in range(Q_SETS):
        sets.append({
            "A": {m: Ad[:m].clone() for m in Q_M},
            "q8": q8.clone().view(Q_N, Q_K), "s8": s8.clone(), "q4": q4.clone(), "s4": s4.clone(),
            "bias": bd.clone(),
            "Y": {m: torch.empty(m, Q_N, dtype=torch.float32, device=ctx.device) for m in Q_M},
        })

    def step(i):
        s = sets[i % Q_SETS]
        for m in Q_M:
            oc.qgemm_w8(s["A"][m], s["q8"], s["s8"], bias=s["bias"], out=s["Y"][m])
            oc.qgemm_w4(s["A"][m], s["q4"], s["s4"], Q_G, bias=s["bias"], out=s["Y"][m])
        return 2 * sum(wo_launches(m, Q_K) for m in Q_M)

    with torch.cuda.stream(ctx.stream):
        for i in range(Q_SETS):  # scratch sized before capture
            step(i)
    ctx.stream.synchronize()
    graphs = []
    for i in range(Q_SETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=ctx.stream):
            launches = step(i)
        graphs.append(g)
    torch.cuda.synchronize()
    if args.profile_once:  # one replay of every set, then one cold-HBM GEMV of each weight type
        for g in graphs:
            g.replay()
        torch.cuda.synchronize()
        qgemm_cold_gemv(ctx, once=True)
        return
    for i in range(args.warmup):
        graphs[i % Q_SETS].replay()
    torch.cuda.synchronize()
    ms_step, clk = ctx.timed(lambda i: graphs[i % Q_SETS].replay(), args.steps)
    value = q_ops() * ctx.world / (ms_step * 1e-3) / 1e12

    # each weight-only call alone (rotating sets: cold weights)
    per = {}
    for kind in ("w8", "w4"):
        for m in Q_M:
            def call(j, kind=kind, m=m):
                s = sets[j]
                if kind == "w8":
                    oc.qgemm_w8(s["A"][m], s["q8"], s["s8"], bias=s["bias"], out=s["Y"][m])
                else:
                    oc.qgemm_w4(s["A"][m], s["q4"], s["s4"], Q_G, bias=s["bias"], out=s["Y"][m])

            us = _rotating_us(ctx, call, Q_SETS)
            ops = 2 * m * Q_K * Q_N
            per[f"{kind}_M{m}"] = {"us": round(us, 3), "TFLOP/s": round(ops / us / 1e6, 2),
                                   "GB/s": round(wo_bytes(kind, m, Q_K, Q_N) / us / 1e3, 1),
                                   "launches": wo_launches(m, Q_K)}
    dom = max(per, key=lambda key: per[key]["us"])
    dkind, dm = dom.split("_M")
    dm = int(dm)
    what = wo_kernel_name(dkind, dm, Q_K, Q_N) + f" {dkind} M={dm}"
    roof = roofline_wo(dkind, dm, Q_K, Q_N, per[dom]["us"], ctx.peaks, what)

    # the int8-activation kernels (W8A8 / W4A8, exact int32) on the same sets
    per_a8 = {}
    pre = [{m: oc.quantize_rows_int8(s["A"][m]) for m in Q_M} for s in sets]
    torch.cuda.synchronize()
    for kind in ("w8", "w4"):
        for m in Q_M:
            def call(j, kind=kind, m=m):
                s, (qa, sa) = sets[j], pre[j][m]
                if kind == "w8":
                    oc.igemm_w8a8(qa, sa, s["q8"], s["s8"], s["bias"], out=s["Y"][m])
                else:
                    oc.igemm_w4a8(qa, sa, s["q4"], s["s4"], Q_G, s["bias"], out=s["Y"][m])

            us = _rotating_us(ctx, call, Q_SETS)
            per_a8[f"{kind}a8_M{m}"] = {"us": round(us, 3), "TOPS": round(2 * m * Q_K * Q_N / us / 1e6, 2),
                                        "GB/s": round(a8_bytes(kind, m) / us / 1e3, 1)}
    del pre

    # e2e through the host-slice C ABI (oc_blas_qgemm_w8 / _w4) with pinned host buffers
    dev = oc.Device(ctx.local)
    s0 = sets[0]
    hA = {m: torch.from_numpy(A[:m]).pin_memory() for m in Q_M}
    hq8, hs8 = s0["q8"].cpu().pin_memory(), s0["s8"].cpu().pin_memory()
    hq4, hs4 = s0["q4"].cpu().pin_memory(), s0["s4"].cpu().pin_memory()
    hb = torch.from_numpy(bias).pin_memory()
    hY = {m: torch.empty(m * Q_N, dtype=torch.float32).pin_memory() for m in Q_M}
    L = oc.lib()

    def e2e_step():
        for m in Q_M:
            oc.check(L.oc_blas_qgemm_w8(dev.handle, m, Q_N, Q_K, hA[m].data_ptr(), hq8.data_ptr(),
                                        hs8.data_ptr(), hb.data_ptr(), hY[m].data_ptr()))
            oc.check(L.oc_blas_qgemm_w4(dev.handle, m, Q_N, Q_K, Q_G, hA[m].data_ptr(), hq4.data_ptr(),
                                        hs4.data_ptr(), hb.data_ptr(), hY[m].data_ptr()))

    for _ in range(max(2, args.warmup)):
        e2e_step()
    n_e2e = max(5, args.steps // 5)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        e2e_step()
    t_e2e = ctx.max_over_ranks((time.perf_counter() - t0) / n_e2e)
    per_m_w = hq8.numel() + hs8.numel() * 4 + hq4.numel() + hs4.numel() * 4 + 2 * hb.numel() * 4
    e2e = {"value": q_ops() * ctx.world / t_e2e / 1e12, "unit": "TOPS",
           "h2d_bytes_per_step": sum(2 * m * Q_K * 4 + per_m_w for m in Q_M),
           "d2h_bytes_per_step": sum(m * Q_N * 4 for m in Q_M) * 2, "ms_per_step": round(t_e2e * 1e3, 3)}
    dev.close()
    extra = {"per_kernel": per, "per_kernel_int8_activations": per_a8}
    ctx.close(*graphs, finish=False)  # the extras below still use the process group
    graphs = []
    extra["gemv_cold_hbm"] = qgemm_cold_gemv(ctx)
    extra["gpt2_batch1"] = qgemm_gpt2_batch1(ctx)
    extra["flash_attention"] = flash_cases(ctx)
    extra["other_configs"] = other_configs(ctx)
    if ctx.world > 1:
        extra["sharded"] = qgemm_sharded(ctx)
        extra["moe_expert_parallel"] = moe_ep_extra(ctx)
    cpu = cpu_qgemm() if ctx.rank == 0 and not args.no_cpu_baseline else None
    config = {"workload": WORKLOADS["qgemm"],
              "parallelism": f"replicas x{ctx.world}",
              "l2": f"{Q_SETS} rotating device input sets (weights alone 185 MB) > 126 MB L2",
              "graph": "one CUDA graph per set (8 weight-only matmuls)"}
    emit(ctx, Q_METRIC, value, "TOPS", ms_step, "f32 (f32 activations x dequantized int8 / int4 weights)", config,
         launches * args.steps, roof, clk, e2e, cpu, extra)
    ctx.finish()


# ----------------------------------------------------------------------------
# qgemm_a8: the same sweep with int8 activations (W8A8 / W4A8, exact int32)
# ----------------------------------------------------------------------------

A8_SETS = 8
A8_BIG = ((2048, 18944), (4096, 18944), (2048, 152064), (4096, 152064))  # W8A8 at K=3584


def cpu_qgemm_a8(target_s: float = 6.0):
    """The exact int8-activation product (the oracle's W8A8 / W4A8, no
    reference counterpart: the reference has no int8-activation path), all
    host cores, rows sampled per call as in cpu_qgemm."""
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    A_full, WT, bias = synth.qgemm_case(max(Q_M), Q_K, Q_N)
    t8 = oracle.quantize_int8(WT.ravel(), Q_K)
    t4 = oracle.quantize_int4(WT.ravel(), Q_G)
    budget = target_s / (2 * len(Q_M))
    t_total, sample = 0.0, []

    def timed(bits, rows):
        t0 = time.perf_counter()
        if bits == 8:
            oracle.qgemm_w8a8(rows, Q_K, Q_N, A_full[:rows], t8.data, t8.scales, bias)
        else:
            oracle.qgemm_w4a8(rows, Q_K, Q_N, Q_G, A_full[:rows], t4.data, t4.scales, bias)
        return time.perf_counter() - t0

    for bits in (8, 4):
        t1, t2 = timed(bits, 1), timed(bits, 8)
        per_row = max((t2 - t1) / 7, 1e-9)
        fixed = max(t1 - per_row, 0.0)
        for m in Q_M:
            rows = max(1, min(m, int(max(budget - fixed, per_row) / per_row)))
            dt = timed(bits, rows)
            t_total += dt if rows == m else (dt - fixed) * (m / rows) + fixed
            sample.append(f"W{bits}A8 M={m}: {rows} rows")
    return {"value": q_ops() / t_total / 1e12, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": "exact int8-activation oracle in C (no reference counterpart); " + "; ".join(sample)
                      + "; sampled calls scaled as fixed + rows * per-row time"}


def run_qgemm_a8(ctx):
    torch, oc, args = ctx.torch, ctx.oc, ctx.args
    import synth

    if args.profile_once and args.a8_k3584:
        m, n, K = A8_BIG[0][0], A8_BIG[0][1], 3584
        g = torch.Generator(device=ctx.device).manual_seed(9)
        qw, sw = oc.quantize_int8((torch.randn(n, K, generator=g, device=ctx.device) * 0.02).view(-1), K)
        qa, sa = oc.quantize_rows_int8(torch.rand(m, K, generator=g, device=ctx.device) * 2 - 1)
        Y = torch.empty(m, n, device=ctx.device)
        for _ in range(2):
            oc.igemm_w8a8(qa, sa, qw.view(n, K), sw, None, out=Y)
        torch.cuda.synchronize()
        return
    A, WT, bias = synth.qgemm_case(max(Q_M), Q_K, Q_N)
    Wd = torch.from_numpy(WT).to(ctx.device)
    q8, s8 = oc.quantize_int8(Wd, Q_K)
    q4, s4 = oc.quantize_int4(Wd, Q_G)
    torch.cuda.synchronize()
    sets = []
    for _ in range(A8_SETS):
        sets.append({
            "A": {m: torch.from_numpy(A[:m]).to(ctx.device) for m in Q_M},
            "q8": q8.clone().view(Q_N, Q_K), "s8": s8.clone(), "q4": q4.clone(), "s4": s4.clone(),
            "bias": torch.from_numpy(bias).to(ctx.device),
            "Y": {m: torch.empty(m, Q_N, dtype=torch.float32, device=ctx.device) for m in Q_M},
        })

    def step(i):
        s = sets[i % A8_SETS]
        for m in Q_M:
            oc.qgemm_w8a8(s["A"][m], s["q8"], s["s8"], s["bias"], out=s["Y"][m])
            oc.qgemm_w4a8(s["A"][m], s["q4"], s["s4"], Q_G, s["bias"], out=s["Y"][m])
        return 4 * len(Q_M)  # row quantization + GEMM per matmul

    oc.workspace(max(Q_M), Q_K, ctx.device)
    with torch.cuda.stream(ctx.stream):
        for i in range(A8_SETS):
            step(i)
    ctx.stream.synchronize()
    graphs = []
    for i in range(A8_SETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=ctx.stream):
            launches = step(i)
        graphs.append(g)
    torch.cuda.synchronize()
    if args.profile_once:
        for g in graphs:
            g.replay()
        torch.cuda.synchronize()
        return
    for i in range(args.warmup):
        graphs[i % A8_SETS].replay()
    torch.cuda.synchronize()
    ms_step, clk = ctx.timed(lambda i: graphs[i % A8_SETS].replay(), args.steps)
    value = q_ops() * ctx.world / (ms_step * 1e-3) / 1e12
    per = {}
    pre = [{m: oc.quantize_rows_int8(s["A"][m]) for m in Q_M} for s in sets]
    torch.cuda.synchronize()
    for kind in ("w8", "w4"):
        for m in Q_M:
            def call(j, kind=kind, m=m):
                s, (qa, sa) = sets[j], pre[j][m]
                if kind == "w8":
                    oc.igemm_w8a8(qa, sa, s["q8"], s["s8"], s["bias"], out=s["Y"][m])
                else:
                    oc.igemm_w4a8(qa, sa, s["q4"], s["s4"], Q_G, s["bias"], out=s["Y"][m])

            us = _rotating_us(ctx, call, A8_SETS)
            per[f"{kind}a8_M{m}"] = {"us": round(us, 3), "TOPS": round(2 * m * Q_K * Q_N / us / 1e6, 2),
                                     "GB/s": round(a8_bytes(kind, m) / us / 1e3, 1)}
    dom = max(per, key=lambda k: per[k]["us"])
    dkind, dm = dom.split("a8_M")
    dm = int(dm)
    roof = roofline(f"gemm_{dkind}a8 M={dm}", 2 * dm * Q_K * Q_N, a8_bytes(dkind, dm), per[dom]["us"], ctx.peaks)
    # W8A8 at 7B-class shapes (K=3584): the kind::i8 GEMM where the epilogue is amortised over a long K
    big = {}
    K = 3584
    g = torch.Generator(device=ctx.device).manual_seed(9)
    for m, n in A8_BIG:
        W = torch.randn(n, K, generator=g, device=ctx.device) * 0.02
        qw, sw = oc.quantize_int8(W.view(-1), K)
        del W
        qa, sa = oc.quantize_rows_int8(torch.rand(m, K, generator=g, device=ctx.device) * 2 - 1)
        Y = torch.empty(m, n, device=ctx.device)
        us = ctx.kernel_us(lambda: oc.igemm_w8a8(qa, sa, qw.view(n, K), sw, None, out=Y), reps=4)
        ops = 2 * m * n * K
        big[f"w8a8_M{m}_K{K}_N{n}"] = {"us": round(us, 1), "TOPS": round(ops / us / 1e6, 1),
                                       "frac_int8_dense": round(ops / us / 1e6 / ctx.peaks[1], 4),
                                       "int8_peak_source": f"{ctx.peaks[3]}: 2 x bf16_tflops"}
        del qw, sw, qa, Y
    torch.cuda.empty_cache()
    # W4A8 at M=2048: the two-term kind::f16 path (the default) against the
    # exact per-group kind::i8 kernel, which runs when the int32 group
    # partials are requested (it writes them: 4 * M * N * K / 32 bytes)
    s0, m = sets[0], max(Q_M)
    acc = torch.empty(m, Q_N, Q_K // Q_G, dtype=torch.int32, device=ctx.device)
    ws = oc.workspace(m, Q_K, ctx.device)
    L = oc.lib()
    us_f16 = ctx.kernel_us(lambda: oc.qgemm_w4a8(s0["A"][m], s0["q4"], s0["s4"], Q_G, s0["bias"], out=s0["Y"][m]),
                           reps=8)
    us_i8 = ctx.kernel_us(lambda: oc.check(L.oc_qgemm_w4a8(m, Q_N, Q_K, Q_G, s0["A"][m].data_ptr(),
                                                           s0["q4"].data_ptr(), s0["s4"].data_ptr(),
                                                           s0["bias"].data_ptr(), s0["Y"][m].data_ptr(),
                                                           ws.data_ptr(), ws.numel(), acc.data_ptr(),
                                                           ctx.stream.cuda_stream)), reps=4)
    ops = 2 * m * Q_K * Q_N
    w4_paths = {"two_term_f16": {"us": round(us_f16, 1), "TOPS": round(ops / us_f16 / 1e6, 1),
                                 "ceiling": "f16 MMA rate (bf16_tflops) / 2 MMAs = 1/4 of INT8 dense"},
                "exact_i8_per_group": {"us": round(us_i8, 1), "TOPS": round(ops / us_i8 / 1e6, 1),
                                       "partials_bytes": int(acc.numel() * 4),
                                       "ceiling": "INT8 dense for the MMAs; the drain promotes M*N*K/32 group sums "
                                                  "in group order and stores the partials"}}
    del acc
    torch.cuda.empty_cache()
    # e2e through the host-slice C ABI (oc_blas_qgemm_w8a8 / _w4a8) with pinned host buffers
    dev = oc.Device(ctx.local)
    hA = {mm: torch.from_numpy(A[:mm]).pin_memory() for mm in Q_M}
    hq8, hs8 = s0["q8"].cpu().pin_memory(), s0["s8"].cpu().pin_memory()
    hq4, hs4 = s0["q4"].cpu().pin_memory(), s0["s4"].cpu().pin_memory()
    hb = torch.from_numpy(bias).pin_memory()
    hY = {mm: torch.empty(mm * Q_N, dtype=torch.float32).pin_memory() for mm in Q_M}

    def e2e_step():
        for mm in Q_M:
            oc.check(L.oc_blas_qgemm_w8a8(dev.handle, mm, Q_N, Q_K, hA[mm].data_ptr(), hq8.data_ptr(),
                                          hs8.data_ptr(), hb.data_ptr(), hY[mm].data_ptr()))
            oc.check(L.oc_blas_qgemm_w4a8(dev.handle, mm, Q_N, Q_K, Q_G, hA[mm].data_ptr(), hq4.data_ptr(),
                                          hs4.data_ptr(), hb.data_ptr(), hY[mm].data_ptr()))

    for _ in range(max(2, args.warmup)):
        e2e_step()
    n_e2e = max(5, args.steps // 5)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        e2e_step()
    t_e2e = ctx.max_over_ranks((time.perf_counter() - t0) / n_e2e)
    per_m_w = hq8.numel() + hs8.numel() * 4 + hq4.numel() + hs4.numel() * 4 + 2 * hb.numel() * 4
    e2e = {"value": q_ops() * ctx.world / t_e2e / 1e12, "unit": "TOPS",
           "h2d_bytes_per_step": sum(2 * mm * Q_K * 4 + per_m_w for mm in Q_M),
           "d2h_bytes_per_step": sum(mm * Q_N * 4 for mm in Q_M) * 2, "ms_per_step": round(t_e2e * 1e3, 3)}
    dev.close()
    cpu = cpu_qgemm_a8() if ctx.rank == 0 and not args.no_cpu_baseline else None
    config = {"workload": WORKLOADS["qgemm_a8"], "parallelism": f"replicas x{ctx.world}",
              "l2": f"{A8_SETS} rotating device input sets (~300 MB) > 126 MB L2",
              "graph": "one CUDA graph per set (row quantization + GEMM per matmul)"}
    emit(ctx, "INT8-activation quantized GEMM TOPS (W8A8 / W4A8, M in {1,16,128,2048}, K=768, N=3072)", value,
         "TOPS", ms_step, "int8 x int8 -> int32 (f32 in/out)", config, launches * args.steps, roof, clk, e2e, cpu,
         {"per_kernel": per, "w8a8_k3584": big, "w4a8_M2048_paths": w4_paths})
    ctx.close(*graphs)


# ----------------------------------------------------------------------------
# sgemm: f32 GEMM of the GPT-2 c_attn shape (f16-term tensor-core GEMM)
# ----------------------------------------------------------------------------

S_M, S_K, S_N = 512, 768, 2304
S_SETS = 16


def s_case():
    import synth

    v = synth.normal(0, S_M * S_K + S_K * S_N + S_N, 0.0, 0.02)
    A = v[: S_M * S_K].reshape(S_M, S_K)
    B = v[S_M * S_K: S_M * S_K + S_K * S_N].reshape(S_K, S_N)
    bias = v[S_M * S_K + S_K * S_N:]
    return A, B, bias


def cpu_sgemm():
    import oracle

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    A, B, bias = s_case()
    ts = []
    for _ in range(2):
        t0 = time.perf_counter()
        C = oracle.sgemm(S_M, S_K, S_N, 1.0, A, B, 0.0, np.zeros(S_M * S_N, np.float32), faithful=True)
        C = C.reshape(S_M, S_N) + bias  # Linear::forward's host bias add
        ts.append(time.perf_counter() - t0)
    v = 2 * S_M * S_K * S_N / min(ts) / 1e12
    return {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": "full call: restated launch_naive_gemm (per-call copies, 256-element tasks) + host bias add"}


def run_sgemm(ctx):
    torch, oc, args = ctx.torch, ctx.oc, ctx.args
    A, B, bias = s_case()
    d = ctx.device
    sets = [{"A": torch.from_numpy(A).to(d), "B": torch.from_numpy(B).to(d), "bias": torch.from_numpy(bias).to(d),
             "C": torch.empty(S_M, S_N, dtype=torch.float32, device=d)} for _ in range(S_SETS)]

    def step(i):
        s = sets[i % S_SETS]
        oc.sgemm(s["A"], s["B"], C=s["C"], bias=s["bias"])
        return 3  # B's column maxima, the f16 terms of A and B, the GEMM

    with torch.cuda.stream(ctx.stream):
        for i in range(S_SETS):
            step(i)
    torch.cuda.synchronize()
    graphs = []
    for i in range(S_SETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=ctx.stream):
            launches = step(i)
        graphs.append(g)
    if args.profile_once:
        for g in graphs:
            g.replay()
        torch.cuda.synchronize()
        return
    for i in range(args.warmup):
        graphs[i % S_SETS].replay()
    ms_step, clk = ctx.timed(lambda i: graphs[i % S_SETS].replay(), args.steps)
    flops = 2 * S_M * S_K * S_N
    value = flops * ctx.world / (ms_step * 1e-3) / 1e12
    # the call alone (column maxima, f16 terms, GEMM), rotating over the sets
    ctr = [0]

    def launch():
        j = ctr[0] % S_SETS
        ctr[0] += 1
        s = sets[j]
        oc.sgemm(s["A"], s["B"], C=s["C"], bias=s["bias"])

    us = ctx.kernel_us(launch, reps=32)
    nbytes = 4 * (S_M * S_K + S_K * S_N + S_N + S_M * S_N)  # A, B, bias, C
    roof = roofline("sgemm call (f32_colmax + f32_terms + gemm_wo<WT=2>) 512x768x2304", flops, nbytes, us,
                    ctx.peaks, ops_unit="F16T3")
    # e2e: the reference's blas-level sgemm (host slices in and out) + the caller's host bias add
    dev = oc.Device(ctx.local)
    hA = torch.from_numpy(A).pin_memory().numpy()
    hB = torch.from_numpy(B).pin_memory().numpy()
    hC = torch.zeros(S_M * S_N, dtype=torch.float32).pin_memory().numpy()

    def e2e_step():
        dev.sgemm(S_M, S_K, S_N, 1.0, hA, hB, 0.0, hC)
        hC.reshape(S_M, S_N).__iadd__(bias)

    for _ in range(3):
        e2e_step()
    n = max(10, args.steps)
    t0 = time.perf_counter()
    for _ in range(n):
        e2e_step()
    t_e2e = ctx.max_over_ranks((time.perf_counter() - t0) / n)
    e2e = {"value": flops * ctx.world / t_e2e / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": 4 * (A.size + B.size + S_M * S_N),
           "d2h_bytes_per_step": 4 * S_M * S_N, "ms_per_step": round(t_e2e * 1e3, 4)}
    dev.close()
    cpu = cpu_sgemm() if ctx.rank == 0 and not args.no_cpu_baseline else None
    config = {"workload": WORKLOADS["sgemm"],
              "parallelism": f"replicas x{ctx.world}", "l2": f"{S_SETS} rotating sets (213 MB) > 126 MB L2",
              "graph": "one CUDA graph per set"}
    emit(ctx, "sgemm TFLOP/s (f32, 512x768x2304 + bias)", value, "TFLOP/s", ms_step,
         "f32 (f16 hi/lo terms of both operands on tensor cores, f32 accumulate)", config, launches * args.steps, roof, clk, e2e, cpu,
         {"call_us": round(us, 3)})
    ctx.close(*graphs)


# ----------------------------------------------------------------------------
# gpt2: GPT-2 124M greedy decode
# ----------------------------------------------------------------------------

G_PROMPT, G_NEW = 32, 128


def cpu_gpt2(new_tokens: int = 4):
    """The reference's generate (q replicated n times, every Linear through
    the naive sgemm with per-call copies) for one sequence, timed for a few
    new tokens; tok/s = new tokens / time (prefill included)."""
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    cfg = oracle.GptConfig(50257, 768, 12, 12, 3072, 1024, 1e-5)
    m = oracle.GptModel(cfg, 3)
    m.set_attention(flash=True, block=64, faithful=True)
    p = synth.gpt_prompts(1, G_PROMPT)[0]
    t0 = time.perf_counter()
    m.generate(p, new_tokens)
    dt = time.perf_counter() - t0
    return {"value": new_tokens / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"batch 1, prompt {G_PROMPT}, {new_tokens} greedy tokens (prefill included), "
                      "reference generate restated in C with naive sgemm and replicated-q flash attention"}


def run_gpt2(ctx):
    torch, args = ctx.torch, ctx.args
    import gpt
    import synth

    batches = (1, 32) if args.profile_once else (32, 1)
    models = {}
    res = {}
    for b in batches:
        m = gpt.GptModel.load_random(gpt.GptConfig.gpt2_124m(), 3, device=ctx.local, max_batch=b,
                                     max_prompt_len=G_PROMPT)
        models[b] = m
        prompts = synth.gpt_prompts(b, G_PROMPT)
        ext = torch.cuda.ExternalStream(m.stream(), device=ctx.device)
        if args.profile_once:  # one generate per batch size
            m.generate(prompts, G_NEW)
            continue
        for _ in range(max(3, args.warmup)):
            m.generate(prompts, G_NEW)
        steps = args.steps if b == 32 else max(3, args.steps // 2)
        n0 = m.kernel_launches()
        ms, clk = ctx.timed(lambda i: m.generate(prompts, G_NEW), steps, stream=ext)
        launches = m.kernel_launches() - n0
        # e2e: generate is the reference-facing call (host prompt ids in, host tokens out)
        t0 = time.perf_counter()
        for _ in range(steps):
            m.generate(prompts, G_NEW)
        t_e2e = ctx.max_over_ranks((time.perf_counter() - t0) / steps)
        toks = b * G_NEW
        res[b] = {"tok_s": toks * ctx.world / (ms * 1e-3), "ms": ms, "clk": clk, "launches": launches,
                  "e2e_tok_s": toks * ctx.world / t_e2e, "e2e_ms": t_e2e * 1e3, "steps": steps}
    if args.profile_once:
        return
    # decode GEMV roofline: the lm_head GEMV at batch 1 dominates the decode step
    m1 = models[1]
    H, V, I = 768, 50257, 3072
    layer_w = 4 * (H * 3 * H + H * H + H * I + I * H)
    step_bytes = 12 * layer_w + 4 * H * V  # every weight read once per decode step (f32)
    per_tok_us = res[1]["ms"] * 1e3 / G_NEW
    roof = {"bound": "hbm", "kernel": "whole decode step, batch 1 (graph of GEMV/attention kernels)",
            "achieved": round(step_bytes / (per_tok_us * 1e-6) / 1e9, 1), "peak": ctx.peaks[0], "unit": "GB/s",
            "frac": round(step_bytes / (per_tok_us * 1e-6) / 1e9 / ctx.peaks[0], 4),
            "peak_source": f"{ctx.peaks[3]} hbm_gbs", "algorithmic_bytes": step_bytes,
            "note": "per-token time includes the amortised 32-token prefill", "traffic": None}
    r = res[32]
    e2e = {"value": r["e2e_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 32 * G_PROMPT * 4,
           "d2h_bytes_per_step": 32 * G_NEW * 4, "ms_per_step": round(r["e2e_ms"], 3)}
    cpu = cpu_gpt2() if ctx.rank == 0 and not args.no_cpu_baseline else None
    config = {"workload": WORKLOADS["gpt2"], "parallelism": f"replicas x{ctx.world}",
              "graph": "decode step captured once, replayed per token", "l2": "weights 497 MB > 126 MB L2"}
    extra = {"batch1": {"tok_s": res[1]["tok_s"], "ms_per_generate": res[1]["ms"],
                        "e2e_tok_s": res[1]["e2e_tok_s"], "gpu_launches": res[1]["launches"]}}
    emit(ctx, "GPT-2 124M greedy decode tok/s (batch 32, prompt 32, 128 new tokens)", r["tok_s"], "tok/s",
         r["ms"], "f32", config, r["launches"], roof, r["clk"], e2e, cpu, extra)
    for m in models.values():
        m.close()
    ctx.close()


# ----------------------------------------------------------------------------
# int4: INT4 group-32 GEMM sweep at 7B-class shapes, N column-sharded
# ----------------------------------------------------------------------------

I_K, I_G = 3584, 32
I_N = (3584, 18944, 152064)
I_M = (1, 8, 64, 512, 4096)


def i_ops() -> int:
    return sum(2 * m * I_K * n for m in I_M for n in I_N)


def cpu_int4(target_s: float = 12.0):
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    total = 0.0
    sample = []
    for n in I_N:
        A, WT, bias = synth.qgemm_case(8, I_K, n, 4, 5, 6)
        t4 = oracle.quantize_int4(WT.ravel(), I_G)

        def timed(rows):
            t0 = time.perf_counter()
            oracle.qgemm_weight_only(4, rows, I_K, n, I_G, A[:rows], t4.data, t4.scales, bias, faithful=True)
            return time.perf_counter() - t0

        t1, t2 = timed(1), timed(4)
        per_row = max((t2 - t1) / 3, 1e-9)
        fixed = max(t1 - per_row, 0.0)
        for m in I_M:
            total += fixed + per_row * m
        sample.append(f"N={n}: 1 and 4 rows")
    v = i_ops() / total / 1e12
    return {"value": v, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": "dequantize + naive sgemm per (M,N): " + "; ".join(sample)
                      + "; every M scaled as fixed + M * per-row time"}


def run_int4(ctx):
    torch, oc, args = ctx.torch, ctx.oc, ctx.args
    import shard
    import synth

    d = ctx.device
    cases = {}
    for n in I_N:
        A, WT, bias = synth.qgemm_case(max(I_M), I_K, n, 4, 5, 6)
        plan = shard.ColumnShard(n, ctx.world)
        r0, r1 = plan.rows(ctx.rank)
        Wl = torch.from_numpy(np.ascontiguousarray(WT[r0:r1])).to(d)
        q4, s4 = oc.quantize_int4(Wl, I_G)  # this rank's rows = its slice of the full quantization
        del Wl
        copies = max(1, -(-160_000_000 // (q4.numel() + s4.numel() * 4)))  # rotate > L2
        cases[n] = {"plan": plan, "A": {m: torch.from_numpy(A[:m]).to(d) for m in I_M},
                    "w": [(q4.clone(), s4.clone()) for _ in range(copies)],
                    "bias": torch.from_numpy(bias[r0:r1]).to(d), "host": (A, WT, bias)}
    torch.cuda.synchronize()

    def step(i):
        n_l = 0
        for n in I_N:
            c = cases[n]
            q4, s4 = c["w"][i % len(c["w"])]
            for m in I_M:
                y = oc.qgemm_w4(c["A"][m], q4, s4, I_G, bias=c["bias"])
                if wo_kernel_name("w4", m, I_K, c["plan"].cols, I_G).startswith("wo4g"):
                    n_l += 2  # digit preparation + GEMM
                else:
                    n_l += wo_launches(m, I_K) * (1 if m <= 16 else -(-c["plan"].cols // wo_chunk_cols(I_K)))
                if ctx.world > 1:
                    shard.gather_columns(y, c["plan"])
                    n_l += 1  # gather kernel (plus the NCCL all-gather)
        return n_l

    with torch.cuda.stream(ctx.stream):
        for i in range(2):
            launches = step(i)
    torch.cuda.synchronize()
    if args.profile_once:
        return
    with torch.cuda.stream(ctx.stream):
        for i in range(args.warmup):
            step(i)
    ms_step, clk = ctx.timed(step, args.steps)
    value = i_ops() / (ms_step * 1e-3) / 1e12
    # the dominant call: time each local GEMM alone
    per = {}
    for n in I_N:
        c = cases[n]
        nl = c["plan"].cols
        Y = {m: torch.empty(m, nl, dtype=torch.float32, device=d) for m in I_M}
        for m in I_M:
            def call(j, c=c, m=m):
                q4, s4 = c["w"][j]
                oc.qgemm_w4(c["A"][m], q4, s4, I_G, bias=c["bias"], out=Y[m])

            us = _rotating_us(ctx, call, len(c["w"]), reps=8)
            per[f"M{m}_N{n}"] = {"us": round(us, 2), "TFLOP/s": round(2 * m * I_K * nl / us / 1e6, 2),
                                 "GB/s": round(wo_bytes("w4", m, I_K, nl, I_G) / us / 1e3, 1)}
    dom = max(per, key=lambda k: per[k]["us"])
    dm, dn = [int(x[1:]) for x in dom.split("_")]
    nl = cases[dn]["plan"].cols
    what = wo_kernel_name("w4", dm, I_K, nl, I_G) + f" M={dm} N={nl}"
    roof = roofline_wo("w4", dm, I_K, nl, per[dom]["us"], ctx.peaks, what)
    # e2e: rank 0 runs the host-slice call for its shard (weights copied per call, as blas does)
    dev = oc.Device(ctx.local)
    L = oc.lib()
    hosts = {}
    for n in I_N:
        c = cases[n]
        q4, s4 = c["w"][0]
        hosts[n] = (q4.cpu().pin_memory(), s4.cpu().pin_memory(), c["bias"].cpu().pin_memory(),
                    {m: torch.from_numpy(c["host"][0][:m]).pin_memory() for m in I_M},
                    {m: torch.empty(m * c["plan"].cols, dtype=torch.float32).pin_memory() for m in I_M})

    def e2e_step():
        for n in I_N:
            hq, hs, hb, hA, hY = hosts[n]
            nl = cases[n]["plan"].cols
            for m in I_M:
                oc.check(L.oc_blas_qgemm_w4(dev.handle, m, nl, I_K, I_G, hA[m].data_ptr(), hq.data_ptr(),
                                            hs.data_ptr(), hb.data_ptr(), hY[m].data_ptr()))

    e2e_step()
    t0 = time.perf_counter()
    ne = 2
    for _ in range(ne):
        e2e_step()
    t_e2e = ctx.max_over_ranks((time.perf_counter() - t0) / ne)
    h2d = sum(hosts[n][0].numel() + hosts[n][1].numel() * 4 + hosts[n][2].numel() * 4 for n in I_N) * len(I_M)
    h2d += sum(m * I_K * 4 for m in I_M) * len(I_N)
    d2h = sum(m * cases[n]["plan"].cols * 4 for m in I_M for n in I_N)
    e2e = {"value": i_ops() / t_e2e / 1e12, "unit": "TOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "ms_per_step": round(t_e2e * 1e3, 2),
           "note": "host-slice oc_blas_qgemm_w4 per rank shard (no gather on the host path)"}
    dev.close()
    cpu = cpu_int4() if ctx.rank == 0 and not args.no_cpu_baseline else None
    config = {"workload": WORKLOADS["int4"],
              "parallelism": f"column shard x{ctx.world} + NCCL all-gather" if ctx.world > 1 else "1 GPU",
              "l2": "weights rotated over copies so every step reads > 126 MB"}
    emit(ctx, "INT4 g32 GEMM TOPS (K=3584 sweep)", value, "TOPS", ms_step,
         "f32 (f32 activations x dequantized int4 weights)",
         config, launches * args.steps, roof, clk, e2e, cpu, {"per_kernel": per}, scaling="strong")
    ctx.close()


# ----------------------------------------------------------------------------
# moe: DeepSeek-style MoE block, experts sharded over the ranks
# ----------------------------------------------------------------------------

E_T, E_D, E_F, E_E, E_K = 8192, 7168, 2048, 256, 8


def e_ops() -> int:
    return 2 * 2 * E_D * E_F * (E_T * E_K + E_T)  # routed + shared expert, two GEMMs each


def cpu_moe(tokens: int = 4):
    """The MoE oracle (W8A8 expert MLPs, per-token loops) on `tokens` tokens
    routed top-8 over 8 experts of the full shape; the per-token work (8
    routed + 1 shared expert MLP) is that of the full block, scaled to 8192."""
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    rng = np.random.default_rng(0)
    E = 8
    w1 = rng.integers(-127, 128, (E, E_F, E_D), dtype=np.int8)
    w2 = rng.integers(-127, 128, (E, E_D, E_F), dtype=np.int8)
    s1 = np.full(E * E_F, 1e-4, np.float32)
    s2 = np.full(E * E_D, 1e-4, np.float32)
    x = synth.uniform(70, tokens * E_D).reshape(tokens, E_D)
    lg = synth.normal(71, tokens * E).reshape(tokens, E)
    t0 = time.perf_counter()
    oracle.moe_forward(x, lg, w1, s1, w2, s2, w1[0], s1[:E_F], w2[0], s2[:E_D], E_K)
    dt = time.perf_counter() - t0
    v = e_ops() / (dt * E_T / tokens) / 1e12
    return {"value": v, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": f"{tokens} tokens through the MoE oracle (8 routed + 1 shared W8A8 expert MLPs of the full "
                      "shape per token), time scaled linearly to 8192 tokens"}


def run_moe(ctx):
    torch, oc, args = ctx.torch, ctx.oc, ctx.args
    import moe
    import synth

    d = ctx.device
    g = ctx.world
    full = moe.random_weights(E_E // g if g > 1 else E_E, E_D, E_F, 5 + ctx.rank, d) if g > 1 else \
        moe.random_weights(E_E, E_D, E_F, 5, d)
    w = full  # with g > 1 each rank draws only its own E/g experts
    T = E_T // g
    x = torch.from_numpy(synth.uniform(70 + ctx.rank, T * E_D).reshape(T, E_D)).to(d)
    lg = torch.from_numpy(synth.normal(71 + ctx.rank, T * E_E).reshape(T, E_E)).to(d)
    torch.cuda.synchronize()

    def step(i):
        if g > 1:
            return moe.moe_forward_ep(x, lg, w, E_E, E_K)
        return moe.moe_forward(x, lg, w, E_K)

    with torch.cuda.stream(ctx.stream):
        for i in range(2 if args.profile_once else max(3, args.warmup)):
            step(i)
    torch.cuda.synchronize()
    if args.profile_once:
        return
    steps = max(3, min(args.steps, 20))
    ms_step, clk = ctx.timed(step, steps)
    value = e_ops() / (ms_step * 1e-3) / 1e12
    # dominant kernel: the grouped expert GEMMs on this rank's routed rows
    with torch.cuda.stream(ctx.stream):
        qx, sx = oc.quantize_rows_int8(x)
        idx, tw = moe.route(lg, E_K)
        e_loc = E_E // g
        keys = idx if g == 1 else torch.remainder(idx, e_loc).to(torch.int32)
        counts, offs, pos, src, xg, sg = moe.dispatch(keys, qx, sx, e_loc)
        H = moe.grouped_gemm(xg, sg, w.w1.reshape(-1, E_D), w.s1, offs, e_loc)
        qh, sh = moe.gelu_quantize_rows(H)
    torch.cuda.synchronize()
    R = xg.shape[0]
    us1 = ctx.kernel_us(lambda: moe.grouped_gemm(xg, sg, w.w1.reshape(-1, E_D), w.s1, offs, e_loc), reps=3,
                        graph=False)
    us2 = ctx.kernel_us(lambda: moe.grouped_gemm(qh, sh, w.w2.reshape(-1, E_F), w.s2, offs, e_loc), reps=3,
                        graph=False)
    ops1 = 2 * R * E_D * E_F
    b1 = R * E_D + R * 4 + e_loc * E_F * E_D + e_loc * E_F * 4 + R * E_F * 4
    roof = roofline(f"grouped_w8a8 fc R={R} N={E_F} K={E_D} G={e_loc}", ops1, b1, us1, ctx.peaks)
    per = {"grouped_fc_us": round(us1, 1), "grouped_fc_TOPS": round(ops1 / us1 / 1e6, 1),
           "grouped_proj_us": round(us2, 1), "grouped_proj_TOPS": round(ops1 / us2 / 1e6, 1)}
    # e2e: tokens and router logits from pinned host memory, y back to pinned host memory
    hx = x.cpu().pin_memory()
    hl = lg.cpu().pin_memory()
    hy = torch.empty(T, E_D, dtype=torch.float32).pin_memory()

    def e2e_step():
        xd = hx.to(d, non_blocking=True)
        ld = hl.to(d, non_blocking=True)
        y = moe.moe_forward_ep(xd, ld, w, E_E, E_K) if g > 1 else moe.moe_forward(xd, ld, w, E_K)
        hy.copy_(y, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step()
    ne = 3
    t0 = time.perf_counter()
    for _ in range(ne):
        e2e_step()
    t_e2e = ctx.max_over_ranks((time.perf_counter() - t0) / ne)
    e2e = {"value": e_ops() / t_e2e / 1e12, "unit": "TOPS", "h2d_bytes_per_step": (T * E_D + T * E_E) * 4,
           "d2h_bytes_per_step": T * E_D * 4, "ms_per_step": round(t_e2e * 1e3, 2)}
    cpu = cpu_moe() if ctx.rank == 0 and not args.no_cpu_baseline else None
    launches = 13 if g == 1 else 13 + 3  # + dispatch by rank, regroup by expert, gather back
    config = {"workload": WORKLOADS["moe"],
              "parallelism": f"expert parallel x{g} (32 experts per GPU at 8), NCCL all-to-all" if g > 1
              else "1 GPU, all experts local",
              "l2": "expert weights 7.5 GB > 126 MB L2"}
    emit(ctx, "MoE block TOPS (8192 tokens, 256 experts top-8 + shared, INT8)", value, "TOPS", ms_step,
         "int8 x int8 -> int32 (f32 in/out)", config, launches * steps, roof, clk, e2e, cpu,
         {"per_kernel": per}, scaling="strong")
    ctx.close()


# ----------------------------------------------------------------------------
# mla: MLA compress / decompress as f16-term tensor-core GEMMs
# ----------------------------------------------------------------------------

L_SEQ, L_DH, L_DC, L_UP = 4 * 4096, 7168, 512, 128 * 128


def l_flops() -> int:
    return 2 * L_SEQ * L_DH * L_DC + 2 * 2 * L_SEQ * L_DC * L_UP


def cpu_mla(rows: int = 8):
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    kv = synth.normal(90, rows * L_DH, 0.0, 0.02).reshape(rows, L_DH)
    down = synth.normal(91, L_DH * L_DC, 0.0, 0.02).reshape(L_DH, L_DC)
    up = synth.normal(92, L_DC * L_UP, 0.0, 0.02).reshape(L_DC, L_UP)

    def once(r):
        t0 = time.perf_counter()
        lat = oracle.mla_compress_kv(r, L_DH, L_DC, kv[:r], down)
        oracle.mla_decompress_kv(r, L_DC, L_UP, lat, up)
        oracle.mla_decompress_kv(r, L_DC, L_UP, lat, up)
        return time.perf_counter() - t0

    t1, t2 = once(1), once(rows)
    per_row = max((t2 - t1) / (rows - 1), 1e-9)
    fixed = max(t1 - per_row, 0.0)
    total = fixed + per_row * L_SEQ
    return {"value": l_flops() / total / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"compress + 2 decompress on 1 and {rows} rows (naive sgemm with per-call copies), "
                      "scaled as fixed + rows * per-row time to 16384 rows"}


def run_mla(ctx):
    torch, oc, args = ctx.torch, ctx.oc, ctx.args
    d = ctx.device
    gen = torch.Generator(device=d)
    gen.manual_seed(90)
    kv = torch.randn(L_SEQ, L_DH, generator=gen, device=d).mul_(0.02)
    down = torch.randn(L_DH, L_DC, generator=gen, device=d).mul_(0.02)
    upk = torch.randn(L_DC, L_UP, generator=gen, device=d).mul_(0.02)
    upv = torch.randn(L_DC, L_UP, generator=gen, device=d).mul_(0.02)

    def step(i):
        lat = oc.mla_compress_kv(kv, down)
        oc.mla_decompress_kv(lat, upk)
        oc.mla_decompress_kv(lat, upv)
        return 9  # each: B's column maxima, the f16 terms of both operands, the GEMM

    with torch.cuda.stream(ctx.stream):
        for i in range(2 if args.profile_once else max(3, args.warmup)):
            launches = step(i)
    torch.cuda.synchronize()
    if args.profile_once:
        return
    steps = max(3, min(args.steps, 20))
    ms_step, clk = ctx.timed(step, steps)
    value = l_flops() * ctx.world / (ms_step * 1e-3) / 1e12
    lat = oc.mla_compress_kv(kv, down)
    us_c = ctx.kernel_us(lambda: oc.mla_compress_kv(kv, down), reps=3, graph=False)
    us_d = ctx.kernel_us(lambda: oc.mla_decompress_kv(lat, upk), reps=3, graph=False)
    fl_d = 2 * L_SEQ * L_DC * L_UP
    roof = roofline("mla_decompress call (f32_colmax + f32_terms + gemm_wo<WT=2>)", fl_d,
                    4 * (L_SEQ * L_DC + L_DC * L_UP + L_SEQ * L_UP), us_d, ctx.peaks, ops_unit="F16T3")
    per = {"compress_us": round(us_c, 1), "compress_TFLOPs": round(2 * L_SEQ * L_DH * L_DC / us_c / 1e6, 1),
           "decompress_us": round(us_d, 1), "decompress_TFLOPs": round(fl_d / us_d / 1e6, 1)}
    # e2e through the host-slice C ABI
    dev = oc.Device(ctx.local)
    L = oc.lib()
    hkv = kv.cpu().pin_memory()
    hdown, hupk, hupv = down.cpu().pin_memory(), upk.cpu().pin_memory(), upv.cpu().pin_memory()
    hlat = torch.empty(L_SEQ * L_DC, dtype=torch.float32).pin_memory()
    hout = torch.empty(L_SEQ * L_UP, dtype=torch.float32).pin_memory()

    def e2e_step():
        oc.check(L.oc_blas_mla_compress_kv(dev.handle, L_SEQ, L_DH, L_DC, hkv.data_ptr(), hdown.data_ptr(),
                                           hlat.data_ptr()))
        for up in (hupk, hupv):
            oc.check(L.oc_blas_mla_decompress_kv(dev.handle, L_SEQ, L_DC, L_UP, hlat.data_ptr(), up.data_ptr(),
                                                 hout.data_ptr()))

    e2e_step()
    t0 = time.perf_counter()
    e2e_step()
    t_e2e = ctx.max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": l_flops() * ctx.world / t_e2e / 1e12, "unit": "TFLOP/s",
           "h2d_bytes_per_step": 4 * (L_SEQ * L_DH + L_DH * L_DC + 2 * (L_SEQ * L_DC + L_DC * L_UP)),
           "d2h_bytes_per_step": 4 * (L_SEQ * L_DC + 2 * L_SEQ * L_UP), "ms_per_step": round(t_e2e * 1e3, 2)}
    dev.close()
    cpu = cpu_mla() if ctx.rank == 0 and not args.no_cpu_baseline else None
    config = {"workload": WORKLOADS["mla"], "parallelism": f"replicas x{ctx.world}",
              "l2": "operands 0.5-1 GB > 126 MB L2"}
    emit(ctx, "MLA compress+decompress TFLOP/s (f32)", value, "TFLOP/s", ms_step,
         "f32 (f16 hi/lo terms of both operands on tensor cores, f32 accumulate)", config, launches * steps, roof, clk, e2e, cpu,
         {"per_kernel": per})
    ctx.close()


# ----------------------------------------------------------------------------
# flash: fused multi-head attention on the tensor cores
# ----------------------------------------------------------------------------

# (batch * heads, seq, head_dim, causal); q_len = kv_len = seq
F_CASES = ((96, 2048, 64, True), (96, 2048, 64, False), (32, 4096, 128, True), (32, 4096, 128, False))
F_METRIC = ("fused attention TFLOP/s (f32; [batch*heads] x seq x head_dim = 96x2048x64 and 32x4096x128, "
            "causal and full)")


def f_flops(case) -> float:
    """4 * d flops per visible (query, key) pair: Q.K^T and P.V."""
    bh, s, d, causal = case
    pairs = s * (s + 1) / 2 if causal else s * s
    return 4.0 * bh * pairs * d


def f_tensor_peak(peaks) -> float:
    """Dense f16 tensor rate (= the measured bf16 rate) / 3: three MMAs per
    f32 product (hi.hi + hi.lo + lo.hi)."""
    return peaks[1] / 2.0 / 3.0


def cpu_flash(target_s: float = 2.0):
    """The reference's flash_attention (blas:589-678, full attention, block
    64) restated in C, query rows spread over all host threads, on whole
    heads of 2048 x 64."""
    import oracle
    import synth

    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    s, d = 2048, 64
    q = synth.normal(95, s * d, 0.0, 1.0)
    k = synth.normal(96, s * d, 0.0, 1.0)
    v = synth.normal(97, s * d, 0.0, 1.0)
    t0 = time.perf_counter()
    oracle.flash_attention(q, k, v, s, d, 64)
    one = time.perf_counter() - t0
    n = max(1, min(64, int(target_s / max(one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(n):
        oracle.flash_attention(q, k, v, s, d, 64)
    dt = time.perf_counter() - t0
    return {"value": 4.0 * s * s * d * n / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{n} heads of {s} x {d} (full attention, block 64), rows over {cores} threads"}


def flash_cases(ctx, reps: int = 5):
    """Device time of each F_CASES launch (median of 3 x `reps`), its TFLOP/s
    and fraction of the f16 tensor rate / 3, beside torch's f32
    scaled_dot_product_attention on the same tensors (a library kernel,
    for context)."""
    torch, oc = ctx.torch, ctx.oc
    F = torch.nn.functional
    out = {}
    peak = f_tensor_peak(ctx.peaks)
    for i, case in enumerate(F_CASES):
        bh, s, d, causal = case
        g = torch.Generator(device=ctx.device).manual_seed(100 + i)
        q, k, v = (torch.randn(bh, s, d, generator=g, device=ctx.device) for _ in range(3))
        us = ctx.kernel_us(lambda: oc.flash_attention_fwd(q, k, v, causal=causal), reps=reps, graph=False)
        us_t = ctx.kernel_us(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal), reps=reps,
                             graph=False)
        tf = f_flops(case) / us / 1e6
        out[f"{bh}x{s}x{d}{'_causal' if causal else ''}"] = {
            "us": round(us, 1), "TFLOPs": round(tf, 1), "frac_tensor": round(tf / peak, 4),
            "kernel": f"flash_tc_kernel<{d}>", "torch_sdpa_f32_us": round(us_t, 1)}
        del q, k, v
    torch.cuda.empty_cache()
    return out


def run_flash(ctx):
    torch, oc, args = ctx.torch, ctx.oc, ctx.args
    gen = torch.Generator(device=ctx.device).manual_seed(100)
    data = [tuple(torch.randn(bh, s, d, generator=gen, device=ctx.device) for _ in range(3))
            for (bh, s, d, _c) in F_CASES]

    def step(i):
        for (q, k, v), case in zip(data, F_CASES):
            oc.flash_attention_fwd(q, k, v, causal=case[3])
        return len(F_CASES)

    with torch.cuda.stream(ctx.stream):
        for i in range(1 if args.profile_once else max(3, args.warmup)):
            launches = step(i)
    torch.cuda.synchronize()
    if args.profile_once:
        return
    steps = max(3, min(args.steps, 20))
    ms_step, clk = ctx.timed(step, steps)
    total = sum(f_flops(c) for c in F_CASES)
    value = total * ctx.world / (ms_step * 1e-3) / 1e12
    per = flash_cases(ctx)
    big = F_CASES[3]
    key = f"{big[0]}x{big[1]}x{big[2]}"
    peak = f_tensor_peak(ctx.peaks)
    us = per[key]["us"]
    roof = {"bound": "tensor", "kernel": f"flash_tc_kernel<{big[2]}> {key} full", "achieved": per[key]["TFLOPs"],
            "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(per[key]["TFLOPs"] / peak, 4),
            "peak_source": f"{ctx.peaks[3]} bf16_tflops / 3 (f16 MMAs at the bf16 rate, three per f32 product)",
            "algorithmic_ops": int(f_flops(big)), "algorithmic_bytes": int(4 * 4 * big[0] * big[1] * big[2]),
            "us_per_launch": us, "traffic": None}
    # e2e: pinned host inputs -> device, the public call, outputs -> host
    host = [tuple(t.cpu().pin_memory() for t in qkv) for qkv in data]
    outs = [torch.empty_like(qkv[0], device="cpu").pin_memory() for qkv in host]

    def e2e_step():
        for (hq, hk, hv), ho, case in zip(host, outs, F_CASES):
            q, k, v = (t.to(ctx.device, non_blocking=True) for t in (hq, hk, hv))
            ho.copy_(oc.flash_attention_fwd(q, k, v, causal=case[3]), non_blocking=True)
        torch.cuda.synchronize()

    e2e_step()
    t0 = time.perf_counter()
    e2e_step()
    t_e2e = ctx.max_over_ranks(time.perf_counter() - t0)
    nbytes = sum(4 * bh * s * d for (bh, s, d, _c) in F_CASES)
    e2e = {"value": total * ctx.world / t_e2e / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": 3 * nbytes,
           "d2h_bytes_per_step": nbytes, "ms_per_step": round(t_e2e * 1e3, 2)}
    cpu = cpu_flash() if ctx.rank == 0 and not args.no_cpu_baseline else None
    config = {"workload": WORKLOADS["flash"], "parallelism": f"replicas x{ctx.world}",
              "l2": "q, k, v of each case 151-201 MB > 126 MB L2"}
    emit(ctx, F_METRIC, value, "TFLOP/s", ms_step, "f32 (f16 hi / lo operand terms on tcgen05, f32 accumulate)",
         config, launches * steps, roof, clk, e2e, cpu, {"per_kernel": per})
    ctx.close()


# ----------------------------------------------------------------------------
# reference arm
# ----------------------------------------------------------------------------

WORKLOADS = {
    "qgemm": "config-2 quantized GEMM sweep: M in {1,16,128,2048}, K=768, N=3072, f32 activations, INT8 per-channel "
             "and INT4 group-32 weights (weight-only: sgemm(A, dequantize(W)^T) + bias), f32 bias and output",
    "qgemm_a8": "config-2 shapes with int8 activations: M in {1,16,128,2048}, K=768, N=3072, W8A8 per-channel + "
                "W4A8 group-32 (activation rows quantized on the device, exact int32 products), f32 bias and output; "
                "W8A8 at K=3584 beside it",
    "sgemm": "config-1 sgemm: A[512x768] . B[768x2304] + bias, N(0,0.02) seed 0",
    "gpt2": "config-3 GPT-2 124M random-init (load_random seed 3), prompt 32, 128 greedy tokens, "
            "batch 32 (32 independent sequences)",
    "int4": "config-4 INT4 group-32 sweep K=3584, N in {3584,18944,152064}, M in {1,8,64,512,4096}, f32 activations "
            "(weight-only)",
    "moe": "config-5 MoE: 8192 tokens x d 7168, 256 experts (d_ff 2048, INT8 per-channel) + 1 shared, top-8 over "
           "N(0,1) router logits, grouped W8A8 GEMMs",
    "mla": "config-5 MLA: KV[16384x7168] . down[7168x512] -> latent; latent . up_K/up_V [512x16384], N(0,0.02) weights",
    "flash": "fused attention (flash_attention, blas:589-678, multi-head): [batch*heads] x seq x head_dim = "
             "96 x 2048 x 64 and 32 x 4096 x 128, causal and full, N(0,1) q/k/v, scale 1/sqrt(head_dim)",
}


REF = {
    "qgemm": (cpu_qgemm, Q_METRIC, "TOPS", lambda v: q_ops() / (v * 1e12) * 1e3),
    "qgemm_a8": (cpu_qgemm_a8, "INT8-activation quantized GEMM TOPS (W8A8 / W4A8, M in {1,16,128,2048}, K=768, "
                 "N=3072)", "TOPS", lambda v: q_ops() / (v * 1e12) * 1e3),
    "sgemm": (cpu_sgemm, "sgemm TFLOP/s (f32, 512x768x2304 + bias)", "TFLOP/s",
              lambda v: 2 * S_M * S_K * S_N / (v * 1e12) * 1e3),
    "gpt2": (cpu_gpt2, "GPT-2 124M greedy decode tok/s (batch 32, prompt 32, 128 new tokens)", "tok/s",
             lambda v: 32 * G_NEW / v * 1e3),
    "int4": (cpu_int4, "INT4 g32 GEMM TOPS (K=3584 sweep)", "TOPS", lambda v: i_ops() / (v * 1e12) * 1e3),
    "moe": (cpu_moe, "MoE block TOPS (8192 tokens, 256 experts top-8 + shared, INT8)", "TOPS",
            lambda v: e_ops() / (v * 1e12) * 1e3),
    "mla": (cpu_mla, "MLA compress+decompress TFLOP/s (f32)", "TFLOP/s", lambda v: l_flops() / (v * 1e12) * 1e3),
    "flash": (cpu_flash, F_METRIC, "TFLOP/s", lambda v: sum(f_flops(c) for c in F_CASES) / (v * 1e12) * 1e3),
}


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    fn, metric, unit, ms_of = REF[args.workload]
    vals, last = [], None
    heavy = args.workload in ("gpt2", "moe", "int4", "flash")  # samples of seconds: fewer of them
    n = max(1, min(args.steps, 3)) if heavy else args.steps
    w = min(args.warmup, 3) if heavy else args.warmup
    for i in range(w + n):
        r = fn()
        if i >= w:
            vals.append(r["value"])
            last = r
    v = statistics.median(vals)
    line = {
        "impl": "reference", "metric": metric, "value": v, "unit": unit, "n_gpus": args.gpus,
        "steps": n, "warmup": w, "ms_per_step": ms_of(v), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": DATA,
        "config": {"workload": WORKLOADS[args.workload],
                   "parallelism": f"reference CPU path restated in C, {last['cores']} host threads, rank 0"},
        "cpu_baseline": {"value": v, "unit": unit, "cores": last["cores"], "kind": last["kind"],
                         "sample": last["sample"]},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    ctx = Ctx(args)
    {"qgemm": run_qgemm, "qgemm_a8": run_qgemm_a8, "sgemm": run_sgemm, "gpt2": run_gpt2, "int4": run_int4, "moe": run_moe,
     "mla": run_mla, "flash": run_flash}[args.workload](ctx)


if __name__ == "__main__":
    main()
