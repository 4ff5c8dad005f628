"""Benchmark of the quantized-linear hot path (one JSON line on stdout).

Workload: FP8 E4M3 W8A16 linears over all seven
Qwen2.5-0.5B projection shapes (K->N: 896->896 q, 896->128 k, 896->128 v,
896->896 o, 896->4864 gate, 896->4864 up, 4864->896 down) at
M in {1, 8, 32, 128, 1024, 8192}: 42 linears per step, each with its own
seeded N(0, 0.02) weight quantised with the reference's per-tensor
absmax/448 scale, bf16 N(0,1) activations. Random init, synthetic data.

  value    TFLOP/s of the whole step (sum 2*M*N*K over the 42 linears / device
           time of one CUDA-graph replay of the step), inputs resident in HBM,
           L2 flushed (256 MiB write) between timed steps.
  e2e      same metric through the public module API (FP8Linear.forward),
           every step copying each x from pinned host memory and each y back.
  roofline dominant kernel = the tcgen05 prefill GEMM (all M > 64 launches),
           timed as its own graph; tensor-bound, vs the measured bf16 peak
           (W8A16 keeps activations in bf16, so bf16 is the parity-preserving
           tensor roofline).
  awq_config0  BASELINE config 0: AWQ W4A16 M=16, K=896, N=9728, cold-L2
           per-linear mean inside a CUDA graph over > 2x L2 of distinct
           weight copies; GB/s vs the measured HBM copy bandwidth.
  decode_large  the same measurement on a large decode layer, Llama-3-8B
           gate 4096 -> 14336 at M = 16 (FP8 and AWQ g128) and AWQ at M = 64
           (config 3's batch): the shapes where the HBM roofline is reachable
           (59 / 31 MB per linear).
  parity   every one of the 42 outputs of the timed graph against an fp32
           product of the bit-exact dequantised weight (max relative
           Frobenius error; the bar is 1e-2). Under torchrun the sharded
           outputs are gathered and checked against the unsharded layer.
  cpu_baseline  the CPU oracle (numpy restatement of the reference path) on
           all of the box's host cores, on the same 42 linears.

--gpus N (under torchrun): tensor parallel over the same sweep, q/k/v/gate/up
column-parallel, o/down row-parallel + NCCL all_reduce; max-over-ranks time;
`tp_breakdown` times the linears alone and the 12 all-reduces alone.
--impl reference: the CPU oracle alone on the same workload (rank 0 only).
--ncu-case NAME: run a few launches of one kernel and exit (no timing, no
JSON), for Nsight Compute captures of a small case (one kernel, <= 4 launches):
  prefill        FP8 gate shape, M=16384 (paired-CTA TMEM-operand GEMM), 3 launches
  down8192       FP8 down 4864->896 at M=8192 (the sweep's paired-kernel launch), 3 launches
  awq0           config-0 AWQ linear (M=16, K=896, N=9728), 4 launches
  awq_llama_gate / fp8_llama_gate   Llama-3-8B gate 4096->14336 at M=16, 3 launches
  sweep_one      sweep linear --ncu-index i (0..41, shape-major, M fastest), 3 launches:
                 one linear per capture for the per-launch DRAM traffic table
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [("q", 896, 896), ("k", 896, 128), ("v", 896, 128), ("o", 896, 896),
          ("gate", 896, 4864), ("up", 896, 4864), ("down", 4864, 896)]  # (name, K, N)
MS = [1, 8, 32, 128, 1024, 8192]
ROW_PARALLEL = {"o", "down"}
PARITY_TOL = 1e-2
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "FP8 W8A16 linear throughput, Qwen2.5-0.5B projection sweep (config 1)"
WORKLOAD = "config1_fp8_sweep_qwen2.5-0.5b_7shapes_x_M{1,8,32,128,1024,8192}"


def sweep_config(world):
    """The workload description both arms print (identical by construction)."""
    return {"workload": WORKLOAD, "linears_per_step": len(SHAPES) * len(MS),
            "weights": "fp8 e4m3, per-tensor scale", "activations": "bf16 N(0,1)", "parallelism": f"tp{world}",
            "l2": "flushed between timed steps (256 MiB write)"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


TRAFFIC_PROFILE = os.path.join(ROOT, "profiles", "traffic_prefill_ts2_kernel_fp8_down_m8192.txt")


def profiled_traffic():
    """DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum) of one launch
    of the sweep's top prefill launch (FP8 down at M = 8192) and its algorithmic
    bytes, from the committed one-kernel capture summary; None if absent."""
    out = {}
    try:
        with open(TRAFFIC_PROFILE) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 2 and parts[0] in ("traffic_bytes_per_launch", "algorithmic_bytes_per_launch"):
                    out[parts[0]] = int(float(parts[1]))
    except OSError:
        return None
    return out or None


def case_bytes_flops(m, k, n, fmt="fp8", gs=128):
    if fmt == "fp8":
        b = n * k + 4 + 2 * m * k + 2 * m * n
    else:
        g = (k + gs - 1) // gs
        b = n * k // 2 + 2 * n * g * 2 + 2 * m * k + 2 * m * n
    return b, 2 * m * n * k


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi, during the timed region)
# ---------------------------------------------------------------------------


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 20 ms from before the
    timed region starts until after it ends; summary() keeps the samples that
    fall inside [t0, t1] (the two nearest ones if the region is shorter than
    the sampling period)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []  # (host time, fields)
        self._proc = None
        self._thread = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self._proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        deadline = time.time() + 5.0
        while not self.samples and time.time() < deadline:
            time.sleep(0.01)

    def _read(self):
        for line in self._proc.stdout:
            parts = [q.strip() for q in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        time.sleep(0.05)
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()

    def summary(self):
        if not self.samples or self.t0 is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        inside = [p for t, p in self.samples if self.t0 <= t <= self.t1]
        note = "inside timed region"
        if not inside:
            near = sorted(self.samples, key=lambda tp: min(abs(tp[0] - self.t0), abs(tp[0] - self.t1)))[:2]
            inside = [p for _, p in near]
            note = "timed region shorter than the 20 ms sampling period: nearest samples"
        sm, mx, pw = [], [], []
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for p in inside:
            try:
                sm.append(float(p[1]))
                mx.append(float(p[2]))
                pw.append(float(p[3]))
            except ValueError:
                continue
            for name, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "reasons": sorted(reasons), "samples": len(sm),
                "note": note}


# ---------------------------------------------------------------------------
# CPU oracle leg (also the --impl reference arm)
# ---------------------------------------------------------------------------


def cpu_sample_cases(seed=0):
    """The same 42 linears as the GPU step (full M, up to 8192 rows)."""
    from oracle import nsq_oracle as O
    rng = np.random.default_rng(seed)
    cases = []
    for name, k, n in SHAPES:
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        codes, scale = O.fp8_quantize(w)
        for m in MS:
            x = O.bf16_round(rng.standard_normal((m, k)).astype(np.float32))
            cases.append((codes, scale, x, 2 * m * n * k))
    return cases


def cpu_oracle_step(cases):
    from oracle import nsq_oracle as O
    for codes, scale, x, _ in cases:
        O.fp8_linear(x, codes, scale)


def host_cores():
    return len(os.sched_getaffinity(0))


def run_cpu_baseline(steps, warmup):
    """The oracle on every host core the process may use (threadpoolctl sets
    the BLAS pool explicitly: under torchrun it would otherwise start at 1)."""
    from threadpoolctl import threadpool_limits
    cores = host_cores()
    with threadpool_limits(limits=cores):
        cases = cpu_sample_cases()
        flops = sum(c[3] for c in cases)
        for _ in range(warmup):
            cpu_oracle_step(cases)
        t = []
        for _ in range(steps):
            t0 = time.perf_counter()
            cpu_oracle_step(cases)
            t.append(time.perf_counter() - t0)
    sec = statistics.median(t)
    return {"value": flops / sec / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"all 42 sweep linears at full M ({flops / 1e9:.1f} GFLOP, the GPU step's work), "
                      f"numpy fp32 dequant+matmul, median of {steps}",
            "same_config": True, "ms_per_step": sec * 1e3}


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------


def build_gpu_cases(torch, ops, device, rank, world):
    """Per-rank shards of the 42 sweep linears (TP over `world` ranks)."""
    cases = []
    g = torch.Generator(device="cpu")
    for si, (name, k, n) in enumerate(SHAPES):
        for mi, m in enumerate(MS):
            g.manual_seed(1000 * si + mi)
            w = (torch.randn(n, k, generator=g) * 0.02).to(device)
            codes, scale, _ = ops.fp8_quantize(w)  # per-tensor scale over the FULL weight
            row = name in ROW_PARALLEL and world > 1
            if world > 1:
                if row:
                    c0, c1 = rank * k // world, (rank + 1) * k // world
                    codes = codes[:, c0:c1].contiguous()
                else:
                    r0, r1 = rank * n // world, (rank + 1) * n // world
                    codes = codes[r0:r1].contiguous()
            ks = codes.shape[1]
            ns = codes.shape[0]
            x = torch.randn(m, ks, generator=g).to(torch.bfloat16).to(device)
            case = {"name": name, "m": m, "k": k, "n": n, "ks": ks, "ns": ns, "codes": codes,
                    "scale": scale, "x": x, "row": row}
            if row:
                # the product's row-parallel layer: local GEMM + all_reduce, chunked
                # and overlapped on a side stream from 2048 tokens on
                from nanosglang_b200.quantization import FP8Linear
                from nanosglang_b200.tensor_parallel import RowParallelLinear
                with torch.device(device):
                    shard = FP8Linear(ks, ns)
                shard.weight_fp8 = codes
                shard.weight_scale = scale
                case["rp"] = RowParallelLinear(k, n, world, rank, linear=shard)
            cases.append(case)
            del w
    return cases


def run_ours(args):
    import torch
    import torch.distributed as dist

    from nanosglang_b200 import _lib, ops
    from nanosglang_b200.quantization import AWQLinear, FP8Linear

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    _lib.load()
    _lib.device_status_reset()
    # weights are written once during set-up and never inside the timed work,
    # so the linears may start streaming them before the previous kernel ends
    _lib.set_pdl(not args.no_pdl)
    peaks, peak_src = load_peaks()

    if args.tp_overlap > 0:
        from nanosglang_b200.tensor_parallel import RowParallelLinear
        RowParallelLinear.overlap_min_tokens = args.tp_overlap
    cases = build_gpu_cases(torch, ops, device, rank, world)
    for c in cases:
        c["y"] = torch.empty(c["m"], c["ns"], dtype=torch.bfloat16, device=device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device)

    def one_linear(c):
        if c["row"]:
            out = c["rp"](c["x"])
        else:
            out = ops.fp8_linear(c["x"], c["codes"], c["scale"])
        c["y"] = out
        return out

    def capture(selected):
        # warm up on the capture stream, then record one graph of the selection
        with torch.cuda.stream(stream):
            for _ in range(2):
                for c in selected:
                    one_linear(c)
        torch.cuda.synchronize()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=stream):
            for c in selected:
                one_linear(c)
        torch.cuda.synchronize()
        return gph

    def time_graph(gph, steps, warmup, sampler=None):
        for _ in range(warmup):
            flush.zero_()
            gph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        if sampler:
            sampler.mark("t0")
        cur = torch.cuda.current_stream()
        for s, e in evs:
            flush.zero_()
            s.record(cur)
            gph.replay()
            e.record(cur)
        torch.cuda.synchronize()
        if sampler:
            sampler.mark("t1")
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ms = sum(s.elapsed_time(e) for s, e in evs)
        if world > 1:
            t = torch.tensor([ms], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms / steps

    # --- headline: whole step as one graph ---------------------------------
    g_all = capture(cases)
    sampler = ClockSampler(local)
    sampler.start()
    ms_step = time_graph(g_all, args.steps, args.warmup, sampler)
    sampler.stop()
    flops_total = sum(2 * c["m"] * c["n"] * c["k"] for c in cases)  # full (unsharded) sweep work
    value = flops_total / (ms_step * 1e-3) / 1e12
    # the timed graph's own outputs (last replay) against the unsharded layer
    parity = check_parity(torch, dist, ops, cases, rank, world, device)
    tp_breakdown = None
    if world > 1:
        tp_breakdown = time_tp_breakdown(cases, capture, time_graph, args, ms_step)

    # --- dominant kernel: all prefill-GEMM launches (M > 64) as one graph ---
    pre = [c for c in cases if c["m"] > 64]
    if world > 1:
        # time the kernel launches alone (no collective) for the roofline
        pre_k = [dict(c, row=False) for c in pre]
    else:
        pre_k = pre
    g_pre = capture(pre_k)
    ms_pre = time_graph(g_pre, args.steps, args.warmup)
    flops_pre = sum(2 * c["m"] * c["ns"] * c["ks"] for c in pre_k)
    bf16_peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    ach = flops_pre / (ms_pre * 1e-3) / 1e12
    roofline = {"kernel": "prefill GEMMs (tcgen05 kind::f16; dequantised weight as the TMEM operand: paired-CTA and one-CTA; split-K cluster)",
                "bound": "tensor", "achieved": round(ach, 2), "peak": bf16_peak, "unit": "TFLOP/s",
                "frac": round(ach / bf16_peak, 4), "peak_source": f"{peak_src} bf16 dense (burst)",
                "launches_per_step": len(pre_k)}
    tr = profiled_traffic() if world == 1 else None
    roofline.update({
        "traffic": tr.get("traffic_bytes_per_launch") if tr else None,
        "traffic_algorithmic_bytes": tr.get("algorithmic_bytes_per_launch") if tr else None,
        "traffic_case": "one launch of the sweep's top prefill linear (FP8 down 4864->896, M=8192), "
                        "ncu dram__bytes_read.sum + dram__bytes_write.sum, one-kernel capture"})
    # decode kernel (M <= 64) class, for context
    dec = [dict(c, row=False) for c in cases if c["m"] <= 64]
    g_dec = capture(dec)
    ms_dec = time_graph(g_dec, args.steps, args.warmup)
    bytes_dec = sum(case_bytes_flops(c["m"], c["ks"], c["ns"])[0] for c in dec)
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    decode_line = {"kernel": "decode kernels (mma.sync swap-AB: single-wave / multi-wave / weight ring, by shape)",
                   "bound": "hbm", "achieved": round(bytes_dec / (ms_dec * 1e-3) / 1e9, 1),
                   "peak": hbm_peak, "unit": "GB/s",
                   "frac": round(bytes_dec / (ms_dec * 1e-3) / 1e9 / hbm_peak, 4),
                   "launches_per_step": len(dec), "us_per_launch": round(ms_dec * 1e3 / len(dec), 2),
                   "algorithmic_bytes_per_launch": int(bytes_dec / len(dec))}
    del g_all, g_pre, g_dec

    # --- e2e through the module API with host buffers -----------------------
    mods = []
    for c in cases:
        mod = FP8Linear(c["ks"], c["ns"]).to(device)
        mod.weight_fp8 = c["codes"]
        mod.weight_scale = c["scale"]
        xh = c["x"].cpu().pin_memory()
        yh = torch.empty(c["m"], c["ns"], dtype=torch.bfloat16).pin_memory()
        mods.append((mod, xh, yh, c))
    h2d = sum(m[1].numel() * 2 for m in mods)
    d2h = sum(m[2].numel() * 2 for m in mods)

    # x uploads on one copy stream, the linears on the compute stream, y
    # downloads on another copy stream (ordered by events), so that the two
    # PCIe directions run at once and overlap the kernels
    compute = torch.cuda.current_stream(device)
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def e2e_step():
        copy_in.wait_stream(compute)
        ins = []
        with torch.cuda.stream(copy_in):
            for mod, xh, yh, c in mods:
                xd = xh.to(device, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_in)
                ins.append((xd, ev))
        for (xd, ev), (mod, xh, yh, c) in zip(ins, mods):
            compute.wait_event(ev)
            xd.record_stream(compute)
            y = mod(xd)
            if c["row"]:
                dist.all_reduce(y)
            done = torch.cuda.Event()
            done.record(compute)
            copy_out.wait_event(done)
            with torch.cuda.stream(copy_out):
                yh.copy_(y, non_blocking=True)
            y.record_stream(copy_out)
        compute.wait_stream(copy_out)  # the step ends when its last result is on the host

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(3, min(args.steps, 10))
    s.record(compute)
    for _ in range(n_e2e):
        e2e_step()
    e.record(compute)
    torch.cuda.synchronize()
    ms_e2e = s.elapsed_time(e) / n_e2e
    if world > 1:
        t = torch.tensor([ms_e2e], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = {"value": round(flops_total / (ms_e2e * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(ms_e2e, 3),
           "steps": n_e2e}
    del mods

    # --- config 0: AWQ W4A16 decode linear, cold L2 -------------------------
    awq = None
    dec_large = None
    if world == 1:
        awq = bench_awq_config0(torch, ops, device, args, peaks, peak_src, flush)
        dec_large = bench_decode_large(torch, ops, device, args, peaks, peak_src, flush)

    # --- model level: configs 2 and 3 (tok/s) -------------------------------
    tok_s = None
    if not args.no_model:
        tok_s = {"config2": bench_config2_tok_s(torch, dist, device, rank, world, args),
                 "config3": bench_config3_tok_s(torch, dist, device, rank, world, args),
                 "config4": bench_config4_tok_s(torch, dist, device, rank, world, args)}

    host = measure_host_overhead(torch, ops, device) if world == 1 else None

    code, where, block = _lib.device_status()
    if code != 0:
        raise RuntimeError(f"device status {code} (tag {where}, block {block})")

    out = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu = run_cpu_baseline(steps=3, warmup=1)
        clocks = sampler.summary()
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": sweep_config(world),
            "roofline": roofline, "decode_kernel": decode_line, "awq_config0": awq, "decode_large": dec_large,
            "cpu_baseline": cpu,
            "e2e": e2e, "gpu_launches": len(cases) * args.steps, "clocks": clocks, "parity": parity,
            "tok_s": tok_s, "host_overhead": host,
        }
        if tp_breakdown is not None:
            out["tp_breakdown"] = tp_breakdown
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


def measure_host_overhead(torch, ops, device):
    """Host time of one eager FP8Linear.forward call (validation, tensor-map
    encoding, launch; no synchronisation), per path: what an eager prefill pays
    per linear outside a CUDA graph. Device work of the calls overlaps."""
    out = {}
    g = torch.Generator().manual_seed(5)
    for name, m, k, n in (("decode M=8 896->4864", 8, 896, 4864), ("prefill M=1024 896->4864", 1024, 896, 4864)):
        codes, scale, _ = ops.fp8_quantize((torch.randn(n, k, generator=g) * 0.02).to(device))
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(device)
        for _ in range(20):
            ops.fp8_linear(x, codes, scale)
        torch.cuda.synchronize()
        reps = 200
        t0 = time.perf_counter()
        for _ in range(reps):
            ops.fp8_linear(x, codes, scale)
        t1 = time.perf_counter()
        torch.cuda.synchronize()
        out[name] = round((t1 - t0) * 1e6 / reps, 2)
    return {"us_per_call": out, "note": "host time per eager ops.fp8_linear call (Python wrapper + C ABI + "
                                        "tensor-map encoding + launch), device not synchronised"}


def check_parity(torch, dist, ops, cases, rank, world, device):
    """Max relative Frobenius error of the step's outputs against an fp32 product
    of the bit-exact dequantised weight (quantization.py:49-52). Under TP the
    shards of x, the weight codes and y are gathered first (column-parallel y
    along N; row-parallel y is already summed by the all-reduce), and rank 0
    checks them against the unsharded layer."""
    def gather(t, dim):
        if world == 1:
            return t
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        return torch.cat(parts, dim=dim)

    worst, worst_name = 0.0, None
    one = torch.ones((), device=device)
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for c in cases:
            codes8 = c["codes"].view(torch.uint8)
            if c["row"]:
                x, codes, y = gather(c["x"], 1), gather(codes8, 1), c["y"]
            else:
                x, codes, y = c["x"], gather(codes8, 0), gather(c["y"], 1)
            if rank != 0:
                continue
            w = ops.fp8_dequant(codes.view(torch.float8_e4m3fn), one, torch.float16).float() * c["scale"]
            ref = x.float() @ w.T
            err = ((y.float() - ref).norm() / ref.norm()).item()
            if err > worst:
                worst, worst_name = err, f'{c["name"]} M={c["m"]}'
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    if rank != 0:
        return None
    return {"max_rel_fro": float(f"{worst:.3e}"), "worst_case": worst_name, "cases": len(cases),
            "tol": PARITY_TOL, "pass": worst <= PARITY_TOL,
            "reference": "fp32 product of the bit-exact dequantised weight (TF32 off)"
                         + (", TP shards gathered to the unsharded layer" if world > 1 else "")}


def time_tp_breakdown(cases, capture, time_graph, args, ms_step):
    """Where a TP step's time goes: the 42 linears alone (no collective) and
    the 12 row-parallel all-reduces alone, each as its own graph."""
    import torch.distributed as dist
    lin = [dict(c, row=False) for c in cases]
    g_lin = capture(lin)
    ms_lin = time_graph(g_lin, args.steps, args.warmup)
    del g_lin
    rows = [c for c in cases if c["row"]]
    import torch
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for c in rows:
            dist.all_reduce(c["y"])
    torch.cuda.synchronize()
    g_ar = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_ar, stream=stream):
        for c in rows:
            dist.all_reduce(c["y"])
    torch.cuda.synchronize()
    ms_ar = time_graph(g_ar, args.steps, args.warmup)
    del g_ar
    return {"step_ms": round(ms_step, 4), "linears_only_ms": round(ms_lin, 4), "allreduce_only_ms": round(ms_ar, 4),
            "allreduces_per_step": len(rows),
            "allreduce_bytes_per_step": int(sum(c["y"].numel() * 2 for c in rows))}


def bench_config2_tok_s(torch, dist, device, rank, world, args):
    """Qwen2.5-0.5B, AWQ int4 on every projection (config-0
    distributions, random init), 32 requests, prompts U[100, 512], outputs
    U[64, 128], greedy, all requests admitted at once; output tokens / wall
    clock through the harness engine (packed prefill + CUDA-graph decode
    steps), prompts up from pinned host memory and tokens back inside the
    timed region. At N GPUs: N independent replicas (the 14 query / 2 KV
    heads do not shard 4 or 8 ways), each serving its own 32-request workload,
    tokens summed, time = the slowest replica."""
    from harness import engine as E
    from harness import model as H
    cfg = H.QWEN2_5_0_5B
    model = H.build_model(cfg, device=device, dtype=torch.bfloat16)
    H.quantize_projections_awq(model)
    H.init_awq(model, 2)
    H.fuse_projections(model)  # q/k/v and gate/up+SiLU as one launch each at decode batch sizes
    # every replica serves the whole 32-request workload (its own seed): the
    # per-GPU batch stays the configuration's, so N replicas serve N x the work
    ps, os_ = E.make_workload(32, 100, 512, 64, 128, cfg.vocab_size, seed=rank)
    eng = E.DecodeEngine(model, max_slots=len(ps), max_len=512 + 128 + 8, max_steps=128)
    eng.capture()
    step_ms = E.time_decode_step(eng, len(ps))
    E.run_workload(eng, ps, os_)  # warm-up (allocator, prefill shapes)
    runs = []
    for _ in range(3):
        if world > 1:
            dist.barrier()
        _, info = E.run_workload(eng, ps, os_)
        el = info["elapsed_s"]
        if world > 1:
            t = torch.tensor([el], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el = float(t.item())
        runs.append(el)
    el = statistics.median(runs)
    total_out = sum(os_)
    if world > 1:
        t = torch.tensor([total_out], device=device, dtype=torch.float64)
        dist.all_reduce(t)
        total_out = int(t.item())
    del eng, model
    torch.cuda.empty_cache()
    return {"workload": "config 2: Qwen2.5-0.5B AWQ int4 (all projections), 32 requests, prompt U[100,512], "
                        "output U[64,128], greedy, bf16 activations", "tok_s": round(total_out / el, 1),
            "unit": "output tokens/s (wall clock)", "elapsed_s": round(el, 4), "output_tokens": total_out,
            "prompt_tokens_per_replica": sum(len(p) for p in ps), "replicas": world, "scaling": "weak",
            "decode_step_ms": round(step_ms, 4), "decode_step_batch": len(ps),
            "method": "packed prefill + one CUDA-graph replay per decode step (harness engine), fused q/k/v and "
                      "gate/up+SiLU launches at decode batch sizes; median of 3 runs after one warm-up"}


def bench_config4_tok_s(torch, dist, device, rank, world, args):
    """Qwen2.5-72B-shaped decoder, FP8 E4M3 on every
    projection (random codes, built without dense projections), tensor
    parallel over the N ranks: one prefill chunk of 8192 tokens (one
    sequence, causal attention) and decode steps at a batch of 128 (context
    2048, random cache), both timed on the device, max over ranks. Runs at
    TP >= 2 (72 GB of weights plus the batch-128 cache exceed one GPU)."""
    if world < 2:
        return {"workload": "config 4: Qwen2.5-72B FP8", "skipped": "runs at TP 2/4/8 (72 GB of FP8 weights and a "
                "44 GB batch-128 cache per 2 GPUs)"}
    from harness import engine as E
    from harness import model as H
    from nanosglang_b200 import tensor_parallel as TP
    cfg = H.QWEN2_5_72B
    prompt, batch, ctx, steps = 8192, 128, 2048, 8
    model = H.build_model_fp8(cfg, device=device, seed=7)
    TP.tensor_parallel_model(model, world, rank)
    torch.cuda.empty_cache()
    wbytes = sum(b.numel() * b.element_size() for n, b in model.named_buffers() if n.endswith("weight_fp8"))
    hd = cfg.head_dim
    proj_params = cfg.num_hidden_layers * cfg.hidden_size * (
        2 * cfg.num_attention_heads * hd + 2 * cfg.num_key_value_heads * hd + 3 * cfg.intermediate_size)
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def max_over_ranks(ms):
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # prefill: one 8192-token chunk into a one-slot cache
    eng = E.DecodeEngine(model, max_slots=1, max_len=prompt + 8, max_steps=4)
    g = torch.Generator(device=device).manual_seed(17)  # the same prompt on every rank
    toks = torch.randint(0, cfg.vocab_size, (prompt,), generator=g, device=device)
    eng.prefill([toks])
    torch.cuda.synchronize()
    dist.barrier()
    reps = 2
    s_ev.record()
    for _ in range(reps):
        eng.prefill([toks])
    e_ev.record()
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(s_ev.elapsed_time(e_ev) / reps)
    del eng
    torch.cuda.empty_cache()
    # decode: batch 128 at context 2048, one CUDA-graph replay per step
    eng = E.DecodeEngine(model, max_slots=batch, max_len=ctx + steps + 8, max_steps=steps + 4)
    gk = torch.Generator(device=device).manual_seed(19 + rank)
    for kc, vc in eng.caches:
        kc.normal_(generator=gk)
        vc.normal_(generator=gk)
    eng.capture([batch])
    eng.tokens.copy_(torch.randint(0, cfg.vocab_size, (batch,), generator=g, device=device))
    gph = eng.graphs[batch]

    def run(n):
        eng.positions.fill_(ctx)
        eng.step.zero_()
        for _ in range(n):
            gph.replay()

    run(2)
    torch.cuda.synchronize()
    dist.barrier()
    eng.positions.fill_(ctx)
    eng.step.zero_()
    s_ev.record()
    for _ in range(steps):
        gph.replay()
    e_ev.record()
    torch.cuda.synchronize()
    decode_ms = max_over_ranks(s_ev.elapsed_time(e_ev) / steps)
    del gph, eng, model
    torch.cuda.empty_cache()
    return {"workload": "config 4: Qwen2.5-72B FP8 E4M3 (all projections), prefill chunk of 8192 tokens + decode "
                        "batch of 128 at context 2048, bf16 activations",
            "tp": world, "fp8_weight_bytes_per_rank": int(wbytes),
            "prefill_ms": round(prefill_ms, 2), "prefill_tok_s": round(prompt / (prefill_ms * 1e-3), 1),
            "prefill_tflops": round(2.0 * prompt * proj_params / world / (prefill_ms * 1e-3) / 1e12, 1),
            "decode_step_ms": round(decode_ms, 3), "decode_tok_s": round(batch / (decode_ms * 1e-3), 1),
            "method": "harness engine: packed prefill (SDPA causal) timed twice after one warm-up; decode-step graph "
                      "replayed 8 times; device time, max over ranks; prefill_tflops = the projections' 2 M N K per "
                      "rank over the whole prefill time (attention, norms and all-reduces included)"}


def bench_config3_tok_s(torch, dist, device, rank, world, args):
    """Llama-3-8B-shaped decoder, AWQ int4 on every
    projection (random init), 64 decode streams at context 2048, tensor
    parallel over the N ranks (q/k/v/gate/up column-parallel, o/down
    row-parallel + NCCL all-reduce, inside the captured decode graph).
    The caches hold 2048 positions of random keys/values (the prefill is not
    part of this figure); tok/s = 64 x steps / device time of the steps,
    max over ranks."""
    from harness import engine as E
    from harness import model as H
    from nanosglang_b200 import tensor_parallel as TP
    cfg = H.LLAMA3_8B
    streams, ctx, steps = 64, 2048, 16
    model = H.build_model(cfg, device=device, dtype=torch.bfloat16)
    H.quantize_projections_awq(model)
    H.init_awq(model, 3)
    peer = False
    if world > 1:
        TP.tensor_parallel_model(model, world, rank)
        if args.peer_allreduce:
            TP.enable_peer_allreduce(4 << 20)  # the step's [64, 4096] bf16 outputs (512 KB) go over NVLink peers
            peer = True
    H.fuse_projections(model)  # fused launches apply to M <= 32 only; 64 streams keep the separate layers
    eng = E.DecodeEngine(model, max_slots=streams, max_len=ctx + steps + 8, max_steps=steps + 4)
    g = torch.Generator(device=device).manual_seed(4 + rank)
    for kc, vc in eng.caches:
        kc.normal_(generator=g)
        vc.normal_(generator=g)
    eng.capture([streams])
    eng.tokens.copy_(torch.randint(0, cfg.vocab_size, (streams,), generator=g, device=device))
    gph = eng.graphs[streams]

    def run(n):
        eng.positions.fill_(ctx)
        eng.step.zero_()
        for _ in range(n):
            gph.replay()

    run(3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    eng.positions.fill_(ctx)
    eng.step.zero_()
    s_ev.record()
    for _ in range(steps):
        gph.replay()
    e_ev.record()
    torch.cuda.synchronize()
    ms = s_ev.elapsed_time(e_ev) / steps
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    wbytes = sum(b.numel() * b.element_size() for n, b in model.named_buffers()
                 if n.endswith(("qweight", "scales", "zeros")))
    ar_ms = None
    if world > 1:
        # the step's 2 x 32 row-parallel all-reduces of [64, 4096] bf16 alone, as one graph
        bufs = [torch.zeros(streams, cfg.hidden_size, device=device, dtype=torch.bfloat16)
                for _ in range(2 * cfg.num_hidden_layers)]
        s2 = torch.cuda.Stream(device)
        with torch.cuda.stream(s2):
            for b in bufs:
                TP._all_reduce_sum(b)
        torch.cuda.synchronize()
        g_ar = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_ar, stream=s2):
            for b in bufs:
                TP._all_reduce_sum(b)
        for _ in range(3):
            g_ar.replay()
        torch.cuda.synchronize()
        dist.barrier()
        s_ev.record()
        for _ in range(steps):
            g_ar.replay()
        e_ev.record()
        torch.cuda.synchronize()
        ar_ms = s_ev.elapsed_time(e_ev) / steps
        t = torch.tensor([ar_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ar_ms = float(t.item())
        del g_ar, bufs
    del gph, eng, model
    if peer:
        torch.cuda.synchronize()
        TP.disable_peer_allreduce()
    torch.cuda.empty_cache()
    return {"workload": "config 3: Llama-3-8B AWQ int4, 64 streams at context 2048, bf16 activations",
            "tok_s": round(streams / (ms * 1e-3), 1), "unit": "tokens/s (device time of decode steps)",
            "ms_per_step": round(ms, 4), "tp": world, "awq_weight_bytes_per_rank": int(wbytes),
            "allreduce_ms_per_step": None if ar_ms is None else round(ar_ms, 4),
            "allreduce_share": None if ar_ms is None else round(ar_ms / ms, 3),
            "allreduce": ("one-shot NVLink peer all-reduce (nsq_peer_allreduce)" if peer else "NCCL")
            if world > 1 else None,
            "method": f"{steps} replays of the batch-64 decode-step graph, max over ranks"}


def bench_decode_large(torch, ops, device, args, peaks, peak_src, flush):
    """Llama-3-8B gate (K=4096 -> N=14336) at M=16, FP8 and AWQ g128, and AWQ at
    M=64 (config 3's decode batch): per-linear mean inside one CUDA graph over
    > 2x L2 of distinct weight copies, through ops (which pass the x-term
    workspace)."""
    k, n, gs = 4096, 14336, 128
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    out = {}
    for key, fmt, m in (("fp8", "fp8", 16), ("awq", "awq", 16), ("awq_m64", "awq", 64)):
        b, f = case_bytes_flops(m, k, n, fmt, gs)
        wbytes = n * k if fmt == "fp8" else n * k // 2
        copies = max(4, math.ceil(2 * l2 / wbytes))
        g = torch.Generator(device=device).manual_seed(11)
        ws = []
        for _ in range(copies):
            if fmt == "fp8":
                codes = torch.randint(0, 126, (n, k), generator=g, device=device, dtype=torch.int16).to(torch.uint8)
                sign = torch.randint(0, 2, (n, k), generator=g, device=device, dtype=torch.int16).to(torch.uint8) << 7
                ws.append(((codes | sign).view(torch.float8_e4m3fn), torch.tensor([0.0003], device=device)))
            else:
                qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), generator=g, device=device,
                                   dtype=torch.int64).to(torch.int32)
                sc = (torch.rand(n, k // gs, generator=g, device=device) * 0.009 + 0.001).half()
                z = torch.randint(0, 16, (n, k // gs), generator=g, device=device).half()
                ws.append((qw, sc, z))
        x = torch.randn(m, k, generator=g, device=device).to(torch.bfloat16)

        def body():
            for w in ws:
                if fmt == "fp8":
                    ops.fp8_linear(x, w[0], w[1])
                else:
                    ops.awq_linear(x, w[0], w[1], w[2], gs)
        stream = torch.cuda.Stream(device)
        with torch.cuda.stream(stream):
            body()
            body()
        torch.cuda.synchronize()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=stream):
            body()
        for _ in range(3):
            gph.replay()
        torch.cuda.synchronize()
        reps = max(3, args.steps // 2)
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tot = 0.0
        for _ in range(reps):
            flush.zero_()
            s_ev.record()
            gph.replay()
            e_ev.record()
            torch.cuda.synchronize()
            tot += s_ev.elapsed_time(e_ev)
        us = tot * 1e3 / (reps * copies)
        gbs = b / (us * 1e-6) / 1e9
        out[key] = {"workload": f"{fmt.upper()} M={m} K={k} N={n}" + (" g128" if fmt == "awq" else ""),
                    "bytes_per_linear": b, "us_per_linear": round(us, 3), "achieved_gbs": round(gbs, 1),
                    "frac": round(gbs / hbm, 4), "copies_in_graph": copies}
        del gph, ws
    out["peak_gbs"] = hbm
    out["peak_source"] = f"{peak_src} HBM copy"
    out["kernels"] = ("x-term kernel + tcgen05 decode kernel: FP8 kind::f8f6f4 with A from the TMA-staged tile; "
                      "AWQ kind::i8 with the nibbles widened into tensor memory")
    out["method"] = "cold-L2 per-linear mean inside one CUDA graph, PDL"
    return out


def bench_awq_config0(torch, ops, device, args, peaks, peak_src, flush):
    """x [16, 896] bf16, K=896 -> N=9728, group 128; per-linear
    mean over > 2x L2 of distinct weight copies replayed in one CUDA graph."""
    m, k, n, gs = 16, 896, 9728, 128
    b, f = case_bytes_flops(m, k, n, "awq", gs)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    copies = max(8, math.ceil(2 * l2 / (n * k // 2)))
    g = torch.Generator().manual_seed(0)
    ws = []
    for _ in range(copies):
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), generator=g, dtype=torch.int64).to(torch.int32)
        s = (torch.rand(n, k // gs, generator=g) * 0.009 + 0.001).half()
        z = torch.randint(0, 16, (n, k // gs), generator=g).half()
        ws.append(tuple(t.to(device) for t in (qw, s, z)))
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(device)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(2):
            for qw, s, z in ws:
                ops.awq_linear(x, qw, s, z, gs)
    torch.cuda.synchronize()
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph, stream=stream):
        for qw, s, z in ws:
            ops.awq_linear(x, qw, s, z, gs)
    for _ in range(3):
        gph.replay()
    torch.cuda.synchronize()
    reps = max(3, args.steps // 2)
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tot = 0.0
    for _ in range(reps):
        flush.zero_()
        s_ev.record()
        gph.replay()
        e_ev.record()
        torch.cuda.synchronize()
        tot += s_ev.elapsed_time(e_ev)
    us = tot * 1e3 / (reps * copies)
    gbs = b / (us * 1e-6) / 1e9
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    return {"workload": "AWQ W4A16 M=16 K=896 N=9728 g128 (config 0)", "bytes_per_linear": b,
            "us_per_linear": round(us, 3), "achieved_gbs": round(gbs, 1), "peak_gbs": hbm,
            "frac": round(gbs / hbm, 4), "peak_source": f"{peak_src} HBM copy",
            "tflops": round(f / (us * 1e-6) / 1e12, 2), "copies_in_graph": copies,
            "method": "cold-L2 per-linear mean inside one CUDA graph"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    r = run_cpu_baseline(steps=args.steps, warmup=args.warmup)
    return {"metric": METRIC, "value": round(r["value"], 5), "unit": "TFLOP/s", "n_gpus": int(os.environ.get(
        "WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_per_step"], 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": sweep_config(int(os.environ.get("WORLD_SIZE", "1"))),
        "cpu_baseline": {"value": round(r["value"], 5), "unit": "TFLOP/s", "cores": r["cores"], "kind": "port",
                         "sample": r["sample"], "same_config": True},
        "e2e": {"value": round(r["value"], 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_ncu_case(name, index=0):
    """A handful of launches of one kernel class, for an Nsight Compute capture."""
    import torch

    from nanosglang_b200 import _lib, ops
    _lib.load()
    _lib.set_pdl(True)
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    if name == "prefill":
        m, k, n = 16384, 896, 4864
        codes, scale, _ = ops.fp8_quantize((torch.randn(n, k, generator=g) * 0.02).to(dev))
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        for _ in range(3):
            ops.fp8_linear(x, codes, scale)
    elif name == "down8192":
        m, k, n = 8192, 4864, 896
        codes, scale, _ = ops.fp8_quantize((torch.randn(n, k, generator=g) * 0.02).to(dev))
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        for _ in range(3):
            ops.fp8_linear(x, codes, scale)
    elif name in ("awq_llama_gate", "fp8_llama_gate"):
        # Llama-3-8B gate 4096 -> 14336 at M = 16, 3 launches (the decode kernel the library picks)
        m, k, n, gs = 16, 4096, 14336, 128
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        if name == "awq_llama_gate":
            qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), generator=g, dtype=torch.int64).to(torch.int32)
            s = (torch.rand(n, k // gs, generator=g) * 0.009 + 0.001).half()
            z = torch.randint(0, 16, (n, k // gs), generator=g).half()
            qw, s, z = qw.to(dev), s.to(dev), z.to(dev)
            for _ in range(3):
                ops.awq_linear(x, qw, s, z, gs)
        else:
            codes, scale, _ = ops.fp8_quantize((torch.randn(n, k, generator=g) * 0.02).to(dev))
            for _ in range(3):
                ops.fp8_linear(x, codes, scale)
    elif name == "sweep_one":
        _, k, n = SHAPES[index // len(MS)]
        m = MS[index % len(MS)]
        codes, scale, _ = ops.fp8_quantize((torch.randn(n, k, generator=g) * 0.02).to(dev))
        x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
        for _ in range(3):
            ops.fp8_linear(x, codes, scale)
    elif name == "awq0":
        m, k, n, gs = 16, 896, 9728, 128
        for _ in range(4):
            qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), generator=g, dtype=torch.int64).to(torch.int32)
            s = (torch.rand(n, k // gs, generator=g) * 0.009 + 0.001).half()
            z = torch.randint(0, 16, (n, k // gs), generator=g).half()
            x = torch.randn(m, k, generator=g).to(torch.bfloat16)
            ops.awq_linear(x.to(dev), qw.to(dev), s.to(dev), z.to(dev), gs)
    else:
        raise SystemExit(f"unknown --ncu-case {name}")
    torch.cuda.synchronize()
    code, where, block = _lib.device_status()
    if code != 0:
        raise RuntimeError(f"device status {code} (tag {where}, block {block})")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU oracle leg")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--no-model", action="store_true", help="skip the model-level tok/s legs (configs 2 and 3)")
    ap.add_argument("--peer-allreduce", action="store_true",
                    help="config 3 under TP: reduce the row-parallel outputs with the NVLink peer all-reduce")
    ap.add_argument("--tp-overlap", type=int, default=0, metavar="TOKENS",
                    help="row-parallel layers overlap chunked GEMMs with their all-reduces from this many tokens "
                         "(0: off, the default)")
    ap.add_argument("--ncu-case", choices=["prefill", "down8192", "awq0", "awq_llama_gate", "fp8_llama_gate",
                                           "sweep_one"],
                    default=None,
                    help="run a small case of one kernel class for a profiler capture, then exit")
    ap.add_argument("--ncu-index", type=int, default=0, help="sweep_one: which of the 42 sweep linears (0..41)")
    args = ap.parse_args()
    if args.ncu_case:
        if not 0 <= args.ncu_index < len(SHAPES) * len(MS):
            raise SystemExit("--ncu-index out of range")
        run_ncu_case(args.ncu_case, args.ncu_index)
        return
    args.warmup = max(3, args.warmup)
    out = run_reference(args) if args.impl == "reference" else run_ours(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
