#!/usr/bin/env python
"""Benchmark of the fused NF4 / fp8 weight-only linear on B200.

One step = one fused quantized linear over one batch of synthetic tokens:
x bf16 [4608, 3072] (one 1024x1024 FLUX image's 4096 latent + 512 text
tokens) times W [12288, 3072] (NF4 by default, the FLUX feed-forward up
projection shape), y bf16 [4608, 12288].  With N GPUs (torchrun, one process
per GPU) every rank runs its own token batch against a replicated weight: data
parallel, no data-path collective, weak scaling; the value is the whole-job
TFLOP/s from the max-over-ranks device time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload nf4|fp8]
    python bench.py --impl reference ...   # the reference's CPU algorithm
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import re
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, N, K = 4608, 12288, 3072
FLOPS_PER_STEP = 2 * M * N * K
ROTATE = 4  # rotating input sets: 4 x (x + W + y) = 650 MB > 126 MB L2
REF_ROW_SLICE = 16  # the CPU reference arm times 1/16 of the weight rows per step

WORKLOADS = {
    "nf4": {
        "desc": "nf4_linear x[4608,3072]bf16 . W[12288,3072]nf4^T (+f32 absmax per 64) -> y[4608,12288]bf16",
        "bytes": M * K * 2 + N * K // 2 + N * K // 64 * 4 + M * N * 2,
    },
    "fp8": {
        "desc": "fp8_linear x[4608,3072]bf16 . W[12288,3072]e4m3^T (per-tensor scale) -> y[4608,12288]bf16",
        "bytes": M * K * 2 + N * K + 4 + M * N * 2,
    },
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["tp_fp8", "flux_dit", "small_nf4", "small_fp8",
                                                           "dequant_nf4", "dequant_fp8"],
                    default="nf4")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-kernels", action="store_true",
                    help="flux_dit: add the per-kernel device-time table of one eager step")
    return ap.parse_args()


# ------------------------------------------------------------------- peaks
def measured_peaks():
    """(burst bf16 TFLOP/s, sustained bf16 TFLOP/s, HBM GB/s, source)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return (float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                float(d["hbm_gbs"]), "measured")
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def profile_traffic(workload: str, plan: dict):
    """DRAM bytes per launch of the planned kernel from its committed ncu summary."""
    kern = "bf16_gemm2" if plan["twophase"] else ("dq_gemm2" if plan["pair"] else "dq_gemm")
    path = os.path.join(ROOT, "profiles", f"{kern}_{workload}_4608x3072x12288.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


# ------------------------------------------------------------------ clocks
REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    """Polls the SM clock and clock-event reasons through NVML while running."""

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            try:
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        nv = self._nvml
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._h is not None:
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if self._h is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml_unavailable"]}
        names = [v for k, v in REASONS.items() if self.reasons & k]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(val: float, world: int, device) -> float:
    if world == 1:
        return val
    import torch.distributed as dist
    t = torch.tensor([val], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_ranks(val: float, world: int, device) -> list:
    if world == 1:
        return [val]
    import torch.distributed as dist
    t = torch.tensor([val], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# --------------------------------------------- the reference's GPU algorithm
NF4_LEVELS = [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
              -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
              0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
              0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
              0.7229568362236023, 1.0]  # R/nf4_ltx23.R:15-21


class RefGpuDequant:
    """The reference's per-forward weight decode, as the libtorch ops it issues
    on the GPU, for timing beside the engine: NF4 per chunk of at most 4 MiB
    packed bytes (R/nf4_ltx23.R:77-115): widen the bytes into an int64
    scratch, gather the bf16 level pairs of the byte table (R/jit_ltx23.R:
    270-281) into the per-shape buffer, multiply each 64-block by its bf16
    absmax; fp8 (R/fp8_ltx23.R:79-80): copy_ (upcast) then mul_ by the bf16
    scale.  The GEMM after it is torch.nn.functional.linear (cuBLAS)."""

    CHUNK_BYTES = 8388608 // 2

    def __init__(self, device):
        pairs = [[NF4_LEVELS[b // 16], NF4_LEVELS[b % 16]] for b in range(256)]
        self.table = torch.tensor(pairs, dtype=torch.bfloat16, device=device)
        self.idx = torch.empty(self.CHUNK_BYTES, dtype=torch.long, device=device)
        self.bufs = {}

    def buffer(self, n, k):
        b = self.bufs.get((n, k))
        if b is None:
            b = self.bufs[(n, k)] = torch.empty(n, k, dtype=torch.bfloat16, device=self.table.device)
        return b

    def nf4(self, packed, absmax, n, k):
        out = self.buffer(n, k)
        pairs, blocks = out.view(-1, 2), out.view(-1, 64)
        am = absmax.to(torch.bfloat16)
        total = packed.numel()
        for s in range(0, total, self.CHUNK_BYTES):
            ln = min(self.CHUNK_BYTES, total - s)
            idx = self.idx[:ln]
            idx.copy_(packed.reshape(-1)[s:s + ln])
            torch.index_select(self.table, 0, idx, out=pairs[s:s + ln])
            b0, nb = 2 * s // 64, 2 * ln // 64
            blocks[b0:b0 + nb].mul_(am.reshape(-1)[b0:b0 + nb].unsqueeze(1))
        return out

    def fp8(self, w8, scale):
        out = self.buffer(*w8.shape)
        out.copy_(w8.view(torch.float8_e4m3fn))
        # the scale is a host scalar tensor (the reference keeps it on the CPU)
        out.mul_(torch.tensor(scale, dtype=torch.float32).to(torch.bfloat16))
        return out


# ----------------------------------------------------------- CPU reference
def cpu_reference_step_fn(workload: str, row_slice: int):
    """The reference's CPU algorithm on 1/row_slice of the weight rows, float32
    (the reference computes in float32 on CPU): per forward, chunked byte-LUT
    dequantization of the NF4 weight (or e4m3 upcast x scale) into a reusable
    buffer, then torch.nn.functional.linear (R/nf4_ltx23.R:235-246,
    R/fp8_ltx23.R:70-83).  Returns (step_fn, flops_per_step, description)."""
    from oracle import torch_ref as T
    n_s = N // row_slice
    g = torch.Generator().manual_seed(0)
    w = torch.randn(n_s, K, generator=g) * 0.02
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(1))
    wbuf = torch.empty(n_s, K, dtype=torch.float32)
    if workload == "nf4":
        packed, absmax = T.ltx23_nf4_quantize(w)

        def step():
            return T.nf4_linear_forward(x, packed, absmax, n_s, K, None, w_buffer=wbuf)
    else:
        w8, scale = T.fp8_quantize(w)

        def step():
            return T.fp8_linear_forward(x, w8, scale, None, w_buffer=wbuf)
    desc = (f"reference CPU op sequence (torch {torch.__version__}, float32) on x[{M},{K}] and "
            f"1/{row_slice} of W ({n_s} of {N} rows) per step")
    return step, 2 * M * n_s * K, desc


def run_cpu_baseline(workload: str, budget_s: float = 12.0):
    step, flops, desc = cpu_reference_step_fn(workload, REF_ROW_SLICE)
    step()
    n = 0
    t0 = time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"value": flops * n / el / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{desc}; {n} steps in {el:.1f} s"}


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    step, flops, desc = cpu_reference_step_fn(args.workload, REF_ROW_SLICE)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    val = flops * args.steps / el / 1e12
    line = {
        "metric": "NF4/fp8 quant-linear TFLOP/s", "value": val, "unit": "TFLOP/s",
        "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOADS[args.workload]["desc"], "format": args.workload,
                   "parallelism": "host cores of rank 0"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": desc},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args, world, rank, local):
    from diffuser_b200 import _lib, modules, ops

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    fmt = args.workload

    # Weights: one seeded fp32 W quantized on the GPU, replicated into ROTATE
    # buffers (distinct addresses, so no launch finds its operands in L2).
    g0 = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(N, K, generator=g0, device=dev) * 0.02
    if fmt == "nf4":
        p0, a0 = ops.ltx23_nf4_quantize(w)
        wsets = [(p0.clone(), a0.clone()) for _ in range(ROTATE)]
        scale = 0.0
    else:
        w80, s0 = ops.fp8_quantize(w)
        wsets = [(w80.view(torch.uint8).clone(), None) for _ in range(ROTATE)]
        scale = float(s0.item())
    del w
    xs, ys = [], []
    for i in range(ROTATE):
        gx = torch.Generator(device=dev).manual_seed(1 + 100 * rank + i)
        xs.append(torch.randn(M, K, generator=gx, device=dev).to(torch.bfloat16))
        ys.append(torch.empty(M, N, dtype=torch.bfloat16, device=dev))
    ws_bytes = ops.workspace_size(M, N, K, 0 if fmt == "nf4" else 1)
    ws = ops.workspace(dev, ws_bytes)
    wsp = ctypes.c_void_p(ws.data_ptr()) if ws is not None else None
    plan0 = ops.plan_info(M, N, K, 0 if fmt == "nf4" else 1)
    # two-phase: one GEMM launch that also decodes the weight (plus a 256-byte
    # memset of its group counters); split-K: GEMM + reduce; else one kernel
    launches_per_step = 2 if plan0["splits"] > 1 else 1

    def launch(i):
        x, y = xs[i % ROTATE], ys[i % ROTATE]
        wp, ap = wsets[i % ROTATE]
        if fmt == "nf4":
            rc = lib.dq_linear_nf4(ctypes.c_void_p(x.data_ptr()), M, K, ctypes.c_void_p(wp.data_ptr()),
                                   ctypes.c_void_p(ap.data_ptr()), None, N, ctypes.c_void_p(y.data_ptr()),
                                   wsp, ws_bytes, sptr)
        else:
            rc = lib.dq_linear_fp8(ctypes.c_void_p(x.data_ptr()), M, K, ctypes.c_void_p(wp.data_ptr()),
                                   ctypes.c_float(scale), None, N, ctypes.c_void_p(y.data_ptr()),
                                   wsp, ws_bytes, sptr)
        if rc != 0:
            raise _lib.DqError("dq_linear", rc)

    for i in range(max(args.warmup, 3)):
        launch(i)
    torch.cuda.synchronize()

    # ---- device-timed region: exactly K steps, events on the launch stream
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            launch(i)
            ev[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    el_ms = t_start.elapsed_time(t_end)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    el_ms_max = max_over_ranks(el_ms, world, dev)
    kern_ms_max = max_over_ranks(kern_ms, world, dev)
    kern_ms_ranks = gather_ranks(kern_ms, world, dev)
    err = ops.device_error(dev)
    if err != 0:
        raise RuntimeError(f"kernel error word {err}")

    # ---- end-to-end through the public module API with host buffers
    e2e = None
    if not args.no_e2e:
        mod = modules.ltx23_nf4_linear(N, K, bias=False) if fmt == "nf4" else \
            modules.ltx23_fp8_linear(N, K, bias=False)
        mod = mod.to(dev)
        if fmt == "nf4":
            mod.set_nf4_weight(wsets[0][0], wsets[0][1])
        else:
            mod.set_fp8_weight(wsets[0][0].view(torch.float8_e4m3fn), torch.tensor(scale))
        # Every step copies its own x in (pinned host -> device) and its whole
        # y back (device -> pinned host).  Copies run on their own streams so
        # step i's download overlaps step i+1's upload and forward, as a
        # caller streaming batches through the module would arrange it.
        xh = [xs[i].cpu().pin_memory() for i in range(2)]
        yh = [torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        xd = [torch.empty(M, K, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        x_free = [torch.cuda.Event() for _ in range(2)]
        y_free = [torch.cuda.Event() for _ in range(2)]
        for e in x_free + y_free:
            e.record(stream)
        n_e2e = max(10, min(args.steps, 200))

        def e2e_step(i):
            bi = i % 2
            s_up.wait_event(x_free[bi])
            with torch.cuda.stream(s_up):
                xd[bi].copy_(xh[bi], non_blocking=True)
                x_ready = torch.cuda.Event()
                x_ready.record(s_up)
            stream.wait_event(x_ready)
            stream.wait_event(y_free[bi])
            y = mod(xd[bi])
            x_free[bi].record(stream)
            y_ready = torch.cuda.Event()
            y_ready.record(stream)
            s_down.wait_event(y_ready)
            with torch.cuda.stream(s_down):
                y.record_stream(s_down)
                yh[bi].copy_(y, non_blocking=True)
                y_free[bi].record(s_down)

        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        a.record(stream)
        s_up.wait_event(a)
        for i in range(n_e2e):
            e2e_step(i)
        done = torch.cuda.Event()
        done.record(s_down)
        stream.wait_event(done)
        b.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        e_ms = max_over_ranks(a.elapsed_time(b), world, dev)
        e2e = {"value": world * FLOPS_PER_STEP * n_e2e / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
               "steps": n_e2e, "ms_per_step": e_ms / n_e2e,
               "api": "diffuser_b200.modules.ltx23_%s_linear.forward" % fmt,
               "copies": "pinned host buffers; upload, forward and download on three streams, "
                         "overlapped across consecutive steps"}

    # ---- the reference's GPU algorithm on the same box, inputs and rotation:
    # decode the weight with its libtorch op sequence into the per-shape
    # buffer, then torch.nn.functional.linear
    ref_gpu = None
    if world == 1:
        rdq = RefGpuDequant(dev)

        def ref_step(i):
            x = xs[i % ROTATE]
            wp, ap = wsets[i % ROTATE]
            wb = rdq.nf4(wp, ap, N, K) if fmt == "nf4" else rdq.fp8(wp, scale)
            return torch.nn.functional.linear(x, wb)

        n_ref = max(10, min(args.steps, 100))
        for i in range(3):
            ref_step(i)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(n_ref):
            ref_step(i)
        b.record(stream)
        torch.cuda.synchronize()
        r_ms = a.elapsed_time(b) / n_ref
        ref_gpu = {"value": FLOPS_PER_STEP / (r_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                   "ms_per_step": r_ms, "steps": n_ref,
                   "algorithm": ("chunked byte-table gather + per-block mul into a bf16 buffer "
                                 "(R/nf4_ltx23.R:77-115), then F.linear (cuBLAS)") if fmt == "nf4"
                   else "copy_ upcast + mul_ by bf16 scale (R/fp8_ltx23.R:79-80), then F.linear (cuBLAS)"}
        del rdq

    if rank == 0:
        burst_tf, sustained_tf, peak_bw, peak_src = measured_peaks()
        clocks = clk.summary()
        # The linear is timed alone (one kernel back to back, ~0.1 s): the
        # burst figure is the denominator; the sustained fraction is reported
        # beside it.
        peak_tf = burst_tf
        peak_kind = "burst"
        achieved = FLOPS_PER_STEP / (kern_ms_max * 1e-3) / 1e12
        plan = ops.plan_info(M, N, K, 0 if fmt == "nf4" else 1)
        traffic = profile_traffic(fmt, plan)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = run_cpu_baseline(fmt)
        line = {
            "metric": "NF4/fp8 quant-linear TFLOP/s",
            "value": world * FLOPS_PER_STEP * args.steps / (el_ms_max * 1e-3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": el_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOADS[fmt]["desc"], "format": fmt, "M": M, "N": N, "K": K,
                       "bias": False, "parallelism": f"dp{world} (own token batch per GPU, replicated weight, no collective)",
                       "l2": f"{ROTATE} rotating input sets ({ROTATE * WORKLOADS[fmt]['bytes'] / 1e6:.0f} MB) > 126 MB L2"},
            # kernel_ms brackets one whole call: with the two-phase plan the
            # counter memset plus the GEMM launch that decodes its weight
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "traffic": traffic,
                         "peak_source": f"{peak_src} bf16 dense, {peak_kind}",
                         "frac_of_burst_peak": achieved / burst_tf,
                         "frac_of_sustained_peak": achieved / sustained_tf,
                         "kernel": (f"bf16_gemm2_kernel<{plan['bm']}, {fmt}> (CTA pair, decodes its "
                                    "weight in-launch), whole call") if plan["twophase"]
                         else f"{plan['kernel']} {fmt} BM={plan['bm']}",
                         "kernel_ms": kern_ms_max,
                         "kernel_ms_per_rank": kern_ms_ranks,
                         "algorithmic_bytes": WORKLOADS[fmt]["bytes"]},
            "cpu_baseline": cpu,
            "reference_gpu_algorithm": ref_gpu,
            "speedup_vs_reference_gpu_algorithm": (
                (world * FLOPS_PER_STEP * args.steps / (el_ms_max * 1e-3) / 1e12) / ref_gpu["value"]
                if ref_gpu else None),
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------- column-parallel
TP_M, TP_N, TP_K = 6144, 12288, 4096  # LTX video tokens x fused q/k/v projection (4096 -> 3 x 4096)


def run_tp(args, world, rank, local):
    """Column-parallel fp8 linear x[6144,4096] . W[12288,4096]^T over `world`
    GPUs: total work fixed (strong scaling).  Each rank's fused kernel writes
    its [M, N/world] block into every rank's y through NVLink peer stores."""
    import torch.distributed as dist
    from diffuser_b200 import ops, tp

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    else:
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29599", rank=0, world_size=1)
    g0 = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(TP_N, TP_K, generator=g0, device=dev) * 0.02
    w8, s0 = ops.fp8_quantize(w)
    del w
    grp = tp.TpGroup(TP_M, TP_N)
    mod = tp.ColumnParallelFp8Linear(TP_K, TP_N, grp, bias=False).to(dev)
    mod.set_fp8_weight(w8, float(s0.item()))
    del w8
    xs = [torch.randn(TP_M, TP_K, generator=torch.Generator(device=dev).manual_seed(1 + i),
                      device=dev).to(torch.bfloat16) for i in range(2)]
    stream = torch.cuda.current_stream(dev)

    def timed(fn, steps):
        for i in range(max(args.warmup, 3)):
            fn(i)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        a.record(stream)
        for i in range(steps):
            fn(i)
        b.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(a.elapsed_time(b) / steps, world, dev)

    with ClockSampler(local) as clk:
        fused_ms = timed(lambda i: mod(xs[i % 2]), args.steps)
    err = ops.device_error(dev)
    nccl_ms = None
    if world > 1:
        nccl_ms = timed(lambda i: mod.forward_nccl(xs[i % 2]), max(10, args.steps // 4))
    grp.close()
    flops = 2 * TP_M * TP_N * TP_K
    peer_bytes = (world - 1) * TP_M * (TP_N // world) * 2  # sent by each rank
    if rank == 0:
        peak_tf, _, _, peak_src = measured_peaks()
        line = {
            "metric": "column-parallel fp8 linear TFLOP/s", "value": flops / (fused_ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": fused_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"fp8_linear x[{TP_M},{TP_K}]bf16 . W[{TP_N},{TP_K}]e4m3^T split over "
                                   f"{world} GPUs by out_features", "parallelism": f"tp{world} column-parallel",
                       "collective": "fused: epilogue peer stores + flag barrier"},
            "per_gpu_tflops": flops / world / (fused_ms * 1e-3) / 1e12,
            "nvlink_gbs_per_gpu": peer_bytes / (fused_ms * 1e-3) / 1e9,
            "compute_bound_ms": flops / world / (peak_tf * 1e12) * 1e3,
            "nccl_allgather_path_ms": nccl_ms,
            "peak_source": f"{peak_src} bf16 dense (burst)",
            "device_error": err, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


# ------------------------------------------------------------ FLUX DiT step
def run_flux(args, world, rank, local):
    """One flow-match Euler step of the FLUX.1 transformer at 1024x1024 (4096
    image + 512 text tokens) with its 494 cast linears in NF4 on the fused
    engine, one image per GPU (latent seed 10 + rank).  Also times the same
    step with the reference's linear algorithm (dequantize each NF4 weight
    into a per-shape bf16 buffer, then cuBLAS) on the same model and box."""
    import torch.distributed as dist
    from diffuser_b200 import flux, modules, ops

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    model = flux.build_flux_nf4(dev, seed=0)
    g = torch.Generator().manual_seed(10 + rank)
    x = flux.pack_latents(torch.randn(1, 16, 128, 128, generator=g)).to(dev, torch.bfloat16)
    g1 = torch.Generator().manual_seed(3)
    text = torch.randn(1, 512, 4096, generator=g1).to(dev, torch.bfloat16)
    pooled = torch.randn(1, 768, generator=g1).to(dev, torch.bfloat16)
    ids = torch.cat([torch.zeros(512, 3), flux.prepare_latent_image_ids(64, 64)], dim=0)
    rope = flux.pos_embed(ids.to(dev), (16, 56, 56))
    t = torch.ones(1, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        with torch.no_grad():
            v = model(x, text, pooled, t, rope)
            return flux.euler_step(v, 1.0, 0.75, x)

    def timed(steps):
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(steps):
            step()
        b.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(a.elapsed_time(b) / steps, world, dev)

    with ClockSampler(local) as clk:
        eager_ms = timed(args.steps)
        # the same step captured once in a CUDA graph and replayed (the engine
        # launches on torch's current stream with cached workspaces, so the
        # whole step captures)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step_out = step()
        graph_steps = lambda: graph.replay()

        def timed_graph(steps):
            for _ in range(3):
                graph_steps()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier(world)
            torch.cuda.synchronize()
            a.record(stream)
            for _ in range(steps):
                graph_steps()
            b.record(stream)
            torch.cuda.synchronize()
            barrier(world)
            return max_over_ranks(a.elapsed_time(b) / steps, world, dev)
        ms = timed_graph(args.steps)
    err = ops.device_error(dev)
    del graph, step_out
    kernels = None
    if args.profile_kernels:
        # one eager step under the torch profiler (outside every timed region)
        torch.cuda.synchronize()
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize()
        ka = prof.key_averages()
        total = sum(e.device_time_total for e in ka)
        kernels = {"total_ms": total / 1e3,
                   "top": [{"kernel": e.key[:120], "launches": e.count, "ms": e.device_time_total / 1e3,
                            "share": e.device_time_total / total}
                           for e in sorted(ka, key=lambda e: -e.device_time_total)[:16]]}
    # The reference's algorithm for every NF4 linear, same weights: its
    # libtorch decode ops into a per-shape bf16 buffer, then cuBLAS; and, for
    # context, the engine's standalone dequantize kernel in place of those ops.
    nf4 = [m for m in model.modules() if isinstance(m, modules.Ltx23Nf4Linear)]
    rdq = RefGpuDequant(dev)

    def swap_forward(decode):
        saved = []
        for m in nf4:
            def fwd(xx, act=None, m=m):
                w = decode(m)
                y = torch.nn.functional.linear(xx, w, m.bias)
                return torch.nn.functional.gelu(y, approximate="tanh") if act else y
            saved.append((m, m.forward))
            m.forward = fwd
        return saved

    # the reference calls q, k and v as three linears and concatenates with torch.cat
    flux.FUSED_QKV = flux.FUSED_CONCAT = False
    saved = swap_forward(lambda m: rdq.nf4(m.weight_nf4, m.weight_absmax, m.out_features,
                                           m.in_features))
    ref_ms = timed(max(3, args.steps // 2))
    for m, f in saved:
        m.forward = f
    saved = swap_forward(lambda m: ops.ltx23_nf4_dequantize(
        m.weight_nf4, m.weight_absmax, (m.out_features, m.in_features),
        out=rdq.buffer(m.out_features, m.in_features)))
    engine_dq_ms = timed(max(3, args.steps // 2))
    for m, f in saved:
        m.forward = f
    flux.FUSED_QKV = flux.FUSED_CONCAT = True
    del rdq
    if rank == 0:
        cast_flops = 59.50e12  # cast linears per step at 1024x1024, B = 1
        line = {
            "metric": "FLUX.1 1024x1024 DiT step ms", "value": ms, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random N(0,0.02) weights, NF4 cast linears)",
            "config": {"workload": "FLUX.1 transformer, 19 double + 38 single blocks, 4096 image + 512 text "
                                   "tokens, one Euler step, one image per GPU",
                       "parallelism": f"dp{world} (replicas, no collective)"},
            "eager_step_ms": eager_ms,
            "images_per_s_4_steps": world / (4 * ms * 1e-3),
            "cast_linear_tflops_if_all_time": cast_flops / (ms * 1e-3) / 1e12,
            "reference_algorithm_step_ms": ref_ms,
            "speedup_vs_reference_algorithm": ref_ms / ms,
            "engine_dequant_plus_cublas_step_ms": engine_dq_ms,
            "note": "value = the step replayed from a CUDA graph; eager_step_ms without; the reference "
                    "algorithm step (its libtorch NF4 decode ops + cuBLAS per cast linear) and the "
                    "engine-dequantize + cuBLAS step are eager",
            "device_error": err, "clocks": clk.summary(),
        }
        if kernels is not None:
            line["kernels_one_eager_step"] = kernels
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------- decode-sized token counts
SMALL_N, SMALL_K = 18432, 3072  # the FLUX AdaLN modulation projection (3072 -> 6 x 3072)
SMALL_MS = (1, 16, 64, 512)
SMALL_ROTATE = 8  # 8 weight copies (255 MB NF4) > 126 MB L2


def run_small(args, world, rank, local):
    """The small-M sweep: x[M, 3072] . W[18432, 3072]^T for M in 1, 16, 64,
    512, each as a CUDA graph of 40 calls over 8 rotating weight copies.
    M <= 64 is HBM-bound on the weight, so the value is GB/s at M = 1 against
    the measured HBM copy bandwidth; every M is reported."""
    from diffuser_b200 import modules, ops
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    fmt = args.workload.split("_")[1]
    n, k = SMALL_N, SMALL_K
    stream = torch.cuda.current_stream(dev)
    g0 = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(n, k, generator=g0, device=dev) * 0.02
    if fmt == "nf4":
        p0, a0 = ops.ltx23_nf4_quantize(w)
        wsets = [(p0.clone(), a0.clone()) for _ in range(SMALL_ROTATE)]
        wbytes = n * k // 2 + n * k // 64 * 4
        call = lambda i, x: ops.nf4_linear(x, *wsets[i % SMALL_ROTATE], n)
    else:
        w80, s0 = ops.fp8_quantize(w)
        scale = float(s0.item())
        wsets = [w80.clone() for _ in range(SMALL_ROTATE)]
        wbytes = n * k
        call = lambda i, x: ops.fp8_linear(x, wsets[i % SMALL_ROTATE], scale)
    del w
    per_graph = 40
    reps = max(1, args.steps // per_graph)
    rows = []
    with ClockSampler(local) as clk:
        for m in SMALL_MS:
            gx = torch.Generator(device=dev).manual_seed(1 + 100 * rank)
            x = torch.randn(m, k, generator=gx, device=dev).to(torch.bfloat16)
            for i in range(max(args.warmup, 3)):
                call(i, x)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(per_graph):
                    call(i, x)
            graph.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier(world)
            torch.cuda.synchronize()
            a.record(stream)
            for _ in range(reps):
                graph.replay()
            b.record(stream)
            torch.cuda.synchronize()
            barrier(world)
            us = max_over_ranks(a.elapsed_time(b) * 1e3 / (reps * per_graph), world, dev)
            del graph
            plan = ops.plan_info(m, n, k, 0 if fmt == "nf4" else 1)
            byts = wbytes + m * k * 2 + m * n * 2
            rows.append({"M": m, "us": us, "GB_per_s": byts / us / 1e3,
                         "TFLOP_per_s": 2 * m * n * k / us / 1e6, "algorithmic_bytes": byts,
                         "kernel": plan["kernel"], "tile_tokens": plan["bm"], "splits": plan["splits"]})
    err = ops.device_error(dev)
    if err != 0:
        raise RuntimeError(f"kernel error word {err}")

    # M = 1 end to end through the public module with host buffers: x up,
    # y down, every call
    mod = (modules.ltx23_nf4_linear(n, k, bias=False) if fmt == "nf4"
           else modules.ltx23_fp8_linear(n, k, bias=False)).to(dev)
    if fmt == "nf4":
        mod.set_nf4_weight(*wsets[0])
    else:
        mod.set_fp8_weight(wsets[0].view(torch.float8_e4m3fn), torch.tensor(scale))
    xh = torch.randn(1, k).to(torch.bfloat16).pin_memory()
    yh = torch.empty(1, n, dtype=torch.bfloat16).pin_memory()
    n_e2e = max(10, min(args.steps, 200))

    def e2e_step():
        y = mod(xh.to(dev, non_blocking=True))
        yh.copy_(y, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n_e2e):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize()
    e_us = max_over_ranks(a.elapsed_time(b) * 1e3 / n_e2e, world, dev)

    # the reference's GPU algorithm at M = 1: decode the whole weight, then cuBLAS
    ref_us = None
    if world == 1:
        rdq = RefGpuDequant(dev)
        x1 = torch.randn(1, k, device=dev).to(torch.bfloat16)

        def ref_step(i):
            wb = rdq.nf4(*wsets[i % SMALL_ROTATE], n, k) if fmt == "nf4" else rdq.fp8(wsets[i % SMALL_ROTATE].view(torch.uint8), scale)
            return torch.nn.functional.linear(x1, wb)
        for i in range(3):
            ref_step(i)
        torch.cuda.synchronize()
        a.record(stream)
        for i in range(20):
            ref_step(i)
        b.record(stream)
        torch.cuda.synchronize()
        ref_us = a.elapsed_time(b) * 1e3 / 20
        del rdq

    if rank == 0:
        _, _, hbm, peak_src = measured_peaks()
        r1 = rows[0]
        line = {
            "metric": f"{fmt.upper()} small-M quant-linear GB/s (M=1, {k}->{n})",
            "value": world * r1["GB_per_s"], "unit": "GB/s", "n_gpus": world,
            "steps": reps * per_graph, "warmup": max(args.warmup, 3), "ms_per_step": r1["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"{fmt}_linear x[M,{k}]bf16 . W[{n},{k}]{fmt}^T, M in {list(SMALL_MS)}",
                       "parallelism": f"dp{world} (replicas, no collective)",
                       "l2": f"{SMALL_ROTATE} rotating weight copies ({SMALL_ROTATE * wbytes / 1e6:.0f} MB) > 126 MB L2",
                       "launch": "CUDA graph of 40 calls"},
            "roofline": {"bound": "hbm", "achieved": r1["GB_per_s"], "peak": hbm, "unit": "GB/s",
                         "frac": r1["GB_per_s"] / hbm, "traffic": None,
                         "peak_source": f"{peak_src} HBM copy bandwidth",
                         "kernel": r1["kernel"], "algorithmic_bytes": r1["algorithmic_bytes"]},
            "sweep": rows,
            "reference_gpu_algorithm_us_M1": ref_us,
            "speedup_vs_reference_gpu_algorithm_M1": (ref_us / r1["us"]) if ref_us else None,
            "cpu_baseline": None,
            "e2e": {"value": world * r1["algorithmic_bytes"] / e_us / 1e3, "unit": "GB/s",
                    "h2d_bytes_per_step": k * 2, "d2h_bytes_per_step": n * 2, "us_per_step": e_us,
                    "api": f"diffuser_b200.modules.ltx23_{fmt}_linear.forward (eager, one call per step)"},
            "gpu_launches": reps * per_graph,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------ standalone decode
def run_dequant(args, world, rank, local):
    """The standalone dequantization (ltx23_nf4_dequantize, R/nf4_ltx23.R:
    77-115; the fp8 upcast x scale, R/fp8_ltx23.R:79-80) of the 12288 x 3072
    weight into bf16, over 4 rotating weight / output sets (387 MB NF4): HBM-
    bound, value = GB/s of packed + scales read and bf16 written."""
    from diffuser_b200 import ops
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    fmt = args.workload.split("_")[1]
    stream = torch.cuda.current_stream(dev)
    g0 = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(N, K, generator=g0, device=dev) * 0.02
    outs = [torch.empty(N, K, dtype=torch.bfloat16, device=dev) for _ in range(ROTATE)]
    if fmt == "nf4":
        p0, a0 = ops.ltx23_nf4_quantize(w)
        sets = [(p0.clone(), a0.clone()) for _ in range(ROTATE)]
        byts = N * K // 2 + N * K // 64 * 4 + N * K * 2
        call = lambda i: ops.ltx23_nf4_dequantize(*sets[i % ROTATE], (N, K), out=outs[i % ROTATE])
    else:
        w80, s0 = ops.fp8_quantize(w)
        scale = float(s0.item())
        sets = [w80.clone() for _ in range(ROTATE)]
        byts = N * K + N * K * 2
        call = lambda i: ops.fp8_dequantize(sets[i % ROTATE], scale, out=outs[i % ROTATE])
    del w
    for i in range(max(args.warmup, 3)):
        call(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        a.record(stream)
        for i in range(args.steps):
            call(i)
        b.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    us = max_over_ranks(a.elapsed_time(b) * 1e3 / args.steps, world, dev)
    err = ops.device_error(dev)
    if err != 0:
        raise RuntimeError(f"kernel error word {err}")
    # end to end through the public op: packed weight up, bf16 weight down
    e2e = None
    if not args.no_e2e:
        if fmt == "nf4":
            hp, ha = sets[0][0].cpu().pin_memory(), sets[0][1].cpu().pin_memory()
            dp, da = torch.empty_like(sets[0][0]), torch.empty_like(sets[0][1])
            h2d = hp.numel() + ha.numel() * 4
        else:
            hp = sets[0].view(torch.uint8).cpu().pin_memory()
            dp = torch.empty_like(sets[0].view(torch.uint8))
            h2d = hp.numel()
        hw = torch.empty(N, K, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            dp.copy_(hp, non_blocking=True)
            if fmt == "nf4":
                da.copy_(ha, non_blocking=True)
                wb = ops.ltx23_nf4_dequantize(dp, da, (N, K), out=outs[0])
            else:
                wb = ops.fp8_dequantize(dp.view(torch.float8_e4m3fn), scale, out=outs[0])
            hw.copy_(wb, non_blocking=True)

        n_e2e = max(5, min(args.steps, 20))
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        e_us = max_over_ranks(a.elapsed_time(b) * 1e3 / n_e2e, world, dev)
        e2e = {"value": world * byts / e_us / 1e3, "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": N * K * 2, "us_per_step": e_us,
               "api": f"diffuser_b200.ops.{'ltx23_nf4_dequantize' if fmt == 'nf4' else 'fp8_dequantize'}"}
    # the reference's GPU op sequence for the same decode
    ref_us = None
    if world == 1:
        rdq = RefGpuDequant(dev)
        ref = (lambda i: rdq.nf4(*sets[i % ROTATE], N, K)) if fmt == "nf4" else \
            (lambda i: rdq.fp8(sets[i % ROTATE].view(torch.uint8), scale))
        for i in range(3):
            ref(i)
        torch.cuda.synchronize()
        a.record(stream)
        for i in range(20):
            ref(i)
        b.record(stream)
        torch.cuda.synchronize()
        ref_us = a.elapsed_time(b) * 1e3 / 20
        del rdq
    if rank == 0:
        _, _, hbm, peak_src = measured_peaks()
        gbs = byts / us / 1e3
        line = {
            "metric": f"{fmt.upper()} dequantize GB/s ({N}x{K} -> bf16)", "value": world * gbs,
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": us / 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8" if fmt == "nf4" else "fp8", "data": "synthetic",
            "config": {"workload": f"{'ltx23_nf4_dequantize' if fmt == 'nf4' else 'fp8 upcast x scale'} "
                                   f"W[{N},{K}] -> bf16", "parallelism": f"dp{world} (replicas)",
                       "l2": f"{ROTATE} rotating weight / output sets ({ROTATE * byts / 1e6:.0f} MB) > 126 MB L2"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "traffic": None, "peak_source": f"{peak_src} HBM copy bandwidth",
                         "kernel": f"dequant_{fmt}_kernel", "algorithmic_bytes": byts},
            "reference_gpu_algorithm_us": ref_us,
            "speedup_vs_reference_gpu_algorithm": (ref_us / us) if ref_us else None,
            "cpu_baseline": None, "e2e": e2e, "gpu_launches": args.steps, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        if args.workload in ("tp_fp8", "flux_dit", "small_nf4", "small_fp8", "dequant_nf4", "dequant_fp8"):
            if rank == 0:
                why = ("the reference runs each linear on one GPU; it has no column-parallel path"
                       if args.workload == "tp_fp8" else
                       "the reference's FLUX step runs in R (not installed); its GPU linear algorithm "
                       "is timed inside the flux_dit line (reference_algorithm_step_ms)"
                       if args.workload == "flux_dit" else
                       "the small-M sweep times the reference's GPU algorithm at M = 1 inside its own line "
                       "(reference_gpu_algorithm_us_M1); the CPU reference arm runs on the default workload"
                       if args.workload.startswith("small_") else
                       "the decode line times the reference's GPU op sequence inside its own line "
                       "(reference_gpu_algorithm_us); the CPU reference arm runs on the default workload")
                print(json.dumps({"impl": "reference", "unavailable": why}))
            return
        run_reference_arm(args, world, rank)
        return
    if args.workload == "tp_fp8":
        run_tp(args, world, rank, local)
        return
    if args.workload == "flux_dit":
        run_flux(args, world, rank, local)
        return
    if args.workload.startswith("small_"):
        run_small(args, world, rank, local)
        return
    if args.workload.startswith("dequant_"):
        run_dequant(args, world, rank, local)
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
