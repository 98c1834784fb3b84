#!/usr/bin/env python
"""Benchmark of the fused NF4 / fp8 weight-only linear on B200.

One step = one fused quantized linear over one batch of synthetic tokens:
x bf16 [4608, 3072] (one 1024x1024 FLUX image's 4096 latent + 512 text
tokens) times W [12288, 3072] (NF4 by default, the FLUX feed-forward up
projection shape), y bf16 [4608, 12288].  With N GPUs (torchrun, one process
per GPU) every rank runs its own token batch against a replicated weight: data
parallel, no data-path collective, weak scaling; the value is the whole-job
TFLOP/s from the max-over-ranks device time.

The same run then measures, into the same JSON line, the rest of the
benchmark suite at this N: the fp8 linear of the same shape (`fp8_linear`),
the small-M sweep of the modulation projection (`small_m`), the four LTX
video linears (`ltx_fp8`: single GPU at N = 1, column-parallel over the N
GPUs with the fused NVLink all-gather at N > 1, with a bit-exactness check
against the single-GPU kernel), and one FLUX.1 1024x1024 DiT step per GPU
(`dit_step`: data parallel, one image per rank).

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
                    help="flux_dit: add the per-kernel device-time table of three graph replays")
    ap.add_argument("--probe", choices=["ring16", "qkv_glue"], default=None,
                    help="run one kernel a few times for an ncu capture and exit (no JSON line): "
                         "ring16 = the two-token-tile small-M ring kernel, NF4 x[16,3072] . "
                         "W[18432,3072]^T, 6 calls; qkv_glue = the FLUX q/k/v norm + RoPE glue at "
                         "4096 + 512 tokens x 24 heads, 4 calls")
    ap.add_argument("--extras", default="fp8,small,ltx,dit",
                    help="default workload: comma list of the sections measured after the "
                         "headline linear (fp8, small, ltx, dit) or 'none'")
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
    """(DRAM bytes per launch, source) of the planned kernel from its committed
    ncu summary, only when that summary was captured on the same plan (its
    `plan_bm:` line equals the x-tile height planned now); else (None, why).
    The number is from an ncu capture, not measured in this run."""
    kern = "bf16_gemm2" if plan["twophase"] else ("dq_gemm2" if plan["pair"] else "dq_gemm")
    name = f"{kern}_{workload}_4608x3072x12288.md"
    try:
        txt = open(os.path.join(ROOT, "profiles", name)).read()
    except OSError:
        return None, f"no ncu summary of {kern} at this shape"
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    b = re.search(r"plan_bm:\s*([0-9]+)", txt)
    if not m or not b or int(b.group(1)) != plan["bm"]:
        return None, f"profiles/{name} was captured on another plan"
    return float(m.group(1)), f"ncu capture of the same plan (profiles/{name}), not this run"


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


def host_threads() -> int:
    """Use every host core this process may run on, whatever OMP_NUM_THREADS
    the launcher set (torchrun sets 1)."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(max(1, n))
    return torch.get_num_threads()


def run_cpu_baseline(workload: str, budget_s: float = 12.0):
    host_threads()
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


def headline_config(fmt: str, world: int) -> dict:
    """The headline workload's `config`, identical in both arms."""
    return {"workload": WORKLOADS[fmt]["desc"], "format": fmt, "M": M, "N": N, "K": K,
            "bias": False,
            "parallelism": f"dp{world} (own token batch per GPU, replicated weight, no collective)",
            "l2": f"{ROTATE} rotating input sets ({ROTATE * WORKLOADS[fmt]['bytes'] / 1e6:.0f} MB) > 126 MB L2"}


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    threads = host_threads()
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
        "config": headline_config(args.workload, world),
        "row_slice": REF_ROW_SLICE,
        "reference_execution": (f"rank 0 only, {threads} host threads; each step runs the whole x "
                                f"against 1/{REF_ROW_SLICE} of the weight rows and is counted by its "
                                "own FLOPs"),
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": desc},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ timing
class Ctx:
    """One rank's device, launch stream and place in the job."""

    def __init__(self, args, world, rank, local):
        self.args, self.world, self.rank, self.local = args, world, rank, local
        torch.cuda.set_device(local)
        self.dev = torch.device("cuda", local)
        self.stream = torch.cuda.current_stream(self.dev)

    def timed(self, fn, steps: int, warmup: int | None = None):
        """Run fn(i) warmup times untimed, then `steps` times between CUDA
        events on the launch stream, bracketed by a barrier and a synchronize
        on both sides.  Returns (max over ranks of ms per step, per-rank ms)."""
        for i in range(max(self.args.warmup if warmup is None else warmup, 3)):
            fn(i)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(self.world)
        torch.cuda.synchronize()
        a.record(self.stream)
        for i in range(steps):
            fn(i)
        b.record(self.stream)
        torch.cuda.synchronize()
        barrier(self.world)
        ms = a.elapsed_time(b) / steps
        return max_over_ranks(ms, self.world, self.dev), gather_ranks(ms, self.world, self.dev)


def release(*_):
    """Free what a section held before the next one starts."""
    from diffuser_b200 import ops
    ops.release_workspaces()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ------------------------------------------------------------------ our arm
def run_ours(args, world, rank, local):
    from diffuser_b200 import _lib, modules, ops

    ctx = Ctx(args, world, rank, local)
    dev, stream = ctx.dev, ctx.stream
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    lib = _lib.lib()
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
        del mod, xh, yh, xd

    # ---- the reference's GPU algorithm on the same box, inputs and rotation:
    # decode the weight with its libtorch op sequence into the per-shape
    # buffer, then torch.nn.functional.linear (every rank, its own GPU)
    rdq = RefGpuDequant(dev)

    def ref_step(i):
        x = xs[i % ROTATE]
        wp, ap = wsets[i % ROTATE]
        wb = rdq.nf4(wp, ap, N, K) if fmt == "nf4" else rdq.fp8(wp, scale)
        return torch.nn.functional.linear(x, wb)

    r_ms, _ = ctx.timed(ref_step, max(10, min(args.steps, 100)))
    ref_gpu = {"value": world * FLOPS_PER_STEP / (r_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": r_ms, "steps": max(10, min(args.steps, 100)),
               "algorithm": ("chunked byte-table gather + per-block mul into a bf16 buffer "
                             "(R/nf4_ltx23.R:77-115), then F.linear (cuBLAS)") if fmt == "nf4"
               else "copy_ upcast + mul_ by bf16 scale (R/fp8_ltx23.R:79-80), then F.linear (cuBLAS)"}
    del rdq, xs, ys, wsets, ws
    release()

    # ---- the rest of the suite at this N, into the same line
    extras = {}
    wanted = [] if args.extras == "none" else [e.strip() for e in args.extras.split(",") if e.strip()]
    if "fp8" in wanted and fmt == "nf4":
        extras["fp8_linear"] = linear_section(ctx, "fp8")
        release()
    if "small" in wanted:
        extras["small_m"] = {f: small_section(ctx, f)[0] for f in ("nf4", "fp8")}
        release()
    if "ltx" in wanted:
        extras["ltx_fp8"] = ltx_section(ctx)
        release()
    if "dit" in wanted:
        extras["dit_step"] = dit_section(ctx, reference=True)
        release()

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
        traffic, traffic_src = profile_traffic(fmt, plan)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = run_cpu_baseline(fmt)
        value = world * FLOPS_PER_STEP * args.steps / (el_ms_max * 1e-3) / 1e12
        line = {
            "metric": "NF4/fp8 quant-linear TFLOP/s",
            "value": value,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": el_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": headline_config(fmt, world),
            # kernel_ms brackets one whole call: with the two-phase plan the
            # counter memset plus the GEMM launch that decodes its weight
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "traffic": traffic, "traffic_source": traffic_src,
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
            "speedup_vs_reference_gpu_algorithm": value / ref_gpu["value"],
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------------ fp8 linear (config 1)
def linear_section(ctx, fmt: str) -> dict:
    """The headline shape x[4608,3072] . W[12288,3072]^T in `fmt`, every rank
    its own tokens, ROTATE input sets; device time per call, max over ranks."""
    from diffuser_b200 import ops
    dev = ctx.dev
    w = torch.randn(N, K, generator=torch.Generator(device=dev).manual_seed(0), device=dev) * 0.02
    if fmt == "nf4":
        p0, a0 = ops.ltx23_nf4_quantize(w)
        wsets = [(p0.clone(), a0.clone()) for _ in range(ROTATE)]
        call = lambda i: ops.nf4_linear(xs[i % ROTATE], *wsets[i % ROTATE], N, out=ys[i % ROTATE])  # noqa: E731
    else:
        w80, s0 = ops.fp8_quantize(w)
        scale = float(s0.item())
        wsets = [w80.clone() for _ in range(ROTATE)]
        call = lambda i: ops.fp8_linear(xs[i % ROTATE], wsets[i % ROTATE], scale, out=ys[i % ROTATE])  # noqa: E731
    del w
    xs = [torch.randn(M, K, generator=torch.Generator(device=dev).manual_seed(1 + 100 * ctx.rank + i),
                      device=dev).to(torch.bfloat16) for i in range(ROTATE)]
    ys = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(ROTATE)]
    ms, ranks = ctx.timed(call, ctx.args.steps)
    plan = ops.plan_info(M, N, K, 0 if fmt == "nf4" else 1)
    burst, sustained, _, src = measured_peaks()
    tf = FLOPS_PER_STEP / (ms * 1e-3) / 1e12
    return {"workload": WORKLOADS[fmt]["desc"], "ms_per_call": ms, "ms_per_call_per_rank": ranks,
            "tflops_per_gpu": tf, "tflops_job": ctx.world * tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": burst, "unit": "TFLOP/s",
                         "frac": tf / burst, "peak_source": f"{src} bf16 dense, burst",
                         "algorithmic_bytes": WORKLOADS[fmt]["bytes"]},
            "mma": "tcgen05.mma kind::f16 (bf16 x bf16): the weight is decoded e4m3 -> bf16 "
                   "bit-exactly as the reference's upcast x bf16(scale)" if fmt == "fp8" else
                   "tcgen05.mma kind::f16 (bf16 x bf16) on the decoded NF4 weight",
            "plan": plan, "l2": f"{ROTATE} rotating input sets > 126 MB L2"}


# ------------------------------------------------------- column-parallel
TP_M, TP_N, TP_K = 6144, 12288, 4096  # LTX video tokens x fused q/k/v projection (4096 -> 3 x 4096)
LTX_M = 6144  # 121-frame 768x512 video: latent 16 x 16 x 24 tokens
# (K, N, name): the LTX-2.3 transformer block's linears (R/dit_ltx23_modules.R:381-386,500-526)
LTX_SHAPES = [(4096, 12288, "attn q/k/v (concatenated)"), (4096, 4096, "attn out"),
              (4096, 16384, "ff up"), (16384, 4096, "ff down")]
PEER_GBS = 770.0  # measured NVLink peer copy per direction per GPU on this B200 pool


def ltx_section(ctx) -> dict:
    """The four LTX video linears in fp8 at M = 6144 tokens.  One GPU: the
    automatic single-GPU plan.  N > 1 GPUs: column-parallel over the ranks
    (each computes [M, N/G] and its epilogue stores the block into every
    rank's y over NVLink, then a bounded flag barrier), strong scaling; beside
    it the NCCL all-gather path, and a bit-for-bit comparison of the assembled
    y with the single-GPU kernel on the full weight."""
    from diffuser_b200 import ops
    dev, world = ctx.dev, ctx.world
    burst, _, _, src = measured_peaks()
    rows = []
    grp = grp_mc = None
    if world > 1:
        from diffuser_b200 import tp
        grp = tp.TpGroup(LTX_M, max(n for _, n, _ in LTX_SHAPES))
        try:  # y buffers bound to an NVLink multicast object: one multimem store per 16 bytes
            grp_mc = tp.TpGroup(LTX_M, max(n for _, n, _ in LTX_SHAPES), multicast=True)
        except RuntimeError:
            grp_mc = None
    try:
        for k, n, name in LTX_SHAPES:
            w = torch.randn(n, k, generator=torch.Generator(device=dev).manual_seed(0), device=dev) * 0.02
            w8, s0 = ops.fp8_quantize(w)  # the same weight on every rank
            del w
            scale = float(s0.item())
            xs = [torch.randn(LTX_M, k, generator=torch.Generator(device=dev).manual_seed(1 + i),
                              device=dev).to(torch.bfloat16) for i in range(2)]
            flops = 2 * LTX_M * n * k
            row = {"shape": f"x[{LTX_M},{k}] . W[{n},{k}]^T", "name": name, "K": k, "N": n,
                   "compute_bound_ms": flops / world / (burst * 1e12) * 1e3}
            if grp is None:
                ys = [torch.empty(LTX_M, n, dtype=torch.bfloat16, device=dev) for _ in range(2)]
                ms, _ = ctx.timed(lambda i: ops.fp8_linear(xs[i % 2], w8, scale, out=ys[i % 2]),
                                  ctx.args.steps)
                row.update({"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12,
                            "frac_of_burst_peak": flops / (ms * 1e-3) / 1e12 / burst,
                            "kernel": ops.plan_info(LTX_M, n, k, 1)["kernel"]})
                del ys
            else:
                from diffuser_b200 import tp
                ref = ops.fp8_linear(xs[0], w8, scale)  # single-GPU kernel, full weight
                mod = tp.ColumnParallelFp8Linear(k, n, grp, bias=False).to(dev)
                mod.set_fp8_weight(w8, scale)
                mods = [mod]
                if grp_mc is not None:
                    mod_mc = tp.ColumnParallelFp8Linear(k, n, grp_mc, bias=False).to(dev)
                    mod_mc.set_fp8_weight(w8, scale)
                    mods.append(mod_mc)
                same = 1.0
                for mm in mods:
                    y = mm(xs[0])
                    torch.cuda.synchronize()
                    same = min(same, float(torch.equal(y, ref)))
                same_all = -max_over_ranks(-same, world, dev)  # min over ranks
                del ref, y
                peer_ms, peer_ranks = ctx.timed(lambda i: mod(xs[i % 2]), ctx.args.steps)
                fused, fused_ranks, mc_ms = peer_ms, peer_ranks, None
                if grp_mc is not None:
                    mc_ms, mc_ranks = ctx.timed(lambda i: mod_mc(xs[i % 2]), ctx.args.steps)
                    if mc_ms < peer_ms:  # the same decision on every rank: both are maxima
                        fused, fused_ranks = mc_ms, mc_ranks
                nccl, _ = ctx.timed(lambda i: mod.forward_nccl(xs[i % 2]), ctx.args.steps)
                peer = (world - 1) * LTX_M * (n // world) * 2  # bytes each rank sends
                nvlink_bound = peer / (PEER_GBS * 1e9) * 1e3
                row.update({"fused_ms": fused, "fused_ms_per_rank": fused_ranks,
                            "fused_stores": "multimem (NVLink multicast)" if fused is mc_ms
                            else "per-rank peer stores",
                            "peer_stores_ms": peer_ms, "multimem_ms": mc_ms,
                            "nccl_allgather_path_ms": nccl,
                            "tflops_job": flops / (fused * 1e-3) / 1e12,
                            "tflops_per_gpu": flops / world / (fused * 1e-3) / 1e12,
                            "nvlink_gbs_per_gpu": peer / (fused * 1e-3) / 1e9,
                            "nvlink_bound_ms": nvlink_bound,
                            "limiter": "nvlink" if nvlink_bound > row["compute_bound_ms"] else "compute",
                            "frac_of_bound": max(nvlink_bound, row["compute_bound_ms"]) / fused,
                            "parity_bitexact_vs_single_gpu": bool(same_all >= 1.0)})
                del mod, mods
            rows.append(row)
            del w8, xs
            release()
    finally:
        if grp_mc is not None:
            grp_mc.close()
        if grp is not None:
            grp.close()
    out = {"workload": f"LTX-2.3 video DiT linears, fp8 e4m3 per-tensor, M={LTX_M} tokens",
           "parallelism": (f"tp{world} column-parallel over out_features, fused NVLink all-gather "
                           "(epilogue peer stores, or multimem stores through an NVLink multicast "
                           "mapping, whichever is faster per shape; bounded flag barrier)")
                          if world > 1 else "single GPU",
           "scaling": "strong" if world > 1 else None,
           "peak_source": f"{src} bf16 dense (burst); NVLink bound at the measured {PEER_GBS:.0f} GB/s "
                          "peer copy per direction", "shapes": rows}
    if world > 1:
        out["parity_bitexact_all"] = all(r["parity_bitexact_vs_single_gpu"] for r in rows)
        out["device_error"] = ops.device_error(dev)
    return out


def run_tp(args, world, rank, local):
    """Column-parallel fp8 linear x[6144,4096] . W[12288,4096]^T over `world`
    GPUs: total work fixed (strong scaling).  Each rank's fused kernel writes
    its [M, N/world] block into every rank's y through NVLink: per-rank peer
    stores, and (N > 1, where the GPUs offer it) multimem stores through a
    multicast mapping; the line reports the faster and lists both."""
    import torch.distributed as dist
    from diffuser_b200 import ops, tp

    ctx = Ctx(args, world, rank, local)
    dev = ctx.dev
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    else:
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29599", rank=0, world_size=1)
    g0 = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(TP_N, TP_K, generator=g0, device=dev) * 0.02
    w8, s0 = ops.fp8_quantize(w)
    del w
    groups = [tp.TpGroup(TP_M, TP_N)]  # per-rank peer stores
    if world > 1:
        try:  # y buffers bound to an NVLink multicast object: one multimem store per 16 bytes
            groups.append(tp.TpGroup(TP_M, TP_N, multicast=True))
        except RuntimeError:
            pass
    mods = []
    for grp in groups:
        mods.append(tp.ColumnParallelFp8Linear(TP_K, TP_N, grp, bias=False).to(dev))
        mods[-1].set_fp8_weight(w8, float(s0.item()))
    del w8
    xs = [torch.randn(TP_M, TP_K, generator=torch.Generator(device=dev).manual_seed(1 + i),
                      device=dev).to(torch.bfloat16) for i in range(2)]

    times = {}
    with ClockSampler(local) as clk:
        for grp, mod in zip(groups, mods):
            key = "multimem" if grp.multicast else "peer_stores"
            times[key], _ = ctx.timed(lambda i, mod=mod: mod(xs[i % 2]), args.steps)
    err = ops.device_error(dev)
    nccl_ms = None
    if world > 1:
        nccl_ms, _ = ctx.timed(lambda i: mods[0].forward_nccl(xs[i % 2]), max(10, args.steps // 4))
    best = min(times, key=times.get)
    fused_ms = times[best]
    multicast = best == "multimem"
    del mods
    for grp in reversed(groups):
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
                       "collective": "fused: epilogue " + ("multimem stores (NVLink multicast)"
                                                           if multicast else "peer stores")
                                     + " + flag barrier"},
            "per_gpu_tflops": flops / world / (fused_ms * 1e-3) / 1e12,
            "nvlink_gbs_per_gpu": peer_bytes / (fused_ms * 1e-3) / 1e9,
            "compute_bound_ms": flops / world / (peak_tf * 1e12) * 1e3,
            "nccl_allgather_path_ms": nccl_ms,
            "fused_ms_by_store_path": times,
            "peak_source": f"{peak_src} bf16 dense (burst)",
            "device_error": err, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


# ------------------------------------------------------------ FLUX DiT step
DIT_CAST_FLOPS = 59.50e12  # the 494 cast linears of one step at 1024x1024, one image
DIT_ATTN_FLOPS = 14.87e12  # 57 blocks x 4 x 4608^2 x 3072 (QK^T and PV)


def dit_section(ctx, reference: bool = True, profile: bool = False) -> dict:
    """One flow-match Euler step of the FLUX.1 transformer at 1024x1024 (4096
    image + 512 text tokens) with its 494 cast linears in NF4 on the fused
    engine, one image per GPU (latent seed 10 + rank): data parallel, no
    collective.  Timed eager and as a replayed CUDA graph; with `reference`
    also the same step with the reference's linear algorithm (its libtorch NF4
    decode ops into a per-shape bf16 buffer, then cuBLAS) and with the
    engine's standalone dequantize kernel + cuBLAS."""
    from diffuser_b200 import flux, modules, ops
    dev, world, args = ctx.dev, ctx.world, ctx.args
    t0 = time.perf_counter()
    model = flux.build_flux_nf4(dev, seed=0)
    build_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(10 + ctx.rank)
    x = flux.pack_latents(torch.randn(1, 16, 128, 128, generator=g)).to(dev, torch.bfloat16)
    g1 = torch.Generator().manual_seed(3)
    text = torch.randn(1, 512, 4096, generator=g1).to(dev, torch.bfloat16)
    pooled = torch.randn(1, 768, generator=g1).to(dev, torch.bfloat16)
    ids = torch.cat([torch.zeros(512, 3), flux.prepare_latent_image_ids(64, 64)], dim=0)
    rope = flux.pos_embed(ids.to(dev), (16, 56, 56))
    t = torch.ones(1, dtype=torch.float32, device=dev)

    def step(_i=0):
        with torch.no_grad():
            v = model(x, text, pooled, t, rope)
            return flux.euler_step(v, 1.0, 0.75, x)

    steps = max(5, args.steps)
    with ClockSampler(ctx.local) as clk:
        eager_ms, eager_ranks = ctx.timed(step, steps)
        # the same step captured once in a CUDA graph and replayed (the engine
        # launches on torch's current stream with cached workspaces, so the
        # whole step captures)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step_out = step()
        graph_ms, graph_ranks = ctx.timed(lambda i: graph.replay(), steps, warmup=3)
    kernels = None
    if profile:
        # Three graph replays back to back under the torch profiler (outside
        # every timed region), bracketed by CUDA events and with the SM clock
        # sampled: the kernels' summed device time per replay against the
        # replay's own event time, at the same clocks, shows how much of the
        # step is gaps between kernels rather than kernel time.
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(ctx.local) as pclk:
            with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
                a.record(ctx.stream)
                for _ in range(3):
                    graph.replay()
                b.record(ctx.stream)
                torch.cuda.synchronize()
        replay_ms = a.elapsed_time(b) / 3
        ka = prof.key_averages()
        total = sum(e.device_time_total for e in ka) / 3
        launches = sum(e.count for e in ka) / 3
        kernels = {"replays": 3, "replay_ms_event": replay_ms, "kernel_ms_sum_per_replay": total / 1e3,
                   "kernels_per_replay": launches,
                   "gap_ms_per_replay": replay_ms - total / 1e3,
                   "clocks": pclk.summary(),
                   "top": [{"kernel": e.key[:120], "launches_per_replay": e.count / 3,
                            "ms_per_replay": e.device_time_total / 3e3,
                            "share": e.device_time_total / 3 / total}
                           for e in sorted(ka, key=lambda e: -e.device_time_total)[:24]]}
    err = ops.device_error(dev)
    del graph, step_out
    ref_ms = engine_dq_ms = None
    if reference:
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
        try:
            saved = swap_forward(lambda m: rdq.nf4(m.weight_nf4, m.weight_absmax, m.out_features,
                                                   m.in_features))
            ref_ms, _ = ctx.timed(step, max(3, steps // 2))
            for m, f in saved:
                m.forward = f
            saved = swap_forward(lambda m: ops.ltx23_nf4_dequantize(
                m.weight_nf4, m.weight_absmax, (m.out_features, m.in_features),
                out=rdq.buffer(m.out_features, m.in_features)))
            engine_dq_ms, _ = ctx.timed(step, max(3, steps // 2))
            for m, f in saved:
                m.forward = f
        finally:
            flux.FUSED_QKV = flux.FUSED_CONCAT = True
        del rdq
    del model
    _, sustained, _, src = measured_peaks()
    flops = DIT_CAST_FLOPS + DIT_ATTN_FLOPS
    tf = flops / (graph_ms * 1e-3) / 1e12
    spread = max(graph_ranks) / min(graph_ranks) - 1.0
    out = {"workload": "FLUX.1-schnell transformer, 19 double + 38 single blocks, 4096 image + 512 "
                       "text tokens (1024x1024), one flow-match Euler step, one image per GPU, NF4 "
                       "cast linears (random N(0,0.02) weights)",
           "parallelism": f"dp{world} (one image per rank, replicated weights, no collective)",
           "graph_ms": graph_ms, "graph_ms_per_rank": graph_ranks,
           "eager_ms": eager_ms, "eager_ms_per_rank": eager_ranks, "steps": steps,
           "images_per_s_4_steps": world / (4 * graph_ms * 1e-3),
           "reference_algorithm_step_ms": ref_ms,
           "speedup_vs_reference_algorithm": (ref_ms / graph_ms) if ref_ms else None,
           "engine_dequant_plus_cublas_step_ms": engine_dq_ms,
           "flops_per_step": flops,
           "roofline": {"bound": "tensor", "achieved": tf, "peak": sustained, "unit": "TFLOP/s",
                        "frac": tf / sustained,
                        "peak_source": f"{src} bf16 dense, sustained (the step runs back to back for seconds)"},
           "limiter": (f"per-rank compute (no collective); slowest rank {spread * 100:.1f}% above the fastest"
                       if world > 1 else "compute (tensor cores; kernel table in profiles/flux_dit_step_1024.md)"),
           "model_build_s": build_s, "device_error": err, "clocks": clk.summary(),
           "note": "graph_ms = the step replayed from a CUDA graph; eager_ms without; the reference "
                   "algorithm step and the engine-dequantize + cuBLAS step are eager"}
    if kernels is not None:
        out["kernels_graph_replay"] = kernels
    return out


def run_flux(args, world, rank, local):
    """The DiT step alone, as its own line (value = graph step ms)."""
    ctx = Ctx(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=ctx.dev)
    d = dit_section(ctx, reference=True, profile=args.profile_kernels)
    if rank == 0:
        line = {
            "metric": "FLUX.1 1024x1024 DiT step ms", "value": d["graph_ms"], "unit": "ms",
            "n_gpus": world, "steps": d["steps"], "warmup": max(args.warmup, 3),
            "ms_per_step": d["graph_ms"], "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random N(0,0.02) weights, NF4 cast linears)",
            "config": {"workload": d["workload"], "parallelism": d["parallelism"]},
            "dit_step": d,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ------------------------------------------------- decode-sized token counts
SMALL_N, SMALL_K = 18432, 3072  # the FLUX AdaLN modulation projection (3072 -> 6 x 3072)
SMALL_MS = (1, 16, 64, 512)
SMALL_ROTATE = 8  # 8 weight copies (255 MB NF4) > 126 MB L2


def small_section(ctx, fmt: str, with_reference: bool = False) -> dict:
    """The small-M sweep: x[M, 3072] . W[18432, 3072]^T for M in 1, 16, 64,
    512, each as a CUDA graph of 40 calls over 8 rotating weight copies.
    M <= 64 is HBM-bound on the weight: GB/s against the measured HBM copy
    bandwidth; M = 512 is compute-bound: TFLOP/s."""
    from diffuser_b200 import ops
    dev, args = ctx.dev, ctx.args
    n, k = SMALL_N, SMALL_K
    w = torch.randn(n, k, generator=torch.Generator(device=dev).manual_seed(0), device=dev) * 0.02
    if fmt == "nf4":
        p0, a0 = ops.ltx23_nf4_quantize(w)
        wsets = [(p0.clone(), a0.clone()) for _ in range(SMALL_ROTATE)]
        wbytes = n * k // 2 + n * k // 64 * 4
        call = lambda i, x: ops.nf4_linear(x, *wsets[i % SMALL_ROTATE], n)  # noqa: E731
    else:
        w80, s0 = ops.fp8_quantize(w)
        scale = float(s0.item())
        wsets = [w80.clone() for _ in range(SMALL_ROTATE)]
        wbytes = n * k
        call = lambda i, x: ops.fp8_linear(x, wsets[i % SMALL_ROTATE], scale)  # noqa: E731
    del w
    per_graph = 40
    reps = max(1, args.steps // per_graph) if args.steps >= per_graph else 1
    _, _, hbm, src = measured_peaks()
    burst = measured_peaks()[0]
    rows = []
    for m in SMALL_MS:
        x = torch.randn(m, k, generator=torch.Generator(device=dev).manual_seed(1 + 100 * ctx.rank),
                        device=dev).to(torch.bfloat16)
        for i in range(max(args.warmup, 3)):
            call(i, x)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(per_graph):
                call(i, x)
        ms, _ = ctx.timed(lambda i: graph.replay(), reps, warmup=1)
        us = ms * 1e3 / per_graph
        del graph
        plan = ops.plan_info(m, n, k, 0 if fmt == "nf4" else 1)
        byts = wbytes + m * k * 2 + m * n * 2
        gbs, tfs = byts / us / 1e3, 2 * m * n * k / us / 1e6
        rows.append({"M": m, "us": us, "GB_per_s": gbs, "frac_of_hbm": gbs / hbm,
                     "TFLOP_per_s": tfs, "frac_of_burst_bf16": tfs / burst,
                     "bound": "hbm" if m <= 64 else "tensor", "algorithmic_bytes": byts,
                     "kernel": plan["kernel"], "tile_tokens": plan["bm"], "splits": plan["splits"]})
    err = ops.device_error(dev)
    if err != 0:
        raise RuntimeError(f"kernel error word {err}")
    out = {"workload": f"{fmt}_linear x[M,{k}]bf16 . W[{n},{k}]{fmt}^T (FLUX AdaLN modulation shape)",
           "launch": f"CUDA graph of {per_graph} calls, {SMALL_ROTATE} rotating weight copies "
                     f"({SMALL_ROTATE * wbytes / 1e6:.0f} MB) > 126 MB L2",
           "peak_source": f"{src} HBM copy bandwidth {hbm:.0f} GB/s", "sweep": rows}
    if with_reference:
        # the reference's GPU algorithm at M = 1: decode the whole weight, then cuBLAS
        rdq = RefGpuDequant(dev)
        x1 = torch.randn(1, k, device=dev).to(torch.bfloat16)

        def ref_step(i):
            wb = rdq.nf4(*wsets[i % SMALL_ROTATE], n, k) if fmt == "nf4" else \
                rdq.fp8(wsets[i % SMALL_ROTATE].view(torch.uint8), scale)
            return torch.nn.functional.linear(x1, wb)
        r_ms, _ = ctx.timed(ref_step, 20)
        out["reference_gpu_algorithm_us_M1"] = r_ms * 1e3
        del rdq
    return out, wsets, (scale if fmt == "fp8" else None)


def run_small(args, world, rank, local):
    """The small-M sweep as its own line (value = GB/s at M = 1)."""
    from diffuser_b200 import modules
    ctx = Ctx(args, world, rank, local)
    dev, stream = ctx.dev, ctx.stream
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    fmt = args.workload.split("_")[1]
    n, k = SMALL_N, SMALL_K
    with ClockSampler(local) as clk:
        sec, wsets, scale = small_section(ctx, fmt, with_reference=(world == 1))
    rows = sec["sweep"]

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

    def e2e_step(_i):
        y = mod(xh.to(dev, non_blocking=True))
        yh.copy_(y, non_blocking=True)

    n_e2e = max(10, min(args.steps, 200))
    e_ms, _ = ctx.timed(e2e_step, n_e2e)
    e_us = e_ms * 1e3
    del stream
    ref_us = sec.get("reference_gpu_algorithm_us_M1")
    if rank == 0:
        _, _, hbm, peak_src = measured_peaks()
        r1 = rows[0]
        line = {
            "metric": f"{fmt.upper()} small-M quant-linear GB/s (M=1, {k}->{n})",
            "value": world * r1["GB_per_s"], "unit": "GB/s", "n_gpus": world,
            "steps": max(1, args.steps // 40) * 40, "warmup": max(args.warmup, 3), "ms_per_step": r1["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"{fmt}_linear x[M,{k}]bf16 . W[{n},{k}]{fmt}^T, M in {list(SMALL_MS)}",
                       "parallelism": f"dp{world} (replicas, no collective)",
                       "l2": sec["launch"], "launch": "CUDA graph of 40 calls"},
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
            "gpu_launches": max(1, args.steps // 40) * 40,
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


def run_probe(which: str):
    """A few launches of one kernel on small inputs, for an ncu capture."""
    from diffuser_b200 import flux, ops
    torch.cuda.set_device(0)
    if which == "ring16":
        k, n, m = 3072, 18432, 16
        w = torch.randn(n, k, device="cuda") * 0.02
        p, a = ops.ltx23_nf4_quantize(w)
        ws = [(p, a), (p.clone(), a.clone())]
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        assert ops.plan_info(m, n, k)["ring"]
        for i in range(6):
            ops.nf4_linear(x, ws[i % 2][0], ws[i % 2][1], n)
    else:
        H, D, S_img, S_txt = 24, 128, 4096, 512
        hd = H * D
        img = torch.randn(1, S_img, 3 * hd, device="cuda").to(torch.bfloat16)
        txt = torch.randn(1, S_txt, 3 * hd, device="cuda").to(torch.bfloat16)
        pi = [img[..., j * hd:(j + 1) * hd] for j in range(3)]
        pt = [txt[..., j * hd:(j + 1) * hd] for j in range(3)]
        w = [torch.ones(D, device="cuda", dtype=torch.bfloat16) for _ in range(4)]
        ids = torch.cat([torch.zeros(S_txt, 3), flux.prepare_latent_image_ids(64, 64)], dim=0)
        rope = flux.pos_embed(ids.cuda(), (16, 56, 56))
        for _ in range(4):
            flux.qkv_norm_rope(pi, pt, H, (w[0], w[1], None), (w[2], w[3], None), (True, True, False),
                               rope, 1e-6)
    torch.cuda.synchronize()
    print(f"probe {which}: ok, device error {ops.device_error()}")


def main():
    args = parse()
    if args.probe is not None:
        run_probe(args.probe)
        return
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
