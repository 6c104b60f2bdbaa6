#!/usr/bin/env python3
"""Benchmark of the fused Winograd 3x3 convolution on B200.

Headline workload (one "step" = one layer over one batch): 3x3 conv, stride 1,
pad 1, F(2x2,3x3), fp32 NCHW in and out, N=64 images, 128->128 channels,
56x56, ReLU; x ~ U(-1,1), Kaiming-normal weights, zero bias.  With --gpus G the
64 images are split across the G ranks (64/G each, contiguous shards) and
every rank holds its own copy of the transformed weights: no collective on the
data path ("strong" scaling; --weak gives every rank the whole batch instead).

Prints one JSON line (rank 0).  `value` = effective conv TFLOP/s of the whole
job (2*N*K*C*H*W*9 over the global batch / max-over-ranks device time);
`ms_per_step` is the time of one layer.  The timed region repeats the K-step
block until it lasts at least --min-time seconds (`timed_repeats`).  `e2e` is
the same metric through the public host-buffer call (cwg_conv3x3_fused_host:
H2D of x, kernel, D2H of y, sync).  After the timed regions, two sampled output
images of every rank (its first and last) are gathered to rank 0 over NCCL and
compared with the CPU oracle (`verify`).  The default run also measures the
bf16 F(4,3) large layer (N=128, 256->256, 112x112) and the ResNet-18-shaped
stride-1 stack (N=256, 13 layers, per-layer and end-to-end) and nests them in
the same line under `workloads`.

  python bench.py [--gpus G] [--steps K] [--warmup W] [--config 1..5 --layer i]
  python bench.py --impl reference ...   # the reference's own CPU kernel
  python bench.py --model resnet18|resnet34|vgg16|alexnet [--n N]   # chained stride-1 stack
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "cache-aware-wino-implementation_b200")
sys.path.insert(0, PKG)

import ranks  # noqa: E402
import workloads  # noqa: E402

METRIC = ("µs/layer and effective conv TFLOP/s (2·N·K·C·H·W·9) "
          "at 1/2/4/8 B200 vs roofline")
L2_BYTES = 126 * 1024 * 1024
# fp32 FFMA peak of a B200 (148 SMs x 128 lanes x 2 flops x 1.965 GHz): the
# compute roof of the CUDA-core kernels, nominal (no measured figure exists)
FFMA_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
# MACs the 2-SM tensor-core MMAs issue per plain-Winograd GEMM MAC: the pair
# kernel stacks two output rows i of At M into the MMA's M dimension (F(2,3):
# both rows, all 16 frequencies: 2x; F(4,3): two passes of two rows, each over
# the 30 of 36 frequencies its At rows do not zero: 4 * 30 / 36).
MMA_ROW_FOLD = {2: 2, 4: 4 * 30 / 36}
# Parity bars (max abs, normwise rel = max|err| / max|ref|), as in the tests.
TOL = {"f23": (1e-4, 1e-3), "f43": (1e-4, 5e-3), "f63": (1e-3, 5e-3), "bf16": (None, 1e-2)}


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic(key: str):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get(key)


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML reads only)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, index: int, period_s: float = 0.005):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001  (clocks are reported when NVML is readable)
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        try:
            self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:  # noqa: BLE001
            self.reasons |= nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self._period)

    def __enter__(self):
        if self._nv is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._nv is not None:
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self) -> dict:
        if self._nv is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workload description shared by both arms
# ---------------------------------------------------------------------------
def config_dict(layer, world: int, weak: bool = False) -> dict:
    """The workload of a line: identical for the GPU arm and the reference arm at the
    same world size (arm-specific facts live outside `config`)."""
    global_n = layer.n * world if weak else layer.n
    per_gpu = layer.n if weak else -(-layer.n // world)
    multi = len(workloads.config_layers(layer.config)) > 1
    return {
        "workload": (f"conv3x3 s1 p1 F({layer.m}x{layer.m},3x3) N={global_n} "
                     f"{layer.c_in}->{layer.c_out} {layer.h}x{layer.w} "
                     f"{'bf16' if layer.bf16 else 'fp32'} I/O{' ReLU' if layer.relu else ''} "
                     f"(config {layer.config}" + (f", layer {layer.index})" if multi else ")")),
        "global_batch": global_n, "n_per_gpu": per_gpu, "c_in": layer.c_in,
        "c_out": layer.c_out, "h": layer.h, "w": layer.w, "m": layer.m,
        "parallelism": (f"dp{world}: " + ("every rank the whole batch" if weak else
                                          "batch split into contiguous shards") +
                        ", replicated U, no collective on the data path"),
    }


def tol_kind(layer) -> str:
    return "bf16" if layer.bf16 else {2: "f23", 4: "f43", 6: "f63"}[layer.m]


# ---------------------------------------------------------------------------
# CPU leg: the reference's own kernel (or the C restatement) on the host cores
# ---------------------------------------------------------------------------
def cpu_time_layer(layer, n_images: int, reps: int = 3):
    """Median seconds of `reps` runs of the CPU reference over n_images images.
    F(2,3): the reference's fused_winograd_f23 compiled from source, driven per
    tile by oracle/ref_layer.c; F(4,3): the C restatement of run_fused."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    g, bias = workloads.make_weights(layer)
    x = workloads.make_input(layer, n_images)
    td = layer.m + 2
    U = oracle.weight_transform(g, td)
    use_ref = layer.m == 2 and oracle.ref_available()
    # every core this process may run on (torchrun exports OMP_NUM_THREADS=1)
    nthreads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()

    def run(xx):
        if use_ref:
            return oracle.ref_conv_layer_f23(xx, U, bias, layer.relu, nthreads)
        return oracle.conv_layer(xx, U, bias, td, layer.relu, nthreads)

    run(x[:1])  # warm-up
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        run(x)
        times.append(time.perf_counter() - t0)
    kind = "reference" if use_ref else "port"
    cores = oracle.ref().refl_max_threads() if use_ref else oracle.max_threads()
    return statistics.median(times), kind, int(cores)


def cpu_baseline(layer, budget_s: float = 12.0) -> dict:
    t1, _, _ = cpu_time_layer(layer, 1, reps=1)
    n = int(max(1, min(layer.n, budget_s / 3.0 / max(t1, 1e-6))))
    t, kind, cores = cpu_time_layer(layer, n, reps=3)
    flops = layer.with_n(n).conv_flops()
    return {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": kind,
            "sample": f"{n} of {layer.n} images of the workload, median of 3 after 1 warm-up; "
                      f"{t * 1e3:.1f} ms per sample ({t / n * 1e6:.0f} us/image)",
            "us_per_layer": t / n * layer.n * 1e6}


def run_reference(args, layer, rank: int, world: int) -> None:
    """The reference arm: rank 0 alone times the reference's CPU kernel on this host's
    cores over a bounded sample of the whole workload (the global batch); other ranks
    exit without work."""
    if rank != 0:
        return
    steps, warm = args.steps, args.warmup
    t1, _, _ = cpu_time_layer(layer, 1, reps=1)
    # each step: a bounded sample of the workload (whole run ~ a few minutes)
    budget = 150.0 / max(1, steps + warm)
    n = int(max(1, min(layer.n, budget / max(t1, 1e-6))))
    t, kind, cores = cpu_time_layer(layer, n, reps=max(1, steps))
    flops = layer.with_n(n).conv_flops()
    value = flops / t / 1e12
    global_n = layer.n * world if args.weak else layer.n
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": t / n * global_n * 1e3,
        "higher_is_better": True, "scaling": "weak" if args.weak else "strong",
        "vs_baseline": None, "dtype": "bf16" if layer.bf16 else "f32", "data": "synthetic",
        "impl": "reference",
        "config": config_dict(layer, world, args.weak),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": kind,
                         "sample": f"{n} of {global_n} images per step, median of {steps}; "
                                   "rank 0 alone on this host's cores (one host whatever "
                                   "the number of GPUs)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# roofline of one layer's kernel
# ---------------------------------------------------------------------------
def roofline(choice, t_ms: float, peaks: dict, peak_src: str, traffic_key: str | None) -> dict:
    """Bound per layer: t_bound = max(alg_bytes / HBM, gemm_flops / compute peak), with the
    algorithmic bytes (x + y + U + bias, each touched once) and the plain-Winograd GEMM flops
    (2 * tiles * K * C * (m+2)^2).  frac = t_bound / t_measured = achieved / peak.  The
    tensor-core kernels issue more MMA work than that (hi/lo products, stacked output rows);
    `issued_*` reports it separately."""
    import cwg

    t = t_ms * 1e-3
    tc = choice.path == cwg.PATH_TC
    t_hbm = choice.alg_bytes / (peaks["hbm_gbs"] * 1e9)
    comp_peak = peaks["bf16_tflops"] if tc else FFMA_TFLOPS
    t_comp = choice.gemm_flops / (comp_peak * 1e12)
    src = f"{peak_src} (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback"
    if t_comp > t_hbm:
        roof = {"bound": "tensor" if tc else "ffma", "achieved": choice.gemm_flops / t / 1e12,
                "peak": comp_peak, "unit": "TFLOP/s",
                "peak_source": src if tc else "nominal fp32 FFMA (148 SMs x 128 x 2 x 1.965 GHz)"}
    else:
        roof = {"bound": "hbm", "achieved": choice.alg_bytes / t / 1e9, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "peak_source": src}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = load_traffic(traffic_key) if traffic_key else None
    roof["t_bound_us"] = max(t_hbm, t_comp) * 1e6
    roof["alg_bytes_per_launch"] = choice.alg_bytes
    roof["gemm_flops_per_launch"] = choice.gemm_flops
    if tc:
        products = max(choice.mma_products, 1)
        issued = choice.gemm_flops * products * MMA_ROW_FOLD.get(choice.m, 1)
        roof["mma_products"] = products
        roof["mma_row_fold"] = MMA_ROW_FOLD.get(choice.m, 1)
        roof["issued_mma_flops_per_launch"] = issued
        roof["issued_tflops"] = issued / t / 1e12
        roof["issued_frac"] = roof["issued_tflops"] / peaks["bf16_tflops"]
    return roof


def plan_dict(choice, flags: int) -> dict:
    import cwg

    tc = choice.path == cwg.PATH_TC
    if tc:
        gemm = {3: "bf16x3 split (fp32 parity)", 2: "fp16 x2 (V split into hi + lo)",
                1: "bf16"}.get(choice.mma_products, "?")
    else:
        gemm = "fp32 FFMA"
    return {"path": choice.path_name, "gemm": gemm, "ctas": choice.ctas,
            "ctas_launched": choice.ctas_launched, "order": choice.order_name,
            "tiles_per_cta": choice.tiles_per_cta, "cout_per_cta": choice.cout_per_cta,
            "flags": flags}


# ---------------------------------------------------------------------------
# timing and verification helpers (shared by every workload)
# ---------------------------------------------------------------------------
def sync_all(rk, dev) -> None:
    import torch

    ranks.barrier(rk)
    torch.cuda.synchronize(dev)


def timed_loop(step, steps: int, min_time_s: float, rk, dev, stream, sample_clocks: bool):
    """Times `steps` calls of step(i), repeated until the region lasts >= min_time_s (the
    repeat count is the same on every rank).  CUDA events on the launching stream, a
    barrier + synchronize on both sides.  Returns (ms per step, max over ranks), repeats,
    libcwg launches in the region, clock summary."""
    import torch

    import cwg

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync_all(rk, dev)
    e0.record(stream)
    for i in range(steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    est = ranks.max_over_ranks(e0.elapsed_time(e1) * 1e-3, rk, dev)
    reps = max(1, int(math.ceil(min_time_s / max(est, 1e-9))))
    sync_all(rk, dev)
    launches0 = cwg.launch_count()
    sampler = ClockSampler(torch.cuda.current_device()) if sample_clocks else None
    if sampler:
        sampler.__enter__()
    e0.record(stream)
    for r in range(reps):
        for i in range(steps):
            step(r * steps + i)
    e1.record(stream)
    sync_all(rk, dev)
    if sampler:
        sampler.__exit__(None, None, None)
    launches = cwg.launch_count() - launches0
    t_ms = e0.elapsed_time(e1) / (steps * reps)
    return ranks.max_over_ranks(t_ms, rk, dev), reps, int(launches), \
        (sampler.summary() if sampler else None)


def oracle_layer(layer, x, g, bias):
    """CPU reference output of a layer on images x (n, C, H, W): (y as float64, oracle name).
    fp32 F(2,3): the reference's own C kernel (else its restatement); fp32 F(4,3)/F(6,3):
    the C restatement of run_fused; bf16: fp64 direct convolution of the bf16 values."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    x = np.ascontiguousarray(x, np.float32)
    if layer.bf16:
        return oracle.direct_conv_f64(x, g, bias, layer.relu), "fp64 direct convolution"
    U = oracle.weight_transform(g, layer.m + 2)
    if layer.m == 2 and oracle.ref_available():
        return (oracle.ref_conv_layer_f23(x, U, bias, layer.relu).astype(np.float64),
                "reference fused_winograd.c")
    return (oracle.conv_layer(x, U, bias, layer.m + 2, layer.relu).astype(np.float64),
            "C restatement of run_fused")


def gather_samples(y, first: int, cnt: int, rk, dev):
    """The first and last output image of this rank's shard, gathered to every rank (NCCL
    over CUDA tensors).  Returns [(rank, global image index, image (K, H, W) fp32 numpy)] on
    rank 0, None elsewhere."""
    import torch

    loc = [0, max(cnt - 1, 0)]
    t = y[loc].float().contiguous()
    idx = torch.tensor([first + i for i in loc], dtype=torch.int64, device=t.device)
    ts = ranks.gather_tensor(t, rk)
    ids = ranks.gather_tensor(idx, rk)
    if rk.rank != 0:
        return None
    out = []
    for r, (tt, ii) in enumerate(zip(ts, ids)):
        a, i = tt.cpu().numpy(), ii.cpu().tolist()
        for j in range(len(loc)):
            out.append((r, int(i[j]), a[j]))
    return out


def check_samples(layer, samples, x_of, g, bias) -> dict:
    """Compares gathered output images with the CPU oracle: per rank, max abs error and
    normwise relative error (max|err| / max|ref|) over its sampled images, against the
    parity bars of the layer's kind.  x_of(global index) -> the input image (C, H, W)."""
    kind = tol_kind(layer)
    atol, rtol = TOL[kind]
    per, name = {}, None
    for r, i, img in samples:
        ref, name = oracle_layer(layer, x_of(i)[None], g, bias)
        ref = ref[0]
        err = float(np.abs(img.astype(np.float64) - ref).max())
        scale = float(np.abs(ref).max())
        d = per.setdefault(r, {"rank": r, "images": [], "max_abs_err": 0.0,
                               "normwise_rel_err": 0.0, "finite": True})
        if i not in d["images"]:
            d["images"].append(i)
        d["max_abs_err"] = max(d["max_abs_err"], err)
        d["normwise_rel_err"] = max(d["normwise_rel_err"], err / scale if scale > 0 else 0.0)
        d["finite"] = d["finite"] and bool(np.isfinite(img).all())
    rows = [per[r] for r in sorted(per)]
    ok = all(d["finite"] and (atol is None or d["max_abs_err"] <= atol) and
             d["normwise_rel_err"] <= rtol for d in rows)
    return {"oracle": name, "tolerance": {"max_abs": atol, "normwise_rel": rtol},
            "per_rank": rows, "ok": ok}


def l2_flusher(dev):
    """A function that overwrites a buffer larger than L2 (flushes it) on a stream."""
    import torch

    buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    def flush(stream):
        with torch.cuda.stream(stream):
            buf.fill_(0.0)
    return flush


# ---------------------------------------------------------------------------
# one layer workload
# ---------------------------------------------------------------------------
def bench_layer(layer, args, rk, dev, peaks, peak_src, *, steps: int, warmup: int,
                extra_flags: int = 0, e2e: bool = True, cpu: bool = True,
                sample_clocks: bool = True) -> dict:
    import torch

    import cwg

    world = rk.world
    global_n = layer.n * world if args.weak else layer.n
    if args.weak:
        first, cnt = rk.rank * layer.n, layer.n
    else:
        if global_n < world:
            raise SystemExit(f"{global_n} images cannot be split across {world} ranks")
        first, cnt = ranks.shard(global_n, rk)
    flags = (cwg.RELU if layer.relu else 0) | (cwg.BF16 if layer.bf16 else 0) | extra_flags
    c, k, h, w, m = layer.c_in, layer.c_out, layer.h, layer.w, layer.m
    nonfused = args.nonfused and layer.config == args.config
    if nonfused:
        if layer.bf16:
            raise SystemExit("--nonfused: the ablation is fp32 only")
        flags |= cwg.FORCE_FFMA  # U in the CUDA-core layout, which the ablation reads
    choice = cwg.select(cnt, c, k, h, w, m, flags)
    dt = torch.bfloat16 if layer.bf16 else torch.float32
    esz = 2 if layer.bf16 else 4
    stream = torch.cuda.current_stream(dev)

    # inputs: this rank's shard of the global batch, resident in HBM
    g, bias = workloads.make_weights(layer)
    x_host = workloads.make_input(layer, cnt, first_image=first)
    x0 = torch.from_numpy(x_host).to(dev).to(dt)
    U = torch.empty(cwg.weight_bytes(c, k, m, flags), dtype=torch.uint8, device=dev)
    cwg.weight_transform(torch.from_numpy(g).to(dev), U, c, k, m, flags)
    b_d = torch.from_numpy(bias).to(dev)
    xbytes, ybytes = cnt * c * h * w * esz, cnt * k * h * w * esz
    # rotate buffer sets so that no step finds its operands in L2
    nsets = max(2, int(np.ceil(2 * L2_BYTES / (xbytes + ybytes))) + 1)
    xs = [x0] + [x0.clone() for _ in range(nsets - 1)]
    ys = [torch.empty((cnt, k, h, w), dtype=dt, device=dev) for _ in range(nsets)]

    if nonfused:
        nf_b = cwg.nonfused_workspace_bytes(cnt, c, k, h, w, m)
        nf_ws = torch.empty(nf_b, dtype=torch.uint8, device=dev)

        def step(i):
            cwg.conv3x3_nonfused(xs[i % nsets], U, b_d, ys[i % nsets], nf_ws, nf_b, cnt, c, k,
                                 h, w, m, flags & cwg.RELU, stream)
    else:
        def step(i):
            cwg.conv3x3_fused(xs[i % nsets], U, b_d, ys[i % nsets], cnt, c, k, h, w, m, flags,
                              stream)

    for i in range(warmup):
        step(i)
    cwg.device_status(stream)
    t_max, reps, launches, clocks = timed_loop(step, steps, args.min_time, rk, dev, stream,
                                               sample_clocks)
    cwg.device_status(stream)

    # ---- end to end through the host-buffer entry point ----
    te_ms = None
    if e2e and not nonfused:
        xh = (torch.from_numpy(x_host).to(dt) if layer.bf16 else
              torch.from_numpy(x_host)).pin_memory()
        yh = torch.empty((cnt, k, h, w), dtype=dt).pin_memory()
        ws_b = cwg.host_workspace_bytes(cnt, c, k, h, w, flags)
        ws = torch.empty(ws_b, dtype=torch.uint8, device=dev)

        def e2e_step(_i):
            cwg.conv3x3_fused_host(int(xh.data_ptr()), U, b_d, int(yh.data_ptr()), ws, ws_b,
                                   cnt, c, k, h, w, m, flags, stream)

        for _ in range(min(warmup, 3)):
            e2e_step(0)
        te_ms, _, _, _ = timed_loop(e2e_step, max(3, min(steps, 10)),
                                           args.min_time / 4, rk, dev, stream, False)
        del ws

    # ---- verification: sampled output images of every rank against the oracle ----
    verify = None
    if not args.no_verify:
        samples = gather_samples(ys[0], first, cnt, rk, dev)
        if rk.rank == 0:
            verify = check_samples(layer, samples,
                                   lambda i: workloads.make_input(layer, 1, first_image=i)[0],
                                   g, bias)

    res = None
    if rk.rank == 0:
        flops_total = layer.with_n(global_n).conv_flops()
        res = {
            "value": flops_total / (t_max * 1e-3) / 1e12, "ms_per_step": t_max,
            "us_per_layer": t_max * 1e3, "timed_repeats": reps,
            "timed_steps_total": steps * reps, "gpu_launches": launches,
            "plan": plan_dict(choice, flags) if not nonfused else
            {"path": "nonfused (input pass, per-frequency GEMM, output pass)", "flags": flags},
            "roofline": roofline(choice, t_max, peaks, peak_src,
                                 f"cfg{layer.config}.{layer.index}:{choice.path_name}")
            if not nonfused else None,
            "e2e": None if te_ms is None else {
                "value": flops_total / (te_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": xbytes, "d2h_bytes_per_step": ybytes,
                "us_per_layer": te_ms * 1e3,
                "note": "per rank: H2D of its shard's x from pinned memory, kernel, D2H of y"},
            "clocks": clocks,
            "verify": verify,
            "l2": f"{nsets} rotating x/y buffer sets ({nsets * (xbytes + ybytes) / 2**20:.0f} MiB)"
                  " > 126 MiB L2",
        }
        if world == 1 and cpu and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(layer, args.cpu_budget)
    del xs, ys
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# the ResNet-18-shaped stride-1 stack (13 layers, chained within each stage)
# ---------------------------------------------------------------------------
def bench_stack(args, rk, dev, peaks, peak_src, reps: int = 5) -> dict | None:
    """Per-layer device time (each layer alone, L2 flushed before it) and the stack's
    end-to-end device time (the 13 launches replayed as one CUDA graph, L2 flushed
    between replays), batch split across ranks, max over ranks."""
    import torch

    import cwg

    layers = workloads.config_layers(4)
    world = rk.world
    global_n = layers[0].n
    first, cnt = ranks.shard(global_n, rk)
    stream = torch.cuda.current_stream(dev)
    flush = l2_flusher(dev)
    plan, prev, x = [], None, None
    for lay in layers:
        flags = cwg.RELU
        g, bias = workloads.make_weights(lay)
        U = torch.empty(cwg.weight_bytes(lay.c_in, lay.c_out, lay.m, flags), dtype=torch.uint8,
                        device=dev)
        cwg.weight_transform(torch.from_numpy(g).to(dev), U, lay.c_in, lay.c_out, lay.m, flags)
        fresh = prev is None or (prev.c_out, prev.h) != (lay.c_in, lay.h)
        if fresh:
            x = torch.from_numpy(workloads.make_input(lay, cnt, first_image=first)).to(dev)
        y = torch.empty((cnt, lay.c_out, lay.h, lay.w), dtype=torch.float32, device=dev)
        plan.append((lay, flags, U, torch.from_numpy(bias).to(dev), x, y, g, bias, fresh))
        x, prev = y, lay

    def launch(i, s):
        lay, flags, U, b, xi, yi = plan[i][:6]
        cwg.conv3x3_fused(xi, U, b, yi, cnt, lay.c_in, lay.c_out, lay.h, lay.w, lay.m, flags, s)

    for i in range(len(plan)):  # eager pass: kernel attributes set before capture
        launch(i, stream)
    cwg.device_status(stream)
    # per layer, cold L2
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in plan] for _ in range(reps)]
    sync_all(rk, dev)
    for r in range(reps):
        for i in range(len(plan)):
            flush(stream)
            ev[r][i][0].record(stream)
            launch(i, stream)
            ev[r][i][1].record(stream)
    sync_all(rk, dev)
    per_layer = [statistics.median(ev[r][i][0].elapsed_time(ev[r][i][1]) for r in range(reps))
                 for i in range(len(plan))]
    per_layer = [ranks.max_over_ranks(t, rk, dev) for t in per_layer]
    # the whole stack as one CUDA graph
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cs = torch.cuda.current_stream(dev)
        for i in range(len(plan)):
            launch(i, cs)
    graph.replay()
    sync_all(rk, dev)
    gev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(reps)]
    for r in range(reps):
        flush(stream)
        gev[r][0].record(stream)
        graph.replay()
        gev[r][1].record(stream)
    sync_all(rk, dev)
    stack_ms = ranks.max_over_ranks(statistics.median(a.elapsed_time(b) for a, b in gev), rk, dev)
    cwg.device_status(stream)
    del graph

    # verification: image 0 and the last image of every rank, layer by layer; a chained
    # layer's oracle input is the gathered GPU output of the layer before it
    verify = None
    if not args.no_verify:
        checks, prev_out = [], None
        for i, (lay, _, _, _, _, y, g, bias, fresh) in enumerate(plan):
            samples = gather_samples(y, first, cnt, rk, dev)
            if rk.rank != 0:
                continue
            if fresh:
                def x_of(gi, lay=lay):
                    return workloads.make_input(lay, 1, first_image=gi)[0]
            else:
                src = {(r, gi): img for r, gi, img in prev_out}
                order = {gi: r for r, gi, _ in samples}

                def x_of(gi, src=src, order=order):
                    return src[(order[gi], gi)]
            v = check_samples(lay, samples, x_of, g, bias)
            checks.append({"layer": i, "ok": v["ok"],
                           "max_abs_err": max(d["max_abs_err"] for d in v["per_rank"]),
                           "normwise_rel_err": max(d["normwise_rel_err"] for d in v["per_rank"])})
            prev_out = samples
        if rk.rank == 0:
            verify = {"oracle": "reference fused_winograd.c on the exact input each layer got",
                      "tolerance": {"max_abs": TOL["f23"][0], "normwise_rel": TOL["f23"][1]},
                      "images": "first and last of every rank's shard", "layers": checks,
                      "ok": all(c["ok"] for c in checks)}
    if rk.rank != 0:
        return None
    flops = sum(lay.with_n(global_n).conv_flops() for lay in layers)
    rows, stages = [], {}
    for i, (lay, flags, *_rest) in enumerate(plan):
        ch = cwg.select(cnt, lay.c_in, lay.c_out, lay.h, lay.w, lay.m, flags)
        roof = roofline(ch, per_layer[i], peaks, peak_src, None)
        rows.append({"layer": i, "c": lay.c_in, "hw": lay.h, "path": ch.path_name,
                     "us": round(per_layer[i] * 1e3, 2),
                     "tflops": round(lay.with_n(global_n).conv_flops() / per_layer[i] / 1e9, 1),
                     "bound": roof["bound"], "frac": round(roof["frac"], 4),
                     "issued_frac": round(roof.get("issued_frac", 0.0), 4)})
        st = stages.setdefault(lay.c_in, {"stage_c": lay.c_in, "hw": lay.h, "layers": 0, "us": 0.0,
                                          "t_bound_us": 0.0})
        st["layers"] += 1
        st["us"] += per_layer[i] * 1e3
        st["t_bound_us"] += roof["t_bound_us"]
    for st in stages.values():
        st["frac"] = st["t_bound_us"] / st["us"]
        st["us"] = round(st["us"], 2)
        st["t_bound_us"] = round(st["t_bound_us"], 2)
    return {
        "config": {"workload": f"ResNet-18 stride-1 3x3 stack (config 4): N={global_n}, "
                               "4x64@56, 3x128@28, 3x256@14, 3x512@7, F(2x2,3x3), fp32, "
                               "bias (BN folded) + ReLU, chained within each stage",
                   "global_batch": global_n, "n_per_gpu": -(-global_n // world),
                   "parallelism": f"dp{world}: batch split, replicated U"},
        "value": flops / (stack_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
        "stack_us": stack_ms * 1e3, "sum_of_layers_us": sum(per_layer) * 1e3,
        "timing": "layers[].us: each layer alone after an L2 flush, median of "
                  f"{reps}; stack_us: the 13 launches as one CUDA graph after an L2 flush, "
                  f"median of {reps}; max over ranks",
        "layers": rows, "stages": list(stages.values()), "verify": verify,
    }


# ---------------------------------------------------------------------------
# model shape feed (1 GPU)
# ---------------------------------------------------------------------------
def run_model(args) -> None:
    """The model's stride-1 3x3 convs (the shapes benchmarks/e2e_benchmark.py:91-137 of the
    reference extracts) as one chained stack per step; per-layer and total device time."""
    import torch

    import cwg
    import model_shapes

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = args.n if args.n > 0 else 1
    for _ in range(args.warmup):
        model_shapes.run_stack(args.model, n, dev, args.flags)
    torch.cuda.synchronize()
    runs = [model_shapes.run_stack(args.model, n, dev, args.flags)[0] for _ in range(args.steps)]
    per_layer = [statistics.median(r[i] for r in runs) for i in range(len(runs[0]))]
    # the whole stack as one CUDA graph: device time without per-layer host gaps
    replay, _ = model_shapes.capture_stack(args.model, n, dev, args.flags)
    for _ in range(args.warmup):
        replay()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(args.steps):
        replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    cwg.device_status()
    total_ms = e0.elapsed_time(e1) / args.steps
    layers = model_shapes.stride1_layers(args.model)
    flops = sum(2.0 * n * s.c_out * s.c_in * s.h * s.w * 9 for s in layers)
    paths = [cwg.select(n, s.c_in, s.c_out, s.h, s.w, 0, args.flags | cwg.RELU).path_name
             for s in layers]
    print(json.dumps({
        "metric": METRIC, "value": flops / (total_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms,
        "us_per_layer": total_ms * 1e3 / len(layers), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16" if args.flags & cwg.BF16 else "f32",
        "data": "synthetic (seeded U(-1,1) inputs, Kaiming-normal weights, bias U(-0.1,0.1))",
        "config": {"workload": f"{args.model} stride-1 3x3 convs at its standard input, "
                               f"{len(layers)} layers chained, N={n}, bias+ReLU",
                   "timing": "ms_per_step: the stack replayed as one CUDA graph; layers[].us: "
                             "each layer timed alone by events around its eager call",
                   "eager_ms": round(sum(per_layer), 3),
                   "layers": [{"c_in": s.c_in, "c_out": s.c_out, "hw": s.h, "path": p,
                               "us": round(t * 1e3, 1)}
                              for s, p, t in zip(layers, paths, per_layer)]},
        "e2e": None,
    }))


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------
def compact(layer, world, weak, r: dict) -> dict:
    """A nested workload entry: its own config, value and measurements."""
    out = {"config": config_dict(layer, world, weak), "value": r["value"], "unit": "TFLOP/s"}
    out.update({k: v for k, v in r.items() if k != "value"})
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--layer", type=int, default=0)
    ap.add_argument("--impl", default="cwg", choices=["cwg", "reference"])
    ap.add_argument("--flags", type=lambda s: int(s, 0), default=0,
                    help="extra CWG_* flags (ablations, e.g. 0x10 = FFMA path)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    ap.add_argument("--n", type=int, default=0,
                    help="batch instead of the workload's own (small profiling cases)")
    ap.add_argument("--weak", action="store_true",
                    help="every rank convolves the whole batch (weak scaling) instead of a shard")
    ap.add_argument("--min-time", type=float, default=0.5,
                    help="the timed region repeats the K-step block until it lasts this long")
    ap.add_argument("--no-verify", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="headline workload only (skip the config-5 layer and config-4 stack)")
    ap.add_argument("--nonfused", action="store_true",
                    help="time the non-fused ablation (3 passes over HBM, fp32) instead")
    ap.add_argument("--model", default="",
                    choices=["", "resnet18", "resnet34", "vgg16", "alexnet"],
                    help="time the model's stride-1 3x3 convs as a chained stack (1 GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.model:
        run_model(args)
        return

    rk = ranks.from_env()
    rank, world, local = rk.rank, rk.world, rk.local
    layer = workloads.config_layers(args.config)[args.layer]
    if args.n > 0:
        layer = layer.with_n(args.n)

    if args.impl == "reference":
        run_reference(args, layer, rank, world)
        return

    import torch

    import cwg  # noqa: F401

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ranks.init(rk, "nccl", device=dev)
    peaks, peak_src = load_peaks()

    r = bench_layer(layer, args, rk, dev, peaks, peak_src, steps=args.steps,
                    warmup=args.warmup, extra_flags=args.flags)
    extra = []
    default_run = (args.config == 3 and args.n == 0 and not args.nonfused and not args.flags
                   and not args.weak)
    if default_run and not args.no_extra:
        l5 = workloads.config_layers(5)[0]
        r5 = bench_layer(l5, args, rk, dev, peaks, peak_src, steps=5, warmup=3,
                         cpu=True, sample_clocks=False)
        if rank == 0:
            extra.append(compact(l5, world, False, r5))
        r4 = bench_stack(args, rk, dev, peaks, peak_src)
        if rank == 0:
            extra.append(r4)

    if rank == 0:
        line = {
            "metric": METRIC, "value": r["value"], "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "us_per_layer": r["us_per_layer"], "timed_repeats": r["timed_repeats"],
            "timed_steps_total": r["timed_steps_total"], "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
            "dtype": "bf16" if layer.bf16 else "f32",
            "data": "synthetic (seeded U(-1,1) inputs, Kaiming-normal weights)",
            "config": config_dict(layer, world, args.weak),
            "plan": r["plan"], "l2": r["l2"],
            "roofline": r["roofline"],
            "e2e": r["e2e"],
            "gpu_launches": r["gpu_launches"],
            "clocks": r["clocks"],
            "verify": r["verify"],
        }
        if "cpu_baseline" in r:
            line["cpu_baseline"] = r["cpu_baseline"]
        if extra:
            line["workloads"] = extra
        print(json.dumps(line), flush=True)

    ranks.finish(rk)


if __name__ == "__main__":
    main()
