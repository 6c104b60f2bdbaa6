#!/usr/bin/env python3
"""Benchmark of the fused Winograd 3x3 convolution on B200.

Default workload (one "step" = one layer over one batch): 3x3 conv, stride 1,
pad 1, F(2x2,3x3), fp32 NCHW in and out, N=64 images per GPU, 128->128
channels, 56x56, ReLU; x ~ U(-1,1), Kaiming-normal weights, zero bias.  With
--gpus N every rank convolves its own 64 images (weak scaling; global batch
64*N) with replicated transformed weights: no collective on the data path.

Prints one JSON line (rank 0).  `value` = effective conv TFLOP/s of the whole
job (2*N*K*C*H*W*9 / max-over-ranks device time); `ms_per_step` is the time
of one layer (us/layer / 1000).  `e2e` is the same metric through the public
host-buffer call (cwg_conv3x3_fused_host: H2D of x, kernel, D2H of y, sync).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1..5 --layer i]
  python bench.py --impl reference ...   # the reference's own CPU kernel
  python bench.py --model resnet18|resnet34|vgg16 [--n N]   # chained stride-1 3x3 stack
"""
from __future__ import annotations

import argparse
import json
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
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": t / n * layer.n * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": config_dict(layer, world, "cpu"),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": kind,
                         "sample": f"{n} of {layer.n} images per step, median of {steps}"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(layer, world: int, path: str, extra: dict | None = None) -> dict:
    d = {
        "workload": (f"conv3x3 s1 p1 F({layer.m}x{layer.m},3x3) N={layer.n}/GPU "
                     f"{layer.c_in}->{layer.c_out} {layer.h}x{layer.w} "
                     f"{'bf16' if layer.bf16 else 'fp32'} I/O{' ReLU' if layer.relu else ''} "
                     f"(config {layer.config}" + (f", layer {layer.index})" if
                                                  len(workloads.config_layers(layer.config)) > 1
                                                  else ")")),
        "n_per_gpu": layer.n, "global_batch": layer.n * world, "c_in": layer.c_in,
        "c_out": layer.c_out, "h": layer.h, "w": layer.w, "m": layer.m,
        "parallelism": f"dp{world} (batch split, replicated U, no collective)",
        "path": path,
    }
    if extra:
        d.update(extra)
    return d


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
        "config": {"workload": f"{args.model} stride-1 3x3 convs at 224x224 input, "
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
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--layer", type=int, default=0)
    ap.add_argument("--impl", default="cwg", choices=["cwg", "reference"])
    ap.add_argument("--flags", type=lambda s: int(s, 0), default=0,
                    help="extra CWG_* flags (ablations, e.g. 0x10 = FFMA path)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--n", type=int, default=0,
                    help="images per GPU instead of the workload's own (small profiling cases)")
    ap.add_argument("--nonfused", action="store_true",
                    help="time the non-fused ablation (3 passes over HBM, fp32) instead")
    ap.add_argument("--model", default="", choices=["", "resnet18", "resnet34", "vgg16"],
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

    import cwg

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ranks.init(rk, "nccl", device=dev)

    flags = (cwg.RELU if layer.relu else 0) | (cwg.BF16 if layer.bf16 else 0) | args.flags
    n, c, k, h, w, m = layer.n, layer.c_in, layer.c_out, layer.h, layer.w, layer.m
    if args.nonfused:
        if layer.bf16:
            raise SystemExit("--nonfused: the ablation is fp32 only")
        flags |= cwg.FORCE_FFMA  # U in the CUDA-core layout, which the ablation reads
    choice = cwg.select(n, c, k, h, w, m, flags)
    dt = torch.bfloat16 if layer.bf16 else torch.float32
    esz = 2 if layer.bf16 else 4

    # inputs: this rank's shard of the global batch, resident in HBM
    g, bias = workloads.make_weights(layer)
    first, _ = ranks.shard(n * world, rk)  # weak scaling: n images per rank
    x_host = workloads.make_input(layer, n, first_image=first)
    x0 = torch.from_numpy(x_host).to(dev).to(dt)
    U = torch.empty(cwg.weight_bytes(c, k, m, flags), dtype=torch.uint8, device=dev)
    cwg.weight_transform(torch.from_numpy(g).to(dev), U, c, k, m, flags)
    b_d = torch.from_numpy(bias).to(dev)
    xbytes, ybytes = n * c * h * w * esz, n * k * h * w * esz
    # rotate buffer sets so that no step finds its operands in L2
    nsets = max(2, int(np.ceil(2 * L2_BYTES / (xbytes + ybytes))) + 1)
    xs = [x0] + [x0.clone() for _ in range(nsets - 1)]
    ys = [torch.empty((n, k, h, w), dtype=dt, device=dev) for _ in range(nsets)]
    stream = torch.cuda.current_stream(dev)

    if args.nonfused:
        nf_b = cwg.nonfused_workspace_bytes(n, c, k, h, w, m)
        nf_ws = torch.empty(nf_b, dtype=torch.uint8, device=dev)

        def step(i):
            cwg.conv3x3_nonfused(xs[i % nsets], U, b_d, ys[i % nsets], nf_ws, nf_b, n, c, k, h,
                                 w, m, flags & cwg.RELU, stream)
    else:
        def step(i):
            cwg.conv3x3_fused(xs[i % nsets], U, b_d, ys[i % nsets], n, c, k, h, w, m, flags,
                              stream)

    for i in range(args.warmup):
        step(i)
    cwg.device_status(stream)

    def barrier():
        ranks.barrier(rk)
        torch.cuda.synchronize(dev)

    # ---- timed region: K steps, events on the launching stream ----
    barrier()
    launches0 = cwg.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        barrier()
    launches = cwg.launch_count() - launches0
    cwg.device_status(stream)
    t_ms = ev0.elapsed_time(ev1) / args.steps
    t_max = ranks.max_over_ranks(t_ms, rk, dev)

    # ---- end to end through the host-buffer entry point (not for the ablation) ----
    te_ms = None
    if not args.nonfused:
        xh = torch.from_numpy(x_host).to(dt).pin_memory() if layer.bf16 else \
            torch.from_numpy(x_host).pin_memory()
        yh = torch.empty((n, k, h, w), dtype=dt).pin_memory()
        ws_b = cwg.host_workspace_bytes(n, c, k, h, w, flags)
        ws = torch.empty(ws_b, dtype=torch.uint8, device=dev)

        def e2e_step():
            cwg.conv3x3_fused_host(int(xh.data_ptr()), U, b_d, int(yh.data_ptr()), ws, ws_b,
                                   n, c, k, h, w, m, flags, stream)

        for _ in range(args.warmup):
            e2e_step()
        e2e_steps = max(3, min(args.steps, 20))
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        te_ms = ranks.max_over_ranks(e0.elapsed_time(e1) / e2e_steps, rk, dev)

    # ---- verification checksum of every rank's output (outside timing) ----
    checksums = ranks.gather_floats(float(ys[0].double().sum().item()), rk, dev)

    if rank == 0:
        peaks, peak_src = load_peaks()
        flops_total = layer.conv_flops() * world
        value = flops_total / (t_max * 1e-3) / 1e12
        # roofline of the dominant (conv) kernel, per launch on this GPU
        products = max(choice.mma_products, 1)
        t_hbm = choice.alg_bytes / (peaks["hbm_gbs"] * 1e9)
        mma_flops = choice.gemm_flops * products
        t_tc = mma_flops / (peaks["bf16_tflops"] * 1e12)
        if choice.path == cwg.PATH_TC and t_tc > t_hbm:
            roof = {"bound": "tensor", "achieved": mma_flops / (t_ms * 1e-3) / 1e12,
                    "peak": peaks["bf16_tflops"], "unit": "TFLOP/s"}
        else:
            roof = {"bound": "hbm", "achieved": choice.alg_bytes / (t_ms * 1e-3) / 1e9,
                    "peak": peaks["hbm_gbs"], "unit": "GB/s"}
        roof["frac"] = roof["achieved"] / roof["peak"]
        roof["traffic"] = load_traffic(f"cfg{layer.config}.{layer.index}:{choice.path_name}")
        roof["peak_source"] = f"{peak_src} (MEASURED_PEAKS.json)" if peak_src == "measured" \
            else "fallback"
        roof["alg_bytes_per_launch"] = choice.alg_bytes
        roof["gemm_flops_per_launch"] = choice.gemm_flops
        roof["mma_products"] = products
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_max,
            "us_per_layer": t_max * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if layer.bf16 else "f32",
            "data": "synthetic (seeded U(-1,1) inputs, Kaiming-normal weights)",
            "config": config_dict(layer, world, "nonfused (input pass, cuBLAS SGEMM per "
                                  "frequency, output pass)" if args.nonfused else
                                  choice.path_name, {
                "gemm": "fp32 cuBLAS SGEMM" if args.nonfused else
                        ("bf16x3 split (fp32 parity)" if products == 3 else
                         ("bf16" if (flags & (cwg.BF16 | cwg.TC_SINGLE)) and
                          choice.path == cwg.PATH_TC else "fp32 FFMA")),
                "l2": f"{nsets} rotating x/y buffer sets ({nsets * (xbytes + ybytes) / 2**20:.0f}"
                      " MiB) > 126 MiB L2",
                "ctas": choice.ctas, "ctas_launched": choice.ctas_launched,
                "order": choice.order_name, "tiles_per_cta": choice.tiles_per_cta,
                "cout_per_cta": choice.cout_per_cta}),
            "roofline": roof,
            "e2e": None if te_ms is None else {
                "value": flops_total / (te_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": xbytes, "d2h_bytes_per_step": ybytes,
                "us_per_layer": te_ms * 1e3},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "checksums": checksums,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(layer)
        print(json.dumps(line), flush=True)

    ranks.finish(rk)


if __name__ == "__main__":
    main()
