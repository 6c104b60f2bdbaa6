"""3x3 convolution shapes of the models the reference's end-to-end driver feeds, and a
chained runner that pushes their stride-1 layers through cwg_conv3x3_fused.

The reference extracts the shapes with forward hooks on torchvision alexnet, resnet18, resnet34
and vgg16 at a 1x3x224x224 input (benchmarks/e2e_benchmark.py:64, 91-137) and times each layer in a
per-layer loop (:206-270).  Here the shapes are written out from the architectures (ResNet
basic blocks with a stride-2 first conv in stages 2-4; VGG16 configuration D; AlexNet's three
3x3 convs after its 11x11 stride-4 and 5x5 layers and two max-pools, at 13x13), so the engine
needs no model library; tests/test_model_shapes.py checks them against torchvision's hooks
where torchvision is installed.  The layer ABI is stride 1, pad 1: stride-2 convs are listed
(as the reference lists them) and skipped by the runner.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ConvShape:
    c_in: int
    c_out: int
    h: int  # input height (= output height at stride 1)
    w: int
    stride: int
    padding: int = 1


def _resnet(blocks: tuple[int, int, int, int]) -> list[ConvShape]:
    out, c_prev, s = [], 64, 56  # after the 7x7 stem and the max-pool
    for stage, (width, n) in enumerate(zip((64, 128, 256, 512), blocks)):
        for b in range(n):
            stride = 2 if (stage > 0 and b == 0) else 1
            out.append(ConvShape(c_prev, width, s, s, stride))
            s //= stride
            out.append(ConvShape(width, width, s, s, 1))
            c_prev = width
    return out


def _vgg16() -> list[ConvShape]:
    out, c_prev, s = [], 3, 224
    for v in (64, 64, "M", 128, 128, "M", 256, 256, 256, "M", 512, 512, 512, "M",
              512, 512, 512, "M"):
        if v == "M":
            s //= 2
            continue
        out.append(ConvShape(c_prev, v, s, s, 1))
        c_prev = v
    return out


def _alexnet() -> list[ConvShape]:
    # 224 -> conv 11x11/4, pad 2: 55 -> max-pool 3/2: 27 -> conv 5x5: 27 -> max-pool: 13
    return [ConvShape(192, 384, 13, 13, 1), ConvShape(384, 256, 13, 13, 1),
            ConvShape(256, 256, 13, 13, 1)]


MODELS = {
    "alexnet": _alexnet,
    "resnet18": lambda: _resnet((2, 2, 2, 2)),
    "resnet34": lambda: _resnet((3, 4, 6, 3)),
    "vgg16": _vgg16,
}
# seed offsets per model (fixed, so that adding a model changes no other model's data)
_MODEL_ID = {"resnet18": 0, "resnet34": 1, "vgg16": 2, "alexnet": 3}


def conv3x3_layers(name: str) -> list[ConvShape]:
    """Every 3x3 conv of the model, in forward order (the reference's list)."""
    return MODELS[name]()


def stride1_layers(name: str) -> list[ConvShape]:
    """The layers the engine runs (stride 1, pad 1)."""
    return [s for s in conv3x3_layers(name) if s.stride == 1 and s.padding == 1]


def layer_params(name: str, index: int, s: ConvShape, bf16: bool = False):
    """Seeded Kaiming-normal weights N(0, sqrt(2/(9 C_in))) and bias U(-0.1, 0.1) (BN
    folded), as for the ResNet-18 stack of the benchmark configurations."""
    seed = 7000 + 100 * _MODEL_ID[name] + index
    rng = np.random.default_rng(seed)
    g = rng.normal(0.0, np.sqrt(2.0 / (9 * s.c_in)), (s.c_out, s.c_in, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, s.c_out).astype(np.float32)
    if bf16:
        from workloads import bf16_round
        g = bf16_round(g)
    return g, bias


def stack_input(name: str, index: int, n: int, s: ConvShape, bf16: bool = False) -> np.ndarray:
    """A fresh U(-1, 1) input for a layer that does not chain from its predecessor."""
    rng = np.random.default_rng(9000 + 100 * _MODEL_ID[name] + index)
    x = rng.uniform(-1.0, 1.0, (n, s.c_in, s.h, s.w)).astype(np.float32)
    if bf16:
        from workloads import bf16_round
        x = bf16_round(x)
    return x


def chains(prev: ConvShape | None, s: ConvShape) -> bool:
    """True when the previous stride-1 layer's output is this layer's input."""
    return prev is not None and prev.c_out == s.c_in and (prev.h, prev.w) == (s.h, s.w)


def run_stack(name: str, n: int, dev, flags: int = 0, keep=None):
    """Runs the model's stride-1 3x3 layers in order on `n` images, each layer on its
    predecessor's output where the shapes chain (bias + ReLU fused), else on a fresh input.

    Returns (per-layer device times in ms, [(layer index, shape, input, output) for the
    indices in `keep`], the prepared layers) -- inputs/outputs as device tensors."""
    import torch

    import cwg

    bf16 = bool(flags & cwg.BF16)
    dt = torch.bfloat16 if bf16 else torch.float32
    flags = flags | cwg.RELU
    layers = stride1_layers(name)
    prepared = []
    for i, s in enumerate(layers):
        g, bias = layer_params(name, i, s, bf16)
        U = torch.empty(cwg.weight_bytes(s.c_in, s.c_out, 0, flags), dtype=torch.uint8,
                        device=dev)
        cwg.weight_transform(torch.from_numpy(g).to(dev), U, s.c_in, s.c_out, 0, flags)
        prepared.append((s, U, torch.from_numpy(bias).to(dev), g, bias))
    times, kept, x, prev = [], [], None, None
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in layers]
    for i, (s, U, b_d, _, _) in enumerate(prepared):
        if not chains(prev, s):
            x = torch.from_numpy(stack_input(name, i, n, s, bf16)).to(dev).to(dt)
        y = torch.empty((n, s.c_out, s.h, s.w), dtype=dt, device=dev)
        ev[i][0].record()
        cwg.conv3x3_fused(x, U, b_d, y, n, s.c_in, s.c_out, s.h, s.w, 0, flags)
        ev[i][1].record()
        if keep is not None and i in keep:
            kept.append((i, s, x, y))
        x, prev = y, s
    cwg.device_status()
    times = [a.elapsed_time(b) for a, b in ev]
    return times, kept, prepared


def capture_stack(name: str, n: int, dev, flags: int = 0):
    """The same chained stack captured once into a CUDA graph: returns a function that
    replays every layer's launches (no per-layer host work) and the output buffer of the
    last layer.  Buffers and transformed weights are allocated up front and stay alive in
    the closure."""
    import torch

    import cwg

    bf16 = bool(flags & cwg.BF16)
    dt = torch.bfloat16 if bf16 else torch.float32
    flags = flags | cwg.RELU
    layers = stride1_layers(name)
    plan, prev, x = [], None, None
    for i, s in enumerate(layers):
        g, bias = layer_params(name, i, s, bf16)
        U = torch.empty(cwg.weight_bytes(s.c_in, s.c_out, 0, flags), dtype=torch.uint8,
                        device=dev)
        cwg.weight_transform(torch.from_numpy(g).to(dev), U, s.c_in, s.c_out, 0, flags)
        if not chains(prev, s):
            x = torch.from_numpy(stack_input(name, i, n, s, bf16)).to(dev).to(dt)
        y = torch.empty((n, s.c_out, s.h, s.w), dtype=dt, device=dev)
        plan.append((s, x, U, torch.from_numpy(bias).to(dev), y))
        x, prev = y, s

    def launch_all(stream):
        for s, xi, U, b, yi in plan:
            cwg.conv3x3_fused(xi, U, b, yi, n, s.c_in, s.c_out, s.h, s.w, 0, flags, stream)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # one eager pass sets the kernels' attributes first
        launch_all(side)
    torch.cuda.synchronize(dev)
    cwg.device_status()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launch_all(torch.cuda.current_stream(dev))
    return graph.replay, plan[-1][4]
