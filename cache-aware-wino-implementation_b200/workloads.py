"""Seeded synthetic workloads for the five benchmark configurations.

The reference measures no public dataset: its benchmarks feed random tiles
(benchmarks/jetson_main_microbench.py:53-56).  These generators produce whole
layers with the stated shapes and distributions:

  1  N=1,  32->32,  56x56, F(2,3), fp32; x~U(-1,1), g~N(0, sqrt(2/(9C))), bias 0
  2  N=1,  (C,K) in the reference's 7 microbench pairs
     (benchmarks/jetson_main_microbench.py:24-32), 56x56, F(2,3) and F(4,3),
     fp32; bias ~U(-0.1, 0.1)
  3  N=64, 128->128, 56x56, F(2,3), fp32 I/O, ReLU; g Kaiming-normal, bias 0
  4  N=256 ResNet-18 stride-1 stack: 4 x 64@56, 3 x 128@28, 3 x 256@14,
     3 x 512@7, F(2,3), fp32, bias ~U(-0.1,0.1) (BN folded), ReLU
  5  N=128, 256->256, 112x112, F(4,3), bf16 x/g/y, fp32 accumulation, bias+ReLU

Seed = config id * 1000 + layer index.  Kaiming-normal here is
N(0, sqrt(2 / fan_in)) with fan_in = 9 * C_in.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

CHANNEL_SWEEP = [(16, 32), (32, 16), (32, 32), (32, 64), (64, 32), (64, 64), (128, 128)]
RN18_STAGES = [(64, 56, 4), (128, 28, 3), (256, 14, 3), (512, 7, 3)]


@dataclass(frozen=True)
class Layer:
    config: int
    index: int
    n: int
    c_in: int
    c_out: int
    h: int
    w: int
    m: int
    relu: bool
    bias: str  # "zero" | "uniform"
    bf16: bool = False

    @property
    def seed(self) -> int:
        return self.config * 1000 + self.index

    @property
    def name(self) -> str:
        dt = "bf16" if self.bf16 else "fp32"
        return (f"cfg{self.config}.{self.index} N={self.n} {self.c_in}->{self.c_out} "
                f"{self.h}x{self.w} F({self.m},3) {dt}{' relu' if self.relu else ''}")

    def conv_flops(self) -> float:
        """2*N*K*C*H*W*9: the effective (direct-convolution) FLOPs of the layer."""
        return 2.0 * self.n * self.c_out * self.c_in * self.h * self.w * 9

    def with_n(self, n: int) -> "Layer":
        return Layer(self.config, self.index, n, self.c_in, self.c_out, self.h, self.w, self.m,
                     self.relu, self.bias, self.bf16)


def config_layers(cfg: int) -> list[Layer]:
    if cfg == 1:
        return [Layer(1, 0, 1, 32, 32, 56, 56, 2, False, "zero")]
    if cfg == 2:
        out, i = [], 0
        for m in (2, 4):
            for c, k in CHANNEL_SWEEP:
                out.append(Layer(2, i, 1, c, k, 56, 56, m, False, "uniform"))
                i += 1
        return out
    if cfg == 3:
        return [Layer(3, 0, 64, 128, 128, 56, 56, 2, True, "zero")]
    if cfg == 4:
        out, i = [], 0
        for c, hw, reps in RN18_STAGES:
            for _ in range(reps):
                out.append(Layer(4, i, 256, c, c, hw, hw, 2, True, "uniform"))
                i += 1
        return out
    if cfg == 5:
        return [Layer(5, 0, 128, 256, 256, 112, 112, 4, True, "uniform", bf16=True)]
    raise ValueError(f"unknown config {cfg}")


def make_weights(layer: Layer):
    """(g, bias) as fp32 numpy arrays; for bf16 layers g is rounded to bf16 values."""
    rng = np.random.default_rng(layer.seed)
    g = rng.normal(0.0, np.sqrt(2.0 / (9 * layer.c_in)),
                   (layer.c_out, layer.c_in, 3, 3)).astype(np.float32)
    if layer.bias == "uniform":
        bias = rng.uniform(-0.1, 0.1, layer.c_out).astype(np.float32)
    else:
        bias = np.zeros(layer.c_out, np.float32)
    if layer.bf16:
        g = bf16_round(g)
    return g, bias


def make_input(layer: Layer, n: int | None = None, first_image: int = 0) -> np.ndarray:
    """x ~ U(-1, 1), shape (n, C, H, W).  Images are generated in blocks keyed by
    the image index so that any shard [first_image, first_image + n) of the batch
    is reproducible on its own (each rank of a multi-GPU run makes only its shard)."""
    n = layer.n if n is None else n
    out = np.empty((n, layer.c_in, layer.h, layer.w), np.float32)
    for j in range(n):
        rng = np.random.default_rng([layer.seed, 7, first_image + j])
        out[j] = rng.uniform(-1.0, 1.0, out.shape[1:]).astype(np.float32)
    if layer.bf16:
        out = bf16_round(out)
    return out


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bfloat16 (ties to even), returned as fp32 values."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    r = np.where(nan, (u | 0x00400000).astype(np.uint32) & np.uint32(0xFFFF0000), r)
    return r.view(np.float32).reshape(a.shape)


def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 values that are already bf16-representable -> uint16 bit patterns."""
    return (np.ascontiguousarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)
