"""Generates the golden vectors under tests/golden/ from the reference itself.

Run where the reference project's source tree is available, after
``make -C oracle REF=<tree>``, naming the tree in ``CWG_REFERENCE`` (required):

    CWG_REFERENCE=<path to the reference tree> python tests/golden/make_golden.py

Sources of truth:
* ``run_fused`` / ``run_non_fused`` of the reference's Python kernel
  (src/fused_winograd_kernel.py:116-181), imported from the reference tree;
* the reference's C kernel ``fused_winograd_f23`` (fused_winograd.c:103-119),
  compiled from the reference sources by oracle/Makefile (oracle/_ref).

Layer-level goldens apply the reference's ``run_fused`` to every tile of a
zero-padded image (the reference has no layer driver; this script's numpy
pad / extract / scatter is the only code of ours involved), with U = G g G^T
computed here in numpy fp64 and rounded once to fp32.  A numpy fp64 direct
convolution of the same inputs is stored beside each layer golden.
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("CWG_REFERENCE", "")

G = {
    4: np.array([[1, 0, 0], [.5, .5, .5], [.5, -.5, .5], [0, 0, 1]]),
    6: np.array([[1 / 4, 0, 0], [-1 / 6, -1 / 6, -1 / 6], [-1 / 6, 1 / 6, -1 / 6],
                 [1 / 24, 1 / 12, 1 / 6], [1 / 24, -1 / 12, 1 / 6], [0, 0, 1]]),
    8: np.array([[1, 0, 0], [-2 / 9, -2 / 9, -2 / 9], [-2 / 9, 2 / 9, -2 / 9],
                 [1 / 90, 1 / 45, 2 / 45], [1 / 90, -1 / 45, 2 / 45],
                 [1 / 45, 1 / 90, 1 / 180], [1 / 45, -1 / 90, 1 / 180], [0, 0, 1]]),
}


def weight_transform(g: np.ndarray, td: int) -> np.ndarray:
    Gm = G[td]
    return np.einsum("ai,kcij,bj->kcab", Gm, g.astype(np.float64), Gm).astype(np.float32)


def direct_conv(x, g, bias, relu):
    N, C, H, W = x.shape
    K = g.shape[0]
    xp = np.zeros((N, C, H + 2, W + 2))
    xp[:, :, 1:-1, 1:-1] = x
    y = np.zeros((N, K, H, W))
    for ky in range(3):
        for kx in range(3):
            y += np.einsum("nchw,kc->nkhw", xp[:, :, ky:ky + H, kx:kx + W],
                           g[:, :, ky, kx].astype(np.float64))
    if bias is not None:
        y += bias[None, :, None, None]
    return np.maximum(y, 0) if relu else y


def layer_via_run_fused(kernel, x, U, bias, td, relu):
    m = td - 2
    N, C, H, W = x.shape
    K = U.shape[0]
    th, tw = -(-H // m), -(-W // m)
    xp = np.zeros((N, C, th * m + 2, tw * m + 2), np.float32)
    xp[:, :, 1:H + 1, 1:W + 1] = x
    y = np.zeros((N, K, th * m, tw * m), np.float32)
    for n in range(N):
        for ty in range(th):
            for tx in range(tw):
                d = xp[n, :, ty * m:ty * m + td, tx * m:tx * m + td]
                y[n, :, ty * m:(ty + 1) * m, tx * m:(tx + 1) * m] = kernel.run_fused(d, U)
    y = y[:, :, :H, :W]
    if bias is not None:
        y = y + bias[None, :, None, None].astype(np.float32)
    if relu:
        y = np.where(y < 0, np.float32(0), y)
    return y.astype(np.float32)


def main() -> None:
    if not REF or not os.path.exists(os.path.join(REF, "src", "fused_winograd_kernel.py")):
        raise SystemExit("set CWG_REFERENCE to the reference project's source tree")
    sys.path.insert(0, REF)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from src.fused_winograd_kernel import FusedWinogradKernel  # the reference
    import oracle

    kernel = FusedWinogradKernel(trace_file=os.path.join(tempfile.mkdtemp(), "trace.json"))
    rng = np.random.default_rng(20240601)

    # ---- per-tile goldens ----
    for td, cases in ((4, [(5, 7), (16, 32)]), (6, [(5, 7), (16, 8)]), (8, [(3, 4)])):
        out = {}
        for i, (c_in, c_out) in enumerate(cases):
            tiles = rng.standard_normal((3, c_in, td, td)).astype(np.float32)
            U = rng.standard_normal((c_out, c_in, td, td)).astype(np.float32)
            U[0, 0, 0, 0] = 0.0  # exercise the reference's zero-skip
            fused = np.stack([kernel.run_fused(t, U) for t in tiles]).astype(np.float32)
            nonfused = np.stack([kernel.run_non_fused(t, U) for t in tiles]).astype(np.float32)
            out[f"tiles_{i}"], out[f"U_{i}"] = tiles, U
            out[f"run_fused_{i}"], out[f"run_non_fused_{i}"] = fused, nonfused
            if td == 4:
                out[f"ref_c_{i}"] = oracle.ref_tiles_f23(tiles, U)
        np.savez_compressed(os.path.join(HERE, f"tiles_td{td}.npz"), **out)

    # ---- layer-level goldens ----
    layers = [
        # name, N, C, K, H, W, td, relu, bias
        ("f23_odd", 1, 3, 4, 7, 5, 4, True, True),
        ("f23_pixel", 1, 2, 2, 1, 1, 4, False, False),
        ("f23_wide", 2, 16, 16, 6, 10, 4, True, True),
        ("f43_odd", 2, 4, 3, 6, 9, 6, False, True),
        ("f43_small", 1, 5, 6, 3, 3, 6, True, False),
        ("f63_square", 1, 8, 8, 8, 8, 8, False, True),
    ]
    for name, N, C, K, H, W, td, relu, use_bias in layers:
        x = rng.uniform(-1, 1, (N, C, H, W)).astype(np.float32)
        g = rng.normal(0, np.sqrt(2 / (9 * C)), (K, C, 3, 3)).astype(np.float32)
        bias = rng.uniform(-0.1, 0.1, K).astype(np.float32) if use_bias else None
        U = weight_transform(g, td)
        y = layer_via_run_fused(kernel, x, U, bias, td, relu)
        yd = direct_conv(x, g, bias, relu)
        d = dict(x=x, g=g, U=U, y=y, y_direct=yd,
                 meta=np.array([N, C, K, H, W, td, int(relu), int(use_bias)], np.int64))
        if bias is not None:
            d["bias"] = bias
        np.savez_compressed(os.path.join(HERE, f"layer_{name}.npz"), **d)
        print(f"{name}: max |run_fused layer - fp64 direct| = {np.abs(y - yd).max():.3e}")


if __name__ == "__main__":
    main()
