"""Drop-in for the reference's ``src/fused_winograd_kernel.py`` backed by the GPU.

Same module-level tables (``_BT_4`` ... ``_AT_8``, ``_TRANSFORMS``), same class
``FusedWinogradKernel`` with the same constructor, attributes and methods
(``run_fused``, ``run_non_fused``, ``_get_transforms``, ``_log_trace``), same
shapes in and out and the same ``ValueError`` for unsupported tile sizes
(reference: src/fused_winograd_kernel.py:18-181).  The arithmetic runs in
libcwg's per-tile CUDA kernel (``cwg_tiles_fused``); numpy only carries the
arrays.  Beyond the reference: ``run_fused`` / ``run_non_fused`` also accept a
batch of tiles ``(T, C_in, td, td)``, and ``conv2d`` runs a whole NCHW layer.
"""
from __future__ import annotations

import json
import os

import numpy as np

import cwg

# Winograd tables, verbatim values of src/fused_winograd_kernel.py:18-67.
_BT_4 = np.array([[1, 0, -1, 0], [0, 1, 1, 0], [0, -1, 1, 0], [0, 1, 0, -1]], dtype=np.float32)
_AT_4 = np.array([[1, 1, 1, 0], [0, 1, -1, -1]], dtype=np.float32)
_BT_6 = np.array([[4, 0, -5, 0, 1, 0], [0, -4, -4, 1, 1, 0], [0, 4, -4, -1, 1, 0],
                  [0, -2, -1, 2, 1, 0], [0, 2, -1, -2, 1, 0], [0, 4, 0, -5, 0, 1]],
                 dtype=np.float32)
_AT_6 = np.array([[1, 1, 1, 1, 1, 0], [0, 1, -1, 2, -2, 0], [0, 1, 1, 4, 4, 0],
                  [0, 1, -1, 8, -8, 1]], dtype=np.float32)
_BT_8 = np.array([
    [1, 0, -21 / 4, 0, 21 / 4, 0, -1, 0],
    [0, 1, 1, -17 / 4, -17 / 4, 1, 1, 0],
    [0, -1, 1, 17 / 4, -17 / 4, -1, 1, 0],
    [0, 1 / 2, 1 / 4, -5 / 2, -5 / 4, 2, 1, 0],
    [0, -1 / 2, 1 / 4, 5 / 2, -5 / 4, -2, 1, 0],
    [0, 2, 4, -5 / 2, -5, 1 / 2, 1, 0],
    [0, -2, 4, 5 / 2, -5, -1 / 2, 1, 0],
    [0, -1, 0, 21 / 4, 0, -21 / 4, 0, 1]], dtype=np.float32)
_AT_8 = np.array([[1, 1, 1, 1, 1, 32, 32, 0], [0, 1, -1, 2, -2, 16, -16, 0],
                  [0, 1, 1, 4, 4, 8, 8, 0], [0, 1, -1, 8, -8, 4, -4, 0],
                  [0, 1, 1, 16, 16, 2, 2, 0], [0, 1, -1, 32, -32, 1, -1, 1]], dtype=np.float32)

_TRANSFORMS = {4: (_BT_4, _AT_4), 6: (_BT_6, _AT_6), 8: (_BT_8, _AT_8)}


class FusedWinogradKernel:
    """GPU-backed counterpart of the reference class (src/fused_winograd_kernel.py:77-181)."""

    def __init__(self, trace_file="artifacts/fusion_trace.json"):
        self.trace_file = trace_file
        self.trace_data = []
        self.BT = _BT_4
        self.AT = _AT_4

    def _get_transforms(self, td):
        if td not in _TRANSFORMS:
            raise ValueError(
                f"Unsupported tile dimension td={td}. "
                f"Supported: {sorted(_TRANSFORMS.keys())} (F(2,3), F(4,3), F(6,3))")
        return _TRANSFORMS[td]

    def _log_trace(self, method, alloc_count, alloc_size_bytes, has_neon=False):
        # Same bounded JSON trace as the reference (:99-110).
        if self.trace_file and len(self.trace_data) < 100:
            self.trace_data.append({
                "method": method,
                "alloc_count": alloc_count,
                "alloc_size_bytes": float(alloc_size_bytes),
                "neon_supported": has_neon,
            })
            d = os.path.dirname(self.trace_file)
            if d:
                os.makedirs(d, exist_ok=True)
            with open(self.trace_file, "w") as f:
                json.dump(self.trace_data, f, indent=2)

    def _run(self, input_tile, U):
        x = np.asarray(input_tile, dtype=np.float32)
        td = x.shape[-1]
        self._get_transforms(td)
        U = np.asarray(U, dtype=np.float32)
        if x.ndim == 3:
            return cwg.tiles_fused(x[None], U)[0], x.shape[0], U.shape[0], td
        return cwg.tiles_fused(x, U), x.shape[1], U.shape[0], td

    def run_non_fused(self, input_tile, U):
        """Same result as run_fused; the reference differs only in the trace
        metadata it logs (four logical allocations, :146-149)."""
        Y, c_in, c_out, td = self._run(input_tile, U)
        m_logical = c_out * c_in * td * td
        alloc = (c_in * td * td + m_logical + c_out * td * td + Y.size) * 4
        self._log_trace("non_fused", 4, alloc, False)
        return Y

    def run_fused(self, input_tile, U):
        Y, c_in, c_out, td = self._run(input_tile, U)
        alloc = (td * td + c_out * td * td + Y.size) * 4
        self._log_trace("fused", 3, alloc, False)
        return Y

    def conv2d(self, x, g, bias=None, m=0, relu=False):
        """Whole 3x3 layer (NCHW, pad=1, stride=1) through cwg_conv3x3_fused_host:
        x (N, C_in, H, W) and g (C_out, C_in, 3, 3) numpy fp32 -> y (N, C_out, H, W)."""
        import torch  # device memory plumbing only

        x = np.ascontiguousarray(x, dtype=np.float32)
        g = np.ascontiguousarray(g, dtype=np.float32)
        n, c_in, h, w = x.shape
        c_out = g.shape[0]
        flags = cwg.RELU if relu else 0
        dev = torch.device("cuda")
        g_d = torch.from_numpy(g).to(dev)
        U = torch.empty(cwg.weight_bytes(c_in, c_out, m, flags), dtype=torch.uint8, device=dev)
        cwg.weight_transform(g_d, U, c_in, c_out, m, flags)
        b_d = None if bias is None else torch.from_numpy(
            np.ascontiguousarray(bias, dtype=np.float32)).to(dev)
        ws_bytes = cwg.host_workspace_bytes(n, c_in, c_out, h, w, flags)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        y = np.empty((n, c_out, h, w), np.float32)
        cwg.conv3x3_fused_host(x.ctypes.data, U, b_d, y.ctypes.data, ws, ws_bytes,
                               n, c_in, c_out, h, w, m, flags)
        return y
