"""The layer call for callers that cannot allocate device memory.

cwg_conv3x3_fused_host needs a device workspace from its caller.  Code that
runs where a framework's allocator owns the device heap, plug-in hosts that
only pass host buffers and a stream, and real-time paths that may not allocate
after start-up cannot provide one; cwg_conv3x3_fused_host_static stages through
a fixed array inside the library instead.  This test calls it through the C ABI
twice in a row (different layers, so stale contents of the shared array would
show) and compares each result with the workspace entry point's; a repeated call
leaves the device's free memory where it was, and a call on a non-blocking
stream of the current device gives the same result.  The file is named to be
collected last.
"""
import ctypes

import numpy as np
import pytest

import cwg
from conftest import assert_close

pytestmark = pytest.mark.gpu


def _static_entry():
    L = cwg.lib()
    fn = L.cwg_conv3x3_fused_host_static
    vp, i, u = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint
    fn.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, u, vp]
    fn.restype = i
    return fn


def _layer(dev, seed, n, c, k, h, w, m, flags):
    import torch

    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    U = torch.empty(cwg.weight_bytes(c, k, m, flags), dtype=torch.uint8, device=dev)
    cwg.weight_transform(torch.from_numpy(g).to(dev), U, c, k, m, flags)
    return x, U, torch.from_numpy(b).to(dev)


def test_static_entry_matches_workspace_entry(cuda_dev):
    import torch

    fn = _static_entry()
    cases = [  # tensor-core layer, then a CUDA-core layer of a different size
        (21, 2, 64, 128, 14, 14, 2, cwg.RELU),
        (22, 1, 16, 24, 9, 11, 4, 0),
    ]
    for seed, n, c, k, h, w, m, flags in cases:
        x, U, b = _layer(cuda_dev, seed, n, c, k, h, w, m, flags)
        y_static = np.full((n, k, h, w), np.nan, np.float32)
        rc = fn(x.ctypes.data, U.data_ptr(), b.data_ptr(), y_static.ctypes.data,
                n, c, k, h, w, m, flags, None)
        assert rc == cwg.OK, cwg.strerror(rc)

        ws_bytes = cwg.host_workspace_bytes(n, c, k, h, w, flags)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_dev)
        y_ws = np.full((n, k, h, w), np.nan, np.float32)
        cwg.conv3x3_fused_host(x.ctypes.data, U, b, y_ws.ctypes.data, ws, ws_bytes,
                               n, c, k, h, w, m, flags)
        assert_close(y_static, y_ws, "f23" if m == 2 else "f43", f"static entry, seed {seed}")

    # the same layer again, on a non-blocking stream: nothing allocated on the device
    stream = torch.cuda.Stream(cuda_dev)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(cuda_dev)[0]
    y_again = np.full((n, k, h, w), np.nan, np.float32)
    rc = fn(x.ctypes.data, U.data_ptr(), b.data_ptr(), y_again.ctypes.data,
            n, c, k, h, w, m, flags, stream.cuda_stream)
    assert rc == cwg.OK, cwg.strerror(rc)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda_dev)[0] >= free0
    assert_close(y_again, y_ws, "f23" if m == 2 else "f43", "static entry, non-blocking stream")


def test_static_entry_rejects_layers_beyond_its_array(cuda_dev):
    fn = _static_entry()
    n, c, k, h, w = 64, 128, 128, 56, 56  # 206 MB of staging > 32 MiB
    assert cwg.host_workspace_bytes(n, c, k, h, w) > 32 << 20
    x = np.zeros(1, np.float32)
    y = np.zeros(1, np.float32)
    rc = fn(x.ctypes.data, 0x1000, None, y.ctypes.data, n, c, k, h, w, 2, 0, None)
    assert rc == cwg.EUNSUPPORTED
    # an empty batch is a no-op, as for the device-pointer call
    assert fn(x.ctypes.data, 0x1000, None, y.ctypes.data, 0, c, k, h, w, 2, 0, None) == cwg.OK
