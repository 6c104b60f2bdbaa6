import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cache-aware-wino-implementation_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


# Parity bars (max abs, normwise rel = max|err| / max|ref|), stated once.
TOL = {
    "f23": (1e-4, 1e-3),   # fp32 F(2x2,3x3) vs the reference C
    "f43": (1e-4, 5e-3),   # fp32 F(4x4,3x3) vs the C restatement of run_fused
    "f63": (1e-3, 5e-3),   # fp32 F(6x6,3x3) vs the C restatement (transform entries up to 32)
    "bf16": (None, 1e-2),  # bf16 I/O vs fp64 direct conv on bf16-rounded x, g
}


def assert_close(y, ref, kind, what=""):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert y.shape == ref.shape, (y.shape, ref.shape)
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    atol, rtol = TOL[kind]
    err = np.abs(y - ref)
    emax = float(err.max()) if err.size else 0.0
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    if atol is not None:
        assert emax <= atol, f"{what}: max abs err {emax:.3e} > {atol}"
    if scale > 0:
        assert emax / scale <= rtol, f"{what}: normwise rel err {emax / scale:.3e} > {rtol}"
    return emax


@pytest.fixture(scope="session")
def cuda_dev():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
