"""ctypes binding of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loaded only by the test suite, by ``__graft_entry__.smoke()`` and by the CPU
baseline leg of ``bench.py``; the product never imports it.

* ``libcwg_oracle.so`` (oracle/cwg_oracle.c): the C restatement of the
  reference's algorithm (fused_winograd.c:19-101 and
  src/fused_winograd_kernel.py:153-181), the weight transform, the layer
  driver and an fp64 direct convolution.
* ``libref_layer.so`` (oracle/ref_layer.c + the reference's own
  fused_winograd.c, compiled from the reference sources): the reference kernel
  itself behind a layer driver.  Optional: present when it was built.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libcwg_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_layer.so")

_fp = ctypes.POINTER(ctypes.c_float)
_dp = ctypes.POINTER(ctypes.c_double)
_i = ctypes.c_int

_orc = None
_ref = None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a, t=_fp):
    return None if a is None else a.ctypes.data_as(t)


def orc() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"oracle not built: {ORACLE_SO} (run make -C oracle)")
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_weight_transform.argtypes = [_fp, _fp, _i, _i, _i]
        L.orc_tiles_fused.argtypes = [_fp, _fp, _fp, _i, _i, _i, _i, _i]
        L.orc_conv_layer.argtypes = [_fp, _fp, _fp, _fp, _i, _i, _i, _i, _i, _i, _i, _i]
        L.orc_direct_conv_f64.argtypes = [_fp, _fp, _fp, _dp, _i, _i, _i, _i, _i, _i, _i]
        L.orc_round_bf16.argtypes = [_fp, ctypes.c_long]
        L.orc_round_bf16.restype = None
        L.orc_max_threads.restype = _i
        _orc = L
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"reference C not built: {REF_SO}")
        L = ctypes.CDLL(REF_SO)
        L.refl_tiles_f23.argtypes = [_fp, _fp, _fp, _i, _i, _i, _i]
        L.refl_conv_layer_f23.argtypes = [_fp, _fp, _fp, _fp, _i, _i, _i, _i, _i, _i, _i]
        L.refl_max_threads.restype = _i
        L.fused_winograd_f23.argtypes = [_fp, _fp, _fp, _i, _i]
        L.fused_winograd_f23.restype = None
        _ref = L
    return _ref


def _ok(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed with {rc}")


def max_threads() -> int:
    return int(orc().orc_max_threads())


def weight_transform(g, td: int) -> np.ndarray:
    """g (K, C, 3, 3) -> U (K, C, td, td), fp64 math rounded once to fp32."""
    g = _f32(g)
    K, C = g.shape[:2]
    U = np.empty((K, C, td, td), np.float32)
    _ok(orc().orc_weight_transform(_p(g), _p(U), K, C, td), "orc_weight_transform")
    return U


def tiles_fused(tiles, U, nthreads: int = 0) -> np.ndarray:
    tiles, U = _f32(tiles), _f32(U)
    nt, C, td = tiles.shape[0], tiles.shape[1], tiles.shape[-1]
    K = U.shape[0]
    out = np.empty((nt, K, td - 2, td - 2), np.float32)
    _ok(orc().orc_tiles_fused(_p(tiles), _p(U), _p(out), nt, C, K, td, nthreads),
        "orc_tiles_fused")
    return out


def conv_layer(x, U, bias, td: int, relu: bool, nthreads: int = 0) -> np.ndarray:
    """Winograd restatement of a whole layer: x (N,C,H,W), U (K,C,td,td) -> y (N,K,H,W)."""
    x, U = _f32(x), _f32(U)
    b = None if bias is None else _f32(bias)
    N, C, H, W = x.shape
    K = U.shape[0]
    y = np.empty((N, K, H, W), np.float32)
    _ok(orc().orc_conv_layer(_p(x), _p(U), _p(b), _p(y), N, C, K, H, W, td, int(relu),
                             nthreads), "orc_conv_layer")
    return y


def direct_conv_f64(x, g, bias, relu: bool, nthreads: int = 0) -> np.ndarray:
    x, g = _f32(x), _f32(g)
    b = None if bias is None else _f32(bias)
    N, C, H, W = x.shape
    K = g.shape[0]
    y = np.empty((N, K, H, W), np.float64)
    _ok(orc().orc_direct_conv_f64(_p(x), _p(g), _p(b), _p(y, _dp), N, C, K, H, W, int(relu),
                                  nthreads), "orc_direct_conv_f64")
    return y


def round_bf16(a) -> np.ndarray:
    a = np.array(a, dtype=np.float32, copy=True, order="C")
    orc().orc_round_bf16(_p(a), a.size)
    return a


def ref_tiles_f23(tiles, U, nthreads: int = 0) -> np.ndarray:
    """The reference's own fused_winograd_f23 on each tile."""
    tiles, U = _f32(tiles), _f32(U)
    nt, C = tiles.shape[:2]
    K = U.shape[0]
    out = np.empty((nt, K, 2, 2), np.float32)
    _ok(ref().refl_tiles_f23(_p(tiles), _p(U), _p(out), nt, C, K, nthreads), "refl_tiles_f23")
    return out


def ref_conv_layer_f23(x, U, bias, relu: bool, nthreads: int = 0) -> np.ndarray:
    """A whole F(2,3) layer through the reference's own per-tile C kernel."""
    x, U = _f32(x), _f32(U)
    b = None if bias is None else _f32(bias)
    N, C, H, W = x.shape
    K = U.shape[0]
    y = np.empty((N, K, H, W), np.float32)
    _ok(ref().refl_conv_layer_f23(_p(x), _p(U), _p(b), _p(y), N, C, K, H, W, int(relu),
                                  nthreads), "refl_conv_layer_f23")
    return y
