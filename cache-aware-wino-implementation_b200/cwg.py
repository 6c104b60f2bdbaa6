"""ctypes binding of libcwg (include/cwg.h) -- the Python side of the C ABI.

This module only forwards to the compiled library: there is no CPU or PyTorch
fallback anywhere.  If ``lib/libcwg.so`` is missing, importing succeeds but the
first call raises ``RuntimeError`` telling the user to build it.

Device-pointer calls take ``torch`` tensors (used here purely as device-memory
and stream plumbing) or raw integer addresses; host-pointer calls take numpy
arrays.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("CWG_LIB") or os.path.join(HERE, "lib", "libcwg.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "cwg.h")

# status codes and flags (include/cwg.h)
OK, EINVAL, EUNSUPPORTED, ECUDA, ETIMEOUT, ENOMEM, ENODEV, ERANGE = 0, -1, -2, -3, -4, -5, -6, -7
RELU, BF16, FORCE_FFMA, FORCE_TC, TC_SINGLE, TC_FULL16 = 0x1, 0x2, 0x10, 0x20, 0x40, 0x80
TC_NOPAIR, NO_SPLIT, TC_X3, NO_PDL = 0x100, 0x200, 0x400, 0x800
PATH_FFMA, PATH_TC = 1, 2
ORDER_GRID, ORDER_RUNS, ORDER_ROUND = 0, 1, 2  # cwg_choice.order

EXPORTED = (
    "fused_winograd_f23", "cwg_tiles_fused", "cwg_last_status", "cwg_weight_bytes",
    "cwg_weight_transform", "cwg_weight_import", "cwg_conv3x3_fused",
    "cwg_host_workspace_bytes", "cwg_conv3x3_fused_host", "cwg_select", "cwg_strerror",
    "cwg_last_cuda_error", "cwg_device_status", "cwg_launch_count", "cwg_version",
    "cwg_nonfused_workspace_bytes", "cwg_conv3x3_nonfused", "cwg_selftest_wait_timeout",
)


class CwgError(RuntimeError):
    """A libcwg call returned a negative status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {strerror(status)} (status {status})")


class cwg_choice(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int), ("path", ctypes.c_int), ("tiles_per_cta", ctypes.c_int),
        ("cout_per_cta", ctypes.c_int), ("cin_chunk", ctypes.c_int), ("threads", ctypes.c_int),
        ("smem_bytes", ctypes.c_int), ("tmem_cols", ctypes.c_int), ("ctas", ctypes.c_longlong),
        ("gemm_flops", ctypes.c_double), ("alg_bytes", ctypes.c_double),
        ("mma_products", ctypes.c_int), ("ctas_launched", ctypes.c_longlong),
        ("order", ctypes.c_int),
    ]


@dataclass
class Choice:
    m: int
    path: int
    tiles_per_cta: int
    cout_per_cta: int
    cin_chunk: int
    threads: int
    smem_bytes: int
    tmem_cols: int
    ctas: int
    gemm_flops: float
    alg_bytes: float
    mma_products: int
    ctas_launched: int
    order: int

    @property
    def path_name(self) -> str:
        return {PATH_FFMA: "ffma", PATH_TC: "tcgen05"}.get(self.path, "?")

    @property
    def order_name(self) -> str:
        return {ORDER_GRID: "one unit per CTA pair", ORDER_RUNS: "persistent pairs, equal tile runs",
                ORDER_ROUND: "persistent pairs, round robin"}.get(self.order, "?")


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libcwg.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"libcwg.so not found at {LIB_PATH}: build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i, u, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, ctypes.c_size_t
    fp = ctypes.POINTER(ctypes.c_float)
    L.fused_winograd_f23.argtypes = [fp, fp, fp, i, i]
    L.fused_winograd_f23.restype = None
    L.cwg_tiles_fused.argtypes = [fp, fp, fp, i, i, i, i]
    L.cwg_tiles_fused.restype = i
    L.cwg_last_status.argtypes = []
    L.cwg_last_status.restype = i
    L.cwg_weight_bytes.argtypes = [i, i, i, u]
    L.cwg_weight_bytes.restype = sz
    L.cwg_weight_transform.argtypes = [vp, vp, i, i, i, u, vp]
    L.cwg_weight_transform.restype = i
    L.cwg_weight_import.argtypes = [vp, vp, i, i, i, u, vp]
    L.cwg_weight_import.restype = i
    L.cwg_conv3x3_fused.argtypes = [vp, vp, vp, vp, i, i, i, i, i, i, u, vp]
    L.cwg_conv3x3_fused.restype = i
    L.cwg_host_workspace_bytes.argtypes = [i, i, i, i, i, u]
    L.cwg_host_workspace_bytes.restype = sz
    L.cwg_conv3x3_fused_host.argtypes = [vp, vp, vp, vp, vp, sz, i, i, i, i, i, i, u, vp]
    L.cwg_conv3x3_fused_host.restype = i
    L.cwg_select.argtypes = [i, i, i, i, i, i, u, ctypes.POINTER(cwg_choice)]
    L.cwg_select.restype = i
    L.cwg_strerror.argtypes = [i]
    L.cwg_strerror.restype = ctypes.c_char_p
    L.cwg_last_cuda_error.argtypes = []
    L.cwg_last_cuda_error.restype = i
    L.cwg_device_status.argtypes = [vp]
    L.cwg_device_status.restype = i
    L.cwg_launch_count.argtypes = []
    L.cwg_launch_count.restype = ctypes.c_longlong
    L.cwg_version.argtypes = []
    L.cwg_version.restype = ctypes.c_char_p
    L.cwg_selftest_wait_timeout.argtypes = [vp]
    L.cwg_selftest_wait_timeout.restype = i
    L.cwg_nonfused_workspace_bytes.argtypes = [i, i, i, i, i, i]
    L.cwg_nonfused_workspace_bytes.restype = sz
    L.cwg_conv3x3_nonfused.argtypes = [vp, vp, vp, vp, vp, sz, i, i, i, i, i, i, u, vp]
    L.cwg_conv3x3_nonfused.restype = i
    _lib = L
    return L


def strerror(status: int) -> str:
    try:
        return lib().cwg_strerror(int(status)).decode()
    except RuntimeError:
        return f"status {status}"


def _check(status: int, what: str) -> None:
    if status != OK:
        if status == ECUDA:
            what = f"{what} (cudaError {lib().cwg_last_cuda_error()})"
        raise CwgError(status, what)


def _ptr(t) -> int | None:
    """Device address of a torch tensor (or an int address, or None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return int(t.data_ptr())


def _stream(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


# ---- selector -----------------------------------------------------------------
def select(n: int, c_in: int, c_out: int, h: int, w: int, m: int = 0, flags: int = 0) -> Choice:
    """Tile/kernel choice for a layer (replaces CacheAdaptiveAutotiler.select_best_tile)."""
    out = cwg_choice()
    _check(lib().cwg_select(n, c_in, c_out, h, w, m, flags, ctypes.byref(out)), "cwg_select")
    return Choice(*(getattr(out, f) for f, _ in cwg_choice._fields_))


def weight_bytes(c_in: int, c_out: int, m: int = 0, flags: int = 0) -> int:
    return int(lib().cwg_weight_bytes(c_in, c_out, m, flags))


# ---- device-pointer layer API -----------------------------------------------------
def weight_transform(g, U, c_in: int, c_out: int, m: int = 0, flags: int = 0, stream=None):
    _check(lib().cwg_weight_transform(_ptr(g), _ptr(U), c_in, c_out, m, flags, _stream(stream)),
           "cwg_weight_transform")


def weight_import(U_ref, U, c_in: int, c_out: int, m: int, flags: int = 0, stream=None):
    _check(lib().cwg_weight_import(_ptr(U_ref), _ptr(U), c_in, c_out, m, flags,
                                   _stream(stream)), "cwg_weight_import")


def conv3x3_fused(x, U, bias, y, n: int, c_in: int, c_out: int, h: int, w: int, m: int = 0,
                  flags: int = 0, stream=None) -> None:
    _check(lib().cwg_conv3x3_fused(_ptr(x), _ptr(U), _ptr(bias), _ptr(y), n, c_in, c_out, h, w,
                                   m, flags, _stream(stream)), "cwg_conv3x3_fused")


def nonfused_workspace_bytes(n, c_in, c_out, h, w, m) -> int:
    return int(lib().cwg_nonfused_workspace_bytes(n, c_in, c_out, h, w, m))


def conv3x3_nonfused(x, U, bias, y, workspace, workspace_bytes: int, n: int, c_in: int,
                     c_out: int, h: int, w: int, m: int, flags: int = 0, stream=None) -> None:
    """Non-fused ablation: three passes over HBM (fp32; U from weight_transform with
    FORCE_FFMA)."""
    _check(lib().cwg_conv3x3_nonfused(_ptr(x), _ptr(U), _ptr(bias), _ptr(y), _ptr(workspace),
                                      workspace_bytes, n, c_in, c_out, h, w, m, flags,
                                      _stream(stream)), "cwg_conv3x3_nonfused")


def host_workspace_bytes(n, c_in, c_out, h, w, flags=0) -> int:
    return int(lib().cwg_host_workspace_bytes(n, c_in, c_out, h, w, flags))


def conv3x3_fused_host(x_host: int, U, bias, y_host: int, workspace, workspace_bytes: int,
                       n, c_in, c_out, h, w, m=0, flags=0, stream=None) -> None:
    _check(lib().cwg_conv3x3_fused_host(_ptr(x_host), _ptr(U), _ptr(bias), _ptr(y_host),
                                        _ptr(workspace), workspace_bytes, n, c_in, c_out, h, w,
                                        m, flags, _stream(stream)), "cwg_conv3x3_fused_host")


def device_status(stream=None) -> None:
    """Raises CwgError(ETIMEOUT) if a bounded device wait gave up since the last check, or
    CwgError(ERANGE) if an fp16 tensor-core operand overflowed."""
    _check(lib().cwg_device_status(_stream(stream)), "device status")


def selftest_wait_timeout(stream=None) -> None:
    """Launches a kernel whose bounded wait runs out; the next device_status() raises
    CwgError(ETIMEOUT)."""
    _check(lib().cwg_selftest_wait_timeout(_stream(stream)), "cwg_selftest_wait_timeout")


def launch_count() -> int:
    return int(lib().cwg_launch_count())


def version() -> str:
    return lib().cwg_version().decode()


# ---- host-pointer per-tile API ----------------------------------------------------
def _f32c(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def tiles_fused(tiles: np.ndarray, U: np.ndarray) -> np.ndarray:
    """Per-tile fused Winograd on the GPU: tiles (T, C_in, td, td), U (C_out, C_in, td, td)
    -> (T, C_out, td-2, td-2); td in {4, 6, 8}."""
    tiles = _f32c(tiles)
    U = _f32c(U)
    if tiles.ndim != 4 or U.ndim != 4:
        raise ValueError("tiles must be (T, C_in, td, td) and U (C_out, C_in, td, td)")
    nt, c_in, td, td2 = tiles.shape
    c_out = U.shape[0]
    if td != td2 or U.shape[1:] != (c_in, td, td):
        raise ValueError(f"shape mismatch: tiles {tiles.shape}, U {U.shape}")
    m = td - 2
    out = np.empty((nt, c_out, max(m, 0), max(m, 0)), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    st = lib().cwg_tiles_fused(tiles.ctypes.data_as(fp), U.ctypes.data_as(fp),
                               out.ctypes.data_as(fp), nt, c_in, c_out, td)
    if st == EINVAL and td not in (4, 6, 8):
        raise ValueError(f"Unsupported tile dimension td={td}. Supported: [4, 6, 8]")
    _check(st, "cwg_tiles_fused")
    return out


def fused_winograd_f23(input_tile: np.ndarray, U: np.ndarray) -> np.ndarray:
    """The reference's C entry point (fused_winograd.c:103) called through ctypes:
    input (C_in, 4, 4), U (C_out, C_in, 4, 4) -> (C_out, 2, 2)."""
    inp = _f32c(input_tile)
    U = _f32c(U)
    c_in, c_out = inp.shape[0], U.shape[0]
    out = np.empty((c_out, 2, 2), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    lib().fused_winograd_f23(inp.ctypes.data_as(fp), U.ctypes.data_as(fp),
                             out.ctypes.data_as(fp), c_in, c_out)
    _check(lib().cwg_last_status(), "fused_winograd_f23")
    return out
