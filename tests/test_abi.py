"""CPU-side checks of the C ABI: the library loads, exports every symbol the
header declares, and its host logic (selector, argument checks, error codes)
behaves -- none of this launches a kernel."""
import ctypes
import os
import re

import numpy as np
import pytest

import cwg

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "cwg.h")



def cuda_present() -> bool:
    import torch

    return torch.cuda.is_available()

def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b([a-z_][a-z0-9_]*)\s*\([^;{]*\)\s*;", text)
    return sorted(set(n for n in names if n not in ("sizeof",)))


def test_library_loads_and_exports_every_declared_symbol():
    L = cwg.lib()
    names = declared_functions()
    assert "fused_winograd_f23" in names and "cwg_conv3x3_fused" in names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(cwg.EXPORTED) <= set(names)


def test_reference_symbol_signature_is_exported_verbatim():
    # fused_winograd.c:103-108: void fused_winograd_f23(const float*, const float*, float*, int, int)
    text = open(HEADER).read()
    assert re.search(r"void\s+fused_winograd_f23\s*\(\s*const float \*input,\s*const float \*U,"
                     r"\s*float \*output,\s*int c_in,\s*int c_out\s*\)", text)


def test_version_and_strerror():
    assert "sm_100a" in cwg.version()
    assert cwg.strerror(cwg.EINVAL) == "invalid argument"
    assert cwg.strerror(cwg.ETIMEOUT).startswith("device-side wait")
    assert cwg.strerror(12345) == "unknown status"


def test_selector_small_channels_take_ffma():
    ch = cwg.select(1, 32, 32, 56, 56)
    assert ch.path == cwg.PATH_FFMA and ch.m == 2
    assert ch.smem_bytes <= 227 * 1024 and ch.tmem_cols == 0
    assert ch.gemm_flops == 2 * 28 * 28 * 32 * 32 * 16
    # bytes: x + y + U + bias
    assert ch.alg_bytes == 32 * 56 * 56 * 4 * 2 + 16 * 32 * 32 * 4 + 4 * 32


def test_selector_auto_m_and_bf16():
    assert cwg.select(1, 16, 32, 56, 56, 0, cwg.BF16 | cwg.FORCE_FFMA).m == 4
    assert cwg.select(1, 16, 32, 56, 56, 4).m == 4
    assert cwg.select(1, 16, 32, 56, 56, 2).m == 2
    # 1-4 input channels: F(2,3) on the one-tile-per-thread kernel, bf16 too
    small = cwg.select(1, 3, 64, 224, 224, 0, cwg.BF16)
    assert small.m == 2 and small.path == cwg.PATH_FFMA and small.threads == 256


def test_selector_grid_covers_layer():
    for (n, c, k, h, w, m) in [(1, 32, 32, 56, 56, 2), (3, 16, 17, 7, 5, 4), (2, 64, 64, 1, 1, 2)]:
        ch = cwg.select(n, c, k, h, w, m, cwg.FORCE_FFMA | cwg.NO_SPLIT)
        th, tw = -(-h // ch.m), -(-w // ch.m)
        side = int(round(ch.tiles_per_cta ** 0.5))
        assert ch.ctas == n * (-(-th // side)) * (-(-tw // side)) * (-(-k // ch.cout_per_cta))


def ffma_slices(ch, n, k, h, w):
    """C_in slices of a CUDA-core choice: CTAs over the grid of its tile and channel blocks."""
    th, tw = -(-h // ch.m), -(-w // ch.m)
    side = int(round(ch.tiles_per_cta ** 0.5))
    grid = n * (-(-th // side)) * (-(-tw // side)) * (-(-k // ch.cout_per_cta))
    assert ch.ctas % grid == 0
    return ch.ctas // grid


def test_selector_ffma_split():
    """The CUDA-core path picks its channel block and C_in slices together from a
    per-CTA cost model: single-image deep layers split (fp32 only, at most one
    slice per 8-channel step, CTAs within one round of the SMs); bf16 layers,
    NO_SPLIT and grids that fill the SMs do not."""
    sms = 148
    for (c, k, h, m) in [(256, 256, 14, 4), (512, 512, 7, 4), (64, 32, 56, 4), (512, 32, 7, 2),
                         (128, 40, 30, 6), (128, 128, 56, 4)]:
        ch = cwg.select(1, c, k, h, h, m, cwg.FORCE_FFMA)
        s = ffma_slices(ch, 1, k, h, h)
        assert 2 <= s <= -(-c // 8) and ch.ctas <= sms, (c, k, h, m, s, ch.ctas)
        for fl in (cwg.BF16, cwg.NO_SPLIT):
            assert ffma_slices(cwg.select(1, c, k, h, h, m, cwg.FORCE_FFMA | fl), 1, k, h, h) == 1
    for (n, c, k, h, m) in [(64, 32, 32, 56, 2), (64, 128, 128, 56, 4), (2, 128, 128, 60, 6),
                            (1, 16, 32, 56, 2), (1, 32, 32, 56, 2)]:
        ch = cwg.select(n, c, k, h, h, m, cwg.FORCE_FFMA)
        assert ffma_slices(ch, n, k, h, h) == 1, (n, c, k, h, m)
    # large layers keep the widest channel block
    assert cwg.select(64, 128, 128, 56, 56, 4, cwg.FORCE_FFMA).cout_per_cta == 64


@pytest.mark.parametrize("args,status", [
    ((1, 0, 32, 56, 56, 2, 0), cwg.EINVAL),
    ((1, 32, 0, 56, 56, 2, 0), cwg.EINVAL),
    ((1, 32, 32, 0, 56, 2, 0), cwg.EINVAL),
    ((1, 32, 32, 56, 56, 3, 0), cwg.EINVAL),
    ((1, 32, 32, 56, 56, 8, 0), cwg.EINVAL),
    ((1, 128, 128, 56, 56, 6, cwg.FORCE_TC), cwg.EUNSUPPORTED),
    ((1, 32, 32, 56, 56, 2, cwg.FORCE_FFMA | cwg.FORCE_TC), cwg.EINVAL),
])
def test_selector_rejects(args, status):
    with pytest.raises(cwg.CwgError) as e:
        cwg.select(*args)
    assert e.value.status == status


def test_weight_bytes():
    assert cwg.weight_bytes(32, 32, 2, cwg.FORCE_FFMA) == 16 * 32 * 32 * 4
    assert cwg.weight_bytes(32, 32, 4, cwg.FORCE_FFMA | cwg.BF16) == 36 * 32 * 32 * 4
    assert cwg.weight_bytes(0, 32, 2) == 0
    assert cwg.weight_bytes(32, 32, 6) == 64 * 32 * 32 * 4  # F(6,3): CUDA cores, fp32 U
    assert cwg.weight_bytes(32, 32, 8) == 0


def test_selector_f63_runs_on_cuda_cores():
    ch = cwg.select(2, 128, 128, 60, 60, 6)
    assert ch.path == cwg.PATH_FFMA and ch.m == 6 and ch.mma_products == 0
    assert ch.tiles_per_cta == 16 and ch.cout_per_cta == 16
    assert ch.ctas == 2 * 3 * 3 * 8  # 10x10 tiles of 6x6 -> 3x3 blocks of 4x4 tiles


def test_selector_tensor_core_variants():
    n, c, k, h, w = 4, 128, 256, 30, 30
    tiles = n * 15 * 15
    pair = cwg.select(n, c, k, h, w, 2, cwg.NO_SPLIT)
    assert pair.path == cwg.PATH_TC and pair.tiles_per_cta == 128 and pair.tmem_cols == 512
    assert pair.ctas == 2 * (-(-tiles // 128)) * 2  # two CTAs per 128-tile block
    # 16 (tile block, channel block) items leave 3/4 of the 74 TPCs idle: the C_in
    # reduction (8 stages of 16 channels) splits into 4 slices of 2 stages
    assert cwg.select(n, c, k, h, w).ctas == pair.ctas * 4
    # 25 items (4 images of 56x56) fill a third of the TPCs: no split
    assert cwg.select(4, c, 128, 56, 56).ctas == cwg.select(4, c, 128, 56, 56, 2, cwg.NO_SPLIT).ctas
    assert cwg.select(n, c, k, h, w, 2, cwg.BF16).ctas == pair.ctas  # fp32 layers only
    assert cwg.select(64, c, k, 56, 56).ctas == cwg.select(64, c, k, 56, 56, 2, cwg.NO_SPLIT).ctas
    single = cwg.select(n, c, k, h, w, 2, cwg.TC_NOPAIR)
    assert single.tiles_per_cta == 64 and single.ctas == (-(-tiles // 64)) * 2
    assert cwg.select(n, c, k, h, w, 2, cwg.TC_FULL16).tiles_per_cta == 32
    # the pair layout holds both At-scaled row sets: [C_out/128][2][C_in/16][16 f][parts]
    # blocks of 4096 bytes
    assert cwg.weight_bytes(c, k, 2) == 2 * cwg.weight_bytes(c, k, 2, cwg.TC_NOPAIR)
    assert cwg.weight_bytes(c, k, 2, cwg.TC_NOPAIR) == 2 * 8 * 16 * 2 * 4096
    assert cwg.weight_bytes(c, k, 2, cwg.BF16) == 2 * 2 * 8 * 16 * 1 * 4096
    with pytest.raises(cwg.CwgError) as e:
        cwg.select(n, c, k, h, w, 2, cwg.TC_NOPAIR | cwg.TC_FULL16)
    assert e.value.status == cwg.EINVAL


def test_selector_64_channel_pair():
    """F(2,3) layers of at most 64 output channels run the pair kernel with M = 128:
    64 channels per CTA and 64-row weight blocks (2048 bytes)."""
    c, k = 96, 64
    ch = cwg.select(4, c, k, 56, 56, 2, cwg.NO_SPLIT)
    assert ch.path == cwg.PATH_TC and ch.cout_per_cta == 64 and ch.tiles_per_cta == 128
    # [1 channel block][2 ranks][6 C_in steps][16 f][hi, lo] blocks of 64 x 16 bf16
    assert cwg.weight_bytes(c, k, 2) == 1 * 2 * 6 * 16 * 2 * 2048
    assert cwg.weight_bytes(c, k, 2, cwg.BF16) == 1 * 2 * 6 * 16 * 1 * 2048
    # 65 channels and up: the M = 256 kernel, 128 channels per CTA
    assert cwg.select(4, c, 65, 56, 56).cout_per_cta == 128
    assert cwg.weight_bytes(c, 65, 2) == 1 * 2 * 6 * 16 * 2 * 4096
    # F(4,3) likewise: up to 64 channels, two output rows x 64 channels per CTA
    # in one pass over all 36 frequencies ([1][2 ranks][6][36 f] fp16 blocks of 128
    # rows); above, 128 channels of one row per CTA in two passes of 30 frequencies
    assert cwg.select(4, c, k, 56, 56, 4, cwg.BF16).cout_per_cta == 64
    assert cwg.weight_bytes(c, k, 4, cwg.BF16) == 1 * 2 * 6 * 36 * 1 * 4096
    assert cwg.weight_bytes(c, k, 4, cwg.BF16 | cwg.TC_X3) == 1 * 2 * 6 * 36 * 2 * 4096
    assert cwg.select(4, c, 65, 56, 56, 4, cwg.BF16).cout_per_cta == 128
    assert cwg.weight_bytes(c, 65, 4, cwg.BF16) == 1 * 2 * 2 * 6 * 30 * 1 * 4096
    # the single-CTA ablations keep their layouts
    assert cwg.select(4, c, k, 56, 56, 2, cwg.TC_NOPAIR).cout_per_cta == 128


def test_selector_launch_plan():
    """Which grid the pair kernel launches (without a device: 74 TPCs, one cluster each)."""
    # 26 units (13 tile blocks x 2 channel blocks) below one wave: one unit per CTA pair
    grid = cwg.select(32, 256, 256, 14, 14)
    assert grid.order == cwg.ORDER_GRID and grid.ctas_launched == grid.ctas == 52
    # 25 tile blocks of one channel block below one wave: shorter equal runs on more pairs
    # (3136 tiles over 74 pairs: 48-tile runs on 66 pairs)
    small = cwg.select(4, 128, 128, 56, 56)
    assert small.ctas == 50
    if not cuda_present():
        assert small.order == cwg.ORDER_RUNS and small.ctas_launched == 2 * 66
    # config 3: 392 blocks = 5.3 waves -> 73 persistent pairs, each 688 tiles (5 x 128 + 48)
    c3 = cwg.select(64, 128, 128, 56, 56)
    assert c3.ctas == 784
    if not cuda_present():
        assert c3.order == cwg.ORDER_RUNS and c3.ctas_launched == 146
    assert c3.order in (cwg.ORDER_RUNS, cwg.ORDER_ROUND) and c3.ctas_launched < c3.ctas
    # config 5 (F(4,3), 4 channel blocks): round robin over (tile block, channel block) units
    c5 = cwg.select(128, 256, 256, 112, 112, 4, cwg.BF16)
    assert c5.ctas == 2 * 1568 * 4
    if not cuda_present():
        assert c5.order == cwg.ORDER_ROUND and c5.ctas_launched == 148
    # a split C_in keeps one unit per pair; so does the CUDA-core path
    split = cwg.select(1, 512, 512, 7, 7)
    assert split.order == cwg.ORDER_GRID and split.ctas_launched == split.ctas
    ffma = cwg.select(1, 16, 32, 56, 56)
    assert ffma.path == cwg.PATH_FFMA and ffma.order == cwg.ORDER_GRID
    assert ffma.ctas_launched == ffma.ctas


def test_selector_f43_tensor_core():
    n, c, k, h, w = 2, 128, 200, 30, 30
    tiles = n * 8 * 8  # 4x4 output tiles
    ch = cwg.select(n, c, k, h, w, 4, cwg.BF16)
    assert ch.path == cwg.PATH_TC and ch.m == 4 and ch.mma_products == 2
    assert ch.tiles_per_cta == 64 and ch.cout_per_cta == 128
    # a CTA pair per (64-tile block, 128-channel block, pass of two output rows)
    assert ch.ctas == 2 * 2 * (-(-tiles // 64)) * (-(-k // 128))
    # weights: [ceil(C_out/128)][2 passes][2 ranks][C_in/16][30 f] fp16 blocks of
    # 128 rows (128 channels of one output row) x 16 channels; a pass stores the
    # 30 frequencies its At rows do not zero; CWG_TC_X3: bf16 hi and lo blocks
    assert cwg.weight_bytes(c, k, 4, cwg.BF16) == 2 * 2 * 2 * 8 * 30 * 4096
    x3 = cwg.select(n, c, k, h, w, 4, cwg.BF16 | cwg.TC_X3)
    assert x3.path == cwg.PATH_TC and x3.mma_products == 3
    assert cwg.weight_bytes(c, k, 4, cwg.BF16 | cwg.TC_X3) == 2 * 2 * 2 * 8 * 30 * 2 * 4096
    # bf16 F(2,3) runs single products; fp32 F(2,3) the hi/lo split
    assert cwg.select(n, c, k, h, w, 0, cwg.BF16).mma_products == 1
    assert cwg.select(n, c, k, h, w, 2).mma_products == 3
    assert cwg.select(1, 32, 32, 8, 8, 4).mma_products == 0  # FFMA
    # fp32 F(4,3) stays on the CUDA cores (tensor-core error above the fp32 bar)
    assert cwg.select(n, c, k, h, w, 4).path == cwg.PATH_FFMA
    # the single-CTA tensor-core kernels are F(2,3) only
    assert cwg.select(n, c, k, h, w, 4, cwg.BF16 | cwg.TC_NOPAIR).path == cwg.PATH_FFMA
    for fl in (cwg.FORCE_TC, cwg.BF16 | cwg.TC_NOPAIR | cwg.FORCE_TC):
        with pytest.raises(cwg.CwgError) as e:
            cwg.select(n, c, k, h, w, 4, fl)
        assert e.value.status == cwg.EUNSUPPORTED


def test_nonfused_workspace_and_argument_checks():
    # F(2,3) (tensor-core GEMM): U and V as UMMA blocks of 128 rows x 16 channels, hi and lo
    # bf16 (8 KiB per block pair), rows padded to 128 and channels to 16; M fp32
    T = 2 * 28 * 28
    blocks = lambda rows, c: 16 * -(-rows // 128) * -(-c // 16) * 8192  # noqa: E731
    assert cwg.nonfused_workspace_bytes(2, 32, 48, 56, 56, 2) == \
        blocks(48, 32) + blocks(T, 32) + 16 * 48 * T * 4
    # F(4,3), F(6,3) (FFMA GEMM): V[td^2][C][T] + M[td^2][K][T] fp32, each rounded up to 256
    T4 = 1 * 3 * 3
    b = cwg.nonfused_workspace_bytes(1, 5, 7, 9, 10, 4)
    assert b == -(-36 * 5 * T4 * 4 // 256) * 256 + -(-36 * 7 * T4 * 4 // 256) * 256
    assert cwg.nonfused_workspace_bytes(1, 8, 8, 8, 8, 8) == 0
    assert cwg.nonfused_workspace_bytes(1, 8, 8, 12, 12, 6) == 2 * (64 * 8 * 4 * 4)
    L = cwg.lib()
    ws = cwg.nonfused_workspace_bytes(1, 8, 8, 8, 8, 2)
    # bf16 / path flags, missing or short workspace: rejected before any CUDA call
    assert L.cwg_conv3x3_nonfused(0x1000, 0x2000, None, 0x3000, 0x4000, ws, 1, 8, 8, 8, 8, 2,
                                  cwg.BF16, None) == cwg.EINVAL
    assert L.cwg_conv3x3_nonfused(0x1000, 0x2000, None, 0x3000, None, ws, 1, 8, 8, 8, 8, 2, 0,
                                  None) == cwg.EINVAL
    assert L.cwg_conv3x3_nonfused(0x1000, 0x2000, None, 0x3000, 0x4000, ws - 1, 1, 8, 8, 8, 8, 2,
                                  0, None) == cwg.EINVAL
    assert L.cwg_conv3x3_nonfused(0x1000, 0x2000, None, 0x3000, 0x4000, ws, 1, 8, 8, 8, 8, 8, 0,
                                  None) == cwg.EINVAL


def test_layer_call_argument_checks_need_no_gpu():
    L = cwg.lib()
    # NULL pointers / bad sizes are rejected before any CUDA call
    assert L.cwg_conv3x3_fused(None, None, None, None, 1, 8, 8, 8, 8, 2, 0, None) == cwg.EINVAL
    assert L.cwg_conv3x3_fused(None, None, None, None, -1, 8, 8, 8, 8, 2, 0, None) == cwg.EINVAL
    assert L.cwg_conv3x3_fused(None, None, None, None, 0, 8, 8, 8, 8, 2, 0, None) == cwg.OK
    # misaligned device pointers (checked on the host)
    assert L.cwg_conv3x3_fused(0x1001, 0x2000, None, 0x3000, 1, 8, 8, 8, 8, 2, 0,
                               None) == cwg.EINVAL
    assert L.cwg_weight_transform(None, None, 8, 8, 2, 0, None) == cwg.EINVAL
    assert L.cwg_weight_import(0x1000, 0x2000, 8, 8, 0, 0, None) == cwg.EINVAL
    assert L.cwg_conv3x3_fused_host(None, None, None, None, None, 0, 1, 8, 8, 8, 8, 2, 0,
                                    None) == cwg.EINVAL
    assert cwg.host_workspace_bytes(2, 3, 4, 5, 6) == 768 + 1024  # 720 B, 960 B, 256-aligned
    assert cwg.host_workspace_bytes(1, 64, 64, 56, 56) == 2 * 64 * 56 * 56 * 4


def test_tiles_argument_checks_need_no_gpu():
    L = cwg.lib()
    fp = ctypes.POINTER(ctypes.c_float)
    a = np.zeros(64, np.float32).ctypes.data_as(fp)
    assert L.cwg_tiles_fused(a, a, a, 1, 1, 1, 5) == cwg.EINVAL
    assert L.cwg_tiles_fused(a, a, a, 1, 0, 1, 4) == cwg.EINVAL
    assert L.cwg_tiles_fused(None, None, None, 1, 1, 1, 4) == cwg.EINVAL
    assert L.cwg_tiles_fused(None, None, None, 0, 1, 1, 4) == cwg.OK
    assert L.cwg_last_status() == cwg.OK


def test_fused_winograd_kernel_mirror_rejects_bad_td():
    from fused_winograd_kernel import FusedWinogradKernel, _TRANSFORMS

    k = FusedWinogradKernel(trace_file=None)
    with pytest.raises(ValueError):
        k.run_fused(np.zeros((2, 5, 5), np.float32), np.zeros((3, 2, 5, 5), np.float32))
    assert sorted(_TRANSFORMS) == [4, 6, 8]
    assert k.BT.shape == (4, 4) and k.AT.shape == (2, 4)


def test_mirror_tables_equal_reference_values():
    from fused_winograd_kernel import _TRANSFORMS
    from conftest import load_golden  # noqa: F401  (tables are checked numerically below)

    # Bt and At must turn a 3x3 correlation into Winograd form with the derived G
    G = {4: np.array([[1, 0, 0], [.5, .5, .5], [.5, -.5, .5], [0, 0, 1]]),
         6: np.array([[1 / 4, 0, 0], [-1 / 6, -1 / 6, -1 / 6], [-1 / 6, 1 / 6, -1 / 6],
                      [1 / 24, 1 / 12, 1 / 6], [1 / 24, -1 / 12, 1 / 6], [0, 0, 1]])}
    for td, Gm in G.items():
        BT, AT = (t.astype(np.float64) for t in _TRANSFORMS[td])
        m = td - 2
        for i in range(m):
            for k in range(3):
                for j in range(td):
                    s = sum(AT[i, f] * Gm[f, k] * BT[f, j] for f in range(td))
                    assert abs(s - (1.0 if j == i + k else 0.0)) < 1e-12
