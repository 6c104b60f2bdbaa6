"""GPU parity: the CUDA path (through the C ABI) against the oracle.

fp32 F(2,3): max abs <= 1e-4 and normwise rel <= 1e-3 against the reference's
own C kernel (compiled from source) driven over the layer; fp32 F(4,3): the
same abs bar and rel <= 5e-3 against the C restatement of run_fused; bf16:
normwise rel <= 1e-2 against an fp64 direct convolution of the bf16-rounded
inputs and weights.  (Tolerances live in conftest.TOL.)
"""
import numpy as np
import pytest

import cwg
import oracle
import workloads
from conftest import assert_close, load_golden

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def make_U(g, c, k, m, flags, dev, U_ref=None):
    import torch

    nbytes = cwg.weight_bytes(c, k, m, flags)
    if nbytes == 0:  # the selector refuses this layer: raise its status
        cwg.select(1, c, k, 8, 8, m, flags)
    U = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    if U_ref is not None:
        cwg.weight_import(_t(U_ref, dev), U, c, k, m, flags)
    else:
        cwg.weight_transform(_t(g, dev), U, c, k, m, flags)
    return U


def gpu_conv(x, g, bias, m, flags, dev, U_ref=None, U=None):
    import torch

    n, c, h, w = x.shape
    k = g.shape[0] if g is not None else U_ref.shape[0]
    bf = bool(flags & cwg.BF16)
    dt = torch.bfloat16 if bf else torch.float32
    x_d = _t(x, dev, dt)
    if U is None:
        U = make_U(g, c, k, m, flags, dev, U_ref)
    b_d = None if bias is None else _t(bias, dev)
    y_d = torch.full((n, k, h, w), float("nan"), dtype=dt, device=dev)
    cwg.conv3x3_fused(x_d, U, b_d, y_d, n, c, k, h, w, m, flags)
    cwg.device_status()
    return y_d.float().cpu().numpy()


def oracle_conv(x, g, bias, m, relu):
    """Reference C for F(2,3) (when built), C restatement for F(4,3) and F(6,3)."""
    td = m + 2
    U = oracle.weight_transform(g, td)
    if m == 2 and oracle.ref_available():
        return oracle.ref_conv_layer_f23(x, U, bias, relu)
    return oracle.conv_layer(x, U, bias, td, relu)


# ---- per-tile entry points ------------------------------------------------------
@pytest.mark.parametrize("td", [4, 6, 8])
def test_tiles_api_vs_reference_run_fused(cuda_dev, td):
    z = load_golden(f"tiles_td{td}.npz")
    i = 0
    while f"tiles_{i}" in z:
        got = cwg.tiles_fused(z[f"tiles_{i}"], z[f"U_{i}"])
        ref = z[f"run_fused_{i}"]
        err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
        assert err < (1e-5 if td == 8 else 2e-6), (td, i, err)
        if td == 4:  # same operation order as the reference C: bit-identical
            np.testing.assert_array_equal(got, z[f"ref_c_{i}"])
        i += 1


def test_fused_winograd_f23_symbol_bit_exact(cuda_dev):
    z = load_golden("tiles_td4.npz")
    for i in range(2):
        for t in range(z[f"tiles_{i}"].shape[0]):
            out = cwg.fused_winograd_f23(z[f"tiles_{i}"][t], z[f"U_{i}"])
            np.testing.assert_array_equal(out, z[f"ref_c_{i}"][t])


def test_reference_class_mirror(cuda_dev, tmp_path):
    from fused_winograd_kernel import FusedWinogradKernel

    k = FusedWinogradKernel(trace_file=str(tmp_path / "trace.json"))
    for td in (4, 6, 8):
        z = load_golden(f"tiles_td{td}.npz")
        tiles, U = z["tiles_0"], z["U_0"]
        for t in range(tiles.shape[0]):
            for fn, key in ((k.run_fused, "run_fused_0"), (k.run_non_fused, "run_non_fused_0")):
                y = fn(tiles[t], U)
                ref = z[key][t]
                assert y.shape == ref.shape
                # normwise: F(6,3)'s coefficients (up to 32) amplify summation order
                assert np.abs(y - ref).max() / np.abs(ref).max() < (1e-5 if td == 8 else 2e-6)
        # batched form
        ref = z["run_fused_0"]
        assert np.abs(k.run_fused(tiles, U) - ref).max() / np.abs(ref).max() < 1e-5
    assert (tmp_path / "trace.json").exists()


def test_reference_class_conv2d(cuda_dev):
    from fused_winograd_kernel import FusedWinogradKernel

    z = load_golden("layer_f23_wide.npz")
    y = FusedWinogradKernel(trace_file=None).conv2d(z["x"], z["g"], z["bias"], m=2, relu=True)
    assert_close(y, z["y"], "f23", "conv2d")


# ---- layer API against the goldens --------------------------------------------
@pytest.mark.parametrize("name", ["f23_odd", "f23_pixel", "f23_wide", "f43_odd", "f43_small"])
@pytest.mark.parametrize("how", ["import", "transform"])
def test_layer_goldens(cuda_dev, name, how):
    z = load_golden(f"layer_{name}.npz")
    N, C, K, H, W, td, relu, _ = (int(v) for v in z["meta"])
    m = td - 2
    flags = cwg.RELU if relu else 0
    bias = z.get("bias")
    y = gpu_conv(z["x"], z["g"], bias, m, flags, cuda_dev,
                 U_ref=z["U"] if how == "import" else None)
    assert_close(y, z["y"], "f23" if m == 2 else "f43", name)


@pytest.mark.parametrize("case", [(1, 8, 8, 12, 12), (2, 21, 35, 17, 23), (1, 128, 128, 60, 60),
                                  (1, 64, 64, 7, 7)], ids=lambda c: "x".join(map(str, c)))
def test_layer_f63(cuda_dev, case):
    """F(6x6,3x3) on the CUDA-core kernel against the C restatement of run_fused
    (td = 8, the reference's _BT_8/_AT_8)."""
    n, c, k, h, w = case
    rng = np.random.default_rng(sum(case) + 700)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    y = gpu_conv(x, g, bias, 6, cwg.RELU, cuda_dev)
    U = oracle.weight_transform(g, 8)
    assert_close(y, oracle.conv_layer(x, U, bias, 8, True), "f63", str(case))


def test_layer_f63_bf16(cuda_dev):
    rng = np.random.default_rng(701)
    x = workloads.bf16_round(rng.uniform(-1, 1, (2, 64, 30, 30)).astype(np.float32))
    g = workloads.bf16_round(rng.normal(0, np.sqrt(2 / 576), (48, 64, 3, 3)).astype(np.float32))
    bias = rng.uniform(-0.1, 0.1, 48).astype(np.float32)
    y = gpu_conv(x, g, bias, 6, cwg.BF16 | cwg.RELU, cuda_dev)
    assert_close(y, oracle.direct_conv_f64(x, g, bias, True), "bf16", "bf16 F(6,3)")


# ---- the benchmark configurations -----------------------------------------------
def _run_cfg_layer(layer, dev, n=None):
    g, bias = workloads.make_weights(layer)
    x = workloads.make_input(layer, n)
    flags = (cwg.RELU if layer.relu else 0) | (cwg.BF16 if layer.bf16 else 0)
    y = gpu_conv(x, g, bias, layer.m, flags, dev)
    return x, g, bias, y


def test_config1(cuda_dev):
    (layer,) = workloads.config_layers(1)
    x, g, bias, y = _run_cfg_layer(layer, cuda_dev)
    assert_close(y, oracle_conv(x, g, bias, 2, layer.relu), "f23", layer.name)


@pytest.mark.parametrize("idx", range(14))
def test_config2_channel_sweep(cuda_dev, idx):
    layer = workloads.config_layers(2)[idx]
    x, g, bias, y = _run_cfg_layer(layer, cuda_dev)
    ref = oracle_conv(x, g, bias, layer.m, layer.relu)
    assert_close(y, ref, "f23" if layer.m == 2 else "f43", layer.name)


def test_config3_full_batch(cuda_dev):
    (layer,) = workloads.config_layers(3)
    x, g, bias, y = _run_cfg_layer(layer, cuda_dev)
    assert_close(y, oracle_conv(x, g, bias, 2, True), "f23", layer.name)


def test_config4_resnet18_stack(cuda_dev):
    """Layers chain within a stage; images 0 and N-1 of every layer are checked
    against the reference C on the very inputs the GPU layer received."""
    import torch

    layers = workloads.config_layers(4)
    sample = [0, layers[0].n - 1]
    prev_stage = None
    for layer in layers:
        g, bias = workloads.make_weights(layer)
        flags = cwg.RELU
        if layer.c_in != prev_stage:
            x_d = _t(workloads.make_input(layer), cuda_dev)
            prev_stage = layer.c_in
        n, c, h, w = x_d.shape
        U = make_U(g, c, layer.c_out, 2, flags, cuda_dev)
        y_d = torch.empty((n, layer.c_out, h, w), dtype=torch.float32, device=cuda_dev)
        cwg.conv3x3_fused(x_d, U, _t(bias, cuda_dev), y_d, n, c, layer.c_out, h, w, 2, flags)
        cwg.device_status()
        xs = x_d[sample].cpu().numpy()
        ys = y_d[sample].cpu().numpy()
        assert_close(ys, oracle_conv(xs, g, bias, 2, True), "f23", layer.name)
        x_d = y_d


def test_config5_bf16_sampled(cuda_dev):
    (layer,) = workloads.config_layers(5)
    g, bias = workloads.make_weights(layer)
    x = workloads.make_input(layer)
    flags = cwg.RELU | cwg.BF16
    y = gpu_conv(x, g, bias, layer.m, flags, cuda_dev)
    for i in (0, layer.n - 1):
        ref = oracle.direct_conv_f64(x[i:i + 1], g, bias, True)
        assert_close(y[i:i + 1], ref, "bf16", f"{layer.name} image {i}")


# ---- edge cases ---------------------------------------------------------------
EDGE = [
    # n, c, k, h, w, m, relu, bias
    (1, 1, 1, 1, 1, 2, False, False),
    (1, 1, 1, 1, 1, 4, True, True),
    (2, 3, 5, 3, 3, 2, True, True),
    (1, 3, 5, 5, 7, 4, False, True),
    (3, 7, 17, 7, 7, 2, False, True),
    (1, 9, 33, 9, 13, 4, True, False),
    (2, 16, 65, 6, 6, 2, True, True),
    (1, 17, 16, 31, 2, 2, False, True),
    (1, 40, 24, 2, 31, 4, True, True),
    (1, 128, 128, 1, 1, 2, False, True),
    (1, 64, 64, 3, 3, 2, True, True),
    (1, 96, 128, 10, 10, 2, True, True),
    (5, 128, 256, 7, 7, 2, True, True),
    (1, 48, 192, 9, 15, 2, False, True),
]


@pytest.mark.parametrize("case", EDGE, ids=lambda c: "x".join(map(str, c[:6])))
def test_edge_shapes(cuda_dev, case):
    n, c, k, h, w, m, relu, use_bias = case
    rng = np.random.default_rng(hash(case) % 2 ** 32)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32) if use_bias else None
    y = gpu_conv(x, g, bias, m, cwg.RELU if relu else 0, cuda_dev)
    assert_close(y, oracle_conv(x, g, bias, m, relu), "f23" if m == 2 else "f43", str(case))


@pytest.mark.parametrize("force", [cwg.FORCE_FFMA, 0])
@pytest.mark.parametrize("case", [(2, 32, 64, 9, 11, 2), (1, 64, 128, 12, 12, 4),
                                  (2, 128, 128, 14, 14, 2)])
def test_bf16_layers(cuda_dev, case, force):
    n, c, k, h, w, m = case
    rng = np.random.default_rng(11)
    x = workloads.bf16_round(rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32))
    g = workloads.bf16_round(rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32))
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    flags = cwg.BF16 | cwg.RELU | force
    try:
        y = gpu_conv(x, g, bias, m, flags, cuda_dev)
    except cwg.CwgError as e:
        assert e.status == cwg.EUNSUPPORTED and force == 0
        return
    assert_close(y, oracle.direct_conv_f64(x, g, bias, True), "bf16", str(case))


def test_paths_agree(cuda_dev):
    """The FFMA and tensor-core kernels agree on a layer both can run."""
    rng = np.random.default_rng(12)
    n, c, k, h, w = 2, 128, 128, 20, 18
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    ref = oracle_conv(x, g, bias, 2, True)
    for force in (cwg.FORCE_FFMA, cwg.FORCE_TC):
        try:
            y = gpu_conv(x, g, bias, 2, cwg.RELU | force, cuda_dev)
        except cwg.CwgError as e:
            assert e.status == cwg.EUNSUPPORTED and force == cwg.FORCE_TC
            continue
        assert_close(y, ref, "f23", f"force={force:#x}")


TC_VARIANTS = [0, cwg.TC_NOPAIR, cwg.TC_FULL16]


@pytest.mark.parametrize("variant", TC_VARIANTS, ids=["pair", "single", "full16"])
@pytest.mark.parametrize("case", [(2, 128, 128, 20, 18), (1, 64, 200, 9, 13),
                                  (3, 96, 128, 7, 7), (1, 256, 64, 3, 33)],
                         ids=lambda c: "x".join(map(str, c)))
def test_tensor_core_variants(cuda_dev, case, variant):
    """Every tcgen05 kernel (2-SM pair, single-CTA half-folded, 16-accumulator)
    against the reference on ragged shapes: partial channel blocks, tile blocks
    that cross images, a last block with no valid tile on one CTA of the pair."""
    n, c, k, h, w = case
    rng = np.random.default_rng(sum(case) + variant)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    y = gpu_conv(x, g, bias, 2, cwg.RELU | cwg.FORCE_TC | variant, cuda_dev)
    assert_close(y, oracle_conv(x, g, bias, 2, True), "f23", f"{case} {variant:#x}")


@pytest.mark.parametrize("variant", TC_VARIANTS, ids=["pair", "single", "full16"])
def test_tensor_core_variants_bf16(cuda_dev, variant):
    n, c, k, h, w = 2, 128, 192, 14, 14
    rng = np.random.default_rng(21)
    x = workloads.bf16_round(rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32))
    g = workloads.bf16_round(rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32))
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    y = gpu_conv(x, g, bias, 2, cwg.BF16 | cwg.RELU | cwg.FORCE_TC | variant, cuda_dev)
    assert_close(y, oracle.direct_conv_f64(x, g, bias, True), "bf16", f"bf16 {variant:#x}")


F43_TC = [(2, 64, 64, 9, 13), (1, 96, 200, 7, 7), (3, 128, 64, 5, 22), (1, 64, 128, 24, 24)]


@pytest.mark.parametrize("products", [0, cwg.TC_X3], ids=["fp16x2", "bf16x3"])
@pytest.mark.parametrize("case", F43_TC, ids=lambda c: "x".join(map(str, c)))
def test_tensor_core_f43_bf16(cuda_dev, case, products):
    """F(4,3) on the pair kernel (6 accumulators, one output row per CTA and pass) for
    bf16 layers, in both product modes (fp16 U * (V_hi + V_lo), the default, and
    the bf16 hi/lo split of CWG_TC_X3): ragged tiles, partial channel blocks,
    tile blocks across images."""
    n, c, k, h, w = case
    rng = np.random.default_rng(sum(case) + 500)
    x = workloads.bf16_round(rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32))
    g = workloads.bf16_round(rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32))
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    y = gpu_conv(x, g, bias, 4, cwg.BF16 | cwg.RELU | cwg.FORCE_TC | products, cuda_dev)
    assert_close(y, oracle.direct_conv_f64(x, g, bias, True), "bf16", f"bf16 {case}")


def test_fp16_products_report_range_overflow(cuda_dev):
    """bf16 data whose Winograd transform leaves fp16's range (|V| up to 100 |x| for
    F(4,3)) cannot run the fp16 products: the kernel finishes, sets the range bit
    and cwg_device_status reports CWG_ERANGE; CWG_TC_X3 runs the same layer
    correctly.  Weights beyond fp16's range are reported by the transform."""
    import torch

    n, c, k, h, w = 1, 64, 64, 12, 12
    rng = np.random.default_rng(77)
    x = workloads.bf16_round(rng.uniform(-2000, 2000, (n, c, h, w)).astype(np.float32))
    g = workloads.bf16_round(rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32))
    bias = np.zeros(k, np.float32)
    flags = cwg.BF16 | cwg.FORCE_TC
    with pytest.raises(cwg.CwgError) as e:
        gpu_conv(x, g, bias, 4, flags, cuda_dev)
    assert e.value.status == cwg.ERANGE
    cwg.device_status()  # the status word was cleared
    y = gpu_conv(x, g, bias, 4, flags | cwg.TC_X3, cuda_dev)
    assert_close(y, oracle.direct_conv_f64(x, g, bias, False), "bf16", "bf16x3, large inputs")
    # weights: |g| = 1e5 overflows fp16 in the transform itself
    U = torch.empty(cwg.weight_bytes(c, k, 4, flags), dtype=torch.uint8, device=cuda_dev)
    g_big = torch.from_numpy(np.full((k, c, 3, 3), 1e5, np.float32)).to(cuda_dev)
    cwg.weight_transform(g_big, U, c, k, 4, flags)
    with pytest.raises(cwg.CwgError) as e:
        cwg.device_status()
    assert e.value.status == cwg.ERANGE


# Layers above one wave of CTA pairs run persistent pairs: each pair walks an
# equal run of tiles in items of up to N tiles (the last a short one, MMA N
# rounded up to 16, possibly empty on the pair's second CTA), every
# output-channel block per tile block, with the next item's first stage written
# ahead of the current item's epilogue.
PERSISTENT = [
    # n, c, k, h, w, m, flags
    (13, 64, 136, 56, 56, 2, 0),                    # fp32 F(2,3), 2 ragged channel blocks
    (13, 64, 64, 56, 56, 2, cwg.BF16),               # bf16 F(2,3): patches outside the V ring
    (13, 96, 64, 56, 56, 2, 0),                      # fp32 F(2,3), 64 channels: M = 128 pair
    (25, 64, 72, 56, 56, 4, cwg.BF16),               # bf16 F(4,3): a ragged block, 2 passes
    # below one wave of units: equal runs shorter than an item on more pairs
    (4, 128, 128, 56, 56, 2, 0),                     # 25 blocks -> 66 runs of 48 tiles
    (8, 64, 128, 37, 41, 2, 0),                      # odd image sizes: runs across rows
    (2, 64, 64, 64, 60, 4, cwg.BF16),                # F(4,3), 64 channels: runs of 32 tiles
    (10, 64, 128, 64, 60, 4, cwg.BF16),              # F(4,3), 2 passes: 76 units, runs
]


@pytest.mark.parametrize("case", PERSISTENT, ids=lambda c: "x".join(map(str, c[:6])))
def test_persistent_pairs(cuda_dev, case):
    n, c, k, h, w, m, extra = case
    rng = np.random.default_rng(sum(case[:6]) + 900)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    bf = bool(extra & cwg.BF16)
    if bf:
        x, g = workloads.bf16_round(x), workloads.bf16_round(g)
    ch = cwg.select(n, c, k, h, w, m, cwg.RELU | cwg.FORCE_TC | extra)
    assert ch.path == cwg.PATH_TC
    assert ch.order in (cwg.ORDER_RUNS, cwg.ORDER_ROUND), ch.order_name
    y = gpu_conv(x, g, bias, m, cwg.RELU | cwg.FORCE_TC | extra, cuda_dev)
    ref = oracle.direct_conv_f64(x, g, bias, True)
    assert_close(y, ref, "bf16" if bf else "f23", f"persistent {case}")


# F(2,3) layers of 1-4 input channels (an RGB input layer) run their own kernel:
# one thread per tile, 8-64 output channels per CTA.
SMALL_CIN = [
    # n, c, k, h, w, flags, bias
    (2, 3, 64, 56, 56, 0, True),      # even width: pair loads, 2-pixel row stores
    (1, 3, 200, 17, 23, 0, True),     # odd sizes: scalar path, ragged channel block
    (3, 2, 40, 30, 31, 0, False),     # odd width, no bias
    (1, 4, 72, 20, 20, 0, True),      # four channels
    (1, 1, 16, 9, 10, 0, True),       # one channel
    (2, 3, 64, 28, 28, cwg.BF16, True),
]


@pytest.mark.parametrize("case", SMALL_CIN, ids=lambda c: "x".join(map(str, c[:5])) + f"f{c[5]:#x}")
def test_small_cin_layers(cuda_dev, case):
    n, c, k, h, w, extra, use_bias = case
    rng = np.random.default_rng(sum(case[:5]) + 1300)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32) if use_bias else None
    flags = cwg.RELU | extra
    ch = cwg.select(n, c, k, h, w, 0, flags)
    assert ch.path == cwg.PATH_FFMA and ch.m == 2 and ch.threads == 256
    if extra & cwg.BF16:
        x, g = workloads.bf16_round(x), workloads.bf16_round(g)
        y = gpu_conv(x, g, bias, 2, flags, cuda_dev)
        assert_close(y, oracle.direct_conv_f64(x, g, bias, True), "bf16", f"small {case}")
    else:
        y = gpu_conv(x, g, bias, 2, flags, cuda_dev)
        assert_close(y, oracle_conv(x, g, bias, 2, True), "f23", f"small {case}")


@pytest.mark.parametrize("case", [
    (128, 200, 2, 0), (128, 200, 2, cwg.BF16), (128, 200, 2, cwg.TC_NOPAIR),
    (128, 200, 2, cwg.TC_FULL16), (96, 200, 4, cwg.BF16), (32, 40, 2, 0), (32, 40, 4, cwg.BF16),
    (80, 64, 2, 0), (80, 64, 2, cwg.BF16),  # the 64-channel pair kernel's 64-row blocks
    (96, 200, 4, cwg.BF16 | cwg.TC_X3),  # F(4,3) in two passes, bf16 hi and lo
    (80, 64, 4, cwg.BF16), (80, 64, 4, cwg.BF16 | cwg.TC_X3)],  # F(4,3), 64 channels, one pass
    ids=lambda c: f"c{c[0]}k{c[1]}m{c[2]}f{c[3]:#x}")
def test_weight_transform_stays_in_its_buffer(cuda_dev, case):
    """Every weight layout is written exactly inside cwg_weight_bytes: guard
    bytes on both sides of the buffer keep their poison."""
    import torch

    c, k, m, flags = case
    g = np.random.default_rng(7).normal(0, 0.1, (k, c, 3, 3)).astype(np.float32)
    nb = cwg.weight_bytes(c, k, m, flags)
    guard = 4096
    buf = torch.full((nb + 2 * guard,), 0xA5, dtype=torch.uint8, device=cuda_dev)
    U = buf[guard:guard + nb]
    cwg.weight_transform(_t(g, cuda_dev), U, c, k, m, flags)
    torch.cuda.synchronize()
    assert bool((buf[:guard] == 0xA5).all()) and bool((buf[guard + nb:] == 0xA5).all())
    assert not bool((U == 0xA5).all())


@pytest.mark.parametrize("case", [(2, 32, 48, 15, 17, 2), (1, 128, 128, 56, 56, 2),
                                  (3, 144, 200, 11, 13, 2), (1, 16, 8, 1, 1, 2),
                                  (1, 64, 64, 21, 19, 4), (2, 16, 32, 9, 9, 4),
                                  (1, 32, 40, 20, 26, 6), (1, 70, 130, 9, 9, 4)],
                         ids=lambda c: "x".join(map(str, c)))
def test_nonfused_ablation_matches_reference(cuda_dev, case):
    """The three-pass ablation (input transform -> HBM -> per-frequency GEMM: tcgen05 bf16x3
    for F(2,3), fp32 FFMA for F(4,3)/F(6,3) -> output transform) computes the same layer;
    ragged tile blocks (T not a multiple of 128), channel counts not multiples of 16 or 128,
    a one-pixel image."""
    import torch

    n, c, k, h, w, m = case
    rng = np.random.default_rng(sum(case) + 600)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    U = make_U(g, c, k, m, cwg.FORCE_FFMA, cuda_dev)
    ws_b = cwg.nonfused_workspace_bytes(n, c, k, h, w, m)
    ws = torch.empty(ws_b, dtype=torch.uint8, device=cuda_dev)
    y = torch.full((n, k, h, w), float("nan"), device=cuda_dev)
    cwg.conv3x3_nonfused(_t(x, cuda_dev), U, _t(bias, cuda_dev), y, ws, ws_b, n, c, k, h, w, m,
                         cwg.RELU)
    cwg.device_status()
    ref = oracle_conv(x, g, bias, m, True)
    assert_close(y.cpu().numpy(), ref, {2: "f23", 4: "f43", 6: "f63"}[m], str(case))


@pytest.mark.parametrize("case", [(1, 512, 512, 7, 7, True, True), (1, 256, 256, 14, 14, False, False),
                                  (1, 128, 128, 28, 28, True, False), (2, 64, 200, 12, 12, True, True),
                                  (1, 96, 64, 9, 5, True, False), (1, 128, 96, 16, 16, False, True)],
                         ids=lambda c: "x".join(map(str, c)))
def test_split_reduction_small_layers(cuda_dev, case):
    """Small fp32 layers split C_in across CTAs (partial sums added into y; bias with
    slice 0, or bias and ReLU in a second pass): same result as the unsplit kernel and
    the reference."""
    n, c, k, h, w, use_bias, relu = case
    rng = np.random.default_rng(sum(case) + 800)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32) if use_bias else None
    assert cwg.select(n, c, k, h, w).ctas > cwg.select(n, c, k, h, w, 2, cwg.NO_SPLIT).ctas
    fl = cwg.RELU if relu else 0
    y = gpu_conv(x, g, bias, 2, fl, cuda_dev)
    y1 = gpu_conv(x, g, bias, 2, fl | cwg.NO_SPLIT, cuda_dev)
    y2 = gpu_conv(x, g, bias, 2, fl | cwg.NO_SPLIT, cuda_dev)
    np.testing.assert_array_equal(y1, y2)  # unsplit: bit-reproducible
    ref = oracle_conv(x, g, bias, 2, relu)
    assert_close(y, ref, "f23", f"split {case}")
    assert_close(y, y1, "f23", f"split vs unsplit {case}")


@pytest.mark.parametrize("case", [(1, 256, 256, 14, 14, 4, True, False), (1, 512, 512, 7, 7, 4, True, True),
                                  (1, 64, 32, 56, 56, 4, False, True), (1, 200, 48, 23, 19, 4, True, False),
                                  (1, 128, 40, 30, 30, 6, True, True), (1, 96, 24, 17, 9, 2, True, True)],
                         ids=lambda c: "x".join(map(str, c)))
def test_ffma_split_reduction(cuda_dev, case):
    """Single-image fp32 layers on the CUDA-core kernel whose grid leaves most SMs
    idle split their C_in steps across CTAs: same result as the unsplit kernel and
    the reference, with and without bias and ReLU."""
    n, c, k, h, w, m, use_bias, relu = case
    rng = np.random.default_rng(sum(case) + 900)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32) if use_bias else None
    fl = cwg.FORCE_FFMA | (cwg.RELU if relu else 0)
    sel = cwg.select(n, c, k, h, w, m, fl)
    blocks = n * (-(-h // (4 * m))) * (-(-w // (4 * m)))  # 4x4 output tiles per CTA
    assert sel.path == cwg.PATH_FFMA and sel.tiles_per_cta == 16
    assert sel.ctas > blocks * (-(-k // sel.cout_per_cta))  # C_in slices
    y = gpu_conv(x, g, bias, m, fl, cuda_dev)
    y1 = gpu_conv(x, g, bias, m, fl | cwg.NO_SPLIT, cuda_dev)
    tol = {2: "f23", 4: "f43", 6: "f63"}[m]
    assert_close(y, oracle_conv(x, g, bias, m, relu), tol, f"ffma split {case}")
    assert_close(y, y1, tol, f"ffma split vs unsplit {case}")


def _random_cases(count, seed=2024):
    """Seeded layer shapes across every kernel the selector can pick: tensor-core
    pairs (both channel counts >= 64), CUDA-core blocks with or without C_in slices,
    the 1-4 input-channel kernel; fp32 and bf16, odd sizes, bias and ReLU on or off."""
    rng = np.random.default_rng(seed)
    cases = []
    for i in range(count):
        regime = i % 3
        bf16 = bool(rng.random() < 0.3)
        if regime == 0:  # tensor cores
            c, k = int(rng.integers(64, 145)), int(rng.integers(64, 145))
            m = 4 if bf16 and rng.random() < 0.5 else 2
        elif regime == 1:  # CUDA cores
            c, k = int(rng.integers(5, 97)), int(rng.integers(1, 64))
            m = int(rng.choice([2, 4, 6]))
        else:  # 1-4 input channels
            c, k, m = int(rng.integers(1, 5)), int(rng.integers(1, 97)), 2
        n = int(rng.integers(1, 3))
        h, w = int(rng.integers(1, 25)), int(rng.integers(1, 25))
        extra = int(rng.choice([0, 0, cwg.NO_SPLIT, cwg.FORCE_FFMA]))
        cases.append((n, c, k, h, w, m, bf16, bool(rng.random() < 0.5), bool(rng.random() < 0.7), extra))
    return cases


@pytest.mark.parametrize("case", _random_cases(24), ids=lambda c: "x".join(map(str, c[:7])))
def test_random_layers(cuda_dev, case):
    """A seeded sweep of layer shapes against the oracle (fp32: the reference C for
    F(2,3), the C restatement for F(4,3)/F(6,3); bf16: fp64 direct convolution of
    the bf16-rounded operands)."""
    n, c, k, h, w, m, bf16, relu, use_bias, extra = case
    rng = np.random.default_rng(abs(hash(case)) % 2 ** 32)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32) if use_bias else None
    flags = extra | (cwg.RELU if relu else 0)
    if bf16:
        x, g = workloads.bf16_round(x), workloads.bf16_round(g)
        y = gpu_conv(x, g, bias, m, flags | cwg.BF16, cuda_dev)
        assert_close(y, oracle.direct_conv_f64(x, g, bias, relu), "bf16", str(case))
    else:
        y = gpu_conv(x, g, bias, m, flags, cuda_dev)
        assert_close(y, oracle_conv(x, g, bias, m, relu), {2: "f23", 4: "f43", 6: "f63"}[m],
                     str(case))


def test_bounded_wait_times_out_and_context_survives(cuda_dev):
    """A device wait on a barrier nothing arrives on gives up after its limit, the host
    reads CWG_ETIMEOUT, the status clears, and the next layer runs normally."""
    cwg.selftest_wait_timeout()
    with pytest.raises(cwg.CwgError) as e:
        cwg.device_status()
    assert e.value.status == cwg.ETIMEOUT
    cwg.device_status()  # read and cleared
    rng = np.random.default_rng(15)
    x = rng.uniform(-1, 1, (1, 64, 12, 12)).astype(np.float32)
    g = rng.normal(0, 0.05, (64, 64, 3, 3)).astype(np.float32)
    y = gpu_conv(x, g, None, 2, cwg.RELU, cuda_dev)
    assert_close(y, oracle_conv(x, g, None, 2, True), "f23", "after a timeout")


def test_host_buffer_entry_matches_device_entry(cuda_dev):
    import torch

    rng = np.random.default_rng(13)
    n, c, k, h, w, m = 2, 32, 48, 15, 17, 2
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    g = rng.normal(0, 0.1, (k, c, 3, 3)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    U = make_U(g, c, k, m, cwg.RELU, cuda_dev)
    y_dev = gpu_conv(x, g, bias, m, cwg.RELU, cuda_dev, U=U)
    ws_b = cwg.host_workspace_bytes(n, c, k, h, w)
    ws = torch.empty(ws_b, dtype=torch.uint8, device=cuda_dev)
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.empty((n, k, h, w), dtype=torch.float32).pin_memory()
    cwg.conv3x3_fused_host(int(xh.data_ptr()), U, _t(bias, cuda_dev), int(yh.data_ptr()), ws,
                           ws_b, n, c, k, h, w, m, cwg.RELU)
    np.testing.assert_array_equal(yh.numpy(), y_dev)


def test_errors_and_launch_counter(cuda_dev):
    import torch

    before = cwg.launch_count()
    rng = np.random.default_rng(14)
    x = rng.uniform(-1, 1, (1, 8, 8, 8)).astype(np.float32)
    g = rng.normal(0, 0.1, (8, 8, 3, 3)).astype(np.float32)
    gpu_conv(x, g, None, 2, 0, cuda_dev)
    assert cwg.launch_count() >= before + 2  # weight transform + conv
    U = make_U(g, 8, 8, 2, 0, cuda_dev)
    x_d = _t(x, cuda_dev)
    y_d = torch.empty((1, 8, 8, 8), device=cuda_dev)
    with pytest.raises(cwg.CwgError) as e:  # misaligned output pointer
        cwg.conv3x3_fused(x_d, U, None, int(y_d.data_ptr()) + 2, 1, 8, 8, 8, 8, 2, 0)
    assert e.value.status == cwg.EINVAL
    # rejected on the host, before any launch
    with pytest.raises(cwg.CwgError) as e:  # no F(8x8,3x3)
        cwg.conv3x3_fused(x_d, U, None, y_d, 1, 8, 8, 8, 8, 8, 0)
    assert e.value.status == cwg.EINVAL
    with pytest.raises(cwg.CwgError) as e:  # F(6,3) has no tensor-core kernel
        cwg.conv3x3_fused(x_d, U, None, y_d, 1, 8, 8, 8, 8, 6, cwg.FORCE_TC)
    assert e.value.status == cwg.EUNSUPPORTED
    cwg.device_status()


@pytest.mark.parametrize("case", [(4, 128, 128, 28, 28, 2, 0), (2, 64, 64, 30, 34, 2, 0),
                                  (2, 256, 256, 28, 28, 4, cwg.BF16)],
                         ids=["f23", "f23_64ch", "f43bf16"])
def test_dependent_launches_ping_pong(cuda_dev, case):
    """Tensor-core layers launched back to back as programmatic dependent launches, with no
    host synchronisation: layer i reads buffer i % 2 and writes the other one, so every
    layer overwrites what the layer before it read.  The chain matches the same chain of
    ordinary launches bit for bit, and its first layer matches the oracle."""
    import torch

    n, c, k, h, w, m, extra = case
    assert c == k
    rng = np.random.default_rng(sum(case) + 77)
    bf = bool(extra & cwg.BF16)
    dt = torch.bfloat16 if bf else torch.float32
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    gs = [rng.normal(0, np.sqrt(2 / (9 * c)), (k, c, 3, 3)).astype(np.float32) for _ in range(6)]
    bias = rng.uniform(-0.1, 0.1, k).astype(np.float32)
    if bf:
        x, gs = workloads.bf16_round(x), [workloads.bf16_round(g) for g in gs]
    flags = cwg.RELU | cwg.FORCE_TC | cwg.NO_SPLIT | extra
    Us = [make_U(g, c, k, m, flags, cuda_dev) for g in gs]
    b_d = _t(bias, cuda_dev)
    stream = torch.cuda.Stream(cuda_dev)
    outs = {}
    for mode in (cwg.NO_PDL, 0):
        bufs = [_t(x, cuda_dev, dt), torch.full((n, k, h, w), float("nan"), dtype=dt,
                                                  device=cuda_dev)]
        first = torch.empty_like(bufs[1])
        torch.cuda.synchronize(cuda_dev)
        with torch.cuda.stream(stream):
            for i, U in enumerate(Us):
                cwg.conv3x3_fused(bufs[i % 2], U, b_d, bufs[(i + 1) % 2], n, c, k, h, w, m,
                                  flags | mode, stream)
                if i == 0:
                    first.copy_(bufs[1])
        stream.synchronize()
        cwg.device_status(stream)
        outs[mode] = (bufs[len(Us) % 2].float().cpu().numpy(), first.float().cpu().numpy())
    np.testing.assert_array_equal(outs[0][0], outs[cwg.NO_PDL][0])
    np.testing.assert_array_equal(outs[0][1], outs[cwg.NO_PDL][1])
    ref = oracle.direct_conv_f64(x, gs[0], bias, True)
    assert_close(outs[0][1], ref, "bf16" if bf else "f23", f"first layer {case}")
