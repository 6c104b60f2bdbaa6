"""The oracle pinned against the reference: golden vectors from the reference's
Python run_fused / run_non_fused and its C kernel compiled from source."""
import numpy as np
import pytest

import oracle
from conftest import load_golden


@pytest.mark.parametrize("td", [4, 6, 8])
def test_restatement_matches_reference_run_fused(td):
    z = load_golden(f"tiles_td{td}.npz")
    i = 0
    while f"tiles_{i}" in z:
        got = oracle.tiles_fused(z[f"tiles_{i}"], z[f"U_{i}"])
        for key in (f"run_fused_{i}", f"run_non_fused_{i}"):
            ref = z[key]
            err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
            assert err < 2e-6, (td, i, key, err)
        i += 1
    assert i > 0


def test_restatement_f23_bit_exact_vs_reference_c_golden():
    z = load_golden("tiles_td4.npz")
    for i in range(2):
        got = oracle.tiles_fused(z[f"tiles_{i}"], z[f"U_{i}"])
        np.testing.assert_array_equal(got, z[f"ref_c_{i}"])


@pytest.mark.skipif(not oracle.ref_available(), reason="reference C not built")
def test_reference_c_layer_equals_restatement_bitwise():
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, (2, 9, 11, 7)).astype(np.float32)
    g = rng.normal(0, 0.1, (6, 9, 3, 3)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 6).astype(np.float32)
    U = oracle.weight_transform(g, 4)
    for relu in (False, True):
        a = oracle.ref_conv_layer_f23(x, U, b, relu)
        c = oracle.conv_layer(x, U, b, 4, relu)
        np.testing.assert_array_equal(a, c)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference C not built")
def test_reference_c_live_matches_golden():
    z = load_golden("tiles_td4.npz")
    got = oracle.ref_tiles_f23(z["tiles_1"], z["U_1"])
    np.testing.assert_array_equal(got, z["ref_c_1"])


LAYERS = ["f23_odd", "f23_pixel", "f23_wide", "f43_odd", "f43_small", "f63_square"]


@pytest.mark.parametrize("name", LAYERS)
def test_layer_oracle_vs_golden(name):
    z = load_golden(f"layer_{name}.npz")
    N, C, K, H, W, td, relu, has_bias = (int(v) for v in z["meta"])
    bias = z.get("bias")
    # weight transform: same fp64 math, rounded once
    U = oracle.weight_transform(z["g"], td)
    np.testing.assert_allclose(U, z["U"], rtol=2e-7, atol=1e-9)
    y = oracle.conv_layer(z["x"], z["U"], bias, td, bool(relu))
    scale = max(np.abs(z["y"]).max(), 1e-30)
    # numpy's matmul/einsum sum in another order; F(6,3)'s large coefficients
    # amplify that rounding difference
    assert np.abs(y - z["y"]).max() / scale < (1e-5 if td == 8 else 2e-6)
    yd = oracle.direct_conv_f64(z["x"], z["g"], bias, bool(relu))
    np.testing.assert_allclose(yd, z["y_direct"], rtol=1e-12, atol=1e-12)
    # Winograd restatement agrees with the independent fp64 direct conv
    assert np.abs(y - yd).max() < (1e-6 if td == 4 else 2e-5)


def test_zero_skip_semantics():
    # the reference skips U == 0 terms, so 0 * inf never reaches the sum
    tiles = np.zeros((1, 1, 4, 4), np.float32)
    tiles[0, 0, 1, 1] = np.inf
    U = np.zeros((1, 1, 4, 4), np.float32)
    out = oracle.tiles_fused(tiles, U)
    np.testing.assert_array_equal(out, 0.0)


def test_bf16_rounding_matches_torch():
    import torch

    rng = np.random.default_rng(3)
    a = (rng.standard_normal(10000) * 10.0 ** rng.integers(-5, 5, 10000)).astype(np.float32)
    a[:4] = [0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8]
    ours = oracle.round_bf16(a)
    ref = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(ours, ref)


def test_workload_bf16_round_matches_oracle():
    import workloads

    rng = np.random.default_rng(4)
    a = rng.standard_normal(5000).astype(np.float32) * 3
    np.testing.assert_array_equal(workloads.bf16_round(a), oracle.round_bf16(a))
