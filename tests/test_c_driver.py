"""The reference's own kind of caller: a C program that declares the kernel entry point
itself and links against the library, the way the reference's generated benchmark drivers
do (benchmarks/ws_model_validation.py:80-92, benchmarks/register_spill_instrument.py:150-170:
an `extern void fused_winograd_f23(...)` declaration, caller-owned host buffers, the call in
a loop).  Here the program fills its buffers from a fixed integer generator instead of
calloc, so that the test can rebuild the same inputs and compare the output bytes with the
reference's C kernel (oracle/_ref).

CPU: the program compiles and links against libcwg.so with `-I include -lcwg` (and also
through include/cwg.h).  GPU: it runs, and its output equals the reference's bit for bit."""
import os
import subprocess

import numpy as np
import pytest

import cwg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.dirname(cwg.LIB_PATH)

DRIVER = r"""
#include <stdio.h>
#include <stdlib.h>
#include <stdint.h>
%(decl)s

/* integer generator shared with the test: 24-bit values in [-1, 1) times a power of 2 */
static uint64_t state = 0x9E3779B97F4A7C15ull;
static float next_value(float scale) {
  state = state * 6364136223846793005ull + 1442695040888963407ull;
  return ((float)((state >> 40) & 0xFFFFFF) / 8388608.0f - 1.0f) * scale;
}

int main(int argc, char **argv) {
  int c_in = %(c_in)d, c_out = %(c_out)d, td = 4, iters = %(iters)d;
  float *input = (float *)malloc(sizeof(float) * c_in * td * td);
  float *U = (float *)malloc(sizeof(float) * c_out * c_in * td * td);
  float *output = (float *)malloc(sizeof(float) * c_out * 4);
  float *first = (float *)malloc(sizeof(float) * c_out * 4);
  for (int i = 0; i < c_in * td * td; ++i) input[i] = next_value(1.0f);
  for (int i = 0; i < c_out * c_in * td * td; ++i) U[i] = next_value(0.0625f);
  for (int it = 0; it < iters; ++it) {
    fused_winograd_f23(input, U, output, c_in, c_out);
    if (it == 0)
      for (int i = 0; i < c_out * 4; ++i) first[i] = output[i];
  }
  for (int i = 0; i < c_out * 4; ++i)
    if (first[i] != output[i]) return 3;  /* repeated calls must agree */
  FILE *f = fopen(argv[1], "wb");
  if (!f) return 2;
  fwrite(output, sizeof(float), (size_t)c_out * 4, f);
  fclose(f);
  free(input); free(U); free(output); free(first);
  return 0;
}
"""

EXTERN = "extern void fused_winograd_f23(const float*, const float*, float*, int, int);"
HEADER = '#include "cwg.h"'


def _inputs(c_in, c_out):
    """The C program's generator, replayed in numpy (uint64 arithmetic wraps the same way)."""
    state = np.uint64(0x9E3779B97F4A7C15)
    a, b = np.uint64(6364136223846793005), np.uint64(1442695040888963407)

    def values(count, scale):
        nonlocal state
        out = np.empty(count, np.float32)
        with np.errstate(over="ignore"):
            for i in range(count):
                state = state * a + b
                v = np.float32(int(state >> np.uint64(40)) & 0xFFFFFF) / np.float32(8388608.0)
                out[i] = (v - np.float32(1.0)) * np.float32(scale)
        return out

    inp = values(c_in * 16, 1.0).reshape(c_in, 4, 4)
    U = values(c_out * c_in * 16, 0.0625).reshape(c_out, c_in, 4, 4)
    return inp, U


def _build(tmp_path, c_in, c_out, iters, decl, libdir=LIBDIR, lib="cwg"):
    src = tmp_path / "driver.c"
    exe = tmp_path / "driver"
    src.write_text(DRIVER % {"decl": decl, "c_in": c_in, "c_out": c_out, "iters": iters})
    if not os.path.exists(os.path.join(libdir, f"lib{lib}.so")):
        pytest.skip(f"lib{lib}.so not built")
    cmd = ["gcc", "-O2", "-std=c99", str(src), "-I", os.path.join(ROOT, "include"),
           "-L", libdir, f"-l{lib}", f"-Wl,-rpath,{libdir}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


@pytest.mark.parametrize("decl", [EXTERN, HEADER], ids=["extern-decl", "cwg.h"])
def test_c_driver_compiles_and_links(tmp_path, decl):
    exe = _build(tmp_path, 8, 8, 1, decl)
    assert exe.exists()


def test_driver_generator_replay_is_exact():
    inp, U = _inputs(3, 2)
    assert inp.dtype == np.float32 and np.all(np.abs(inp) <= 1.0)
    assert np.all(np.abs(U) <= 0.0625)
    assert len(np.unique(inp)) == inp.size  # a real sequence, not a constant


def test_same_driver_on_the_reference_kernel(tmp_path):
    """The identical program linked against the reference's own fused_winograd.c (compiled
    from source into oracle/_ref) reproduces the test's replay of its inputs: this pins
    the generator and the output comparison below without a GPU."""
    import oracle

    exe = _build(tmp_path, 16, 8, 2, EXTERN, os.path.join(ROOT, "oracle", "_ref"), "ref_layer")
    out_file = tmp_path / "out.bin"
    r = subprocess.run([str(exe), str(out_file)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(out_file, np.float32).reshape(8, 2, 2)
    inp, U = _inputs(16, 8)
    want = oracle.ref_tiles_f23(inp[None], U)[0]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("c_in,c_out,iters", [(32, 32, 50), (128, 128, 5), (7, 19, 3)])
def test_c_driver_output_equals_reference_bitwise(tmp_path, cuda_dev, c_in, c_out, iters):
    import oracle

    exe = _build(tmp_path, c_in, c_out, iters, EXTERN)
    out_file = tmp_path / "out.bin"
    r = subprocess.run([str(exe), str(out_file)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    got = np.fromfile(out_file, np.float32).reshape(c_out, 2, 2)
    inp, U = _inputs(c_in, c_out)
    want = oracle.ref_tiles_f23(inp[None], U)[0]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        float(np.abs(got - want).max())
