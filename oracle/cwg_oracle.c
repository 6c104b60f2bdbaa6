/*
 * cwg_oracle.c -- CPU oracle for the fused Winograd F(m x m, 3 x 3) convolution.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product: only
 * the test suite, the smoke check and the CPU-baseline leg of the benchmark load
 * it.  The product (libcwg.so) neither links nor calls anything in this
 * directory and fails loudly when its CUDA code is unavailable.
 *
 * What it restates (reference paths are relative to the reference project):
 *   - Winograd tables Bt/At for F(2,3), F(4,3), F(6,3):
 *       src/fused_winograd_kernel.py:18-74 (_BT_4, _AT_4, _BT_6, _AT_6, _BT_8, _AT_8)
 *   - per-tile fused algorithm  V = Bt d B ;  M = sum_ic U (.) V ;  Y = At M A
 *       fused_winograd.c:19-101 (F(2,3), sequential fp32 accumulation over ic,
 *       zero-skip on U) and src/fused_winograd_kernel.py:153-181 (run_fused, any td)
 *   - the weight transform U = G g G^T.  The reference has none (it takes U as
 *     an input, fused_winograd.c:21); G is the unique matrix that makes the
 *     reference's Bt/At compute a 3x3 cross-correlation (Lavin & Gray 2015,
 *     the paper cited at src/fused_winograd_kernel.py:14-15).
 *   - layer driver (pad=1, stride=1, tile extraction in the reference's
 *     ic*td*td + r*td + c layout of fused_winograd.c:45, scatter of
 *     oc*m*m + i*m + j of fused_winograd.c:93-96, bias, ReLU).  The reference
 *     has no layer driver; its benchmarks loop a single tile
 *     (benchmarks/jetson_main_microbench.py:47-80).
 *   - an fp64 direct cross-correlation (independent of Winograd).
 *
 * Parity pins: the F(2,3) restatement is bit-identical to the reference C
 * compiled from source (oracle/_ref), and every td is checked against golden
 * vectors produced by the reference's own Python run_fused
 * (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- transform tables (src/fused_winograd_kernel.py:18-67) ---------------- */
static const float BT4[16] = {1, 0, -1, 0, 0, 1, 1, 0, 0, -1, 1, 0, 0, 1, 0, -1};
static const float AT4[8] = {1, 1, 1, 0, 0, 1, -1, -1};
static const float BT6[36] = {4, 0, -5, 0, 1, 0,  0, -4, -4, 1, 1, 0,
                              0, 4, -4, -1, 1, 0, 0, -2, -1, 2, 1, 0,
                              0, 2, -1, -2, 1, 0, 0, 4, 0, -5, 0, 1};
static const float AT6[24] = {1, 1, 1, 1, 1, 0,  0, 1, -1, 2, -2, 0,
                              0, 1, 1, 4, 4, 0,  0, 1, -1, 8, -8, 1};
static const float BT8[64] = {
    1, 0, -21.f / 4, 0, 21.f / 4, 0, -1, 0,
    0, 1, 1, -17.f / 4, -17.f / 4, 1, 1, 0,
    0, -1, 1, 17.f / 4, -17.f / 4, -1, 1, 0,
    0, 0.5f, 0.25f, -2.5f, -1.25f, 2, 1, 0,
    0, -0.5f, 0.25f, 2.5f, -1.25f, -2, 1, 0,
    0, 2, 4, -2.5f, -5, 0.5f, 1, 0,
    0, -2, 4, 2.5f, -5, -0.5f, 1, 0,
    0, -1, 0, 21.f / 4, 0, -21.f / 4, 0, 1};
static const float AT8[48] = {1, 1, 1, 1, 1, 32, 32, 0,   0, 1, -1, 2, -2, 16, -16, 0,
                              0, 1, 1, 4, 4, 8, 8, 0,     0, 1, -1, 8, -8, 4, -4, 0,
                              0, 1, 1, 16, 16, 2, 2, 0,   0, 1, -1, 32, -32, 1, -1, 1};

/* G (td x 3) such that At[(G g G^T) . (Bt d B)]A == corr(d, g); exact rationals. */
static const double G4[12] = {1, 0, 0, .5, .5, .5, .5, -.5, .5, 0, 0, 1};
static const double G6[18] = {1. / 4, 0, 0,
                              -1. / 6, -1. / 6, -1. / 6,
                              -1. / 6, 1. / 6, -1. / 6,
                              1. / 24, 1. / 12, 1. / 6,
                              1. / 24, -1. / 12, 1. / 6,
                              0, 0, 1};
static const double G8[24] = {1, 0, 0,
                              -2. / 9, -2. / 9, -2. / 9,
                              -2. / 9, 2. / 9, -2. / 9,
                              1. / 90, 1. / 45, 2. / 45,
                              1. / 90, -1. / 45, 2. / 45,
                              1. / 45, 1. / 90, 1. / 180,
                              1. / 45, -1. / 90, 1. / 180,
                              0, 0, 1};

static int tables(int td, const float **bt, const float **at, const double **g) {
  switch (td) {
    case 4: *bt = BT4; *at = AT4; *g = G4; return 0;
    case 6: *bt = BT6; *at = AT6; *g = G6; return 0;
    case 8: *bt = BT8; *at = AT8; *g = G8; return 0;
    default: return -1;
  }
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Weight transform: g [K][C][3][3] -> U [K][C][td][td] (the reference's U layout,
 * fused_winograd.c:74), computed in fp64 and rounded once to fp32. */
int orc_weight_transform(const float *g, float *U, int K, int C, int td) {
  const float *bt, *at;
  const double *G;
  if (tables(td, &bt, &at, &G)) return -1;
  for (long kc = 0; kc < (long)K * C; ++kc) {
    const float *gk = g + kc * 9;
    double t[8 * 3];
    for (int a = 0; a < td; ++a)
      for (int j = 0; j < 3; ++j) {
        double s = 0;
        for (int i = 0; i < 3; ++i) s += G[a * 3 + i] * (double)gk[i * 3 + j];
        t[a * 3 + j] = s;
      }
    float *u = U + kc * td * td;
    for (int a = 0; a < td; ++a)
      for (int b = 0; b < td; ++b) {
        double s = 0;
        for (int j = 0; j < 3; ++j) s += t[a * 3 + j] * G[b * 3 + j];
        u[a * td + b] = (float)s;
      }
  }
  return 0;
}

/* F(2,3) tile, operation order of fused_winograd.c:44-97 (bit-identical). */
static void tile_f23(const float *input, const float *U, float *output, int c_in, int c_out,
                     float *V) {
  for (int ic = 0; ic < c_in; ic++) {
    const float *d = input + ic * 16;
    float *v = V + ic * 16;
    float t[16];
    for (int i = 0; i < 4; i++) {
      t[0 * 4 + i] = d[0 * 4 + i] - d[2 * 4 + i];
      t[1 * 4 + i] = d[1 * 4 + i] + d[2 * 4 + i];
      t[2 * 4 + i] = -d[1 * 4 + i] + d[2 * 4 + i];
      t[3 * 4 + i] = d[1 * 4 + i] - d[3 * 4 + i];
    }
    for (int i = 0; i < 4; i++) {
      v[i * 4 + 0] = t[i * 4 + 0] - t[i * 4 + 2];
      v[i * 4 + 1] = t[i * 4 + 1] + t[i * 4 + 2];
      v[i * 4 + 2] = -t[i * 4 + 1] + t[i * 4 + 2];
      v[i * 4 + 3] = t[i * 4 + 1] - t[i * 4 + 3];
    }
  }
  for (int oc = 0; oc < c_out; oc++) {
    float M[16] = {0};
    for (int ic = 0; ic < c_in; ic++) {
      const float *u = U + ((long)oc * c_in + ic) * 16;
      const float *v = V + ic * 16;
      for (int i = 0; i < 16; i++)
        if (u[i] != 0.0f) M[i] += u[i] * v[i];
    }
    float t[8];
    for (int i = 0; i < 4; i++) {
      t[0 * 4 + i] = M[0 * 4 + i] + M[1 * 4 + i] + M[2 * 4 + i];
      t[1 * 4 + i] = M[1 * 4 + i] - M[2 * 4 + i] - M[3 * 4 + i];
    }
    float *y = output + oc * 4;
    for (int i = 0; i < 2; i++) {
      y[i * 2 + 0] = t[i * 4 + 0] + t[i * 4 + 1] + t[i * 4 + 2];
      y[i * 2 + 1] = t[i * 4 + 1] - t[i * 4 + 2] - t[i * 4 + 3];
    }
  }
}

/* Generic td tile (run_fused, src/fused_winograd_kernel.py:153-181):
 * V = (Bt d) Bt^T, M = sum_ic U (.) V (sequential fp32), Y = (At M) At^T. */
static void tile_generic(const float *input, const float *U, float *output, int c_in,
                         int c_out, int td, const float *bt, const float *at, float *V) {
  const int m = td - 2, n2 = td * td;
  for (int ic = 0; ic < c_in; ic++) {
    const float *d = input + (long)ic * n2;
    float *v = V + (long)ic * n2;
    float t[64];
    for (int a = 0; a < td; ++a)
      for (int j = 0; j < td; ++j) {
        float s = 0.f;
        for (int i = 0; i < td; ++i) s += bt[a * td + i] * d[i * td + j];
        t[a * td + j] = s;
      }
    for (int a = 0; a < td; ++a)
      for (int b = 0; b < td; ++b) {
        float s = 0.f;
        for (int j = 0; j < td; ++j) s += t[a * td + j] * bt[b * td + j];
        v[a * td + b] = s;
      }
  }
  for (int oc = 0; oc < c_out; oc++) {
    float M[64];
    for (int i = 0; i < n2; ++i) M[i] = 0.f;
    for (int ic = 0; ic < c_in; ic++) {
      const float *u = U + ((long)oc * c_in + ic) * n2;
      const float *v = V + (long)ic * n2;
      for (int i = 0; i < n2; i++)
        if (u[i] != 0.0f) M[i] += u[i] * v[i];
    }
    float t[6 * 8];
    for (int i = 0; i < m; ++i)
      for (int b = 0; b < td; ++b) {
        float s = 0.f;
        for (int a = 0; a < td; ++a) s += at[i * td + a] * M[a * td + b];
        t[i * td + b] = s;
      }
    float *y = output + (long)oc * m * m;
    for (int i = 0; i < m; ++i)
      for (int j = 0; j < m; ++j) {
        float s = 0.f;
        for (int b = 0; b < td; ++b) s += t[i * td + b] * at[j * td + b];
        y[i * m + j] = s;
      }
  }
}

/* Per-tile entry with the reference's argument order (fused_winograd.c:103-108),
 * generalised to td in {4,6,8}; n_tiles tiles laid out back to back. */
int orc_tiles_fused(const float *tiles, const float *U, float *out, int n_tiles, int c_in,
                    int c_out, int td, int nthreads) {
  const float *bt, *at;
  const double *G;
  if (tables(td, &bt, &at, &G) || c_in <= 0 || c_out <= 0 || n_tiles < 0) return -1;
  const int m = td - 2;
  set_threads(nthreads);
  int err = 0;
#pragma omp parallel
  {
    float *V = (float *)malloc(sizeof(float) * (size_t)c_in * td * td);
    if (!V) {
#pragma omp atomic write
      err = -2;
    } else {
#pragma omp for schedule(static)
      for (long t = 0; t < n_tiles; ++t) {
        const float *in = tiles + t * (long)c_in * td * td;
        float *o = out + t * (long)c_out * m * m;
        if (td == 4)
          tile_f23(in, U, o, c_in, c_out, V);
        else
          tile_generic(in, U, o, c_in, c_out, td, bt, at, V);
      }
      free(V);
    }
  }
  return err;
}

/* Layer driver: x [N][C][H][W], U [K][C][td][td], bias [K] (may be NULL),
 * y [N][K][H][W]; pad=1, stride=1.  Tiles cover ceil(H/m) x ceil(W/m); inputs
 * outside the image read as zero and outputs outside it are dropped. */
int orc_conv_layer(const float *x, const float *U, const float *bias, float *y, int N, int C,
                   int K, int H, int W, int td, int relu, int nthreads) {
  const float *bt, *at;
  const double *G;
  if (tables(td, &bt, &at, &G) || N < 0 || C <= 0 || K <= 0 || H <= 0 || W <= 0) return -1;
  const int m = td - 2, th = (H + m - 1) / m, tw = (W + m - 1) / m;
  set_threads(nthreads);
  int err = 0;
#pragma omp parallel
  {
    float *d = (float *)malloc(sizeof(float) * (size_t)C * td * td);
    float *V = (float *)malloc(sizeof(float) * (size_t)C * td * td);
    float *o = (float *)malloc(sizeof(float) * (size_t)K * m * m);
    if (!d || !V || !o) {
#pragma omp atomic write
      err = -2;
    } else {
#pragma omp for schedule(dynamic, 4)
      for (long job = 0; job < (long)N * th * tw; ++job) {
        const int n = (int)(job / ((long)th * tw));
        const int ty = (int)((job / tw) % th), tx = (int)(job % tw);
        const int y0 = ty * m - 1, x0 = tx * m - 1;
        for (int c = 0; c < C; ++c) {
          const float *xc = x + ((long)n * C + c) * H * W;
          for (int r = 0; r < td; ++r)
            for (int s = 0; s < td; ++s) {
              const int yy = y0 + r, xx = x0 + s;
              d[(c * td + r) * td + s] =
                  (yy >= 0 && yy < H && xx >= 0 && xx < W) ? xc[(long)yy * W + xx] : 0.f;
            }
        }
        if (td == 4)
          tile_f23(d, U, o, C, K, V);
        else
          tile_generic(d, U, o, C, K, td, bt, at, V);
        for (int k = 0; k < K; ++k) {
          float *yk = y + ((long)n * K + k) * H * W;
          const float b = bias ? bias[k] : 0.f;
          for (int i = 0; i < m; ++i)
            for (int j = 0; j < m; ++j) {
              const int yy = ty * m + i, xx = tx * m + j;
              if (yy < H && xx < W) {
                float v = o[(k * m + i) * m + j] + b;
                if (relu && v < 0.f) v = 0.f;
                yk[(long)yy * W + xx] = v;
              }
            }
        }
      }
    }
    free(d);
    free(V);
    free(o);
  }
  return err;
}

/* fp64 direct 3x3 cross-correlation, pad=1, stride=1: y [N][K][H][W] (double). */
int orc_direct_conv_f64(const float *x, const float *g, const float *bias, double *y, int N,
                        int C, int K, int H, int W, int relu, int nthreads) {
  if (N < 0 || C <= 0 || K <= 0 || H <= 0 || W <= 0) return -1;
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) {
      double *yk = y + ((long)n * K + k) * H * W;
      const double b = bias ? (double)bias[k] : 0.0;
      for (long p = 0; p < (long)H * W; ++p) yk[p] = 0.0;
      for (int c = 0; c < C; ++c) {
        const float *xc = x + ((long)n * C + c) * H * W;
        const float *gk = g + ((long)k * C + c) * 9;
        for (int ky = 0; ky < 3; ++ky)
          for (int kx = 0; kx < 3; ++kx) {
            const double w = gk[ky * 3 + kx];
            for (int oy = 0; oy < H; ++oy) {
              const int iy = oy + ky - 1;
              if (iy < 0 || iy >= H) continue;
              for (int ox = 0; ox < W; ++ox) {
                const int ix = ox + kx - 1;
                if (ix < 0 || ix >= W) continue;
                yk[(long)oy * W + ox] += w * (double)xc[(long)iy * W + ix];
              }
            }
          }
      }
      for (long p = 0; p < (long)H * W; ++p) {
        double v = yk[p] + b;
        if (relu && v < 0.0) v = 0.0;
        yk[p] = v;
      }
    }
  return 0;
}

/* Round fp32 values to the nearest bfloat16 (ties to even), in place, keeping
 * them as fp32 bit patterns; NaN stays NaN. */
void orc_round_bf16(float *x, long n) {
  for (long i = 0; i < n; ++i) {
    uint32_t u;
    memcpy(&u, &x[i], 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
      u |= 0x00400000u;
    } else {
      u += 0x7fffu + ((u >> 16) & 1u);
    }
    u &= 0xffff0000u;
    memcpy(&x[i], &u, 4);
  }
}
