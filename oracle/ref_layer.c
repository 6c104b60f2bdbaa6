/*
 * ref_layer.c -- layer driver around the reference's own per-tile kernel.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the CPU baseline, never the
 * product).  This file is linked with the reference's unmodified
 * fused_winograd.c, compiled from the reference source tree by
 * oracle/Makefile into oracle/_ref/libref_layer.so.  It adds only what the
 * reference lacks for a whole layer: zero padding (pad=1), extraction of each
 * 4x4 input tile in the ic*16 + r*4 + c layout the kernel reads
 * (fused_winograd.c:45), the scatter of its oc*4 + i*2 + j output
 * (fused_winograd.c:93-96), bias and ReLU, and an OpenMP loop over
 * (image, tile row, tile column).
 */
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* fused_winograd.c:103-108 */
void fused_winograd_f23(const float *input, const float *U, float *output, int c_in, int c_out);

int refl_tiles_f23(const float *tiles, const float *U, float *out, int n_tiles, int c_in,
                   int c_out, int nthreads) {
  if (c_in <= 0 || c_out <= 0 || n_tiles < 0) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
#pragma omp parallel for schedule(static)
  for (long t = 0; t < n_tiles; ++t)
    fused_winograd_f23(tiles + t * (long)c_in * 16, U, out + t * (long)c_out * 4, c_in, c_out);
  return 0;
}

int refl_conv_layer_f23(const float *x, const float *U, const float *bias, float *y, int N,
                        int C, int K, int H, int W, int relu, int nthreads) {
  if (N < 0 || C <= 0 || K <= 0 || H <= 0 || W <= 0) return -1;
  const int th = (H + 1) / 2, tw = (W + 1) / 2;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  int err = 0;
#pragma omp parallel
  {
    float *d = (float *)malloc(sizeof(float) * (size_t)C * 16);
    float *o = (float *)malloc(sizeof(float) * (size_t)K * 4);
    if (!d || !o) {
#pragma omp atomic write
      err = -2;
    } else {
#pragma omp for schedule(dynamic, 4)
      for (long job = 0; job < (long)N * th * tw; ++job) {
        const int n = (int)(job / ((long)th * tw));
        const int ty = (int)((job / tw) % th), tx = (int)(job % tw);
        const int y0 = 2 * ty - 1, x0 = 2 * tx - 1;
        for (int c = 0; c < C; ++c) {
          const float *xc = x + ((long)n * C + c) * H * W;
          for (int r = 0; r < 4; ++r)
            for (int s = 0; s < 4; ++s) {
              const int yy = y0 + r, xx = x0 + s;
              d[c * 16 + r * 4 + s] =
                  (yy >= 0 && yy < H && xx >= 0 && xx < W) ? xc[(long)yy * W + xx] : 0.f;
            }
        }
        fused_winograd_f23(d, U, o, C, K);
        for (int k = 0; k < K; ++k) {
          float *yk = y + ((long)n * K + k) * H * W;
          const float b = bias ? bias[k] : 0.f;
          for (int i = 0; i < 2; ++i)
            for (int j = 0; j < 2; ++j) {
              const int yy = 2 * ty + i, xx = 2 * tx + j;
              if (yy < H && xx < W) {
                float v = o[k * 4 + i * 2 + j] + b;
                if (relu && v < 0.f) v = 0.f;
                yk[(long)yy * W + xx] = v;
              }
            }
        }
      }
    }
    free(d);
    free(o);
  }
  return err;
}

int refl_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
