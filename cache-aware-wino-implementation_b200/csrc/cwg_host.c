/*
 * cwg_host.c -- host side of libcwg, in C: argument checking, the tile /
 * kernel selector, weight-layout bookkeeping, the reference-compatible per-tile
 * entry points, and the host-buffer (end-to-end) layer call.  Kernels are
 * reached only through the launch shims of cwg_internal.h.
 *
 * Reference counterparts (paths relative to the reference project):
 *   cwg_select ........... CacheAdaptiveAutotiler.select_best_tile and
 *                          compute_working_set (src/cache_adaptive_autotiler.py:25-82):
 *                          the reference fits a per-tile working set into
 *                          alpha * L1; here every candidate kernel's per-CTA
 *                          footprint is checked against shared memory (227 KiB)
 *                          and tensor memory (512 columns), and the grid
 *                          replaces LocalityScheduler's task list
 *                          (src/locality_scheduler.py:10-43): one CTA per
 *                          (tile block, output-channel block, image), output-
 *                          channel blocks outermost so CTAs sharing a slice of U
 *                          run together.
 *   fused_winograd_f23 ... fused_winograd.c:103-108 (void, no error return).
 *   cwg_tiles_fused ...... src/fused_winograd_kernel.py:153-181 (run_fused) for
 *                          td in {4,6,8}; ValueError for other td there
 *                          (:92-97) is CWG_EINVAL here.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "../../include/cwg.h"
#include "cwg_internal.h"

#define CWG_VERSION "cwg 0.1 (sm_100a)"
#define B200_SMS 148
#define SMEM_LIMIT (227 * 1024)

const char *cwg_version(void) { return CWG_VERSION; }

const char *cwg_strerror(int status) {
  switch (status) {
    case CWG_OK: return "ok";
    case CWG_EINVAL: return "invalid argument";
    case CWG_EUNSUPPORTED: return "unsupported configuration";
    case CWG_ECUDA: return "CUDA runtime error";
    case CWG_ETIMEOUT: return "device-side wait timed out";
    case CWG_ENOMEM: return "out of memory";
    case CWG_ENODEV: return "no usable sm_100 device";
    case CWG_ERANGE: return "an operand left the range of the kernel's fp16 arithmetic";
    default: return "unknown status";
  }
}

int cwg_last_cuda_error(void) { return cwgk_get_cuda_error(); }
long long cwg_launch_count(void) { return cwgk_launches(); }

static int cuda_fail(cudaError_t e) {
  cwgk_set_cuda_error((int)e);
  return CWG_ECUDA;
}

/* SM count of the current device; B200's 148 when no device is visible (the
 * selector is pure host arithmetic and must work without a GPU). */
static int num_sms(void) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return B200_SMS;
  }
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0) {
    cudaGetLastError();
    return B200_SMS;
  }
  return sms;
}

/* ---- path decision (depends only on c_in, c_out, m, flags, so that the
 * weight layout chosen at transform time matches the conv call) ----------- */
/* Tensor-core kernel variant: the 2-SM pair kernel unless a flag asks for one
 * of the single-CTA kernels.  Layers of at most 64 output channels run it with
 * 64 channels per CTA: F(2,3) as M = 128 (half the weight rows of the M = 256
 * kernel, whose other half would be zero), F(4,3) with two output rows x 64
 * channels per CTA in one pass over all 36 frequencies (the 128-channel form's
 * two passes would each leave half their rows zero). */
static int tc_variant(unsigned flags, int m, int c_out) {
  if (flags & CWG_TC_FULL16) return CWGK_TC_FULL16;
  if (flags & CWG_TC_NOPAIR) return CWGK_TC_HALF;
  return c_out <= 64 ? CWGK_TC_PAIR64 : CWGK_TC_PAIR;
}

/* Products per multiply-accumulate on the tensor cores:
 *   3  bf16 hi/lo split, fp32-accurate: fp32 layers (and bf16 F(4,3) layers
 *      with CWG_TC_X3);
 *   2  fp16 operands with V split into hi + lo: bf16 F(4,3) layers.  F(4,3)'s
 *      output transform (coefficients up to 8) turns single bf16 products into
 *      ~6% errors; fp16's 11 significant bits bring two products to ~5e-3
 *      normwise against a direct convolution, at two thirds of the MMAs and half
 *      the weight stream of the split;
 *   1  bf16 F(2,3) layers, or when CWG_TC_SINGLE asks for it. */
static int tc_products(int m, unsigned flags) {
  if (flags & CWG_TC_SINGLE) return 1;
  if (flags & CWG_BF16) return m == 4 ? ((flags & CWG_TC_X3) ? 3 : 2) : 1;
  return 3;
}

/* F(4,3) runs on the tensor cores for bf16 layers only: with fp32 data the
 * hi/lo split's dropped lo*lo terms, amplified by the output transform, leave
 * ~4e-4 absolute error against fp32 F(4,3) -- outside the fp32 parity bar. */
static int tc_available(int m, unsigned flags, int c_out) {
  cwgk_tc_cfg cfg;
  if (m == 4 && !(flags & CWG_BF16)) return 0;
  return cwgk_tc_get_cfg(tc_products(m, flags), tc_variant(flags, m, c_out), m, &cfg) == 0;
}

/* Tensor cores only where the per-frequency GEMM is a real contraction: both
 * channel counts >= 64 (the kernels zero-pad C_in to 16 and C_out to the
 * channel block). */
static int tc_shape_ok(int c_in, int c_out) { return c_in >= 64 && c_out >= 64; }

/* Resolves m and the path; returns CWG_OK or an error. */
static int decide(int c_in, int c_out, int m, unsigned flags, int *m_out, int *path_out) {
  if (c_in <= 0 || c_out <= 0) return CWG_EINVAL;
  if (m != 0 && m != 2 && m != 4 && m != 6) return CWG_EINVAL;
  if ((flags & CWG_FORCE_FFMA) && (flags & CWG_FORCE_TC)) return CWG_EINVAL;
  if ((flags & CWG_TC_FULL16) && (flags & CWG_TC_NOPAIR)) return CWG_EINVAL;
  /* the tensor-core path runs F(2,3) unless F(4,3) is asked for */
  const int m_tc = m ? m : 2;
  const int tc_ok = tc_shape_ok(c_in, c_out) && tc_available(m_tc, flags, c_out);
  if (flags & CWG_FORCE_TC) {
    if (!tc_ok) return CWG_EUNSUPPORTED;
    *m_out = m_tc;
    *path_out = CWG_PATH_TC;
    return CWG_OK;
  }
  if (!(flags & CWG_FORCE_FFMA) && tc_ok) {
    *m_out = m_tc;
    *path_out = CWG_PATH_TC;
    return CWG_OK;
  }
  /* CUDA-core path: F(4,3) needs 2.25 multiplies per output against 4 for
   * F(2,3); take it for bf16 data, whose rounding already dominates the error,
   * and keep F(2,3) (the reference's default, src/cache_adaptive_autotiler.py:70-73)
   * for fp32. */
  *m_out = m ? m : ((flags & CWG_BF16) && c_in > 4 ? 4 : 2);  /* 1-4 channels: own F(2,3) kernel */
  *path_out = CWG_PATH_FFMA;
  return CWG_OK;
}

static int layout_of(int path, int m, unsigned flags, int c_out) {
  if (path == CWG_PATH_TC) {
    const int pm = tc_products(m, flags), x3 = pm == 3;
    const int v = tc_variant(flags, m, c_out);
    if (v == CWGK_TC_PAIR && pm == 2) return CWGK_LAYOUT_TC2_H2;
    if (v == CWGK_TC_PAIR64 && pm == 2) return CWGK_LAYOUT_TC2H_H2;
    if (v == CWGK_TC_PAIR) return x3 ? CWGK_LAYOUT_TC2_X3 : CWGK_LAYOUT_TC2_X1;
    if (v == CWGK_TC_PAIR64) return x3 ? CWGK_LAYOUT_TC2H_X3 : CWGK_LAYOUT_TC2H_X1;
    return x3 ? CWGK_LAYOUT_TC_X3 : CWGK_LAYOUT_TC_X1;
  }
  /* The CUDA-core kernel keeps U in fp32 for bf16 layers too: rounding U to
   * bf16 loses ~4% through F(4,3)'s output transform (coefficients up to 8). */
  return CWGK_LAYOUT_FFMA_F32;
}

static size_t weight_bytes_for(int c_in, int c_out, int m, int layout) {
  size_t nf = (size_t)(m + 2) * (m + 2);
  switch (layout) {
    case CWGK_LAYOUT_FFMA_F32: return nf * c_in * c_out * 4;
    case CWGK_LAYOUT_TC_X3:
    case CWGK_LAYOUT_TC_X1:
    case CWGK_LAYOUT_TC2_X3:
    case CWGK_LAYOUT_TC2_X1:
    case CWGK_LAYOUT_TC2H_X3:
    case CWGK_LAYOUT_TC2H_X1:
    case CWGK_LAYOUT_TC2_H2:
    case CWGK_LAYOUT_TC2H_H2: {
      /* [ceil(C_out / kb)][passes][sets][C_pad / 16][nf][parts] blocks of `rows`
       * rows x 16 channels (rows x 32 bytes).  Pair layouts: one set per rank;
       * 128 channels of one output row per block and m/2 passes (pairs of
       * output rows; an F(4,3) pass stores the 30 frequencies whose At row pair
       * is not all zero), or, for layers of at most 64 channels (TC2H), one
       * pass: 64 channels of one output row (F(2,3)) or of two (F(4,3)). */
      const int half = layout == CWGK_LAYOUT_TC2H_X3 || layout == CWGK_LAYOUT_TC2H_X1 ||
                       layout == CWGK_LAYOUT_TC2H_H2;
      const int pair = half || layout == CWGK_LAYOUT_TC2_X3 || layout == CWGK_LAYOUT_TC2_X1 ||
                       layout == CWGK_LAYOUT_TC2_H2;
      const size_t kb = half ? 64 : 128;
      const size_t rows = (half && m == 4) ? 128 : kb;
      const size_t passes = (pair && !half) ? (size_t)(m / 2) : 1;
      if (pair && !half && m == 4) nf -= (size_t)(m + 2);
      const size_t nkb = ((size_t)c_out + kb - 1) / kb * passes;
      const size_t c16 = ((size_t)c_in + 15) / 16;
      const size_t parts = (layout == CWGK_LAYOUT_TC_X3 || layout == CWGK_LAYOUT_TC2_X3 ||
                            layout == CWGK_LAYOUT_TC2H_X3)
                               ? 2
                               : 1;
      const size_t sets = pair ? 2 : 1;
      return nkb * sets * c16 * nf * parts * rows * 32;
    }
    default: return 0;
  }
}

static int find_ffma_ty(int m, int kb, int ty, cwgk_ffma_cfg *c) {
  const int ncfg = cwgk_ffma_num_cfgs();
  for (int i = 0; i < ncfg; ++i)
    if (cwgk_ffma_get_cfg(i, c) == 0 && c->m == m && c->kb == kb && c->ty == ty) return i;
  return -1;
}

/* F(2,3) layers of 1-4 input channels (an RGB input layer) run the one-tile-per-
 * thread kernel: they are bound by writing the output planes, and the general
 * kernel's per-CTA staging of 8-channel weight chunks costs more than the math. */
static int small_cin(int c_in, int m) { return m == 2 && c_in <= 4; }

/* Cost of one CTA of the 4x4-tile CUDA-core kernel, c0 + steps * b microseconds
 * for `steps` 8-channel input steps, fitted to B200 sweeps of single-image 56x56
 * layers over channel block x C_in slices (6 % rms).  The kernels run one CTA per
 * SM (72-168 registers a thread), so a grid of G CTAs takes ceil(G / SMs) such
 * rounds.  A C_in split adds the zeroing of y and its atomics, and with ReLU the
 * bias/ReLU pass. */
typedef struct {
  int m, kb;
  double c0, b;
} ffma_cost;
static const ffma_cost kFfmaCost[] = {
    {2, 16, 1.8, 0.92}, {2, 32, 2.1, 1.10}, {2, 64, 2.5, 1.66}, {4, 16, 4.3, 1.95},
    {4, 32, 4.5, 2.56}, {4, 64, 6.3, 4.27}, {6, 16, 6.0, 4.6},
};
#define FFMA_SPLIT_US 4.5
#define FFMA_RELU_PASS_US 3.5

/* Picks the FFMA configuration for a layer (index into the shim's table) and its
 * C_in slices (1 unless fp32 and allowed):
 *   - large layers whose grid of 8x8-tile blocks of 32 channels still fills every
 *     SM take that kernel: a CTA's weight chunk then serves 64 tiles instead of
 *     16, and each CTA pays its load / transform / store latency once (a 3->64
 *     layer at 224x224, 32 images: 521 vs 791 us);
 *   - otherwise the (channel block, slices) of least modelled time (kFfmaCost):
 *     wide blocks use fewer instructions per output channel, narrow blocks and
 *     slices fill more SMs.  Single-image F(4,3) at 56x56 (us, model pick vs the
 *     previous widest-block-filling-the-SMs rule): 64->64 14.7 vs 23.7, 128->128
 *     31.3 vs 39.6. */
static int pick_ffma(int n, int c_in, int c_out, int h, int w, int m, unsigned flags,
                     cwgk_ffma_cfg *cfg_out, int *slices_out) {
  const int sms = num_sms();
  const long long th = (h + m - 1) / m, tw = (w + m - 1) / m;
  if (slices_out) *slices_out = 1;
  if (c_out >= 32 && n <= 65535) { /* the kernel's grid.z holds the images */
    cwgk_ffma_cfg c;
    const int idx = find_ffma_ty(m, 32, 8, &c);
    if (idx >= 0) {
      const long long ctas = (long long)n * ((th + c.ty - 1) / c.ty) * ((tw + c.tx - 1) / c.tx) *
                             ((c_out + c.kb - 1) / c.kb);
      if (ctas >= sms) {
        if (cfg_out) *cfg_out = c;
        return idx;
      }
    }
  }
  const int can_split = !(flags & (CWG_BF16 | CWG_NO_SPLIT));
  const int relu = (flags & CWG_RELU) != 0;
  int best = -1, best_s = 1;
  double best_t = 0.0;
  cwgk_ffma_cfg best_c;
  memset(&best_c, 0, sizeof(best_c));
  static const int kbs[3] = {64, 32, 16}; /* ties keep the wider block */
  for (int i = 0; i < 3; ++i) {
    cwgk_ffma_cfg c;
    const int idx = find_ffma_ty(m, kbs[i], 4, &c);
    if (idx < 0) continue;
    const ffma_cost *cost = NULL;
    for (size_t j = 0; j < sizeof(kFfmaCost) / sizeof(kFfmaCost[0]); ++j)
      if (kFfmaCost[j].m == m && kFfmaCost[j].kb == c.kb) cost = &kFfmaCost[j];
    if (!cost) continue;
    const long long grid = (long long)n * ((th + c.ty - 1) / c.ty) * ((tw + c.tx - 1) / c.tx) *
                           ((c_out + c.kb - 1) / c.kb);
    const int steps = (c_in + c.cc - 1) / c.cc;
    /* splitting a grid that already fills the SMs only adds rounds */
    const int max_s = (can_split && grid < sms) ? steps : 1;
    for (int s = 1; s <= max_s; ++s) {
      const int per = (steps + s - 1) / s;
      if ((steps + per - 1) / per != s) continue; /* same steps per slice as a smaller s */
      if ((long long)n * s > 65535) break;
      const double rounds = (double)((grid * s + sms - 1) / sms);
      const double t = rounds * (cost->c0 + per * cost->b) +
                       (s > 1 ? FFMA_SPLIT_US + (relu ? FFMA_RELU_PASS_US : 0.0) : 0.0);
      if (best < 0 || t < best_t) {
        best = idx;
        best_s = s;
        best_t = t;
        best_c = c;
      }
    }
  }
  if (best < 0) return -1;
  if (cfg_out) *cfg_out = best_c;
  if (slices_out) *slices_out = best_s;
  return best;
}

int cwg_select(int n, int c_in, int c_out, int h, int w, int m, unsigned flags,
               cwg_choice *out) {
  if (!out || n < 0 || h <= 0 || w <= 0) return CWG_EINVAL;
  int mm = 0, path = 0;
  const int rc = decide(c_in, c_out, m, flags, &mm, &path);
  if (rc) return rc;
  memset(out, 0, sizeof(*out));
  out->m = mm;
  out->path = path;
  const long long th = (h + mm - 1) / mm, tw = (w + mm - 1) / mm;
  const double td2 = (double)(mm + 2) * (mm + 2);
  const int esz = (flags & CWG_BF16) ? 2 : 4;
  out->gemm_flops = 2.0 * (double)n * th * tw * c_out * c_in * td2;
  out->alg_bytes = (double)n * c_in * h * w * esz + (double)n * c_out * h * w * esz +
                   (double)weight_bytes_for(c_in, c_out, mm, layout_of(path, mm, flags, c_out)) +
                   4.0 * c_out;
  if (path == CWG_PATH_TC) {
    cwgk_tc_cfg t;
    cwgk_tc_get_cfg(tc_products(mm, flags), tc_variant(flags, mm, c_out), mm, &t);
    out->mma_products = tc_products(mm, flags);
    out->tiles_per_cta = t.tiles;
    out->cout_per_cta = t.kb;
    out->cin_chunk = t.cc;
    out->threads = t.threads;
    out->smem_bytes = t.smem;
    out->tmem_cols = t.tmem_cols;
    const int v = tc_variant(flags, mm, c_out);
    const int bf = (flags & CWG_BF16) != 0, split = !(flags & CWG_NO_SPLIT);
    out->ctas = ((long long)n * th * tw + t.tiles - 1) / t.tiles * ((c_out + t.kb - 1) / t.kb) *
                t.ctas_per_tile_block *
                cwgk_tc_splits(n, c_in, c_out, h, w, mm, v, bf, split, num_sms());
    out->ctas_launched = out->ctas;
    out->order = CWG_ORDER_GRID;
    if (n > 0 && cwgk_tc_plan(n, c_in, c_out, h, w, mm, tc_products(mm, flags), v, bf, split,
                              num_sms(), &out->ctas_launched, &out->order) != 0) {
      out->ctas_launched = out->ctas;
      out->order = CWG_ORDER_GRID;
    }
  } else if (small_cin(c_in, mm)) {
    const long long gx = ((long long)n * th * tw + 255) / 256;
    int kc = 64; /* the launch's rule: halve while the grid leaves SMs idle */
    while (kc > 8 && gx * ((c_out + kc - 1) / kc) < 2LL * num_sms()) kc /= 2;
    out->tiles_per_cta = 256; /* one thread per tile */
    out->cout_per_cta = kc;
    out->cin_chunk = c_in;
    out->threads = 256;
    out->smem_bytes = 64 * 16 * c_in * 4;
    out->tmem_cols = 0;
    out->ctas = gx * ((c_out + kc - 1) / kc);
    out->ctas_launched = out->ctas;
    out->order = CWG_ORDER_GRID;
  } else {
    cwgk_ffma_cfg c;
    int slices = 1;
    if (pick_ffma(n, c_in, c_out, h, w, mm, flags, &c, &slices) < 0) return CWG_EUNSUPPORTED;
    out->tiles_per_cta = c.ty * c.tx;
    out->cout_per_cta = c.kb;
    out->cin_chunk = c.cc;
    out->threads = c.threads;
    out->smem_bytes = c.smem;
    out->tmem_cols = 0;
    out->ctas = (long long)n * ((th + c.ty - 1) / c.ty) * ((tw + c.tx - 1) / c.tx) *
                ((c_out + c.kb - 1) / c.kb) * slices;
    out->ctas_launched = out->ctas;
    out->order = CWG_ORDER_GRID;
  }
  if (out->smem_bytes > SMEM_LIMIT || out->tmem_cols > 512) return CWG_EUNSUPPORTED;
  return CWG_OK;
}

size_t cwg_weight_bytes(int c_in, int c_out, int m, unsigned flags) {
  int mm = 0, path = 0;
  if (decide(c_in, c_out, m, flags, &mm, &path)) return 0;
  return weight_bytes_for(c_in, c_out, mm, layout_of(path, mm, flags, c_out));
}

static int weight_common(const float *src, void *U, int c_in, int c_out, int m, unsigned flags,
                         int from_ref, void *stream) {
  if (!src || !U) return CWG_EINVAL;
  if (((uintptr_t)src & 3) || ((uintptr_t)U & 15)) return CWG_EINVAL;
  int mm = 0, path = 0;
  const int rc = decide(c_in, c_out, m, flags, &mm, &path);
  if (rc) return rc;
  if (from_ref && m == 0) return CWG_EINVAL; /* a reference-layout U fixes td */
  return cwgk_weight_transform(src, U, c_in, c_out, mm, layout_of(path, mm, flags, c_out), from_ref,
                               stream);
}

int cwg_weight_transform(const float *g, void *U, int c_in, int c_out, int m, unsigned flags,
                         void *stream) {
  return weight_common(g, U, c_in, c_out, m, flags, 0, stream);
}

int cwg_weight_import(const float *U_ref, void *U, int c_in, int c_out, int m, unsigned flags,
                      void *stream) {
  return weight_common(U_ref, U, c_in, c_out, m, flags, 1, stream);
}

int cwg_conv3x3_fused(const void *x, const void *U, const float *bias, void *y, int n, int c_in,
                      int c_out, int h, int w, int m, unsigned flags, void *stream) {
  if (n < 0 || h <= 0 || w <= 0 || c_in <= 0 || c_out <= 0) return CWG_EINVAL;
  if (n == 0) return CWG_OK;
  if (!x || !U || !y) return CWG_EINVAL;
  const size_t esz = (flags & CWG_BF16) ? 2 : 4;
  if (((uintptr_t)x % esz) || ((uintptr_t)y % esz) || ((uintptr_t)U & 15) ||
      ((uintptr_t)bias & 3))
    return CWG_EINVAL;
  if ((long long)h * w > (1LL << 30) || (long long)n * c_in > (1LL << 31)) return CWG_EINVAL;
  int mm = 0, path = 0;
  int rc = decide(c_in, c_out, m, flags, &mm, &path);
  if (rc) return rc;
  const int relu = (flags & CWG_RELU) ? 1 : 0;
  const int bf16 = (flags & CWG_BF16) ? 1 : 0;
  if (path == CWG_PATH_TC) {
    return cwgk_conv_tc(x, U, bias, y, n, c_in, c_out, h, w, mm, tc_products(mm, flags),
                        tc_variant(flags, mm, c_out), bf16, relu, !(flags & CWG_NO_SPLIT),
                        !(flags & CWG_NO_PDL), stream);
  }
  if (small_cin(c_in, mm))
    return cwgk_conv_small(x, U, bias, y, n, c_in, c_out, h, w, bf16, relu, stream);
  cwgk_ffma_cfg cfg;
  int slices = 1;
  const int idx = pick_ffma(n, c_in, c_out, h, w, mm, flags, &cfg, &slices);
  if (idx < 0) return CWG_EUNSUPPORTED;
  return cwgk_conv_ffma(idx, x, U, bias, y, n, c_in, c_out, h, w, bf16, relu, slices, stream);
}

/* ---- per-thread context: staging for the per-tile calls, copy streams ---- */

/* Per-thread staging: a stream and one device buffer that grows on demand.
 * Freed by the thread-exit destructor; the main thread's copy lives until
 * process exit. */
typedef struct tile_ctx {
  int dev;
  cudaStream_t stream;
  void *buf;
  size_t cap;
  /* copy streams and events of the pipelined host-buffer layer call */
  cudaStream_t s_in, s_out;
  cudaEvent_t ev_start, ev_in, ev_comp, ev_done;
  int pipe_ready;
} tile_ctx;

static pthread_key_t g_ctx_key;
static pthread_once_t g_ctx_once = PTHREAD_ONCE_INIT;
static __thread int t_status = CWG_OK;

static void ctx_free(void *p) {
  tile_ctx *c = (tile_ctx *)p;
  if (!c) return;
  if (c->buf) cudaFree(c->buf);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->pipe_ready) {
    cudaStreamDestroy(c->s_in);
    cudaStreamDestroy(c->s_out);
    cudaEventDestroy(c->ev_start);
    cudaEventDestroy(c->ev_in);
    cudaEventDestroy(c->ev_comp);
    cudaEventDestroy(c->ev_done);
  }
  free(c);
}

static void ctx_key_init(void) { pthread_key_create(&g_ctx_key, ctx_free); }

static int ctx_get(size_t need, tile_ctx **out) {
  pthread_once(&g_ctx_once, ctx_key_init);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (e == cudaErrorNoDevice) ? CWG_ENODEV : cuda_fail(e);
  tile_ctx *c = (tile_ctx *)pthread_getspecific(g_ctx_key);
  if (c && c->dev != dev) {
    ctx_free(c);
    c = NULL;
    pthread_setspecific(g_ctx_key, NULL);
  }
  if (!c) {
    c = (tile_ctx *)calloc(1, sizeof(*c));
    if (!c) return CWG_ENOMEM;
    c->dev = dev;
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      free(c);
      return cuda_fail(e);
    }
    pthread_setspecific(g_ctx_key, c);
  }
  if (need > 0 && c->cap < need) {
    if (c->buf) cudaFree(c->buf);
    c->buf = NULL;
    c->cap = 0;
    e = cudaMalloc(&c->buf, need);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return (e == cudaErrorMemoryAllocation) ? CWG_ENOMEM : cuda_fail(e);
    }
    c->cap = need;
  }
  *out = c;
  return CWG_OK;
}

size_t cwg_host_workspace_bytes(int n, int c_in, int c_out, int h, int w, unsigned flags) {
  if (n < 0 || c_in <= 0 || c_out <= 0 || h <= 0 || w <= 0) return 0;
  const size_t esz = (flags & CWG_BF16) ? 2 : 4;
  const size_t xb = ((size_t)n * c_in * h * w * esz + 255) / 256 * 256;
  const size_t yb = ((size_t)n * c_out * h * w * esz + 255) / 256 * 256;
  return xb + yb;
}

/* One stream: copy x in, convolve, copy y out, synchronise.  Creates nothing
 * and allocates nothing (the no-allocation entry point relies on that). */
int cwgh_conv_host_serial(const void *x_host, const void *U, const float *bias, void *y_host,
                          char *xd, char *yd, size_t xbytes, size_t ybytes, int n, int c_in,
                          int c_out, int h, int w, int m, unsigned flags, void *stream) {
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(xd, x_host, xbytes, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e);
  /* an ordinary launch between the copies: nothing to overlap here */
  int rc = cwg_conv3x3_fused(xd, U, bias, yd, n, c_in, c_out, h, w, m, flags | CWG_NO_PDL, s);
  if (rc) return rc;
  e = cudaMemcpyAsync(y_host, yd, ybytes, cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e);
  return CWG_OK;
}

static int pipe_ready(tile_ctx *c) {
  if (c->pipe_ready) return CWG_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&c->s_in, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->s_out, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_start, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_in, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_comp, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_done, cudaEventDisableTiming);
  if (e != cudaSuccess) return cuda_fail(e);
  c->pipe_ready = 1;
  return CWG_OK;
}

/* Large layers: the batch is cut into image chunks; chunk i's copy-in (copy
 * stream), convolution (caller's stream) and copy-out (second copy stream)
 * overlap with the neighbouring chunks, so the call costs about one
 * direction of host<->device traffic instead of both plus the kernel.  Chunk
 * sizes ramp up (1, 2, 4, ... images) to the steady size and back down at the
 * end: the first copy-in and the last copy-out, which nothing overlaps, stay
 * short. */
#define HOST_PIPE_MIN_BYTES (8u << 20)
#define HOST_PIPE_STEADY 5 /* steady chunks: about n / 5 images each */
#define HOST_PIPE_MAX_CHUNKS 64

/* Chunk sizes for n images; returns the number of chunks (<= HOST_PIPE_MAX_CHUNKS). */
static int pipe_chunks(int n, int *sizes) {
  int steady = n / HOST_PIPE_STEADY;
  if (steady < 1) steady = 1;
  int head[8], nh = 0;
  for (int r = 1; r < steady && nh < 8; r *= 2) head[nh++] = r;
  int ramp = 0;
  for (int i = 0; i < nh; ++i) ramp += 2 * head[i];
  while (nh > 0 && ramp > n) {  /* batch too small for the full ramp */
    --nh;
    ramp -= 2 * head[nh];
  }
  int k = 0;
  for (int i = 0; i < nh; ++i) sizes[k++] = head[i];
  int mid = n - ramp;
  const int nmid = mid > 0 ? (mid + steady - 1) / steady : 0;
  for (int i = 0; i < nmid && k < HOST_PIPE_MAX_CHUNKS - nh; ++i) {
    const int cnt = (mid - (mid / nmid) * nmid > i) ? mid / nmid + 1 : mid / nmid;
    sizes[k++] = cnt;
  }
  for (int i = nh - 1; i >= 0; --i) sizes[k++] = head[i];
  return k;
}

int cwg_conv3x3_fused_host(const void *x_host, const void *U, const float *bias, void *y_host,
                           void *workspace, size_t workspace_bytes, int n, int c_in, int c_out,
                           int h, int w, int m, unsigned flags, void *stream) {
  const size_t need = cwg_host_workspace_bytes(n, c_in, c_out, h, w, flags);
  if (need == 0 || !x_host || !y_host || !workspace || workspace_bytes < need ||
      ((uintptr_t)workspace & 255))
    return CWG_EINVAL;
  const size_t esz = (flags & CWG_BF16) ? 2 : 4;
  const size_t xbytes = (size_t)n * c_in * h * w * esz;
  const size_t ybytes = (size_t)n * c_out * h * w * esz;
  char *xd = (char *)workspace;
  char *yd = xd + (xbytes + 255) / 256 * 256;
  cudaStream_t s = (cudaStream_t)stream;
  if (n < 2 || xbytes + ybytes < HOST_PIPE_MIN_BYTES)
    return cwgh_conv_host_serial(x_host, U, bias, y_host, xd, yd, xbytes, ybytes, n, c_in, c_out,
                                 h, w, m, flags, s);
  tile_ctx *c = NULL;
  int rc = ctx_get(0, &c);
  if (rc) return rc;
  rc = pipe_ready(c);
  if (rc) return rc;
  const size_t xi = xbytes / (size_t)n, yi = ybytes / (size_t)n;  /* bytes per image */
  int sizes[HOST_PIPE_MAX_CHUNKS];
  const int chunks = pipe_chunks(n, sizes);
  /* everything already queued on the caller's stream comes first */
  cudaError_t e = cudaEventRecord(c->ev_start, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(c->s_in, c->ev_start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(c->s_out, c->ev_start, 0);
  if (e != cudaSuccess) return cuda_fail(e);
  int done = 0;
  for (int i = 0; i < chunks; ++i) {
    const int cnt = sizes[i];
    const size_t xo = (size_t)done * xi, yo = (size_t)done * yi;
    e = cudaMemcpyAsync(xd + xo, (const char *)x_host + xo, (size_t)cnt * xi,
                        cudaMemcpyHostToDevice, c->s_in);
    if (e == cudaSuccess) e = cudaEventRecord(c->ev_in, c->s_in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, c->ev_in, 0);
    if (e != cudaSuccess) return cuda_fail(e);
    /* ordinary launches: each chunk's kernel follows an event wait on its copy */
    rc = cwg_conv3x3_fused(xd + xo, U, bias, yd + yo, cnt, c_in, c_out, h, w, m,
                           flags | CWG_NO_PDL, stream);
    if (rc) return rc;
    e = cudaEventRecord(c->ev_comp, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(c->s_out, c->ev_comp, 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync((char *)y_host + yo, yd + yo, (size_t)cnt * yi,
                          cudaMemcpyDeviceToHost, c->s_out);
    if (e != cudaSuccess) return cuda_fail(e);
    done += cnt;
  }
  e = cudaEventRecord(c->ev_done, c->s_out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, c->ev_done, 0);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e);
  return CWG_OK;
}

int cwg_device_status(void *stream) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e);
  unsigned st = 0;
  if (cwgk_read_clear_status(&st)) return CWG_ECUDA;
  if (st & 1u) return CWG_ETIMEOUT;
  return st ? CWG_ERANGE : CWG_OK;
}

static size_t al256(size_t b) { return (b + 255) / 256 * 256; }

int cwg_tiles_fused(const float *tiles, const float *U, float *out, int n_tiles, int c_in,
                    int c_out, int td) {
  int rc = CWG_OK;
  if (td != 4 && td != 6 && td != 8)
    rc = CWG_EINVAL;
  else if (c_in <= 0 || c_out <= 0 || n_tiles < 0)
    rc = CWG_EINVAL;
  else if (n_tiles > 0 && (!tiles || !U || !out))
    rc = CWG_EINVAL;
  if (rc || n_tiles == 0) return t_status = rc;
  const size_t m = (size_t)td - 2, nf = (size_t)td * td;
  const size_t tb = (size_t)n_tiles * c_in * nf * 4, ub = (size_t)c_out * c_in * nf * 4,
               ob = (size_t)n_tiles * c_out * m * m * 4;
  tile_ctx *c = NULL;
  rc = ctx_get(al256(tb) + al256(ub) + al256(ob), &c);
  if (rc) return t_status = rc;
  char *dt = (char *)c->buf, *du = dt + al256(tb), *dout = du + al256(ub);
  cudaError_t e = cudaMemcpyAsync(dt, tiles, tb, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(du, U, ub, cudaMemcpyHostToDevice, c->stream);
  if (e != cudaSuccess) return t_status = cuda_fail(e);
  rc = cwgk_tiles((const float *)dt, (const float *)du, (float *)dout, n_tiles, c_in, c_out, td,
                  c->stream);
  if (rc) return t_status = rc;
  e = cudaMemcpyAsync(out, dout, ob, cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return t_status = cuda_fail(e);
  return t_status = CWG_OK;
}

int cwg_last_status(void) { return t_status; }

void fused_winograd_f23(const float *input, const float *U, float *output, int c_in, int c_out) {
  const int rc = cwg_tiles_fused(input, U, output, 1, c_in, c_out, 4);
  if (rc != CWG_OK && output && c_out > 0) {
    const float qnan = nanf("");
    for (int i = 0; i < 4 * c_out; ++i) output[i] = qnan;
  }
}
