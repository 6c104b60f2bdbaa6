/*
 * cwg_internal.h -- the thin C boundary between the host code (cwg_host.c,
 * plain C) and the CUDA translation units.  Not installed; not part of the
 * public ABI in include/cwg.h.
 */
#ifndef CWG_INTERNAL_H
#define CWG_INTERNAL_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Layouts of the transformed weights U in device memory. */
enum {
  CWGK_LAYOUT_FFMA_F32 = 1,  /* fp32 [td*td][C_in][C_out] (fp32 and bf16 layers)  */
  CWGK_LAYOUT_TC_X3 = 3,     /* bf16 hi+lo UMMA blocks (fp32-parity tensor path)  */
  CWGK_LAYOUT_TC_X1 = 4,     /* bf16 UMMA blocks (single product)                 */
  CWGK_LAYOUT_TC2_X3 = 5,    /* pair kernel: At-scaled hi+lo blocks, 2 rank sets  */
  CWGK_LAYOUT_TC2_X1 = 6,    /* pair kernel: At-scaled blocks, single product     */
  CWGK_LAYOUT_TC2H_X3 = 7,   /* 64-channel pair kernel: 64-row hi+lo blocks       */
  CWGK_LAYOUT_TC2H_X1 = 8,   /* 64-channel pair kernel: 64-row blocks, 1 product  */
  CWGK_LAYOUT_TC2_H2 = 9,    /* pair kernel: At-scaled fp16 blocks (F(4,3), bf16) */
  CWGK_LAYOUT_TC2H_H2 = 10   /* the same for F(4,3) layers of <= 64 channels      */
};

/* Tensor-core kernel variants. */
enum {
  CWGK_TC_PAIR = 0,   /* 2-SM pair, M = 256 (stacked output rows), F(2,3) and F(4,3) */
  CWGK_TC_HALF = 1,   /* one CTA, half-folded, M = 128, N = 64                  */
  CWGK_TC_FULL16 = 2, /* one CTA, 16 frequency accumulators, N = 32             */
  CWGK_TC_PAIR64 = 3  /* 2-SM pair, 64 output channels per CTA: F(2,3) M = 128;
                         F(4,3) two output rows x 64 channels                   */
};

/* One compiled FFMA kernel configuration. */
typedef struct cwgk_ffma_cfg {
  int m;       /* 2 or 4 */
  int ty, tx;  /* tiles per CTA along y and x */
  int kb;      /* output channels per CTA */
  int cc;      /* input channels per pipeline step */
  int threads; /* threads per CTA */
  int smem;    /* dynamic shared memory bytes */
} cwgk_ffma_cfg;

/* Tensor-core kernel geometry (fixed per build). */
typedef struct cwgk_tc_cfg {
  int m;          /* output tile edge (2) */
  int tiles;      /* output tiles per CTA (per pair for the pair kernel) */
  int kb;         /* output channels per CTA (MMA M) */
  int cc;         /* input channels per pipeline stage */
  int threads;    /* threads per CTA */
  int smem;       /* dynamic shared memory bytes */
  int tmem_cols;  /* TMEM columns allocated */
  int ctas_per_tile_block; /* CTAs that share one block of `tiles` tiles */
} cwgk_tc_cfg;

int cwgk_ffma_num_cfgs(void);
int cwgk_ffma_get_cfg(int idx, cwgk_ffma_cfg *out);
/* pm: products per multiply-accumulate (1 bf16, 2 fp16 with V split, 3 bf16 split) */
int cwgk_tc_get_cfg(int pm, int variant, int m, cwgk_tc_cfg *out);

/* g (or U_ref when from_ref) -> U in `layout`.  Device pointers. */
int cwgk_weight_transform(const float *src, void *U, int c_in, int c_out, int m, int layout,
                          int from_ref, void *stream);

/* Tensor-core weight layouts (CWGK_LAYOUT_TC_*), defined with the tcgen05 kernel. */
int cwgk_weight_transform_tc(const float *src, void *U, int c_in, int c_out, int m, int layout,
                             int from_ref, void *stream);

/* F(2,3) for layers of 1-4 input channels (csrc/cwg_small.cu): one thread per tile,
 * 64 output channels per CTA, weights in the CUDA-core layout. */
int cwgk_conv_small(const void *x, const void *U, const float *bias, void *y, int n, int c_in,
                    int c_out, int h, int w, int bf16, int relu, void *stream);

/* FFMA fused convolution with configuration `cfg_idx`.  slices > 1 (fp32 only)
 * splits the C_in steps across that many CTAs per tile block (y zeroed, partial
 * sums added atomically, bias with slice 0 or, with ReLU, in a second pass). */
int cwgk_conv_ffma(int cfg_idx, const void *x, const void *U, const float *bias, void *y, int n,
                   int c_in, int c_out, int h, int w, int bf16, int relu, int slices,
                   void *stream);
/* bias + ReLU in place over the n*c_out fp32 planes of h*w in y (after a split
 * reduction). */
int cwgk_bias_relu(float *y, const float *bias, int n, int c_out, int h, int w, int relu,
                   void *stream);

/* tcgen05 fused convolution F(m x m, 3x3) (C_in padded to 16 and C_out to the
 * channel block by the weight layout), kernel `variant` (CWGK_TC_*; the
 * single-CTA variants are F(2,3) only).  allow_split: the pair kernel may split
 * the C_in reduction of small fp32 layers across CTAs (y zeroed, partial sums
 * added atomically, bias and ReLU in a second pass).  allow_pdl: the pair
 * kernel is a programmatic dependent launch (see CWG_NO_PDL). */
int cwgk_conv_tc(const void *x, const void *U, const float *bias, void *y, int n, int c_in,
                 int c_out, int h, int w, int m, int pm, int variant, int bf16, int relu,
                 int allow_split, int allow_pdl, void *stream);

/* C_in slices the tensor-core path uses for this layer (1 = no split). */
int cwgk_tc_splits(int n, int c_in, int c_out, int h, int w, int m, int variant, int bf16,
                   int allow_split, int sms);
/* The pair kernel's launch plan for a layer on the current device (or, without
 * one, `sms` SMs): CTAs launched and CWG_ORDER_*. */
int cwgk_tc_plan(int n, int c_in, int c_out, int h, int w, int m, int pm, int variant, int bf16,
                 int allow_split, int sms, long long *ctas, int *order);

/* Non-fused ablation on the tensor cores.  Bytes of one operand in UMMA blocks of
 * 128 rows x 16 channels, hi and lo bf16 (rows = output channels or tiles). */
size_t cwgk_gemm_blocks_bytes(int nf, int rows, int c_in);
/* U (CUDA-core layout, fp32 [nf][C][K]) -> Ug blocks, and the input pass x -> V = Bt d B
 * in Vg blocks (nf = (m+2)^2 frequencies, T = n ceil(h/m) ceil(w/m) tiles). */
int cwgk_gemm_prepare(const float *U, void *Ug, const float *x, void *Vg, int m, int n, int c_in,
                      int c_out, int h, int w, void *stream);
/* M[f][k][t] = sum_c U_f[k][c] V_f[c][t] (fp32 out) with three bf16 products per MAC. */
int cwgk_gemm_x3(const void *Ug, const void *Vg, float *Mf, int nf, int c_in, int c_out, int T,
                 void *stream);

/* Per-tile kernel on device buffers (reference layouts). */
int cwgk_tiles(const float *tiles, const float *U, float *out, int n_tiles, int c_in, int c_out,
               int td, void *stream);

/* Host-buffer layer call on one stream (copy in, convolve, copy out, sync),
 * staging in xd/yd; creates and allocates nothing. */
int cwgh_conv_host_serial(const void *x_host, const void *U, const float *bias, void *y_host,
                          char *xd, char *yd, size_t xbytes, size_t ybytes, int n, int c_in,
                          int c_out, int h, int w, int m, unsigned flags, void *stream);

/* Reads and clears the device status word (after the caller synchronised):
 * bit 0 a bounded wait gave up, bit 1 an fp16 operand left fp16's range. */
int cwgk_read_clear_status(unsigned *status);

/* Launch counter shared by all translation units. */
void cwgk_count_launch(void);
long long cwgk_launches(void);

/* Records the last CUDA error code for the calling thread. */
void cwgk_set_cuda_error(int err);
int cwgk_get_cuda_error(void);

#ifdef __cplusplus
}
#endif
#endif /* CWG_INTERNAL_H */
