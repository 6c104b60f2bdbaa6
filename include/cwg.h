/*
 * cwg.h -- C ABI of libcwg, a B200 (sm_100a) fused Winograd 3x3 convolution.
 *
 * Every entry point is plain C: pointers, sizes and an opaque CUDA stream
 * (`void *stream`, a cudaStream_t; NULL means the legacy default stream).
 * Nothing here allocates device memory on the per-layer path: the caller owns
 * every buffer.  Functions return CWG_OK (0) or a negative CWG_E* status, and
 * never abort the process.
 *
 * Reference interfaces (paths relative to the reference project):
 *   fused_winograd_f23 ...... fused_winograd.c:103-108, same symbol, argument
 *                             order and per-tile layouts; host pointers.
 *   cwg_tiles_fused ......... the batch form of the same per-tile operation for
 *                             every tile size run_fused accepts
 *                             (src/fused_winograd_kernel.py:153-181, td 4/6/8).
 *   cwg_weight_transform .... U = G g G^T; the reference has no weight
 *                             transform and takes U as input (fused_winograd.c:21).
 *   cwg_weight_import ....... takes U already transformed, in the reference's
 *                             [C_out][C_in][td][td] layout (fused_winograd.c:74).
 *   cwg_conv3x3_fused ....... the layer-level convolution (NCHW, pad=1, stride=1)
 *                             the reference's benchmarks emulate by looping one
 *                             tile (benchmarks/jetson_main_microbench.py:47-80);
 *                             argument order follows fused_winograd.c:103
 *                             (input, U, output, then sizes).
 *   cwg_select .............. tile-size / kernel selector replacing
 *                             CacheAdaptiveAutotiler.select_best_tile
 *                             (src/cache_adaptive_autotiler.py:50-82) and the
 *                             task grid of LocalityScheduler.generate_tile_tasks
 *                             (src/locality_scheduler.py:10-43).
 */
#ifndef CWG_H
#define CWG_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define CWG_OK 0
#define CWG_EINVAL (-1)       /* bad size, NULL pointer, misaligned pointer */
#define CWG_EUNSUPPORTED (-2) /* valid request this build cannot serve (e.g. m=6 per layer) */
#define CWG_ECUDA (-3)        /* a CUDA runtime call failed (see cwg_last_cuda_error) */
#define CWG_ETIMEOUT (-4)     /* a bounded device-side wait gave up; results invalid */
#define CWG_ENOMEM (-5)       /* host or device allocation failed (per-tile entries only) */
#define CWG_ENODEV (-6)       /* no usable sm_100 device */
#define CWG_ERANGE (-7)       /* an operand left the range of the kernel's fp16 arithmetic
                                 (bf16 F(4,3) tensor-core layers: |x| above ~650 or |g|
                                 above ~900); results invalid, rerun with CWG_TC_X3 */

/* ---- flags for the layer-level calls -------------------------------------- */
#define CWG_RELU 0x1u        /* fused ReLU after bias */
#define CWG_BF16 0x2u        /* x, y and U in bfloat16, fp32 accumulation */
#define CWG_FORCE_FFMA 0x10u /* ablation: always take the CUDA-core (FFMA) kernel */
#define CWG_FORCE_TC 0x20u   /* ablation: always take the tcgen05 kernel (EUNSUPPORTED if it cannot) */
#define CWG_TC_SINGLE 0x40u  /* ablation: fp32 I/O with ONE bf16 product per MAC (below fp32 parity) */
#define CWG_TC_FULL16 0x80u  /* ablation: single-CTA tensor-core kernel with all 16 frequency
                                accumulators (32-tile blocks) */
#define CWG_TC_NOPAIR 0x100u /* ablation: single-CTA half-folded tensor-core kernel (64-tile
                                blocks) instead of the 2-SM pair kernel (128-tile blocks) */
#define CWG_NO_SPLIT 0x200u  /* bit-reproducible results: never split the C_in reduction of a small
                                fp32 layer across CTAs (a split adds partial sums atomically, so
                                the last bits of y vary between runs) */
#define CWG_TC_X3 0x400u     /* bf16 F(4,3) layers on the tensor cores: three bf16 products per
                                MAC (hi/lo split of both operands, any bf16 range) instead of the
                                default two fp16 products (U * V_hi + U * V_lo, ~2/3 of the
                                time; inputs must stay within fp16's range after the transform,
                                else cwg_device_status reports CWG_ERANGE) */
#define CWG_NO_PDL 0x800u    /* launch the tensor-core kernel as an ordinary stream launch; by
                                default it is a programmatic dependent launch: its CTAs may
                                start (barriers, TMEM) while the previous kernel in the stream
                                finishes, and wait for that kernel's completion before they
                                touch global memory */

/* Kernel paths reported by cwg_select. */
#define CWG_PATH_FFMA 1 /* warp register-blocked FFMA fused kernel */
#define CWG_PATH_TC 2   /* tcgen05/TMEM fused kernel */

/* Result of the tile selector.  All fields are outputs. */
typedef struct cwg_choice {
  int m;             /* output tile edge: 2 -> F(2x2,3x3), 4 -> F(4x4,3x3), 6 -> F(6x6,3x3)
                        (CUDA-core path only) */
  int path;          /* CWG_PATH_* */
  int tiles_per_cta; /* output tiles one CTA owns (one CTA pair, for the 2-SM kernel) */
  int cout_per_cta;  /* output channels one CTA owns */
  int cin_chunk;     /* input channels staged per pipeline step */
  int threads;       /* threads per CTA */
  int smem_bytes;    /* dynamic shared memory per CTA */
  int tmem_cols;     /* tensor-memory columns per CTA (0 on the FFMA path) */
  long long ctas;    /* CTAs in the grid */
  double gemm_flops; /* 2 * tiles * C_out * C_in * (m+2)^2 */
  double alg_bytes;  /* x + y + U + bias, each touched once */
  int mma_products;  /* tensor-core products per multiply-accumulate: 3 (bf16 hi/lo split,
                        fp32-accurate), 2 (fp16, V split into hi + lo: bf16 F(4,3) layers)
                        or 1 (bf16); 0 on the FFMA path */
  long long ctas_launched; /* CTAs the launch really uses: `ctas`, or for a layer larger than
                              one wave of CTA pairs, two per co-resident cluster of the current
                              device (B200's 74 TPCs when no device is present) */
  int order;         /* CWG_ORDER_*: how the tensor-core kernel walks its work */
} cwg_choice;

/* cwg_choice.order */
#define CWG_ORDER_GRID 0  /* one work unit (tile block x channel block x C_in slice) per CTA
                             or CTA pair */
#define CWG_ORDER_RUNS 1  /* persistent pairs, each an equal run of tiles */
#define CWG_ORDER_ROUND 2 /* persistent pairs, round robin over the work units */

/* ---- reference-compatible per-tile entry points (HOST pointers) ----------- */

/* fused_winograd.c:103-108.  input [c_in][4][4], U [c_out][c_in][4][4],
 * output [c_out][2][2], all fp32 host memory.  Runs on the current CUDA
 * device.  Like the reference it returns nothing: on failure the output is
 * filled with NaN and cwg_last_status() reports why.  Reentrant: every host
 * thread gets its own stream and staging buffers. */
void fused_winograd_f23(const float *input, const float *U, float *output, int c_in, int c_out);

/* n_tiles independent tiles: tiles [n_tiles][c_in][td][td], U
 * [c_out][c_in][td][td], out [n_tiles][c_out][td-2][td-2]; td in {4, 6, 8}
 * (F(2,3), F(4,3), F(6,3)); fp32 host memory. */
int cwg_tiles_fused(const float *tiles, const float *U, float *out, int n_tiles, int c_in,
                    int c_out, int td);

/* Status of the calling thread's last per-tile call. */
int cwg_last_status(void);

/* ---- layer-level API (DEVICE pointers) ----------------------------------- */

/* Bytes of transformed weights for (c_in, c_out, m, flags); 0 if invalid. */
size_t cwg_weight_bytes(int c_in, int c_out, int m, unsigned flags);

/* g: fp32 [c_out][c_in][3][3] on the device -> U (cwg_weight_bytes bytes) in
 * the layout the selected kernel reads.  m = 0 lets cwg_select choose. */
int cwg_weight_transform(const float *g, void *U, int c_in, int c_out, int m, unsigned flags,
                         void *stream);

/* U_ref: fp32 [c_out][c_in][m+2][m+2] on the device (reference layout) -> U. */
int cwg_weight_import(const float *U_ref, void *U, int c_in, int c_out, int m, unsigned flags,
                      void *stream);

/* y = [ReLU](conv3x3(x, g) + bias), x [n][c_in][h][w], y [n][c_out][h][w],
 * fp32 (or bf16 with CWG_BF16), pad=1, stride=1.  U from cwg_weight_transform
 * or cwg_weight_import with the same (c_in, c_out, m, flags); bias may be
 * NULL.  Asynchronous on `stream`. */
int cwg_conv3x3_fused(const void *x, const void *U, const float *bias, void *y, int n, int c_in,
                      int c_out, int h, int w, int m, unsigned flags, void *stream);

/* End-to-end form: x_host and y_host are host buffers (pinned for full copy
 * speed); the call copies x in, runs cwg_conv3x3_fused on the device staging
 * buffers in `workspace` (at least cwg_host_workspace_bytes bytes), copies y
 * out and synchronises the stream. */
size_t cwg_host_workspace_bytes(int n, int c_in, int c_out, int h, int w, unsigned flags);
int cwg_conv3x3_fused_host(const void *x_host, const void *U, const float *bias, void *y_host,
                           void *workspace, size_t workspace_bytes, int n, int c_in, int c_out,
                           int h, int w, int m, unsigned flags, void *stream);

/* For callers that cannot allocate device memory (a framework's allocator
 * owns the device heap, a plug-in host hands over only host buffers and a
 * stream, or a real-time path may not allocate after start-up): the same call
 * as cwg_conv3x3_fused_host, but staging x and y in a fixed device array of
 * CWG_STATIC_WORKSPACE_BYTES that the library holds on every GPU that loads
 * it, so the call allocates nothing.  No counterpart in the reference.
 * Limits: cwg_host_workspace_bytes(n, c_in, c_out, h, w, flags) must not
 * exceed CWG_STATIC_WORKSPACE_BYTES (CWG_EUNSUPPORTED otherwise).  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture.  All calls share the one
 * array: calls whose work overlaps on the GPU (different streams or threads
 * without ordering) race on it.  `stream` must belong to the current device
 * (CWG_EINVAL otherwise); n == 0 returns CWG_OK; a device reset after the
 * first call on that device is not supported. */
#define CWG_STATIC_WORKSPACE_BYTES (32u << 20)
int cwg_conv3x3_fused_host_static(const void *x_host, const void *U, const float *bias,
                                  void *y_host, int n, int c_in, int c_out, int h, int w, int m,
                                  unsigned flags, void *stream);

/* ---- non-fused ablation ---------------------------------------------------- */

/* The same fp32 layer as three passes over HBM, for measuring what the fused
 * kernels save: input transform -> V in `workspace`, one GEMM per frequency ->
 * M[(m+2)^2][c_out][T] fp32, output transform + bias (+ ReLU with CWG_RELU) -> y;
 * T = n*ceil(h/m)*ceil(w/m).  The GEMM does the arithmetic of the fused kernel
 * of the same layer: tcgen05 MMAs with the bf16 hi/lo split for m = 2 (V and U
 * as bf16 UMMA blocks), fp32 FFMA for m = 4 and 6.
 * Mirrors the reference's run_non_fused (src/fused_winograd_kernel.py:116-151),
 * whose math equals run_fused.  U in the CUDA-core layout: produce it with
 * cwg_weight_transform(..., m, CWG_FORCE_FFMA, ...).  m = 2, 4 or 6; fp32 only
 * (any flag but CWG_RELU -> CWG_EINVAL); workspace 256-byte aligned, at least
 * cwg_nonfused_workspace_bytes() bytes.  Device pointers; `stream` as above. */
size_t cwg_nonfused_workspace_bytes(int n, int c_in, int c_out, int h, int w, int m);
int cwg_conv3x3_nonfused(const float *x, const float *U, const float *bias, float *y,
                         void *workspace, size_t workspace_bytes, int n, int c_in, int c_out,
                         int h, int w, int m, unsigned flags, void *stream);

/* ---- selector, diagnostics ----------------------------------------------- */

/* Chooses m (when m == 0), the kernel path and its blocking for a layer on the
 * current device.  Pure host computation: launches nothing. */
int cwg_select(int n, int c_in, int c_out, int h, int w, int m, unsigned flags, cwg_choice *out);

/* Human-readable text for a CWG_* status. */
const char *cwg_strerror(int status);

/* cudaError_t of the last failing CUDA call in this thread (0 if none). */
int cwg_last_cuda_error(void);

/* Synchronises `stream`, then reads and clears the device-side status word
 * that bounded waits inside the kernels set when they give up, and that the
 * fp16 tensor-core path sets when an operand leaves fp16's range.  Returns
 * CWG_ETIMEOUT if any kernel since the last call timed out, else CWG_ERANGE if
 * an operand overflowed, else CWG_OK (or CWG_ECUDA if the synchronisation
 * itself failed). */
int cwg_device_status(void *stream);

/* Self-test of the failure path: launches one CTA whose bounded device wait can
 * never complete (an mbarrier nothing arrives on).  After the wait limit (~2 s)
 * it gives up and sets the status word, so the next cwg_device_status(stream)
 * returns CWG_ETIMEOUT; the context stays usable.  No reference counterpart. */
int cwg_selftest_wait_timeout(void *stream);

/* Number of kernel launches this process made through libcwg (all threads). */
long long cwg_launch_count(void);

/* Library version string. */
const char *cwg_version(void);

#ifdef __cplusplus
}
#endif
#endif /* CWG_H */
