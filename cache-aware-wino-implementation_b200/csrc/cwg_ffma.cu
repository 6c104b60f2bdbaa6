// cwg_ffma.cu -- CUDA-core kernels of libcwg:
//   * wt_transform        U = G g G^T (or an import of a reference-layout U)
//   * wino_fused_ffma     the fused layer kernel for small channel counts
//                         (halo load -> Bt d B -> per-frequency register-blocked
//                         FFMA GEMMs -> At M A + bias + ReLU -> store)
//   * tiles_fused         the reference's per-tile operation on device buffers
// plus the launch shims declared in cwg_internal.h.
#include <atomic>
#include <cstdio>

#include "cwg_common.cuh"

namespace cwg {

static std::atomic<long long> g_launches{0};
static thread_local int t_cuda_error = 0;

// ============================================================================
// Weight transform
// ============================================================================
// One thread per (c, k); k fastest so the [f][C][K] stores coalesce.
template <int M>
__global__ void wt_transform_ffma(const float *__restrict__ src, float *__restrict__ U, int C,
                                  int K, int from_ref) {
  constexpr int NF = (M + 2) * (M + 2);
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)C * K) return;
  const int k = (int)(idx % K), c = (int)(idx / K);
  float u[NF];
  transform_one<M>(src + ((long)k * C + c) * (from_ref ? NF : 9), from_ref, u);
#pragma unroll
  for (int f = 0; f < NF; ++f) U[((long)f * C + c) * K + k] = u[f];
}

// ============================================================================
// Fused FFMA kernel
// ============================================================================
// CTA = TY x TX output tiles of one image x KB output channels, looping over
// the input channels in steps of CC.  Per step:
//   * U[f][c0:c0+CC][k0:k0+KB] arrives by 16-byte cp.async into one of two
//     buffers while the previous step computes (double buffering);
//   * the (TY*M+2) x (TX*M+2) input halo of the step (zero outside the image =
//     pad 1) was loaded into registers during the previous step and is now
//     written to shared memory;
//   * every thread transforms a slice of frequency rows of one (channel, tile)
//     patch (Bt d B), so the whole CTA shares the transform;
//   * each warp runs the GEMM of FPW frequencies, every lane holding a TR x KR
//     register block (tiles x output channels).
// The epilogue regroups the frequency accumulators through shared memory and
// applies At M A, bias and ReLU, storing NCHW.  With `slices` > 1 (fp32 only) the
// steps are split into that many C_in ranges, one per CTA (blockIdx.z = image *
// slices + slice): each CTA adds its partial At M A into the zeroed y with fp32
// atomics, slice 0 adding the bias; ReLU, if any, then needs a second pass.
template <int M, int TY, int TX, int KB, int CC, int FPW>
struct FG {
  static constexpr int TD = M + 2, NF = TD * TD, T = TY * TX;
  static constexpr int HR = TY * M + 2, WR = TX * M + 2;
  static constexpr int KR = 4, KG = KB / KR, TG = 32 / KG, TR = T / TG;
  static constexpr int NW = NF / FPW, NT = NW * 32;
  static constexpr int XS = CC * HR * WR, VS = NF * CC * T, US = NF * CC * KB;
  static constexpr int XPT = (XS + NT - 1) / NT;          // halo elements per thread
  static constexpr int U4 = US / 4, U4PT = (U4 + NT - 1) / NT;  // 16-byte U chunks per thread
  static constexpr int PAIRS = CC * T;                     // (channel, tile) patches per step
  static constexpr int PARTS = NT / PAIRS;                 // threads per patch
  static constexpr int ROWS = TD / PARTS;                  // frequency rows per thread
  static constexpr int MAIN = XS + VS + 2 * US;
  static constexpr int EPI = NF * KG * (T + 1);
  static constexpr int SMEM = 4 * (MAIN > EPI ? MAIN : EPI);
  static_assert(NF % FPW == 0, "frequencies per warp must divide td^2");
  static_assert(KB % KR == 0 && 32 % KG == 0 && T % TG == 0, "lane grid must tile 32");
  static_assert(TR == 2 || TR % 4 == 0, "tile register block must vectorise");
  static_assert(NT % PAIRS == 0 && TD % PARTS == 0, "transform slices must tile the CTA");
  static_assert(KB % 4 == 0, "U rows copy in 16-byte chunks");
};

template <int N>
__device__ __forceinline__ void lds_vec(const float *p, float (&v)[N]) {
  if constexpr (N == 2) {
    const float2 a = *reinterpret_cast<const float2 *>(p);
    v[0] = a.x;
    v[1] = a.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 a = *reinterpret_cast<const float4 *>(p + i);
      v[i] = a.x;
      v[i + 1] = a.y;
      v[i + 2] = a.z;
      v[i + 3] = a.w;
    }
  }
}

// 16-byte global -> shared async copy; src_bytes < 16 zero-fills the rest.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Row A of V = Bt d B: (Bt d)[A][:] then times B, coefficients as immediates.
template <int M, int A>
__device__ __forceinline__ void v_row(const float (&d)[M + 2][M + 2], float (&out)[M + 2]) {
  constexpr int TD = M + 2;
  float trow[TD];
#pragma unroll
  for (int j = 0; j < TD; ++j) {
    float sacc = 0.f;
    bool first = true;
#pragma unroll
    for (int i = 0; i < TD; ++i) {
      const float cf = Wino<M>::bt(A, i);
      if (cf == 0.f) continue;
      sacc = first ? first_term<false>(cf, d[i][j]) : fmaf(cf, d[i][j], sacc);
      first = false;
    }
    trow[j] = sacc;
  }
#pragma unroll
  for (int b = 0; b < TD; ++b) {
    float sacc = 0.f;
    bool first = true;
#pragma unroll
    for (int j = 0; j < TD; ++j) {
      const float cf = Wino<M>::bt(b, j);
      if (cf == 0.f) continue;
      sacc = first ? first_term<false>(cf, trow[j]) : fmaf(cf, trow[j], sacc);
      first = false;
    }
    out[b] = sacc;
  }
}

template <int M>
__device__ __forceinline__ void v_row_dispatch(int a, const float (&d)[M + 2][M + 2],
                                               float (&out)[M + 2]) {
  switch (a) {
    case 0: v_row<M, 0>(d, out); break;
    case 1: v_row<M, 1>(d, out); break;
    case 2: v_row<M, 2>(d, out); break;
    case 3: v_row<M, 3>(d, out); break;
    default:
      if constexpr (M + 2 > 4) {
        if (a == 4) {
          v_row<M, 4>(d, out);
        } else if (a == 5) {
          v_row<M, 5>(d, out);
        } else if constexpr (M + 2 > 6) {
          if (a == 6) v_row<M, 6>(d, out);
          else v_row<M, 7>(d, out);
        }
      }
  }
}

template <int M, int TY, int TX, int KB, int CC, int FPW, typename Tio>
__global__ void __launch_bounds__(FG<M, TY, TX, KB, CC, FPW>::NT, 1)
    wino_fused_ffma(const Tio *__restrict__ x, const float *__restrict__ U,
                    const float *__restrict__ bias, Tio *__restrict__ y, int C, int K, int H,
                    int W, int tiles_y, int tiles_x, int relu, int slices) {
  using G = FG<M, TY, TX, KB, CC, FPW>;
  constexpr int TD = G::TD, T = G::T, NT = G::NT, KR = G::KR, TR = G::TR, KG = G::KG;
  extern __shared__ __align__(16) float smem[];
  float *xs = smem;
  float *vs = xs + G::XS;
  float *us0 = vs + G::VS;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tg = lane / KG, kg = lane % KG;
  const int nbx = (tiles_x + TX - 1) / TX;
  const int by = blockIdx.x / nbx, bx = blockIdx.x - by * nbx;
  // blockIdx.z = image * slices + C_in slice; a slice owns steps [st0, st1)
  const int k0 = blockIdx.y * KB, n = blockIdx.z / slices, slice = blockIdx.z - n * slices;
  const int ty0 = by * TY, tx0 = bx * TX;
  const int iy0 = ty0 * M - 1, ix0 = tx0 * M - 1;
  const size_t plane = (size_t)H * W;
  const Tio *xn = x + (size_t)n * C * plane;
  const int steps = (C + CC - 1) / CC, per = (steps + slices - 1) / slices;
  const int st0 = slice * per, st1 = min(steps, st0 + per);
  const bool u_vec = (K & 3) == 0;  // every U row starts on a 16-byte boundary

  // ---- U step s -> us buffer (s & 1), 16-byte chunks (scalar if K % 4 != 0)
  auto issue_u = [&](int st) {
    float *dst = us0 + (st & 1) * G::US;
    const int c0 = st * CC;
#pragma unroll
    for (int j = 0; j < G::U4PT; ++j) {
      const int q = tid + j * NT;
      if (q < G::U4) {
        const int row = q / (KB / 4), k4 = (q - row * (KB / 4)) * 4;  // row = f * CC + c
        const int f = row / CC, c = row - f * CC;
        const int cg = c0 + c, kk = k0 + k4;
        const float *src = U + ((size_t)f * C + (cg < C ? cg : 0)) * K + (kk < K ? kk : 0);
        float *d = dst + row * KB + k4;
        if (u_vec) {
          const int bytes = (cg < C && kk < K) ? 16 : 0;
          cp_async16(d, src, bytes);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            d[e] = (cg < C && kk + e < K) ? U[((size_t)f * C + cg) * K + kk + e] : 0.f;
        }
      }
    }
    cp_async_commit();
  };
  // ---- input halo of step s -> registers (stored to xs at the start of step s)
  // per element, fixed across steps: (window row << 10) | (window column << 4) |
  // chunk channel, or -1 outside the image / past the halo
  float xr[G::XPT];
  int xpk[G::XPT];
  static_assert(G::HR <= 64 && G::WR <= 64 && CC <= 16, "halo coordinates pack into 16 bits");
#pragma unroll
  for (int j = 0; j < G::XPT; ++j) {
    const int i = tid + j * NT;
    int pk = -1;
    if (i < G::XS) {
      const int c = i / (G::HR * G::WR), rem = i - c * (G::HR * G::WR);
      const int r = rem / G::WR, s2 = rem - r * G::WR;
      const int iy = iy0 + r, ix = ix0 + s2;
      if (iy >= 0 && iy < H && ix >= 0 && ix < W) pk = (r << 10) | (s2 << 4) | c;
    }
    xpk[j] = pk;
  }
  auto load_x = [&](int st) {
    const int cl = C - st * CC;  // chunk channels c < cl exist
#pragma unroll
    for (int j = 0; j < G::XPT; ++j) {
      const int pk = xpk[j];
      float v = 0.f;
      if (pk >= 0 && (pk & 15) < cl)
        v = to_f32(xn[(size_t)(st * CC + (pk & 15)) * plane +
                      (size_t)(iy0 + (pk >> 10)) * W + (ix0 + ((pk >> 4) & 63))]);
      xr[j] = v;
    }
  };

  float acc[FPW][TR][KR];
#pragma unroll
  for (int a = 0; a < FPW; ++a)
#pragma unroll
    for (int b = 0; b < TR; ++b)
#pragma unroll
      for (int c = 0; c < KR; ++c) acc[a][b][c] = 0.f;

  // this thread's transform slice: one (channel, tile) patch and ROWS
  // frequency rows; the slice (part) is uniform across a warp.
  const int part = warp % G::PARTS, tp = (warp / G::PARTS) * 32 + lane;
  const int tc = tp / T, tt = tp - tc * T, tyl = tt / TX, txl = tt - tyl * TX;

  issue_u(st0);
  load_x(st0);
  for (int st = st0; st < st1; ++st) {
    // stage this step's halo, prefetch the next step
#pragma unroll
    for (int j = 0; j < G::XPT; ++j) {
      const int i = tid + j * NT;
      if (i < G::XS) xs[i] = xr[j];
    }
    if (st + 1 < st1) {
      issue_u(st + 1);
      load_x(st + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // transform: rows [part*ROWS, part*ROWS+ROWS) of V for patch (tc, tt)
    {
      const float *src = xs + tc * G::HR * G::WR + (tyl * M) * G::WR + txl * M;
      float d[TD][TD];
#pragma unroll
      for (int r = 0; r < TD; ++r)
#pragma unroll
        for (int c2 = 0; c2 < TD; ++c2) d[r][c2] = src[r * G::WR + c2];
#pragma unroll
      for (int ra = 0; ra < G::ROWS; ++ra) {
        const int a = part * G::ROWS + ra;
        float vrow[TD];
        v_row_dispatch<M>(a, d, vrow);
#pragma unroll
        for (int b2 = 0; b2 < TD; ++b2) vs[((a * TD + b2) * CC + tc) * T + tt] = vrow[b2];
      }
    }
    __syncthreads();
    // per-frequency GEMM on the CUDA cores
    const float *us = us0 + (st & 1) * G::US;
#pragma unroll 2
    for (int c = 0; c < CC; ++c) {
#pragma unroll
      for (int fi = 0; fi < FPW; ++fi) {
        const int f = warp * FPW + fi;
        float vv[TR], uu[KR];
        lds_vec<TR>(vs + (f * CC + c) * T + tg * TR, vv);
        lds_vec<KR>(us + (f * CC + c) * KB + kg * KR, uu);
#pragma unroll
        for (int r = 0; r < TR; ++r)
#pragma unroll
          for (int q = 0; q < KR; ++q) acc[fi][r][q] = fmaf(vv[r], uu[q], acc[fi][r][q]);
      }
    }
    __syncthreads();
  }

  // epilogue: regroup the NF accumulators of each (tile, channel), one
  // register column q at a time, then At M A + bias + ReLU.
  float *ms = smem;  // [NF][KG][T+1]
#pragma unroll
  for (int q = 0; q < KR; ++q) {
#pragma unroll
    for (int fi = 0; fi < FPW; ++fi)
#pragma unroll
      for (int r = 0; r < TR; ++r)
        ms[((warp * FPW + fi) * KG + kg) * (T + 1) + tg * TR + r] = acc[fi][r][q];
    __syncthreads();
    for (int p = tid; p < T * KG; p += NT) {
      const int t = p % T, kgp = p / T;
      const int k = k0 + kgp * KR + q;
      const int tyl2 = t / TX, txl2 = t - tyl2 * TX;
      const int ty = ty0 + tyl2, tx = tx0 + txl2;
      if (k < K && ty < tiles_y && tx < tiles_x) {
        float mm[TD][TD], yy[M][M];
#pragma unroll
        for (int a = 0; a < TD; ++a)
#pragma unroll
          for (int b2 = 0; b2 < TD; ++b2)
            mm[a][b2] = ms[((a * TD + b2) * KG + kgp) * (T + 1) + t];
        output_transform<M>(mm, yy);
        const float bb = (bias && slice == 0) ? bias[k] : 0.f;
        Tio *yk = y + ((size_t)n * K + k) * plane;
#pragma unroll
        for (int i = 0; i < M; ++i)
#pragma unroll
          for (int j = 0; j < M; ++j) {
            const int oy = ty * M + i, ox = tx * M + j;
            if (oy < H && ox < W) {
              float v = yy[i][j] + bb;
              if (slices > 1) {
                // partial sum of this slice into the zeroed y (fp32 only)
                if constexpr (sizeof(Tio) == 4) atomicAdd(&yk[(size_t)oy * W + ox], v);
              } else {
                if (relu) v = v < 0.f ? 0.f : v;
                yk[(size_t)oy * W + ox] = from_f32<Tio>(v);
              }
            }
          }
      }
    }
    __syncthreads();
  }
}

// ============================================================================
// Per-tile kernel (reference layouts; fused_winograd.c:19-101 semantics)
// ============================================================================
// CTA = one tile x 128 output channels; thread = one output channel.  V for a
// chunk of input channels is staged in shared memory; the accumulation over
// input channels is sequential with the reference's zero-skip and separate
// multiply/add, so F(2,3) reproduces the reference C bit for bit.
constexpr int kTileThreads = 128;
constexpr int kTileChunk = 64;

template <int M>
__global__ void __launch_bounds__(kTileThreads)
    tiles_fused(const float *__restrict__ tiles, const float *__restrict__ U,
                float *__restrict__ out, int C, int K) {
  constexpr int TD = M + 2, NF = TD * TD;
  __shared__ float vsh[kTileChunk * NF];
  const int tile = blockIdx.x;
  const int oc = blockIdx.y * kTileThreads + threadIdx.x;
  const float *in = tiles + (size_t)tile * C * NF;
  float acc[NF];
#pragma unroll
  for (int f = 0; f < NF; ++f) acc[f] = 0.f;
  for (int c0 = 0; c0 < C; c0 += kTileChunk) {
    const int cn = min(kTileChunk, C - c0);
    __syncthreads();
    for (int ic = threadIdx.x; ic < cn; ic += kTileThreads) {
      float d[TD][TD], v[TD][TD];
#pragma unroll
      for (int r = 0; r < TD; ++r)
#pragma unroll
        for (int s = 0; s < TD; ++s) d[r][s] = in[(size_t)(c0 + ic) * NF + r * TD + s];
      input_transform<M, true>(d, v);
#pragma unroll
      for (int a = 0; a < TD; ++a)
#pragma unroll
        for (int b = 0; b < TD; ++b) vsh[ic * NF + a * TD + b] = v[a][b];
    }
    __syncthreads();
    if (oc < K) {
      const float *u = U + ((size_t)oc * C + c0) * NF;
      for (int ic = 0; ic < cn; ++ic) {
#pragma unroll
        for (int f = 0; f < NF; ++f) {
          const float uf = u[(size_t)ic * NF + f];
          if (uf != 0.0f) acc[f] = __fadd_rn(acc[f], __fmul_rn(uf, vsh[ic * NF + f]));
        }
      }
    }
  }
  if (oc < K) {
    float mm[TD][TD], yy[M][M];
#pragma unroll
    for (int a = 0; a < TD; ++a)
#pragma unroll
      for (int b = 0; b < TD; ++b) mm[a][b] = acc[a * TD + b];
    output_transform<M, true>(mm, yy);
    float *o = out + ((size_t)tile * K + oc) * M * M;
#pragma unroll
    for (int i = 0; i < M; ++i)
#pragma unroll
      for (int j = 0; j < M; ++j) o[i * M + j] = yy[i][j];
  }
}

// ============================================================================
// Configuration table + launch shims
// ============================================================================
typedef void (*ffma_fn)(const void *, const void *, const float *, void *, int, int, int, int,
                        int, int, int, int);

struct FfmaEntry {
  cwgk_ffma_cfg cfg;
  const void *fn_f32;
  const void *fn_bf16;
};

#define CWG_FFMA_ENTRY(M_, TY_, TX_, KB_, CC_, FPW_)                                         \
  {{M_, TY_, TX_, KB_, CC_, FG<M_, TY_, TX_, KB_, CC_, FPW_>::NT,                            \
    FG<M_, TY_, TX_, KB_, CC_, FPW_>::SMEM},                                                 \
   (const void *)wino_fused_ffma<M_, TY_, TX_, KB_, CC_, FPW_, float>,                      \
   (const void *)wino_fused_ffma<M_, TY_, TX_, KB_, CC_, FPW_, __nv_bfloat16>}

static const FfmaEntry kFfma[] = {
    CWG_FFMA_ENTRY(2, 4, 4, 16, 8, 1), CWG_FFMA_ENTRY(2, 4, 4, 32, 8, 1),
    CWG_FFMA_ENTRY(2, 4, 4, 64, 8, 1), CWG_FFMA_ENTRY(2, 8, 8, 32, 8, 1),
    CWG_FFMA_ENTRY(4, 4, 4, 16, 8, 3), CWG_FFMA_ENTRY(4, 4, 4, 32, 8, 3),
    CWG_FFMA_ENTRY(4, 4, 4, 64, 8, 3),
    // F(6,3): a 32-channel block spills ~290 B per thread (64 accumulators beside
    // the 8x8 window rows); the 16-channel block fits in 128 registers but for a
    // few bytes.
    CWG_FFMA_ENTRY(6, 4, 4, 16, 8, 4),
};
constexpr int kNumFfma = sizeof(kFfma) / sizeof(kFfma[0]);

static int fail(cudaError_t e) {
  t_cuda_error = (int)e;
  return -3; /* CWG_ECUDA */
}

}  // namespace cwg

using namespace cwg;

extern "C" {

void cwgk_count_launch(void) { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long cwgk_launches(void) { return g_launches.load(std::memory_order_relaxed); }
void cwgk_set_cuda_error(int err) { t_cuda_error = err; }
int cwgk_get_cuda_error(void) { return t_cuda_error; }

int cwgk_ffma_num_cfgs(void) { return kNumFfma; }

int cwgk_ffma_get_cfg(int idx, cwgk_ffma_cfg *out) {
  if (idx < 0 || idx >= kNumFfma || !out) return -1;
  *out = kFfma[idx].cfg;
  return 0;
}

int cwgk_weight_transform(const float *src, void *U, int c_in, int c_out, int m, int layout,
                          int from_ref, void *stream) {
  if (layout != CWGK_LAYOUT_FFMA_F32) return cwgk_weight_transform_tc(src, U, c_in, c_out, m,
                                                                      layout, from_ref, stream);
  const long total = (long)c_in * c_out;
  const int threads = 256;
  const unsigned blocks = (unsigned)((total + threads - 1) / threads);
  cudaStream_t s = (cudaStream_t)stream;
  if (m == 2)
    wt_transform_ffma<2><<<blocks, threads, 0, s>>>(src, (float *)U, c_in, c_out, from_ref);
  else if (m == 4)
    wt_transform_ffma<4><<<blocks, threads, 0, s>>>(src, (float *)U, c_in, c_out, from_ref);
  else if (m == 6)
    wt_transform_ffma<6><<<blocks, threads, 0, s>>>(src, (float *)U, c_in, c_out, from_ref);
  else
    return -2;
  cwgk_count_launch();
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : fail(e);
}

int cwgk_conv_ffma(int cfg_idx, const void *x, const void *U, const float *bias, void *y, int n,
                   int c_in, int c_out, int h, int w, int bf16, int relu, int slices,
                   void *stream) {
  if (cfg_idx < 0 || cfg_idx >= kNumFfma) return -1;
  const FfmaEntry &e = kFfma[cfg_idx];
  const int m = e.cfg.m;
  const int tiles_y = (h + m - 1) / m, tiles_x = (w + m - 1) / m;
  const unsigned gx = (unsigned)(((tiles_y + e.cfg.ty - 1) / e.cfg.ty) *
                                 ((tiles_x + e.cfg.tx - 1) / e.cfg.tx));
  const unsigned gy = (unsigned)((c_out + e.cfg.kb - 1) / e.cfg.kb);
  if (n > 65535 || gy > 65535) return -2;
  // slices: fp32 only, at most one per step, none empty
  const int steps = (c_in + e.cfg.cc - 1) / e.cfg.cc;
  if (slices < 1 || bf16) slices = 1;
  if (slices > steps) slices = steps;
  const int per = (steps + slices - 1) / slices;
  slices = (steps + per - 1) / per;
  if ((long long)n * slices > 65535) return -2;
  const void *fn = bf16 ? e.fn_bf16 : e.fn_f32;
  static std::atomic<unsigned long long> attr_done[kNumFfma][2];
  cudaError_t err = smem_attr_once(attr_done[cfg_idx][bf16 ? 1 : 0], fn, e.cfg.smem);
  if (err != cudaSuccess) return fail(err);
  cudaStream_t s = (cudaStream_t)stream;
  // split: y zeroed and accumulated; with ReLU the bias joins in the second pass
  const float *kbias = (slices > 1 && relu) ? nullptr : bias;
  int krelu = slices > 1 ? 0 : relu;
  if (slices > 1 &&
      (err = cudaMemsetAsync(y, 0, (size_t)n * c_out * h * w * sizeof(float), s)) != cudaSuccess)
    return fail(err);
  void *args[] = {(void *)&x,     (void *)&U, (void *)&kbias,   (void *)&y,
                  (void *)&c_in,  (void *)&c_out, (void *)&h,   (void *)&w,
                  (void *)&tiles_y, (void *)&tiles_x, (void *)&krelu, (void *)&slices};
  err = cudaLaunchKernel(fn, dim3(gx, gy, (unsigned)(n * slices)),
                         dim3((unsigned)e.cfg.threads), args, (size_t)e.cfg.smem, s);
  cwgk_count_launch();
  if (err != cudaSuccess) return fail(err);
  if (slices > 1 && relu) return cwgk_bias_relu((float *)y, bias, n, c_out, h, w, 1, stream);
  return 0;
}

int cwgk_tiles(const float *tiles, const float *U, float *out, int n_tiles, int c_in, int c_out,
               int td, void *stream) {
  if (n_tiles == 0) return 0;
  if (n_tiles > 0x7fffffff || c_out <= 0) return -1;
  const dim3 grid((unsigned)n_tiles, (unsigned)((c_out + kTileThreads - 1) / kTileThreads));
  cudaStream_t s = (cudaStream_t)stream;
  switch (td) {
    case 4: tiles_fused<2><<<grid, kTileThreads, 0, s>>>(tiles, U, out, c_in, c_out); break;
    case 6: tiles_fused<4><<<grid, kTileThreads, 0, s>>>(tiles, U, out, c_in, c_out); break;
    case 8: tiles_fused<6><<<grid, kTileThreads, 0, s>>>(tiles, U, out, c_in, c_out); break;
    default: return -2;
  }
  cwgk_count_launch();
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : fail(e);
}

}  // extern "C"
