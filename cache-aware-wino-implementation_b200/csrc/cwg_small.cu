// cwg_small.cu -- F(2x2,3x3) for layers with at most 4 input channels (a network's
// RGB input layer).
//
// With C_in <= 4 a layer is bound by writing its C_out output planes, and the
// general CUDA-core kernel (shared-memory stages of 8 input channels, one warp per
// frequency) spends its time on per-CTA latency instead: each CTA stages a weight
// chunk for a few dozen tiles.  Here one thread owns one 2x2 output tile: it loads
// its 4x4 window of every input channel once, keeps V = Bt d B (16 x C values) in
// registers, and then walks the CTA's 64 output channels: M_f = sum_c U[f][c][k] V[f][c]
// (the weights of channel k are a broadcast read from shared memory), Y = At M A,
// bias, ReLU, two 2-pixel row stores.  Consecutive threads own consecutive tiles of
// an image row, so a warp's stores of one channel cover 64 contiguous pixels.  A
// small batch gets fewer channels per CTA (down to 8) so that the grid still fills
// the SMs.
//
// Weights: the CUDA-core layout, fp32 [16 f][C_in][C_out] (csrc/cwg_ffma.cu), the
// same buffer the general kernel reads.  Per-tile math as in the reference
// (fused_winograd.c:19-119): V = Bt d B, M = sum over input channels of U (.) V,
// Y = At M A.
#include <cstdint>

#include "../../include/cwg.h"
#include "cwg_common.cuh"
#include "cwg_internal.h"

namespace cwg {
namespace small {

constexpr int kThreads = 256;  // tiles per CTA
constexpr int kKb = 64;        // output channels per CTA, at most

template <int C, typename Tio>
__global__ void __launch_bounds__(kThreads)
    wino_small_cin(const Tio *__restrict__ x, const float *__restrict__ U,
                   const float *__restrict__ bias, Tio *__restrict__ y, int K, int H, int W,
                   int tiles_y, int tiles_x, long long total_tiles, int relu, int pairs,
                   int kc) {
  constexpr int NF = 16;
  __shared__ __align__(16) float su[kKb][NF * C];  // [k][f * C + c]
  const int k0 = blockIdx.y * kc;                  // kc <= kKb channels per CTA
  const int kn = K - k0 < kc ? K - k0 : kc;
  for (int i = threadIdx.x; i < kKb * NF * C; i += kThreads) {
    const int k = i % kKb, fc = i / kKb;  // consecutive threads: consecutive k
    su[k][fc] = k < kn ? U[(size_t)fc * K + k0 + k] : 0.f;
  }
  __syncthreads();
  const long long T = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (T >= total_tiles) return;
  const long long per_img = (long long)tiles_y * tiles_x;
  const int n = (int)(T / per_img);
  const int rem = (int)(T - (long long)n * per_img);
  const int ty = rem / tiles_x, tx = rem - ty * tiles_x;
  const int y0 = 2 * ty - 1, x0 = 2 * tx - 1;
  const size_t plane = (size_t)H * W;

  // V[f][c] of this tile, every input channel
  float v[NF][C];
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const Tio *xc = x + ((size_t)n * C + c) * plane;
    float d[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int yy = y0 + i;
      const bool rok = yy >= 0 && yy < H;
      if (pairs) {
        // columns x0 - 1 .. x0 + 4 as three aligned pairs (even width)
        const Tio *row = xc + (size_t)(rok ? yy : 0) * W + (x0 - 1);
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          const int c0 = x0 - 1 + 2 * p;
          const bool ok = rok && c0 >= 0 && c0 + 1 < W;
          float a0 = 0.f, a1 = 0.f;
          if (ok) {
            if constexpr (sizeof(Tio) == 4) {
              const float2 q = *reinterpret_cast<const float2 *>(row + 2 * p);
              a0 = q.x;
              a1 = q.y;
            } else {
              const uint32_t q = *reinterpret_cast<const uint32_t *>(row + 2 * p);
              a0 = __uint_as_float(q << 16);
              a1 = __uint_as_float(q & 0xFFFF0000u);
            }
          }
          if (p > 0) d[i][2 * p - 1] = a0;
          if (p < 2) d[i][2 * p] = a1;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int xx = x0 + j;
          d[i][j] = (rok && xx >= 0 && xx < W) ? to_f32(xc[(size_t)yy * W + xx]) : 0.f;
        }
      }
    }
    float vt[4][4];
    input_transform<2>(d, vt);
#pragma unroll
    for (int f = 0; f < NF; ++f) v[f][c] = vt[f / 4][f % 4];
  }

  const int oy = 2 * ty, ox = 2 * tx;
  const bool row1 = oy + 1 < H, col1 = ox + 1 < W;
  const bool vec = pairs && col1;  // both pixels of a row, 8-byte (4-byte) aligned
  Tio *yt = y + ((size_t)n * K + k0) * plane + (size_t)oy * W + ox;
#pragma unroll 2
  for (int k = 0; k < kn; ++k) {
    float m[4][4];
    const float *uk = &su[k][0];
#pragma unroll
    for (int f = 0; f < NF; ++f) {
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) s = fmaf(uk[f * C + c], v[f][c], s);
      m[f / 4][f % 4] = s;
    }
    float o[2][2];
    output_transform<2>(m, o);
    const float b = bias ? bias[k0 + k] : 0.f;
    Tio *yk = yt + (size_t)k * plane;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (i == 1 && !row1) break;
      float a0 = o[i][0] + b, a1 = o[i][1] + b;
      if (relu) {
        a0 = a0 < 0.f ? 0.f : a0;
        a1 = a1 < 0.f ? 0.f : a1;
      }
      Tio *dst = yk + (size_t)i * W;
      if (vec) {
        if constexpr (sizeof(Tio) == 4) {
          *reinterpret_cast<float2 *>(dst) = make_float2(a0, a1);
        } else {
          __nv_bfloat162 h;
          h.x = __float2bfloat16_rn(a0);
          h.y = __float2bfloat16_rn(a1);
          *reinterpret_cast<__nv_bfloat162 *>(dst) = h;
        }
      } else {
        dst[0] = from_f32<Tio>(a0);
        if (col1) dst[1] = from_f32<Tio>(a1);
      }
    }
  }
}

}  // namespace small
}  // namespace cwg

using namespace cwg;

extern "C" int cwgk_conv_small(const void *x, const void *U, const float *bias, void *y, int n,
                               int c_in, int c_out, int h, int w, int bf16, int relu,
                               void *stream) {
  if (c_in < 1 || c_in > 4) return -2;
  const int tiles_y = (h + 1) / 2, tiles_x = (w + 1) / 2;
  const long long total = (long long)n * tiles_y * tiles_x;
  const long long gx = (total + small::kThreads - 1) / small::kThreads;
  // channels per CTA: 64, halved (down to 8) while the grid would leave SMs idle
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    (void)cudaGetLastError();
    sms = 148;
  }
  int kc = small::kKb;
  while (kc > 8 && gx * ((c_out + kc - 1) / kc) < 2LL * sms) kc /= 2;
  const int gy = (c_out + kc - 1) / kc;
  if (gx > 0x7fffffffLL || gy > 65535) return -2;
  // pair loads and row stores need an even row length and x, y aligned to two elements
  const size_t esz = bf16 ? 2 : 4;
  const int pairs = (w % 2 == 0) && ((uintptr_t)x % (2 * esz) == 0) &&
                    ((uintptr_t)y % (2 * esz) == 0);
  const dim3 grid((unsigned)gx, (unsigned)gy);
  cudaStream_t s = (cudaStream_t)stream;
#define CWG_SMALL(C_)                                                                          \
  (bf16 ? (small::wino_small_cin<C_, __nv_bfloat16><<<grid, small::kThreads, 0, s>>>(          \
               (const __nv_bfloat16 *)x, (const float *)U, bias, (__nv_bfloat16 *)y, c_out, h, \
               w, tiles_y, tiles_x, total, relu, pairs, kc),                                   \
           0)                                                                                  \
        : (small::wino_small_cin<C_, float><<<grid, small::kThreads, 0, s>>>(                  \
               (const float *)x, (const float *)U, bias, (float *)y, c_out, h, w, tiles_y,     \
               tiles_x, total, relu, pairs, kc),                                               \
           0))
  switch (c_in) {
    case 1: CWG_SMALL(1); break;
    case 2: CWG_SMALL(2); break;
    case 3: CWG_SMALL(3); break;
    default: CWG_SMALL(4); break;
  }
#undef CWG_SMALL
  cwgk_count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return -3;
  }
  return 0;
}
