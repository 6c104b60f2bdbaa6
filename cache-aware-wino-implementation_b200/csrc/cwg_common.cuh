// cwg_common.cuh -- shared device helpers: Winograd tables, element I/O,
// launch bookkeeping.  Device code for sm_100a only.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "cwg_internal.h"

namespace cwg {

// ---- launch bookkeeping ---------------------------------------------------------
// The opt-in shared-memory size of a kernel, set once per (kernel, device): later
// launches skip the call, so per-layer host cost stays low and a stream capture
// into a CUDA graph sees launches only.  `done` holds one bit per device.
inline cudaError_t smem_attr_once(std::atomic<unsigned long long> &done, const void *fn,
                                  int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? 1ull << dev : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
  return e;
}
template <auto Kernel>
inline cudaError_t smem_attr_once(int bytes) {
  static std::atomic<unsigned long long> done{0};
  return smem_attr_once(done, (const void *)Kernel, bytes);
}

// ---- weight transform G g G^T ------------------------------------------------
// G for F(2,3), F(4,3) and F(6,3): the unique matrices that make the reference's Bt/At
// (src/fused_winograd_kernel.py:18-67) compute a 3x3 cross-correlation.
template <int M>
__device__ __forceinline__ double gmat(int a, int i);
template <>
__device__ __forceinline__ double gmat<2>(int a, int i) {
  const double g[4][3] = {{1, 0, 0}, {.5, .5, .5}, {.5, -.5, .5}, {0, 0, 1}};
  return g[a][i];
}
template <>
__device__ __forceinline__ double gmat<4>(int a, int i) {
  const double g[6][3] = {{1. / 4, 0, 0},          {-1. / 6, -1. / 6, -1. / 6},
                          {-1. / 6, 1. / 6, -1. / 6}, {1. / 24, 1. / 12, 1. / 6},
                          {1. / 24, -1. / 12, 1. / 6}, {0, 0, 1}};
  return g[a][i];
}

template <>
__device__ __forceinline__ double gmat<6>(int a, int i) {
  const double g[8][3] = {{1, 0, 0},
                          {-2. / 9, -2. / 9, -2. / 9},
                          {-2. / 9, 2. / 9, -2. / 9},
                          {1. / 90, 1. / 45, 2. / 45},
                          {1. / 90, -1. / 45, 2. / 45},
                          {1. / 45, 1. / 90, 1. / 180},
                          {1. / 45, -1. / 90, 1. / 180},
                          {0, 0, 1}};
  return g[a][i];
}

// u[f] for one (k, c) pair, in fp64 with the same operation order as the CPU
// oracle (no contraction), rounded once to fp32.
template <int M>
__device__ __forceinline__ void transform_one(const float *src, int from_ref, float *u) {
  constexpr int TD = M + 2, NF = TD * TD;
  if (from_ref) {
#pragma unroll
    for (int f = 0; f < NF; ++f) u[f] = src[f];
    return;
  }
  double gk[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) gk[i] = (double)src[i];
  double t[TD][3];
#pragma unroll
  for (int a = 0; a < TD; ++a)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      double s = 0.0;
#pragma unroll
      for (int i = 0; i < 3; ++i) s = __dadd_rn(s, __dmul_rn(gmat<M>(a, i), gk[i * 3 + j]));
      t[a][j] = s;
    }
#pragma unroll
  for (int a = 0; a < TD; ++a)
#pragma unroll
    for (int b = 0; b < TD; ++b) {
      double s = 0.0;
#pragma unroll
      for (int j = 0; j < 3; ++j) s = __dadd_rn(s, __dmul_rn(t[a][j], gmat<M>(b, j)));
      u[a * TD + b] = (float)s;
    }
}


// ---- element conversion -----------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// ---- Winograd tables ----------------------------------------------------------
// Bt (td x td) and At (m x td) are the reference's tables
// (src/fused_winograd_kernel.py:18-67).  They are spelled out as local
// constant arrays so that, once the loops are unrolled, every coefficient is a
// compile-time immediate and the zero terms vanish.
template <int M>
struct Wino;

template <>
struct Wino<2> {
  static constexpr int TD = 4;
  __device__ __forceinline__ static float bt(int a, int i) {
    const float t[4][4] = {{1, 0, -1, 0}, {0, 1, 1, 0}, {0, -1, 1, 0}, {0, 1, 0, -1}};
    return t[a][i];
  }
  __device__ __forceinline__ static float at(int a, int i) {
    const float t[2][4] = {{1, 1, 1, 0}, {0, 1, -1, -1}};
    return t[a][i];
  }
};

template <>
struct Wino<4> {
  static constexpr int TD = 6;
  __device__ __forceinline__ static float bt(int a, int i) {
    const float t[6][6] = {{4, 0, -5, 0, 1, 0},  {0, -4, -4, 1, 1, 0}, {0, 4, -4, -1, 1, 0},
                           {0, -2, -1, 2, 1, 0}, {0, 2, -1, -2, 1, 0}, {0, 4, 0, -5, 0, 1}};
    return t[a][i];
  }
  __device__ __forceinline__ static float at(int a, int i) {
    const float t[4][6] = {
        {1, 1, 1, 1, 1, 0}, {0, 1, -1, 2, -2, 0}, {0, 1, 1, 4, 4, 0}, {0, 1, -1, 8, -8, 1}};
    return t[a][i];
  }
};

template <>
struct Wino<6> {
  static constexpr int TD = 8;
  __device__ __forceinline__ static float bt(int a, int i) {
    const float t[8][8] = {{1, 0, -5.25f, 0, 5.25f, 0, -1, 0},
                           {0, 1, 1, -4.25f, -4.25f, 1, 1, 0},
                           {0, -1, 1, 4.25f, -4.25f, -1, 1, 0},
                           {0, 0.5f, 0.25f, -2.5f, -1.25f, 2, 1, 0},
                           {0, -0.5f, 0.25f, 2.5f, -1.25f, -2, 1, 0},
                           {0, 2, 4, -2.5f, -5, 0.5f, 1, 0},
                           {0, -2, 4, 2.5f, -5, -0.5f, 1, 0},
                           {0, -1, 0, 5.25f, 0, -5.25f, 0, 1}};
    return t[a][i];
  }
  __device__ __forceinline__ static float at(int a, int i) {
    const float t[6][8] = {{1, 1, 1, 1, 1, 32, 32, 0},   {0, 1, -1, 2, -2, 16, -16, 0},
                           {0, 1, 1, 4, 4, 8, 8, 0},     {0, 1, -1, 8, -8, 4, -4, 0},
                           {0, 1, 1, 16, 16, 2, 2, 0},   {0, 1, -1, 32, -32, 1, -1, 1}};
    return t[a][i];
  }
};

// s + c*d.  EXACT keeps the reference's separate multiply and add (two
// roundings, as the reference's C compiles on x86-64); otherwise one FMA.
template <bool EXACT>
__device__ __forceinline__ float madd(float c, float d, float s) {
  return EXACT ? __fadd_rn(s, __fmul_rn(c, d)) : fmaf(c, d, s);
}

// Sum of coefficient * value over the nonzero coefficients of one table row,
// in index order.  The sum starts from the first term itself (a +-1
// coefficient costs nothing), so only one add per further term remains.
template <bool EXACT>
__device__ __forceinline__ float first_term(float c, float d) {
  return c == 1.f ? d : (c == -1.f ? -d : (EXACT ? __fmul_rn(c, d) : c * d));
}

// v = Bt d B (td x td, row-major), sequential in the reference's index order.
template <int M, bool EXACT = false>
__device__ __forceinline__ void input_transform(const float (&d)[M + 2][M + 2],
                                                float (&v)[M + 2][M + 2]) {
  constexpr int TD = M + 2;
  float t[TD][TD];
#pragma unroll
  for (int a = 0; a < TD; ++a)
#pragma unroll
    for (int j = 0; j < TD; ++j) {
      float s = 0.f;
      bool first = true;
#pragma unroll
      for (int i = 0; i < TD; ++i) {
        const float c = Wino<M>::bt(a, i);
        if (c == 0.f) continue;
        s = first ? first_term<EXACT>(c, d[i][j]) : madd<EXACT>(c, d[i][j], s);
        first = false;
      }
      t[a][j] = s;
    }
#pragma unroll
  for (int a = 0; a < TD; ++a)
#pragma unroll
    for (int b = 0; b < TD; ++b) {
      float s = 0.f;
      bool first = true;
#pragma unroll
      for (int j = 0; j < TD; ++j) {
        const float c = Wino<M>::bt(b, j);
        if (c == 0.f) continue;
        s = first ? first_term<EXACT>(c, t[a][j]) : madd<EXACT>(c, t[a][j], s);
        first = false;
      }
      v[a][b] = s;
    }
}

// y = At m A (m x m) from the td x td accumulator tile.
template <int M, bool EXACT = false>
__device__ __forceinline__ void output_transform(const float (&mm)[M + 2][M + 2],
                                                 float (&y)[M][M]) {
  constexpr int TD = M + 2;
  float t[M][TD];
#pragma unroll
  for (int i = 0; i < M; ++i)
#pragma unroll
    for (int b = 0; b < TD; ++b) {
      float s = 0.f;
      bool first = true;
#pragma unroll
      for (int a = 0; a < TD; ++a) {
        const float c = Wino<M>::at(i, a);
        if (c == 0.f) continue;
        s = first ? first_term<EXACT>(c, mm[a][b]) : madd<EXACT>(c, mm[a][b], s);
        first = false;
      }
      t[i][b] = s;
    }
#pragma unroll
  for (int i = 0; i < M; ++i)
#pragma unroll
    for (int j = 0; j < M; ++j) {
      float s = 0.f;
      bool first = true;
#pragma unroll
      for (int b = 0; b < TD; ++b) {
        const float c = Wino<M>::at(j, b);
        if (c == 0.f) continue;
        s = first ? first_term<EXACT>(c, t[i][b]) : madd<EXACT>(c, t[i][b], s);
        first = false;
      }
      y[i][j] = s;
    }
}

}  // namespace cwg
