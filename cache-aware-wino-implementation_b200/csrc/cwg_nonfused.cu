// cwg_nonfused.cu -- the non-fused ablation: the same Winograd convolution as three
// passes over HBM, for measuring what the fused kernels save.
//
// The reference's run_non_fused (src/fused_winograd_kernel.py:116-151) computes the
// same per-tile math as run_fused; its "non-fused" difference is only logged metadata.
// Here the three stages really are separate kernels with HBM round trips between them:
//   1. input transform  x -> V[td^2][C][T]          (fp32, one thread per (c, tile))
//   2. per-frequency GEMM M_f = U_f^T V_f -> M[td^2][K][T]  (cuBLAS SGEMM, strided batch)
//   3. output transform M -> y, bias, ReLU           (one thread per (k, tile))
// T = n * ceil(h/m) * ceil(w/m).  fp32 only; U in the FFMA layout [td^2][C][K].
#include <cublas_v2.h>

#include <mutex>

#include "../../include/cwg.h"
#include "cwg_common.cuh"

namespace cwg {
namespace nonfused {

// V[f][c][t] for one (c, tile): the 4x4 (6x6) window with zero padding.
template <int M>
__global__ void input_pass(const float *__restrict__ x, float *__restrict__ V, int C, int H,
                           int W, int tiles_y, int tiles_x, long long T) {
  constexpr int TD = M + 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)C * T) return;
  const int c = (int)(idx / T);
  const long long t = idx - (long long)c * T;
  const long long per_img = (long long)tiles_y * tiles_x;
  const int n = (int)(t / per_img);
  const int rem = (int)(t - (long long)n * per_img);
  const int ty = rem / tiles_x, tx = rem - ty * tiles_x;
  const int y0 = M * ty - 1, x0 = M * tx - 1;
  const float *xc = x + ((size_t)n * C + c) * H * W;
  float d[TD][TD], v[TD][TD];
#pragma unroll
  for (int i = 0; i < TD; ++i)
#pragma unroll
    for (int j = 0; j < TD; ++j) {
      const int yy = y0 + i, xx = x0 + j;
      d[i][j] = (yy >= 0 && yy < H && xx >= 0 && xx < W) ? xc[(size_t)yy * W + xx] : 0.f;
    }
  input_transform<M, true>(d, v);
#pragma unroll
  for (int f = 0; f < TD * TD; ++f) V[((size_t)f * C + c) * T + t] = v[f / TD][f % TD];
}

// y for one (k, tile): At M A, bias, ReLU, clipped to the image.
template <int M>
__global__ void output_pass(const float *__restrict__ Mf, const float *__restrict__ bias,
                            float *__restrict__ y, int K, int H, int W, int tiles_y,
                            int tiles_x, long long T, int relu) {
  constexpr int TD = M + 2;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)K * T) return;
  const int k = (int)(idx / T);
  const long long t = idx - (long long)k * T;
  const long long per_img = (long long)tiles_y * tiles_x;
  const int n = (int)(t / per_img);
  const int rem = (int)(t - (long long)n * per_img);
  const int ty = rem / tiles_x, tx = rem - ty * tiles_x;
  float mm[TD][TD], o[M][M];
#pragma unroll
  for (int f = 0; f < TD * TD; ++f) mm[f / TD][f % TD] = Mf[((size_t)f * K + k) * T + t];
  output_transform<M, true>(mm, o);
  const float b = bias ? bias[k] : 0.f;
  float *yk = y + ((size_t)n * K + k) * H * W;
#pragma unroll
  for (int i = 0; i < M; ++i)
#pragma unroll
    for (int j = 0; j < M; ++j) {
      const int yy = M * ty + i, xx = M * tx + j;
      if (yy < H && xx < W) {
        float val = o[i][j] + b;
        if (relu) val = val < 0.f ? 0.f : val;
        yk[(size_t)yy * W + xx] = val;
      }
    }
}

// One cuBLAS handle per device, created on first use (plain FP32 math: no TF32).
constexpr int kMaxDevices = 64;
cublasHandle_t g_handle[kMaxDevices];
std::mutex g_mu;

cublasHandle_t handle_for(int dev) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_handle[dev]) {
    cublasHandle_t h = nullptr;
    if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) return nullptr;
    if (cublasSetMathMode(h, CUBLAS_PEDANTIC_MATH) != CUBLAS_STATUS_SUCCESS) {
      cublasDestroy(h);
      return nullptr;
    }
    g_handle[dev] = h;
  }
  return g_handle[dev];
}

}  // namespace nonfused
}  // namespace cwg

using namespace cwg;

static size_t al256(size_t b) { return (b + 255) / 256 * 256; }

extern "C" size_t cwg_nonfused_workspace_bytes(int n, int c_in, int c_out, int h, int w, int m) {
  if (n <= 0 || c_in <= 0 || c_out <= 0 || h <= 0 || w <= 0 || (m != 2 && m != 4 && m != 6))
    return 0;
  const size_t T = (size_t)n * ((h + m - 1) / m) * ((w + m - 1) / m);
  const size_t nf = (size_t)(m + 2) * (m + 2);
  return al256(nf * c_in * T * 4) + al256(nf * c_out * T * 4);
}

extern "C" int cwg_conv3x3_nonfused(const float *x, const float *U, const float *bias, float *y,
                                    void *workspace, size_t workspace_bytes, int n, int c_in,
                                    int c_out, int h, int w, int m, unsigned flags,
                                    void *stream) {
  if (flags & ~(unsigned)CWG_RELU) return CWG_EINVAL;  // fp32 only, no path switches
  const size_t need = cwg_nonfused_workspace_bytes(n, c_in, c_out, h, w, m);
  if (need == 0) return CWG_EINVAL;
  if (!x || !U || !y || !workspace || workspace_bytes < need) return CWG_EINVAL;
  if (((uintptr_t)x & 3) || ((uintptr_t)y & 3) || ((uintptr_t)U & 3) || ((uintptr_t)bias & 3) ||
      ((uintptr_t)workspace & 255))
    return CWG_EINVAL;
  const int tiles_y = (h + m - 1) / m, tiles_x = (w + m - 1) / m;
  const long long T = (long long)n * tiles_y * tiles_x;
  const int nf = (m + 2) * (m + 2);
  if (T > 0x7fffffffLL) return CWG_EUNSUPPORTED;
  float *V = static_cast<float *>(workspace);
  float *Mf = reinterpret_cast<float *>(static_cast<char *>(workspace) +
                                        al256((size_t)nf * c_in * T * 4));
  cudaStream_t s = (cudaStream_t)stream;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= nonfused::kMaxDevices) {
    cwgk_set_cuda_error((int)e);
    return CWG_ECUDA;
  }
  cublasHandle_t hb = nonfused::handle_for(dev);
  if (!hb) return CWG_ECUDA;
  const int threads = 256;
  const unsigned bx = (unsigned)(((long long)c_in * T + threads - 1) / threads);
  if (m == 2)
    nonfused::input_pass<2><<<bx, threads, 0, s>>>(x, V, c_in, h, w, tiles_y, tiles_x, T);
  else if (m == 4)
    nonfused::input_pass<4><<<bx, threads, 0, s>>>(x, V, c_in, h, w, tiles_y, tiles_x, T);
  else
    nonfused::input_pass<6><<<bx, threads, 0, s>>>(x, V, c_in, h, w, tiles_y, tiles_x, T);
  cwgk_count_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return CWG_ECUDA;
  }
  // Row-major V_f [C][T], U_f [C][K], M_f [K][T]; in cuBLAS's column-major view
  // M_f (T x K) = V_f (T x C) * U_f^T, with U_f stored as K x C (ld K).
  const float one = 1.f, zero = 0.f;
  if (cublasSetStream(hb, s) != CUBLAS_STATUS_SUCCESS ||
      cublasSgemmStridedBatched(hb, CUBLAS_OP_N, CUBLAS_OP_T, (int)T, c_out, c_in, &one, V,
                                (int)T, (long long)c_in * T, U, c_out, (long long)c_in * c_out,
                                &zero, Mf, (int)T, (long long)c_out * T,
                                nf) != CUBLAS_STATUS_SUCCESS)
    return CWG_ECUDA;
  const unsigned by = (unsigned)(((long long)c_out * T + threads - 1) / threads);
  const int relu = (flags & CWG_RELU) ? 1 : 0;
  if (m == 2)
    nonfused::output_pass<2>
        <<<by, threads, 0, s>>>(Mf, bias, y, c_out, h, w, tiles_y, tiles_x, T, relu);
  else if (m == 4)
    nonfused::output_pass<4>
        <<<by, threads, 0, s>>>(Mf, bias, y, c_out, h, w, tiles_y, tiles_x, T, relu);
  else
    nonfused::output_pass<6>
        <<<by, threads, 0, s>>>(Mf, bias, y, c_out, h, w, tiles_y, tiles_x, T, relu);
  cwgk_count_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return CWG_ECUDA;
  }
  return CWG_OK;
}
