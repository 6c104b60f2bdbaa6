// cwg_nonfused.cu -- the non-fused ablation: the same Winograd convolution as three
// passes over HBM, for measuring what the fused kernels save.
//
// The reference's run_non_fused (src/fused_winograd_kernel.py:116-151) computes the
// same per-tile math as run_fused; its "non-fused" difference is only logged metadata.
// Here the three stages really are separate kernels with HBM round trips between them:
//   1. input transform  x -> V (one thread per (channel, tile))
//   2. per-frequency GEMM M_f = U_f V_f -> M[td^2][K][T]  (fp32 results)
//   3. output transform M -> y, bias, ReLU           (one thread per (k, tile))
// T = n * ceil(h/m) * ceil(w/m).  The GEMM runs the same arithmetic as the fused
// kernel of the same layer, so that the two differ only in fusion:
//   F(2,3): tcgen05 MMAs with the bf16 hi/lo split (three products), as the fused
//           pair kernel; V goes to HBM as UMMA blocks (hi and lo bf16, 4 bytes per
//           element like fp32) and U is re-laid into such blocks by a small pass;
//   F(4,3), F(6,3): fp32 FFMA (the fused path of fp32 layers of these sizes is the
//           CUDA-core kernel), V fp32 [td^2][C][T].
// fp32 only; U in the CUDA-core layout [td^2][C][K].
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

// M_f[k][t] = sum_c U_f[c][k] V_f[c][t], fp32 FFMA: a CTA computes 64 channels x
// 128 tiles of one frequency through shared-memory tiles of 16 input channels; a
// thread accumulates 4 channels x 8 tiles in registers.
constexpr int kGk = 64, kGt = 128, kGc = 16;
__global__ void __launch_bounds__(256)
    gemm_freq_ffma(const float *__restrict__ U, const float *__restrict__ V, float *__restrict__ Mf,
                   int C, int K, int T) {
  __shared__ float As[kGc][kGk];
  __shared__ float Bs[kGc][kGt];
  const int f = blockIdx.z;
  const int k0 = blockIdx.y * kGk, t0 = blockIdx.x * kGt;
  const float *Uf = U + (size_t)f * C * K;
  const float *Vf = V + (size_t)f * C * T;
  const int tid = threadIdx.x;
  const int tk = (tid / 16) * 4, tt = (tid % 16) * 8;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int c0 = 0; c0 < C; c0 += kGc) {
#pragma unroll
    for (int r = 0; r < kGc * kGk / 256; ++r) {
      const int e = tid + r * 256, c = e / kGk, k = e % kGk;
      As[c][k] = (c0 + c < C && k0 + k < K) ? Uf[(size_t)(c0 + c) * K + k0 + k] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < kGc * kGt / 256; ++r) {
      const int e = tid + r * 256, c = e / kGt, t = e % kGt;
      Bs[c][t] = (c0 + c < C && t0 + t < T) ? Vf[(size_t)(c0 + c) * T + t0 + t] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kGc; ++c) {
      float a[4], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[c][tk + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[c][tt + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = k0 + tk + i;
    if (k >= K) continue;
    float *row = Mf + ((size_t)f * K + k) * T;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (t0 + tt + j < T) row[t0 + tt + j] = acc[i][j];
  }
}

}  // namespace nonfused
}  // namespace cwg

using namespace cwg;

static size_t al256(size_t b) { return (b + 255) / 256 * 256; }

// Workspace: [U blocks (F(2,3))][V][M], each 256-byte aligned.
static void nonfused_parts(int n, int c_in, int c_out, int h, int w, int m, size_t *ub,
                           size_t *vb, size_t *mb) {
  const size_t T = (size_t)n * ((h + m - 1) / m) * ((w + m - 1) / m);
  const int nf = (m + 2) * (m + 2);
  if (m == 2) {
    *ub = al256(cwgk_gemm_blocks_bytes(nf, c_out, c_in));
    *vb = al256(cwgk_gemm_blocks_bytes(nf, (int)T, c_in));
  } else {
    *ub = 0;
    *vb = al256((size_t)nf * c_in * T * 4);
  }
  *mb = al256((size_t)nf * c_out * T * 4);
}

extern "C" size_t cwg_nonfused_workspace_bytes(int n, int c_in, int c_out, int h, int w, int m) {
  if (n <= 0 || c_in <= 0 || c_out <= 0 || h <= 0 || w <= 0 || (m != 2 && m != 4 && m != 6))
    return 0;
  const size_t T = (size_t)n * ((h + m - 1) / m) * ((w + m - 1) / m);
  if (T > 0x7fffff00u) return 0;
  size_t ub, vb, mb;
  nonfused_parts(n, c_in, c_out, h, w, m, &ub, &vb, &mb);
  return ub + vb + mb;
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
  size_t ub, vb, mb;
  nonfused_parts(n, c_in, c_out, h, w, m, &ub, &vb, &mb);
  char *ws = static_cast<char *>(workspace);
  void *Ug = ws;
  void *V = ws + ub;
  float *Mf = reinterpret_cast<float *>(ws + ub + vb);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  const int threads = 256;
  if (m == 2) {
    int rc = cwgk_gemm_prepare(U, Ug, x, V, m, n, c_in, c_out, h, w, stream);
    if (rc == 0) rc = cwgk_gemm_x3(Ug, V, Mf, nf, c_in, c_out, (int)T, stream);
    if (rc != 0) return rc == -2 ? CWG_EUNSUPPORTED : CWG_ECUDA;
  } else {
    float *Vf = static_cast<float *>(V);
    const unsigned bx = (unsigned)(((long long)c_in * T + threads - 1) / threads);
    if (m == 4)
      nonfused::input_pass<4><<<bx, threads, 0, s>>>(x, Vf, c_in, h, w, tiles_y, tiles_x, T);
    else
      nonfused::input_pass<6><<<bx, threads, 0, s>>>(x, Vf, c_in, h, w, tiles_y, tiles_x, T);
    cwgk_count_launch();
    const long long gt = (T + nonfused::kGt - 1) / nonfused::kGt;
    const int gk = (c_out + nonfused::kGk - 1) / nonfused::kGk;
    if (gt > 0x7fffffffLL || gk > 65535) return CWG_EUNSUPPORTED;
    nonfused::gemm_freq_ffma<<<dim3((unsigned)gt, (unsigned)gk, (unsigned)nf), 256, 0, s>>>(
        U, Vf, Mf, c_in, c_out, (int)T);
    cwgk_count_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) {
      cwgk_set_cuda_error((int)e);
      return CWG_ECUDA;
    }
  }
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
