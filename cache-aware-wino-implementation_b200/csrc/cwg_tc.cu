// cwg_tc.cu -- the tcgen05/TMEM fused Winograd F(2x2,3x3) kernels (sm_100a).
//
// wino_fused_tc_pair (default; defined after the single-CTA kernel): a 2-SM CTA
// pair computes items of up to 128 output tiles x 128 output channels (F(2,3)) with
// tcgen05.mma.cta_group::2; a layer larger than one wave runs one persistent pair
// per co-resident cluster, which writes its next item's first stage while the
// current item's epilogue drains TMEM; see the comments above it.
//
// wino_fused_tc (ablations CWG_TC_NOPAIR / CWG_TC_FULL16): one CTA computes 128
// output channels x 64 (half-folded) or 32 (16 accumulators) output tiles:
//   * A = U_f   (128 output channels x 16 input channels, bf16, K-major), one
//                per Winograd frequency f, streamed from global memory by
//                cp.async.bulk (the weight transform already wrote each
//                (channel block, 16-channel step, frequency) as the exact
//                shared-memory image the tensor core reads);
//   * B = V_f   (tiles x 16 input channels, bf16, K-major), written into shared
//                memory by the transform warps, which load the 4x4 input patches
//                from global memory and compute Bt d B in registers;
//   * D in TMEM: 8 half-folded or 16 frequency accumulators fill all 512
//                columns, so the whole C_in reduction completes on chip;
//   * epilogue: the same warps read D (lane = output channel) with tcgen05.ld,
//                finish At M A, add bias, apply ReLU and store NCHW.
// fp32 parity ("x3"): every fp32 operand v is split into hi = bf16(v) and
// lo = bf16(v - hi); each product runs as three MMAs (hi*hi + hi*lo + lo*hi)
// into the same fp32 accumulator.  "x1" (bf16 layers) runs one MMA.
//
// Warp roles: warp 0 allocates TMEM and issues the MMAs from one elected lane;
// warp 1 issues the bulk copies of U; the other warps transform and run the
// epilogue.  Every mbarrier wait is bounded by %globaltimer: on timeout the
// kernel sets g_tc_status, drains what it has in flight, frees TMEM and
// returns, and the host reports CWG_ETIMEOUT.
#include <cstdint>

#include <cuda_fp16.h>

#include "../../include/cwg.h"
#include "cwg_common.cuh"

namespace cwg {
namespace tc {

constexpr int kCout = 128;     // MMA M
constexpr int kCc = 16;        // input channels per pipeline stage (one MMA K step)
constexpr int kNF = 16;        // frequencies of F(2,3)
constexpr int kFPerU = 2;      // frequencies per U stage
constexpr int kNV = 2;         // V stages
constexpr int kTmemCols = 512;
constexpr int kCoreBytes = 4096;               // one 128x16 bf16 operand block
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

// Two accumulation schemes share the kernel:
//   HALF  ("half-folded", the default): the row pass of the output transform,
//         Z[i][b] = sum_a At[i][a] M[a][b], runs inside the GEMM (the MMA's
//         negate-A bit supplies At's -1 entries), so 8 accumulators of 64 tiles
//         fill TMEM.  1.5x the MACs of plain Winograd, but every U byte serves 64
//         tiles instead of 32 and N=64 MMAs run ~1.7x closer to peak than N=32.
//   full: the 16 frequency accumulators M[a][b] of 32 tiles (plain Winograd).
template <bool HALF>
struct Geo {
  static constexpr int kTiles = HALF ? 64 : 32;         // MMA N
  static constexpr int kAcc = HALF ? 8 : 16;            // TMEM accumulators
  static constexpr int kXWarps = HALF ? 16 : 4;         // transform + epilogue warps
  static constexpr int kCpt = kTiles * 16 / (32 * kXWarps);  // channels per transform thread
  static constexpr int kThreads = (2 + kXWarps) * 32;
  static constexpr int kMinBlocks = HALF ? 1 : 2;       // CTAs per SM
  static constexpr int kNU = HALF ? 5 : 3;              // U stages
  static constexpr int kVBytes = kTiles * kCc * 2;      // one N x 16 bf16 operand block
  static_assert(kAcc * kTiles == kTmemCols, "accumulators fill TMEM");
};

// At of F(2,3) (src/fused_winograd_kernel.py:25-28), for the half-folded GEMM.
__host__ __device__ constexpr int at23(int i, int a) {
  return i == 0 ? (a == 3 ? 0 : 1) : (a == 0 ? 0 : (a == 1 ? 1 : -1));
}

template <bool X3, bool HALF>
struct Layout {
  using G = Geo<HALF>;
  static constexpr int kNU = G::kNU;
  static constexpr int kParts = X3 ? 2 : 1;                       // hi (+ lo)
  static constexpr int kVStage = kParts * kNF * G::kVBytes;       // up to 64 KiB
  static constexpr int kUStage = kFPerU * kParts * kCoreBytes;    // 8 or 16 KiB
  static constexpr int kVOff = 0;
  static constexpr int kUOff = kVOff + kNV * kVStage;
  static constexpr int kBarOff = kUOff + kNU * kUStage;
  // barriers: v_full[kNV], v_empty[kNV], u_full[kNU], u_empty[kNU], acc_full, drain
  static constexpr int kNumBars = 2 * kNV + 2 * kNU + 2;
  static constexpr int kTmemSlot = kBarOff + 8 * kNumBars;
  static constexpr int kAbortSlot = kTmemSlot + 4;
  static constexpr int kSmem = kAbortSlot + 4;
};

__device__ unsigned int g_tc_status;

// ---- PTX wrappers -------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase completed; false on timeout or when another
// role already aborted (the abort flag lives in shared memory).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      *abort = 1;
      atomicOr(&g_tc_status, 1u);
      return false;
    }
  }
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                   "r"(bar)
               : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 x bf16 -> fp32.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r0, r1, r2, r3;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(taddr)
               : "memory");
  v[0] = __uint_as_float(r0);
  v[1] = __uint_as_float(r1);
  v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3);
}
// One lane of a converged warp (elect.sync).  Issuing tcgen05 instructions this
// way, from warp-uniform control flow, keeps their operands in uniform
// registers: a per-lane branch around them costs ~3x in MMA issue rate.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred px;\n\telect.sync _|px, %1;\n\t@px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xFFFFFFFFu));
  return pred != 0;
}

// Named barrier 1: TMEM address handoff from warp 0 to the epilogue warps.
constexpr int kBarTmem = 1;
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, no swizzle.  Core matrices are
// 8 rows x 16 bytes; `lbo` = byte distance between the two K-adjacent core
// matrices of one MMA step, `sbo` = byte distance between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;                // base offset 0, legacy LBO mode, SWIZZLE_NONE
}

// Instruction descriptor: kind::f16, A = B = bf16 (or both fp16), D = fp32, both
// K-major.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool f16 = false) {
  return (1u << 4)                         // D format fp32
         | ((f16 ? 0u : 1u) << 7)          // A format: bf16 (1) or fp16 (0)
         | ((f16 ? 0u : 1u) << 10)         // B format: the same as A
         | ((uint32_t)(n >> 3) << 17)      // N / 8
         | ((uint32_t)(m >> 4) << 24);     // M / 16
}

// Byte offset of element (row, k) inside one K-major no-swizzle operand block
// of 16 K-elements: 8-row groups 256 B apart, K halves 128 B apart.
__host__ __device__ constexpr uint32_t blk_off(int row, int k) {
  return (uint32_t)((row >> 3) * 256 + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2);
}

// Two fp32 values -> packed bf16x2 (first value in the low half), one cvt.
__device__ __forceinline__ uint32_t pack_bf16(float first, float second) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(first, second);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// hi = bf16(v), lo = bf16(v - hi) for a pair of values; each result packs the
// pair (first value in the low half).  Two paired conversions and the unpacking
// of hi: fewer instructions than rounding hi with integer arithmetic, which the
// transform warps measured slower (173.4 vs 169.9 us on 64 images of 128->128 at
// 56x56, 281 vs 273.5 us on 256 images of 64->64).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &hi, uint32_t &lo) {
  hi = pack_bf16(a, b);
  lo = pack_bf16(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xFFFF0000u));
}

// ---- weight transform into UMMA blocks ------------------------------------------
// U layout: [K_pad/128][C_pad/16][16 f][parts][4096 B block], block element
// (k % 128, c % 16) at blk_off.  Channels past C_out / C_in are zero.
template <bool X3>
__global__ void wt_transform_tc(const float *__restrict__ src, uint8_t *__restrict__ U, int C,
                                int K, int Cp, int Kp, int from_ref) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)Cp * Kp) return;
  const int c = (int)(idx % Cp), k = (int)(idx / Cp);
  float u[kNF];
  if (k < K && c < C) {
    if (from_ref) {
#pragma unroll
      for (int f = 0; f < kNF; ++f) u[f] = src[((long)k * C + c) * kNF + f];
    } else {
      // fp64 G g G^T, same operation order as the CPU oracle, rounded once
      const double G[4][3] = {{1, 0, 0}, {.5, .5, .5}, {.5, -.5, .5}, {0, 0, 1}};
      const float *g = src + ((long)k * C + c) * 9;
      double t[4][3];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          double s = 0.0;
#pragma unroll
          for (int i = 0; i < 3; ++i) s = __dadd_rn(s, __dmul_rn(G[a][i], (double)g[i * 3 + j]));
          t[a][j] = s;
        }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          double s = 0.0;
#pragma unroll
          for (int j = 0; j < 3; ++j) s = __dadd_rn(s, __dmul_rn(t[a][j], G[b][j]));
          u[a * 4 + b] = (float)s;
        }
    }
  } else {
#pragma unroll
    for (int f = 0; f < kNF; ++f) u[f] = 0.f;
  }
  constexpr int parts = X3 ? 2 : 1;
  const int C16 = Cp / kCc;
  const long blk0 = (long)(k / kCout) * C16 + c / kCc;
  const uint32_t off = blk_off(k % kCout, c % kCc);
#pragma unroll
  for (int f = 0; f < kNF; ++f) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(u[f]);
    uint8_t *b = U + ((blk0 * kNF + f) * parts) * kCoreBytes;
    *reinterpret_cast<__nv_bfloat16 *>(b + off) = hi;
    if (X3) {
      const __nv_bfloat16 lo = __float2bfloat16_rn(u[f] - __bfloat162float(hi));
      *reinterpret_cast<__nv_bfloat16 *>(b + kCoreBytes + off) = lo;
    }
  }
}

// ---- the fused kernel -------------------------------------------------------------
template <bool X3, bool HALF, typename Tio>
__global__ void __launch_bounds__(Geo<HALF>::kThreads, Geo<HALF>::kMinBlocks)
    wino_fused_tc(const Tio *__restrict__ x, const uint8_t *__restrict__ U,
                  const float *__restrict__ bias, Tio *__restrict__ y, int C, int K, int H, int W,
                  int tiles_y, int tiles_x, long long total_tiles, int relu) {
  using L = Layout<X3, HALF>;
  using G = Geo<HALF>;
  constexpr int P = L::kParts;
  constexpr int kTiles = G::kTiles, kNU = G::kNU, kVBytes = G::kVBytes;
  constexpr int kEpiThreads = 32 * G::kXWarps;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t v_full = sbase + L::kBarOff, v_empty = v_full + 8 * kNV;
  const uint32_t u_full = v_empty + 8 * kNV, u_empty = u_full + 8 * kNU;
  const uint32_t acc_full = u_empty + 8 * kNU, drain = acc_full + 8;
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::kAbortSlot);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kTmemSlot);

  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);  // warp-uniform
  const int lane = threadIdx.x & 31;
  const int C16 = (C + kCc - 1) / kCc;
  const int kblk = blockIdx.y;
  const long long tile0 = (long long)blockIdx.x * kTiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNV; ++i) {
      mbar_init(v_full + 8 * i, G::kXWarps);
      mbar_init(v_empty + 8 * i, 1);
    }
    for (int i = 0; i < kNU; ++i) {
      mbar_init(u_full + 8 * i, 1);
      mbar_init(u_empty + 8 * i, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------- TMEM owner + MMA issuer ----------------
    // The allocation may wait for a co-resident CTA to free its columns; the
    // producer and transform warps meanwhile fill the first stages.
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    tc_fence_before();
    __syncwarp();
    named_bar_arrive(kBarTmem, 32 + kEpiThreads);  // hands the address to the epilogue warps
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    {
      // The whole warp walks the pipeline; one elected lane issues.
      constexpr uint32_t idesc = instr_desc(kCout, kTiles);
      constexpr uint32_t idesc_neg = idesc | (1u << 13);  // negate A
      constexpr uint32_t kLo = (uint32_t)(kNF * kVBytes) >> 4;  // V hi -> V lo
      const uint64_t a0 = smem_desc(sbase + L::kUOff, 128, 256);
      // V blocks are K-half-major: the two 8-channel halves kTiles*16 bytes
      // apart, 8-tile row groups 128 bytes apart.
      const uint64_t b0 = smem_desc(sbase + L::kVOff, (uint32_t)(kTiles * 16), 128);
      bool ok = true;
      int ui = 0;
      for (int cs = 0; cs < C16; ++cs) {
        const int vs = cs % kNV;
        ok = __all_sync(0xffffffffu, mbar_wait(v_full + 8 * vs, (cs / kNV) & 1, abort));
        if (!ok) break;
        tc_fence_after();
        const uint64_t bst = b0 + (uint64_t)((uint32_t)(vs * L::kVStage) >> 4);
        const uint32_t acc0 = cs > 0 ? 1u : 0u;
#pragma unroll
        for (int fp = 0; fp < kNF / kFPerU; ++fp, ++ui) {
          const int us = ui % kNU;
          ok = __all_sync(0xffffffffu, mbar_wait(u_full + 8 * us, (ui / kNU) & 1, abort));
          if (!ok) break;
          tc_fence_after();
          const uint64_t ast = a0 + (uint64_t)((uint32_t)(us * L::kUStage) >> 4);
#pragma unroll
          for (int fi = 0; fi < kFPerU; ++fi) {
            const int f = fp * kFPerU + fi;
            const uint64_t ah = ast + (uint64_t)((uint32_t)(fi * P * kCoreBytes) >> 4);
            const uint64_t bh = bst + (uint64_t)((uint32_t)(f * kVBytes) >> 4);
#pragma unroll
            for (int i = 0; i < (HALF ? 2 : 1); ++i) {
              const int a = f >> 2, b = f & 3;
              const int sgn = HALF ? at23(i, a) : 1;
              if (sgn == 0) continue;
              // accumulator: Z[i][b] (half-folded) or M[a][b]
              const int q = HALF ? i * 4 + b : f;
              const uint32_t d = tmem + (uint32_t)(q * kTiles);
              const uint32_t id = sgn < 0 ? idesc_neg : idesc;
              // the first term of Z[i][b] is a = i (At[0][0] = At[1][1] = 1)
              const uint32_t first = HALF ? (a == i ? acc0 : 1u) : acc0;
              if (elect_one()) mma_bf16(d, ah, bh, id, first);
              if (X3) {
                if (elect_one()) mma_bf16(d, ah, bh + kLo, id, 1u);
                if (elect_one()) mma_bf16(d, ah + (uint64_t)(kCoreBytes >> 4), bh, id, 1u);
              }
            }
          }
          __syncwarp();
          if (elect_one()) tc_commit(u_empty + 8 * us);
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) tc_commit(v_empty + 8 * vs);
        __syncwarp();
      }
      if (ok) {
        if (elect_one()) tc_commit(acc_full);
        __syncwarp();
      } else {
        // drain whatever was issued before giving up
        if (elect_one()) tc_commit(drain);
        __syncwarp();
        const unsigned long long t0 = globaltimer();
        while (!mbar_try(drain, 0) && globaltimer() - t0 < kTimeoutNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- producer: U stages by bulk copy ----------------
    const int nstages = C16 * (kNF / kFPerU);
    const uint8_t *ublk = U + (size_t)kblk * C16 * kNF * P * kCoreBytes;
    int issued = 0;
    for (int i = 0; i < nstages; ++i) {
      const int s = i % kNU;
      if (!__all_sync(0xffffffffu, mbar_wait(u_empty + 8 * s, ((i / kNU) & 1) ^ 1, abort)))
        break;
      if (elect_one()) {
        mbar_expect_tx(u_full + 8 * s, L::kUStage);
        bulk_g2s(sbase + L::kUOff + s * L::kUStage, ublk + (size_t)i * L::kUStage, L::kUStage,
                 u_full + 8 * s);
      }
      __syncwarp();
      issued = i + 1;
    }
    // never leave the CTA with a copy still writing shared memory
    for (int i = issued - kNU > 0 ? issued - kNU : 0; i < issued; ++i) {
      const int s = i % kNU;
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(u_full + 8 * s, (i / kNU) & 1) && globaltimer() - t0 < kTimeoutNs) {
      }
    }
  } else {
    // ---------------- transform warps, then epilogue ----------------
    const int tw = warp - 2;            // 0 .. kXWarps-1
    // warp -> (16-tile block, group of 2*CPT channels); lane -> (tile, CPT
    // channels).  A warp load then reads 16 consecutive tiles of 2 channel
    // planes (2 x 64-128 contiguous bytes) and a warp store fills one
    // contiguous run of the K-half-major V block.
    constexpr int kTileBlocks = kTiles / 16, CPT = G::kCpt;
    const int cgrp = tw / kTileBlocks;
    const int cbase = cgrp * (2 * CPT) + (lane & 1) * CPT;  // first channel of the stage
    const int kh = cbase >> 3;                               // K half of the MMA step
    const int t = (tw % kTileBlocks) * 16 + (lane >> 1);  // tile within the CTA
    const long long T = tile0 + t;
    const bool tile_ok = T < total_tiles;
    int n = 0, ty = 0, tx = 0;
    if (tile_ok) {
      const long long per_img = (long long)tiles_y * tiles_x;
      n = (int)(T / per_img);
      const int rem = (int)(T - (long long)n * per_img);
      ty = rem / tiles_x;
      tx = rem - ty * tiles_x;
    }
    const int y0 = 2 * ty - 1, x0 = 2 * tx - 1;
    const size_t plane = (size_t)H * W;
    const Tio *xn = x + (size_t)n * C * plane;
    // row/column validity of the 4x4 patch (pad = 1)
    bool rv[4], cv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rv[i] = tile_ok && (y0 + i) >= 0 && (y0 + i) < H;
      cv[i] = (x0 + i) >= 0 && (x0 + i) < W;
    }
    float d[CPT][4][4];  // [channel][row][col]
    auto load_stage = [&](int cs) {
#pragma unroll
      for (int q = 0; q < CPT; ++q) {
        const int c = cs * kCc + cbase + q;
        const bool cok = c < C;
        const Tio *xc = xn + (size_t)c * plane;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            d[q][i][j] = (cok && rv[i] && cv[j])
                             ? to_f32(xc[(size_t)(y0 + i) * W + (x0 + j)])
                             : 0.f;
      }
    };
    bool ok = true;
    if (C16 > 0) load_stage(0);
    for (int cs = 0; cs < C16; ++cs) {
      const int vs = cs % kNV;
      ok = __all_sync(0xffffffffu, mbar_wait(v_empty + 8 * vs, ((cs / kNV) & 1) ^ 1, abort));
      if (!ok) break;
      uint8_t *vb = smem + L::kVOff + vs * L::kVStage;
      const uint32_t off = (uint32_t)(kh * (kTiles * 16) + t * 16 + (cbase & 7) * 2);
      float v[CPT][4][4];
#pragma unroll
      for (int q = 0; q < CPT; ++q) input_transform<2>(d[q], v[q]);
#pragma unroll
      for (int f = 0; f < kNF; ++f) {
        const int a = f >> 2, b = f & 3;
        if constexpr (CPT == 4) {
          const float e0 = v[0][a][b], e1 = v[1][a][b], e2 = v[2][a][b], e3 = v[3][a][b];
          uint2 hi, lo;
          if (X3) {
            split_pair(e0, e1, hi.x, lo.x);
            split_pair(e2, e3, hi.y, lo.y);
            *reinterpret_cast<uint2 *>(vb + (kNF + f) * kVBytes + off) = lo;
          } else {
            hi.x = pack_bf16(e0, e1);
            hi.y = pack_bf16(e2, e3);
          }
          *reinterpret_cast<uint2 *>(vb + f * kVBytes + off) = hi;
        } else {
          const float e0 = v[0][a][b], e1 = v[1][a][b];
          uint32_t hi, lo;
          if (X3) {
            split_pair(e0, e1, hi, lo);
            *reinterpret_cast<uint32_t *>(vb + (kNF + f) * kVBytes + off) = lo;
          } else {
            hi = pack_bf16(e0, e1);
          }
          *reinterpret_cast<uint32_t *>(vb + f * kVBytes + off) = hi;
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(v_full + 8 * vs);
      if (cs + 1 < C16) load_stage(cs + 1);
    }

    // ---------------- epilogue ----------------
    named_bar_sync(kBarTmem, 32 + kEpiThreads);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort));
    tc_fence_after();
    if (ok) {
      // Lane = output channel after tcgen05.ld.  Each group of 8 tiles is
      // transposed through a private shared-memory patch (row stride 33
      // floats: conflict-free both ways) so that every warp store then writes
      // two contiguous 64-byte row segments of one channel plane.  The operand
      // stages are free: every MMA has completed.
      const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
      constexpr int kCols = kTiles * 4 / G::kXWarps;  // tile columns per epilogue warp
      const int col0 = (tw / 4) * kCols;
      const int kq = kblk * kCout + quad * 32;
      const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
      float *patch = reinterpret_cast<float *>(smem) + tw * (32 * 33);
      const float bk = (bias != nullptr && kq + lane < K) ? bias[kq + lane] : 0.f;
      const long long per_img = (long long)tiles_y * tiles_x;
      // this lane's output pixel in the read-back phase: tile j, pixel (pi, pj)
      const int jt = lane >> 2, pi = (lane >> 1) & 1, pj = lane & 1;
#pragma unroll 1
      for (int gq = 0; gq < kCols / 8; ++gq) {
        const int cbase = col0 + gq * 8;
        float acc[G::kAcc][8];
#pragma unroll
        for (int q = 0; q < G::kAcc; ++q) {
          float lo4[4], hi4[4];
          tmem_ld4(trow + (uint32_t)(q * kTiles + cbase), lo4);
          tmem_ld4(trow + (uint32_t)(q * kTiles + cbase + 4), hi4);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[q][e] = lo4[e];
            acc[q][4 + e] = hi4[e];
          }
        }
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float o[2][2];
          if (HALF) {
            // Y[i][j'] = sum_b Z[i][b] At[j'][b]
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float z0 = acc[i * 4 + 0][j], z1 = acc[i * 4 + 1][j];
              const float z2 = acc[i * 4 + 2][j], z3 = acc[i * 4 + 3][j];
              o[i][0] = (z0 + z1) + z2;
              o[i][1] = (z1 - z2) - z3;
            }
          } else {
            float mm[4][4];
#pragma unroll
            for (int f = 0; f < kNF; ++f) mm[f >> 2][f & 3] = acc[f][j];
            output_transform<2>(mm, o);
          }
#pragma unroll
          for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              float val = o[i][jj] + bk;
              if (relu) val = val < 0.f ? 0.f : val;
              patch[lane * 33 + j * 4 + i * 2 + jj] = val;
            }
        }
        __syncwarp();
        const long long TT = tile0 + cbase + jt;
        if (TT < total_tiles) {
          const int nn = (int)(TT / per_img);
          const int rem = (int)(TT - (long long)nn * per_img);
          const int yy = rem / tiles_x, xx = rem - yy * tiles_x;
          const int oy = 2 * yy + pi, ox = 2 * xx + pj;
          if (oy < H && ox < W) {
            Tio *dst = y + ((size_t)nn * K + kq) * plane + (size_t)oy * W + ox;
            const int kmax = K - kq < 32 ? K - kq : 32;
#pragma unroll 4
            for (int cc = 0; cc < kmax; ++cc)
              dst[(size_t)cc * plane] = from_f32<Tio>(patch[cc * 33 + jt * 4 + pi * 2 + pj]);
          }
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot),
                 "r"(kTmemCols));
  }
}

template <bool X3, bool HALF, typename Tio>
static cudaError_t launch(const void *x, const void *U, const float *bias, void *y, int n, int c,
                          int k, int h, int w, int relu, cudaStream_t s) {
  constexpr int kTiles = Geo<HALF>::kTiles;
  const int tiles_y = (h + 1) / 2, tiles_x = (w + 1) / 2;
  const long long total = (long long)n * tiles_y * tiles_x;
  const long long gx = (total + kTiles - 1) / kTiles;
  const int gy = (k + kCout - 1) / kCout;
  if (gx > 0x7fffffffLL || gy > 65535) return cudaErrorInvalidValue;
  auto fn = wino_fused_tc<X3, HALF, Tio>;
  cudaError_t e = smem_attr_once<wino_fused_tc<X3, HALF, Tio>>(Layout<X3, HALF>::kSmem);
  if (e != cudaSuccess) return e;
  fn<<<dim3((unsigned)gx, (unsigned)gy), Geo<HALF>::kThreads, Layout<X3, HALF>::kSmem, s>>>(
      (const Tio *)x, (const uint8_t *)U, bias, (Tio *)y, c, k, h, w, tiles_y, tiles_x, total,
      relu);
  return cudaGetLastError();
}

// ==== 2-SM pair kernel (tcgen05.mma.cta_group::2) ====================================
//
// A CTA pair (a cluster of two, on the two SMs of one TPC) computes one block
// of output channels x N tiles.  The half-folded accumulation
// Z[i][b] = sum_a At[i][a] M[a][b] is stacked along M = 256:
//   A = [At[i0][a] U_ab ; At[i0 + 1][a] U_ab]  -- the rows of two output-row
//        indices, pre-scaled by At (exact in bf16); rank r holds those of
//        i0 + r (128 output channels);
//   B = V_ab of the pair's N tiles             -- rank r holds half of them;
//   D = Z[i][b]: rank r's TMEM holds, for its rows, (m+2) accumulators x N.
// F(2,3): 128 channels x 128 tiles, rank r = output row 2ty + r.  F(4,3): 128
// channels x 64 tiles per pass, pass p: rank r = output row 4ty + 2p + r; a
// pass multiplies only the 30 frequencies whose two At rows are not both zero.
// One MMA per (frequency, product) serves both output rows and N tiles: for
// F(2,3) the tensor core reads 6 KB of shared memory per 262K MACs of an SM
// instead of 6 KB per 131K in the single-CTA kernel.
//
// Rank 0 issues every MMA and commit for the pair.  Readiness of rank 1's
// operands reaches rank 0 by remote mbarrier arrivals: rank 1's warp 0 (idle
// otherwise) relays each of its completed V stages and landed weight stages.
// Releases (operand stages, accumulators) are multicast commits that arrive on
// both CTAs' barriers.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrival on a barrier of another CTA of the cluster.  Default (CTA-scope)
// release: a cluster-scope release costs ~1.4K cycles per arrival, and what it
// would order is already complete -- bulk copies by their own mbarrier, thread
// writes to V by fence.proxy.async and the local barrier the relay observed.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Programmatic dependent launch: wait for the previous grid of the stream to
// complete (its memory operations visible); allow the next grid to launch.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
// completion of this thread's earlier MMAs -> one arrival on the barrier at
// offset `bar` of every CTA in `mask`
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void mma_pair_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[e]);
}

// y[0..3] += v, one 16-byte vector reduction in L2 (16-byte aligned address).
__device__ __forceinline__ void red_add_v4(float *y, float4 v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(y), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

// Two consecutive elements (an aligned pair) as fp32; zeros when !ok.
__device__ __forceinline__ void ld_pair(const float *p, bool ok, float &a, float &b) {
  float2 v = make_float2(0.f, 0.f);
  if (ok) v = *reinterpret_cast<const float2 *>(p);
  a = v.x;
  b = v.y;
}
__device__ __forceinline__ void ld_pair(const __nv_bfloat16 *p, bool ok, float &a, float &b) {
  uint32_t v = 0;
  if (ok) v = *reinterpret_cast<const uint32_t *>(p);
  a = __uint_as_float(v << 16);
  b = __uint_as_float(v & 0xFFFF0000u);
}

// Products per multiply-accumulate of the pair kernel (its PM parameter):
//   kPmX3  bf16 operands split as hi + lo, three MMAs hi*hi + hi*lo + lo*hi:
//          fp32-accurate (fp32 layers);
//   kPmH2  fp16 operands, weights in one part and V split as hi + lo, two MMAs
//          U*V_hi + U*V_lo (bf16 F(4,3) layers: fp16's 11 significant bits keep
//          F(4,3)'s amplified rounding error near 5e-3 normwise, where single
//          bf16 products reach ~6e-2);
//   kPmX1  one bf16 MMA (bf16 F(2,3) layers).
enum : int { kPmX1 = 1, kPmH2 = 2, kPmX3 = 3 };
template <int PM>
struct Prod {
  static constexpr int kUParts = PM == kPmX3 ? 2 : 1;  // weight blocks per frequency
  static constexpr int kVParts = PM == kPmX1 ? 1 : 2;  // V blocks per frequency
  static constexpr bool kF16 = PM == kPmH2;            // fp16 rather than bf16 operands
};
// Largest finite fp16; bit of g_tc_status set when an fp16 operand would overflow.
constexpr float kF16Max = 65504.f;
constexpr unsigned kStatusRange = 2u;

// Division of a non-negative int below 2^31 by a divisor fixed for the launch,
// as a multiply-high: with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (umulhi(m, n) + n) >> l (Granlund and Montgomery, "Division by
// invariant integers using multiplication", 1994; the sum stays below 2^32 for
// n < 2^31).  Tile indices and their remainders within an image take it.
struct FastDiv {
  uint32_t m, l;
};
__host__ __device__ inline FastDiv fast_div(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  return FastDiv{(uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1), l};
}
__device__ __forceinline__ int fdiv(int n, FastDiv f) {
  return (int)((__umulhi(f.m, (uint32_t)n) + (uint32_t)n) >> f.l);
}
// n / d: the multiply-high form in the F(2,3) kernels (measured 169.4 vs 171.3 and
// 173.0 vs 174.6 us on 64 images of 128->128 at 56x56), the plain division in
// F(4,3), where the multiply-high form measured no faster (32 images of 256->256
// at 112x112: 1254 vs 1229 us, then 1246 vs 1249 us)
template <int M>
__device__ __forceinline__ int tile_div(int n, int d, FastDiv f) {
  if constexpr (M == 2)
    return fdiv(n, f);
  else
    return n / d;
}

// r = Bt x for F(4x4,3x3) (Bt rows 4 0 -5 0 1 0 / 0 -4 -4 1 1 0 / 0 4 -4 -1 1 0 /
// 0 -2 -1 2 1 0 / 0 2 -1 -2 1 0 / 0 4 0 -5 0 1), factored over the sums and
// differences the rows share: 6 additions and 8 multiply-adds.
template <typename T>
__device__ __forceinline__ void bt6(const T &x, float (&r)[6]) {
  const float a = x[1] + x[2], b = x[3] + x[4];
  const float c = x[1] - x[2], d = x[4] - x[3];
  const float e = x[4] - x[2], f = x[3] - x[1];
  r[0] = fmaf(4.f, x[0], fmaf(-5.f, x[2], x[4]));
  r[1] = fmaf(-4.f, a, b);
  r[2] = fmaf(4.f, c, d);
  r[3] = fmaf(2.f, f, e);
  r[4] = fmaf(-2.f, f, e);
  r[5] = fmaf(4.f, x[1], fmaf(-5.f, x[3], x[5]));
}

// Geometry of the pair kernel for F(M x M, 3x3).
//   F(2,3): rank r holds the 128 rows (i = r, output channel), 64 tiles of V;
//           N = 128, 4 accumulators Z[r][b] x 128 columns.
//   F(4,3): two passes (items) per channel block; in pass p rank r holds the
//           128 rows of output row i = 2p + r (output channel), 32 tiles of V;
//           N = 64, 6 accumulators x 64 columns.  Layers of at most 64 output
//           channels (RP = 2) keep one pass of two rows x 64 channels per rank
//           over all 36 frequencies, which is also what every F(4,3) layer ran
//           before the passes (1346 vs 1272 us on 32 images of 256->256 at
//           112x112).
//   HM ("half M", F(2,3) layers of at most 64 output channels): M = 128, rank r
//           holds 64 rows (i = r, output channel); in TMEM the accumulator's
//           columns [0, N/2) sit in lanes 0-63 and [N/2, N) in lanes 64-127,
//           both at columns 0 .. N/2-1.
template <int M, bool HM = false, int RP = 1>
struct PairGeo {
  static_assert(!HM || M == 2, "the M = 128 pair kernel is F(2,3) only");
  static_assert(RP == 1 || (M == 4 && !HM && RP == 2), "two rows per CTA: F(4,3) only");
  static constexpr int TD = M + 2, NF = TD * TD;
  // A pass of the pair computes RP output rows of every tile on each rank
  // (rank r: rows (2p + r) RP ..), for kCoutCta output channels.  F(4,3) with
  // RP = 1 runs two passes (rows 0-1, rows 2-3) as separate items; each skips
  // the frequency row a that both of its At rows leave zero (a = 5 for rows 0
  // and 1, a = 0 for rows 2 and 3), so a pass multiplies 30 of the 36
  // frequencies.  RP = 2 (layers of at most 64 output channels): one pass, 2
  // rows x 64 channels per rank, all 36 frequencies.
  static constexpr int kPasses = M / 2 / RP;
  static constexpr int kRowsI = RP;                 // output rows i per CTA and pass
  static constexpr int kRowsCta = HM ? 64 : kCout;  // A rows (MMA M / 2) per CTA
  static constexpr int kMmaM = 2 * kRowsCta;        // MMA M of the pair
  static constexpr int kCoutCta = kRowsCta / RP;    // output channels per CTA
  static constexpr int NFP = (M == 4 && RP == 1) ? NF - TD : NF;  // frequencies a pass multiplies
  // first frequency of pass p (frequencies f0 .. f0 + NFP - 1, f = a * TD + b)
  __host__ __device__ static constexpr int f0(int p) { return (M == 4 && RP == 1 && p) ? TD : 0; }
  static constexpr int kBlkBytes = kRowsCta * kCc * 2;  // one weight block (rows x 16 ch)
  static constexpr int kTiles = M == 2 ? 64 : 32;   // V columns (tiles) per CTA
  static constexpr int kN = 2 * kTiles;             // MMA N of the pair
  static constexpr int kXWarps = 16;                // transform + epilogue warps
  static constexpr int kThreads = (2 + kXWarps) * 32;
  // A thread transforms 2 channels of one tile.  F(2,3): all 16 warps take
  // every stage, with the next stage's patches in registers meanwhile.
  // F(4,3): two groups of 8 warps take alternate stages (two 6x6 windows fill
  // the registers).  Splitting F(2,3) the same way, with 4 channels per thread
  // and conflict-free 8-byte V stores, was slower (207 vs 190 us on a 64-image
  // 128->128 56x56 layer): with two V slots each group's slot then stays busy
  // through its own transform and the MMAs.
  static constexpr int kGroups = M == 2 ? 1 : 2;
  static constexpr int kGroupWarps = kXWarps / kGroups;
  static constexpr int kCpt = 2;
  // weight stages in flight.  Fewer than the stream could use: every KB of
  // shared memory left unallocated serves as L1 cache for the input windows,
  // and their misses refill the same SRAM the tensor core reads its operands
  // from.  Measured on B200 (us/layer, 2 / 3 / 4 / 5 stages): 64 images of
  // 128->128 at 56x56 (F(2,3), 16 KB stages) 198 / 177 / 179 / 182; 256 images
  // of 64->64 at 56x56 (8 KB stages, 3 / 4 / 6 / 8) 285 / 286 / 289 / 288.
  static constexpr int kNU = HM ? 4 : 3;
  static constexpr int kVBytes = kTiles * kCc * 2;  // one frequency of V
  static constexpr int kEpiTiles = 32 / M;          // tiles per 32-pixel epilogue patch row
  static_assert(TD * kN <= kTmemCols, "accumulators fit TMEM");
  static_assert(kTiles * kCc == kGroupWarps * 32 * kCpt, "one (tile, channels) per thread");
};

// Pair weight layout: [ceil(C_out/cout_cta)][pass][rank = 2][C_pad/16][NFP f][parts][block]
// (blocks of rows_cta rows x 16 channels: 4096 B, or 2048 B for HM; a pass
// stores its NFP frequencies f0(pass) ..): block row k' of rank r holds
// At[2 pass + r][a] * U_ab for output channel kblk * cout_cta + k' (scaling by
// 0, +-1, +-2, +-4, +-8 is exact in bf16 and fp16).  Channels past C_out / C_in are zero.  Parts: bf16 hi and
// lo (kPmX3), one bf16 block (kPmX1) or one fp16 block (kPmH2).  An fp16 weight
// beyond the fp16 range sets the range bit of the status word.
template <int M, int PM, bool HM, int RP = 1>
__global__ void wt_transform_tc_pair(const float *__restrict__ src, uint8_t *__restrict__ U,
                                     int C, int K, int Cp, int Kp, int from_ref) {
  using G = PairGeo<M, HM, RP>;
  using P = Prod<PM>;
  constexpr int NF = G::NF, TD = G::TD;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)Cp * Kp) return;
  const int c = (int)(idx % Cp), k = (int)(idx / Cp);
  float u[NF];
  if (k < K && c < C) {
    transform_one<M>(src + ((long)k * C + c) * (from_ref ? NF : 9), from_ref, u);
  } else {
#pragma unroll
    for (int f = 0; f < NF; ++f) u[f] = 0.f;
  }
  constexpr int parts = P::kUParts;
  const int C16 = Cp / kCc;
  const int kb = k / G::kCoutCta, kr = k % G::kCoutCta;
  float umax = 0.f;
#pragma unroll
  for (int pass = 0; pass < G::kPasses; ++pass)
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int il = 0; il < G::kRowsI; ++il) {
        const long blk0 = (((long)kb * G::kPasses + pass) * 2 + r) * C16 + c / kCc;
        const uint32_t off = blk_off(il * G::kCoutCta + kr, c % kCc);
#pragma unroll
        for (int fp = 0; fp < G::NFP; ++fp) {
          const int f = G::f0(pass) + fp;
          const float s = Wino<M>::at((2 * pass + r) * G::kRowsI + il, f / TD) * u[f];
          uint8_t *b = U + ((blk0 * G::NFP + fp) * parts) * G::kBlkBytes;
          if constexpr (P::kF16) {
            *reinterpret_cast<__half *>(b + off) = __float2half_rn(s);
            umax = fmaxf(umax, fabsf(s));
          } else {
            const __nv_bfloat16 hi = __float2bfloat16_rn(s);
            *reinterpret_cast<__nv_bfloat16 *>(b + off) = hi;
            if (P::kUParts == 2)
              *reinterpret_cast<__nv_bfloat16 *>(b + G::kBlkBytes + off) =
                  __float2bfloat16_rn(s - __bfloat162float(hi));
          }
        }
      }
  if (P::kF16 && !(umax <= kF16Max)) atomicOr(&g_tc_status, kStatusRange);
}

// Shared memory of one CTA of the pair.
template <int M, int PM, bool HM = false, int RP = 1>
struct PairLayout {
  using G = PairGeo<M, HM, RP>;
  using P = Prod<PM>;
  // weight stages: PairGeo::kNU for F(2,3) (twice that for one-part bf16 stages,
  // the same bytes in flight); five for F(4,3) (32 images of 256->256 at
  // 112x112, fp16 stages, 2 / 3 / 4 / 5 / 10 stages: 1959 / 1500 / 1364 / 1356 /
  // 1368 us)
  static constexpr int kNU = M == 2 ? G::kNU * (PM == kPmX1 ? 2 : 1) : 5;
  static constexpr int kVStage = P::kVParts * G::NF * G::kVBytes;
  static constexpr int kUStage = kFPerU * P::kUParts * G::kBlkBytes;
  static constexpr int kVOff = 0;
  static constexpr int kUOff = kVOff + kNV * kVStage;
  static constexpr int kBarOff = kUOff + kNU * kUStage;
  // v_full[kNV], v_empty[kNV], v_peer[kNV] (rank 0: rank 1's V stage written),
  // u_full[kNU], u_empty[kNU], u_peer[kNU] (rank 0: rank 1's weights landed),
  // acc_full, drain, tmem_empty (rank 0: both CTAs have read the accumulators)
  static constexpr int kNumBars = 3 * kNV + 3 * kNU + 3;
  static constexpr int kTmemSlot = kBarOff + 8 * kNumBars;
  static constexpr int kAbortSlot = kTmemSlot + 4;
  // epilogue transpose patch of one warp: 32 output channels x 32 pixels, the
  // pixel index XOR the channel (conflict-free both ways, no padding)
  static constexpr int kPx = G::kEpiTiles * M;  // output pixels per patch row
  static_assert(kPx == 32, "one 32 x 32 patch per warp");
  static constexpr int kPatchFloats = 32 * 32;
  static constexpr int kPatchBytes = G::kXWarps * kPatchFloats * 4;
  // An item's patches live in the V slot that the next item's second stage
  // takes (free once the item's MMAs have completed); where one V slot is too
  // small for them (one-product layouts), in a region of their own.
  static constexpr bool kPatchInV = kPatchBytes <= kVStage;
  static constexpr int kPatchOff = (kAbortSlot + 4 + 127) / 128 * 128;
  static constexpr int kSmem = kPatchInV ? kAbortSlot + 4 : kPatchOff + kPatchBytes;
  static_assert(kSmem <= 227 * 1024, "fits the opt-in shared memory of one CTA");
  static_assert(G::NFP % kFPerU == 0, "whole frequencies per weight stage");
};

// Work of one CTA pair p = blockIdx.x / 2, as a sequence of items.
//   chunk > 0: the tiles [p * chunk, min((p + 1) * chunk, total)), cut into items
//     of at most kN tiles; each tile block runs for kb_count output-channel
//     blocks in turn (kb_count == 1: the block blockIdx.y).  A layer of at most
//     one wave launches chunk = kN, one item per pair; a larger one may launch one
//     pair per co-resident cluster with equal chunks, so that the last items are
//     short ones (MMA N rounded up to 16) instead of a last wave that leaves most
//     TPCs idle.
//   chunk == 0: round robin over the (kN-tile block, output-channel block) units,
//     unit u = p + idx * pairs, u = block * kb_count + channel block: the
//     pairs at work at one time share their input tiles through L2.
// Either way a pair writes the first stage of its next item ahead of the
// current item's epilogue.
struct PairItem {
  int t0;   // first tile of the item
  int cnt;       // tiles in the item, 1..kN
  int kb;        // output-channel block
};
template <int KN>
__device__ __forceinline__ PairItem pair_item(int chunk, int total, int kb_count, int idx) {
  PairItem it;
  int hi = total;
  if (chunk == 0) {
    const int u = (int)(blockIdx.x >> 1) + idx * (int)(gridDim.x >> 1);
    const int tb = u / kb_count;
    it.kb = u - tb * kb_count;
    it.t0 = tb * KN;
  } else {
    const int lo = (int)(blockIdx.x >> 1) * chunk;
    hi = total - lo > chunk ? lo + chunk : total;
    int tbi = idx / kb_count;
    it.kb = kb_count == 1 ? (int)blockIdx.y : idx - tbi * kb_count;
    // odd pairs take their short last block first: the pairs' epilogues (and
    // their bursts of output stores) then alternate instead of coinciding
    const int nb = (hi - lo + KN - 1) / KN;
    if ((blockIdx.x >> 1) & 1) tbi = tbi == 0 ? nb - 1 : tbi - 1;
    it.t0 = lo + tbi * KN;
  }
  const int left = hi - it.t0;
  it.cnt = left < KN ? left : KN;
  return it;
}
// MMA N of an item (M = 256 takes N in steps of 16); each CTA holds N/2 rows of B
__device__ __forceinline__ int item_n(int cnt) { return (cnt + 15) & ~15; }

// Named barrier 2: the epilogue warps have finished with their patches.
constexpr int kBarEpi = 2;

// Epilogue of item e of a pair, run by every transform warp: output rows M ty + i
// of the item's tiles.  TMEM lane = (il, output channel).  Each group of
// kEpiTiles tiles (32 output pixels of one row) goes through the warp's 32 x 32
// patch, then out as 16-byte stores of 4 pixels of one channel (or, at image
// edges and odd alignments, one channel plane per warp store).  Every warp runs
// every item's epilogue, also after an abort (then only its barrier arrivals), so
// that the named barriers match.  Not inlined: its registers stay out of the
// transform loop, which calls it once per item.
template <int M, int PM, typename Tio, bool HM, int RP>
__device__ __noinline__ bool pair_epilogue(int e, bool run, int nst, uint8_t *smem,
                                           const float *__restrict__ bias, Tio *__restrict__ y,
                                           int K, int H, int W, int tiles_y, int tiles_x,
                                           int total_tiles, int chunk, int kb_count,
                                           int relu, int split, FastDiv fd_img,
                                           FastDiv fd_tx) {
  using L = PairLayout<M, PM, HM, RP>;
  using G = PairGeo<M, HM, RP>;
  constexpr int TD = G::TD, kN = G::kN, kNU = L::kNU;
  constexpr int kEpiThreads = 32 * G::kXWarps;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t acc_full = sbase + L::kBarOff + 8 * (3 * kNV + 3 * kNU);
  const uint32_t tmem_empty = acc_full + 16;
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::kAbortSlot);
  const uint32_t *tmem_slot = reinterpret_cast<const uint32_t *>(smem + L::kTmemSlot);
  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int tw = warp - 2;
  const uint32_t rank = cluster_rank();
  const size_t plane = (size_t)H * W;
  const int per_img = tiles_y * tiles_x;

  if (e == 0) named_bar_sync(kBarTmem, 32 + kEpiThreads);  // TMEM address published
  // the item and its bias load before the wait for the accumulators
  const PairItem it = pair_item<kN>(chunk, total_tiles, kb_count, e);
  const int quad = warp & 3;
  // TMEM lanes 32 quad .. 32 quad + 31: channels kq .. kq + 31 of output row
  // irow; HM: lanes 64-127 repeat channels 0-63 for the second half of the columns
  const int kq = (it.kb / G::kPasses) * G::kCoutCta +
                 (HM ? 32 * (quad & 1) : (quad * 32) % G::kCoutCta);
  // a split adds its partial sums into y (zeroed by the host); slice 0 adds
  // the bias unless a ReLU must follow the full sum, in which case a separate
  // pass applies both once every slice has landed
  const bool add_bias = !split || (!relu && blockIdx.z == 0);
  const float bk = (run && add_bias && bias != nullptr && kq + lane < K) ? bias[kq + lane] : 0.f;
  if (run) run = __all_sync(0xffffffffu, mbar_wait(acc_full, (uint32_t)e & 1u, abort));
  tc_fence_after();
  if (run) {
    constexpr int kE = G::kEpiTiles;
    const uint32_t tmem = *tmem_slot;
    const int il = HM ? 0 : (quad * 32) / G::kCoutCta;
    // output row i of the tile
    const int irow = (2 * (it.kb % G::kPasses) + (int)rank) * G::kRowsI + il;
    // item columns [col0, lim) of this warp, at TMEM column (column - tshift):
    // 32 (F2) or 16 (F4) per warp; HM: 16 per warp within its lanes' half
    int col0 = (tw >> 2) * (kN / 4), lim = it.cnt, tshift = 0;
    if constexpr (HM) {
      const int nh = item_n(it.cnt) >> 1, hq = quad >> 1;
      tshift = hq * nh;
      col0 = tshift + (tw >> 2) * kE;
      lim = it.cnt < tshift + nh ? it.cnt : tshift + nh;
    }
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const int pslot = ((e + 1) * nst + 1) % kNV;
    float *patch =
        reinterpret_cast<float *>(smem + (L::kPatchInV ? L::kVOff + pslot * L::kVStage
                                                       : L::kPatchOff)) +
        tw * L::kPatchFloats;
    const bool do_relu = relu && !split;
    const int kmax = K - kq < 32 ? K - kq : 32;
#pragma unroll 1
    for (int gq = 0; gq < (HM ? 1 : (kN / 4) / kE); ++gq) {
      const int cb = col0 + gq * kE;
      if (cb >= lim) break;
      // 8 tiles (columns) at a time from TMEM: TD x 8 registers
#pragma unroll 1
      for (int h = 0; h < kE; h += 8) {
        float z[TD][8];
#pragma unroll
        for (int b = 0; b < TD; ++b)
          tmem_ld8(trow + (uint32_t)(b * kN + cb - tshift + h), z[b]);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 2 * M; ++q) {  // 4 pixels (px = 4q ..) of this 8-tile half
          float o[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int e2 = (4 * q + r) / M, j = (4 * q + r) % M;
            // Y[i][j] = sum_b Z[i][b] At[j][b]
            float s = 0.f;
#pragma unroll
            for (int b = 0; b < TD; ++b) {
              const float cf = Wino<M>::at(j, b);
              if (cf != 0.f) s = fmaf(cf, z[b][e2], s);
            }
            s += bk;
            o[r] = do_relu && s < 0.f ? 0.f : s;
          }
          const int qg = (h * M) / 4 + q;  // 4-pixel chunk of the 32-pixel row
          *reinterpret_cast<float4 *>(patch + lane * 32 + ((qg ^ (lane & 7)) << 2)) =
              make_float4(o[0], o[1], o[2], o[3]);  // lane = channel
        }
      }
      __syncwarp();
      // Vector stores (a split: vector reductions): lane -> (4-pixel chunk q,
      // channel 4 cc + lane / 8), each lane's 4 pixels (4 / M consecutive tiles
      // of the item) contiguous in one image row and 16-byte aligned.
      // Otherwise (image edges, odd alignments): lane -> pixel, one channel
      // plane per warp store.
      const int q = lane & 7, chs = lane >> 3;
      long long off0 = -1;  // element offset of the lane's first pixel in channel kq
      bool vec = ((plane & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
#pragma unroll
      for (int u = 0; u < 4 / M; ++u) {
        const int tt = cb + (4 * q) / M + u;  // column = tile of the item
        long long o = -1;
        if (tt < lim) {
          const int TT = it.t0 + tt;
          const int nn = tile_div<M>(TT, per_img, fd_img);
          const int rem = TT - nn * per_img;
          const int yy = tile_div<M>(rem, tiles_x, fd_tx), xx = rem - yy * tiles_x;
          const int oy = M * yy + irow, ox = M * xx;
          if (oy < H && ox + M <= W)
            o = ((long long)nn * K + kq) * (long long)plane + (long long)oy * W + ox;
        }
        if (u == 0) off0 = o;
        vec = vec && o >= 0 && o == off0 + u * M;
      }
      vec = vec && (off0 & 3) == 0;
      if (__all_sync(0xffffffffu, vec)) {
#pragma unroll 2
        for (int cc = 0; cc < 8; ++cc) {
          const int ch = 4 * cc + chs;
          if (ch >= kmax) continue;
          const float4 v =
              *reinterpret_cast<const float4 *>(patch + ch * 32 + ((q ^ (ch & 7)) << 2));
          Tio *dst = y + off0 + (long long)ch * plane;
          if constexpr (sizeof(Tio) == 4) {
            if (split)
              red_add_v4(reinterpret_cast<float *>(dst), v);
            else
              *reinterpret_cast<float4 *>(dst) = v;
          } else {
            uint2 pk;
            pk.x = pack_bf16(v.x, v.y);
            pk.y = pack_bf16(v.z, v.w);
            *reinterpret_cast<uint2 *>(dst) = pk;
          }
        }
      } else {
        const int tt = cb + lane / M, j = lane % M;  // lane = pixel
        if (tt < lim) {
          const int TT = it.t0 + tt;
          const int nn = tile_div<M>(TT, per_img, fd_img);
          const int rem = TT - nn * per_img;
          const int yy = tile_div<M>(rem, tiles_x, fd_tx), xx = rem - yy * tiles_x;
          const int oy = M * yy + irow, ox = M * xx + j;
          if (oy < H && ox < W) {
            Tio *dst = y + ((size_t)nn * K + kq) * plane + (size_t)oy * W + ox;
            // the slices of a split start on different channels, so that their
            // atomic adds do not meet on the same lines at the same time
            const int rot = split ? (int)(blockIdx.z * 8) & 31 : 0;
#pragma unroll 4
            for (int c2 = 0; c2 < 32; ++c2) {
              const int ch = (c2 + rot) & 31;
              if (ch >= kmax) continue;
              const float v = patch[ch * 32 + ((((lane >> 2) ^ (ch & 7)) << 2) | (lane & 3))];
              if constexpr (sizeof(Tio) == 4) {
                if (split)
                  atomicAdd(reinterpret_cast<float *>(dst + (size_t)ch * plane), v);
                else
                  dst[(size_t)ch * plane] = v;
              } else {
                dst[(size_t)ch * plane] = from_f32<Tio>(v);
              }
            }
          }
        }
      }
      __syncwarp();
    }
  }
  // this warp's accumulator reads are complete: rank 0 may reuse TMEM
  tc_fence_before();
  __syncwarp();
  if (lane == 0) {
    if (rank == 0)
      mbar_arrive(tmem_empty);
    else
      mbar_arrive_cluster(mapa_shared(tmem_empty, 0));
  }
  named_bar_sync(kBarEpi, kEpiThreads);  // patches done before the slot takes V
  return run;
}

template <int M, int PM, typename Tio, bool HM, int RP = 1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairGeo<M, HM, RP>::kThreads, 1)
    wino_fused_tc_pair(const Tio *__restrict__ x, const uint8_t *__restrict__ U,
                       const float *__restrict__ bias, Tio *__restrict__ y, int C, int K, int H,
                       int W, int tiles_y, int tiles_x, int total_tiles, int relu,
                       int cs_per_split, int split, int chunk, int kb_count,
                       FastDiv fd_img, FastDiv fd_tx) {
  using L = PairLayout<M, PM, HM, RP>;
  using G = PairGeo<M, HM, RP>;
  constexpr int UP = L::P::kUParts, TD = G::TD, NF = G::NF;
  constexpr int kTiles = G::kTiles, kN = G::kN, kNU = L::kNU, kVBytes = G::kVBytes;
  constexpr int kXW = G::kXWarps;
  constexpr int kEpiThreads = 32 * kXW;
  constexpr int kUPerStage = G::NFP / kFPerU;  // weight stages per 16-channel stage (a pass)
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t v_full = sbase + L::kBarOff, v_empty = v_full + 8 * kNV;
  const uint32_t v_peer = v_empty + 8 * kNV;
  const uint32_t u_full = v_peer + 8 * kNV, u_empty = u_full + 8 * kNU;
  const uint32_t u_peer = u_empty + 8 * kNU, acc_full = u_peer + 8 * kNU;
  const uint32_t drain = acc_full + 8, tmem_empty = drain + 8;
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::kAbortSlot);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kTmemSlot);

  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);  // warp-uniform
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0: issues the MMAs
  const int C16 = (C + kCc - 1) / kCc;
  // this CTA's slice of the C_in reduction (blockIdx.z; one slice unless split)
  const int cs0 = (int)blockIdx.z * cs_per_split;
  const int nst = C16 - cs0 < cs_per_split ? C16 - cs0 : cs_per_split;
  // this pair's tiles and work items; every role walks the same sequence, and
  // the pipeline counters run on across items
  int n_items = 0;
  if (chunk == 0) {
    const int units = (total_tiles + kN - 1) / kN * kb_count;
    const int p = (int)(blockIdx.x >> 1);
    n_items = p < units ? (units - 1 - p) / (int)(gridDim.x >> 1) + 1 : 0;
  } else {
    const int lo = (int)(blockIdx.x >> 1) * chunk;
    const int hi = total_tiles - lo > chunk ? lo + chunk : total_tiles;
    n_items = lo < hi ? (hi - lo + kN - 1) / kN * kb_count : 0;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNV; ++i) {
      mbar_init(v_full + 8 * i, G::kGroupWarps);
      mbar_init(v_empty + 8 * i, 1);
      mbar_init(v_peer + 8 * i, 1);
    }
    for (int i = 0; i < kNU; ++i) {
      mbar_init(u_full + 8 * i, 1);
      mbar_init(u_empty + 8 * i, 1);
      mbar_init(u_peer + 8 * i, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    mbar_init(tmem_empty, 2 * kXW);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrival
  // Launched as a programmatic dependent launch, this CTA may have started while
  // the previous kernel of the stream was still running: nothing above touched
  // global memory, and nothing below does before that kernel has completed and
  // its writes are visible.  (Without such a launch both are no-ops.)
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- TMEM (both CTAs) + MMA issue (rank 0) / relay (rank 1) ----------
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    tc_fence_before();
    __syncwarp();
    named_bar_arrive(kBarTmem, 32 + kEpiThreads);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (rank == 0) {
      constexpr uint32_t kLo = (uint32_t)(NF * kVBytes) >> 4;  // V hi -> V lo
      const uint64_t a0 = smem_desc(sbase + L::kUOff, 128, 256);
      const uint64_t b0 = smem_desc(sbase + L::kVOff, (uint32_t)(kTiles * 16), 128);
      bool ok = true;
      int ui = 0, g = 0;
      for (int j = 0; ok && j < n_items; ++j) {
        const PairItem it = pair_item<kN>(chunk, total_tiles, kb_count, j);
        const uint32_t idesc = instr_desc(G::kMmaM, item_n(it.cnt), L::P::kF16);
        const int fb = G::f0(it.kb % G::kPasses);  // the pass's first frequency
        if (j > 0) {
          // both CTAs' epilogue warps have read item j-1's accumulators
          ok = __all_sync(0xffffffffu, mbar_wait(tmem_empty, (j - 1) & 1, abort));
          if (!ok) break;
          tc_fence_after();
        }
        for (int cs = 0; cs < nst; ++cs, ++g) {
          const int vs = g % kNV;
          ok = __all_sync(0xffffffffu, mbar_wait(v_full + 8 * vs, (g / kNV) & 1, abort) &&
                                           mbar_wait(v_peer + 8 * vs, (g / kNV) & 1, abort));
          if (!ok) break;
          tc_fence_after();
          const uint64_t bst = b0 + (uint64_t)((uint32_t)(vs * L::kVStage) >> 4);
#pragma unroll 2
          for (int fp = 0; fp < kUPerStage; ++fp, ++ui) {
            const int us = ui % kNU;
            const uint32_t ph = (ui / kNU) & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(u_full + 8 * us, ph, abort) &&
                                             mbar_wait(u_peer + 8 * us, ph, abort));
            if (!ok) break;
            tc_fence_after();
            const uint64_t ast = a0 + (uint64_t)((uint32_t)(us * L::kUStage) >> 4);
#pragma unroll
            for (int fi = 0; fi < kFPerU; ++fi) {
              const int f = fb + fp * kFPerU + fi;
              const uint64_t ah = ast + (uint64_t)((uint32_t)(fi * UP * G::kBlkBytes) >> 4);
              const uint64_t bh = bst + (uint64_t)((uint32_t)(f * kVBytes) >> 4);
              // accumulator Z[.][b], b = f % TD; its first term is the pass's
              // first row a of stage 0
              const uint32_t d = tmem + (uint32_t)((f % TD) * kN);
              const uint32_t first = (cs > 0 || f >= fb + TD) ? 1u : 0u;
              if (elect_one()) mma_pair_bf16(d, ah, bh, idesc, first);
              if (PM != kPmX1) {  // U * V_lo
                if (elect_one()) mma_pair_bf16(d, ah, bh + kLo, idesc, 1u);
              }
              if (PM == kPmX3) {  // U_lo * V_hi
                if (elect_one())
                  mma_pair_bf16(d, ah + (uint64_t)(G::kBlkBytes >> 4), bh, idesc, 1u);
              }
            }
            __syncwarp();
            if (elect_one()) tc_commit_pair(u_empty + 8 * us, 3);
            __syncwarp();
          }
          if (!ok) break;
          if (elect_one()) tc_commit_pair(v_empty + 8 * vs, 3);
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) tc_commit_pair(acc_full, 3);
        __syncwarp();
      }
      if (!ok) {
        // drain whatever was issued before giving up (the MMAs read both CTAs)
        if (elect_one()) tc_commit_pair(drain, 1);
        __syncwarp();
        const unsigned long long t0 = globaltimer();
        while (!mbar_try(drain, 0) && globaltimer() - t0 < kTimeoutNs) {
        }
      }
    } else {
      // relay, in the order rank 0 consumes them: each V stage written and each
      // weight stage landed here -> one arrival on rank 0's barrier.
      const uint32_t v_peer_r0 = mapa_shared(v_peer, 0), u_peer_r0 = mapa_shared(u_peer, 0);
      int ui = 0, g = 0;
      bool ok = true;
      for (int j = 0; ok && j < n_items; ++j) {
        for (int cs = 0; ok && cs < nst; ++cs, ++g) {
          const int vs = g % kNV;
          ok = __all_sync(0xffffffffu, mbar_wait(v_full + 8 * vs, (g / kNV) & 1, abort));
          if (!ok) break;
          if (elect_one()) mbar_arrive_cluster(v_peer_r0 + 8 * vs);
          __syncwarp();
          for (int fp = 0; fp < kUPerStage; ++fp, ++ui) {
            const int us = ui % kNU;
            ok = __all_sync(0xffffffffu, mbar_wait(u_full + 8 * us, (ui / kNU) & 1, abort));
            if (!ok) break;
            if (elect_one()) mbar_arrive_cluster(u_peer_r0 + 8 * us);
            __syncwarp();
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- producer: this CTA's weight rows by bulk copy ----------------
    int issued = 0;
    bool ok = true;
    for (int j = 0; ok && j < n_items; ++j) {
      const PairItem it = pair_item<kN>(chunk, total_tiles, kb_count, j);
      const uint8_t *ublk = U + ((size_t)it.kb * 2 + rank) * C16 * G::NFP * UP * G::kBlkBytes +
                            (size_t)cs0 * kUPerStage * L::kUStage;
      for (int q = 0; q < nst * kUPerStage; ++q) {
        const int s = issued % kNU;
        if (!__all_sync(0xffffffffu,
                        mbar_wait(u_empty + 8 * s, ((issued / kNU) & 1) ^ 1, abort))) {
          ok = false;
          break;
        }
        if (elect_one()) {
          mbar_expect_tx(u_full + 8 * s, L::kUStage);
          bulk_g2s(sbase + L::kUOff + s * L::kUStage, ublk + (size_t)q * L::kUStage,
                   L::kUStage, u_full + 8 * s);
        }
        __syncwarp();
        ++issued;
      }
    }
    for (int i = issued - kNU > 0 ? issued - kNU : 0; i < issued; ++i) {
      const int s = i % kNU;
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(u_full + 8 * s, (i / kNU) & 1) && globaltimer() - t0 < kTimeoutNs) {
      }
    }
  } else {
    // ---------------- transform warps (this CTA's tiles) + epilogues ----------------
    const int tw = warp - 2;
    const int grp = tw / G::kGroupWarps, gw = tw % G::kGroupWarps;
    // warp -> (16-tile block, K half cgrp >> 1, 4-channel quarter); lane -> (tile,
    // CPT channels).  Lanes 0-15 (the block's tiles 0-7) and lanes 16-31 (tiles
    // 8-15) take the two opposite quarters of the K half: B rows t and t + 8 share
    // a bank group, so their 4-byte V stores then land on different words and a
    // warp store fills all 32 banks once (the same quarter for all 16 tiles
    // replayed every store).  A warp load reads 8 consecutive tiles of 4 channel
    // planes.
    constexpr int CPT = G::kCpt;
    constexpr int kTileBlocks = kTiles / 16;
    const int cgrp = gw / kTileBlocks;  // 0..3
    const int cbase = (cgrp >> 1) * 8 + ((cgrp & 1) ^ (lane >> 4)) * 4 + (lane & 1) * CPT;
    const int kh = cbase >> 3;
    const int tb16 = (gw % kTileBlocks) * 16;  // first of the warp's 16 B rows
    const int t = tb16 + (lane >> 1);          // this lane's B row
    const size_t plane = (size_t)H * W;
    const int per_img = tiles_y * tiles_x;
    const int S = n_items * nst;  // every stage of every item, in order
    // Two-pixel loads need an even row length (every pair then lies inside or
    // outside the image as a whole) and x aligned to two elements.
    const bool pairs =
        ((W & 1) == 0) && ((reinterpret_cast<uintptr_t>(x) & (2 * sizeof(Tio) - 1)) == 0);

    // The lane's tile in the current item: rank r holds B rows [0, N/2) = the
    // item's tiles [r N/2, (r + 1) N/2).  A group meets each item first at its
    // stage 0 or 1.
    int cnt_cta = 0;
    unsigned vmask = 0;        // window rows (bits 0..TD-1) / columns (bits 8..) inside the image
    long long xoff = 0;        // element offset of the window's corner in x, channel 0
    auto set_item = [&](int j) {
      const PairItem it = pair_item<kN>(chunk, total_tiles, kb_count, j);
      const int half = item_n(it.cnt) >> 1;
      const int c = it.cnt - (int)rank * half;
      cnt_cta = c < 0 ? 0 : (c < half ? c : half);
      int n = 0, ty = 0, tx = 0;
      const bool tile_ok = t < cnt_cta;
      if (tile_ok) {
        const int T = it.t0 + (int)rank * half + t;
        n = tile_div<M>(T, per_img, fd_img);
        const int rem = T - n * per_img;
        ty = tile_div<M>(rem, tiles_x, fd_tx);
        tx = rem - ty * tiles_x;
      }
      const int y0 = M * ty - 1, x0 = M * tx - 1;
      xoff = (long long)n * C * (long long)plane + (long long)y0 * W + x0;
      vmask = 0;
#pragma unroll
      for (int i = 0; i < TD; ++i) {
        if (tile_ok && (y0 + i) >= 0 && (y0 + i) < H) vmask |= 1u << i;
        if ((x0 + i) >= 0 && (x0 + i) < W) vmask |= 256u << i;
      }
      // column pairs (x0 - 1 + 2p, x0 + 2p), p = 0 .. TD/2, for the pair loads
#pragma unroll
      for (int p = 0; p <= TD / 2; ++p)
        if (x0 - 1 + 2 * p >= 0 && x0 + 2 * p < W) vmask |= 65536u << p;
    };
    float d[CPT][TD][TD];  // [channel][row][col]
    // input patches of stage s; a lane whose tile is past the item's end loads
    // nothing (all-zero window mask: every load is predicated off)
    auto load_stage = [&](int s) {
      const int j = s / nst, cs = s - j * nst;
      if (cs < G::kGroups) set_item(j);
#pragma unroll
      for (int q = 0; q < CPT; ++q) {
        const int c = (cs0 + cs) * kCc + cbase + q;
        const bool cok = c < C;
        const Tio *xc = x + xoff + (long long)c * (long long)plane;
        if (pairs) {
          // TD/2 + 1 aligned two-pixel loads per window row instead of TD
#pragma unroll
          for (int i = 0; i < TD; ++i) {
            const Tio *row = xc + i * W - 1;  // column x0 - 1: even
#pragma unroll
            for (int p = 0; p <= TD / 2; ++p) {
              float a0, a1;
              ld_pair(row + 2 * p, cok && ((vmask >> i) & 1u) && ((vmask >> (16 + p)) & 1u), a0,
                      a1);
              if (p > 0) d[q][i][2 * p - 1] = a0;
              if (p < TD / 2) d[q][i][2 * p] = a1;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < TD; ++i)
#pragma unroll
            for (int j2 = 0; j2 < TD; ++j2)
              d[q][i][j2] = (cok && ((vmask >> i) & 1u) && ((vmask >> (8 + j2)) & 1u))
                                ? to_f32(xc[i * W + j2])
                                : 0.f;
        }
      }
    };
    // V of frequency f, channels cbase .. cbase+CPT-1 of row t: 2*CPT bytes per part
    const uint32_t voff = (uint32_t)(kh * (kTiles * 16) + t * 16 + (cbase & 7) * 2);
    float vmax = 0.f;  // largest |V| an fp16 layout stored (range check)
    auto put_v = [&](uint8_t *vb, int f, const float (&e)[CPT]) {
      uint32_t hi2, lo2;
      if constexpr (PM == kPmH2) {
        const __half2 h = __floats2half2_rn(e[0], e[1]);
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn(e[0] - hf.x, e[1] - hf.y);
        hi2 = *reinterpret_cast<const uint32_t *>(&h);
        lo2 = *reinterpret_cast<const uint32_t *>(&l);
        vmax = fmaxf(vmax, fmaxf(fabsf(e[0]), fabsf(e[1])));
        *reinterpret_cast<uint32_t *>(vb + (NF + f) * kVBytes + voff) = lo2;
      } else if constexpr (PM == kPmX3) {
        split_pair(e[0], e[1], hi2, lo2);
        *reinterpret_cast<uint32_t *>(vb + (NF + f) * kVBytes + voff) = lo2;
      } else {
        hi2 = pack_bf16(e[0], e[1]);
      }
      *reinterpret_cast<uint32_t *>(vb + f * kVBytes + voff) = hi2;
    };
    static_assert(CPT == 2, "two channels per transform thread");

    // Group g takes the stages s = g (mod kGroups) of the whole sequence.
    // F(2,3): the next stage's patches load while this one is transformed and
    // stored.  F(4,3): a stage's patches load before the wait for its V slot
    // (the registers are free by then), overlapping the other group's stage and
    // the MMAs.  Item e's epilogue follows the warp's last stage up to item
    // e+1's first: that stage is written ahead, so the MMAs of item e+1 start as
    // soon as the accumulators are read.
    bool ok = true;
    int ep = 0;  // next item whose epilogue this warp owes
    if constexpr (M == 2) {
      if (grp < S) load_stage(grp);
    }
    for (int s = grp; s < S; s += G::kGroups) {
      // (F(2,3): stage s's patches are already in registers, their loads having
      // overlapped the last MMAs and the epilogue)
      while (ep < n_items && s > (ep + 1) * nst)
        ok = pair_epilogue<M, PM, Tio, HM, RP>(ep++, ok, nst, smem, bias, y, K, H, W, tiles_y,
                                           tiles_x, total_tiles, chunk, kb_count, relu, split, fd_img,
                                           fd_tx) &&
             ok;
      if (!ok) break;
      const int vs = s % kNV;
      if constexpr (M != 2) load_stage(s);
      ok = __all_sync(0xffffffffu, mbar_wait(v_empty + 8 * vs, ((s / kNV) & 1) ^ 1, abort));
      if (!ok) break;
      uint8_t *vb = smem + L::kVOff + vs * L::kVStage;
      const int sn = s + G::kGroups;  // this group's next stage
      if (tb16 < cnt_cta) {
        if constexpr (M == 2) {
          float v[CPT][TD][TD];
#pragma unroll
          for (int q = 0; q < CPT; ++q) input_transform<M>(d[q], v[q]);
#pragma unroll
          for (int f = 0; f < NF; ++f) {
            float e[CPT];
#pragma unroll
            for (int q = 0; q < CPT; ++q) e[q] = v[q][f / TD][f % TD];
            put_v(vb, f, e);
          }
        } else {
          // Bt d Bt^T with the factored 6-point transform (14 operations instead
          // of 22 multiply-adds): the row pass runs in place, then each column
          // b is transformed and its six frequencies packed and stored, so two
          // 6x6 windows fit the registers.
#pragma unroll
          for (int q = 0; q < CPT; ++q)
#pragma unroll
            for (int i = 0; i < TD; ++i) {
              float w[TD];
              bt6(d[q][i], w);
#pragma unroll
              for (int b = 0; b < TD; ++b) d[q][i][b] = w[b];
            }
#pragma unroll
          for (int b = 0; b < TD; ++b) {
            float col[CPT][TD], r[CPT][TD];
#pragma unroll
            for (int q = 0; q < CPT; ++q) {
#pragma unroll
              for (int i = 0; i < TD; ++i) col[q][i] = d[q][i][b];
              bt6(col[q], r[q]);
            }
#pragma unroll
            for (int a = 0; a < TD; ++a) {
              float e[CPT];
#pragma unroll
              for (int q = 0; q < CPT; ++q) e[q] = r[q][a];
              put_v(vb, a * TD + b, e);
            }
          }
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(v_full + 8 * vs);
      // the next stage's loads go out after this stage's V stores (issuing them
      // between the transform and the stores measured 188.8 vs 180.8 us on
      // 64 images of 128->128 at 56x56)
      if constexpr (M == 2) {
        if (sn < S) load_stage(sn);
      }
    }
    while (ep < n_items)
      ok = pair_epilogue<M, PM, Tio, HM, RP>(ep++, ok, nst, smem, bias, y, K, H, W, tiles_y, tiles_x,
                                         total_tiles, chunk, kb_count, relu, split, fd_img, fd_tx) &&
           ok;
    if (n_items == 0) named_bar_sync(kBarTmem, 32 + kEpiThreads);
    if constexpr (PM == kPmH2) {
      // an input whose transform left the fp16 range made the result invalid
      if (__any_sync(0xffffffffu, !(vmax <= kF16Max)) && lane == 0)
        atomicOr(&g_tc_status, kStatusRange);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // rank 0's MMAs read both CTAs' shared memory and TMEM
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot),
                 "r"(kTmemCols));
  }
}

// bias + ReLU over y after a split reduction (fp32, in place).  blockIdx.y walks
// the (image, channel) planes, blockIdx.x strides over a plane; 16-byte accesses
// when the planes are 16-byte aligned.
__global__ void bias_relu_pass(float *__restrict__ y, const float *__restrict__ bias, int K,
                               long long plane, long long planes, int relu) {
  const long long step = (long long)gridDim.x * blockDim.x;
  const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = (plane & 3) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  for (long long pl = blockIdx.y; pl < planes; pl += gridDim.y) {
    const float b = bias ? bias[pl % K] : 0.f;
    float *p = y + (size_t)pl * plane;
    if (vec) {
      float4 *p4 = reinterpret_cast<float4 *>(p);
      for (long long i = i0; i < plane / 4; i += step) {
        float4 v = p4[i];
        v.x += b;
        v.y += b;
        v.z += b;
        v.w += b;
        if (relu) {
          v.x = v.x < 0.f ? 0.f : v.x;
          v.y = v.y < 0.f ? 0.f : v.y;
          v.z = v.z < 0.f ? 0.f : v.z;
          v.w = v.w < 0.f ? 0.f : v.w;
        }
        p4[i] = v;
      }
    } else {
      for (long long i = i0; i < plane; i += step) {
        float v = p[i] + b;
        if (relu) v = v < 0.f ? 0.f : v;
        p[i] = v;
      }
    }
  }
}

// bias_relu_pass over n*k planes of h*w floats: one grid row per plane (up to
// 65535), the columns capped so that the grid stays near 8 CTAs per SM.
static cudaError_t launch_bias_relu(float *y, const float *bias, int n, int k, int h, int w,
                                    int relu, int sms, cudaStream_t s) {
  cwgk_count_launch();
  const long long plane = (long long)h * w, planes = (long long)n * k;
  const unsigned gy = (unsigned)(planes < 65535 ? planes : 65535);
  long long bx = (plane / 4 + 255) / 256;
  if (bx < 1) bx = 1;
  if (bx * gy > 8LL * sms) bx = (8LL * sms + gy - 1) / gy;
  bias_relu_pass<<<dim3((unsigned)bx, gy), 256, 0, s>>>(y, bias, k, plane, planes, relu);
  return cudaGetLastError();
}

// C_in slices for a layer whose CTA pairs would leave three quarters of the TPCs
// idle: one slice per idle TPC, down to one 16-channel stage per slice.  1 = no
// split.  (Above that occupancy the extra zeroing, atomics and bias pass cost
// more than the shorter C_in loop saves.  One-stage slices rather than two:
// resnet18's 13 stride-1 layers at N=1, one CUDA graph, 248.7 -> 226.0 us.)
template <int M, bool HM, int RP = 1>
static int split_stages(int n, int c, int k, int h, int w, int tpcs, int *per) {
  using G = PairGeo<M, HM, RP>;
  const int C16 = (c + kCc - 1) / kCc;
  const long long tiles = (long long)n * ((h + M - 1) / M) * ((w + M - 1) / M);
  const long long items =
      (tiles + G::kN - 1) / G::kN * ((k + G::kCoutCta - 1) / G::kCoutCta) * G::kPasses;
  *per = C16;
  if (4 * items > tpcs || C16 < 2) return 1;
  long long s = tpcs / items;
  if (s > C16) s = C16;
  if (s < 2) return 1;
  *per = (C16 + (int)s - 1) / (int)s;
  return (C16 + *per - 1) / *per;
}

// Clusters of a pair kernel that fit on the device at once, cached per device
// (a TPC whose two SMs are not both free cannot take a pair).
template <auto Kernel>
static int resident_pairs(int threads, int smem, int sms) {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return sms / 2;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(sms / 2 * 2), 1, 1);
  cfg.blockDim = dim3((unsigned)threads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (const void *)Kernel, &cfg) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    n = sms / 2;
  }
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Work split of a pair launch: pairs, chunk (0: round robin), grid rows,
// output-channel blocks per pair.  Up to one wave of (tile block, channel block)
// units, or a split C_in: one unit per pair.  More: one pair per resident
// cluster, in whichever of the two persistent orders costs less by a simple
// model of an item's time: a share kFixed (weight stream, A operand reads,
// epilogue) that does not shrink with the item's tiles, the rest in proportion;
// plus a prologue (kPrologue of an item) that only the first item pays.
struct PairPlan {
  long long pairs, chunk;
  int gy, kb_count;
  int order;  // CWG_ORDER_*
};
template <int M, bool HM>
static PairPlan plan_pairs(long long total, int gy, int splits, int resident) {
  using G = PairGeo<M, HM>;
  constexpr double kFixed = M == 2 ? 0.5 : 0.75, kPrologue = 0.1;
  const long long blocks = (total + G::kN - 1) / G::kN, units = blocks * gy;
  PairPlan p{blocks, G::kN, gy, 1, CWG_ORDER_GRID};
  if (splits > 1 || resident <= 0) return p;
  // one wave of whole units: one item per pair
  const double grid = units <= resident ? 1.0 + kPrologue : 1e300;
  // round robin: every pair takes ceil(units / resident) whole units at most
  const double rr = units > resident ? (double)((units + resident - 1) / resident) + kPrologue
                                     : 1e300;
  // equal runs of tiles over every resident pair: whole items plus one short item
  // per channel block (a layer of less than one wave of full items then runs
  // shorter items on more pairs: 8 images of 128->128 at 56x56, 49 blocks of 128
  // tiles, run as 66 items of 96 tiles)
  // runs start on a multiple of 16 tiles: a lane's pixels then stay in one image
  // row and aligned for a vector store whenever the row holds an even number of tiles
  const long long chunk = ((total + resident - 1) / resident + 15) / 16 * 16;
  const long long full = chunk / G::kN, rem = chunk % G::kN;
  const double eq =
      (double)gy * ((double)full + (rem ? kFixed + (1 - kFixed) * (double)rem / G::kN : 0.0)) +
      kPrologue;
  if (grid <= eq && grid <= rr) return p;
  if (eq < rr) {
    p.chunk = chunk;
    p.pairs = (total + chunk - 1) / chunk;
    p.order = CWG_ORDER_RUNS;
  } else {
    p.chunk = 0;
    p.pairs = resident;
    p.order = CWG_ORDER_ROUND;
  }
  p.gy = 1;
  p.kb_count = gy;
  return p;
}

template <int M, int PM, typename Tio, bool HM, int RP = 1>
static cudaError_t launch_pair(const void *x, const void *U, const float *bias, void *y, int n,
                               int c, int k, int h, int w, int relu, int allow_split,
                               int allow_pdl, cudaStream_t s) {
  using G = PairGeo<M, HM, RP>;
  using L = PairLayout<M, PM, HM, RP>;
  const int tiles_y = (h + M - 1) / M, tiles_x = (w + M - 1) / M;
  const long long total = (long long)n * tiles_y * tiles_x;
  const int gy = (k + G::kCoutCta - 1) / G::kCoutCta * G::kPasses;  // (channel block, pass)
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  int per = (c + kCc - 1) / kCc;
  const int splits = (allow_split && sizeof(Tio) == 4) ? split_stages<M, HM, RP>(n, c, k, h, w, sms / 2,
                                                                         &per)
                                                       : 1;
  auto fn = wino_fused_tc_pair<M, PM, Tio, HM, RP>;
  e = smem_attr_once<wino_fused_tc_pair<M, PM, Tio, HM, RP>>(L::kSmem);
  if (e != cudaSuccess) return e;
  const int resident =
      resident_pairs<wino_fused_tc_pair<M, PM, Tio, HM, RP>>(G::kThreads, L::kSmem, sms);
  const PairPlan plan = plan_pairs<M, HM>(total, gy, splits, resident);
  // tile indices, item counts and units are 32-bit in the kernel
  if (total * gy > 0x7fffffffLL || 2 * plan.pairs > 0x7fffffffLL || plan.gy > 65535)
    return cudaErrorInvalidValue;
  const size_t ybytes = (size_t)n * k * h * w * sizeof(Tio);
  if (splits > 1 && (e = cudaMemsetAsync(y, 0, ybytes, s)) != cudaSuccess) return e;
  // Programmatic dependent launch: the pair's CTAs may become resident while the
  // previous kernel in the stream drains (they set up barriers and TMEM, then
  // wait for its completion before any global access).  After a memset (split
  // layers) the launch is an ordinary one.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * plan.pairs), (unsigned)plan.gy, (unsigned)splits);
  cfg.blockDim = dim3((unsigned)G::kThreads);
  cfg.dynamicSmemBytes = (size_t)L::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (allow_pdl && splits == 1) ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, fn, (const Tio *)x, (const uint8_t *)U, bias, (Tio *)y, c, k, h, w,
                         tiles_y, tiles_x, (int)total, relu, per, (int)(splits > 1),
                         (int)plan.chunk, plan.kb_count,
                         fast_div((uint32_t)(tiles_y * tiles_x)), fast_div((uint32_t)tiles_x));
  if (e != cudaSuccess || (e = cudaGetLastError()) != cudaSuccess || splits == 1) return e;
  if (relu) e = launch_bias_relu((float *)y, bias, n, k, h, w, relu, sms, s);
  return e;
}

// The launch plan of a layer as launch_pair would make it on the current device
// (without one: `sms` SMs and one cluster per TPC).
template <int M, int PM, typename Tio, bool HM, int RP = 1>
static void plan_layer(int n, int c, int k, int h, int w, int allow_split, int sms,
                       long long *ctas, int *order) {
  using G = PairGeo<M, HM, RP>;
  using L = PairLayout<M, PM, HM, RP>;
  const long long total = (long long)n * ((h + M - 1) / M) * ((w + M - 1) / M);
  const int gy = (k + G::kCoutCta - 1) / G::kCoutCta * G::kPasses;  // (channel block, pass)
  int per = 0;
  const int splits =
      (allow_split && sizeof(Tio) == 4) ? split_stages<M, HM, RP>(n, c, k, h, w, sms / 2, &per) : 1;
  int resident = sms / 2, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess &&
      smem_attr_once<wino_fused_tc_pair<M, PM, Tio, HM, RP>>(L::kSmem) == cudaSuccess)
    resident = resident_pairs<wino_fused_tc_pair<M, PM, Tio, HM, RP>>(G::kThreads, L::kSmem, sms);
  else
    (void)cudaGetLastError();
  const PairPlan p = plan_pairs<M, HM>(total, gy, splits, resident);
  *ctas = 2 * p.pairs * p.gy * splits;
  *order = p.order;
}

// ==== batched per-frequency GEMM of the non-fused ablation ===========================
//
// M_f[k][t] = sum_c U_f[k][c] V_f[c][t] for every frequency f, fp32 results in HBM
// ([f][K][T], t contiguous), on the tensor cores with the fp32-parity products of
// the fused kernels (bf16 hi/lo split, three MMAs per 16-channel step).  Both
// operands arrive in HBM as ready-made UMMA blocks of 128 rows x 16 channels
// (the blk_off layout, hi and lo blocks adjacent):
//   A: Ug [nf][Kp/128][C16][hi, lo][4096 B]   rows = output channels
//   B: Vg [nf][Tp/128][C16][hi, lo][4096 B]   rows = tiles
// One CTA per (128-tile block, 128-channel block, frequency): warp 0 owns 128
// TMEM columns and issues the MMAs, warp 1 streams the 16 KB stages by
// cp.async.bulk, warps 2-5 read the accumulator (lane = output channel) and
// store rows of M.  Every wait is bounded, as in the fused kernels.
constexpr int kGemmStages = 4;
constexpr int kGemmStage = 4 * kCoreBytes;  // A hi, A lo, B hi, B lo
constexpr int kGemmThreads = 6 * 32;
constexpr int kGemmBarOff = kGemmStages * kGemmStage;
// full[stages], empty[stages], acc_full, drain; then the TMEM slot and abort flag
constexpr int kGemmSmem = kGemmBarOff + 8 * (2 * kGemmStages + 2) + 8;

__global__ void __launch_bounds__(kGemmThreads)
    gemm_freq_x3(const uint8_t *__restrict__ Ug, const uint8_t *__restrict__ Vg,
                 float *__restrict__ Mf, int K, int T, int C16, int Kb, int Tb) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t full = sbase + kGemmBarOff, empty = full + 8 * kGemmStages;
  const uint32_t acc_full = empty + 8 * kGemmStages, drain = acc_full + 8;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kGemmBarOff + 8 * (2 * kGemmStages + 2));
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  const int tb = blockIdx.x, kb = blockIdx.y, f = blockIdx.z;
  const uint8_t *a_src = Ug + ((size_t)f * Kb + kb) * C16 * 2 * kCoreBytes;
  const uint8_t *b_src = Vg + ((size_t)f * Tb + tb) * C16 * 2 * kCoreBytes;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGemmStages; ++i) {
      mbar_init(full + 8 * i, 1);
      mbar_init(empty + 8 * i, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(128));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    tc_fence_before();
    __syncwarp();
    named_bar_arrive(kBarTmem, 32 + 4 * 32);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t idesc = instr_desc(128, 128);
    constexpr uint64_t kBlk = (uint64_t)(kCoreBytes >> 4);
    bool ok = true;
    for (int cs = 0; cs < C16; ++cs) {
      const int st = cs % kGemmStages;
      ok = __all_sync(0xffffffffu, mbar_wait(full + 8 * st, (cs / kGemmStages) & 1, abort));
      if (!ok) break;
      tc_fence_after();
      const uint64_t a = smem_desc(sbase + st * kGemmStage, 128, 256);
      const uint64_t b = a + 2 * kBlk;
      if (elect_one()) mma_bf16(tmem, a, b, idesc, cs > 0 ? 1u : 0u);  // hi * hi
      if (elect_one()) mma_bf16(tmem, a, b + kBlk, idesc, 1u);         // hi * lo
      if (elect_one()) mma_bf16(tmem, a + kBlk, b, idesc, 1u);         // lo * hi
      __syncwarp();
      if (elect_one()) tc_commit(empty + 8 * st);
      __syncwarp();
    }
    if (ok) {
      if (elect_one()) tc_commit(acc_full);
      __syncwarp();
    } else {
      if (elect_one()) tc_commit(drain);
      __syncwarp();
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(drain, 0) && globaltimer() - t0 < kTimeoutNs) {
      }
    }
  } else if (warp == 1) {
    int issued = 0;
    for (int cs = 0; cs < C16; ++cs) {
      const int st = cs % kGemmStages;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(empty + 8 * st, ((cs / kGemmStages) & 1) ^ 1, abort)))
        break;
      if (elect_one()) {
        mbar_expect_tx(full + 8 * st, kGemmStage);
        bulk_g2s(sbase + st * kGemmStage, a_src + (size_t)cs * 2 * kCoreBytes, 2 * kCoreBytes,
                 full + 8 * st);
        bulk_g2s(sbase + st * kGemmStage + 2 * kCoreBytes, b_src + (size_t)cs * 2 * kCoreBytes,
                 2 * kCoreBytes, full + 8 * st);
      }
      __syncwarp();
      issued = cs + 1;
    }
    // never leave the CTA with a copy still writing shared memory
    for (int i = issued - kGemmStages > 0 ? issued - kGemmStages : 0; i < issued; ++i) {
      const int st = i % kGemmStages;
      const unsigned long long t0 = globaltimer();
      while (!mbar_try(full + 8 * st, (i / kGemmStages) & 1) && globaltimer() - t0 < kTimeoutNs) {
      }
    }
  } else {
    // epilogue: TMEM lanes 32 quad .. 32 quad + 31 = output channels, columns = tiles
    named_bar_sync(kBarTmem, 32 + 4 * 32);
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort));
    tc_fence_after();
    if (ok) {
      const int quad = warp & 3;
      const int k = kb * 128 + quad * 32 + lane;
      const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
      float *row = Mf + ((size_t)f * K + (k < K ? k : 0)) * (size_t)T;
      const bool vec = (T & 3) == 0 && (reinterpret_cast<uintptr_t>(Mf) & 15) == 0;
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 8) {
        float v[8];
        tmem_ld8(trow + (uint32_t)c0, v);  // whole warp, converged
        tmem_wait_ld();
        const int t0 = tb * 128 + c0;
        if (k < K && t0 < T) {
          if (vec && t0 + 8 <= T) {
            *reinterpret_cast<float4 *>(row + t0) = make_float4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<float4 *>(row + t0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (t0 + e < T) row[t0 + e] = v[e];
          }
        }
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot),
                 "r"(128));
  }
}

// U in the CUDA-core layout, fp32 [nf][C][K] -> Ug blocks (hi, lo); zero past C, K.
__global__ void gemm_u_blocks(const float *__restrict__ U, uint8_t *__restrict__ Ug, int nf, int C,
                              int K, int C16, int Kb) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long Kp = (long long)Kb * 128, Cp = (long long)C16 * 16;
  if (idx >= (long long)nf * Cp * Kp) return;
  const int k = (int)(idx % Kp);
  const int c = (int)((idx / Kp) % Cp);
  const int f = (int)(idx / (Kp * Cp));
  const float u = (k < K && c < C) ? U[((size_t)f * C + c) * K + k] : 0.f;
  const __nv_bfloat16 hi = __float2bfloat16_rn(u);
  const __nv_bfloat16 lo = __float2bfloat16_rn(u - __bfloat162float(hi));
  uint8_t *blk = Ug + ((((size_t)f * Kb + k / 128) * C16 + c / 16) * 2) * kCoreBytes;
  const uint32_t off = blk_off(k % 128, c % 16);
  *reinterpret_cast<__nv_bfloat16 *>(blk + off) = hi;
  *reinterpret_cast<__nv_bfloat16 *>(blk + kCoreBytes + off) = lo;
}

// Input pass of the ablation for the tensor-core GEMM (F(2,3)): V = Bt d B of one
// tile and 8 input channels, written as hi/lo bf16 into the Vg blocks -- per
// frequency one 16-byte row of each block, so that consecutive threads (tiles)
// fill consecutive rows; zero past C and T (the blocks cover the padded ranges,
// so no memset is needed).
__global__ void __launch_bounds__(128)
    gemm_v_blocks(const float *__restrict__ x, uint8_t *__restrict__ Vg, int C, int H, int W,
                  int tiles_y, int tiles_x, int T, int C16, int Tb) {
  constexpr int NF = 16;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long Tp = (long long)Tb * 128;
  if (idx >= (long long)C16 * 2 * Tp) return;
  const int t = (int)(idx % Tp);
  const int c8 = (int)(idx / Tp);  // 8-channel group: channels 8 c8 .. 8 c8 + 7
  const int per_img = tiles_y * tiles_x;
  const bool tok = t < T;
  const int n = tok ? t / per_img : 0;
  const int rem = tok ? t - n * per_img : 0;
  const int ty = rem / tiles_x, tx = rem - ty * tiles_x;
  const int y0 = 2 * ty - 1, x0 = 2 * tx - 1;
  uint32_t hi[NF][4], lo[NF][4];  // per frequency: 8 channels as 4 bf16 pairs
#pragma unroll
  for (int q2 = 0; q2 < 4; ++q2) {
    float v[2][4][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = 8 * c8 + 2 * q2 + h;
      const bool ok = tok && c < C;
      const float *xc = x + ((size_t)n * C + (ok ? c : 0)) * H * W;
      float d[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int yy = y0 + i, xx = x0 + j;
          d[i][j] =
              (ok && yy >= 0 && yy < H && xx >= 0 && xx < W) ? xc[(size_t)yy * W + xx] : 0.f;
        }
      input_transform<2, true>(d, v[h]);
    }
#pragma unroll
    for (int f = 0; f < NF; ++f)
      split_pair(v[0][f / 4][f % 4], v[1][f / 4][f % 4], hi[f][q2], lo[f][q2]);
  }
  // row t of the block (t / 128, c8 / 2), K half c8 % 2: 8-row groups 256 B apart,
  // K halves 128 B apart, rows 16 B apart (blk_off)
  const uint32_t off = blk_off(t % 128, (c8 % 2) * 8);
#pragma unroll
  for (int f = 0; f < NF; ++f) {
    uint8_t *blk = Vg + ((((size_t)f * Tb + t / 128) * C16 + c8 / 2) * 2) * kCoreBytes;
    *reinterpret_cast<uint4 *>(blk + off) = make_uint4(hi[f][0], hi[f][1], hi[f][2], hi[f][3]);
    *reinterpret_cast<uint4 *>(blk + kCoreBytes + off) =
        make_uint4(lo[f][0], lo[f][1], lo[f][2], lo[f][3]);
  }
}

// Diagnostics: one CTA waits, through the kernels' own bounded wait, on an
// mbarrier that nothing ever arrives on.  After kTimeoutNs the wait gives up,
// sets g_tc_status and the kernel returns: the host sees CWG_ETIMEOUT and the
// context stays usable.  No spin is unbounded and nothing faults.
__global__ void wait_selftest() {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  (void)mbar_wait(smem_u32(&bar), 0, &abort_flag);
}

}  // namespace tc
}  // namespace cwg

using namespace cwg;

extern "C" {

int cwgk_tc_get_cfg(int pm, int variant, int m, cwgk_tc_cfg *out) {
  using namespace tc;
  if (!out || pm < kPmX1 || pm > kPmX3) return -1;
  const bool x3 = pm == kPmX3;
  out->m = m;
  out->kb = tc::kCout;
  out->cc = tc::kCc;
  out->tmem_cols = tc::kTmemCols;
  if (variant == CWGK_TC_PAIR) {
    if (m == 2 && pm != kPmH2) {  // fp16 products serve the F(4,3) layers only
      out->tiles = PairGeo<2>::kN;
      out->kb = PairGeo<2>::kCoutCta;
      out->threads = PairGeo<2>::kThreads;
      out->smem = x3 ? PairLayout<2, kPmX3>::kSmem : PairLayout<2, kPmX1>::kSmem;
    } else if (m == 4) {
      out->tiles = PairGeo<4>::kN;
      out->kb = PairGeo<4>::kCoutCta;
      out->threads = PairGeo<4>::kThreads;
      out->smem = pm == kPmX3 ? PairLayout<4, kPmX3>::kSmem
                              : (pm == kPmH2 ? PairLayout<4, kPmH2>::kSmem
                                             : PairLayout<4, kPmX1>::kSmem);
    } else {
      return -1;
    }
    // a CTA pair per (tile block, channel block, pass of output rows)
    out->ctas_per_tile_block = 2 * (m == 4 ? PairGeo<4>::kPasses : PairGeo<2>::kPasses);
    return 0;
  }
  if (variant == CWGK_TC_PAIR64 && m == 4) {  // two output rows x 64 channels per CTA
    using G4 = PairGeo<4, false, 2>;
    out->tiles = G4::kN;
    out->kb = G4::kCoutCta;
    out->threads = G4::kThreads;
    out->smem = pm == kPmX3 ? PairLayout<4, kPmX3, false, 2>::kSmem
                            : (pm == kPmH2 ? PairLayout<4, kPmH2, false, 2>::kSmem
                                           : PairLayout<4, kPmX1, false, 2>::kSmem);
    out->ctas_per_tile_block = 2 * G4::kPasses;
    return 0;
  }
  if (pm == kPmH2) return -1;
  if (variant == CWGK_TC_PAIR64) {
    if (m != 2) return -1;
    out->tiles = PairGeo<2, true>::kN;
    out->kb = PairGeo<2, true>::kCoutCta;
    out->threads = PairGeo<2, true>::kThreads;
    out->smem = x3 ? PairLayout<2, kPmX3, true>::kSmem : PairLayout<2, kPmX1, true>::kSmem;
    out->ctas_per_tile_block = 2;
    return 0;
  }
  if (m != 2) return -1;
  switch (variant) {
    case CWGK_TC_HALF:
      out->tiles = tc::Geo<true>::kTiles;
      out->threads = tc::Geo<true>::kThreads;
      out->smem = x3 ? tc::Layout<true, true>::kSmem : tc::Layout<false, true>::kSmem;
      out->ctas_per_tile_block = 1;
      return 0;
    case CWGK_TC_FULL16:
      out->tiles = tc::Geo<false>::kTiles;
      out->threads = tc::Geo<false>::kThreads;
      out->smem = x3 ? tc::Layout<true, false>::kSmem : tc::Layout<false, false>::kSmem;
      out->ctas_per_tile_block = 1;
      return 0;
    default: return -1;
  }
}

int cwgk_weight_transform_tc(const float *src, void *U, int c_in, int c_out, int m, int layout,
                             int from_ref, void *stream) {
  // TC2H: 64 output channels per CTA (F(2,3): M = 128 pair; F(4,3): two rows x 64)
  const bool half = layout == CWGK_LAYOUT_TC2H_X3 || layout == CWGK_LAYOUT_TC2H_X1 ||
                    layout == CWGK_LAYOUT_TC2H_H2;
  const bool h2 = layout == CWGK_LAYOUT_TC2_H2 || layout == CWGK_LAYOUT_TC2H_H2;
  const bool pair = half || h2 || layout == CWGK_LAYOUT_TC2_X3 || layout == CWGK_LAYOUT_TC2_X1;
  const bool x3 = layout == CWGK_LAYOUT_TC_X3 || layout == CWGK_LAYOUT_TC2_X3 ||
                  layout == CWGK_LAYOUT_TC2H_X3;
  if (!(m == 2 || (m == 4 && pair))) return -2;
  if (h2 && m != 4) return -2;
  if (!pair && layout != CWGK_LAYOUT_TC_X1 && layout != CWGK_LAYOUT_TC_X3) return -2;
  const int kb = half ? (m == 4 ? tc::PairGeo<4, false, 2>::kCoutCta
                                : tc::PairGeo<2, true>::kCoutCta)
                      : (pair ? (m == 2 ? tc::PairGeo<2>::kCoutCta : tc::PairGeo<4>::kCoutCta)
                              : tc::kCout);
  const int Cp = (c_in + tc::kCc - 1) / tc::kCc * tc::kCc;
  const int Kp = (c_out + kb - 1) / kb * kb;
  const long total = (long)Cp * Kp;
  const int threads = 256;
  const unsigned blocks = (unsigned)((total + threads - 1) / threads);
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t *u = (uint8_t *)U;
#define CWG_WT(KERNEL) KERNEL<<<blocks, threads, 0, s>>>(src, u, c_in, c_out, Cp, Kp, from_ref)
  if (!pair) {
    if (x3)
      CWG_WT(tc::wt_transform_tc<true>);
    else
      CWG_WT(tc::wt_transform_tc<false>);
  } else if (half && m == 4) {
    if (x3)
      CWG_WT((tc::wt_transform_tc_pair<4, tc::kPmX3, false, 2>));
    else if (h2)
      CWG_WT((tc::wt_transform_tc_pair<4, tc::kPmH2, false, 2>));
    else
      CWG_WT((tc::wt_transform_tc_pair<4, tc::kPmX1, false, 2>));
  } else if (half) {
    if (x3)
      CWG_WT((tc::wt_transform_tc_pair<2, tc::kPmX3, true>));
    else
      CWG_WT((tc::wt_transform_tc_pair<2, tc::kPmX1, true>));
  } else if (m == 2) {
    if (x3)
      CWG_WT((tc::wt_transform_tc_pair<2, tc::kPmX3, false>));
    else
      CWG_WT((tc::wt_transform_tc_pair<2, tc::kPmX1, false>));
  } else {
    if (x3)
      CWG_WT((tc::wt_transform_tc_pair<4, tc::kPmX3, false>));
    else if (h2)
      CWG_WT((tc::wt_transform_tc_pair<4, tc::kPmH2, false>));
    else
      CWG_WT((tc::wt_transform_tc_pair<4, tc::kPmX1, false>));
  }
#undef CWG_WT
  cwgk_count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return -3;
  }
  return 0;
}

int cwgk_bias_relu(float *y, const float *bias, int n, int c_out, int h, int w, int relu,
                   void *stream) {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = tc::launch_bias_relu(y, bias, n, c_out, h, w, relu, sms, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return -3;
  }
  return 0;
}

int cwgk_tc_splits(int n, int c_in, int c_out, int h, int w, int m, int variant, int bf16,
                   int allow_split, int sms) {
  int per = 0;
  if ((variant != CWGK_TC_PAIR && variant != CWGK_TC_PAIR64) || bf16 || !allow_split) return 1;
  if (variant == CWGK_TC_PAIR64)
    return m == 2 ? tc::split_stages<2, true>(n, c_in, c_out, h, w, sms / 2, &per) : 1;
  return m == 2 ? tc::split_stages<2, false>(n, c_in, c_out, h, w, sms / 2, &per)
                : tc::split_stages<4, false>(n, c_in, c_out, h, w, sms / 2, &per);
}

int cwgk_tc_plan(int n, int c_in, int c_out, int h, int w, int m, int pm, int variant, int bf16,
                 int allow_split, int sms, long long *ctas, int *order) {
  using namespace tc;
  if (!((variant == CWGK_TC_PAIR || variant == CWGK_TC_PAIR64) && (m == 2 || m == 4)))
    return -1;
  if (pm == kPmH2 && !(m == 4 && bf16)) return -1;
#define CWG_PLAN(M_, PM_, T_, HM_) \
  plan_layer<M_, PM_, T_, HM_>(n, c_in, c_out, h, w, allow_split, sms, ctas, order)
  const bool x3 = pm == kPmX3;
  if (variant == CWGK_TC_PAIR64 && m == 4) {  // bf16 layers only
    if (!bf16) return -1;
    if (pm == kPmH2)
      plan_layer<4, kPmH2, __nv_bfloat16, false, 2>(n, c_in, c_out, h, w, allow_split, sms,
                                                     ctas, order);
    else if (x3)
      plan_layer<4, kPmX3, __nv_bfloat16, false, 2>(n, c_in, c_out, h, w, allow_split, sms,
                                                     ctas, order);
    else
      plan_layer<4, kPmX1, __nv_bfloat16, false, 2>(n, c_in, c_out, h, w, allow_split, sms,
                                                     ctas, order);
  } else if (variant == CWGK_TC_PAIR64) {
    if (bf16)
      x3 ? CWG_PLAN(2, kPmX3, __nv_bfloat16, true) : CWG_PLAN(2, kPmX1, __nv_bfloat16, true);
    else
      x3 ? CWG_PLAN(2, kPmX3, float, true) : CWG_PLAN(2, kPmX1, float, true);
  } else if (m == 2) {
    if (bf16)
      x3 ? CWG_PLAN(2, kPmX3, __nv_bfloat16, false) : CWG_PLAN(2, kPmX1, __nv_bfloat16, false);
    else
      x3 ? CWG_PLAN(2, kPmX3, float, false) : CWG_PLAN(2, kPmX1, float, false);
  } else if (pm == kPmH2) {
    CWG_PLAN(4, kPmH2, __nv_bfloat16, false);
  } else {
    if (bf16)
      x3 ? CWG_PLAN(4, kPmX3, __nv_bfloat16, false) : CWG_PLAN(4, kPmX1, __nv_bfloat16, false);
    else
      x3 ? CWG_PLAN(4, kPmX3, float, false) : CWG_PLAN(4, kPmX1, float, false);
  }
#undef CWG_PLAN
  return 0;
}

int cwgk_conv_tc(const void *x, const void *U, const float *bias, void *y, int n, int c_in,
                 int c_out, int h, int w, int m, int pm, int variant, int bf16, int relu,
                 int allow_split, int allow_pdl, void *stream) {
  using tc::kPmH2;
  using tc::kPmX1;
  using tc::kPmX3;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  const bool x3 = pm == kPmX3;
#define CWG_TC_LAUNCH(X3_, HALF_)                                                              \
  (bf16 ? tc::launch<X3_, HALF_, __nv_bfloat16>(x, U, bias, y, n, c_in, c_out, h, w, relu, s) \
        : tc::launch<X3_, HALF_, float>(x, U, bias, y, n, c_in, c_out, h, w, relu, s))
#define CWG_TC_LAUNCH_PAIR(M_, PM_, HM_)                                                        \
  (bf16 ? tc::launch_pair<M_, PM_, __nv_bfloat16, HM_>(x, U, bias, y, n, c_in, c_out, h, w,   \
                                                        relu, allow_split, allow_pdl, s)      \
        : tc::launch_pair<M_, PM_, float, HM_>(x, U, bias, y, n, c_in, c_out, h, w, relu,     \
                                               allow_split, allow_pdl, s))
  if (variant == CWGK_TC_PAIR64 && m == 4) {  // bf16 F(4,3), two rows x 64 channels per CTA
    if (!bf16) return -2;
    if (pm == kPmH2)
      e = tc::launch_pair<4, kPmH2, __nv_bfloat16, false, 2>(x, U, bias, y, n, c_in, c_out, h, w,
                                                             relu, allow_split, allow_pdl, s);
    else if (x3)
      e = tc::launch_pair<4, kPmX3, __nv_bfloat16, false, 2>(x, U, bias, y, n, c_in, c_out, h, w,
                                                             relu, allow_split, allow_pdl, s);
    else
      e = tc::launch_pair<4, kPmX1, __nv_bfloat16, false, 2>(x, U, bias, y, n, c_in, c_out, h, w,
                                                             relu, allow_split, allow_pdl, s);
  } else if (pm == kPmH2) {  // bf16 F(4,3) layers only
    if (!(variant == CWGK_TC_PAIR && m == 4 && bf16)) return -2;
    e = tc::launch_pair<4, kPmH2, __nv_bfloat16, false>(x, U, bias, y, n, c_in, c_out, h, w,
                                                        relu, allow_split, allow_pdl, s);
  } else if (variant == CWGK_TC_PAIR && m == 2)
    e = x3 ? CWG_TC_LAUNCH_PAIR(2, kPmX3, false) : CWG_TC_LAUNCH_PAIR(2, kPmX1, false);
  else if (variant == CWGK_TC_PAIR64 && m == 2)
    e = x3 ? CWG_TC_LAUNCH_PAIR(2, kPmX3, true) : CWG_TC_LAUNCH_PAIR(2, kPmX1, true);
  else if (variant == CWGK_TC_PAIR && m == 4)
    e = x3 ? CWG_TC_LAUNCH_PAIR(4, kPmX3, false) : CWG_TC_LAUNCH_PAIR(4, kPmX1, false);
  else if (variant == CWGK_TC_HALF && m == 2)
    e = x3 ? CWG_TC_LAUNCH(true, true) : CWG_TC_LAUNCH(false, true);
  else if (variant == CWGK_TC_FULL16 && m == 2)
    e = x3 ? CWG_TC_LAUNCH(true, false) : CWG_TC_LAUNCH(false, false);
  else
    return -2;
#undef CWG_TC_LAUNCH
#undef CWG_TC_LAUNCH_PAIR
  cwgk_count_launch();
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return -3;
  }
  return 0;
}

size_t cwgk_gemm_blocks_bytes(int nf, int rows, int c_in) {
  return (size_t)nf * ((rows + 127) / 128) * ((c_in + 15) / 16) * 2 * tc::kCoreBytes;
}

int cwgk_gemm_prepare(const float *U, void *Ug, const float *x, void *Vg, int m, int n, int c_in,
                      int c_out, int h, int w, void *stream) {
  cudaStream_t s = (cudaStream_t)stream;
  if (m != 2) return -2;  // the tensor-core ablation serves F(2,3) layers
  const int nf = (m + 2) * (m + 2);
  const int tiles_y = (h + m - 1) / m, tiles_x = (w + m - 1) / m;
  const long long T = (long long)n * tiles_y * tiles_x;
  if (T > 0x7fffffffLL - 128) return -2;
  const int C16 = (c_in + 15) / 16, Kb = (c_out + 127) / 128, Tb = (int)((T + 127) / 128);
  const int threads = 256;
  const long long nu = (long long)nf * C16 * 16 * Kb * 128;
  tc::gemm_u_blocks<<<(unsigned)((nu + threads - 1) / threads), threads, 0, s>>>(
      U, (uint8_t *)Ug, nf, c_in, c_out, C16, Kb);
  cwgk_count_launch();
  const long long nv = (long long)C16 * 2 * Tb * 128;
  const unsigned bv = (unsigned)((nv + 127) / 128);
  tc::gemm_v_blocks<<<bv, 128, 0, s>>>(x, (uint8_t *)Vg, c_in, h, w, tiles_y, tiles_x, (int)T,
                                        C16, Tb);
  cwgk_count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return -3;
  }
  return 0;
}

int cwgk_gemm_x3(const void *Ug, const void *Vg, float *Mf, int nf, int c_in, int c_out, int T,
                 void *stream) {
  const int C16 = (c_in + 15) / 16, Kb = (c_out + 127) / 128, Tb = (T + 127) / 128;
  if (Kb > 65535 || nf > 65535) return -2;
  cudaError_t e = smem_attr_once<tc::gemm_freq_x3>(tc::kGemmSmem);
  if (e == cudaSuccess) {
    tc::gemm_freq_x3<<<dim3((unsigned)Tb, (unsigned)Kb, (unsigned)nf), tc::kGemmThreads,
                       tc::kGemmSmem, (cudaStream_t)stream>>>(
        (const uint8_t *)Ug, (const uint8_t *)Vg, Mf, c_out, T, C16, Kb, Tb);
    cwgk_count_launch();
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return -3;
  }
  return 0;
}

int cwg_selftest_wait_timeout(void *stream) {
  tc::wait_selftest<<<1, 32, 0, (cudaStream_t)stream>>>();
  cwgk_count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return CWG_ECUDA;
  }
  return CWG_OK;
}

int cwgk_read_clear_status(unsigned *status) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tc::g_tc_status, sizeof(v));
  if (e == cudaSuccess && v) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(tc::g_tc_status, &zero, sizeof(zero));
  }
  if (e != cudaSuccess) {
    cwgk_set_cuda_error((int)e);
    return -3;
  }
  *status = v;
  return 0;
}

}  // extern "C"
