// Fused NVFP4 quantiser: fp16 activations -> e2m1 codes + e4m3 block scales,
// the scales written directly in the 128x4 blocked layout that the tcgen05
// GEMMs read (no separate swizzle pass).
//
// Per 16-element block of a row (global scale 1.0):
//   amax  = max |x_i|                                   (exact in f32)
//   s     = e4m3(amax / 6)   round-to-nearest-even, saturating at 448
//   inv   = 1 / s            one IEEE f32 division per block
//   q_i   = e2m1(x_i * inv)  f32 product, then round-to-nearest-even,
//                            saturating at +-6
//   (s == 0, i.e. an all-zero or tiny block: every code is 0)
// Every step is a correctly rounded f32 operation, so the result is
// reproducible bit for bit.  (An IEEE division per element made the kernel
// compute-bound at 45 % of HBM bandwidth.)
//
// Every (row, block) position of the PADDED blocked scale matrix is written
// (padding rows / columns get a zero scale byte), so the whole scale buffer is
// defined after one launch.  Memory bound: 2 bytes read and 0.5625 bytes
// written per element.
#include <cuda_fp16.h>
#include <algorithm>
#include <cstdint>
#include "ptx.cuh"
#include "common.h"

namespace nvfp4 {
namespace {

__device__ __forceinline__ uint32_t e2m1x2_from_f32(float lo, float hi) {
  uint32_t r;
  asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n cvt.u32.u8 %0, t;\n}\n"
      : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ uint32_t e4m3_from_f32(float v) {
  uint32_t r;
  asm("{\n .reg .b16 t;\n cvt.rn.satfinite.e4m3x2.f32 t, %1, %1;\n cvt.u32.u16 %0, t;\n}\n" : "=r"(r) : "f"(v));
  return r & 0xFFu;
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
  float lo, hi;
  h2_to_f2(cvt_e4m3x2(byte), lo, hi);
  return lo;
}

__device__ __forceinline__ void load_block(const __half* xp, uint32_t (&w)[8]) {
  if ((reinterpret_cast<uintptr_t>(xp) & 15u) == 0) {
    const uint4 u0 = reinterpret_cast<const uint4*>(xp)[0];
    const uint4 u1 = reinterpret_cast<const uint4*>(xp)[1];
    w[0] = u0.x; w[1] = u0.y; w[2] = u0.z; w[3] = u0.w;
    w[4] = u1.x; w[5] = u1.y; w[6] = u1.z; w[7] = u1.w;
  } else {   // any 2-byte alignment
#pragma unroll
    for (int j = 0; j < 8; ++j)
      w[j] = (uint32_t)__half_as_ushort(xp[2 * j]) | ((uint32_t)__half_as_ushort(xp[2 * j + 1]) << 16);
  }
}

// Quantises one 16-element block held as 8 packed half2 words: writes its 8
// code bytes to qp and returns the scale byte.
__device__ __forceinline__ uint32_t quant_block(const uint32_t (&w)[8], uint8_t* qp) {
  // amax in half2: |x| and max are exact in fp16; starting from zero,
  // __hmax2 (like fmaxf) ignores NaN inputs
  __half2 m = __float2half2_rn(0.f);
#pragma unroll
  for (int j = 0; j < 8; ++j) m = __hmax2(m, __habs2(*reinterpret_cast<const __half2*>(&w[j])));
  const float amax = fmaxf(__low2float(m), __high2float(m));
  const uint32_t sbyte = e4m3_from_f32(__fdiv_rn(amax, 6.0f));
  const float s = e4m3_to_f32(sbyte);
  uint32_t packed[2] = {0u, 0u};
  if (s > 0.f) {
    const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
      const uint32_t b = e2m1x2_from_f32(__fmul_rn(__low2float(h), inv), __fmul_rn(__high2float(h), inv));
      packed[j / 4] |= b << (8 * (j % 4));
    }
  }
  if ((reinterpret_cast<uintptr_t>(qp) & 7u) == 0) {
    *reinterpret_cast<uint2*>(qp) = make_uint2(packed[0], packed[1]);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) qp[j] = (uint8_t)(packed[j / 4] >> (8 * (j % 4)));
  }
  return sbyte;
}

// One CTA walks whole rows of the padded scale matrix, RPI rows per pass
// (grid-strided), loading all of a pass's blocks before quantising any so
// that RPI x 32 bytes per thread are in flight; its threads take consecutive
// 16-element blocks of a row, so no index needs a division.  Each warp covers
// 32 consecutive blocks: 1 KB of fp16 in, 256 B of codes and 32 scale bytes
// out (four lanes' bytes are one 4-byte store: the blocked layout keeps blocks
// 4j..4j+3 of a row adjacent).  Rows past M and blocks past K/16 write zero
// scale bytes only.  I indexes the scale buffer.
template <typename I, int RPI>
__global__ void __launch_bounds__(1024) quantize_kernel(const __half* __restrict__ x, int64_t M, int64_t K,
                                                        int64_t ldx, uint8_t* __restrict__ codes, int64_t ldq,
                                                        uint8_t* __restrict__ sf, int kbp, int64_t mp) {
  const int kb = (int)(K / 16);
  const int lane = threadIdx.x & 31;
  const I tile_stride = (I)(kbp / 4) * 512;   // bytes per 128-row tile of the blocked layout
  for (int64_t r0 = blockIdx.x; r0 < mp; r0 += (int64_t)RPI * gridDim.x) {
    for (int c0 = threadIdx.x & ~31; c0 < kbp; c0 += blockDim.x) {   // whole warps: the shuffles need all lanes
      const int c = c0 + lane;
      uint32_t w[RPI][8];
      bool live[RPI];
#pragma unroll
      for (int q = 0; q < RPI; ++q) {
        const int64_t r = r0 + (int64_t)q * gridDim.x;
        live[q] = r < M && c < kb;
        if (live[q]) load_block(x + r * ldx + (int64_t)c * 16, w[q]);
      }
#pragma unroll
      for (int q = 0; q < RPI; ++q) {
        const int64_t r = r0 + (int64_t)q * gridDim.x;
        const uint32_t sbyte = live[q] ? quant_block(w[q], codes + r * ldq + (int64_t)c * 8) : 0u;
        // blocks 4j..4j+3 of the row are adjacent bytes of the blocked layout
        const uint32_t b1 = __shfl_down_sync(0xffffffffu, sbyte, 1);
        const uint32_t b2 = __shfl_down_sync(0xffffffffu, sbyte, 2);
        const uint32_t b3 = __shfl_down_sync(0xffffffffu, sbyte, 3);
        if ((lane & 3) == 0 && c < kbp && r < mp) {
          const I off = (I)(r >> 7) * tile_stride + (I)((r & 31) * 16 + ((r >> 5) & 3) * 4) + (I)(c >> 2) * 512;
          *reinterpret_cast<uint32_t*>(sf + off) = sbyte | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
      }
    }
  }
}

// Rows per pass: 1.  Loading 2 or 4 rows' blocks before quantising any (more
// bytes in flight per thread, fewer resident threads) measured slower (32.6 /
// 33.1 vs 30.9 us at M=8192, K=7168).
constexpr int kQuantRowsPerPass = 1;

template <int RPI>
int launch_quant(bool small, int threads, const __half* x, int64_t M, int64_t K, int64_t ldx, uint8_t* codes,
                 int64_t ldq, uint8_t* sf, int kbp, int64_t mp, cudaStream_t stream) {
  auto kern = small ? quantize_kernel<uint32_t, RPI> : quantize_kernel<uint64_t, RPI>;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(quantize)");
  const int64_t grid = std::min<int64_t>((mp + RPI - 1) / RPI, (int64_t)sm_count() * std::max(per_sm, 1));
  kern<<<(unsigned)grid, threads, 0, stream>>>(x, M, K, ldx, codes, ldq, sf, kbp, mp);
  return check_launch("quantize_kernel");
}

}  // namespace
}  // namespace nvfp4

extern "C" int nvfp4_quantize(const void* x, int64_t M, int64_t K, int64_t ldx, void* codes, int64_t ldq,
                              void* sf_blocked, void* stream) {
  using namespace nvfp4;
  if (!x || !codes || !sf_blocked) return fail(NVFP4_ERR_INVALID, "nvfp4_quantize: null pointer");
  if (M < 1 || K < 16 || K % 16) return fail(NVFP4_ERR_INVALID, "nvfp4_quantize: need M >= 1 and K a multiple of 16");
  if (ldx < K || ldq < K / 2) return fail(NVFP4_ERR_INVALID, "nvfp4_quantize: row strides below the row length");
  if (reinterpret_cast<uintptr_t>(x) & 1) return fail(NVFP4_ERR_ALIGNMENT, "nvfp4_quantize: fp16 input not 2-byte aligned");
  const int64_t mp = (M + 127) / 128 * 128, kbp = (K / 16 + 3) / 4 * 4;
  if (kbp > INT32_MAX / 32) return fail(NVFP4_ERR_INVALID, "nvfp4_quantize: K too large");
  if (reinterpret_cast<uintptr_t>(sf_blocked) & 3)
    return fail(NVFP4_ERR_ALIGNMENT, "nvfp4_quantize: scale buffer not 4-byte aligned");
  // one warp per 32 blocks of a row, up to 1024 threads; rows grid-strided
  // over as many CTAs as fit at once
  const int threads = (int)std::min<int64_t>(1024, (kbp + 31) / 32 * 32);
  const bool small = mp * kbp + 1024 < (int64_t)UINT32_MAX;   // the largest scale offset is below mp * kbp + 512
  return launch_quant<kQuantRowsPerPass>(small, threads, static_cast<const __half*>(x), M, K, ldx,
                                         static_cast<uint8_t*>(codes), ldq, static_cast<uint8_t*>(sf_blocked),
                                         (int)kbp, mp, static_cast<cudaStream_t>(stream));
}
