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
// One thread per (row, block) position of the PADDED blocked scale matrix:
// threads on padding rows / columns write a zero scale byte and nothing else,
// so the whole scale buffer is defined after one launch.  Memory bound: 2 bytes
// read and 0.5625 bytes written per element.
#include <cuda_fp16.h>
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

// Index type I: 32-bit when every index fits (64-bit division is slow).
template <typename I>
__global__ void __launch_bounds__(256) quantize_kernel(const __half* __restrict__ x, int64_t M, int64_t K,
                                                       int64_t ldx, uint8_t* __restrict__ codes, int64_t ldq,
                                                       uint8_t* __restrict__ sf, int64_t kbp_, int64_t total_) {
  const I kb = (I)(K / 16), kbp = (I)kbp_, total = (I)total_;
  const I nkt = kbp / 4;  // 4-block column tiles
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
    const I r = i / kbp, c = i % kbp;   // consecutive threads: consecutive blocks of one row
    const I off = ((r / 128) * nkt + c / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (c % 4);
    if (r >= M || c >= kb) {
      sf[off] = 0;
      continue;
    }
    const __half* xp = x + (int64_t)r * ldx + (int64_t)c * 16;
    float v[16];
    if ((reinterpret_cast<uintptr_t>(xp) & 15u) == 0) {
      const uint4 u0 = reinterpret_cast<const uint4*>(xp)[0];
      const uint4 u1 = reinterpret_cast<const uint4*>(xp)[1];
      const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
        v[2 * j] = __low2float(h);
        v[2 * j + 1] = __high2float(h);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = __half2float(xp[j]);
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const uint32_t sbyte = e4m3_from_f32(__fdiv_rn(amax, 6.0f));
    const float s = e4m3_to_f32(sbyte);
    uint32_t packed[2] = {0u, 0u};
    if (s > 0.f) {
      const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t b = e2m1x2_from_f32(__fmul_rn(v[2 * j], inv), __fmul_rn(v[2 * j + 1], inv));
        packed[j / 4] |= b << (8 * (j % 4));
      }
    }
    uint8_t* qp = codes + (int64_t)r * ldq + (int64_t)c * 8;
    if ((reinterpret_cast<uintptr_t>(qp) & 7u) == 0) {
      *reinterpret_cast<uint2*>(qp) = make_uint2(packed[0], packed[1]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) qp[j] = (uint8_t)(packed[j / 4] >> (8 * (j % 4)));
    }
    sf[off] = (uint8_t)sbyte;
  }
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
  const int64_t total = mp * kbp;
  int64_t grid = (total + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (grid > cap) grid = cap;
  // the largest index the kernel forms is the scale offset, below total + 512
  auto kern = (total + 1024 < (int64_t)UINT32_MAX) ? quantize_kernel<uint32_t> : quantize_kernel<uint64_t>;
  kern<<<(unsigned)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), M, K, ldx, static_cast<uint8_t*>(codes), ldq, static_cast<uint8_t*>(sf_blocked),
      kbp, total);
  return check_launch("quantize_kernel");
}
