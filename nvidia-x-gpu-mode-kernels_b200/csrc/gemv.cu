// Batched NVFP4 block-scaled GEMV for sm_100a.
//
//   c[m, l] = sum_k e2m1(A[m,k,l]) e2m1(b[k,l]) e4m3(SFA[m,k/16,l]) e4m3(SFB[k/16,l])
//
// The reference (blackwell_nvfp4_gemv.cu:295-475) streams one tensor-map tile
// per K step into a single shared buffer and computes with all threads, so loads
// and math alternate inside each CTA.  This kernel is HBM-streaming instead:
//
//   * a persistent grid (a multiple of the SM count) splits the M*L output rows
//     into equal contiguous ranges, one per CTA, so every CTA streams the same
//     number of bytes;
//   * one producer warp fills a STAGES-deep shared-memory ring with 1-D bulk
//     (TMA) copies: each lane copies one row's K-slice of A and of SFA, and the
//     matching slice of b/SFB rides along in the same stage;
//   * CONSUMER_WARPS warps own rows; each lane owns 16-byte chunks (32 e2m1 codes,
//     two scale blocks).  b is decoded to f16x2 once per stage per warp and kept
//     in registers while the warp walks its rows;
//   * e2m1 -> f16x2 with cvt.rn.f16x2.e2m1x2, products summed with fma.rn.f16x2
//     inside a 16-element block.  Each half-lane sums 8 products that are
//     multiples of 1/4 below 36 in magnitude, so every partial sum is a multiple
//     of 1/4 below 512 and f16 holds it exactly.  The block sum is widened to
//     f32 and scaled by sfa*sfb in f32 (exact: 4 x 4 significant bits), then
//     accumulated in f32 - unlike the reference, which scales and sums in f16
//     (:126-131) and overflows for scale products above 65504;
//   * the lanes' partial sums of a row meet in a xor-shuffle reduction and one
//     lane stores the fp16 result.
//
// Every wait is bounded (2 s) and reports into the device error word.
#include <cuda_fp16.h>
#include "ptx.cuh"
#include "common.h"

namespace nvfp4 {
namespace {

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

struct GemvArgs {
  const uint8_t* a;
  const uint8_t* b;
  const uint8_t* sfa;
  const uint8_t* sfb;
  __half* c;
  int64_t M, K, L;
  int64_t a_sm, a_sl, b_sl, sfa_sm, sfa_sl, sfb_sl, c_sm, c_sl;
  uint32_t* err;
};

template <int ROWS_, int KTB_, int STAGES_, int CONSUMER_WARPS_>
struct GemvCfg {
  static constexpr int ROWS = ROWS_;            // rows per stage tile
  static constexpr int KTB = KTB_;              // A bytes per row per stage
  static constexpr int STAGES = STAGES_;
  static constexpr int CW = CONSUMER_WARPS_;
  static constexpr int THREADS = (CW + 1) * 32;
  static constexpr int SFB_BYTES = KTB / 8;     // scale bytes per row per stage
  static constexpr int NCH = KTB / 512;         // 16-byte chunks per lane per row
  static constexpr int RPW = (ROWS + CW - 1) / CW;  // rows per warp per tile (max)
  static constexpr int OFF_SFA = ROWS * KTB;
  static constexpr int OFF_B = OFF_SFA + ROWS * SFB_BYTES;
  static constexpr int OFF_SFB = OFF_B + KTB;
  static constexpr int STAGE_BYTES = ((OFF_SFB + SFB_BYTES) + 127) / 128 * 128;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 2 * STAGES * 8 + 16;
  static_assert(KTB % 512 == 0, "KTB must cover whole warp-wide chunk rows");
  static_assert(ROWS <= 32, "one producer lane per row");
};

// The rows a CTA owns: [row_begin, row_end) of the flattened (l, m) space.
__device__ __forceinline__ void cta_rows(int64_t total, int64_t& r0, int64_t& r1) {
  const int64_t g = gridDim.x, c = blockIdx.x;
  r0 = total * c / g;
  r1 = total * (c + 1) / g;
}

template <class C>
__global__ void __launch_bounds__(C::THREADS, 1) gemv_tma_kernel(const __grid_constant__ GemvArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + C::STAGES * C::STAGE_BYTES;
  const uint32_t bar_empty = bar_full + 8 * C::STAGES;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, C::CW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t M = p.M, KB = p.K / 2;  // KB: A bytes per row
  const int nk = (int)((KB + C::KTB - 1) / C::KTB);
  int64_t r0, r1;
  cta_rows(M * p.L, r0, r1);

  if (warp == C::CW) {
    // ---------------- producer warp ----------------
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    uint32_t it = 0;
    for (int64_t r = r0; r < r1;) {
      const int64_t l = r / M, m = r % M;
      const int n = (int)imin64(imin64(C::ROWS, r1 - r), M - m);
      const uint8_t* a_rows = p.a + l * p.a_sl + m * p.a_sm;
      const uint8_t* sa_rows = p.sfa + l * p.sfa_sl + m * p.sfa_sm;
      const uint8_t* b_l = p.b + l * p.b_sl;
      const uint8_t* sb_l = p.sfb + l * p.sfb_sl;
      for (int kt = 0; kt < nk; ++kt, ++it) {
        const int s = it % C::STAGES;
        const uint32_t ph = (it / C::STAGES) & 1;
        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, p.err, kDevErrTimeoutEmpty)) return;
        const int64_t k0 = (int64_t)kt * C::KTB;
        const uint32_t kb = (uint32_t)imin64(C::KTB, KB - k0);
        const uint32_t fb = kb / 8;
        const uint32_t st = sbase + s * C::STAGE_BYTES;
        if (lane == 0) mbar_arrive_expect_tx(bar_full + 8 * s, (uint32_t)(n + 1) * (kb + fb));
        __syncwarp();
        if (lane < n) {
          bulk_g2s_hint(st + lane * C::KTB, a_rows + lane * p.a_sm + k0, kb, bar_full + 8 * s, pol_stream);
          bulk_g2s_hint(st + C::OFF_SFA + lane * C::SFB_BYTES, sa_rows + lane * p.sfa_sm + k0 / 8, fb,
                        bar_full + 8 * s, pol_stream);
        }
        if (lane == 31) {
          bulk_g2s_hint(st + C::OFF_B, b_l + k0, kb, bar_full + 8 * s, pol_keep);
          bulk_g2s_hint(st + C::OFF_SFB, sb_l + k0 / 8, fb, bar_full + 8 * s, pol_keep);
        }
      }
      r += n;
    }
    return;
  }

  // ---------------- consumer warps ----------------
  uint32_t it = 0;
  for (int64_t r = r0; r < r1;) {
    const int64_t l = r / M, m = r % M;
    const int n = (int)imin64(imin64(C::ROWS, r1 - r), M - m);
    float acc[C::RPW];
#pragma unroll
    for (int j = 0; j < C::RPW; ++j) acc[j] = 0.f;

    for (int kt = 0; kt < nk; ++kt, ++it) {
      const int s = it % C::STAGES;
      const uint32_t ph = (it / C::STAGES) & 1;
      if (!mbar_wait(bar_full + 8 * s, ph, p.err, kDevErrTimeoutFull)) return;
      const int64_t k0 = (int64_t)kt * C::KTB;
      const int kb = (int)imin64(C::KTB, KB - k0);
      const uint8_t* st = smem + s * C::STAGE_BYTES;

      // b slice for this lane: chunk i at byte 512*i + 16*lane.
      uint32_t bh[C::NCH][16];
      float sb[C::NCH][2];
#pragma unroll
      for (int i = 0; i < C::NCH; ++i) {
        const int off = 512 * i + 16 * lane;
        if (off < kb) {
          const uint4 bv = *reinterpret_cast<const uint4*>(st + C::OFF_B + off);
          cvt_e2m1x8(bv.x, *reinterpret_cast<uint32_t(*)[4]>(&bh[i][0]));
          cvt_e2m1x8(bv.y, *reinterpret_cast<uint32_t(*)[4]>(&bh[i][4]));
          cvt_e2m1x8(bv.z, *reinterpret_cast<uint32_t(*)[4]>(&bh[i][8]));
          cvt_e2m1x8(bv.w, *reinterpret_cast<uint32_t(*)[4]>(&bh[i][12]));
          const uint32_t s2 = *reinterpret_cast<const uint16_t*>(st + C::OFF_SFB + off / 8);
          h2_to_f2(cvt_e4m3x2(s2), sb[i][0], sb[i][1]);
        }
      }

#pragma unroll
      for (int j = 0; j < C::RPW; ++j) {
        const int row = warp + j * C::CW;
        if (row < n) {
          const uint8_t* arow = st + row * C::KTB;
          const uint8_t* srow = st + C::OFF_SFA + row * C::SFB_BYTES;
#pragma unroll
          for (int i = 0; i < C::NCH; ++i) {
            const int off = 512 * i + 16 * lane;
            if (off < kb) {
              const uint4 av = *reinterpret_cast<const uint4*>(arow + off);
              const uint32_t s2 = *reinterpret_cast<const uint16_t*>(srow + off / 8);
              uint32_t h[4], c0 = 0u, c1 = 0u;
              cvt_e2m1x8(av.x, h);
              c0 = hfma2(h[0], bh[i][0], c0); c0 = hfma2(h[1], bh[i][1], c0);
              c0 = hfma2(h[2], bh[i][2], c0); c0 = hfma2(h[3], bh[i][3], c0);
              cvt_e2m1x8(av.y, h);
              c0 = hfma2(h[0], bh[i][4], c0); c0 = hfma2(h[1], bh[i][5], c0);
              c0 = hfma2(h[2], bh[i][6], c0); c0 = hfma2(h[3], bh[i][7], c0);
              cvt_e2m1x8(av.z, h);
              c1 = hfma2(h[0], bh[i][8], c1); c1 = hfma2(h[1], bh[i][9], c1);
              c1 = hfma2(h[2], bh[i][10], c1); c1 = hfma2(h[3], bh[i][11], c1);
              cvt_e2m1x8(av.w, h);
              c1 = hfma2(h[0], bh[i][12], c1); c1 = hfma2(h[1], bh[i][13], c1);
              c1 = hfma2(h[2], bh[i][14], c1); c1 = hfma2(h[3], bh[i][15], c1);
              float sa0, sa1, x0, y0, x1, y1;
              h2_to_f2(cvt_e4m3x2(s2), sa0, sa1);
              h2_to_f2(c0, x0, y0);
              h2_to_f2(c1, x1, y1);
              acc[j] = fmaf(x0 + y0, sa0 * sb[i][0], acc[j]);
              acc[j] = fmaf(x1 + y1, sa1 * sb[i][1], acc[j]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);
    }

#pragma unroll
    for (int j = 0; j < C::RPW; ++j) {
      float v = acc[j];
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
      const int row = warp + j * C::CW;
      if (lane == 0 && row < n) p.c[l * p.c_sl + (m + row) * p.c_sm] = __float2half_rn(v);
    }
    r += n;
  }
}

// Plain-load kernel for shapes the bulk-copy path cannot take (K % 256 != 0 or
// strides / pointers not 16-byte aligned).  One warp per output row; lane t
// handles 16-element blocks t, t+32, ...; same exact per-block arithmetic.
__global__ void __launch_bounds__(256) gemv_generic_kernel(const __grid_constant__ GemvArgs p) {
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nblk = p.K / 16;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < p.M * p.L;
       r += warps_total) {
    const int64_t l = r / p.M, m = r % p.M;
    const uint8_t* arow = p.a + l * p.a_sl + m * p.a_sm;
    const uint8_t* srow = p.sfa + l * p.sfa_sl + m * p.sfa_sm;
    const uint8_t* bl = p.b + l * p.b_sl;
    const uint8_t* sbl = p.sfb + l * p.sfb_sl;
    float acc = 0.f;
    for (int64_t blk = lane; blk < nblk; blk += 32) {
      uint32_t c = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c = hfma2(cvt_e2m1x2(arow[blk * 8 + j]), cvt_e2m1x2(bl[blk * 8 + j]), c);
      }
      float x, y, sa, sb, d0, d1;
      h2_to_f2(c, x, y);
      h2_to_f2(cvt_e4m3x2(srow[blk]), sa, d0);
      h2_to_f2(cvt_e4m3x2(sbl[blk]), sb, d1);
      acc = fmaf(x + y, sa * sb, acc);
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
    if (lane == 0) p.c[l * p.c_sl + m * p.c_sm] = __float2half_rn(acc);
  }
}

template <class C>
int launch_tma(const GemvArgs& args, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_tma_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
    attr_set[dev] = true;
  }
  const int64_t total = args.M * args.L;
  int64_t grid = sm_count();
  // Small problems: keep at least one full tile per CTA.
  const int64_t tiles = (total + C::ROWS - 1) / C::ROWS;
  if (tiles < grid) grid = tiles;
  if (grid < 1) grid = 1;
  gemv_tma_kernel<C><<<(unsigned)grid, C::THREADS, C::SMEM, stream>>>(args);
  return check_launch("gemv_tma_kernel");
}

}  // namespace

}  // namespace nvfp4

using nvfp4::fail;

extern "C" int nvfp4_gemv(const void* a, const void* b, const void* sfa, const void* sfb, void* c,
                          int64_t M, int64_t K, int64_t L, int64_t a_sm, int64_t a_sl, int64_t b_sl,
                          int64_t sfa_sm, int64_t sfa_sl, int64_t sfb_sl, int64_t c_sm, int64_t c_sl,
                          void* stream) {
  using namespace nvfp4;
  if (!a || !b || !sfa || !sfb || !c) return fail(NVFP4_ERR_INVALID, "nvfp4_gemv: null pointer");
  if (M < 1 || L < 1 || K < 16 || K % 16 != 0)
    return fail(NVFP4_ERR_INVALID, "nvfp4_gemv: need M>=1, L>=1, K>=16 and K%%16==0 (got M=%lld K=%lld L=%lld)",
                (long long)M, (long long)K, (long long)L);
  if (a_sm < K / 2 || sfa_sm < K / 16 || (L > 1 && (a_sl <= 0 || b_sl <= 0 || sfa_sl <= 0 || sfb_sl <= 0)) ||
      c_sm == 0 || (L > 1 && c_sl == 0))
    return fail(NVFP4_ERR_INVALID, "nvfp4_gemv: invalid strides");
  GemvArgs args{static_cast<const uint8_t*>(a), static_cast<const uint8_t*>(b),
                static_cast<const uint8_t*>(sfa), static_cast<const uint8_t*>(sfb),
                static_cast<__half*>(c), M, K, L, a_sm, a_sl, b_sl, sfa_sm, sfa_sl, sfb_sl, c_sm, c_sl,
                device_error_word()};
  if (!args.err) return fail(NVFP4_ERR_CUDA, "nvfp4_gemv: cannot resolve the device error word");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool tma_ok = (K % 256 == 0) && aligned16(a) && aligned16(b) && aligned16(sfa) && aligned16(sfb) &&
                      a_sm % 16 == 0 && sfa_sm % 16 == 0 && (L == 1 || (a_sl % 16 == 0 && b_sl % 16 == 0 &&
                      sfa_sl % 16 == 0 && sfb_sl % 16 == 0));
  if (tma_ok) {
    using C = GemvCfg<32, 1024, 5, 8>;
    return launch_tma<C>(args, st);
  }
  const int64_t rows = M * L;
  int64_t grid = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (grid > cap) grid = cap;
  gemv_generic_kernel<<<(unsigned)grid, 256, 0, st>>>(args);
  return check_launch("gemv_generic_kernel");
}
