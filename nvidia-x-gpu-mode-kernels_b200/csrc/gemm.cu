// NVFP4 block-scaled GEMMs on the tcgen05 tensor cores (sm_100a):
//
//   grouped:  C_g[M_g, N_g] = A_g[M_g, K_g] . B_g[N_g, K_g]^T          (fp16 out)
//   dual:     C[M, N] = silu(A . B1^T) * (A . B2^T)                    (fp16 out)
//
// Operands are e2m1 codes packed two per byte, K-major (rows of K/2 bytes),
// with one e4m3 scale per 16 K-elements stored in the 128x4 blocked layout
// (128-row x 4-scale tiles of 512 bytes, row-tile major; inside a tile the
// scale (r, c) sits at byte (r%32)*16 + (r/32)*4 + c).  That layout is what a
// tcgen05.cp 32x128b.warpx4 copy turns into the tensor-memory arrangement the
// block-scaled MMA reads, so scales go global -> shared -> tensor memory with
// plain copies.  The MMA reads scales as unsigned e4m3 (sign bit must be 0).
//
// One persistent CTA per SM walks output tiles of 128 x BN (tile t, t+grid,
// ...).  Tiles of a group are ordered M-tile fastest, so CTAs running at the
// same time share B tiles through L2.  Warp roles:
//   warp 0  TMA producer: per 256-element K step, one 128x128-byte box of A and
//           one BNx128-byte box of B (and B2) with 128-byte swizzle, plus 1-D
//           bulk copies of the 2 KB scale blocks, into a STAGES-deep ring;
//   warp 1  allocates tensor memory; one thread copies the stage's scales into
//           tensor memory and issues 4 MMAs of K=64 (kind::mxf4nvf4,
//           scale_vec::4X) per B operand, then commits the stage back to the
//           producer and, after the last K step, the accumulator to the
//           epilogue;
//   warps 2-5  epilogue: tcgen05.ld of the fp32 accumulator rows (one row per
//           thread), SiLU-gate or plain conversion to fp16, 16-byte stores.
// Every mbarrier wait is bounded (2 s) and reports into the device error word.
#include <cuda_fp16.h>
#include <cstring>
#include <mutex>
#include "ptx.cuh"
#include "tcgen05.cuh"
#include "common.h"
#include "tmap.h"

namespace nvfp4 {
namespace {

constexpr int BM = 128;          // rows per tile (one MMA of M=128)
constexpr int KSTEP = 256;       // K elements per stage = 128 bytes per row
constexpr int KSTEP_BYTES = 128;

struct GemmGroup {
  CUtensorMap ta, tb, tb2;       // A [M, K/2], B [N, K/2] (B2 for the dual GEMM)
  CUtensorMap tc;                // C [M, N] fp16, 64-column boxes, 128-byte swizzle
  CUtensorMap tsa, tsb, tsb2;    // blocked scales as [row tiles][K/64][128 x u32]
  const uint8_t* sfa;            // blocked scales of A, B, B2
  const uint8_t* sfb;
  const uint8_t* sfb2;
  __half* c;
  int64_t ldc;                   // elements
  int M, N, K;
  int tiles_m, tiles_n, tile_begin;
  int vec_ok;                    // c 16-byte aligned and ldc % 8 == 0: 16-byte stores
  int tma_store;                 // tc is valid: the epilogue stores through shared memory + TMA
};

template <int MAXG>
struct GemmParams {
  GemmGroup g[MAXG];
  int ngroups;
  int total_tiles;
  uint32_t* err;
};

// DBG is a tuning knob (0 in every product instantiation): bit 0 skips the
// scale copies, bit 1 the MMAs, bit 2 the loads, bit 3 the epilogue's
// tensor-memory loads and stores, to time each link alone.
// SFST selects how block scales reach tensor memory: 0 = tcgen05.cp issued by
// the MMA thread, 1 = four scale warps that tcgen05.st them (off the MMA queue).
// EPI 1 stages the fp16 tile in shared memory and writes it with TMA stores
// (needs BM*BN*2 bytes of shared memory); EPI 0 stores rows from registers.
// POL picks the L2 policy of B loads: 0 evict-first, 1 normal.
// SEPSF 1: the stage's scale boxes complete on their own barrier, issued
// before the operand boxes, so the scale warps stage them while the operand
// bytes are still in flight (needs SFST and SFTMA).
// TRANS 1 (skinny GEMM): A holds weight rows, B the token rows, and the
// epilogue writes C^T, i.e. out[token][weight row]; one N tile only.
template <int BN_, bool DUAL_, int STAGES_, int DBG_ = 0, int SFST_ = 1, int EPI_ = 1, int POL_ = 0, int SFTMA_ = 1,
          int SEPSF_ = 1, int TRANS_ = 0, int KA_ = 1>
struct GemmCfg {
  static constexpr int TRANS = TRANS_;
  // KA 128-byte K atoms (256 elements each) per stage: one TMA box per atom and
  // operand, 4 * KA MMAs per stage, scale boxes of 4 * KA K-blocks
  static constexpr int KA = KA_;
  static constexpr int KPS = 4 * KA_;    // 64-element K blocks per stage
  static constexpr int SFTMA = SFTMA_;   // scales by tensor-map TMA (1) or 1-D bulk copies (0)
  static constexpr int SEPSF = (SEPSF_ && SFST_ && SFTMA_) ? 1 : 0;
  static constexpr int DBG = DBG_;
  static constexpr int EPI = EPI_;
  static constexpr int POL = POL_;
  static constexpr int SFST = SFST_;
  static constexpr int BN = BN_;
  static constexpr bool DUAL = DUAL_;
  static constexpr int STAGES = STAGES_;
  static constexpr int NB = (BN + 127) / 128;              // 128-row scale blocks per B tile
  static_assert(BN % 128 == 0 || (BN < 128 && 128 % BN == 0 && (BN % 32 == 0 || (TRANS_ && BN == 16))),
                "B tiles must not straddle scale blocks");
  static constexpr int A_ATOM = BM * KSTEP_BYTES;          // 16 KB per K atom
  static constexpr int B_ATOM = BN * KSTEP_BYTES;
  static constexpr int A_BYTES = KA * A_ATOM;
  static constexpr int B_BYTES = KA * B_ATOM;
  static constexpr int SFA_BYTES = KPS * 512;              // KPS K-blocks of 64
  static constexpr int SFB_ROWTILE = KPS * 512;            // per 128-row block of B
  static constexpr int SFB_BYTES = NB * SFB_ROWTILE;
  static constexpr int OFF_B = A_BYTES;
  static constexpr int OFF_B2 = OFF_B + B_BYTES;
  static constexpr int OFF_SFA = OFF_B2 + (DUAL ? B_BYTES : 0);
  static constexpr int OFF_SFB = OFF_SFA + SFA_BYTES;
  static constexpr int OFF_SFB2 = OFF_SFB + SFB_BYTES;
  static constexpr int STAGE_BYTES = ((OFF_SFB2 + (DUAL ? SFB_BYTES : 0)) + 1023) / 1024 * 1024;
  static constexpr int OFF_C = STAGES * STAGE_BYTES;      // fp16 output tile, BN/64 swizzled boxes
  static constexpr int C_BYTES = EPI ? BM * BN * 2 : 0;
  static constexpr int OFF_BAR = OFF_C + C_BYTES;
  static constexpr int SMEM = OFF_BAR + (4 * STAGES + 4) * 8 + 16;   // base is 1024-aligned
  // tensor memory columns
  static constexpr int ACC_COLS = DUAL ? 2 * BN : BN;
  static constexpr int SF_BASE = ACC_COLS;
  static constexpr int SFB_COLS_PER_KB = NB * 4;
  static constexpr int SFA_COLS = 4 * KPS;
  static constexpr int SF_STAGE_COLS = SFA_COLS + KPS * SFB_COLS_PER_KB * (DUAL ? 2 : 1);
  static constexpr int TMEM_COLS = 512;
  static_assert(SF_BASE + STAGES * SF_STAGE_COLS <= TMEM_COLS, "tensor memory budget");
  static_assert(KA == 1 || SFTMA_, "wide stages load scales by tensor map");
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int THREADS = SFST ? 320 : 192;   // + 4 scale warps (warps 6-9)
  static constexpr bool PAIR = false;
  static constexpr int TILE_M = BM;
  static constexpr int B_BOX = BN;
  static constexpr uint32_t IDESC = tc::idesc_mxf4nvf4(BM, BN);
};

__device__ __forceinline__ int find_group(const GemmGroup* g, int ng, int t) {
  int i = 0;
  while (i + 1 < ng && g[i + 1].tile_begin <= t) ++i;
  return i;
}

// Scale blocks of one 256-element K step with 1-D bulk copies: the A row
// tile and the B row tiles [rt_b, rt_b + NB).  The caller registered the
// full-box byte count (as for tensor-map loads); bytes that are not copied
// (blocks past the end of a matrix or of K) are completed here directly.
template <class C>
__device__ __forceinline__ void load_sf_bulk(uint32_t st, const GemmGroup& G, int rt_a, int rt_b, int nk64, int ks,
                                             uint32_t bar) {
  const int nch = min(4, nk64 - 4 * ks);
  const int nrt_a = (G.M + 127) / 128, nrt_b = (G.N + 127) / 128;
  uint32_t missing = 0;
  if (rt_a < nrt_a) bulk_g2s(st + C::OFF_SFA, G.sfa + ((size_t)rt_a * nk64 + 4 * ks) * 512, nch * 512, bar);
  missing += (rt_a < nrt_a) ? (4 - nch) * 512 : 2048;
  for (int nb = 0; nb < C::NB; ++nb) {
    const int rt = rt_b + nb;
    const int ops = C::DUAL ? 2 : 1;
    if (rt >= nrt_b) { missing += 2048 * ops; continue; }
    bulk_g2s(st + C::OFF_SFB + nb * 2048, G.sfb + ((size_t)rt * nk64 + 4 * ks) * 512, nch * 512, bar);
    if (C::DUAL) bulk_g2s(st + C::OFF_SFB2 + nb * 2048, G.sfb2 + ((size_t)rt * nk64 + 4 * ks) * 512, nch * 512, bar);
    missing += (4 - nch) * 512 * ops;
  }
  if (missing) {   // complete the uncopied bytes ourselves
    asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(missing) : "memory");
  }
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// The first n (<= 8) fp16 values of a packed 16-byte piece, one element at a
// time (unaligned or ragged output rows).  Out of line so the epilogue's
// unrolled row loop does not hold a store path per element in registers.
__device__ __noinline__ void store_piece(__half* dst, uint4 piece, int n) {
  const uint32_t w[4] = {piece.x, piece.y, piece.z, piece.w};
  for (int j = 0; j < n; ++j) dst[j] = __ushort_as_half((unsigned short)(w[j / 2] >> (16 * (j & 1))));
}

template <class C, int MAXG>
__global__ void __launch_bounds__(C::THREADS, 1) gemm_kernel(const __grid_constant__ GemmParams<MAXG> P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = raw;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (raw & 1023u) {  // the swizzled tiles need a 1024-aligned base; the launch guarantees it
    if (threadIdx.x == 0) atomicOr(P.err, kDevErrTimeoutMma);
    return;
  }
  const uint32_t bar_full = sbase + C::OFF_BAR;
  const uint32_t bar_empty = bar_full + 8 * C::STAGES;
  const uint32_t bar_sfr = bar_empty + 8 * C::STAGES;      // scales in tensor memory (SFST)
  const uint32_t bar_sff = bar_sfr + 8 * C::STAGES;        // scale boxes landed (SEPSF)
  const uint32_t bar_accf = bar_sff + 8 * C::STAGES;
  const uint32_t bar_acce = bar_accf + 8;
  const uint32_t bar_done = bar_acce + 8;
  const uint32_t tmem_slot = bar_done + 8;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - raw));

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
      mbar_init(bar_sfr + 8 * s, 4);
      mbar_init(bar_sff + 8 * s, 1);
    }
    mbar_init(bar_accf, 1);
    mbar_init(bar_acce, 4);
    mbar_init(bar_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot_ptr;

  if (warp == 0) {
    // ---------------------------- producer ----------------------------
    if (lane == 0) {
      for (int i = 0; i < P.ngroups; ++i) {
        prefetch_tmap(&P.g[i].ta);
        prefetch_tmap(&P.g[i].tb);
        if (C::DUAL) prefetch_tmap(&P.g[i].tb2);
        if (C::SFTMA) {
          prefetch_tmap(&P.g[i].tsa);
          prefetch_tmap(&P.g[i].tsb);
          if (C::DUAL) prefetch_tmap(&P.g[i].tsb2);
        }
      }
      const uint64_t pol_a = policy_evict_last();   // A tiles are re-read by every N tile
      const uint64_t pol_b = C::POL ? policy_evict_normal() : policy_evict_first();
      uint32_t it = 0;
      for (int t = blockIdx.x; t < P.total_tiles; t += gridDim.x) {
        const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
        const int local = t - G.tile_begin;
        const int mt = local % G.tiles_m, nt = local / G.tiles_m;
        const int nk64 = G.K / 64;
        const int nks = (nk64 + C::KPS - 1) / C::KPS;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(bar_empty + 8 * s, ((it / C::STAGES) & 1) ^ 1, P.err, kDevErrTimeoutEmpty)) goto done;
          const uint32_t st = sbase + s * C::STAGE_BYTES;
          const uint32_t fb = bar_full + 8 * s;
          // scale boxes always count in full (blocks past the end read as zeros)
          const uint32_t sf_bytes = (C::DBG & 16) ? 0 : C::SFA_BYTES + C::SFB_BYTES * (C::DUAL ? 2 : 1);
          const uint32_t bytes = C::A_BYTES + C::B_BYTES * (C::DUAL ? 2 : 1) + (C::SEPSF ? 0 : sf_bytes);
          if (C::DBG & 4) {
            mbar_arrive(fb);
            if (C::SEPSF) mbar_arrive(bar_sff + 8 * s);
            continue;
          }
          if (C::SEPSF) {   // scales first, on their own barrier
            const uint32_t sb = bar_sff + 8 * s;
            mbar_arrive_expect_tx(sb, sf_bytes);
            if (!(C::DBG & 16)) {
              tma_load_3d(st + C::OFF_SFA, &G.tsa, sb, 0, C::KPS * ks, mt, pol_a);
              tma_load_3d(st + C::OFF_SFB, &G.tsb, sb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
              if (C::DUAL) tma_load_3d(st + C::OFF_SFB2, &G.tsb2, sb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
            }
          }
          mbar_arrive_expect_tx(fb, bytes);
#pragma unroll
          for (int a = 0; a < C::KA; ++a) {   // atoms past K read as zeros (and count in full)
            const int x = (ks * C::KA + a) * KSTEP_BYTES;
            tma_load_2d(st + a * C::A_ATOM, &G.ta, fb, x, mt * BM, pol_a);
            tma_load_2d(st + C::OFF_B + a * C::B_ATOM, &G.tb, fb, x, nt * C::BN, pol_b);
            if (C::DUAL) tma_load_2d(st + C::OFF_B2 + a * C::B_ATOM, &G.tb2, fb, x, nt * C::BN, pol_b);
          }
          if (!(C::DBG & 16) && !C::SEPSF) {
            if (C::SFTMA) {
              tma_load_3d(st + C::OFF_SFA, &G.tsa, fb, 0, C::KPS * ks, mt, pol_a);
              tma_load_3d(st + C::OFF_SFB, &G.tsb, fb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
              if (C::DUAL) tma_load_3d(st + C::OFF_SFB2, &G.tsb2, fb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
            } else {
              load_sf_bulk<C>(st, G, mt, (nt * C::BN) / 128, nk64, ks, fb);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA -------------------------------
    if (lane == 0) {
      uint32_t it = 0, tile_it = 0;
      for (int t = blockIdx.x; t < P.total_tiles; t += gridDim.x, ++tile_it) {
        const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
        const int nk64 = G.K / 64;
        const int nks = (nk64 + C::KPS - 1) / C::KPS;
        // a B tile narrower than 128 rows starts inside its scale block: its
        // scales begin (tile row offset / 32) columns into the block's 4
        const uint32_t sfb_off = (uint32_t)((((t - G.tile_begin) / G.tiles_m) * C::BN) % 128) / 32;
        if (!mbar_wait(bar_acce, (tile_it & 1) ^ 1, P.err, kDevErrTimeoutMma)) goto done;
        tc::fence_after_sync();
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait((C::SFST ? bar_sfr : bar_full) + 8 * s, (it / C::STAGES) & 1, P.err, kDevErrTimeoutFull))
            goto done;
          if (C::SEPSF && !mbar_wait(bar_full + 8 * s, (it / C::STAGES) & 1, P.err, kDevErrTimeoutFull)) goto done;
          tc::fence_after_sync();
          const uint32_t st = sbase + s * C::STAGE_BYTES;
          const int nch = min(C::KPS, nk64 - C::KPS * ks);
          const uint32_t sf = tmem + C::SF_BASE + s * C::SF_STAGE_COLS;
          const uint32_t sfa_t = sf, sfb_t = sf + C::SFA_COLS, sfb2_t = sf + C::SFA_COLS + C::KPS * C::SFB_COLS_PER_KB;
          for (int kk = 0; kk < nch && !(C::DBG & 1) && !C::SFST; ++kk) {
            tc::cp_sf_32x128b_x4(sfa_t + 4 * kk, tc::desc_sf_block(st + C::OFF_SFA + kk * 512));
            for (int nb = 0; nb < C::NB; ++nb) {
              tc::cp_sf_32x128b_x4(sfb_t + kk * C::SFB_COLS_PER_KB + 4 * nb,
                                   tc::desc_sf_block(st + C::OFF_SFB + nb * C::SFB_ROWTILE + kk * 512));
              if (C::DUAL)
                tc::cp_sf_32x128b_x4(sfb2_t + kk * C::SFB_COLS_PER_KB + 4 * nb,
                                     tc::desc_sf_block(st + C::OFF_SFB2 + nb * C::SFB_ROWTILE + kk * 512));
            }
          }
          for (int kk = 0; kk < nch && !(C::DBG & 2); ++kk) {
            const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
            // atom kk / 4 of the stage; its (kk % 4)-th 64-element slice starts
            // 32 bytes further (encoded >> 4)
            const int at = kk >> 2, sl = kk & 3;
            const uint64_t da = tc::desc_sw128(st + at * C::A_ATOM) + 2 * sl;
            const uint64_t db = tc::desc_sw128(st + C::OFF_B + at * C::B_ATOM) + 2 * sl;
            tc::mma_mxf4nvf4(tmem, da, db, C::IDESC, sfa_t + 4 * kk, sfb_t + kk * C::SFB_COLS_PER_KB + sfb_off, accum);
            if (C::DUAL) {
              const uint64_t db2 = tc::desc_sw128(st + C::OFF_B2 + at * C::B_ATOM) + 2 * sl;
              tc::mma_mxf4nvf4(tmem + C::BN, da, db2, C::IDESC, sfa_t + 4 * kk,
                               sfb2_t + kk * C::SFB_COLS_PER_KB + sfb_off, accum);
            }
          }
          tc::commit(bar_empty + 8 * s);
        }
        tc::commit(bar_accf);
      }
    }
  } else if (warp >= 6) {
    // ------------------- scale warps (SFST == 1 only) -------------------
    // Each warp copies, for its tensor-memory lane quarter, the 16 bytes of
    // every 512-byte scale block of the stage (row `lane` of the block) into 4
    // consecutive columns: the same image a 32x128b.warpx4 copy would make.
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t it = 0;
    bool dead = false;
    for (int t = blockIdx.x; t < P.total_tiles; t += gridDim.x) {
      const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
      const int nk64 = G.K / 64;
      const int nks = (nk64 + C::KPS - 1) / C::KPS;
      for (int ks = 0; ks < nks; ++ks, ++it) {
        const int s = it % C::STAGES;
        if (!dead && !mbar_wait((C::SEPSF ? bar_sff : bar_full) + 8 * s, (it / C::STAGES) & 1, P.err,
                                kDevErrTimeoutFull))
          dead = true;
        if (dead) break;
        const uint8_t* st = smem_raw + (sbase - raw) + s * C::STAGE_BYTES;
        const int nch = min(C::KPS, nk64 - C::KPS * ks);
        const uint32_t sf = tmem + lane_base + C::SF_BASE + s * C::SF_STAGE_COLS;
        const uint32_t sfa_t = sf, sfb_t = sf + C::SFA_COLS, sfb2_t = sf + C::SFA_COLS + C::KPS * C::SFB_COLS_PER_KB;
        for (int kk = 0; kk < nch && !(C::DBG & 1); ++kk) {
          uint4 v = *reinterpret_cast<const uint4*>(st + C::OFF_SFA + kk * 512 + lane * 16);
          tc::st_32x32b_x4(sfa_t + 4 * kk, v.x, v.y, v.z, v.w);
#pragma unroll
          for (int nb = 0; nb < C::NB; ++nb) {
            v = *reinterpret_cast<const uint4*>(st + C::OFF_SFB + nb * C::SFB_ROWTILE + kk * 512 + lane * 16);
            tc::st_32x32b_x4(sfb_t + kk * C::SFB_COLS_PER_KB + 4 * nb, v.x, v.y, v.z, v.w);
            if (C::DUAL) {
              v = *reinterpret_cast<const uint4*>(st + C::OFF_SFB2 + nb * C::SFB_ROWTILE + kk * 512 + lane * 16);
              tc::st_32x32b_x4(sfb2_t + kk * C::SFB_COLS_PER_KB + 4 * nb, v.x, v.y, v.z, v.w);
            }
          }
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_sfr + 8 * s);
      }
      if (dead) break;
    }
  } else {
    // ---------------------------- epilogue ----------------------------
    const int sub = warp & 3;                 // tensor-memory lane quarter of this warp
    const uint32_t lane_base = (uint32_t)(sub * 32) << 16;
    uint32_t tile_it = 0;
    for (int t = blockIdx.x; t < P.total_tiles; t += gridDim.x, ++tile_it) {
      const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
      const int local = t - G.tile_begin;
      const int mt = local % G.tiles_m, nt = local / G.tiles_m;
      if (!mbar_wait(bar_accf, tile_it & 1, P.err, kDevErrTimeoutMma)) break;
      tc::fence_after_sync();
      const int rloc = sub * 32 + lane;        // row of the tile held by this thread
      const int row = mt * BM + rloc;
      if constexpr (C::TRANS) {
        // C^T: this thread's accumulator row is output column `row`; its BN
        // columns are tokens.  A warp stores 32 consecutive output columns of
        // one token per instruction.
        constexpr int CHUNK = C::BN < 32 ? C::BN : 32;
#pragma unroll 1
        for (int cb = 0; cb < C::BN / CHUNK; ++cb) {
          uint32_t v[32];
          if constexpr (CHUNK == 32) tc::ld_32x32b_x32(tmem + lane_base + cb * 32, v);
          else tc::ld_32x32b_x16(tmem + lane_base + cb * CHUNK, v);
          tc::wait_ld();
          if (cb == C::BN / CHUNK - 1) {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acce);
          }
          if (row < G.M) {
#pragma unroll
            for (int j = 0; j < CHUNK; ++j) {
              const int tok = nt * C::BN + cb * CHUNK + j;
              if (tok < G.N) G.c[(int64_t)tok * G.ldc + row] = __float2half_rn(__uint_as_float(v[j]));
            }
          }
        }
        continue;
      }
      if (!(C::EPI && G.tma_store) && !(C::DBG & 8) && !C::DUAL) {
        // Drain the whole accumulator row into registers (packed fp16) and
        // release it before storing anything, so the next tile's MMAs run while
        // this tile's global stores drain.  Storing chunk by chunk between the
        // tensor-memory loads held the accumulator ~3 us per tile (the 16-byte
        // row-strided stores are slow to issue).  The dual GEMM keeps the
        // chunked order below: with ~1.5 tiles per CTA its last epilogue is on
        // the critical path, where interleaving loads and stores is shorter
        // (31.7 vs 33.4 us on the dual workload; 74.1 vs 74.9 grouped).
        uint32_t h[C::BN / 2];
#pragma unroll
        for (int cb = 0; cb < C::BN / 16; ++cb) {   // 16 columns per load keeps the live set small
          uint32_t v[32];
          tc::ld_32x32b_x16(tmem + lane_base + cb * 16, v);
          tc::wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) h[cb * 8 + j] = pack_h2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_acce);
        if (row < G.M) {
          __half* crow = G.c + (int64_t)row * G.ldc + (int64_t)nt * C::BN;
          const int col0 = nt * C::BN;
          const bool vec = col0 + C::BN <= G.N && G.vec_ok;
#pragma unroll
          for (int q = 0; q < C::BN / 8; ++q) {   // 8 columns per piece; h stays register-indexed
            if (vec) {
              reinterpret_cast<uint4*>(crow)[q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
            } else if (col0 + 8 * q < G.N) {
              store_piece(crow + 8 * q, make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]),
                          min(8, G.N - col0 - 8 * q));
            }
          }
        }
        continue;
      }
      if (C::EPI && G.tma_store) {
        // previous tile's TMA stores must have finished reading the staging tile
        if (threadIdx.x == 64) bulk_wait_read_all();
        asm volatile("bar.sync 2, 128;" ::: "memory");
      }
      __half* crow = G.c + (int64_t)row * G.ldc + (int64_t)nt * C::BN;
#pragma unroll 1
      for (int cb = 0; cb < C::BN / 32 && !(C::DBG & 8); ++cb) {
        uint32_t v[32];
        tc::ld_32x32b_x32(tmem + lane_base + cb * 32, v);
        uint32_t h[16];
        if constexpr (C::DUAL) {
          uint32_t u[32];
          tc::ld_32x32b_x32(tmem + lane_base + C::BN + cb * 32, u);
          tc::wait_ld();
          if (cb == C::BN / 32 - 1) {   // accumulator fully read: let the next tile's MMAs start
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acce);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j)
            h[j] = pack_h2(silu_mul(__uint_as_float(v[2 * j]), __uint_as_float(u[2 * j])),
                           silu_mul(__uint_as_float(v[2 * j + 1]), __uint_as_float(u[2 * j + 1])));
        } else {
          tc::wait_ld();
          if (cb == C::BN / 32 - 1) {
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_acce);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) h[j] = pack_h2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        }
        if (C::EPI && G.tma_store) {
          // box cb/2 holds 64 columns: row rloc at 128 * rloc, 16-byte chunk q at (q ^ (rloc % 8))
          uint8_t* box = smem_raw + C::OFF_C + (cb >> 1) * (BM * 128) + rloc * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = ((cb & 1) * 4 + q) ^ (rloc & 7);
            *reinterpret_cast<uint4*>(box + chunk * 16) = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
          }
          continue;
        }
        const int col0 = nt * C::BN + cb * 32;
        if (row < G.M) {
          if (col0 + 32 <= G.N && G.vec_ok) {
            uint4* dst = reinterpret_cast<uint4*>(crow + cb * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
          } else {
            const __half* hs = reinterpret_cast<const __half*>(h);
            for (int j = 0; j < 32 && col0 + j < G.N; ++j) crow[cb * 32 + j] = hs[j];
          }
        }
      }
      if (C::DBG & 8) {
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_acce);
      }
      if (C::EPI && G.tma_store && !(C::DBG & 8)) {
        fence_proxy_async_smem();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          for (int b = 0; b < C::BN / 64; ++b)
            tma_store_2d(&G.tc, sbase + C::OFF_C + b * (BM * 128), nt * C::BN + 64 * b, mt * BM);
          bulk_commit_group();
        }
      }
    }
    if (threadIdx.x == 64) bulk_wait_all();
  }
done:
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ===========================================================================
// CTA-pair variant (tcgen05.mma.cta_group::2).  A cluster of two CTAs on two
// SMs computes a 256 x BN tile: each CTA holds 128 rows of A and BN/2 rows of
// each B operand in its shared memory and the 128 x BN accumulator of its own
// rows in its tensor memory; the leader CTA (cluster rank 0) issues every MMA.
// Against the single-CTA kernel each CTA streams a third fewer bytes per FLOP
// (B is split across the pair instead of loaded by both), which is what the
// single-CTA kernel is limited by (shared-memory fill bandwidth per SM).
//   * each CTA loads its operand halves and its scale blocks with ordinary TMA
//     into its own shared memory on one local barrier (`sf_full`); the paired
//     .cta_group::2 load form, which completes on the leader's barrier,
//     measured slower (loads-only pipeline 65.6 vs 49.3 us on config 4);
//   * four scale warps per CTA wait for that barrier, write the scales into
//     this CTA's tensor memory in the
//     single-CTA arrangement (A: this CTA's 128 rows; B: all BN rows of the
//     tile, 4 columns per 128-row block, replicated in every lane quarter),
//     then arrive on the leader's `sf_ready` barrier across the cluster: that
//     arrival tells the leader this CTA's whole stage is ready;
//   * the leader commits each stage to both CTAs' `empty` barriers and each
//     finished accumulator to both CTAs' `accf` with one multicast commit; the
//     scale warps and the epilogue warps of each CTA meet at a named barrier
//     and send one arrival per CTA to the leader (`sf_ready`, `acce`).
// ===========================================================================
template <int BN_, bool DUAL_, int STAGES_, int DBG_ = 0, int SFTMA_ = 1, int KA_ = 1>
struct Gemm2Cfg {
  static constexpr int KA = KA_;                           // 128-byte K atoms per stage (as in GemmCfg)
  static constexpr int SFTMA = SFTMA_;
  static constexpr int DBG = DBG_;                         // tuning knob as in GemmCfg (0 in the product)
  static constexpr int BN = BN_;                           // N per pair MMA (per B operand)
  static constexpr bool DUAL = DUAL_;
  static constexpr int STAGES = STAGES_;
  static constexpr int HB = BN / 2;                        // B rows per CTA
  static constexpr int KPS = 4 * KA_;                      // 64-element K blocks per stage
  static constexpr int NB = (BN + 127) / 128;              // 128-row scale blocks of B per tile
  static constexpr int A_ATOM = BM * KSTEP_BYTES;
  static constexpr int B_ATOM = HB * KSTEP_BYTES;
  static constexpr int A_BYTES = KA * A_ATOM;
  static constexpr int B_BYTES = KA * B_ATOM;
  static constexpr int OFF_B = A_BYTES;
  static constexpr int OFF_B2 = OFF_B + B_BYTES;
  static constexpr int OFF_SFA = OFF_B2 + (DUAL ? B_BYTES : 0);
  static constexpr int SFA_BYTES = KPS * 512;
  static constexpr int SFB_ROWTILE = KPS * 512;
  static constexpr int OFF_SFB = OFF_SFA + SFA_BYTES;
  static constexpr int SFB_BYTES = NB * SFB_ROWTILE;
  static constexpr int OFF_SFB2 = OFF_SFB + SFB_BYTES;
  static constexpr int STAGE_BYTES = ((OFF_SFB2 + (DUAL ? SFB_BYTES : 0)) + 1023) / 1024 * 1024;
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int NBARS = 5 * STAGES + 2;
  static constexpr int SMEM = OFF_BAR + NBARS * 8 + 16;
  static constexpr int ACC_COLS = DUAL ? 2 * BN : BN;
  static constexpr int SF_BASE = ACC_COLS;
  static constexpr int SFBC = NB * 4;                      // B-scale columns per 64-element K block
  static constexpr int SFA_COLS = 4 * KPS;
  static constexpr int SF_STAGE_COLS = SFA_COLS + KPS * SFBC * (DUAL ? 2 : 1);
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 320;
  static constexpr bool PAIR = true;
  static constexpr int TILE_M = 2 * BM;
  static constexpr int B_BOX = HB;
  static constexpr uint32_t IDESC = tc::idesc_mxf4nvf4(256, BN);
  static constexpr uint32_t TX_AB = 2u * (A_BYTES + B_BYTES * (DUAL ? 2 : 1));   // both CTAs' operand bytes
  static_assert(BN % 64 == 0 && BN <= 256 && (BN % 128 == 0 || BN == 64), "pair tile N");
  static_assert(KA == 1 || SFTMA_, "wide stages load scales by tensor map");
  static_assert(SF_BASE + STAGES * SF_STAGE_COLS <= TMEM_COLS, "tensor memory budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <class C, int MAXG>
__global__ void __launch_bounds__(C::THREADS, 1) gemm2_kernel(const __grid_constant__ GemmParams<MAXG> P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const uint32_t pair = cluster_id_x(), npairs = nclusters_x();
  if (sbase & 1023u) {  // a uniform condition: both CTAs of a pair leave together
    if (threadIdx.x == 0) atomicOr(P.err, kDevErrTimeoutMma);
    return;
  }
  const uint32_t bar_full = sbase + C::OFF_BAR;            // leader: both CTAs' operand bytes
  const uint32_t bar_sff = bar_full + 8 * C::STAGES;       // local: this CTA's scale bytes
  const uint32_t bar_empty = bar_sff + 8 * C::STAGES;      // local: stage consumed by the pair MMAs
  const uint32_t bar_sfr = bar_empty + 8 * C::STAGES;      // leader: scales of both CTAs in tensor memory
  const uint32_t bar_accf = bar_sfr + 8 * C::STAGES;       // local: accumulator ready
  const uint32_t bar_acce = bar_accf + 8;                  // leader: both epilogues drained
  const uint32_t bar_opf = bar_acce + 8;                   // local: this CTA's operand bytes
  const uint32_t tmem_slot = bar_opf + 8 * C::STAGES;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_sff + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
      mbar_init(bar_sfr + 8 * s, 2);
      mbar_init(bar_opf + 8 * s, 1);
    }
    mbar_init(bar_accf, 1);
    mbar_init(bar_acce, 2);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tc::tmem_relinquish_pair();
  }
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync();   // barriers of both CTAs initialised before any cross-CTA arrival
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - sbase));

  if (warp == 0) {
    // --------------------------- producer (both CTAs) ---------------------------
    if (lane == 0) {
      for (int i = 0; i < P.ngroups; ++i) {
        prefetch_tmap(&P.g[i].ta);
        prefetch_tmap(&P.g[i].tb);
        if (C::DUAL) prefetch_tmap(&P.g[i].tb2);
        if (C::SFTMA) {
          prefetch_tmap(&P.g[i].tsa);
          prefetch_tmap(&P.g[i].tsb);
          if (C::DUAL) prefetch_tmap(&P.g[i].tsb2);
        }
      }
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_first();
      uint32_t it = 0;
      for (int t = pair; t < P.total_tiles; t += npairs) {
        const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
        const int local = t - G.tile_begin;
        const int mt = local % G.tiles_m, nt = local / G.tiles_m;
        const int nk64 = G.K / 64, nks = (nk64 + C::KPS - 1) / C::KPS;
        const int rt_a = mt * 2 + (int)cta;
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(bar_empty + 8 * s, ((it / C::STAGES) & 1) ^ 1, P.err, kDevErrTimeoutEmpty)) goto done;
          const uint32_t st = sbase + s * C::STAGE_BYTES;
          const uint32_t fb_leader = mapa(bar_full + 8 * s, 0);
          if (C::DBG & 4) {
            mbar_arrive(bar_sff + 8 * s);
            mbar_arrive(bar_opf + 8 * s);
            continue;
          }
          // this CTA's scales first, on their own local barrier, so the scale
          // warps stage them into tensor memory while the operands are in flight
          const uint32_t lb = bar_sff + 8 * s, ob = bar_opf + 8 * s;
          mbar_arrive_expect_tx(lb, (C::DBG & 16) ? 0 : C::SFA_BYTES + C::SFB_BYTES * (C::DUAL ? 2 : 1));
          mbar_arrive_expect_tx(ob, C::TX_AB / 2);
#pragma unroll
          for (int a = 0; a < C::KA; ++a) {
            const int x = (ks * C::KA + a) * KSTEP_BYTES;
            tma_load_2d(st + a * C::A_ATOM, &G.ta, ob, x, rt_a * BM, pol_a);
            tma_load_2d(st + C::OFF_B + a * C::B_ATOM, &G.tb, ob, x, nt * C::BN + (int)cta * C::HB, pol_b);
            if (C::DUAL)
              tma_load_2d(st + C::OFF_B2 + a * C::B_ATOM, &G.tb2, ob, x, nt * C::BN + (int)cta * C::HB, pol_b);
          }
          if (!(C::DBG & 16)) {
            if (C::SFTMA) {
              tma_load_3d(st + C::OFF_SFA, &G.tsa, lb, 0, C::KPS * ks, rt_a, pol_a);
              tma_load_3d(st + C::OFF_SFB, &G.tsb, lb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
              if (C::DUAL) tma_load_3d(st + C::OFF_SFB2, &G.tsb2, lb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
            } else {
              load_sf_bulk<C>(st, G, rt_a, (nt * C::BN) / 128, nk64, ks, lb);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA (leader) ------------------------------
    if (lane == 0 && cta == 0) {
      uint32_t it = 0, tile_it = 0;
      for (int t = pair; t < P.total_tiles; t += npairs, ++tile_it) {
        const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
        const int nk64 = G.K / 64, nks = (nk64 + C::KPS - 1) / C::KPS;
        const uint32_t sfb_off = (uint32_t)((((t - G.tile_begin) / G.tiles_m) * C::BN) % 128) / 32;
        if (!mbar_wait_cluster(bar_acce, (tile_it & 1) ^ 1, P.err, kDevErrTimeoutMma)) goto done;
        tc::fence_after_sync();
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          // both CTAs' operands landed and their scales are in tensor memory
          if (!mbar_wait_cluster(bar_sfr + 8 * s, ph, P.err, kDevErrTimeoutFull)) goto done;
          tc::fence_after_sync();
          const uint32_t st = sbase + s * C::STAGE_BYTES;
          const int nch = min(C::KPS, nk64 - C::KPS * ks);
          const uint32_t sf = tmem + C::SF_BASE + s * C::SF_STAGE_COLS;
          const uint32_t sfa_t = sf, sfb_t = sf + C::SFA_COLS, sfb2_t = sf + C::SFA_COLS + C::KPS * C::SFBC;
          for (int kk = 0; kk < nch && !(C::DBG & 2); ++kk) {
            const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
            const int at = kk >> 2, sl = kk & 3;   // K atom of the stage, 64-element slice in it
            const uint64_t da = tc::desc_sw128(st + at * C::A_ATOM) + 2 * sl;
            const uint64_t db = tc::desc_sw128(st + C::OFF_B + at * C::B_ATOM) + 2 * sl;
            tc::mma_mxf4nvf4_pair(tmem, da, db, C::IDESC, sfa_t + 4 * kk, sfb_t + kk * C::SFBC + sfb_off, accum);
            if (C::DUAL) {
              const uint64_t db2 = tc::desc_sw128(st + C::OFF_B2 + at * C::B_ATOM) + 2 * sl;
              tc::mma_mxf4nvf4_pair(tmem + C::BN, da, db2, C::IDESC, sfa_t + 4 * kk,
                                    sfb2_t + kk * C::SFBC + sfb_off, accum);
            }
          }
          tc::commit_pair_both(bar_empty + 8 * s, 3);
        }
        tc::commit_pair_both(bar_accf, 3);
      }
    }
  } else if (warp >= 6) {
    // --------------------------- scale warps (both CTAs) ---------------------------
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t sfr_leader = mapa(bar_sfr, 0);
    uint32_t it = 0;
    for (int t = pair; t < P.total_tiles; t += npairs) {
      const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
      const int nk64 = G.K / 64, nks = (nk64 + C::KPS - 1) / C::KPS;
      for (int ks = 0; ks < nks; ++ks, ++it) {
        const int s = it % C::STAGES;
        if (!mbar_wait(bar_sff + 8 * s, (it / C::STAGES) & 1, P.err, kDevErrTimeoutFull)) goto done;
        const uint8_t* st = smem_raw + s * C::STAGE_BYTES;
        const int nch = min(C::KPS, nk64 - C::KPS * ks);
        const uint32_t sf = tmem + lane_base + C::SF_BASE + s * C::SF_STAGE_COLS;
        const uint32_t sfa_t = sf, sfb_t = sf + C::SFA_COLS, sfb2_t = sf + C::SFA_COLS + C::KPS * C::SFBC;
        for (int kk = 0; kk < nch && !(C::DBG & 1); ++kk) {
          const uint4 v = *reinterpret_cast<const uint4*>(st + C::OFF_SFA + kk * 512 + lane * 16);
          tc::st_32x32b_x4(sfa_t + 4 * kk, v.x, v.y, v.z, v.w);
          // B scales: every 128-row block of the tile into 4 columns, in every
          // lane quarter (the same image as for a single-CTA MMA of N = BN)
#pragma unroll
          for (int op = 0; op < (C::DUAL ? 2 : 1); ++op) {
#pragma unroll
            for (int nb = 0; nb < C::NB; ++nb) {
              const uint4 w = *reinterpret_cast<const uint4*>(st + (op ? C::OFF_SFB2 : C::OFF_SFB) +
                                                              nb * C::SFB_ROWTILE + kk * 512 + lane * 16);
              tc::st_32x32b_x4((op ? sfb2_t : sfb_t) + kk * C::SFBC + 4 * nb, w.x, w.y, w.z, w.w);
            }
          }
        }
        tc::wait_st();
        tc::fence_before_sync();
        asm volatile("bar.sync 3, 128;" ::: "memory");     // the 4 scale warps of this CTA
        // once this CTA's operands landed too, its whole stage is ready for the
        // pair MMA (an expired wait is recorded and the arrival skipped: the
        // leader's own bounded wait then ends the pipeline)
        if (threadIdx.x == 192 && mbar_wait(bar_opf + 8 * s, (it / C::STAGES) & 1, P.err, kDevErrTimeoutFull))
          mbar_arrive_cluster(sfr_leader + 8 * s);
      }
    }
  } else {
    // ----------------------------- epilogue (both CTAs) -----------------------------
    const int sub = warp & 3;
    const uint32_t lane_base = (uint32_t)(sub * 32) << 16;
    const uint32_t acce_leader = mapa(bar_acce, 0);
    uint32_t tile_it = 0;
    for (int t = pair; t < P.total_tiles; t += npairs, ++tile_it) {
      const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
      const int local = t - G.tile_begin;
      const int mt = local % G.tiles_m, nt = local / G.tiles_m;
      if (!mbar_wait(bar_accf, tile_it & 1, P.err, kDevErrTimeoutMma)) break;
      tc::fence_after_sync();
      const int row = mt * 256 + (int)cta * BM + sub * 32 + lane;
      __half* crow = G.c + (int64_t)row * G.ldc + (int64_t)nt * C::BN;
      // whole accumulator row -> packed fp16 registers, release, then store
      uint32_t h[C::BN / 2];
#pragma unroll
      for (int cb = 0; cb < C::BN / 16; ++cb) {
        uint32_t v[32];
        tc::ld_32x32b_x16(tmem + lane_base + cb * 16, v);
        if constexpr (C::DUAL) {
          uint32_t u[32];
          tc::ld_32x32b_x16(tmem + lane_base + C::BN + cb * 16, u);
          tc::wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            h[cb * 8 + j] = pack_h2(silu_mul(__uint_as_float(v[2 * j]), __uint_as_float(u[2 * j])),
                                    silu_mul(__uint_as_float(v[2 * j + 1]), __uint_as_float(u[2 * j + 1])));
        } else {
          tc::wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) h[cb * 8 + j] = pack_h2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        }
      }
      tc::fence_before_sync();
      asm volatile("bar.sync 4, 128;" ::: "memory");   // the 4 epilogue warps of this CTA
      if (threadIdx.x == 64) mbar_arrive_cluster(acce_leader);
      if (row < G.M) {
        const int col0 = nt * C::BN;
        const bool vec = col0 + C::BN <= G.N && G.vec_ok;
#pragma unroll
        for (int q = 0; q < C::BN / 8; ++q) {
          if (vec)
            reinterpret_cast<uint4*>(crow)[q] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
          else if (col0 + 8 * q < G.N)
            store_piece(crow + 8 * q, make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]),
                        min(8, G.N - col0 - 8 * q));
        }
      }
    }
  }
done:
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync();   // the leader's MMAs read this CTA's shared memory until here
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

}  // namespace

namespace {

template <class C, int MAXG>
int launch_gemm(const GemmParams<MAXG>& P, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<C, MAXG>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
    attr_set[dev] = true;
  }
  int grid = sm_count();
  if (P.total_tiles < grid) grid = P.total_tiles;
  if (grid < 1) return NVFP4_OK;
  gemm_kernel<C, MAXG><<<grid, C::THREADS, C::SMEM, stream>>>(P);
  return check_launch("gemm_kernel");
}

template <class C, int MAXG>
int launch_gemm2(const GemmParams<MAXG>& P, cudaStream_t stream) {
  static bool attr_set[64] = {};
  static int max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm2_kernel<C, MAXG>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dev >= 64) return fail(NVFP4_ERR_UNSUPPORTED, "device index out of range");
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm2)");
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n < 1) return fail(NVFP4_ERR_UNSUPPORTED, "no CTA pairs fit on this device");
    max_pairs[dev] = n;
    attr_set[dev] = true;
  }
  int pairs = max_pairs[dev];
  if (P.total_tiles < pairs) pairs = P.total_tiles;
  if (pairs < 1) return NVFP4_OK;
  cfg.gridDim = dim3(2 * pairs);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, P);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemm2)");
  return check_launch("gemm2_kernel");
}

template <class C, int MAXG>
int launch_any(const GemmParams<MAXG>& P, cudaStream_t stream) {
  if constexpr (C::PAIR) return launch_gemm2<C, MAXG>(P, stream);
  else return launch_gemm<C, MAXG>(P, stream);
}

int operand_map(CUtensorMap* m, const void* p, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  const uint64_t dims[2] = {(uint64_t)(K / 2), (uint64_t)rows};
  const uint64_t str[1] = {(uint64_t)ld};
  const uint32_t box[2] = {KSTEP_BYTES, (uint32_t)box_rows};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Blocked scales viewed as u32 [row tiles][K/64 blocks][128]: a box of
// {128, 4, n} is n row tiles x one 256-element K step (2 KB per row tile).
int sf_map(CUtensorMap* m, const void* sf, int64_t rows, int64_t K, int box_tiles, int box_kb = 4) {
  const uint64_t nk64 = (uint64_t)(K / 64);
  const uint64_t dims[3] = {128, nk64, (uint64_t)((rows + 127) / 128)};
  const uint64_t str[2] = {512, nk64 * 512};
  const uint32_t box[3] = {128, (uint32_t)box_kb, (uint32_t)box_tiles};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, sf, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int check_operand(const char* name, const void* p, const void* sf, int64_t rows, int64_t K, int64_t ld) {
  if (!p || !sf) return fail(NVFP4_ERR_INVALID, "%s: null pointer", name);
  if (rows < 1) return fail(NVFP4_ERR_INVALID, "%s: need at least one row", name);
  if (ld < K / 2) return fail(NVFP4_ERR_INVALID, "%s: row stride %lld below K/2", name, (long long)ld);
  if (!aligned16(p) || !aligned16(sf) || ld % 16)
    return fail(NVFP4_ERR_ALIGNMENT, "%s: pointers and row stride must be multiples of 16 bytes", name);
  return NVFP4_OK;
}

int check_out(void* c, int64_t N, int64_t ldc) {
  if (!c) return fail(NVFP4_ERR_INVALID, "output: null pointer");
  if (ldc < N) return fail(NVFP4_ERR_INVALID, "output: ldc below N");
  if (reinterpret_cast<uintptr_t>(c) & 1) return fail(NVFP4_ERR_ALIGNMENT, "output: fp16 pointer not 2-byte aligned");
  return NVFP4_OK;
}

int vec_ok(const void* c, int64_t ldc) { return aligned16(c) && ldc % 8 == 0; }

// Output map for the TMA-store epilogue: fp16 [M, N], 64-column x 128-row boxes
// with 128-byte swizzle (the staging tile's layout).
int out_map(CUtensorMap* m, void* c, int64_t M, int64_t N, int64_t ldc) {
  const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
  const uint64_t str[1] = {(uint64_t)ldc * 2};
  const uint32_t box[2] = {64, (uint32_t)BM};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, c, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

namespace nvfp4 {
template <class C>
int dual_run(const void* a, const void* b1, const void* b2, const void* sfa, const void* sfb1,
             const void* sfb2, void* c, int64_t M, int64_t N, int64_t K, int64_t lda,
             int64_t ldb, int64_t ldc, void* stream) {
  if (K < 64 || K % 64) return fail(NVFP4_ERR_INVALID, "nvfp4_dual_gemm: K must be a positive multiple of 64");
  int rc;
  if ((rc = check_operand("a", a, sfa, M, K, lda)) || (rc = check_operand("b1", b1, sfb1, N, K, ldb)) ||
      (rc = check_operand("b2", b2, sfb2, N, K, ldb)) || (rc = check_out(c, N, ldc)))
    return rc;
  GemmParams<1> P;
  std::memset(&P, 0, sizeof(P));
  GemmGroup& G = P.g[0];
  if ((rc = operand_map(&G.ta, a, M, K, lda, BM)) || (rc = operand_map(&G.tb, b1, N, K, ldb, C::B_BOX)) ||
      (rc = operand_map(&G.tb2, b2, N, K, ldb, C::B_BOX)))
    return rc;
  if ((rc = sf_map(&G.tsa, sfa, M, K, 1, C::KPS)) || (rc = sf_map(&G.tsb, sfb1, N, K, C::NB, C::KPS)) ||
      (rc = sf_map(&G.tsb2, sfb2, N, K, C::NB, C::KPS)))
    return rc;
  G.sfa = static_cast<const uint8_t*>(sfa);
  G.sfb = static_cast<const uint8_t*>(sfb1);
  G.sfb2 = static_cast<const uint8_t*>(sfb2);
  G.c = static_cast<__half*>(c);
  G.ldc = ldc;
  G.vec_ok = vec_ok(c, ldc);
  G.tma_store = G.vec_ok && out_map(&G.tc, c, M, N, ldc) == NVFP4_OK;
  G.M = (int)M; G.N = (int)N; G.K = (int)K;
  G.tiles_m = (int)((M + C::TILE_M - 1) / C::TILE_M);
  G.tiles_n = (int)((N + C::BN - 1) / C::BN);
  G.tile_begin = 0;
  P.ngroups = 1;
  P.total_tiles = G.tiles_m * G.tiles_n;
  P.err = device_error_word();
  if (!P.err) return fail(NVFP4_ERR_CUDA, "nvfp4_dual_gemm: cannot resolve the device error word");
  return launch_any<C, 1>(P, static_cast<cudaStream_t>(stream));
}

}  // namespace nvfp4

extern "C" int nvfp4_dual_gemm(const void* a, const void* b1, const void* b2, const void* sfa, const void* sfb1,
                               const void* sfb2, void* c, int64_t M, int64_t N, int64_t K, int64_t lda,
                               int64_t ldb, int64_t ldc, void* stream) {
  // two 512-element K stages of 108 KB: half the stage handshakes of four 256-element
  // stages at the same bytes in flight (30.9 vs 33.3 us on the dual workload, same box)
  return dual_run<GemmCfg<128, true, 2, 0, 1, 0, 0, 1, 1, 0, 2>>(a, b1, b2, sfa, sfb1, sfb2, c, M, N, K, lda, ldb,
                                                                   ldc, stream);
}

namespace nvfp4 {
// out[T, N] = X[T, K] . W[N, K]^T for T <= BN tokens: W streams as the MMA's A
// operand (128 weight rows per tile), X is one BN-row B tile, C^T epilogue.
template <class C>
int skinny_run(const void* x, const void* w, const void* sfx, const void* sfw, void* out, int64_t T, int64_t N,
               int64_t K, int64_t ldx, int64_t ldw, int64_t ldo, void* stream) {
  if (K < 64 || K % 64) return fail(NVFP4_ERR_INVALID, "nvfp4_gemm_skinny: K must be a positive multiple of 64");
  int rc;
  if ((rc = check_operand("x", x, sfx, T, K, ldx)) || (rc = check_operand("w", w, sfw, N, K, ldw)) ||
      (rc = check_out(out, N, ldo)))
    return rc;
  GemmParams<1> P;
  std::memset(&P, 0, sizeof(P));
  GemmGroup& G = P.g[0];
  if ((rc = operand_map(&G.ta, w, N, K, ldw, BM)) || (rc = operand_map(&G.tb, x, T, K, ldx, C::BN)) ||
      (rc = sf_map(&G.tsa, sfw, N, K, 1, C::KPS)) || (rc = sf_map(&G.tsb, sfx, T, K, 1, C::KPS)))
    return rc;
  G.sfa = static_cast<const uint8_t*>(sfw);
  G.sfb = static_cast<const uint8_t*>(sfx);
  G.c = static_cast<__half*>(out);
  G.ldc = ldo;
  G.M = (int)N;
  G.N = (int)T;
  G.K = (int)K;
  G.tiles_m = (int)((N + BM - 1) / BM);
  G.tiles_n = 1;
  P.ngroups = 1;
  P.total_tiles = G.tiles_m;
  P.err = device_error_word();
  if (!P.err) return fail(NVFP4_ERR_CUDA, "nvfp4_gemm_skinny: cannot resolve the device error word");
  return launch_any<C, 1>(P, static_cast<cudaStream_t>(stream));
}

template <class C, int MAXG>
int grouped_launches(const nvfp4_group* groups, int num_groups, void* stream) {
  uint32_t* err = device_error_word();
  if (!err) return fail(NVFP4_ERR_CUDA, "nvfp4_grouped_gemm: cannot resolve the device error word");
  static GemmParams<MAXG> P;          // large; built under a lock, copied into the launch
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  for (int g0 = 0; g0 < num_groups; g0 += MAXG) {
    std::memset(&P, 0, sizeof(P));
    int tiles = 0, n = 0;
    for (int i = g0; i < num_groups && n < MAXG; ++i) {
      const nvfp4_group& q = groups[i];
      if (q.M == 0) continue;
      int rc;
      if (q.K < 64 || q.K % 64 || q.N < 1 || q.M < 0)
        return fail(NVFP4_ERR_INVALID, "group %d: need M>=0, N>=1 and K a positive multiple of 64", i);
      if ((rc = check_operand("a", q.a, q.sfa, q.M, q.K, q.lda)) ||
          (rc = check_operand("b", q.b, q.sfb, q.N, q.K, q.ldb)) || (rc = check_out(q.c, q.N, q.ldc)))
        return rc;
      GemmGroup& G = P.g[n];
      if ((rc = operand_map(&G.ta, q.a, q.M, q.K, q.lda, BM)) || (rc = operand_map(&G.tb, q.b, q.N, q.K, q.ldb, C::B_BOX)))
        return rc;
      if ((rc = sf_map(&G.tsa, q.sfa, q.M, q.K, 1, C::KPS)) || (rc = sf_map(&G.tsb, q.sfb, q.N, q.K, C::NB, C::KPS)))
        return rc;
      G.sfa = static_cast<const uint8_t*>(q.sfa);
      G.sfb = static_cast<const uint8_t*>(q.sfb);
      G.c = static_cast<__half*>(q.c);
      G.ldc = q.ldc;
      G.vec_ok = vec_ok(q.c, q.ldc);
      G.tma_store = G.vec_ok && out_map(&G.tc, q.c, q.M, q.N, q.ldc) == NVFP4_OK;
      G.M = (int)q.M; G.N = (int)q.N; G.K = (int)q.K;
      G.tiles_m = (int)((q.M + C::TILE_M - 1) / C::TILE_M);
      G.tiles_n = (int)((q.N + C::BN - 1) / C::BN);
      G.tile_begin = tiles;
      tiles += G.tiles_m * G.tiles_n;
      ++n;
    }
    if (n == 0) continue;
    P.ngroups = n;
    P.total_tiles = tiles;
    P.err = err;
    int rc = launch_any<C, MAXG>(P, static_cast<cudaStream_t>(stream));
    if (rc) return rc;
  }
  return NVFP4_OK;
}

// The kernel parameters carry every group's tensor maps (about 1 KB a group):
// up to 8 groups launch with an 8-group parameter block instead of paying for
// 24 groups' worth on every launch.
template <class C>
int grouped_run(const nvfp4_group* groups, int num_groups, void* stream) {
  if (!groups || num_groups < 1) return fail(NVFP4_ERR_INVALID, "nvfp4_grouped_gemm: no groups");
  if (num_groups <= 8) return grouped_launches<C, 8>(groups, num_groups, stream);
  return grouped_launches<C, 24>(groups, num_groups, stream);
}
}  // namespace nvfp4

extern "C" int nvfp4_grouped_gemm(const nvfp4_group* groups, int num_groups, void* stream) {
  return grouped_run<GemmCfg<256, false, 4, 0, 1, 0, 0>>(groups, num_groups, stream);
}

extern "C" int nvfp4_gemm_skinny(const void* x, const void* w, const void* sfx, const void* sfw, void* out,
                                 int64_t T, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldo,
                                 void* stream) {
  if (T < 1 || T > 64) return fail(NVFP4_ERR_INVALID, "nvfp4_gemm_skinny: 1..64 token rows (got %lld)", (long long)T);
  // 512-element K stages (32 KB of weights each): half the per-stage handshakes of
  // 256-element stages (13.8 vs 16.3 us at T=16, N=14336, K=4096)
  if (T <= 16)
    return skinny_run<GemmCfg<16, false, 4, 0, 1, 0, 0, 1, 1, 1, 2>>(x, w, sfx, sfw, out, T, N, K, ldx, ldw, ldo, stream);
  if (T <= 32)
    return skinny_run<GemmCfg<32, false, 4, 0, 1, 0, 0, 1, 1, 1, 2>>(x, w, sfx, sfw, out, T, N, K, ldx, ldw, ldo, stream);
  return skinny_run<GemmCfg<64, false, 4, 0, 1, 0, 0, 1, 1, 1, 2>>(x, w, sfx, sfw, out, T, N, K, ldx, ldw, ldo, stream);
}

// ---------------------------------------------------------------------------
// FP4 tensor-core peak probe: every CTA (one per SM) issues `iters` dense
// 128x256x64 kind::mxf4nvf4 MMAs back to back from shared memory into one
// tensor-memory accumulator, with nothing else in the loop.  The operand bytes
// are whatever shared memory holds; only the issue rate matters.  It gives the
// denominator of the GEMMs' tensor-core roofline fraction.
// ---------------------------------------------------------------------------
namespace nvfp4 {
namespace {
// Dense FP4 throughput probe: back-to-back 128x256x64 kind::mxf4nvf4 MMAs
// on every SM.  pattern 0: one fixed scale column pair and whatever shared
// memory holds.  pattern 1 (the GEMMs' conditions): pseudo-random operand
// bytes, e4m3 scales in 2^[-3, 3], and the scale columns advancing per K
// step through four 48-column stages exactly as the GEMM's tensor-memory
// layout does.  The tensor pipe's rate depends on both.
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int iters, int pattern, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  const uint32_t bar = sbase + 49152;
  const uint32_t slot = bar + 8;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(slot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem_raw + (slot - raw));
  if (pattern == 1) {
    uint32_t* ops = reinterpret_cast<uint32_t*>(smem_raw + (sbase - raw));
    for (int i = threadIdx.x; i < 49152 / 4; i += blockDim.x) {
      uint32_t x = (uint32_t)i * 2654435761u ^ (blockIdx.x * 40503u);
      x ^= x >> 15; x *= 0x2c1b3c6du; x ^= x >> 12;
      ops[i] = x;
    }
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    for (int c = 256; c < 256 + 4 * 48; c += 2) {   // each warp: its 32-lane quarter, two columns per store
      const uint32_t x = (uint32_t)(c * 131 + (threadIdx.x & 31) * 7 + blockIdx.x);
      uint32_t v = 0;
      for (int b = 0; b < 4; ++b) v |= (((x >> (3 * b)) % 7u) + 4u) << 3 << (8 * b);   // bytes 0x20..0x50: 2^-3 .. 2^3
      tc::st_32x32b_x2(tmem + lane_base + c, v, v ^ 0x08080808u);
    }
    tc::wait_st();
    fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }
  if (threadIdx.x == 0) {
    const uint64_t da = tc::desc_sw128(sbase), db = tc::desc_sw128(sbase + 16384);
    const uint32_t idesc = tc::idesc_mxf4nvf4(128, 256);
    for (int i = 0; i < iters; ++i) {
      const int k = i & 3;
      const uint32_t st = 256u + 48u * (uint32_t)((i >> 2) & 3);
      const uint32_t sfa = pattern ? st + 4 * k : 256u, sfb = pattern ? st + 16 + 8 * k : 272u;
      tc::mma_mxf4nvf4(tmem, da + 2 * k, db + 2 * k, idesc, tmem + sfa, tmem + sfb, i > 0 ? 1u : 0u);
    }
    tc::commit(bar);
    mbar_wait(bar, 0, err, kDevErrTimeoutMma);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}
}  // namespace
}  // namespace nvfp4

extern "C" int nvfp4_mma_peak_pattern(int iters, int pattern, void* stream) {
  if (iters < 1) return fail(NVFP4_ERR_INVALID, "nvfp4_mma_peak: iters must be positive");
  if (pattern != 0 && pattern != 1) return fail(NVFP4_ERR_INVALID, "nvfp4_mma_peak_pattern: pattern must be 0 or 1");
  uint32_t* err = device_error_word();
  if (!err) return fail(NVFP4_ERR_CUDA, "nvfp4_mma_peak: cannot resolve the device error word");
  constexpr int kSmem = 49152 + 64 + 1024;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(mma_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(mma_peak)");
    attr_set[dev] = true;
  }
  mma_peak_kernel<<<sm_count(), 128, kSmem, static_cast<cudaStream_t>(stream)>>>(iters, pattern, err);
  return check_launch("mma_peak_kernel");
}

extern "C" int nvfp4_mma_peak(int iters, void* stream) { return nvfp4_mma_peak_pattern(iters, 0, stream); }
