// The CTA-pair (cta_group::2) kernel of the grouped and dual GEMMs.  Included
// by gemm.cu only.
//
// A cluster of two CTAs on two SMs computes a 256 x BN output tile with
// 256 x BN x 64 pair MMAs issued by the leader (cluster rank 0).  Each CTA
// holds 128 rows of A and BN/2 rows of B (and of B2, dual GEMM) in its shared
// memory and the 128 x BN accumulator(s) of its own rows in its tensor memory.  Against the
// single-CTA kernel (128 x 256 tiles) every SM moves a third fewer operand
// bytes from L2 per FLOP (B is split across the pair instead of loaded by
// both).  Measured on config 4 on one box: 64.6 us against 68.5 us, outputs
// bit-identical.  Both are bound by the TMA round trip: a stage's operands
// land ~1.3 us after issue (per-stage %globaltimer stamps), and 5 stages of
// 38 KB (all of shared memory) cover ~0.35 us of MMAs each.
//   * each CTA's producer loads its operand halves (one local barrier, `full`)
//     and its scale blocks (`sff`: A scales of its 128 rows, B scales of all BN
//     rows) with ordinary TMA into its own shared memory, 5 stages of 38 KB;
//   * four scale warps per CTA copy the scales into this CTA's tensor memory
//     (tcgen05.st, the single-CTA image: B scales of all BN rows in every lane
//     quarter), wait for this CTA's operands, and send one arrival to the
//     leader's `sfr`: the stage is ready on this SM;
//   * the leader waits for both arrivals, issues the stage's pair MMAs
//     (unrolled) and commits the stage to both CTAs' `empty` barriers, and each
//     finished accumulator to both CTAs' `accf`, with one multicast commit;
//   * each CTA's epilogue drains its 128 accumulator rows into registers, sends
//     one arrival to the leader's `acce`, and stores them.
// No TMA load uses cluster multicast; every wait is bounded (2 s).
#pragma once

namespace nvfp4 {
namespace {

// DUAL: two B operands sharing A (the dual GEMM), SiLU-gated epilogue.
template <int BN_, int STAGES_, bool DUAL_ = false>
struct PairCfg {
  static constexpr int BN = BN_;                           // N per pair MMA (per B operand)
  static constexpr int STAGES = STAGES_;
  static constexpr bool DUAL = DUAL_;
  static constexpr int HB = BN / 2;                        // B rows per CTA
  static constexpr int KPS = 4;                            // 64-element K blocks per stage
  static constexpr int NB = (BN + 127) / 128;              // 128-row scale blocks of B per tile
  static constexpr int A_BYTES = BM * KSTEP_BYTES;         // 16 KB
  static constexpr int B_BYTES = HB * KSTEP_BYTES;
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
  static constexpr int NBARS = 4 * STAGES + 2;
  static constexpr int SMEM = OFF_BAR + NBARS * 8 + 16;
  static constexpr int SF_BASE = DUAL ? 2 * BN : BN;      // accumulator columns first
  static constexpr int SFBC = NB * 4;                      // B-scale columns per 64-element K block
  static constexpr int SFA_COLS = 4 * KPS;
  static constexpr int SF_STAGE_COLS = SFA_COLS + KPS * SFBC * (DUAL ? 2 : 1);
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 320;
  static constexpr bool PAIR = true;
  static constexpr int TILE_M = 2 * BM;
  static constexpr int B_BOX = HB;
  static constexpr uint32_t IDESC = tc::idesc_mxf4nvf4(256, BN);
  static constexpr uint32_t OP_BYTES = A_BYTES + B_BYTES * (DUAL ? 2 : 1);
  static constexpr uint32_t SF_BYTES = SFA_BYTES + SFB_BYTES * (DUAL ? 2 : 1);
  static_assert(BN % 128 == 0 && BN <= 256, "pair tile N: whole 128-row scale blocks");
  static_assert(SF_BASE + STAGES * SF_STAGE_COLS <= TMEM_COLS, "tensor memory budget");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(SMEM < (1 << 18), "descriptor address field");
};

template <class C, int MAXG>
__global__ void __launch_bounds__(C::THREADS, 1) pair_kernel(const __grid_constant__ GemmParams<MAXG> P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const uint32_t pair = cluster_id_x(), npairs = nclusters_x();
  if (sbase & 1023u) {  // the same layout in both CTAs: both leave together
    if (threadIdx.x == 0) atomicOr(P.err, kDevErrTimeoutMma);
    return;
  }
  const uint32_t bar_full = sbase + C::OFF_BAR;            // local: this CTA's operand bytes
  const uint32_t bar_sff = bar_full + 8 * C::STAGES;       // local: this CTA's scale bytes
  const uint32_t bar_empty = bar_sff + 8 * C::STAGES;      // local: stage consumed by the pair MMAs
  const uint32_t bar_sfr = bar_empty + 8 * C::STAGES;      // leader: both CTAs' stages ready
  const uint32_t bar_accf = bar_sfr + 8 * C::STAGES;       // local: accumulator ready
  const uint32_t bar_acce = bar_accf + 8;                  // leader: both epilogues drained
  const uint32_t tmem_slot = bar_acce + 8;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_sff + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
      mbar_init(bar_sfr + 8 * s, 2);
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
  cluster_sync();   // both CTAs' barriers initialised before any cross-CTA arrival
  tc::fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem_raw + (tmem_slot - sbase));

  if (warp == 0) {
    // --------------------------- producer (both CTAs) ---------------------------
    if (lane == 0) {
      for (int i = 0; i < P.ngroups; ++i) {
        prefetch_tmap(&P.g[i].ta);
        prefetch_tmap(&P.g[i].tb);
        prefetch_tmap(&P.g[i].tsa);
        prefetch_tmap(&P.g[i].tsb);
        if (C::DUAL) {
          prefetch_tmap(&P.g[i].tb2);
          prefetch_tmap(&P.g[i].tsb2);
        }
      }
      const uint64_t pol_a = policy_evict_last();   // A tiles are re-read by every N tile
      const uint64_t pol_b = policy_evict_first();
      uint32_t it = 0;
      for (int t = pair; t < P.total_tiles; t += npairs) {
        const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
        const int local = t - G.tile_begin;
        const int mt = local % G.tiles_m, nt = local / G.tiles_m;
        const int nks = G.K / KSTEP;                           // K is a multiple of 256 on this path
        const int rt_a = mt * 2 + (int)cta;                    // this CTA's 128-row block of A
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(bar_empty + 8 * s, ((it / C::STAGES) & 1) ^ 1, P.err, kDevErrTimeoutEmpty)) goto done;
          const uint32_t st = sbase + s * C::STAGE_BYTES;
          const uint32_t sb = bar_sff + 8 * s, fb = bar_full + 8 * s;
          mbar_arrive_expect_tx(sb, C::SF_BYTES);
          tma_load_3d(st + C::OFF_SFA, &G.tsa, sb, 0, C::KPS * ks, rt_a, pol_a);
          tma_load_3d(st + C::OFF_SFB, &G.tsb, sb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
          if (C::DUAL) tma_load_3d(st + C::OFF_SFB2, &G.tsb2, sb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
          mbar_arrive_expect_tx(fb, C::OP_BYTES);
          const int x = ks * KSTEP_BYTES;
          tma_load_2d(st, &G.ta, fb, x, rt_a * BM, pol_a);
          tma_load_2d(st + C::OFF_B, &G.tb, fb, x, nt * C::BN + (int)cta * C::HB, pol_b);
          if (C::DUAL) tma_load_2d(st + C::OFF_B2, &G.tb2, fb, x, nt * C::BN + (int)cta * C::HB, pol_b);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA (leader) ------------------------------
    if (lane == 0 && cta == 0) {
      const uint64_t da0 = tc::desc_sw128(sbase);
      const uint64_t db0 = tc::desc_sw128(sbase + C::OFF_B);
      const uint64_t db20 = tc::desc_sw128(sbase + C::OFF_B2);
      uint32_t it = 0, tile_it = 0;
      for (int t = pair; t < P.total_tiles; t += npairs, ++tile_it) {
        const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
        const int nks = G.K / KSTEP;
        if (!mbar_wait(bar_acce, (tile_it & 1) ^ 1, P.err, kDevErrTimeoutMma)) goto done;
        tc::fence_after_sync();
        for (int ks = 0; ks < nks; ++ks, ++it) {
          const int s = it % C::STAGES;
          // both CTAs' operands landed and their scales are in tensor memory
          if (!mbar_wait(bar_sfr + 8 * s, (it / C::STAGES) & 1, P.err, kDevErrTimeoutFull)) goto done;
          tc::fence_after_sync();
          const uint64_t soff = (uint64_t)((s * C::STAGE_BYTES) >> 4);
          const uint32_t sf = tmem + C::SF_BASE + s * C::SF_STAGE_COLS;
#pragma unroll
          for (int kk = 0; kk < C::KPS; ++kk) {
            const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
            tc::mma_mxf4nvf4_pair(tmem, da0 + soff + 2 * kk, db0 + soff + 2 * kk, C::IDESC, sf + 4 * kk,
                                  sf + C::SFA_COLS + kk * C::SFBC, accum);
            if (C::DUAL)
              tc::mma_mxf4nvf4_pair(tmem + C::BN, da0 + soff + 2 * kk, db20 + soff + 2 * kk, C::IDESC, sf + 4 * kk,
                                    sf + C::SFA_COLS + C::KPS * C::SFBC + kk * C::SFBC, accum);
          }
          tc::commit_pair_both(bar_empty + 8 * s, 3);
        }
        tc::commit_pair_both(bar_accf, 3);
      }
    }
  } else if (warp >= 6) {
    // --------------------------- scale warps (both CTAs) ---------------------------
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t sfr_leader = mapa(bar_sfr, 0);
    uint32_t it = 0;
    for (int t = pair; t < P.total_tiles; t += npairs) {
      const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
      const int nks = G.K / KSTEP;
      for (int ks = 0; ks < nks; ++ks, ++it) {
        const int s = it % C::STAGES;
        const uint32_t par = (it / C::STAGES) & 1;
        if (!mbar_wait(bar_sff + 8 * s, par, P.err, kDevErrTimeoutFull)) goto done;
        const uint8_t* st = smem_raw + s * C::STAGE_BYTES;
        const uint32_t sf = tmem + lane_base + C::SF_BASE + s * C::SF_STAGE_COLS;
#pragma unroll
        for (int kk = 0; kk < C::KPS; ++kk) {
          uint4 v = *reinterpret_cast<const uint4*>(st + C::OFF_SFA + kk * 512 + lane * 16);
          tc::st_32x32b_x4(sf + 4 * kk, v.x, v.y, v.z, v.w);
#pragma unroll
          for (int nb = 0; nb < C::NB; ++nb) {
            v = *reinterpret_cast<const uint4*>(st + C::OFF_SFB + nb * C::SFB_ROWTILE + kk * 512 + lane * 16);
            tc::st_32x32b_x4(sf + C::SFA_COLS + kk * C::SFBC + 4 * nb, v.x, v.y, v.z, v.w);
            if (C::DUAL) {
              v = *reinterpret_cast<const uint4*>(st + C::OFF_SFB2 + nb * C::SFB_ROWTILE + kk * 512 + lane * 16);
              tc::st_32x32b_x4(sf + C::SFA_COLS + C::KPS * C::SFBC + kk * C::SFBC + 4 * nb, v.x, v.y, v.z, v.w);
            }
          }
        }
        tc::wait_st();
        tc::fence_before_sync();
        asm volatile("bar.sync 3, 128;" ::: "memory");     // the 4 scale warps of this CTA
        // once this CTA's operands landed too, its whole stage is ready for the
        // pair MMA (an expired wait is recorded and the arrival skipped: the
        // leader's own bounded wait then ends the pipeline)
        if (threadIdx.x == 192 && mbar_wait(bar_full + 8 * s, par, P.err, kDevErrTimeoutFull))
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
      const int row = mt * C::TILE_M + (int)cta * BM + sub * 32 + lane;
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
        __half* crow = G.c + (int64_t)row * G.ldc + (int64_t)nt * C::BN;
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
}  // namespace nvfp4
