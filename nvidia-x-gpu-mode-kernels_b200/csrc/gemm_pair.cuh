// The CTA-pair (cta_group::2) variant of the GEMM kernel: exact, measured
// no faster than the single-CTA kernel, not instantiated by the library's
// entry points.  Included by gemm.cu only.
#pragma once

namespace nvfp4 {
namespace {

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
}  // namespace nvfp4
