// The tcgen05 GEMM kernel (dual, grouped and skinny GEMMs; see gemm.cu for
// the design).  Included by gemm.cu only.
#pragma once

namespace nvfp4 {
namespace {

// Issues the MMAs of one stage.  `kb` K-blocks of 64 (KPS on full stages: a
// compile-time count, so the loop unrolls into straight-line MMA issues; a
// runtime-bounded loop measured ~25 % slower per stage).  Descriptors advance
// by whole atoms (A_ATOM / B_ATOM bytes, >> 4) and by 32 bytes (>> 4 = 2) per
// 64-element slice inside a 128-byte swizzled atom.
template <class C, int KB>
__device__ __forceinline__ void issue_stage_mmas(uint32_t tmem, uint64_t da, uint64_t db, uint64_t db2,
                                                 uint32_t sfa_t, uint32_t sfb_t, uint32_t sfb2_t,
                                                 uint32_t first_accum) {
#pragma unroll
  for (int kk = 0; kk < KB; ++kk) {
    const uint32_t accum = kk == 0 ? first_accum : 1u;
    const uint64_t off = (uint64_t)((kk >> 2) * (C::A_ATOM >> 4) + 2 * (kk & 3));
    const uint64_t offb = (uint64_t)((kk >> 2) * (C::B_ATOM >> 4) + 2 * (kk & 3));
    tc::mma_mxf4nvf4(tmem, da + off, db + offb, C::IDESC, sfa_t + 4 * kk, sfb_t + kk * C::SFB_COLS_PER_KB, accum);
    if (C::DUAL)
      tc::mma_mxf4nvf4(tmem + C::BN, da + off, db2 + offb, C::IDESC, sfa_t + 4 * kk,
                       sfb2_t + kk * C::SFB_COLS_PER_KB, accum);
  }
}

// Copies, for this warp's tensor-memory lane quarter, row `lane` of every
// 512-byte scale block of `kb` K-blocks into 4 consecutive columns each: the
// image a 32x128b.warpx4 copy would make, without occupying the tensor pipe.
template <class C, int KB>
__device__ __forceinline__ void stage_scales(const uint8_t* st, uint32_t sf, int lane) {
  const uint32_t sfa_t = sf, sfb_t = sf + C::SFA_COLS, sfb2_t = sf + C::SFA_COLS + C::KPS * C::SFB_COLS_PER_KB;
#pragma unroll
  for (int kk = 0; kk < KB; ++kk) {
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
  const uint32_t bar_full = sbase + C::OFF_BAR;             // operand boxes landed
  const uint32_t bar_empty = bar_full + 8 * C::STAGES;      // stage consumed by the MMAs
  const uint32_t bar_sfr = bar_empty + 8 * C::STAGES;       // scales staged in tensor memory
  const uint32_t bar_sff = bar_sfr + 8 * C::STAGES;         // scale boxes landed
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
          // Scales first, on their own barrier, so the scale warps stage them
          // while the operand bytes are still in flight.  Boxes always count in
          // full: blocks past the end of a matrix or of K read as zeros.
          const uint32_t sb = bar_sff + 8 * s;
          mbar_arrive_expect_tx(sb, C::SF_BYTES);
          tma_load_3d(st + C::OFF_SFA, &G.tsa, sb, 0, C::KPS * ks, mt, pol_a);
          tma_load_3d(st + C::OFF_SFB, &G.tsb, sb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
          if (C::DUAL) tma_load_3d(st + C::OFF_SFB2, &G.tsb2, sb, 0, C::KPS * ks, (nt * C::BN) / 128, pol_b);
          mbar_arrive_expect_tx(fb, C::OP_BYTES);
#pragma unroll
          for (int a = 0; a < C::KA; ++a) {   // atoms past K read as zeros (and count in full)
            const int x = (ks * C::KA + a) * KSTEP_BYTES;
            tma_load_2d(st + a * C::A_ATOM, &G.ta, fb, x, mt * BM, pol_a);
            tma_load_2d(st + C::OFF_B + a * C::B_ATOM, &G.tb, fb, x, nt * C::BN, pol_b);
            if (C::DUAL) tma_load_2d(st + C::OFF_B2 + a * C::B_ATOM, &G.tb2, fb, x, nt * C::BN, pol_b);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA -------------------------------
    if (lane == 0) {
      const uint64_t da0 = tc::desc_sw128(sbase);
      const uint64_t db0 = tc::desc_sw128(sbase + C::OFF_B);
      const uint64_t db20 = tc::desc_sw128(sbase + C::OFF_B2);
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
          const uint32_t par = (it / C::STAGES) & 1;
          if (!mbar_wait(bar_sfr + 8 * s, par, P.err, kDevErrTimeoutFull)) goto done;
          if (!mbar_wait(bar_full + 8 * s, par, P.err, kDevErrTimeoutFull)) goto done;
          tc::fence_after_sync();
          const uint64_t soff = (uint64_t)((s * C::STAGE_BYTES) >> 4);
          const uint32_t sf = tmem + C::SF_BASE + s * C::SF_STAGE_COLS;
          const uint32_t sfa_t = sf, sfb_t = sf + C::SFA_COLS + sfb_off;
          const uint32_t sfb2_t = sf + C::SFA_COLS + C::KPS * C::SFB_COLS_PER_KB + sfb_off;
          const uint32_t first = ks > 0 ? 1u : 0u;
          const int nch = min(C::KPS, nk64 - C::KPS * ks);
          if (nch == C::KPS) {
            issue_stage_mmas<C, C::KPS>(tmem, da0 + soff, db0 + soff, db20 + soff, sfa_t, sfb_t, sfb2_t, first);
          } else {
            // the last stage of a K that is not a multiple of the stage width
            for (int kk = 0; kk < nch; ++kk) {
              const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
              const uint64_t off = soff + (uint64_t)((kk >> 2) * (C::A_ATOM >> 4) + 2 * (kk & 3));
              const uint64_t offb = soff + (uint64_t)((kk >> 2) * (C::B_ATOM >> 4) + 2 * (kk & 3));
              tc::mma_mxf4nvf4(tmem, da0 + off, db0 + offb, C::IDESC, sfa_t + 4 * kk, sfb_t + kk * C::SFB_COLS_PER_KB,
                               accum);
              if (C::DUAL)
                tc::mma_mxf4nvf4(tmem + C::BN, da0 + off, db20 + offb, C::IDESC, sfa_t + 4 * kk,
                                 sfb2_t + kk * C::SFB_COLS_PER_KB, accum);
            }
          }
          tc::commit(bar_empty + 8 * s);
        }
        tc::commit(bar_accf);
      }
    }
  } else if (warp >= 6) {
    // --------------------------- scale warps ---------------------------
    // Each warp copies the stage's scale blocks into its tensor-memory lane
    // quarter (the MMA reads every quarter).  Issuing the same copies as
    // tcgen05.cp from the MMA thread serialises them with the MMAs on the
    // tensor pipe (~23 ns each, 12 per stage).
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t it = 0;
    bool dead = false;
    for (int t = blockIdx.x; t < P.total_tiles && !dead; t += gridDim.x) {
      const GemmGroup& G = P.g[find_group(P.g, P.ngroups, t)];
      const int nk64 = G.K / 64;
      const int nks = (nk64 + C::KPS - 1) / C::KPS;
      for (int ks = 0; ks < nks; ++ks, ++it) {
        const int s = it % C::STAGES;
        if (!mbar_wait(bar_sff + 8 * s, (it / C::STAGES) & 1, P.err, kDevErrTimeoutFull)) {
          dead = true;
          break;
        }
        const uint8_t* st = smem_raw + (sbase - raw) + s * C::STAGE_BYTES;
        const uint32_t sf = tmem + lane_base + C::SF_BASE + s * C::SF_STAGE_COLS;
        // on a last, partial stage the blocks past K arrived as zeros (the
        // box reads past the end as zeros) and no MMA reads them
        stage_scales<C, C::KPS>(st, sf, lane);
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_sfr + 8 * s);
      }
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
      } else if constexpr (!C::DUAL) {
        // Drain the whole accumulator row into registers (packed fp16) and
        // release it before storing anything, so the next tile's MMAs run while
        // this tile's global stores drain.  Storing chunk by chunk between the
        // tensor-memory loads held the accumulator ~3 us per tile (the 16-byte
        // row-strided stores are slow to issue).
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
      } else {
        // Dual GEMM: 32 columns of both accumulators at a time, SiLU gate,
        // stores interleaved with the loads.  With ~1.5 tiles per CTA the last
        // epilogue is on the critical path, where interleaving is shorter than
        // draining first (31.7 vs 33.4 us on the dual workload).
        __half* crow = G.c + (int64_t)row * G.ldc + (int64_t)nt * C::BN;
#pragma unroll 1
        for (int cb = 0; cb < C::BN / 32; ++cb) {
          uint32_t v[32], u[32], h[16];
          tc::ld_32x32b_x32(tmem + lane_base + cb * 32, v);
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
      }
    }
  }
done:
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace
}  // namespace nvfp4
