// Shared definitions of the tcgen05 GEMM kernels: per-group launch
// parameters, the single-CTA kernel's compile-time configuration, and small
// device helpers.  Included by gemm.cu only (one translation unit).
#pragma once

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

}  // namespace
}  // namespace nvfp4
