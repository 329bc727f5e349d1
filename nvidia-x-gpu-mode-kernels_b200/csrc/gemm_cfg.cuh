// Shared definitions of the tcgen05 GEMM kernel: per-group launch parameters,
// the kernel's compile-time configuration, and small device helpers.
// Included by gemm.cu only (one translation unit).
#pragma once

namespace nvfp4 {
namespace {

constexpr int BM = 128;          // rows per tile (one MMA of M=128)
constexpr int KSTEP = 256;       // K elements per K atom = 128 bytes per row
constexpr int KSTEP_BYTES = 128;

struct GemmGroup {
  CUtensorMap ta, tb, tb2;       // A [M, K/2], B [N, K/2] (B2 for the dual GEMM)
  CUtensorMap tsa, tsb, tsb2;    // blocked scales as [row tiles][K/64][128 x u32]
  __half* c;
  int64_t ldc;                   // elements
  int M, N, K;
  int tiles_m, tiles_n, tile_begin;
  int vec_ok;                    // c 16-byte aligned and ldc % 8 == 0: 16-byte stores
};

template <int MAXG>
struct GemmParams {
  GemmGroup g[MAXG];
  int ngroups;
  int total_tiles;
  uint32_t* err;
};

// BN: columns of a tile (rows of B per tile).  DUAL: two B operands sharing A,
// SiLU-gated epilogue.  STAGES: depth of the shared-memory ring.
// TRANS 1 (skinny GEMM): A holds weight rows, B the token rows, and the
// epilogue writes C^T, i.e. out[token][weight row]; one N tile only.
// KA: 128-byte K atoms (256 elements each) per stage: one TMA box per atom and
// operand, 4 * KA MMAs per B operand per stage, scale boxes of 4 * KA K-blocks.
template <int BN_, bool DUAL_, int STAGES_, int TRANS_ = 0, int KA_ = 1>
struct GemmCfg {
  static constexpr int TRANS = TRANS_;
  static constexpr int KA = KA_;
  static constexpr int KPS = 4 * KA_;    // 64-element K blocks (one MMA each) per stage
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
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int SMEM = OFF_BAR + (4 * STAGES + 4) * 8 + 16;   // base is 1024-aligned
  static constexpr uint32_t OP_BYTES = A_BYTES + B_BYTES * (DUAL ? 2 : 1);
  static constexpr uint32_t SF_BYTES = SFA_BYTES + SFB_BYTES * (DUAL ? 2 : 1);
  // tensor memory columns
  static constexpr int ACC_COLS = DUAL ? 2 * BN : BN;
  static constexpr int SF_BASE = ACC_COLS;
  static constexpr int SFB_COLS_PER_KB = NB * 4;
  static constexpr int SFA_COLS = 4 * KPS;
  static constexpr int SF_STAGE_COLS = SFA_COLS + KPS * SFB_COLS_PER_KB * (DUAL ? 2 : 1);
  static constexpr int TMEM_COLS = 512;
  static_assert(SF_BASE + STAGES * SF_STAGE_COLS <= TMEM_COLS, "tensor memory budget");
  static_assert(SMEM <= 232448, "shared memory budget");
  // shared-memory descriptors hold address >> 4 in 14 bits: stage offsets are
  // added to a base descriptor without carrying out of the field
  static_assert(SMEM < (1 << 18), "descriptor address field");
  // warp 0 producer, warp 1 MMA, warps 2-5 epilogue, warps 6-9 scale staging
  static constexpr int THREADS = 320;
  static constexpr uint32_t IDESC = tc::idesc_mxf4nvf4(BM, BN);
  static constexpr bool PAIR = false;
  static constexpr int TILE_M = BM;   // output rows per tile
  static constexpr int B_BOX = BN;    // B rows per TMA box
};

__device__ __forceinline__ int find_group(const GemmGroup* g, int ng, int t) {
  int i = 0;
  while (i + 1 < ng && g[i + 1].tile_begin <= t) ++i;
  return i;
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
