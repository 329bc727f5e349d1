// Batched NVFP4 block-scaled GEMV for sm_100a.
//
//   c[m, l] = sum_k e2m1(A[m,k,l]) e2m1(b[k,l]) e4m3(SFA[m,k/16,l]) e4m3(SFB[k/16,l])
//
// The reference (blackwell_nvfp4_gemv.cu:295-475) loads one tile per K step
// into a single shared buffer and computes with all threads, so loads and math
// alternate inside each CTA.  This kernel streams HBM instead:
//
//   * work unit = a tile of ROWS output rows of one batch l.  The tiles are
//     split into equal contiguous ranges, one per CTA of a persistent grid
//     (SM count x MINB CTAs), so every CTA streams the same number of bytes;
//   * one producer thread fills a STAGES-deep shared-memory ring: per stage one
//     tensor-map TMA box of A (ROWS rows x KTB bytes, read as u64 elements so a
//     row slice of up to 2 KB is one box row), one box of SFA (ROWS x KTB/8),
//     and the matching slices of b and SFB.  Whole-tile boxes keep the TMA
//     issue count at four per stage (per-row 1-D bulk copies measured at under
//     5 TB/s even with the math switched off).  Rows past M and K past the end
//     read as zeros (TMA out-of-bounds fill) and contribute nothing;
//   * CW consumer warps split a stage by K: warp w takes 512-byte column chunk
//     w % NCH of every row in its row group w / NCH, so it decodes its slice of
//     b once per stage (to f16x2 registers) and reuses it for RPW rows;
//   * per lane, 16 bytes = 32 e2m1 codes = two scale blocks.  Codes go to f16x2
//     with cvt.rn.f16x2.e2m1x2 and multiply-add into f16x2 accumulators inside
//     a 16-element block.  A half-lane sums at most 8 products, each a multiple
//     of 1/4 below 36 in magnitude, so every partial sum is a multiple of 1/4
//     below 512 and f16 represents it exactly.  The block sum is widened to f32
//     and scaled by sfa*sfb in f32 (exact: 4 x 4 significant bits), then
//     accumulated in f32.  The reference instead scales and sums in f16
//     (:126-131), which rounds, and overflows once sfa*sfb exceeds 65504;
//   * at the end of a tile each warp reduces its per-row partials across lanes
//     (xor shuffles), the NCH column chunks of a row meet in shared memory, and
//     one thread per row stores the fp16 result.
//
// Every wait is bounded (2 s) and reports into the device error word.
#include <cuda_fp16.h>
#include <cstring>
#include <atomic>
#include <mutex>
#include "ptx.cuh"
#include "common.h"
#include "tmap.h"

namespace nvfp4 {
namespace {

constexpr int kMaxRanks = 8;
// Staging buffer of the fused all-gather (32-bit words): control words first,
// then 64-bit lines from word kLineWord on: (epoch << 32) | two fp16 values
// (elements 2i, 2i+1 in line i) when M_total is even, (epoch << 32) | one
// fp16 value (element i in line i) when it is odd.
constexpr int kCtaCounter = 16;   // counts this rank's finished CTAs (reset per call)
constexpr int kEpochWord = 20;    // the last epoch (device-epoch mode)
constexpr int kStampWord = 32;    // words 32-37: %globaltimer at start / rows sent / all rows present
constexpr int kLineWord = 64;     // first line: 64-bit index kLineWord / 2


struct GemvArgs {
  const uint8_t* a;
  const uint8_t* b;
  const uint8_t* sfa;
  const uint8_t* sfb;
  __half* c;
  int64_t M, K, L;
  int64_t a_sm, a_sl, b_sl, sfa_sm, sfa_sl, sfb_sl, c_sm, c_sl;
  uint32_t* err;
  // Fused all-gather (world > 0): every result also goes, as one 64-bit line
  // (epoch << 32 | fp16 bits), to element index l * M_total + m_off + row of
  // every rank's staging buffer; then each CTA unpacks its slice of the full
  // output from this rank's staging buffer into c, once the slice's lines
  // carry this call's epoch.
  uint64_t* peer_stage[kMaxRanks];
  int world;
  int rank;
  int64_t m_off;
  int64_t M_total;
  int per_line;      // output elements per 64-bit line: 2 (M_total even) or 1
  uint32_t epoch;    // 1-based call count of this gather (same on every rank); 0 = device epoch
  uint64_t peer_wait_ns;   // budget of the wait for the other ranks' rows
};

struct GemvMaps {
  CUtensorMap a, sfa, b, sfb;
};

// ROWS rows x KTB A-bytes per stage; CW consumer warps; MINB CTAs per SM.
template <int ROWS_, int KTB_, int STAGES_, int CW_, int MINB_ = 1>
struct GemvCfg {
  static constexpr int ROWS = ROWS_;
  static constexpr int KTB = KTB_;
  static constexpr int STAGES = STAGES_;
  static constexpr int CW = CW_;
  static constexpr int MINB = MINB_;
  static constexpr int THREADS = (CW + 1) * 32;
  static constexpr int NCH = KTB / 512;          // 512-byte column chunks per row
  static constexpr int GROUPS = CW / NCH;        // row groups
  static constexpr int RPW = ROWS / GROUPS;      // rows per consumer warp
  static constexpr int SFK = KTB / 8;            // scale bytes per row per stage
  static constexpr int OFF_SFA = ROWS * KTB;
  static constexpr int OFF_B = ((OFF_SFA + ROWS * SFK) + 127) / 128 * 128;
  static constexpr int OFF_SFB = OFF_B + KTB;
  static constexpr int STAGE_BYTES = ((OFF_SFB + SFK) + 127) / 128 * 128;
  static constexpr uint32_t TX = ROWS * KTB + ROWS * SFK + KTB + SFK;
  static constexpr int OFF_RED = STAGES * STAGE_BYTES;                  // float [2][ROWS][NCH]
  static constexpr int OFF_BAR = (OFF_RED + 2 * ROWS * NCH * 4 + 15) / 16 * 16;
  static constexpr int SMEM = OFF_BAR + 2 * STAGES * 8 + 128;           // + alignment slack
  static_assert(KTB % 512 == 0 && KTB <= 2048, "KTB: 512-byte chunks, box row <= 256 u64");
  static_assert(CW % NCH == 0 && ROWS % GROUPS == 0, "warps must tile (rows x chunks)");
  static_assert(ROWS <= 256, "TMA box height");
};

}  // namespace

namespace {

// One 16-byte chunk (two 16-element scale blocks) of a row against the
// decoded b chunk: returns the f32 contribution sum_blk blocksum * sfa * sfb.
__device__ __forceinline__ float chunk_dot(const uint4 av, uint32_t sfa2, const uint32_t (&bh)[16],
                                           float sb0, float sb1) {
  uint32_t h[4], p0, p1, q0, q1;
  cvt_e2m1x8(av.x, h);
  p0 = hfma2(h[0], bh[0], 0u);
  p1 = hfma2(h[1], bh[1], 0u);
  p0 = hfma2(h[2], bh[2], p0);
  p1 = hfma2(h[3], bh[3], p1);
  cvt_e2m1x8(av.y, h);
  p0 = hfma2(h[0], bh[4], p0);
  p1 = hfma2(h[1], bh[5], p1);
  p0 = hfma2(h[2], bh[6], p0);
  p1 = hfma2(h[3], bh[7], p1);
  cvt_e2m1x8(av.z, h);
  q0 = hfma2(h[0], bh[8], 0u);
  q1 = hfma2(h[1], bh[9], 0u);
  q0 = hfma2(h[2], bh[10], q0);
  q1 = hfma2(h[3], bh[11], q1);
  cvt_e2m1x8(av.w, h);
  q0 = hfma2(h[0], bh[12], q0);
  q1 = hfma2(h[1], bh[13], q1);
  q0 = hfma2(h[2], bh[14], q0);
  q1 = hfma2(h[3], bh[15], q1);
  // each half-lane of p0+p1 sums 8 products: exact in f16 (see file comment)
  const uint32_t p = hadd2(p0, p1), q = hadd2(q0, q1);
  float sa0, sa1, x0, y0, x1, y1;
  h2_to_f2(cvt_e4m3x2(sfa2), sa0, sa1);
  h2_to_f2(p, x0, y0);
  h2_to_f2(q, x1, y1);
  return fmaf(x0 + y0, sa0 * sb0, (x1 + y1) * (sa1 * sb1));
}

template <class C>
__global__ void __launch_bounds__(C::THREADS, C::MINB)
gemv_tma_kernel(const __grid_constant__ GemvMaps maps, const __grid_constant__ GemvArgs p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 127u) & ~127u;
  uint8_t* smem = smem_raw + (sbase - raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t bar_full = sbase + C::OFF_BAR;
  const uint32_t bar_empty = bar_full + 8 * C::STAGES;
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, C::CW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Launched with programmatic dependent launch: everything above overlapped
  // the previous kernel on the stream; wait for it before touching global
  // memory (a no-op when launched without the attribute).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // fused all-gather: this launch's epoch, for every thread.  Device-epoch
  // mode (p.epoch == 0) numbers the launch (stored + 1); every CTA reads the
  // word before the last CTA (which counts in after all others have started)
  // stores the new value.
  __shared__ uint32_t s_epoch;
  uint32_t* const ctl = p.world > 0 ? reinterpret_cast<uint32_t*>(p.peer_stage[p.rank]) : nullptr;
  if (p.world > 0 && threadIdx.x == 0) {
    s_epoch = p.epoch ? p.epoch : *reinterpret_cast<volatile uint32_t*>(ctl + kEpochWord) + 1u;
    if (blockIdx.x == 0) {
      const uint64_t t = globaltimer();
      ctl[kStampWord] = (uint32_t)t;
      ctl[kStampWord + 1] = (uint32_t)(t >> 32);
    }
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int64_t M = p.M;
  const int nk = (int)((p.K / 2 + C::KTB - 1) / C::KTB);
  const int64_t tpl = (M + C::ROWS - 1) / C::ROWS;  // tiles per batch
  const int64_t ntiles = tpl * p.L;
  const int64_t t0 = ntiles * blockIdx.x / gridDim.x, t1 = ntiles * (blockIdx.x + 1) / gridDim.x;

  if (warp == C::CW) {
    // ---------------- producer: one elected thread ----------------
    if (lane == 0) {
      prefetch_tmap(&maps.a);
      prefetch_tmap(&maps.sfa);
      prefetch_tmap(&maps.b);
      prefetch_tmap(&maps.sfb);
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      uint32_t it = 0;
      for (int64_t t = t0; t < t1; ++t) {
        const int l = (int)(t / tpl);
        const int m0 = (int)((t % tpl) * C::ROWS);
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait(bar_empty + 8 * s, ((it / C::STAGES) & 1) ^ 1, p.err, kDevErrTimeoutEmpty)) return;
          const uint32_t st = sbase + s * C::STAGE_BYTES;
          const uint32_t fb = bar_full + 8 * s;
          const int x = kt * (C::KTB / 8);  // u64 units of A == bytes of SFA
          mbar_arrive_expect_tx(fb, C::TX);
          tma_load_3d(st, &maps.a, fb, x, m0, l, pol_stream);
          tma_load_3d(st + C::OFF_SFA, &maps.sfa, fb, x, m0, l, pol_stream);
          tma_load_2d(st + C::OFF_B, &maps.b, fb, x, l, pol_keep);
          tma_load_2d(st + C::OFF_SFB, &maps.sfb, fb, x, l, pol_keep);
        }
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int chunk = warp % C::NCH;
  const int group = warp / C::NCH;
  const int off = 512 * chunk + 16 * lane;   // this lane's byte offset inside a stage row
  uint32_t it = 0;
  int parity = 0;
  bool dead = false;  // a wait expired: stop waiting, keep joining the named barrier
  for (int64_t t = t0; t < t1; ++t, parity ^= 1) {
    const int64_t l = t / tpl;
    const int64_t m0 = (t % tpl) * C::ROWS;
    float acc[C::RPW];
#pragma unroll
    for (int j = 0; j < C::RPW; ++j) acc[j] = 0.f;

    for (int kt = 0; kt < nk; ++kt, ++it) {
      const int s = it % C::STAGES;
      if (!dead && !mbar_wait(bar_full + 8 * s, (it / C::STAGES) & 1, p.err, kDevErrTimeoutFull)) dead = true;
      const uint8_t* st = smem + s * C::STAGE_BYTES;
      {
        uint32_t bh[16];
        float sb0, sb1;
        {
          const uint4 bv = *reinterpret_cast<const uint4*>(st + C::OFF_B + off);
          cvt_e2m1x8(bv.x, *reinterpret_cast<uint32_t(*)[4]>(&bh[0]));
          cvt_e2m1x8(bv.y, *reinterpret_cast<uint32_t(*)[4]>(&bh[4]));
          cvt_e2m1x8(bv.z, *reinterpret_cast<uint32_t(*)[4]>(&bh[8]));
          cvt_e2m1x8(bv.w, *reinterpret_cast<uint32_t(*)[4]>(&bh[12]));
          const uint32_t s2 = *reinterpret_cast<const uint16_t*>(st + C::OFF_SFB + off / 8);
          h2_to_f2(cvt_e4m3x2(s2), sb0, sb1);
        }
#pragma unroll
        for (int j = 0; j < C::RPW; ++j) {
          const int row = group * C::RPW + j;
          const uint4 av = *reinterpret_cast<const uint4*>(st + row * C::KTB + off);
          const uint32_t s2 = *reinterpret_cast<const uint16_t*>(st + C::OFF_SFA + row * C::SFK + off / 8);
          acc[j] += chunk_dot(av, s2, bh, sb0, sb1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);
    }

    // lanes -> per-row partial of this chunk -> shared memory
    float* rb = red + parity * C::ROWS * C::NCH;
#pragma unroll
    for (int j = 0; j < C::RPW; ++j) {
      float v = acc[j];
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
      if (lane == 0) rb[(group * C::RPW + j) * C::NCH + chunk] = v;
    }
    asm volatile("bar.sync 1, %0;" :: "r"(C::CW * 32) : "memory");
    if (p.world == 0) {
      for (int row = threadIdx.x; row < C::ROWS; row += C::CW * 32) {
        float v = 0.f;
#pragma unroll
        for (int c = 0; c < C::NCH; ++c) v += rb[row * C::NCH + c];
        if (m0 + row < M) p.c[l * p.c_sl + (m0 + row) * p.c_sm] = __float2half_rn(v);
      }
    } else {
      // one 64-bit line per (row group, rank), a row group being per_line
      // consecutive rows (rows are split at even boundaries when per_line is
      // 2, so a pair never straddles two ranks): thread t sends group t % G to
      // rank t / G.  A naturally aligned 64-bit store is single-copy atomic, so
      // a line that carries this call's epoch carries this call's values: no
      // fence or count is needed before the receiver may use it.  Two values
      // per line halve the small NVLink stores, whose rate limits the gather.
      const int pl = p.per_line, G = C::ROWS / pl;
      for (int t = threadIdx.x; t < G * p.world; t += C::CW * 32) {
        const int row = (t % G) * pl, r = t / G;
        if (m0 + row >= M) continue;
        uint64_t line = (uint64_t)epoch << 32;
        for (int j = 0; j < pl; ++j) {
          float v = 0.f;
#pragma unroll
          for (int c = 0; c < C::NCH; ++c) v += rb[(row + j) * C::NCH + c];
          line |= (uint64_t)__half_as_ushort(__float2half_rn(v)) << (16 * j);
        }
        uint64_t* dst = p.peer_stage[r] + kLineWord / 2 + (l * p.M_total + p.m_off + m0 + row) / pl;
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(dst), "l"(line) : "memory");   // NVLink peer store
      }
    }
  }
  if (p.world > 0) {
    // Completion: CTA b unpacks slice b of the full output (all ranks' rows)
    // from this rank's staging buffer, waiting (bounded) for each line to carry
    // this call's epoch; the launch ends when every slice is in c.  Thread 0 of
    // the CTA that finishes last resets the CTA count, stamps the time and, in
    // device-epoch mode, stores the epoch for the next launch.
    asm volatile("bar.sync 1, %0;" :: "r"(C::CW * 32) : "memory");
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      const uint64_t ts = globaltimer();
      ctl[kStampWord + 2] = (uint32_t)ts;
      ctl[kStampWord + 3] = (uint32_t)(ts >> 32);
    }
    const int64_t total = p.M_total * p.L / p.per_line;   // lines
    const int64_t e0 = total * blockIdx.x / gridDim.x, e1 = total * (blockIdx.x + 1) / gridDim.x;
    const uint64_t* lines = p.peer_stage[p.rank] + kLineWord / 2;
    bool late = false;
    for (int64_t e = e0 + threadIdx.x; e < e1; e += C::CW * 32) {
      uint64_t v = 0;
      uint64_t t0 = 0;
      for (uint32_t it = 0;; ++it) {
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(lines + e) : "memory");
        if ((uint32_t)(v >> 32) == epoch) break;
        if (late) break;   // this thread already gave up once: do not wait again
        if ((it & 63u) == 0) {
          const uint64_t t = globaltimer();
          if (it == 0) t0 = t;
          else if (t - t0 > p.peer_wait_ns) {
            atomicOr(p.err, kDevErrTimeoutPeer);
            late = true;
            break;
          }
        }
      }
      if ((uint32_t)(v >> 32) == epoch) {
        for (int j = 0; j < p.per_line; ++j) {
          const int64_t x = e * p.per_line + j, l = x / p.M_total, m = x % p.M_total;
          p.c[l * p.c_sl + m * p.c_sm] = __ushort_as_half((unsigned short)((v >> (16 * j)) & 0xFFFFu));
        }
      }
    }
    asm volatile("bar.sync 1, %0;" :: "r"(C::CW * 32) : "memory");
    if (threadIdx.x == 0) {
      const uint32_t done = atomicAdd(ctl + kCtaCounter, 1u) + 1u;
      if (done == gridDim.x) {
        ctl[kCtaCounter] = 0u;
        const uint64_t te = globaltimer();
        ctl[kStampWord + 4] = (uint32_t)te;
        ctl[kStampWord + 5] = (uint32_t)(te >> 32);
        if (p.epoch == 0) ctl[kEpochWord] = epoch;
      }
    }
  }
}

// Plain-load kernel for inputs the TMA path cannot take (a pointer or byte
// stride that is not a multiple of 16).  One warp per output row; lane t
// handles 16-element blocks t, t+32, ...; the same exact per-block arithmetic.
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
      for (int j = 0; j < 8; ++j) c = hfma2(cvt_e2m1x2(arow[blk * 8 + j]), cvt_e2m1x2(bl[blk * 8 + j]), c);
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

}  // namespace

// Stride along L for a tensor map when L == 1 (any 16-byte multiple is valid).
static inline uint64_t l_stride(int64_t L, int64_t given, int64_t fallback) {
  if (L > 1) return (uint64_t)given;
  return (uint64_t)((fallback + 15) / 16 * 16);
}

// Tensor maps depend only on the pointers, shape, strides and tile config, so
// they are cached by value (a small LRU per process): repeated calls on the
// same buffers skip the four driver encodes.
struct MapKey {
  const void* a;
  const void* b;
  const void* sfa;
  const void* sfb;
  int64_t M, K, L, a_sm, a_sl, b_sl, sfa_sm, sfa_sl, sfb_sl;
  int cfg;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};

struct MapCache {
  static constexpr int N = 16;
  MapKey key[N];
  GemvMaps maps[N];
  uint64_t stamp[N] = {};
  uint64_t clock = 0;
  std::mutex mu;
};
MapCache g_map_cache;

template <class C>
int build_maps(const GemvArgs& p, GemvMaps& maps) {
  const uint64_t kq = (uint64_t)(p.K / 16);  // A/b row length in u64 units == scale bytes per row
  {
    const uint64_t dims[3] = {kq, (uint64_t)p.M, (uint64_t)p.L};
    const uint64_t str[2] = {(uint64_t)p.a_sm, l_stride(p.L, p.a_sl, p.a_sm * p.M)};
    const uint32_t box[3] = {C::KTB / 8, C::ROWS, 1};
    int rc = encode_tmap(&maps.a, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, p.a, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {kq, (uint64_t)p.M, (uint64_t)p.L};
    const uint64_t str[2] = {(uint64_t)p.sfa_sm, l_stride(p.L, p.sfa_sl, p.sfa_sm * p.M)};
    const uint32_t box[3] = {C::KTB / 8, C::ROWS, 1};
    int rc = encode_tmap(&maps.sfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, p.sfa, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {kq, (uint64_t)p.L};
    const uint64_t str[1] = {l_stride(p.L, p.b_sl, p.K / 2)};
    const uint32_t box[2] = {C::KTB / 8, 1};
    int rc = encode_tmap(&maps.b, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, p.b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {kq, (uint64_t)p.L};
    const uint64_t str[1] = {l_stride(p.L, p.sfb_sl, p.K / 16)};
    const uint32_t box[2] = {C::KTB / 8, 1};
    return encode_tmap(&maps.sfb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, p.sfb, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
}

template <class C>
int cached_maps(const GemvArgs& p, GemvMaps& out) {
  MapKey k;
  std::memset(&k, 0, sizeof(k));
  k.a = p.a; k.b = p.b; k.sfa = p.sfa; k.sfb = p.sfb;
  k.M = p.M; k.K = p.K; k.L = p.L;
  k.a_sm = p.a_sm; k.a_sl = p.L > 1 ? p.a_sl : 0; k.b_sl = p.L > 1 ? p.b_sl : 0;
  k.sfa_sm = p.sfa_sm; k.sfa_sl = p.L > 1 ? p.sfa_sl : 0; k.sfb_sl = p.L > 1 ? p.sfb_sl : 0;
  k.cfg = C::ROWS * 1000000 + C::KTB;
  MapCache& c = g_map_cache;
  {
    std::lock_guard<std::mutex> lk(c.mu);
    for (int i = 0; i < MapCache::N; ++i)
      if (c.stamp[i] && c.key[i] == k) {
        c.stamp[i] = ++c.clock;
        out = c.maps[i];
        return NVFP4_OK;
      }
  }
  int rc = build_maps<C>(p, out);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(c.mu);
  int victim = 0;
  for (int i = 1; i < MapCache::N; ++i)
    if (c.stamp[i] < c.stamp[victim]) victim = i;
  c.key[victim] = k;
  c.maps[victim] = out;
  c.stamp[victim] = ++c.clock;
  return NVFP4_OK;
}

template <class C>
int64_t grid_of(const GemvArgs& p) {
  const int64_t ntiles = (p.M + C::ROWS - 1) / C::ROWS * p.L;
  int64_t grid = (int64_t)sm_count() * C::MINB;
  return ntiles < grid ? ntiles : grid;
}

template <class C>
int launch_tma(const GemvArgs& p, cudaStream_t stream, int64_t* grid_out) {
  if (grid_out) {
    *grid_out = grid_of<C>(p);
    return NVFP4_OK;
  }
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_tma_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemv)");
    attr_set[dev] = true;
  }
  GemvMaps maps;
  int rc = cached_maps<C>(p, maps);
  if (rc) return rc;
  const int64_t grid = grid_of<C>(p);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_tma_kernel<C>, maps, p);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemv)");
  return check_launch("gemv_tma_kernel");
}

int launch_generic(const GemvArgs& p, cudaStream_t stream) {
  const int64_t rows = p.M * p.L;
  int64_t grid = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (grid > cap) grid = cap;
  gemv_generic_kernel<<<(unsigned)grid, 256, 0, stream>>>(p);
  return check_launch("gemv_generic_kernel");
}

// Configuration by shape.  The stage width KTB (bytes of a row per stage) is
// chosen from K alone: a row's f32 summation order, and so every bit of its
// result, depends on KTB and on nothing else (not on the row tile, the warp
// count, the grid, M, L or the rank's share), so a row-sharded GEMV returns
// exactly the single-GPU bits.  Small problems then use short tiles and more
// CTAs per SM so that every SM gets work.
// With grid_out set, only reports the grid the launch would use.
int gemv_dispatch(const GemvArgs& p, cudaStream_t st, int64_t* grid_out = nullptr) {
  const int64_t kb = p.K / 2;
  const int64_t rows = p.M * p.L;
  const int64_t sms = sm_count();
  // widest row slice whose last stage is not mostly padding: K/2 = 7168
  // bytes is 3.5 slices of 2 KB (a half-empty last stage per tile, 52.3 us on
  // config 2) but exactly 7 slices of 1 KB (48.6 us)
  auto pad = [kb](int64_t w) { return ((kb + w - 1) / w) * w - kb; };
  const int ktb = (kb >= 2048 && pad(2048) <= pad(1024)) ? 2048 : (kb >= 1024 ? 1024 : 512);
  if (ktb == 2048) {
    // fewer than 16 rows per SM (the 8-rank share of config 1): 4-row tiles,
    // four CTAs per SM (M=2048, K=16384: 11.5 vs 12.0 us with 1 KB stages)
    if (rows < sms * 16) return launch_tma<GemvCfg<4, 2048, 4, 4, 4>>(p, st, grid_out);
    // fewer than two 16-row tiles per SM (the 4-rank share): 8-row tiles,
    // two CTAs per SM
    if (rows < sms * 32) return launch_tma<GemvCfg<8, 2048, 4, 4, 2>>(p, st, grid_out);
    return launch_tma<GemvCfg<16, 2048, 4, 8, 1>>(p, st, grid_out);
  }
  if (ktb == 1024) {
    if (rows < sms * 16) return launch_tma<GemvCfg<4, 1024, 3, 4, 4>>(p, st, grid_out);
    return launch_tma<GemvCfg<16, 1024, 4, 8, 2>>(p, st, grid_out);
  }
  if (rows < sms * 16) return launch_tma<GemvCfg<2, 512, 2, 2, 8>>(p, st, grid_out);
  return launch_tma<GemvCfg<16, 512, 4, 8, 2>>(p, st, grid_out);
}

}  // namespace nvfp4

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
  GemvArgs args{};
  args.a = static_cast<const uint8_t*>(a);
  args.b = static_cast<const uint8_t*>(b);
  args.sfa = static_cast<const uint8_t*>(sfa);
  args.sfb = static_cast<const uint8_t*>(sfb);
  args.c = static_cast<__half*>(c);
  args.M = M; args.K = K; args.L = L;
  args.a_sm = a_sm; args.a_sl = a_sl; args.b_sl = b_sl;
  args.sfa_sm = sfa_sm; args.sfa_sl = sfa_sl; args.sfb_sl = sfb_sl;
  args.c_sm = c_sm; args.c_sl = c_sl;
  args.err = device_error_word();
  if (!args.err) return fail(NVFP4_ERR_CUDA, "nvfp4_gemv: cannot resolve the device error word");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool tma_ok = aligned16(a) && aligned16(b) && aligned16(sfa) && aligned16(sfb) && a_sm % 16 == 0 &&
                      sfa_sm % 16 == 0 &&
                      (L == 1 || (a_sl % 16 == 0 && b_sl % 16 == 0 && sfa_sl % 16 == 0 && sfb_sl % 16 == 0));
  if (!tma_ok) return launch_generic(args, st);
  return gemv_dispatch(args, st);
}

extern "C" int nvfp4_gemv_grid(int64_t M, int64_t K, int64_t L, int64_t* grid) {
  using namespace nvfp4;
  if (!grid || M < 1 || L < 1 || K < 16 || K % 16) return fail(NVFP4_ERR_INVALID, "nvfp4_gemv_grid: bad shape");
  GemvArgs args{};
  args.M = M; args.K = K; args.L = L;
  return gemv_dispatch(args, nullptr, grid);
}

namespace nvfp4 {
namespace {
std::atomic<uint64_t> g_peer_wait_ns{kWaitBudgetNs};
}
}  // namespace nvfp4

extern "C" int nvfp4_set_peer_wait_ns(uint64_t ns) {
  using namespace nvfp4;
  if (ns == 0) ns = kWaitBudgetNs;
  if (ns < 1000ull || ns > kWaitBudgetNs)
    return fail(NVFP4_ERR_INVALID, "nvfp4_set_peer_wait_ns: budget must be 0 (default) or 1e3..2e9 ns, got %llu",
                (unsigned long long)ns);
  g_peer_wait_ns.store(ns, std::memory_order_relaxed);
  return NVFP4_OK;
}

extern "C" int nvfp4_gemv_allgather(const void* a, const void* b, const void* sfa, const void* sfb,
                                    int64_t M_local, int64_t K, int64_t L, int64_t a_sm, int64_t a_sl,
                                    int64_t b_sl, int64_t sfa_sm, int64_t sfa_sl, int64_t sfb_sl,
                                    void* out, int64_t c_sm, int64_t c_sl, int64_t m_off, int64_t M_total,
                                    void* const* peer_stage, int world, int rank, uint32_t epoch, void* stream) {
  using namespace nvfp4;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || !peer_stage || !out)
    return fail(NVFP4_ERR_INVALID, "nvfp4_gemv_allgather: need 1 <= world <= %d, 0 <= rank < world and an output",
                kMaxRanks);
  for (int r = 0; r < world; ++r) {
    if (!peer_stage[r]) return fail(NVFP4_ERR_INVALID, "nvfp4_gemv_allgather: null staging buffer");
    if (reinterpret_cast<uintptr_t>(peer_stage[r]) & 7u)
      return fail(NVFP4_ERR_ALIGNMENT, "nvfp4_gemv_allgather: staging buffers must be 8-byte aligned");
  }
  if (!a || !b || !sfa || !sfb) return fail(NVFP4_ERR_INVALID, "nvfp4_gemv_allgather: null input");
  if (M_local < 1 || L < 1 || K < 16 || K % 16 || m_off < 0 || M_total < m_off + M_local || c_sm == 0 ||
      (L > 1 && c_sl == 0))
    return fail(NVFP4_ERR_INVALID, "nvfp4_gemv_allgather: bad shape or strides");
  const bool tma_ok = aligned16(a) && aligned16(b) && aligned16(sfa) && aligned16(sfb) && a_sm % 16 == 0 &&
                      sfa_sm % 16 == 0 &&
                      (L == 1 || (a_sl % 16 == 0 && b_sl % 16 == 0 && sfa_sl % 16 == 0 && sfb_sl % 16 == 0));
  if (!tma_ok) return fail(NVFP4_ERR_ALIGNMENT, "nvfp4_gemv_allgather: needs 16-byte aligned pointers and strides");
  if (M_total % 2 == 0 && (m_off % 2 || M_local % 2))
    return fail(NVFP4_ERR_INVALID,
                "nvfp4_gemv_allgather: with an even M_total, every rank's m_off and M_local must be even "
                "(two results travel per line)");
  GemvArgs args{};
  args.a = static_cast<const uint8_t*>(a);
  args.b = static_cast<const uint8_t*>(b);
  args.sfa = static_cast<const uint8_t*>(sfa);
  args.sfb = static_cast<const uint8_t*>(sfb);
  args.c = static_cast<__half*>(out);
  args.M = M_local; args.K = K; args.L = L;
  args.a_sm = a_sm; args.a_sl = a_sl; args.b_sl = b_sl;
  args.sfa_sm = sfa_sm; args.sfa_sl = sfa_sl; args.sfb_sl = sfb_sl;
  args.c_sm = c_sm; args.c_sl = c_sl;
  args.err = device_error_word();
  if (!args.err) return fail(NVFP4_ERR_CUDA, "nvfp4_gemv_allgather: cannot resolve the device error word");
  for (int r = 0; r < world; ++r) args.peer_stage[r] = static_cast<uint64_t*>(peer_stage[r]);
  args.world = world;
  args.rank = rank;
  args.m_off = m_off;
  args.M_total = M_total;
  args.per_line = M_total % 2 == 0 ? 2 : 1;
  args.epoch = epoch;
  args.peer_wait_ns = g_peer_wait_ns.load(std::memory_order_relaxed);
  return gemv_dispatch(args, static_cast<cudaStream_t>(stream));
}
