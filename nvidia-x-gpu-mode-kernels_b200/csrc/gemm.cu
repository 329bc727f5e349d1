// NVFP4 block-scaled GEMMs on the tcgen05 tensor cores (sm_100a):
//
//   grouped:  C_g[M_g, N_g] = A_g[M_g, K_g] . B_g[N_g, K_g]^T          (fp16 out)
//   dual:     C[M, N] = silu(A . B1^T) * (A . B2^T)                    (fp16 out)
//   skinny:   out[T, N] = X[T, K] . W[N, K]^T, T <= 64 (weights as the MMA's
//             128-row operand, the epilogue writes C^T)
//
// Operands are e2m1 codes packed two per byte, K-major (rows of K/2 bytes),
// with one e4m3 scale per 16 K-elements stored in the 128x4 blocked layout
// (128-row x 4-scale tiles of 512 bytes, row-tile major; inside a tile the
// scale (r, c) sits at byte (r%32)*16 + (r/32)*4 + c).  That layout is the
// image a 32x128b.warpx4 copy turns into the tensor-memory arrangement the
// block-scaled MMA reads.  The MMA reads scales as unsigned e4m3 (sign bit 0).
//
// gemm_kernel (gemm_kernel.cuh): one persistent CTA per SM walks output tiles
// of 128 x BN (tile t, t+grid, ...); tiles of a group are ordered M-tile
// fastest, so CTAs running at the same time share B tiles through L2.  A stage
// holds KA 128-byte K atoms (256 elements each).  Warp roles:
//   warp 0     TMA producer: per stage, tensor-map boxes of the stage's scale
//              blocks (on their own barrier, issued first) and one 128-byte
//              swizzled box per K atom of A and of B (and B2);
//   warp 1     allocates tensor memory; one thread issues 4*KA MMAs of K=64
//              (kind::mxf4nvf4, scale_vec::4X) per B operand, commits the
//              stage back to the producer and, after the last K step, the
//              accumulator to the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of the fp32 accumulator (one row per
//              thread), SiLU gate or plain conversion to fp16, 16-byte stores;
//              the grouped GEMM drains the whole row to registers and releases
//              the accumulator before storing;
//   warps 6-9  scale warps: copy each stage's scale blocks from shared memory
//              into tensor memory with tcgen05.st, each its lane quarter.
// Every mbarrier wait is bounded (2 s) and reports into the device error word.
#include <cuda_fp16.h>
#include <cstring>
#include <mutex>
#include "ptx.cuh"
#include "tcgen05.cuh"
#include "common.h"
#include "tmap.h"

#include "gemm_cfg.cuh"
#include "gemm_kernel.cuh"
#include "gemm_pair.cuh"

namespace nvfp4 {

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
int launch_pair(const GemmParams<MAXG>& P, cudaStream_t stream) {
  static bool attr_set[64] = {};
  static int max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(NVFP4_ERR_UNSUPPORTED, "device index out of range");
  auto kern = pair_kernel<C, MAXG>;
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
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair gemm)");
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
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(pair gemm)");
  return check_launch("pair_kernel");
}

template <class C, int MAXG>
int launch_any(const GemmParams<MAXG>& P, cudaStream_t stream) {
  if constexpr (C::PAIR) return launch_pair<C, MAXG>(P, stream);
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
  G.c = static_cast<__half*>(c);
  G.ldc = ldc;
  G.vec_ok = vec_ok(c, ldc);
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
  // CTA pairs (256 x 128 tiles per B operand, 5 stages of 38 KB) when K is a
  // multiple of the 256-element stage: 16.x vs 30.6 us on the dual workload.
  // Otherwise the single-CTA kernel with two 512-element K stages of 108 KB.
  if (K % 256 == 0)
    return dual_run<PairCfg<128, 5, true>>(a, b1, b2, sfa, sfb1, sfb2, c, M, N, K, lda, ldb, ldc, stream);
  return dual_run<GemmCfg<128, true, 2, 0, 2>>(a, b1, b2, sfa, sfb1, sfb2, c, M, N, K, lda, ldb, ldc, stream);
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
  return launch_gemm<C, 1>(P, static_cast<cudaStream_t>(stream));
}

template <class C, int MAXG>
int grouped_launches(const nvfp4_group* groups, int num_groups, void* stream) {
  uint32_t* err = device_error_word();
  if (!err) return fail(NVFP4_ERR_CUDA, "nvfp4_grouped_gemm: cannot resolve the device error word");
  static GemmParams<MAXG> P;          // large; built under a lock, copied into the launch
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  // Groups go into launches of up to MAXG non-empty groups each; `next` is the
  // first group not yet placed (empty groups are skipped, not counted).
  int next = 0;
  while (next < num_groups) {
    std::memset(&P, 0, sizeof(P));
    int tiles = 0, n = 0;
    int i = next;
    for (; i < num_groups && n < MAXG; ++i) {
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
      G.c = static_cast<__half*>(q.c);
      G.ldc = q.ldc;
      G.vec_ok = vec_ok(q.c, q.ldc);
      G.M = (int)q.M; G.N = (int)q.N; G.K = (int)q.K;
      G.tiles_m = (int)((q.M + C::TILE_M - 1) / C::TILE_M);
      G.tiles_n = (int)((q.N + C::BN - 1) / C::BN);
      G.tile_begin = tiles;
      tiles += G.tiles_m * G.tiles_n;
      ++n;
    }
    next = i;
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
  // CTA pairs (256 x 256 tiles, 5 stages) when every group's K is a multiple
  // of the 256-element stage; the single-CTA kernel handles the rest
  bool k256 = groups != nullptr && num_groups > 0;
  for (int i = 0; k256 && i < num_groups; ++i) k256 = groups[i].M == 0 || groups[i].K % 256 == 0;
  if (k256) return grouped_run<PairCfg<256, 5>>(groups, num_groups, stream);
  return grouped_run<GemmCfg<256, false, 4>>(groups, num_groups, stream);
}

extern "C" int nvfp4_gemm_skinny(const void* x, const void* w, const void* sfx, const void* sfw, void* out,
                                 int64_t T, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldo,
                                 void* stream) {
  if (T < 1 || T > 64) return fail(NVFP4_ERR_INVALID, "nvfp4_gemm_skinny: 1..64 token rows (got %lld)", (long long)T);
  // 512-element K stages (32 KB of weights each): half the per-stage handshakes of
  // 256-element stages (13.8 vs 16.3 us at T=16, N=14336, K=4096)
  if (T <= 16)
    return skinny_run<GemmCfg<16, false, 4, 1, 2>>(x, w, sfx, sfw, out, T, N, K, ldx, ldw, ldo, stream);
  if (T <= 32)
    return skinny_run<GemmCfg<32, false, 4, 1, 2>>(x, w, sfx, sfw, out, T, N, K, ldx, ldw, ldo, stream);
  return skinny_run<GemmCfg<64, false, 4, 1, 2>>(x, w, sfx, sfw, out, T, N, K, ldx, ldw, ldo, stream);
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
