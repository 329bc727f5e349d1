/*
 * nvfp4_b200.h — C ABI of libnvfp4_b200.so, a B200 (sm_100a) NVFP4 kernel library.
 *
 * Data formats (all entry points):
 *   - FP4 operands are e2m1 codes packed two per byte, K contiguous ("K-major"),
 *     the even K index in the low nibble.
 *   - Block scales are e4m3fn bytes, one per 16 consecutive K elements.
 *   - Outputs are IEEE fp16.  Accumulation is fp32.
 *
 * Conventions: every function returns 0 (NVFP4_OK) or a positive status code and
 * never throws; nvfp4_last_error() gives the calling thread's last message.
 * Work is enqueued on the caller's stream (a cudaStream_t passed as void*; NULL is
 * the legacy default stream) on the current device; no function synchronises
 * unless its comment says so.  Pointers are device pointers.
 */
#ifndef NVFP4_B200_H_
#define NVFP4_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define NVFP4_API __attribute__((visibility("default")))
#else
#define NVFP4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum nvfp4_status {
  NVFP4_OK = 0,
  NVFP4_ERR_INVALID = 1,      /* bad shape, stride or null pointer */
  NVFP4_ERR_ALIGNMENT = 2,    /* a pointer or stride breaks a 16-byte rule */
  NVFP4_ERR_CUDA = 3,         /* a CUDA runtime / driver call failed */
  NVFP4_ERR_TIMEOUT = 4,      /* a device-side bounded wait expired */
  NVFP4_ERR_UNSUPPORTED = 5,  /* no kernel for this device or shape */
};

/* Message for the last non-zero status returned on this thread. */
NVFP4_API const char* nvfp4_last_error(void);

/* Library version as 10000*major + 100*minor + patch. */
NVFP4_API int nvfp4_version(void);

/*
 * Batched block-scaled GEMV.
 *   c[m, l] = sum_k e2m1(a[m, k, l]) * e2m1(b[k, l]) * e4m3(sfa[m, k/16, l]) * e4m3(sfb[k/16, l])
 *
 * Replaces the reference's pybind entry
 *   void nvfp4_gemv_forward(const at::Tensor& a, const at::Tensor& b,
 *                           const at::Tensor& sa, const at::Tensor& sb,
 *                           at::Tensor& c, int64_t M, int64_t K, int64_t L)
 * (Nvidia-x-GPU-MODE-Kernels, blackwell_nvfp4_gemv.cu:500-524), whose tensors are
 * a [M, K/2, L], b [>=1, K/2, L] (row 0 read), sa [M, K/16, L], sb [>=1, K/16, L],
 * c [M, 1, L]; the strides that the reference reads from the tensors
 * (blackwell_nvfp4_gemv.cu:226-227, 257-258, 270-271, 284-285, 495-497) are explicit
 * here.  Innermost (K) strides are 1.
 *
 *   a_sm, a_sl      : byte strides of a along M and L
 *   b_sl            : byte stride of b along L
 *   sfa_sm, sfa_sl  : byte strides of sfa along M and L
 *   sfb_sl          : byte stride of sfb along L
 *   c_sm, c_sl      : element strides of c along M and L
 *
 * Requirements: M, L >= 1; K >= 16 and K % 16 == 0.  The TMA-streaming kernel is
 * used when K % 256 == 0 and every pointer and byte stride is a multiple of 16;
 * other valid shapes run a plain-load kernel with the same arithmetic.
 */
NVFP4_API int nvfp4_gemv(const void* a, const void* b, const void* sfa, const void* sfb, void* c,
               int64_t M, int64_t K, int64_t L,
               int64_t a_sm, int64_t a_sl, int64_t b_sl,
               int64_t sfa_sm, int64_t sfa_sl, int64_t sfb_sl,
               int64_t c_sm, int64_t c_sl, void* stream);

/* Number of CTAs the nvfp4_gemv TMA path launches for this shape (aligned inputs). */
NVFP4_API int nvfp4_gemv_grid(int64_t M, int64_t K, int64_t L, int64_t* grid);

/*
 * Row-sharded GEMV with the output all-gather fused in (one launch per rank,
 * one rank per GPU).  This rank computes rows [m_off, m_off + M_local) of the
 * full M_total-row output (its a / sfa hold only those rows) and sends each
 * result to every rank; the launch returns once `out` holds the full output
 * [M_total, 1, L] (fp16, element strides c_sm / c_sl, on this GPU).
 *
 * peer_stage[r] is rank r's staging buffer, a device pointer valid on this GPU
 * (peer memory over NVLink, e.g. from torch symmetric memory), 8-byte aligned,
 * zero-initialised, of at least 64 + 2 * M_total * L 32-bit words.  Protocol:
 * results travel as 64-bit lines (epoch << 32 | fp16 bits) to every rank's
 * buffer, from 64-bit index 32 on.  When M_total is even a line holds two
 * elements, e = 2i and 2i + 1 (e = l * M_total + m) in line i, low half first,
 * and every rank's m_off and M_local must then be even (NVFP4_ERR_INVALID
 * otherwise); when M_total is odd a line holds element e = i.  A naturally
 * aligned 64-bit store is single-copy atomic, so a line carrying this call's
 * epoch carries this call's values and no fence or counter gates it.  Each CTA
 * then copies its slice of the lines into `out`, waiting for each to carry the
 * epoch.  Words 0-63 of this rank's buffer are control words: 16 counts
 * finished CTAs (reset by the last one), 20 holds the epoch in device-epoch
 * mode, 32-37 receive three 64-bit %globaltimer stamps (low word first): the
 * launch's start, CTA 0 having sent its rows, and the last CTA holding its
 * slice.
 *
 * `epoch` is the 1-based count of calls made with these staging buffers (the
 * same on every rank; the shape must stay the same between calls).
 * epoch == 0 selects device-epoch mode: the kernel keeps the count in word 20
 * of this rank's buffer, so a captured CUDA graph of the call advances it on
 * every replay (use one mode per set of buffers).  Every wait is bounded (2 s
 * by default, see nvfp4_set_peer_wait_ns; error bit 16 in nvfp4_device_errors()).
 * Requires the aligned (TMA) path; world <= 8.  Replaces "nvfp4_gemv_forward
 * + an output all-gather" (the reference has no distributed code; the north
 * star asks for row sharding with an output all-gather).
 */
NVFP4_API int nvfp4_gemv_allgather(const void* a, const void* b, const void* sfa, const void* sfb,
                                   int64_t M_local, int64_t K, int64_t L,
                                   int64_t a_sm, int64_t a_sl, int64_t b_sl,
                                   int64_t sfa_sm, int64_t sfa_sl, int64_t sfb_sl,
                                   void* out, int64_t c_sm, int64_t c_sl, int64_t m_off, int64_t M_total,
                                   void* const* peer_stage, int world, int rank, uint32_t epoch,
                                   void* stream);

/*
 * Budget of the fused all-gather's wait for the other ranks' rows, in
 * nanoseconds, for launches made after the call (process-wide).  0 restores the
 * default of 2 s; other values must lie in [1e3, 2e9].  A short budget lets a
 * caller (or a test) detect a rank that never delivers without stalling for the
 * default.  No counterpart in the reference, whose waits never expire
 * (blackwell_nvfp4_gemv.cu:150-157).
 */
NVFP4_API int nvfp4_set_peer_wait_ns(uint64_t ns);

/*
 * Reads this device's error word (bits set by device-side bounded waits that
 * expired) and, when `clear` is non-zero, resets it.  Synchronises the device.
 * No counterpart in the reference, whose waits never expire
 * (blackwell_nvfp4_gemv.cu:150-157).
 */
NVFP4_API int nvfp4_device_errors(uint32_t* out_bits, int clear);

/*
 * Self-test of the bounded-wait machinery: launches one block that waits on an
 * mbarrier nothing will ever complete, with a budget of `budget_ns` nanoseconds
 * (clamped to [1e3, 1e9]); synchronises and returns NVFP4_ERR_TIMEOUT when the
 * wait expired as designed, NVFP4_OK if it (impossibly) completed.  No
 * counterpart in the reference.
 */
NVFP4_API int nvfp4_selftest_wait_timeout(uint64_t budget_ns, void* stream);

/*
 * The same self-test without any device allocation, for callers that cannot
 * allocate device memory (a serving process whose allocator already owns all
 * of the GPU's memory, or a host runtime with no device-allocation hook).
 * Launches `waiters` blocks (1..64), each waiting with budget `budget_ns` on a
 * barrier nothing completes, and stores in *expired how many waits gave up;
 * returns NVFP4_ERR_TIMEOUT when any did (the expected outcome), and
 * NVFP4_ERR_INVALID for more than 64 waiters.  The outcome words live in a
 * fixed 256-byte array inside the library that every GPU loading the library
 * keeps until exit; the first call on a device resolves its address (make that
 * call before any stream capture).  Calls share the array and clear the words
 * they use, so calls that overlap on the GPU race.  Synchronises `stream`.
 * No counterpart in the reference.
 */
NVFP4_API int nvfp4_selftest_wait_timeout_noalloc(uint64_t budget_ns, int waiters, int* expired, void* stream);


/*
 * NVFP4 GEMM operands (dual and grouped GEMM): an operand with `rows` rows is
 *   codes   [rows, K/2] bytes, row stride ld (bytes, a multiple of 16), K-major;
 *   scales  e4m3 (unsigned: sign bit 0), one per 16 K-elements, in the 128x4
 *           blocked layout: 128-row x 4-column tiles of 512 bytes, row-tile
 *           major; inside a tile the scale of (row r, block c) sits at byte
 *           (r % 32) * 16 + (r / 32 % 4) * 4 + c % 4; rows padded to 128 and
 *           K/16 to a multiple of 4 with zeros.
 * K must be a multiple of 64; operand pointers 16-byte aligned.  Outputs are
 * fp16 with row stride ldc elements (16-byte stores when the pointer is 16-byte
 * aligned and ldc % 8 == 0, element stores otherwise).  No counterpart exists in the
 * reference, which ships only the GEMV and announces a dual GEMM
 * (Nvidia-x-GPU-MODE-Kernels README.md:3); the contract is
 * fp32 accumulation of the dequantised products, one rounding to fp16.
 */

/* out[M, N] = silu(A . B1^T) * (A . B2^T); B1, B2 are [N, K/2] with row stride ldb. */
NVFP4_API int nvfp4_dual_gemm(const void* a, const void* b1, const void* b2,
                              const void* sfa, const void* sfb1, const void* sfb2, void* out,
                              int64_t M, int64_t N, int64_t K,
                              int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/* One problem of a grouped GEMM: c[M, N] = a[M, K] . b[N, K]^T. */
typedef struct nvfp4_group {
  const void* a;
  const void* b;
  const void* sfa;
  const void* sfb;
  void* c;
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
} nvfp4_group;

/*
 * Grouped GEMM over `num_groups` independent problems (host array of
 * descriptors; groups with M == 0 are skipped).  One persistent launch covers
 * up to 24 groups; its CTAs walk the tiles of all groups.
 */
NVFP4_API int nvfp4_grouped_gemm(const nvfp4_group* groups, int num_groups, void* stream);

/*
 * Skinny GEMM for decode batches: out[T, N] = x[T, K] . w[N, K]^T with
 * 1 <= T <= 64 token rows (operand conventions as above; out row stride ldo
 * elements).  The weights stream through the tensor cores as the MMA's
 * 128-row operand ("swap-AB"), the tokens form one 16/32/64-wide tile, and
 * the epilogue writes the transposed accumulator.  One CTA per 128 weight
 * rows.  No counterpart in the reference.
 */
NVFP4_API int nvfp4_gemm_skinny(const void* x, const void* w, const void* sfx, const void* sfw, void* out,
                                int64_t T, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldo,
                                void* stream);

/*
 * Fused NVFP4 quantiser for GEMM activations: x [M, K] fp16 (row stride ldx
 * elements, K % 16 == 0) -> codes [M, K/2] (row stride ldq bytes) and e4m3
 * scales written straight into the 128x4 blocked layout (buffer of
 * ceil(M/128) * ceil(K/64) * 512 bytes; padding bytes are written as 0).
 * Per 16-element block, global scale 1.0:  s = e4m3_rne_satfinite(amax / 6),
 * q_i = e2m1_rne_satfinite(x_i * fl32(1 / s)) (one IEEE f32 reciprocal per
 * block, f32 products); a block whose s is 0 gets all-zero codes.  Finite inputs.  No counterpart in the reference
 * (its inputs arrive already quantised); it produces the operands of
 * nvfp4_dual_gemm / nvfp4_grouped_gemm.
 */
NVFP4_API int nvfp4_quantize(const void* x, int64_t M, int64_t K, int64_t ldx, void* codes, int64_t ldq,
                             void* sf_blocked, void* stream);

/*
 * Tensor-core peak probe: one CTA per SM issues `iters` dense 128x256x64
 * kind::mxf4nvf4 MMAs (4,194,304 FLOP each) from shared memory.  Time it with
 * events on `stream` to get the device's FP4 tensor throughput, the
 * denominator of the GEMMs' roofline fraction.  No counterpart in the reference.
 */
NVFP4_API int nvfp4_mma_peak(int iters, void* stream);

/*
 * The same probe under a chosen operand pattern: 0 = one fixed scale column
 * pair and whatever shared memory holds (what nvfp4_mma_peak runs); 1 = the
 * GEMMs' conditions: pseudo-random operand bytes, e4m3 scales in 2^[-3, 3],
 * scale columns advancing per K step through four 48-column stages.  The
 * tensor pipe's rate depends on both, so pattern 1 is the attainable rate for
 * the GEMM kernels' instruction stream.
 */
NVFP4_API int nvfp4_mma_peak_pattern(int iters, int pattern, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_B200_H_ */
