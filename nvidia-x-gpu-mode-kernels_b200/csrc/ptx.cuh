// Inline-PTX primitives for sm_100a shared by the NVFP4 kernels:
// mbarriers with bounded waits, tensor-map TMA loads, numeric conversions,
// and the device-side error word every bounded wait reports into.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace nvfp4 {

// Error bits recorded by kernels (OR-ed into the device error word).
enum : uint32_t {
  kDevErrTimeoutFull  = 1u << 0,   // consumer gave up waiting for a stage to fill
  kDevErrTimeoutEmpty = 1u << 1,   // producer gave up waiting for a stage to drain
  kDevErrTimeoutMma   = 1u << 2,   // MMA / epilogue handshake gave up
  kDevErrTimeoutTest  = 1u << 3,   // deliberately unsatisfied wait (self-test)
  kDevErrTimeoutPeer  = 1u << 4,   // a peer GPU's rows did not arrive (fused all-gather)
};

// Wait budget for every spin in this library: 2 s of %globaltimer.  A healthy
// pipeline waits microseconds; a stage that never fills (a lost copy) makes the
// waiter record an error bit and leave instead of hanging the GPU.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}

// Non-blocking-to-the-caller probe of a phase (try_wait may suspend the
// thread briefly until the phase completes).
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (after
// OR-ing `err_bit` into *err) when the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          uint32_t* err, uint32_t err_bit,
                                          uint64_t budget_ns = kWaitBudgetNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 15u && globaltimer() - t0 > budget_ns) {
      if (err) atomicOr(err, err_bit);
      return false;
    }
  }
}

// ---- thread-block clusters (CTA pairs) ------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %nclusterid.x;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (a shared::cluster
// address from mapa), with the instruction's default semantics, as cluster
// pipelines conventionally do; the explicit .release.cluster form compiles to
// a full memory barrier per arrival.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Tensor-map TMA loads (no multicast anywhere in this library).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar,
                                            int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4}], [%2], %5;"
      :: "r"(dst), "l"(tmap), "r"(bar), "r"(x), "r"(y), "l"(policy) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar,
                                            int x, int y, int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4, %5}], [%2], %6;"
      :: "r"(dst), "l"(tmap), "r"(bar), "r"(x), "r"(y), "r"(z), "l"(policy) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(tmap) : "memory");
}

// ---- numeric conversions used by the dequantising dot products ----------

// Two e2m1 codes (one byte) -> f16x2 (low nibble -> low half).
__device__ __forceinline__ uint32_t cvt_e2m1x2(uint32_t byte) {
  uint32_t r;
  asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}\n"
      : "=r"(r) : "r"(byte));
  return r;
}

// Four e2m1 byte pairs of a 32-bit word -> four f16x2 values.
__device__ __forceinline__ void cvt_e2m1x8(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n"
      " mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}\n"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3]) : "r"(w));
}

// Two e4m3 bytes (low 16 bits) -> f16x2.
__device__ __forceinline__ uint32_t cvt_e4m3x2(uint32_t two) {
  uint32_t r;
  asm("{\n .reg .b16 t;\n cvt.u16.u32 t, %1;\n cvt.rn.f16x2.e4m3x2 %0, t;\n}\n"
      : "=r"(r) : "r"(two));
  return r;
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// f16x2 -> (low, high) as f32.
__device__ __forceinline__ void h2_to_f2(uint32_t h, float& lo, float& hi) {
  asm("{\n .reg .f16 l, h;\n mov.b32 {l, h}, %2;\n cvt.f32.f16 %0, l;\n cvt.f32.f16 %1, h;\n}\n"
      : "=f"(lo), "=f"(hi) : "r"(h));
}

}  // namespace nvfp4
