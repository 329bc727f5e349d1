// Library-wide C ABI pieces: error messages, version, the per-device error word
// that bounded waits report into, and the bounded-wait self-test kernel.
#include <atomic>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include "ptx.cuh"
#include "common.h"
#include "tmap.h"

namespace nvfp4 {

namespace {
thread_local char g_msg[512] = "";

// One word per device (a __device__ variable exists once per device context).
__device__ uint32_t g_error_word;

constexpr int kMaxDevices = 64;
// Per-device addresses, published with release stores and read with acquire
// loads outside the lock (double-checked initialisation).
std::atomic<uint32_t*> g_err_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
std::mutex g_mu;

__global__ void selftest_wait_kernel(uint32_t* err, uint64_t budget_ns, uint32_t* done) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait must run out and report.
  const bool ok = mbar_wait(b, 0, err, kDevErrTimeoutTest, budget_ns);
  if (threadIdx.x == 0) *done = ok ? 1u : 2u;
}
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

uint32_t* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (uint32_t* p = g_err_ptr[dev].load(std::memory_order_acquire)) return p;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev].load(std::memory_order_relaxed)) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev].store(static_cast<uint32_t*>(p), std::memory_order_release);
  }
  return g_err_ptr[dev].load(std::memory_order_relaxed);
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (!g_sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  if (g_encode) return g_encode;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return g_encode;
}
}  // namespace

namespace {
// Cache of encoded tensor maps keyed by every encoding argument (a map depends
// on nothing else), so repeated calls on the same buffers skip the driver.
struct TmapKey {
  const void* base;
  uint64_t dims[5];
  uint64_t strides[4];
  uint32_t box[5];
  int dtype, rank, swizzle, promo;
  bool operator==(const TmapKey& o) const { return std::memcmp(this, &o, sizeof(TmapKey)) == 0; }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    const uint64_t* w = reinterpret_cast<const uint64_t*>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(TmapKey) / 8; ++i) h = (h ^ w[i]) * 1099511628211ull;
    return (size_t)h;
  }
};
std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> g_tmap_cache;
std::mutex g_tmap_mu;
constexpr size_t kTmapCacheMax = 4096;
}  // namespace

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  TmapKey key;
  std::memset(&key, 0, sizeof(key));
  key.base = base;
  key.dtype = (int)dtype;
  key.rank = rank;
  key.swizzle = (int)swizzle;
  key.promo = (int)promo;
  for (int i = 0; i < rank && i < 5; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) key.strides[i] = strides_bytes[i];
  }
  {
    std::lock_guard<std::mutex> lk(g_tmap_mu);
    auto it = g_tmap_cache.find(key);
    if (it != g_tmap_cache.end()) {
      *map = it->second;
      return NVFP4_OK;
    }
  }
  auto fn = encode_fn();
  if (!fn) return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t gd[5], gs[4];
  cuuint32_t bd[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bd[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) gs[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bd, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rank %d dims[0]=%llu box[0]=%u", (int)r,
                rank, (unsigned long long)dims[0], box[0]);
  std::lock_guard<std::mutex> lk(g_tmap_mu);
  if (g_tmap_cache.size() >= kTmapCacheMax) g_tmap_cache.clear();
  g_tmap_cache.emplace(key, *map);
  return NVFP4_OK;
}

}  // namespace nvfp4

extern "C" const char* nvfp4_last_error(void) { return nvfp4::g_msg; }

extern "C" int nvfp4_version(void) { return 100; }

extern "C" int nvfp4_device_errors(uint32_t* out_bits, int clear) {
  using namespace nvfp4;
  if (!out_bits) return fail(NVFP4_ERR_INVALID, "nvfp4_device_errors: null output");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  uint32_t v = 0;
  e = cudaMemcpyFromSymbol(&v, g_error_word, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(error word)");
  *out_bits = v;
  if (clear) {
    const uint32_t z = 0;
    e = cudaMemcpyToSymbol(g_error_word, &z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(error word)");
  }
  return NVFP4_OK;
}

extern "C" int nvfp4_selftest_wait_timeout(uint64_t budget_ns, void* stream) {
  using namespace nvfp4;
  if (budget_ns < 1000ull) budget_ns = 1000ull;
  if (budget_ns > 1000000000ull) budget_ns = 1000000000ull;
  uint32_t* err = device_error_word();
  if (!err) return fail(NVFP4_ERR_CUDA, "selftest: no device error word");
  // The kernel reports how its wait ended through a small device flag.
  uint32_t* done = nullptr;
  cudaError_t e = cudaMalloc(&done, sizeof(uint32_t));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(selftest flag)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaMemsetAsync(done, 0, sizeof(uint32_t), st);
  selftest_wait_kernel<<<1, 32, 0, st>>>(err, budget_ns, done);
  int rc = check_launch("selftest_wait_kernel");
  uint32_t h = 0;
  if (rc == NVFP4_OK) {
    e = cudaMemcpyAsync(&h, done, sizeof(h), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = cuda_fail(e, "selftest sync");
  }
  cudaFree(done);
  if (rc != NVFP4_OK) return rc;
  if (h == 2u) return fail(NVFP4_ERR_TIMEOUT, "selftest: wait expired after %llu ns (expected)",
                           (unsigned long long)budget_ns);
  return NVFP4_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free form of the bounded-wait self-test.
//
// nvfp4_selftest_wait_timeout allocates a 4-byte device word for each run.
// Some callers cannot allocate device memory at all: a serving process whose
// allocator has reserved every byte of the GPU up front, or a host runtime
// that has no hook for device allocations, still wants to check that the
// library's waits give up instead of hanging.  This entry point keeps the
// words it needs in a fixed array inside the library: 64 32-bit words
// (256 bytes), one per waiting block, resident on every GPU that loads the
// library until the process exits.  The caller passes the budget and the
// number of waiting blocks, and gets back how many waits expired.
// ---------------------------------------------------------------------------
namespace nvfp4 {
namespace {

constexpr int kSelftestMaxWaiters = 64;
static __device__ __align__(256) uint32_t g_selftest_scratch[kSelftestMaxWaiters];

std::atomic<uint32_t*> g_selftest_ptr[kMaxDevices] = {};

// Each block waits on its own mbarrier that nothing completes; thread 0
// records 1 (completed) or 2 (expired) in word blockIdx.x of `outcome`.
__global__ void selftest_wait_noalloc_kernel(uint32_t* err, uint64_t budget_ns, uint32_t* outcome) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait(b, 0, err, kDevErrTimeoutTest, budget_ns);
  if (threadIdx.x == 0) outcome[blockIdx.x] = ok ? 1u : 2u;
}

// Device address of this device's array, resolved once with the device
// current (the array's name is only a host-side stand-in).
int selftest_scratch(uint32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NVFP4_ERR_UNSUPPORTED, "device index %d out of range", dev);
  uint32_t* ptr = g_selftest_ptr[dev].load(std::memory_order_acquire);
  if (!ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    ptr = g_selftest_ptr[dev].load(std::memory_order_relaxed);
    if (!ptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_selftest_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(self-test scratch)");
      ptr = static_cast<uint32_t*>(p);
      g_selftest_ptr[dev].store(ptr, std::memory_order_release);
    }
  }
  *out = ptr;
  return NVFP4_OK;
}

}  // namespace
}  // namespace nvfp4

extern "C" int nvfp4_selftest_wait_timeout_noalloc(uint64_t budget_ns, int waiters, int* expired, void* stream) {
  using namespace nvfp4;
  if (!expired) return fail(NVFP4_ERR_INVALID, "nvfp4_selftest_wait_timeout_noalloc: null output");
  if (waiters < 1 || waiters > kSelftestMaxWaiters)
    return fail(NVFP4_ERR_INVALID,
                "nvfp4_selftest_wait_timeout_noalloc: waiters must be 1..%d (the built-in scratch holds %d words), "
                "got %d", kSelftestMaxWaiters, kSelftestMaxWaiters, waiters);
  if (budget_ns < 1000ull) budget_ns = 1000ull;
  if (budget_ns > 1000000000ull) budget_ns = 1000000000ull;
  uint32_t* err = device_error_word();
  if (!err) return fail(NVFP4_ERR_CUDA, "self-test: no device error word");
  uint32_t* words = nullptr;
  int rc = selftest_scratch(&words);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the array keeps the previous call's outcomes: clear the words this call uses
  cudaError_t e = cudaMemsetAsync(words, 0, sizeof(uint32_t) * waiters, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(self-test scratch)");
  selftest_wait_noalloc_kernel<<<waiters, 32, 0, st>>>(err, budget_ns, words);
  rc = check_launch("selftest_wait_noalloc_kernel");
  if (rc) return rc;
  uint32_t h[kSelftestMaxWaiters] = {};
  e = cudaMemcpyAsync(h, words, sizeof(uint32_t) * waiters, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "self-test readback");
  int n = 0;
  for (int i = 0; i < waiters; ++i) n += (h[i] == 2u) ? 1 : 0;
  *expired = n;
  if (n > 0) return fail(NVFP4_ERR_TIMEOUT, "self-test: %d of %d waits expired after %llu ns (expected)", n, waiters,
                         (unsigned long long)budget_ns);
  return NVFP4_OK;
}
