// Library-wide C ABI pieces: error messages, version, the per-device error word
// that bounded waits report into, and the bounded-wait self-test kernel.
#include <cstring>
#include <mutex>
#include "ptx.cuh"
#include "common.h"
#include "tmap.h"

namespace nvfp4 {

namespace {
thread_local char g_msg[512] = "";

// One word per device (a __device__ variable exists once per device context).
__device__ uint32_t g_error_word;

constexpr int kMaxDevices = 64;
uint32_t* g_err_ptr[kMaxDevices] = {};
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
  if (g_err_ptr[dev]) return g_err_ptr[dev];
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<uint32_t*>(p);
  }
  return g_err_ptr[dev];
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

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
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
