/*
 * A plain C caller of the C ABI, compiled with gcc against include/nvfp4_b200.h
 * and linked against the built library: the shape of the binding a non-Python
 * host (a cgo / JNI / FFI layer) would write.  It runs without a GPU: it checks
 * the version, and that invalid calls return the documented status codes with
 * a message, before any CUDA work.  Prints one line per check; exit code 0 when
 * all pass.
 */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "nvfp4_b200.h"

static int failures = 0;

static void expect(const char* what, int got, int want, const char* needle) {
  const char* msg = nvfp4_last_error();
  int ok = got == want && (needle == NULL || (msg != NULL && strstr(msg, needle) != NULL));
  printf("%s %s (status %d, message \"%s\")\n", ok ? "ok  " : "FAIL", what, got, msg ? msg : "");
  if (!ok) ++failures;
}

int main(void) {
  /* a 16-byte aligned stand-in: validation rejects before dereferencing */
  static unsigned char buf[64] __attribute__((aligned(16)));
  void* p = buf;
  printf("nvfp4_version %d\n", nvfp4_version());
  if (nvfp4_version() < 100) ++failures;

  /* GEMV: K must be a multiple of 16; null inputs */
  expect("gemv K%16", nvfp4_gemv(p, p, p, p, p, 4, 24, 1, 12, 0, 0, 2, 0, 0, 1, 0, NULL), NVFP4_ERR_INVALID, "K%16");
  expect("gemv null a", nvfp4_gemv(NULL, p, p, p, p, 4, 32, 1, 16, 0, 0, 2, 0, 0, 1, 0, NULL), NVFP4_ERR_INVALID,
         "null");
  /* dual GEMM: K granularity; misaligned operand */
  expect("dual K%64", nvfp4_dual_gemm(p, p, p, p, p, p, p, 128, 128, 100, 64, 64, 128, NULL), NVFP4_ERR_INVALID,
         NULL);
  expect("dual misaligned", nvfp4_dual_gemm(buf + 8, p, p, p, p, p, p, 128, 128, 256, 128, 128, 128, NULL),
         NVFP4_ERR_ALIGNMENT, NULL);
  /* grouped GEMM: no groups */
  expect("grouped none", nvfp4_grouped_gemm(NULL, 0, NULL), NVFP4_ERR_INVALID, "no groups");
  /* skinny GEMM: token count */
  expect("skinny T=0", nvfp4_gemm_skinny(p, p, p, p, p, 0, 128, 256, 128, 128, 128, NULL), NVFP4_ERR_INVALID,
         "1..64");
  /* quantiser: odd fp16 address */
  expect("quantize odd", nvfp4_quantize(buf + 1, 8, 32, 32, p, 16, p, NULL), NVFP4_ERR_ALIGNMENT, NULL);
  /* tensor-core probe: pattern */
  expect("peak pattern", nvfp4_mma_peak_pattern(16, 7, NULL), NVFP4_ERR_INVALID, "pattern");

  printf("%s\n", failures ? "FAILED" : "all passed");
  return failures ? 1 : 0;
}
