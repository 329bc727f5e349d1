// Tensor-map (TMA descriptor) encoding through the driver entry point, so the
// library needs no link-time libcuda.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace nvfp4 {

// Encodes a tiled tensor map.  dims/box are innermost-first; strides are the
// byte strides of dims 1..rank-1.  Returns NVFP4_OK or an error status (with
// the message recorded).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

}  // namespace nvfp4
