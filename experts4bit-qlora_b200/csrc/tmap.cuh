// Host-side tensor-map encoding through the driver entry point (no libcuda link).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace e4b {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Encodes a tiled map; false on failure.
inline bool encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
                         const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn f = encode_tiled_fn();
  if (!f) return false;
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return f(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace e4b
