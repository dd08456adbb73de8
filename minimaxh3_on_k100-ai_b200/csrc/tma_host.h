// Host-side construction of TMA tensor maps.  cuTensorMapEncodeTiled is a
// driver entry point; it is resolved once through cudaGetDriverEntryPoint so the
// library does not link libcuda directly.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/h3_b200.h"

namespace h3 {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// BF16 tensor map with 128-byte swizzle.  dims/strides innermost first; strides
// in bytes for dims 1..rank-1; box innermost first.  Returns H3 status.
inline int make_tmap_bf16(CUtensorMap *map, void *base, int rank, const cuuint64_t *dims,
                          const cuuint64_t *strides_bytes, const cuuint32_t *box) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return H3_ERR_DRIVER;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, base, dims, strides_bytes, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? H3_OK : H3_ERR_BAD_LAYOUT;
}

}  // namespace h3
