// Host-side TMA tensor-map encoding through the driver entry point (no link against libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// 3-D bf16/fp16 tensor [d2][d1][d0] (d0 contiguous, elements), strides in elements for d1 and d2,
// box (64 elements of d0 = 128 bytes, 1, box2) with 128-byte swizzle: one tile = box2 rows of 128 B.
// Out-of-range rows read as zero. Returns false on failure (alignment, driver).
inline bool make_tmap_3d_sw128(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                               uint64_t stride1_elems, uint64_t stride2_elems, uint32_t box2, int elem_bytes = 2) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || ((uintptr_t)base & 15)) return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1_elems * elem_bytes, stride2_elems * elem_bytes};
    const cuuint32_t box[3] = {(cuuint32_t)(128 / elem_bytes), 1, box2};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gdn
