// tmap.h — host-side TMA tensor-map encoding for the tcgen05 kernels.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

// cuTensorMapEncodeTiled, looked up through the runtime so the library does
// not link the driver library directly (it loads where no driver exists).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
inline EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// BF16 row-major [rows x cols] as a 2-D tensor map with 64 x box_rows boxes
// and 128-byte swizzle (the UMMA K-major canonical layout). Rows past `rows`
// read as zeros (partial tiles).
inline bool tmap_bf16(CUtensorMap *m, const void *base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc || !base) return false;
    cuuint64_t dims[2] = {cols, rows < 1 ? 1 : rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
