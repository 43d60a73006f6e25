// capi.cu -- library-wide entry points and host helpers of libssparse.so.
#include <mutex>

#include "common.cuh"

namespace ss {

int attention_prepare(int device);
int router_prepare(int device);
int attention_i8_prepare(int device);

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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

static int encode_2d_bf16(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                          uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return SS_ERR_DRIVER;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : SS_ERR_DRIVER;
}

// 2-D bf16 tensor map over a row-major [outer][inner] view, 128-byte swizzle, zero fill outside.
int encode_tmap_2d_bf16(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                        uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
    return encode_2d_bf16(map, base, inner, outer, row_stride_bytes, box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
}

// The same without swizzle: a box lands in shared memory as plain rows of box_inner elements.
int encode_tmap_2d_bf16_rows(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                             uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
    return encode_2d_bf16(map, base, inner, outer, row_stride_bytes, box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// 2-D uint8 tensor map over a row-major [outer][inner] view (int8 data), 128-byte swizzle.
int encode_tmap_2d_u8(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                      uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return SS_ERR_DRIVER;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : SS_ERR_DRIVER;
}

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

// The calling thread's current CUDA context (nullptr if none), through the driver entry point so
// the library does not link libcuda directly.
int current_context(void **ctx) {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    if (!fn) return SS_ERR_DRIVER;
    CUcontext c = nullptr;
    if (fn(&c) != CUDA_SUCCESS) return SS_ERR_DRIVER;
    *ctx = static_cast<void *>(c);
    return 0;
}

}  // namespace ss

extern "C" int ss_version(void) { return 101; }

extern "C" int ss_prepare_device(void) {
    int device;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return (int)e;
    int rc = ss::attention_prepare(device);
    if (rc) return rc;
    rc = ss::attention_i8_prepare(device);
    if (rc) return rc;
    return ss::router_prepare(device);
}
