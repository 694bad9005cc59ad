// tma.cu -- host side of tma.cuh: tensor-map encoding through the driver entry point
// (fetched once from the runtime, so the library needs no link-time libcuda).
#include <mutex>

#include "tma.cuh"

namespace dfsnn {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();   // leave no sticky error behind
    });
    return fn;
}

}  // namespace

bool encode_rows_map(CUtensorMap* map, const float* base, long long N, int rows, int box_n) {
    // box coordinates are signed 32-bit: keep every tile start below 2^31
    if (!base || N < 1 || N > (1ll << 31) - 256 || (N % 4) != 0) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
    if (rows < 1 || rows > 256 || box_n < 4 || box_n > 256 || (box_n % 4) != 0) return false;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)N * sizeof(float)};
    const cuuint32_t box[2] = {(cuuint32_t)box_n, (cuuint32_t)rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace dfsnn
