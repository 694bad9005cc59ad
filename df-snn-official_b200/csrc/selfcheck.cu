// selfcheck.cu -- dfsnn_check_surrogate_quotient: the Markstein quotient of
// lif_common.cuh against __fdiv_rn, and its refined reciprocal against __frcp_rn, over
// every denominator mantissa of the requested binades.
#include "../../include/dfsnn_b200.h"
#include "kernels.h"
#include "lif_common.cuh"

namespace dfsnn {
namespace {

__global__ void check_reciprocal(unsigned long long* bad) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (1u << 23)) return;
    const float b = __uint_as_float(0x3f800000u | i);
    const float y0 = rcp_approx(b);
    const float y = __fmaf_rn(__fmaf_rn(-b, y0, 1.0f), y0, y0);
    if (__float_as_uint(y) != __float_as_uint(__frcp_rn(b))) atomicAdd(bad, 1ull);
}

__global__ void check_quotient(const float* a, int na, int expo, unsigned long long* bad) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (1u << 23)) return;
    const float b = __uint_as_float(((uint32_t)expo << 23) | i);
    unsigned long long nb = 0;
    for (int k = 0; k < na; ++k)
        if (__float_as_uint(div_markstein(a[k], b)) != __float_as_uint(__fdiv_rn(a[k], b))) ++nb;
    if (nb) atomicAdd(bad, nb);
}

}  // namespace
}  // namespace dfsnn

extern "C" int dfsnn_check_surrogate_quotient(const float* a, int n_numerators, int exp_lo,
                                              int exp_hi, unsigned long long* mismatches,
                                              void* stream) {
    if (!a || !mismatches) return DFSNN_ERR_NULL;
    if (n_numerators < 1 || exp_lo < 128 || exp_hi > 191 || exp_lo > exp_hi) return DFSNN_ERR_PARAM;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(mismatches, 0, 2 * sizeof(unsigned long long), st);
    if (e != cudaSuccess) return dfsnn::record_cuda_error(e);
    const unsigned blocks = (1u << 23) / 256;
    for (int ex = exp_lo; ex <= exp_hi; ++ex)
        dfsnn::check_quotient<<<blocks, 256, 0, st>>>(a, n_numerators, ex, mismatches);
    dfsnn::check_reciprocal<<<blocks, 256, 0, st>>>(mismatches + 1);
    e = cudaGetLastError();
    return e == cudaSuccess ? DFSNN_OK : dfsnn::record_cuda_error(e);
}
