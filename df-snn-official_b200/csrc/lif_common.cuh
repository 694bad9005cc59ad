// lif_common.cuh -- shared device helpers for the LIF-FDE kernels (sm_100a).
//
// Arithmetic contract: every kernel reproduces the operation order of the reference CUDA
// kernels (spikeDE_dis/fde_cupy_kernels_all.py, examples/cnn128/aligned_glmulti.py,
// spikeDE_dis/direct_euler_cupy.py).  The reference is compiled by NVRTC with
// --fmad=true (library kernels) or --fmad=false (aligned kernels); here every rounding
// step is an explicit intrinsic (__fmaf_rn, __fmul_rn, __fadd_rn, __fsub_rn, __fdiv_rn)
// so the compiler cannot contract or reorder differently from the reference.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dfsnn {

constexpr float kPiHalf = 1.57079632679489661923f;          // fde_cupy_kernels_all.py:100
constexpr float kAlignedPiHalf = 1.5707963267948966f;        // aligned_glmulti.py:25

// Arctan surrogate derivative of the library kernels: u = (pi/2*a)*z; a / (2*(1+u*u)),
// with 1+u*u contracted to one fma (fde_cupy_kernels_all.py:143-146, :1862-1864).
__device__ __forceinline__ float surrogate_fma(float z, float sg) {
    const float u = __fmul_rn(__fmul_rn(kPiHalf, sg), z);
    return __fdiv_rn(sg, __fmul_rn(2.0f, __fmaf_rn(u, u, 1.0f)));
}

// Division by tau.  The reference divides (IEEE).  When tau is a power of two the
// quotient equals the product with 1/tau exactly, so the kernels may multiply instead.
template <bool TAU_POW2>
__device__ __forceinline__ float div_tau(float a, float tau, float inv_tau) {
    if constexpr (TAU_POW2) return __fmul_rn(a, inv_tau);
    else return __fdiv_rn(a, tau);
}

__device__ __forceinline__ float ld_stream(const float* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float* p, float v) { __stcs(p, v); }

}  // namespace dfsnn
