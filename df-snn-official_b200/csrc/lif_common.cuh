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

// Correctly rounded a / b without the general IEEE division sequence, by Markstein's
// FMA-corrected quotient (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990; Theorem 8.10 of his
// "IA-64 and Elementary Functions", 2000): with y = RN(1/b) and a quotient q0 within one
// ulp of a/b, the remainder r = a - b*q0 is exact in one FMA and RN(q0 + r*y) = RN(a/b).
// y comes from the hardware reciprocal approximation refined by one Newton step.  Valid
// when a, b, 1/b and a/b stay in the normal range (callers guarantee 2 <= b <= 2^64 and
// 2^-60 <= |a| <= 2^60 and take __fdiv_rn otherwise); the tests compare it bit for bit
// with __fdiv_rn over every b mantissa.
__device__ __forceinline__ float rcp_approx(float b) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
    return y;
}

__device__ __forceinline__ float div_markstein(float a, float b) {
    const float y0 = rcp_approx(b);
    const float y = __fmaf_rn(__fmaf_rn(-b, y0, 1.0f), y0, y0);
    const float q0 = __fmul_rn(a, y);
    return __fmaf_rn(__fmaf_rn(-b, q0, a), y, q0);
}

// surrogate_fma with the quotient by div_markstein (sg checked on the host to lie in
// [2^-60, 2^60] in magnitude); 1+u*u >= 1 so only a huge or NaN denominator takes the
// IEEE division.  Bit-identical to surrogate_fma.
__device__ __forceinline__ float surrogate_fast(float z, float sg) {
    const float u = __fmul_rn(__fmul_rn(kPiHalf, sg), z);
    const float b = __fmul_rn(2.0f, __fmaf_rn(u, u, 1.0f));
    float q = div_markstein(sg, b);
    if (!(b <= 0x1p64f)) q = __fdiv_rn(sg, b);
    return q;
}

// Division by tau.  The reference divides (IEEE).  When tau is a power of two the
// quotient equals the product with 1/tau exactly, so the kernels may multiply instead.
template <bool TAU_POW2>
__device__ __forceinline__ float div_tau(float a, float tau, float inv_tau) {
    if constexpr (TAU_POW2) return __fmul_rn(a, inv_tau);
    else return __fdiv_rn(a, tau);
}

// Block-wide check that W (row stride T) is Toeplitz on its strict lower triangle and that
// scale is constant: W[t,i] == W[t-i,0] and scale[t] == scale[0], bitwise.  This is how the
// reference builds every glmulti schedule (spikeDE_dis/neuron.py:1494-1514); kernels then
// keep the T-1 distinct weights and the scale in registers.  Contains a block barrier.
__device__ __forceinline__ bool block_toeplitz(const float* W, const float* scale, int T) {
    int ok = 1;
    for (int e = threadIdx.x; e < T * T; e += blockDim.x) {
        const int t = e / T, i = e % T;
        if (i < t && __float_as_uint(W[e]) != __float_as_uint(W[(t - i) * T])) ok = 0;
    }
    for (int t = threadIdx.x; t < T; t += blockDim.x)
        if (__float_as_uint(scale[t]) != __float_as_uint(scale[0])) ok = 0;
    return __syncthreads_and(ok) != 0;
}

// Weight of history term (t, i): registers wr[t-i] (Toeplitz) or shared sW[t*TB+i].
template <int TB, bool FAST>
__device__ __forceinline__ float wgt(const float* sW, const float (&wr)[TB], int t, int i) {
    if constexpr (FAST) return wr[t - i];
    else return sW[t * TB + i];
}

__device__ __forceinline__ float ld_stream(const float* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float* p, float v) { __stcs(p, v); }

// Grid for a grid-stride ("persistent") kernel: enough blocks to fill every SM at the
// kernel's occupancy, never more than there are 256-neuron tiles.
template <class K>
inline unsigned persistent_grid(K kernel, int threads, size_t smem, long long N) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, threads, smem);
    if (per < 1) per = 1;
    const long long tiles = (N + threads - 1) / threads;
    long long g = (long long)sms * per;
    if (g > tiles) g = tiles;
    return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace dfsnn
