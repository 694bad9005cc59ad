// pack2.cuh -- two neurons per thread with Blackwell's packed fp32x2 arithmetic.
//
// sm_100 issues FFMA2/FADD2/FMUL2: one instruction applies the same IEEE fp32 operation,
// rounded to nearest, to both halves of a float2.  Each half is therefore bit-identical to
// the scalar operation the reference performs on that neuron.  Subtractions are written as
// fma(b, -1, a) = round(a - b) and histories that enter with a minus sign are accumulated
// negated (round-to-nearest is symmetric: round(-x) = -round(x)), so no separate negations
// are issued.  Only the sign of an exact zero can differ from the scalar form.
#pragma once
#include <cuda_runtime.h>

namespace dfsnn {

__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
// round(a - b) per half
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __ffma2_rn(b, f2(-1.0f), a); }

// The same operations as inline PTX (fma/add/sub/mul .rn.f32x2, sm_100+).
//
// Rule for every packed kernel here: a packed product never feeds a packed sum (unless it is
// formed by pmz2 below).  GPU probes
// (2^17 neuron pairs) showed that a packed multiply whose result is consumed by a packed
// add/sub can be fused into one packed FMA by the optimised code -- for the intrinsics and
// for these .rn PTX forms alike, depending on context -- which changes the rounding.  Such
// sums are written with the per-half scalar helpers below (sadd2/ssub2), which are never
// contracted.  A packed Kahan chain whose running sum is a packed add was also seen to lose
// its compensation; that add is scalar too (single_order.cu).
__device__ __forceinline__ unsigned long long pk(float2 a) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
    return r;
}
__device__ __forceinline__ float2 upk(unsigned long long r) {
    float2 a;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
    return a;
}
__device__ __forceinline__ float2 pfma2(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
    return upk(d);
}
__device__ __forceinline__ float2 padd2(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
    return upk(d);
}
__device__ __forceinline__ float2 psub2(float2 a, float2 b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
    return upk(d);
}
__device__ __forceinline__ float2 pmul2(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk(a)), "l"(pk(b)));
    return upk(d);
}

// A packed product that a packed sum may consume: fma(a, b, z) with z = -0 per half equals
// round(a*b) bit for bit (signed zeros included), and because z is a kernel argument the
// compiler cannot tell the fma from a product, so it has nothing to contract the following
// add with.  GPU probe: 0 of 6.7e7 accumulated values differ from the per-half scalar
// product-then-sum, against 43 % for a packed multiply feeding a packed add.  Callers pass
// nz = f2(args.negz) with negz == -0.0f set by the host.
__device__ __forceinline__ float2 pmz2(float2 a, float2 b, float2 nz) { return pfma2(a, b, nz); }

// per-half scalar operations (separately rounded, never contracted)
__device__ __forceinline__ float2 sadd2(float2 a, float2 b) {
    return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
}
__device__ __forceinline__ float2 ssub2(float2 a, float2 b) {
    return make_float2(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y));
}
__device__ __forceinline__ float2 smul2(float2 a, float2 b) {
    return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
}


// Per-half division by tau (IEEE) or product with 1/tau when tau is a power of two.
template <bool TAU_POW2>
__device__ __forceinline__ float2 div_tau2(float2 a, float tau, float2 inv_tau) {
    if constexpr (TAU_POW2) return mul2(a, inv_tau);
    else return make_float2(__fdiv_rn(a.x, tau), __fdiv_rn(a.y, tau));
}

__device__ __forceinline__ float2 ld2_stream(const float* p) {
    return __ldcs(reinterpret_cast<const float2*>(p));
}
__device__ __forceinline__ void st2_stream(float* p, float2 v) {
    __stcs(reinterpret_cast<float2*>(p), v);
}

// Spike of each half (p >= th) as 0/1 floats.
__device__ __forceinline__ float2 fire2(float2 p, float th) {
    return make_float2(p.x >= th ? 1.0f : 0.0f, p.y >= th ? 1.0f : 0.0f);
}

}  // namespace dfsnn
