// aligned.cu -- "aligned" distributed-order GL LIF kernels for sm_100a.
//
// Replaces AlignedGLMulti of examples/cnn128/aligned_glmulti.py (the glmulti semantics the
// CNN128 / Spikformer256 examples install over LIFFDEGLMultiFunction, :157-162):
//   forward  aligned_forward (:7-17): spike decided on the predicted voltage v+d, reset
//            folded into the drift;
//   backward aligned_backward (:20-32), the exact discrete VJP with history weight rho,
//            plus aligned_scale (:33-41) and the strictly-lower weight gradient
//            -(ga@h^T)*tril(-1) (:141-144).
// The reference compiles these with --fmad=false: every product and sum here is a
// separately rounded intrinsic, in the reference's order.
// The forward writes only spikes (the reference also writes pred and hist: 12 B vs 4 B
// per neuron-step); the backward is the same persistent, bulk-staged design as the glmulti
// backward (glmulti.cu), reducing grad a / grad W in-kernel.
#include <atomic>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "bulk_pipe.cuh"
#include "kernels.h"
#include "pack2.cuh"
#include "param_reduce.cuh"
#include "warp_tile.cuh"

namespace dfsnn {

struct AlnArgs {
    float negz;          // -0.0f, set by the host (pmz2: products a packed sum may consume)
    const float* x;
    const float* v0;
    const float* a;      // [T] per-step gain (the schedule's scale)
    const float* W;      // [T, T]
    const float* g;      // [T, N] upstream grad of the spikes
    float* spike;
    const void* xio;     // forward input x in the element type E of the forward kernels
    void* sio;           // forward spikes in the element type E
    float* gx;
    float* gv0;
    double* part;
    unsigned int* err;
    int T;
    long long N;
    float tau, inv_tau, th, sg, rho;
};

// Element I/O of the forward kernels: fp32, or the fp16 / bf16 activations that reach the
// layer under autocast.  The reference casts x with .float() and returns the spikes with
// .to(x.dtype) (aligned_glmulti.py:112-121); a half-precision value converts to fp32
// exactly and 0 / 1 spikes are exact in either type, so reading and writing the element
// type directly gives the same values with a quarter of the cast traffic.
template <typename E>
struct Io;
template <>
struct Io<float> {
    using Raw2 = float2;                                  // two elements as loaded
    static __device__ __forceinline__ Raw2 ld2raw(const void* p, long long i) { return ld2(p, i); }
    static __device__ __forceinline__ float2 cvt2(Raw2 r) { return r; }
    static __device__ __forceinline__ float ld(const void* p, long long i) {
        return __ldcs(static_cast<const float*>(p) + i);
    }
    static __device__ __forceinline__ float2 ld2(const void* p, long long i) {
        return __ldcs(reinterpret_cast<const float2*>(static_cast<const float*>(p) + i));
    }
    static __device__ __forceinline__ void st(void* p, long long i, float v) {
        __stcs(static_cast<float*>(p) + i, v);
    }
    static __device__ __forceinline__ void st2(void* p, long long i, float2 v) {
        __stcs(reinterpret_cast<float2*>(static_cast<float*>(p) + i), v);
    }
};
// two adjacent 16-bit elements as one 32-bit streaming access
__device__ __forceinline__ uint32_t ld_cs_b32(const void* p) {
    uint32_t v;
    asm("ld.global.cs.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void st_cs_b32(void* p, uint32_t v) {
    asm volatile("st.global.cs.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned short ld_cs_b16(const void* p) {
    unsigned short v;
    asm("ld.global.cs.b16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void st_cs_b16(void* p, unsigned short v) {
    asm volatile("st.global.cs.b16 [%0], %1;" ::"l"(p), "h"(v) : "memory");
}

template <>
struct Io<__half> {
    using Raw2 = uint32_t;
    static __device__ __forceinline__ Raw2 ld2raw(const void* p, long long i) {
        return ld_cs_b32(static_cast<const __half*>(p) + i);
    }
    static __device__ __forceinline__ float2 cvt2(Raw2 u) {
        return make_float2(__half2float(__ushort_as_half((unsigned short)(u & 0xffffu))),
                           __half2float(__ushort_as_half((unsigned short)(u >> 16))));
    }
    static __device__ __forceinline__ float ld(const void* p, long long i) {
        return __half2float(__ushort_as_half(ld_cs_b16(static_cast<const __half*>(p) + i)));
    }
    static __device__ __forceinline__ float2 ld2(const void* p, long long i) {
        const uint32_t u = ld_cs_b32(static_cast<const __half*>(p) + i);
        return make_float2(__half2float(__ushort_as_half((unsigned short)(u & 0xffffu))),
                           __half2float(__ushort_as_half((unsigned short)(u >> 16))));
    }
    static __device__ __forceinline__ void st(void* p, long long i, float v) {
        st_cs_b16(static_cast<__half*>(p) + i, __half_as_ushort(__float2half_rn(v)));
    }
    static __device__ __forceinline__ void st2(void* p, long long i, float2 v) {
        st_cs_b32(static_cast<__half*>(p) + i,
                  (uint32_t)__half_as_ushort(__float2half_rn(v.x)) |
                      ((uint32_t)__half_as_ushort(__float2half_rn(v.y)) << 16));
    }
};
template <>
struct Io<__nv_bfloat16> {
    using Raw2 = uint32_t;
    static __device__ __forceinline__ Raw2 ld2raw(const void* p, long long i) {
        return ld_cs_b32(static_cast<const __nv_bfloat16*>(p) + i);
    }
    static __device__ __forceinline__ float2 cvt2(Raw2 u) {
        return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    }
    static __device__ __forceinline__ float ld(const void* p, long long i) {
        return __uint_as_float((uint32_t)ld_cs_b16(static_cast<const __nv_bfloat16*>(p) + i) << 16);
    }
    static __device__ __forceinline__ float2 ld2(const void* p, long long i) {
        const uint32_t u = ld_cs_b32(static_cast<const __nv_bfloat16*>(p) + i);
        return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    }
    static __device__ __forceinline__ void st(void* p, long long i, float v) {
        st_cs_b16(static_cast<__nv_bfloat16*>(p) + i, __bfloat16_as_ushort(__float2bfloat16_rn(v)));
    }
    static __device__ __forceinline__ void st2(void* p, long long i, float2 v) {
        st_cs_b32(static_cast<__nv_bfloat16*>(p) + i,
                  (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v.x)) |
                      ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v.y)) << 16));
    }
};

// One forward step of aligned_forward (:11-14) given the step's history sum h (accumulated
// in push form by the caller, in the reference's term order).  Returns v_t.
template <bool TP2>
__device__ __forceinline__ float aligned_step(float x, float v, float a_t, float h, float tau,
                                              float inv_tau, float th, float& pred, bool& fire) {
    const float d = div_tau<TP2>(__fsub_rn(x, v), tau, inv_tau);
    pred = __fadd_rn(v, d);
    fire = pred >= th;
    const float spike = fire ? 1.0f : 0.0f;
    const float f = __fsub_rn(d, div_tau<TP2>(__fmul_rn(spike, th), tau, inv_tau));
    return __fsub_rn(__fmul_rn(a_t, f), h);
}

// Fold v_t into the history sums of all later steps: hs[u] += round(W[u,t] * v_t) (the
// reference's sequential h += w*hist order, no fused multiply-add).
template <int TB, bool FAST>
__device__ __forceinline__ void aligned_push(float (&hs)[TB], const float* sW, const float (&wr)[TB],
                                             int t, float v) {
#pragma unroll
    for (int u = t + 1; u < TB; ++u) hs[u] = __fadd_rn(hs[u], __fmul_rn(wgt<TB, FAST>(sW, wr, u, t), v));
}

template <int TB, bool TP2, bool FAST, typename E>
__device__ __forceinline__ void aln_fwd_body(const AlnArgs& a, const float* sW, const float* sA,
                                             long long n) {
    const int T = a.T;
    const long long N = a.N;
    float wr[TB];
#pragma unroll
    for (int d = 0; d < TB; ++d) wr[d] = (FAST && d > 0) ? sW[d * TB] : 0.0f;
    float xr[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t)
        if (t < T) xr[t] = Io<E>::ld(a.xio, t * N + n);
    float v = a.v0[n];
    float hs[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) hs[t] = 0.0f;
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        if (t < T) {
            float pred;
            bool fire;
            v = aligned_step<TP2>(xr[t], v, FAST ? sA[0] : sA[t], hs[t], a.tau, a.inv_tau, a.th,
                                  pred, fire);
            aligned_push<TB, FAST>(hs, sW, wr, t, v);
            Io<E>::st(a.sio, t * N + n, fire ? 1.0f : 0.0f);
        }
    }
}

template <int TB, bool TP2, typename E>
__global__ void __launch_bounds__(256) aln_fwd_reg(AlnArgs a) {
    __shared__ float sW[TB * TB];
    __shared__ float sA[TB];
    const int T = a.T;
    for (int e = threadIdx.x; e < TB * TB; e += blockDim.x) {
        const int t = e / TB, i = e % TB;
        sW[e] = (t < T && i < T) ? a.W[t * T + i] : 0.0f;
    }
    for (int e = threadIdx.x; e < TB; e += blockDim.x) sA[e] = e < T ? a.a[e] : 0.0f;
    const bool fast = block_toeplitz(a.W, a.a, T);
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    if (fast) aln_fwd_body<TB, TP2, true, E>(a, sW, sA, n);
    else aln_fwd_body<TB, TP2, false, E>(a, sW, sA, n);
}

// Forward, T <= TB <= 16, two neurons per thread (Toeplitz schedule; a general W runs the
// scalar body per neuron).  Every product is formed by pmz2 and every sum is packed
// (pack2.cuh).  The history sum h is accumulated negated, h' = h' + round(-w*v), so
// v = round(a*f) - h is an add.
template <int TB, bool TP2, typename E>
__global__ void __launch_bounds__(128, 5) aln_fwd_x2(AlnArgs a) {
    __shared__ float sW[TB * TB];
    __shared__ float sA[TB];
    const int T = a.T;
    // this thread's x rows and v0 are requested before the block stages W and checks it, so
    // their memory latency overlaps the staging and the block barrier
    const long long n = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
    // the rows as loaded (half-precision pairs stay packed until their step uses them, so the
    // loads are all in flight before any conversion waits on one)
    typename Io<E>::Raw2 xr[TB];
    float2 v = f2(0.0f);
    if (n < a.N) {
#pragma unroll
        for (int t = 0; t < TB; ++t)
            if (t < T) xr[t] = Io<E>::ld2raw(a.xio, t * a.N + n);
        v = *reinterpret_cast<const float2*>(a.v0 + n);
    }
    for (int e = threadIdx.x; e < TB * TB; e += blockDim.x) {
        const int t = e / TB, i = e % TB;
        sW[e] = (t < T && i < T) ? a.W[t * T + i] : 0.0f;
    }
    for (int e = threadIdx.x; e < TB; e += blockDim.x) sA[e] = e < T ? a.a[e] : 0.0f;
    const bool fast = block_toeplitz(a.W, a.a, T);
    if (n >= a.N) return;
    if (!fast) {
        aln_fwd_body<TB, TP2, false, E>(a, sW, sA, n);
        aln_fwd_body<TB, TP2, false, E>(a, sW, sA, n + 1);
        return;
    }
    const long long N = a.N;
    float2 nw[TB];
#pragma unroll
    for (int d = 0; d < TB; ++d) nw[d] = f2(d > 0 ? -sW[d * TB] : 0.0f);
    const float2 a2 = f2(sA[0]);
    const float2 inv2 = f2(a.inv_tau);
    const float2 mth = f2(-a.th);
    float2 hn[TB];                                                   // -h, push form
    const float2 nz2 = f2(a.negz);
#pragma unroll
    for (int t = 0; t < TB; ++t) hn[t] = f2(-0.0f);
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        if (t < T) {
            // every product is a pmz2 product, so the sums that consume them may be packed
            const float2 xm = psub2(Io<E>::cvt2(xr[t]), v);
            const float2 d = TP2 ? pmz2(xm, inv2, nz2)
                                 : make_float2(__fdiv_rn(xm.x, a.tau), __fdiv_rn(xm.y, a.tau));
            const float2 pred = padd2(v, d);
            const float2 s = fire2(pred, a.th);
            const float2 sm = pmz2(s, mth, nz2);
            const float2 smt = TP2 ? pmz2(sm, inv2, nz2)
                                   : make_float2(__fdiv_rn(sm.x, a.tau), __fdiv_rn(sm.y, a.tau));
            const float2 f = padd2(d, smt);                          // d - s*th/tau
            v = padd2(pmz2(a2, f, nz2), hn[t]);                      // a*f - h
#pragma unroll
            for (int u = t + 1; u < TB; ++u) hn[u] = padd2(hn[u], pmz2(nw[u - t], v, nz2));
            Io<E>::st2(a.sio, t * N + n, s);
        }
    }
}

// Backward tile.  Stage X holds x_t, then v_t + h_t, then e_t = r_t (v_t + h_t) / a_t;
// stage G holds grad_spike_t, then q_t (surrogate term), then the adjoint r_t.
template <int TB, bool TP2, bool FAST>
__device__ __forceinline__ void aln_bwd_tile(const AlnArgs& a, const float* sW, const float* sA,
                                             const float (&wr)[TB], const float (&rw)[TB],
                                             float zc, float one_m, float* X, float* G, float* V,
                                             const float* V0, long long n0, int tid) {
    const int T = a.T;
    const long long N = a.N;
    const long long n = n0 + tid;
    const bool live = n < N;
    float v = live ? V0[tid] : 0.0f;
    float hs[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) hs[t] = 0.0f;
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        if (t < T) {
            float pred;
            bool fire;
            const float h = hs[t];
            v = aligned_step<TP2>(X[t * kTile + tid], v, FAST ? sA[0] : sA[t], h, a.tau, a.inv_tau,
                                  a.th, pred, fire);
            aligned_push<TB, FAST>(hs, sW, wr, t, v);
            const float z = __fmul_rn(zc, __fsub_rn(pred, a.th));
            const float den = __fmul_rn(2.0f, __fadd_rn(1.0f, __fmul_rn(z, z)));
            G[t * kTile + tid] = __fdiv_rn(__fmul_rn(G[t * kTile + tid], a.sg), den);   // q_t
            X[t * kTile + tid] = __fadd_rn(v, h);                                       // v_t + h_t
        } else {
            v = 0.0f;
        }
        if (!live) v = 0.0f;
        V[t * kTile + tid] = v;
    }
    float A[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) A[t] = 0.0f;
#pragma unroll
    for (int t = TB - 1; t >= 0; --t) {
        float r = 0.0f, e = 0.0f;
        if (t < T) {
            const float a_t = FAST ? sA[0] : sA[t];
            const float q = G[t * kTile + tid];
            r = A[t];
            const float ra = __fmul_rn(r, a_t);
            if (live) st_stream(a.gx + t * N + n, div_tau<TP2>(__fadd_rn(q, ra), a.tau, a.inv_tau));
            const float prev = __fsub_rn(__fmul_rn(q, one_m), div_tau<TP2>(ra, a.tau, a.inv_tau));
            if (t) A[t - 1] = __fadd_rn(A[t - 1], prev);
            else if (live) a.gv0[n] = prev;
#pragma unroll
            for (int j = 0; j < t; ++j) {
                const float rwj = FAST ? rw[t - j] : __fmul_rn(a.rho, sW[t * TB + j]);
                A[j] = __fsub_rn(A[j], __fmul_rn(rwj, r));
            }
            e = __fdiv_rn(__fmul_rn(r, X[t * kTile + tid]), a_t);
        }
        G[t * kTile + tid] = live ? r : 0.0f;
        X[t * kTile + tid] = live ? e : 0.0f;
    }
}

template <int TB>
struct AlnBwdSmem {
    // per stage: X [TB][256], G [TB][256], v0 row [256]; then V [TB][256]
    static constexpr size_t kStageFloats = size_t(2) * TB * kTile + kTile;
    static constexpr size_t kBytes = sizeof(float) * (2 * kStageFloats + size_t(TB) * kTile);
    static_assert(size_t(kTile) * 20 * sizeof(double) <= kBytes, "reduction scratch must fit");
};

template <int TB, bool TP2, bool BULK>
__global__ void __launch_bounds__(256) aln_bwd(AlnArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    constexpr size_t kSF = AlnBwdSmem<TB>::kStageFloats;
    float* base = reinterpret_cast<float*>(smem_raw);
    float* V = base + 2 * kSF;
    __shared__ float sW[TB * TB];
    __shared__ float sA[TB];
    __shared__ __align__(8) uint64_t bars[2];
    const int T = a.T;
    const long long N = a.N;
    const int tid = threadIdx.x;
    for (int e = tid; e < TB * TB; e += blockDim.x) {
        const int t = e / TB, i = e % TB;
        sW[e] = (t < T && i < T) ? a.W[t * T + i] : 0.0f;
    }
    for (int e = tid; e < TB; e += blockDim.x) sA[e] = e < T ? a.a[e] : 1.0f;
    BulkPipe<2> pipe;
    pipe.bar = bars;
    pipe.T = T;
    pipe.N = N;
    pipe.src[0] = a.x;
    pipe.src[1] = a.g;
    pipe.row_src = a.v0;
    for (int s = 0; s < 2; ++s) {
        pipe.stage[s][0] = base + s * kSF;
        pipe.stage[s][1] = base + s * kSF + TB * kTile;
        pipe.row_stage[s] = base + s * kSF + 2 * TB * kTile;
    }
    if (BULK && tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    const bool fast = block_toeplitz(a.W, a.a, T);
    float wr[TB], rw[TB];
#pragma unroll
    for (int d = 0; d < TB; ++d) {
        wr[d] = (fast && d > 0) ? sW[d * TB] : 0.0f;
        rw[d] = __fmul_rn(a.rho, wr[d]);                  // (rho * w) as the reference rounds it
    }
    const float zc = __fmul_rn(kAlignedPiHalf, a.sg);
    const float one_m = __fsub_rn(1.0f, __fdiv_rn(1.0f, a.tau));      // 1 - 1/tau
    TileProduct<TB, false> prod;
    prod.init(tid);
    const long long ntiles = (N + kTile - 1) / kTile;
    const long long first = blockIdx.x, stride = gridDim.x;
    if (BULK && tid == 0) {
        if (first < ntiles) pipe.issue(0, first);
        if (first + stride < ntiles) pipe.issue(1, first + stride);
    }
    bool failed = false;
    int j = 0;
    for (long long tile = first; tile < ntiles; tile += stride, ++j) {
        const int s = BULK ? (j & 1) : 0;
        float* X = base + s * kSF;
        float* G = X + TB * kTile;
        float* V0 = G + TB * kTile;
        if constexpr (BULK) {
            const bool ok = mbar_wait_bounded(&bars[s], (uint32_t)((j >> 1) & 1));
            if (__syncthreads_or(!ok)) { failed = true; break; }
        } else {
            const long long n = tile * kTile + tid;
            for (int t = 0; t < T; ++t) {
                X[t * kTile + tid] = n < N ? ld_stream(a.x + t * N + n) : 0.0f;
                G[t * kTile + tid] = n < N ? ld_stream(a.g + t * N + n) : 0.0f;
            }
            V0[tid] = n < N ? a.v0[n] : 0.0f;
        }
        if (fast) aln_bwd_tile<TB, TP2, true>(a, sW, sA, wr, rw, zc, one_m, X, G, V, V0, tile * kTile, tid);
        else aln_bwd_tile<TB, TP2, false>(a, sW, sA, wr, rw, zc, one_m, X, G, V, V0, tile * kTile, tid);
        __syncthreads();
        prod.accumulate(G, V, X);
        __syncthreads();
        if (BULK && tid == 0 && tile + 2 * stride < ntiles) pipe.issue(s, tile + 2 * stride);
    }
    if (failed) {
        if (tid == 0) {
            atomicOr(a.err, 1u);
            mbar_wait_bounded(&bars[j & 1], (uint32_t)((j >> 1) & 1));
            if (first + (long long)(j + 1) * stride < ntiles)
                mbar_wait_bounded(&bars[(j + 1) & 1], (uint32_t)(((j + 1) >> 1) & 1));
        }
        return;
    }
    prod.finish(reinterpret_cast<double*>(smem_raw), a.part + (size_t)blockIdx.x * ProdCfg<TB>::NOUT, tid);
}

// ------------------------------------------------------------------------------------
// backward, T in {8, 16} exactly: the warp-tiled persistent design of glm_bwd_w
// (warp_tile.cuh) with the aligned arithmetic: every product and sum separately rounded
// (packed fp32x2 per neuron pair), IEEE divisions for the surrogate term and for e_t.
// Stage X holds x_t, then v_t + h_t; G holds grad_spike_t, then grad_x_t; V0 holds v0,
// then grad_v0.  GP receives the adjoint r_t, V the membrane v_t.
// ------------------------------------------------------------------------------------
// Reverse sweep of one aligned tile (SLOW: IEEE division for the surrogate term q_t).
template <int T, bool TP2, bool FAST, bool SLOW>
__device__ __forceinline__ void aln_bwd_warp_reverse(const AlnArgs& a, const float* sW,
                                                     const float* sA, const float* sInvA,
                                                     const float2 (&rw)[T], const float* X,
                                                     float* G, float* V0, float* GP,
                                                     const float2 (&den)[T], float2 (&gsa)[T]) {
    constexpr int RS = WarpBwdCfg<T>::RS;
    constexpr int TN = WarpBwdCfg<T>::TN;
    const int c2 = 2 * (threadIdx.x & 31);
    const float2 inv2 = f2(a.inv_tau), sg2 = f2(a.sg);
    const float2 one_m2 = f2(__fsub_rn(1.0f, __fdiv_rn(1.0f, a.tau)));
    const float2 nz2 = f2(a.negz);
    float2 A[T];
#pragma unroll
    for (int t = 0; t < T; ++t) A[t] = f2(0.0f);
#pragma unroll
    for (int t = T - 1; t >= 0; --t) {
        const float2 a2 = f2(FAST ? sA[0] : sA[t]);
        const float2 gnum = pmul2(*reinterpret_cast<const float2*>(G + t * TN + c2), sg2);
        const float2 q = quot2<SLOW>(gnum, den[t]);                     // (g*sg)/den, exact
        const float2 r = A[t];
        const float2 ra = pmz2(r, a2, nz2);
        const float2 qa = padd2(q, ra);
        const float2 gx = TP2 ? pmul2(qa, inv2)
                              : make_float2(__fdiv_rn(qa.x, a.tau), __fdiv_rn(qa.y, a.tau));
        *reinterpret_cast<float2*>(G + t * TN + c2) = gx;
        const float2 rat = TP2 ? pmz2(ra, inv2, nz2)
                               : make_float2(__fdiv_rn(ra.x, a.tau), __fdiv_rn(ra.y, a.tau));
        const float2 prev = psub2(pmz2(q, one_m2, nz2), rat);
        if (t) A[t - 1] = padd2(A[t - 1], prev);
        else *reinterpret_cast<float2*>(V0 + c2) = prev;
#pragma unroll
        for (int j = 0; j < t; ++j) {
            const float2 rwj = FAST ? rw[t - j] : f2(__fmul_rn(a.rho, sW[t * T + j]));
            A[j] = psub2(A[j], pmz2(rwj, r, nz2));
        }
        *reinterpret_cast<float2*>(GP + t * RS + c2) = r;
        // e_t = r_t (v_t + h_t) / a_t feeds only the grad_a reduction: product with the
        // correctly rounded reciprocal of a_t (within an ulp of the quotient per term)
        const float2 rx = pmz2(r, *reinterpret_cast<const float2*>(X + t * TN + c2), nz2);
        gsa[t] = padd2(gsa[t], pmz2(rx, f2(FAST ? sInvA[0] : sInvA[t]), nz2));
    }
}

// One aligned tile: forward recompute (v -> V rows, v + h -> X, surrogate denominators in
// registers), then the reverse sweep with the fast or the IEEE surrogate quotient.
template <int T, bool TP2, bool FAST>
__device__ __forceinline__ void aln_bwd_warp_tile(const AlnArgs& a, const float* sW, const float* sA,
                                                  const float* sInvA, const float2 (&wr)[T],
                                                  const float2 (&rw)[T], float* X, float* G,
                                                  float* V0, float* GP, float* Vs,
                                                  float2 (&gsa)[T]) {
    constexpr int RS = WarpBwdCfg<T>::RS;
    constexpr int TN = WarpBwdCfg<T>::TN;
    const int c2 = 2 * (threadIdx.x & 31);
    const float th = a.th;
    const float2 th2 = f2(th), inv2 = f2(a.inv_tau), zc2 = f2(__fmul_rn(kAlignedPiHalf, a.sg));
    const float sg = a.sg;
    const float2 thr_tau = f2(div_tau<TP2>(th, a.tau, a.inv_tau));   // spike*th/tau for spike = 1
    float2 v = *reinterpret_cast<const float2*>(V0 + c2);
    float2 hs[T], den[T];
    const float2 nz2 = f2(a.negz);
    bool bad = false;
#pragma unroll
    for (int t = 0; t < T; ++t) hs[t] = f2(0.0f);
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const float2 a2 = f2(FAST ? sA[0] : sA[t]);
        const float2 xs = *reinterpret_cast<const float2*>(X + t * TN + c2);
        const float2 xm = psub2(xs, v);
        const float2 d = TP2 ? pmz2(xm, inv2, nz2)
                             : make_float2(__fdiv_rn(xm.x, a.tau), __fdiv_rn(xm.y, a.tau));
        const float2 pred = padd2(v, d);
        // f = d - spike*th/tau; spike*th/tau is exactly thr_tau or 0 (and d - 0 == d)
        const float2 dm = psub2(d, thr_tau);
        const float2 f = make_float2(pred.x >= th ? dm.x : d.x, pred.y >= th ? dm.y : d.y);
        const float2 h = hs[t];
        v = psub2(pmz2(a2, f, nz2), h);
#pragma unroll
        for (int u = t + 1; u < T; ++u) {
            const float2 w = FAST ? wr[u - t] : f2(sW[u * T + t]);
            hs[u] = padd2(hs[u], pmz2(w, v, nz2));
        }
        const float2 z = pmz2(zc2, psub2(pred, th2), nz2);
        const float2 dn = pmul2(f2(2.0f), padd2(f2(1.0f), pmz2(z, z, nz2)));
        den[t] = dn;
        const float2 g = *reinterpret_cast<const float2*>(G + t * TN + c2);
        bad |= !(dn.x <= 0x1p64f) || !(dn.y <= 0x1p64f) ||
               !quot_num_ok(__fmul_rn(g.x, sg)) || !quot_num_ok(__fmul_rn(g.y, sg));
        *reinterpret_cast<float2*>(Vs + t * RS + c2) = v;
        *reinterpret_cast<float2*>(X + t * TN + c2) = padd2(v, h);     // v_t + h_t
    }
    if (__any_sync(0xffffffffu, bad))
        aln_bwd_warp_reverse<T, TP2, FAST, true>(a, sW, sA, sInvA, rw, X, G, V0, GP, den, gsa);
    else
        aln_bwd_warp_reverse<T, TP2, FAST, false>(a, sW, sA, sInvA, rw, X, G, V0, GP, den, gsa);
}

template <int T, bool TP2>
__global__ void __launch_bounds__(256, WarpBwdCfg<T>::kMinBlocks)
    aln_bwd_w(AlnArgs a, const __grid_constant__ TileMaps m) {
    using C = WarpBwdCfg<T>;
    constexpr int RS = C::RS;
    constexpr int TN = C::TN;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ float sW[T * T];
    __shared__ float sA[T];
    __shared__ float sInvA[T];
    __shared__ __align__(8) uint64_t bars[C::kWarps][2];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long N = a.N;
    for (int e = tid; e < T * T; e += blockDim.x) sW[e] = a.W[e];
    for (int e = tid; e < T; e += blockDim.x) {
        sA[e] = a.a[e];
        sInvA[e] = __frcp_rn(a.a[e]);
    }
    if (lane == 0) {
        mbar_init(&bars[warp][0], 1);
        mbar_init(&bars[warp][1], 1);
        fence_mbar_init();
    }
    const bool fast = block_toeplitz(a.W, a.a, T);     // block barrier
    unsigned char* aligned_smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    float* wbase = reinterpret_cast<float*>(aligned_smem) + warp * C::PER_WARP;
    float* GP = wbase + 2 * C::STAGE;
    float* Vs = GP + T * RS;
    float2 wr[T], rw[T];
#pragma unroll
    for (int d = 0; d < T; ++d) {
        const float w = (fast && d > 0) ? sW[d * T] : 0.0f;
        wr[d] = f2(w);
        rw[d] = f2(__fmul_rn(a.rho, w));                // (rho * w) as the reference rounds it
    }
    float acc[C::NACC];
    float2 gsa[T];
#pragma unroll
    for (int e = 0; e < C::NACC; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int t = 0; t < T; ++t) gsa[t] = f2(0.0f);
    const long long ntiles = (N + TN - 1) / TN;
    const long long first = (long long)blockIdx.x * C::kWarps + warp;
    const long long stride = (long long)gridDim.x * C::kWarps;
    if (lane == 0 && first < ntiles) warp_load<T>(wbase, &bars[warp][0], m, first * TN);
    bool failed = false;
    int j = 0;
    for (long long tile = first; tile < ntiles; tile += stride, ++j) {
        const int s = j & 1;
        float* X = wbase + s * C::STAGE;
        float* G = X + T * TN;
        float* V0 = X + 2 * T * TN;
        const bool ok = mbar_wait_bounded(&bars[warp][s], (uint32_t)((j >> 1) & 1));
        if (__any_sync(0xffffffffu, !ok)) { failed = true; break; }
        if (lane == 0 && tile + stride < ntiles)
            warp_load<T>(wbase + (s ^ 1) * C::STAGE, &bars[warp][s ^ 1], m, (tile + stride) * TN);
        // lanes past N compute on zero-filled inputs (finite); the stores clip them
        if (fast) aln_bwd_warp_tile<T, TP2, true>(a, sW, sA, sInvA, wr, rw, X, G, V0, GP, Vs, gsa);
        else aln_bwd_warp_tile<T, TP2, false>(a, sW, sA, sInvA, wr, rw, X, G, V0, GP, Vs, gsa);
        __syncwarp();
        warp_product<T>(GP, Vs, lane, acc);
        warp_store<T>(X, m, tile * TN, lane);
    }
    if (lane == 0) {
        if (failed) {
            atomicOr(a.err, 1u);
            mbar_wait_bounded(&bars[warp][j & 1], (uint32_t)((j >> 1) & 1));
        }
        bulk_wait_all();
    }
    warp_tiles_finish<T>(acc, gsa, aligned_smem, a.part, tid);
}

namespace {

int tb_of(int T) { return T <= 8 ? 8 : (T <= 16 ? 16 : 32); }

template <class K>
int aln_resident(K k, size_t smem) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, kTile, smem);
    if (per < 1) per = 1;
    return (sms < 1 ? 1 : sms) * per;
}

template <int TB>
int aln_grid_t(long long N) {
    static std::atomic<int> cached[64];
    int dev = 0;
    cudaGetDevice(&dev);
    int res = (dev >= 0 && dev < 64) ? cached[dev].load(std::memory_order_relaxed) : 0;
    if (res <= 0) {
        if constexpr (TB == 8 || TB == 16)
            res = aln_resident(aln_bwd_w<TB, false>, WarpBwdCfg<TB>::kBytes);
        else
            res = aln_resident(aln_bwd<TB, false, true>, AlnBwdSmem<TB>::kBytes);
        if (dev >= 0 && dev < 64) cached[dev].store(res, std::memory_order_relaxed);
    }
    const long long ntiles = (N + kTile - 1) / kTile;
    long long g = res;
    if (g > ntiles) g = ntiles;
    return g < 1 ? 1 : (int)g;
}

// ------------------------------------------------------------------------------------
// 32 < T <= 64: one thread per neuron, history in shared memory ([T][64] floats per block;
// the backward's adjoint sums another [T][64]).  Pull-form history in the reference's
// order (h += w*hist, separately rounded).  The backward writes v_t, the adjoint r_t (ga)
// and e_t = r_t*(v_t + h_t)/a_t to [T, N] scratch for param_long.
// ------------------------------------------------------------------------------------
constexpr int kAlnLongThreads = 64;

template <bool TP2, typename E>
__global__ void __launch_bounds__(kAlnLongThreads) aln_fwd_long(AlnArgs a) {
    extern __shared__ float sh[];
    const long long n = (long long)blockIdx.x * kAlnLongThreads + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int T = a.T;
    float* vh = sh + threadIdx.x;
    float v = a.v0[n];
    for (int t = 0; t < T; ++t) {
        const float* wrow = a.W + (size_t)t * T;
        float h = 0.0f;
        for (int j = 0; j < t; ++j) h = __fadd_rn(h, __fmul_rn(__ldg(wrow + j), vh[j * kAlnLongThreads]));
        float pred;
        bool fire;
        v = aligned_step<TP2>(Io<E>::ld(a.xio, t * N + n), v, __ldg(a.a + t), h, a.tau, a.inv_tau,
                              a.th, pred, fire);
        vh[t * kAlnLongThreads] = v;
        Io<E>::st(a.sio, t * N + n, fire ? 1.0f : 0.0f);
    }
}

template <bool TP2>
__global__ void __launch_bounds__(kAlnLongThreads) aln_bwd_long(AlnArgs a, float* Vs, float* Es,
                                                                float* Rs) {
    extern __shared__ float sh[];
    const long long n = (long long)blockIdx.x * kAlnLongThreads + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int T = a.T;
    float* vh = sh + threadIdx.x;
    float* A = sh + (size_t)T * kAlnLongThreads + threadIdx.x;
    const float zc = __fmul_rn(kAlignedPiHalf, a.sg);
    const float one_m = __fsub_rn(1.0f, __fdiv_rn(1.0f, a.tau));
    float v = a.v0[n];
    for (int t = 0; t < T; ++t) {
        const float* wrow = a.W + (size_t)t * T;
        float h = 0.0f;
        for (int j = 0; j < t; ++j) h = __fadd_rn(h, __fmul_rn(__ldg(wrow + j), vh[j * kAlnLongThreads]));
        float pred;
        bool fire;
        v = aligned_step<TP2>(ld_stream(a.x + t * N + n), v, __ldg(a.a + t), h, a.tau, a.inv_tau,
                              a.th, pred, fire);
        vh[t * kAlnLongThreads] = v;
        const float z = __fmul_rn(zc, __fsub_rn(pred, a.th));
        const float den = __fmul_rn(2.0f, __fadd_rn(1.0f, __fmul_rn(z, z)));
        Rs[t * N + n] = __fdiv_rn(__fmul_rn(ld_stream(a.g + t * N + n), a.sg), den);   // q_t
        Es[t * N + n] = __fadd_rn(v, h);                                               // v_t + h_t
        Vs[t * N + n] = v;
        A[t * kAlnLongThreads] = 0.0f;
    }
    for (int t = T - 1; t >= 0; --t) {
        const float a_t = __ldg(a.a + t);
        const float q = Rs[t * N + n];
        const float r = A[t * kAlnLongThreads];
        const float ra = __fmul_rn(r, a_t);
        st_stream(a.gx + t * N + n, div_tau<TP2>(__fadd_rn(q, ra), a.tau, a.inv_tau));
        const float prev = __fsub_rn(__fmul_rn(q, one_m), div_tau<TP2>(ra, a.tau, a.inv_tau));
        if (t) A[(t - 1) * kAlnLongThreads] = __fadd_rn(A[(t - 1) * kAlnLongThreads], prev);
        else a.gv0[n] = prev;
        const float* wrow = a.W + (size_t)t * T;
        for (int j = 0; j < t; ++j)
            A[j * kAlnLongThreads] = __fsub_rn(A[j * kAlnLongThreads],
                                               __fmul_rn(__fmul_rn(a.rho, __ldg(wrow + j)), r));
        Rs[t * N + n] = r;
        Es[t * N + n] = __fdiv_rn(__fmul_rn(r, Es[t * N + n]), a_t);
    }
}

template <int TB, bool TP2, bool BULK>
cudaError_t aln_bwd_launch_t(const AlnArgs& a, int grid, cudaStream_t st) {
    const size_t smem = AlnBwdSmem<TB>::kBytes;
    auto k = aln_bwd<TB, TP2, BULK>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, kTile, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace

int aligned_bwd_blocks(int T, long long N, bool) {
    const int TB = tb_of(T);
    if (TB == 8) return aln_grid_t<8>(N);
    if (TB == 16) return aln_grid_t<16>(N);
    return aln_grid_t<32>(N);
}

int aligned_part_stride(int T) {
    if (T > 32) return T + T * T;
    const int TB = tb_of(T);
    return TB + TB * TB;
}

cudaError_t aligned_backward_long_launch(const float* g, const float* x, const float* v0,
                                         const float* a_, const float* W, float* gx, float* gv0,
                                         float* ga, float* gW, int T, long long N, float tau,
                                         float th, float sg, float rho, bool tau_pow2,
                                         double* part, int slices, float* scratch,
                                         unsigned int* err, cudaStream_t st) {
    AlnArgs a{};
    a.negz = -0.0f;
    a.x = x; a.v0 = v0; a.a = a_; a.W = W; a.g = g; a.gx = gx; a.gv0 = gv0;
    a.T = T; a.N = N; a.tau = tau; a.inv_tau = 1.0f / tau; a.th = th; a.sg = sg; a.rho = rho;
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return e;
    float* Vs = scratch;
    float* Es = scratch + (size_t)T * N;
    float* Rs = scratch + 2 * (size_t)T * N;
    if (N > 0) {
        const size_t smem = sizeof(float) * 2 * (size_t)T * kAlnLongThreads;
        const unsigned grid = (unsigned)((N + kAlnLongThreads - 1) / kAlnLongThreads);
        auto k = tau_pow2 ? aln_bwd_long<true> : aln_bwd_long<false>;
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<grid, kAlnLongThreads, smem, st>>>(a, Vs, Es, Rs);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (!ga && !gW) return cudaSuccess;
    e = param_long_launch(Rs, Vs, Es, T, N, false, part, slices, st);
    if (e != cudaSuccess) return e;
    return launch_param_finalize(part, slices, T, T, ga, gW, 1, err, st);
}

namespace {

template <typename E>
cudaError_t aligned_forward_t(AlnArgs& a, const void* x, const void* spike, int T, long long N,
                              bool tau_pow2, cudaStream_t st) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(a.v0) |
                         reinterpret_cast<uintptr_t>(spike);
    if (T <= 16 && (N % 2) == 0 && (al & (2 * sizeof(E) - 1)) == 0 &&
        (reinterpret_cast<uintptr_t>(a.v0) & 7u) == 0) {
        const unsigned g2 = (unsigned)((N / 2 + 127) / 128);        // 128-thread blocks
        if (T <= 8) {
            if (tau_pow2) aln_fwd_x2<8, true, E><<<g2, 128, 0, st>>>(a);
            else aln_fwd_x2<8, false, E><<<g2, 128, 0, st>>>(a);
        } else {
            if (tau_pow2) aln_fwd_x2<16, true, E><<<g2, 128, 0, st>>>(a);
            else aln_fwd_x2<16, false, E><<<g2, 128, 0, st>>>(a);
        }
        return cudaGetLastError();
    }
    if (T > 32) {
        const unsigned gl = (unsigned)((N + kAlnLongThreads - 1) / kAlnLongThreads);
        const size_t smem = sizeof(float) * (size_t)T * kAlnLongThreads;
        auto k = tau_pow2 ? aln_fwd_long<true, E> : aln_fwd_long<false, E>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<gl, kAlnLongThreads, smem, st>>>(a);
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned)((N + 255) / 256);
    const int TB = tb_of(T);
#define DFSNN_AF(TBV)                                                       \
    if (TB == TBV) {                                                        \
        if (tau_pow2) aln_fwd_reg<TBV, true, E><<<grid, 256, 0, st>>>(a);   \
        else aln_fwd_reg<TBV, false, E><<<grid, 256, 0, st>>>(a);           \
    }
    DFSNN_AF(8) DFSNN_AF(16) DFSNN_AF(32)
#undef DFSNN_AF
    return cudaGetLastError();
}

}  // namespace

cudaError_t aligned_forward_launch_io(const void* x, int dtype, const float* v0, const float* a_,
                                      const float* W, void* spike, int T, long long N, float tau,
                                      float th, bool tau_pow2, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    AlnArgs a{};
    a.negz = -0.0f;
    a.v0 = v0; a.a = a_; a.W = W; a.xio = x; a.sio = spike; a.T = T; a.N = N; a.tau = tau;
    a.inv_tau = 1.0f / tau; a.th = th;
    if (dtype == kIoF16) return aligned_forward_t<__half>(a, x, spike, T, N, tau_pow2, st);
    if (dtype == kIoBF16) return aligned_forward_t<__nv_bfloat16>(a, x, spike, T, N, tau_pow2, st);
    return aligned_forward_t<float>(a, x, spike, T, N, tau_pow2, st);
}

cudaError_t aligned_forward_launch(const float* x, const float* v0, const float* a_,
                                   const float* W, float* spike, int T, long long N, float tau,
                                   float th, bool tau_pow2, cudaStream_t st) {
    return aligned_forward_launch_io(x, kIoF32, v0, a_, W, spike, T, N, tau, th, tau_pow2, st);
}

cudaError_t aligned_backward_launch(const float* g, const float* x, const float* v0,
                                    const float* a_, const float* W, float* gx, float* gv0,
                                    float* ga, float* gW, int T, long long N, float tau, float th,
                                    float sg, float rho, bool tau_pow2, double* part,
                                    unsigned int* err, int nblocks, cudaStream_t st) {
    AlnArgs a{};
    a.negz = -0.0f;
    a.x = x; a.v0 = v0; a.a = a_; a.W = W; a.g = g; a.gx = gx; a.gv0 = gv0; a.part = part;
    a.err = err; a.T = T; a.N = N; a.tau = tau; a.inv_tau = 1.0f / tau; a.th = th; a.sg = sg;
    a.rho = rho;
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return e;
    const int TB = tb_of(T);
    TileMaps maps;
    if ((T == 8 || T == 16) && encode_tile_maps(&maps, x, g, v0, gx, gv0, T, N)) {
        auto k = T == 8 ? (tau_pow2 ? aln_bwd_w<8, true> : aln_bwd_w<8, false>)
                        : (tau_pow2 ? aln_bwd_w<16, true> : aln_bwd_w<16, false>);
        const size_t smem = T == 8 ? WarpBwdCfg<8>::kBytes : WarpBwdCfg<16>::kBytes;
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<nblocks, 256, smem, st>>>(a, maps);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        if (ga || gW) e = launch_param_finalize(part, nblocks, TB, T, ga, gW, 1, err, st);
        return e;
    }
    const bool bulk = bulk_eligible(x, g, v0, N);
#define DFSNN_AB(TBV)                                                                          \
    if (TB == TBV) {                                                                           \
        if (bulk) e = tau_pow2 ? aln_bwd_launch_t<TBV, true, true>(a, nblocks, st)             \
                               : aln_bwd_launch_t<TBV, false, true>(a, nblocks, st);           \
        else e = tau_pow2 ? aln_bwd_launch_t<TBV, true, false>(a, nblocks, st)                 \
                          : aln_bwd_launch_t<TBV, false, false>(a, nblocks, st);               \
    }
    DFSNN_AB(8) DFSNN_AB(16) DFSNN_AB(32)
#undef DFSNN_AB
    if (e != cudaSuccess) return e;
    if (ga || gW) e = launch_param_finalize(part, nblocks, TB, T, ga, gW, 1, err, st);
    return e;
}

}  // namespace dfsnn
