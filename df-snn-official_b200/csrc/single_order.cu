// single_order.cu -- single-order fractional LIF kernels for sm_100a:
//   GL        lif_fde_gl_forward/backward_kernel         (fde_cupy_kernels_all.py:24-163)
//   GL1       lif_fde_gl1_forward/backward_kernel        (:170-320)
//   TRAP      lif_fde_trap_forward/backward_kernel       (:327-472)
//   PREDICTOR lif_fde_predictor_forward/backward_kernel  (:479-637)
// The forward reproduces the reference's Kahan-compensated history sum term by term.
// The reference backward recomputes the whole forward (O(T^2) per neuron, 2 KB of local
// arrays per thread) only to recover v_t and spike_t; here the forward also emits a spike
// bitmask (one bit per step) and the backward streams the saved membrane v[T,N] and the
// bits: O(T) per neuron, no recompute, bit-identical surrogate inputs (v_t + s_t*theta).
#include "kernels.h"
#include "lif_common.cuh"
#include "pack2.cuh"

namespace dfsnn {

struct SingleArgs {
    const float* x;      // [T, N]
    const float* v0;     // [N]
    const float* w;      // [T+1] reversed weights (c_rev / trap_w / pred_w)
    float* spike;        // [T, N]
    float* v;            // [T, N]
    uint32_t* bits;      // [ceil(T/32), N] spike bitmask
    const float* gS;     // [T, N]
    const float* gV;     // [T, N]
    const float* vs;     // [T, N] saved membrane (backward input)
    const uint32_t* bits_in;
    float* gx;           // [T, N]
    float* gv0;          // [N]
    int T;
    long long N;
    float tau, inv_tau, beta, th, sg, h_beta, gamma1;
};

// Per-step update of the pre-reset potential given drift dv and history sum hist.
template <int SCHEME>
__device__ __forceinline__ float single_update(float v, float dv, float hist, float trap_factor,
                                               float pred_scale, float w_cur, float h_beta) {
    if constexpr (SCHEME == kGL) return __fsub_rn(dv, hist);                         // :66
    else if constexpr (SCHEME == kGL1) return __fmaf_rn(h_beta, dv, -hist);          // :213
    else if constexpr (SCHEME == kTRAP1) return __fsub_rn(__fmaf_rn(h_beta, dv, v), hist);  // :2059
    else if constexpr (SCHEME == kPRED1)
        return __fmaf_rn(h_beta, __fmaf_rn(w_cur, dv, hist), v);                     // :2326
    else if constexpr (SCHEME == kTRAP) return __fadd_rn(v, __fmaf_rn(trap_factor, dv, -hist));  // :372
    else return __fmaf_rn(pred_scale, __fmaf_rn(w_cur, dv, hist), v);                // :528
}

// ------------------------------------------------------------------------------------
// forward, T <= TB <= 32: history in registers
// ------------------------------------------------------------------------------------
template <int SCHEME, int TB, bool TP2>
__global__ void __launch_bounds__(256) single_fwd_reg(SingleArgs a) {
    __shared__ float sw[TB + 1];
    const int T = a.T;
    for (int e = threadIdx.x; e <= T; e += blockDim.x) sw[e] = a.w[e];
    __syncthreads();
    const long long N = a.N;
    const float trap_factor = __fmaf_rn(1.5f, a.beta, 0.5f);     // :346
    const float pred_scale = __fdiv_rn(a.h_beta, a.gamma1);       // :528
    // history weight of lag L = k - i is w[T - L] (k >= 1, i < k); keep the table in
    // registers indexed by the (compile-time) lag so the Kahan loop reads no memory
    float wr[TB + 1];
#pragma unroll
    for (int L = 0; L <= TB; ++L) wr[L] = (L <= T) ? sw[T - L] : 0.0f;
    const float w_cur = wr[0];
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float xr[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t)
        if (t < T) xr[t] = ld_stream(a.x + t * N + n);
    float v = a.v0[n];
    float hv[TB];
    uint32_t bits = 0;
#pragma unroll
    for (int k = 0; k < TB; ++k) {
        if (k < T) {
            const float dv = div_tau<TP2>(__fsub_rn(xr[k], v), a.tau, a.inv_tau);
            float sum = 0.0f, c = 0.0f;                            // Kahan, :52-63
#pragma unroll
            for (int i = 0; i < k; ++i) {
                const float y = __fmaf_rn(wr[k - i], hv[i], -c);
                const float t = __fadd_rn(sum, y);
                c = __fsub_rn(__fsub_rn(t, sum), y);
                sum = t;
            }
            const float p = single_update<SCHEME>(v, dv, sum, trap_factor, pred_scale, w_cur, a.h_beta);
            const bool fire = p >= a.th;
            const float s = fire ? 1.0f : 0.0f;
            v = __fsub_rn(p, s * a.th);
            hv[k] = (SCHEME == kPRED || SCHEME == kPRED1) ? div_tau<TP2>(-v, a.tau, a.inv_tau) : v;
            bits |= (fire ? 1u : 0u) << k;
            st_stream(a.spike + k * N + n, s);
            st_stream(a.v + k * N + n, v);
        }
    }
    a.bits[n] = bits;
}

// ------------------------------------------------------------------------------------
// forward, T in {8, 16} exactly, two neurons per thread (n, n+1): both Kahan chains advance
// with packed fp32x2 instructions (inline PTX, so no compiler pass can rewrite the
// compensation).  The history is summed negated (weights -w) for the schemes that use
// -hist, which makes every update a single packed operation; round-to-nearest is
// symmetric, so only the sign of an exact zero can differ from the scalar kernel.
// Used when N is even and x / v0 / spike / v / bits are 8-byte aligned.
// ------------------------------------------------------------------------------------
template <int SCHEME, int T, bool TP2>
__global__ void __launch_bounds__(256) single_fwd_x2(SingleArgs a) {
    __shared__ float sw[T + 1];
    for (int e = threadIdx.x; e <= T; e += blockDim.x) sw[e] = a.w[e];
    __syncthreads();
    const long long N = a.N;
    const long long n = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
    if (n >= N) return;
    constexpr bool NEG = SCHEME != kPRED && SCHEME != kPRED1;
    float2 wr[T + 1];
#pragma unroll
    for (int L = 1; L <= T; ++L) wr[L] = f2(NEG ? -sw[T - L] : sw[T - L]);
    const float th = a.th;
    const float2 th2 = f2(th), inv2 = f2(a.inv_tau), ninv2 = f2(-a.inv_tau);
    const float2 tf2 = f2(__fmaf_rn(1.5f, a.beta, 0.5f));                 // :346
    const float2 ps2 = f2(__fdiv_rn(a.h_beta, a.gamma1));                 // :528
    const float2 wc2 = f2(sw[T]), hb2 = f2(a.h_beta);
    float2 xr[T];
#pragma unroll
    for (int t = 0; t < T; ++t) xr[t] = ld2_stream(a.x + t * N + n);
    float2 v = *reinterpret_cast<const float2*>(a.v0 + n);
    float2 hv[T];
    uint32_t b0 = 0, b1 = 0;
#pragma unroll
    for (int k = 0; k < T; ++k) {
        const float2 xm = psub2(xr[k], v);
        const float2 dv = TP2 ? pmul2(xm, inv2)
                              : make_float2(__fdiv_rn(xm.x, a.tau), __fdiv_rn(xm.y, a.tau));
        float2 s = f2(0.0f), cn = f2(-0.0f);       // Kahan sum (negated when NEG), cn = -c
#pragma unroll
        for (int i = 0; i < k; ++i) {
            const float2 y = pfma2(wr[k - i], hv[i], cn);
            // the running sum is formed by two scalar adds: with a packed add here the
            // optimised code was seen to lose the compensation in some chains (the GPU
            // suite compares every instantiation of this kernel bit for bit)
            const float2 t = make_float2(__fadd_rn(s.x, y.x), __fadd_rn(s.y, y.y));
            cn = padd2(y, psub2(s, t));
            s = t;
        }
        float2 p;
        if constexpr (SCHEME == kGL) p = sadd2(dv, s);                          // dv - hist (dv is a product)
        else if constexpr (SCHEME == kGL1) p = pfma2(hb2, dv, s);               // fma(hb, dv, -hist)
        else if constexpr (SCHEME == kTRAP1) p = padd2(pfma2(hb2, dv, v), s);   // fma(hb, dv, v) - hist
        else if constexpr (SCHEME == kPRED1) p = pfma2(hb2, pfma2(wc2, dv, s), v);
        else if constexpr (SCHEME == kTRAP) p = padd2(v, pfma2(tf2, dv, s));    // v + fma(tf, dv, -hist)
        else p = pfma2(ps2, pfma2(wc2, dv, s), v);                              // predictor
        // v = p - spike*th with spike*th exactly th or 0
        const float2 z = psub2(p, th2);
        const bool f0 = p.x >= th, f1 = p.y >= th;
        v = make_float2(f0 ? z.x : p.x, f1 ? z.y : p.y);
        if constexpr (SCHEME == kPRED || SCHEME == kPRED1)
            hv[k] = TP2 ? pmul2(v, ninv2)
                        : make_float2(__fdiv_rn(-v.x, a.tau), __fdiv_rn(-v.y, a.tau));
        else
            hv[k] = v;
        b0 |= (f0 ? 1u : 0u) << k;
        b1 |= (f1 ? 1u : 0u) << k;
        st2_stream(a.spike + k * N + n, make_float2(f0 ? 1.0f : 0.0f, f1 ? 1.0f : 0.0f));
        st2_stream(a.v + k * N + n, v);
    }
    *reinterpret_cast<uint2*>(a.bits + n) = make_uint2(b0, b1);
}

constexpr int kLongBlock = 64;

// ------------------------------------------------------------------------------------
// forward, T > 32: blocked pull form.  The history sum of step k is one Kahan chain over
// i = 0..k-1 whose loop-carried path (fma, add, sub, sub) is ~16 cycles per term, and the
// shared-memory history (T floats per neuron) leaves room for only ~200 neurons (6 warps)
// per SM: one chain per thread left the FP32 pipes less than half busy (ncu: issue stalls on
// fixed-latency dependencies).  The chains of the kBlk steps k0..k0+kBlk-1 are independent
// over the terms i < k0, which are known before step k0 starts, so they advance together
// there (kBlk chains per thread, four terms per iteration, one history load per term and a
// sliding window of weights); inside the block, each new history value is folded into the
// later chains of the block as soon as it exists.  Every chain still takes its terms in the
// reference's order i = 0, 1, ..., k-1: the sums are bit-identical.
// ------------------------------------------------------------------------------------
#define DFSNN_KAHAN(S, C, W, H)                                                           \
    do {                                                                                  \
        const float y_ = __fmaf_rn((W), (H), -(C));                                       \
        const float t_ = __fadd_rn((S), y_);                                              \
        (C) = __fsub_rn(__fsub_rn(t_, (S)), y_);                                          \
        (S) = t_;                                                                         \
    } while (0)

constexpr int kBlkPad = 16;       // zeros in front of the weight table (window reads, KB <= 16)

// KB chains advance together (8 or 16; a multiple of 8, so every k0 gives an even trip count
// of the unrolled term loop).  The 6 warps per SM that fit leave the FP32 pipes idle between
// dependent operations unless each thread carries enough independent chains.
template <int SCHEME, bool TP2, int KB>
__global__ void __launch_bounds__(kLongBlock) single_fwd_blk(SingleArgs a) {
    static_assert(KB % 8 == 0 && KB <= kBlkPad, "KB: 8 or 16");
    constexpr int kBlk = KB;
    extern __shared__ float sh[];
    const int T = a.T;
    float* sw = sh + kBlkPad;                        // [T+1] after kBlkPad zeros
    float* hv = sh + ((kBlkPad + T + 1 + 3) & ~3) + threadIdx.x;   // [T][kLongBlock]
    if (threadIdx.x < kBlkPad) sh[threadIdx.x] = 0.0f;
    for (int e = threadIdx.x; e <= T; e += blockDim.x) sw[e] = a.w[e];
    __syncthreads();
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const float trap_factor = __fmaf_rn(1.5f, a.beta, 0.5f);
    const float pred_scale = __fdiv_rn(a.h_beta, a.gamma1);
    const float w_cur = sw[T];
    float v = a.v0[n];
    uint32_t bits = 0;
    for (int k0 = 0; k0 < T; k0 += kBlk) {
        float xk[kBlk];
#pragma unroll
        for (int j = 0; j < kBlk; ++j)
            if (k0 + j < T) xk[j] = ld_stream(a.x + (long long)(k0 + j) * N + n);
        float sm[kBlk], cm[kBlk];
#pragma unroll
        for (int j = 0; j < kBlk; ++j) sm[j] = cm[j] = 0.0f;
        // chains k0 + j over the known terms i < k0 (k0 % 4 == 0): weight sw[T - k0 - j + i]
        // = wb[i - j]; per iteration the window holds wb[i - kBlk + 1 .. i + 3]
        const float* wb = sw + (T - k0);             // i - j >= -(kBlk - 1) stays in sh
        float wm[kBlk];                              // wm[d] = wb[i - d], d = 1..kBlk-1
#pragma unroll
        for (int d = 1; d < kBlk; ++d) wm[d] = wb[-d];
        // operands of iteration i are loaded during iteration i - 4 (shared-memory latency
        // off the dependency chains: only ~6 warps per SM are resident to hide it)
        float wa[4], h[4];
        if (k0 > 0) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                wa[u] = wb[u];
                h[u] = hv[u * kLongBlock];
            }
        }
#pragma unroll 2
        for (int i = 0; i < k0; i += 4) {           // k0 % 8 == 0: an even trip count
            float wn[4], hn[4];
            if (i + 4 < k0) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    wn[u] = wb[i + 4 + u];
                    hn[u] = hv[(i + 4 + u) * kLongBlock];
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int j = 0; j < kBlk; ++j) {
                    // weight of term i + u for chain j: wb[i + u - j]
                    const int d = j - u;                 // > 0: from the carried window
                    const float w = d > 0 ? wm[d > 0 ? d : 1] : wa[d > 0 ? 0 : -d];
                    DFSNN_KAHAN(sm[j], cm[j], w, h[u]);
                }
#pragma unroll
            for (int d = kBlk - 1; d >= 1; --d)         // slide by four terms
                wm[d] = d > 4 ? wm[d - 4] : wa[4 - d];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                wa[u] = wn[u];
                h[u] = hn[u];
            }
        }
        // the block's own steps, in order; each new history value goes into the later chains
#pragma unroll
        for (int j = 0; j < kBlk; ++j) {
            const int k = k0 + j;
            if (k < T) {
                const float dv = div_tau<TP2>(__fsub_rn(xk[j], v), a.tau, a.inv_tau);
                const float p = single_update<SCHEME>(v, dv, sm[j], trap_factor, pred_scale,
                                                      w_cur, a.h_beta);
                const bool fire = p >= a.th;
                const float s = fire ? 1.0f : 0.0f;
                v = __fsub_rn(p, s * a.th);
                const float hk = (SCHEME == kPRED || SCHEME == kPRED1)
                                     ? div_tau<TP2>(-v, a.tau, a.inv_tau) : v;
                hv[k * kLongBlock] = hk;
#pragma unroll
                for (int jj = j + 1; jj < kBlk; ++jj)    // term k of chain k0 + jj: sw[T - jj + j]
                    DFSNN_KAHAN(sm[jj], cm[jj], sw[T - jj + j], hk);
                bits |= (fire ? 1u : 0u) << (k & 31);
                st_stream(a.spike + (long long)k * N + n, s);
                st_stream(a.v + (long long)k * N + n, v);
                if ((k & 31) == 31 || k == T - 1) {
                    a.bits[(long long)(k >> 5) * N + n] = bits;
                    bits = 0;
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------
// forward, T >= 128, history read back from the membrane output.  Same blocked pull form and
// term order as single_fwd_blk, but the history value of step i is re-read from row i of v,
// which this thread wrote when it finished step i (the PREDICTOR schemes convert it with the
// same -v/tau that produced it), instead of being kept in shared memory.  With no T floats of
// shared memory per neuron, residency is set by registers instead of shared memory, and the
// rows of the resident neurons (T floats each) stay in L2: the history loads are cache hits,
// issued two iterations (eight terms) before their use.
// ------------------------------------------------------------------------------------
constexpr int kL2Block = 128;
constexpr int kL2MinT = 128;      // history read back from v from this T on (T = 64: 7 % slower,
                                  // T = 256: 9 % faster than shared memory)
constexpr int kL2Chains = 16;

template <int SCHEME, bool TP2, int KB>
__global__ void __launch_bounds__(kL2Block) single_fwd_l2(SingleArgs a) {
    static_assert(KB % 8 == 0 && KB <= kBlkPad, "KB: 8 or 16");
    constexpr int kBlk = KB;
    constexpr bool PRED = SCHEME == kPRED || SCHEME == kPRED1;
    extern __shared__ __align__(16) float sh[];
    const int T = a.T;
    // weight table sw[0..T] placed so that sw + T is 16-byte aligned, with at least 16 zeros
    // in front of it: the window wb[i-16 .. i+3] of every term iteration is five float4 loads
    const int off = kBlkPad + ((4 - (T & 3)) & 3);
    float* sw = sh + off;
    if (threadIdx.x < off) sh[threadIdx.x] = 0.0f;
    for (int e = threadIdx.x; e <= T; e += blockDim.x) sw[e] = a.w[e];
    __syncthreads();
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const float* hrow = a.v + n;                     // v of step i at hrow[i * N]
    auto hist = [&](float vv) { return PRED ? div_tau<TP2>(-vv, a.tau, a.inv_tau) : vv; };
    const float trap_factor = __fmaf_rn(1.5f, a.beta, 0.5f);
    const float pred_scale = __fdiv_rn(a.h_beta, a.gamma1);
    const float w_cur = sw[T];
    float v = a.v0[n];
    uint32_t bits = 0;
    for (int k0 = 0; k0 < T; k0 += kBlk) {
        float xk[kBlk];
#pragma unroll
        for (int j = 0; j < kBlk; ++j)
            if (k0 + j < T) xk[j] = ld_stream(a.x + (long long)(k0 + j) * N + n);
        float sm[kBlk], cm[kBlk];
#pragma unroll
        for (int j = 0; j < kBlk; ++j) sm[j] = cm[j] = 0.0f;
        const float* wb = sw + (T - k0);             // weight of term i, chain j: wb[i - j]
        // four terms i..i+3 against all chains; hb holds their raw v and is refilled with
        // terms i+8..i+11 once used (two buffers, so the loads are two iterations ahead)
        auto terms = [&](int i, float (&hb)[4]) {
            const float4* w4 = reinterpret_cast<const float4*>(wb + i - 16);
            float wl[20];                            // wl[16 + d] = wb[i + d]
#pragma unroll
            for (int q = 0; q < 5; ++q) {
                const float4 t4 = w4[q];
                wl[4 * q] = t4.x;
                wl[4 * q + 1] = t4.y;
                wl[4 * q + 2] = t4.z;
                wl[4 * q + 3] = t4.w;
            }
            float hu[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) hu[u] = hist(hb[u]);
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int j = 0; j < kBlk; ++j) DFSNN_KAHAN(sm[j], cm[j], wl[16 + u - j], hu[u]);
            if (i + 8 < k0) {                        // k0 % 4 == 0: i + 11 < k0 as well
#pragma unroll
                for (int u = 0; u < 4; ++u) hb[u] = hrow[(long long)(i + 8 + u) * N];
            }
        };
        if (k0 > 0) {                                // k0 >= kBlk >= 8 terms are known
            float ha[4], hc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                ha[u] = hrow[(long long)u * N];
                hc[u] = hrow[(long long)(4 + u) * N];
            }
            for (int i = 0; i < k0; i += 8) {       // k0 % 8 == 0
                terms(i, ha);
                terms(i + 4, hc);
            }
        }
        // weights of lags 1..15 for the block's own terms: wlag[16 - L] = sw[T - L] (16-byte
        // aligned, T >= 16)
        float wlag[16];
        {
            const float4* l4 = reinterpret_cast<const float4*>(sw + T - 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 t4 = l4[q];
                wlag[4 * q] = t4.x;
                wlag[4 * q + 1] = t4.y;
                wlag[4 * q + 2] = t4.z;
                wlag[4 * q + 3] = t4.w;
            }
        }
#pragma unroll
        for (int j = 0; j < kBlk; ++j) {
            const int k = k0 + j;
            if (k < T) {
                const float dv = div_tau<TP2>(__fsub_rn(xk[j], v), a.tau, a.inv_tau);
                const float p = single_update<SCHEME>(v, dv, sm[j], trap_factor, pred_scale,
                                                      w_cur, a.h_beta);
                const bool fire = p >= a.th;
                const float s = fire ? 1.0f : 0.0f;
                v = __fsub_rn(p, s * a.th);
                const float hk = hist(v);
#pragma unroll
                for (int jj = j + 1; jj < kBlk; ++jj)
                    DFSNN_KAHAN(sm[jj], cm[jj], wlag[16 - (jj - j)], hk);
                bits |= (fire ? 1u : 0u) << (k & 31);
                st_stream(a.spike + (long long)k * N + n, s);
                a.v[(long long)k * N + n] = v;          // re-read as history: keep it cached
                if ((k & 31) == 31 || k == T - 1) {
                    a.bits[(long long)(k >> 5) * N + n] = bits;
                    bits = 0;
                }
            }
        }
    }
}
#undef DFSNN_KAHAN

// ------------------------------------------------------------------------------------
// backward: truncated reverse sweep from the saved membrane and spike bits (any T)
// ------------------------------------------------------------------------------------
template <int SCHEME, bool TP2, class WFn>
__device__ __forceinline__ void single_bwd_step(const SingleArgs& a, int t, float vt, bool fire,
                                                float gst, float gvt, float& gv, float trap_factor,
                                                float pred_scale, float w_cur, float* gx_out,
                                                WFn lag_weight) {
    gv = __fadd_rn(gv, gvt);
    const float p = __fmaf_rn(fire ? 1.0f : 0.0f, a.th, vt);          // v + spike*theta
    const float surr = surrogate_fma(__fsub_rn(p, a.th), a.sg);
    gv = __fmaf_rn(gst, surr, gv);
    float gvm;
    if constexpr (SCHEME == kGL) {                                      // :150-154
        *gx_out = div_tau<TP2>(gv, a.tau, a.inv_tau);
        gvm = div_tau<TP2>(-gv, a.tau, a.inv_tau);
    } else if constexpr (SCHEME == kTRAP) {                             // :459-463
        const float gsd = __fmul_rn(gv, trap_factor);
        const float q = div_tau<TP2>(gsd, a.tau, a.inv_tau);
        *gx_out = q;
        gvm = __fsub_rn(gv, q);
    } else if constexpr (SCHEME == kPRED) {                             // :621-629
        const float gdc = __fmul_rn(__fmul_rn(gv, pred_scale), w_cur);
        const float q = div_tau<TP2>(gdc, a.tau, a.inv_tau);
        *gx_out = q;
        gvm = __fsub_rn(gv, q);
    } else if constexpr (SCHEME == kEULER) {                            // LIFEuler :2645-2647
        *gx_out = div_tau<TP2>(gv, a.tau, a.inv_tau);
        gvm = __fmul_rn(gv, __fsub_rn(1.0f, __fdiv_rn(1.0f, a.tau)));
    } else {                                                            // GL1 :296-312
        const float gd = __fmul_rn(a.h_beta, gv);
        *gx_out = div_tau<TP2>(gd, a.tau, a.inv_tau);
        gvm = div_tau<TP2>(-gd, a.tau, a.inv_tau);
        for (int i = 0; i < t; ++i) gvm = __fmaf_rn(-lag_weight(t - i), gv, gvm);
    }
    gv = gvm;
}

template <int SCHEME, int TB, bool TP2>
__global__ void __launch_bounds__(256) single_bwd_reg(SingleArgs a) {
    __shared__ float sw[(SCHEME == kGL1) ? TB + 1 : 1];
    const int T = a.T;
    if constexpr (SCHEME == kGL1) {
        for (int e = threadIdx.x; e <= T; e += blockDim.x) sw[e] = a.w[e];
        __syncthreads();
    }
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const float trap_factor = __fmaf_rn(1.5f, a.beta, 0.5f);
    const float pred_scale = __fdiv_rn(a.h_beta, a.gamma1);
    const float w_cur = (SCHEME == kPRED) ? __ldg(a.w + T) : 0.0f;
    float vr[TB], gsr[TB], gvr[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        if (t < T) {
            vr[t] = ld_stream(a.vs + t * N + n);
            gsr[t] = ld_stream(a.gS + t * N + n);
            gvr[t] = ld_stream(a.gV + t * N + n);
        }
    }
    const uint32_t bits = a.bits_in[n];
    float wr[(SCHEME == kGL1) ? TB + 1 : 1];
    if constexpr (SCHEME == kGL1) {
#pragma unroll
        for (int L = 0; L <= TB; ++L) wr[L] = (L <= T) ? sw[T - L] : 0.0f;
    }
    float gv = 0.0f;
#pragma unroll
    for (int t = TB - 1; t >= 0; --t) {
        if (t < T) {
            float gxt;
            single_bwd_step<SCHEME, TP2>(a, t, vr[t], (bits >> t) & 1u, gsr[t], gvr[t], gv,
                                         trap_factor, pred_scale, w_cur, &gxt,
                                         [&](int L) { return wr[(SCHEME == kGL1) ? L : 0]; });
            st_stream(a.gx + t * N + n, gxt);
        }
    }
    a.gv0[n] = gv;
}

template <int SCHEME, bool TP2>
__global__ void __launch_bounds__(256) single_bwd_loop(SingleArgs a) {
    extern __shared__ float sw[];
    const int T = a.T;
    if constexpr (SCHEME == kGL1) {
        for (int e = threadIdx.x; e <= T; e += blockDim.x) sw[e] = a.w[e];
        __syncthreads();
    }
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const float trap_factor = __fmaf_rn(1.5f, a.beta, 0.5f);
    const float pred_scale = __fdiv_rn(a.h_beta, a.gamma1);
    const float w_cur = (SCHEME == kPRED) ? __ldg(a.w + T) : 0.0f;
    float gv = 0.0f;
    uint32_t bits = 0;
    // rows are consumed from t = T-1 down; the loads of the next kPf rows are issued before
    // the current kPf rows are processed, so each thread keeps two groups of loads in flight
    constexpr int kPf = 4;
    float vb[kPf], gsb[kPf], gvb[kPf];
    auto load_rows = [&](int t0, float (&vr)[kPf], float (&sr)[kPf], float (&gr)[kPf]) {
#pragma unroll
        for (int u = 0; u < kPf; ++u) {
            const long long t = t0 - u;
            if (t >= 0) {
                vr[u] = ld_stream(a.vs + t * N + n);
                sr[u] = ld_stream(a.gS + t * N + n);
                gr[u] = ld_stream(a.gV + t * N + n);
            }
        }
    };
    load_rows(T - 1, vb, gsb, gvb);
    for (int t0 = T - 1; t0 >= 0; t0 -= kPf) {
        float vn[kPf], gsn[kPf], gvn[kPf];
        if (t0 >= kPf) load_rows(t0 - kPf, vn, gsn, gvn);
#pragma unroll
        for (int u = 0; u < kPf; ++u) {
            const int t = t0 - u;
            if (t >= 0) {
                if (t == T - 1 || (t & 31) == 31) bits = a.bits_in[(long long)(t >> 5) * N + n];
                float gxt;
                single_bwd_step<SCHEME, TP2>(a, t, vb[u], (bits >> (t & 31)) & 1u, gsb[u],
                                             gvb[u], gv, trap_factor, pred_scale, w_cur, &gxt,
                                             [&](int L) { return sw[T - L]; });
                st_stream(a.gx + (long long)t * N + n, gxt);
            }
        }
#pragma unroll
        for (int u = 0; u < kPf; ++u) {
            vb[u] = vn[u];
            gsb[u] = gsn[u];
            gvb[u] = gvn[u];
        }
    }
    a.gv0[n] = gv;
}

// ------------------------------------------------------------------------------------
// LIFEuler forward (fde_cupy_kernels_all.py:2546-2584): v + (x - v)/tau, no history; one
// neuron per thread, streaming, spike bitmask for the backward as for the other schemes.
// ------------------------------------------------------------------------------------
template <bool TP2>
__global__ void __launch_bounds__(256) euler_lif_fwd(SingleArgs a) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int T = a.T;
    float v = a.v0[n];
    uint32_t word = 0;
    for (int k = 0; k < T; ++k) {
        const float dv = div_tau<TP2>(__fsub_rn(ld_stream(a.x + k * N + n), v), a.tau, a.inv_tau);
        const float p = __fadd_rn(v, dv);
        const bool fire = p >= a.th;
        v = fire ? __fsub_rn(p, a.th) : p;                   // p - spike*th
        st_stream(a.spike + k * N + n, fire ? 1.0f : 0.0f);
        st_stream(a.v + k * N + n, v);
        word |= (fire ? 1u : 0u) << (k & 31);
        if ((k & 31) == 31 || k == T - 1) {
            a.bits[(k >> 5) * N + n] = word;
            word = 0;
        }
    }
}

// ------------------------------------------------------------------------------------
// TRAP1 / PREDICTOR1 backward (fde_cupy_kernels_all.py:2072-2161, :2337-2432).  The
// reference recomputes the trajectory here with a plain fused multiply-add history sum --
// not the forward's Kahan sum, so its membranes and spikes may differ from the forward's --
// and the reverse step's history term touches only the current gradient.  Both are
// reproduced operation by operation: one thread per neuron, the recomputed membranes (and
// PREDICTOR1's history derivatives -v/tau) in shared memory [T][64], spikes as bits.
// ------------------------------------------------------------------------------------
constexpr int kS1Threads = 64;

template <int SCHEME, bool TP2>
__global__ void __launch_bounds__(kS1Threads) single1_bwd(SingleArgs a) {
    extern __shared__ float sh[];
    const int T = a.T;
    const int tid = threadIdx.x;
    const int wpad = (T + 1 + 3) & ~3;
    float* sw = sh;                                            // [T+1] weights
    float* hbw = sh + wpad;                                    // [T+1] h_beta * w (PREDICTOR1)
    float* VL = sh + 2 * wpad;                                 // [T][64] recomputed v
    float* HV = (SCHEME == kPRED1) ? VL + (size_t)T * kS1Threads : VL;   // [T][64] history
    uint32_t* SB = reinterpret_cast<uint32_t*>(HV + (size_t)T * kS1Threads);   // [8][64] spikes
    for (int e = tid; e <= T; e += blockDim.x) {
        sw[e] = a.w[e];
        hbw[e] = __fmul_rn(a.h_beta, a.w[e]);
    }
    __syncthreads();
    const long long n = (long long)blockIdx.x * kS1Threads + tid;
    if (n >= a.N) return;
    const long long N = a.N;
    const float hb = a.h_beta, th = a.th;
    for (int wdx = 0; wdx < (T + 31) / 32; ++wdx) SB[wdx * kS1Threads + tid] = 0u;
    float v = a.v0[n];
    for (int k = 0; k < T; ++k) {
        const float dv = div_tau<TP2>(__fsub_rn(ld_stream(a.x + k * N + n), v), a.tau, a.inv_tau);
        float hist = 0.0f;
        for (int i = 0; i < k; ++i) hist = __fmaf_rn(sw[T - k + i], HV[i * kS1Threads + tid], hist);
        const float p = SCHEME == kTRAP1 ? __fsub_rn(__fmaf_rn(hb, dv, v), hist)
                                         : __fmaf_rn(hb, __fmaf_rn(sw[T], dv, hist), v);
        const bool fire = p >= th;
        const float vn = fire ? __fsub_rn(p, th) : p;           // p - spike*th
        VL[k * kS1Threads + tid] = vn;
        if constexpr (SCHEME == kPRED1) HV[k * kS1Threads + tid] = div_tau<TP2>(-vn, a.tau, a.inv_tau);
        if (fire) SB[(k >> 5) * kS1Threads + tid] |= 1u << (k & 31);
        v = vn;
    }
    const float m1 = SCHEME == kTRAP1 ? __fsub_rn(1.0f, div_tau<TP2>(hb, a.tau, a.inv_tau))
                                      : __fsub_rn(1.0f, div_tau<TP2>(hbw[T], a.tau, a.inv_tau));
    const float gxs = SCHEME == kTRAP1 ? hb : hbw[T];           // h_beta (* w_T)
    float gv = 0.0f;
    for (int t = T - 1; t >= 0; --t) {
        gv = __fadd_rn(gv, ld_stream(a.gV + t * N + n));
        const float vl = VL[t * kS1Threads + tid];
        const bool fire = (SB[(t >> 5) * kS1Threads + tid] >> (t & 31)) & 1u;
        const float pp = fire ? __fadd_rn(vl, th) : vl;         // v + spike*th
        gv = __fmaf_rn(ld_stream(a.gS + t * N + n), surrogate_fma(__fsub_rn(pp, th), a.sg), gv);
        st_stream(a.gx + t * N + n, div_tau<TP2>(__fmul_rn(gxs, gv), a.tau, a.inv_tau));
        float gvm = __fmul_rn(gv, m1);
        if constexpr (SCHEME == kTRAP1) {
            for (int i = 0; i < t; ++i) gvm = __fmaf_rn(-sw[T - t + i], gv, gvm);
        } else {
            for (int i = 0; i < t; ++i)
                gvm = __fsub_rn(gvm, div_tau<TP2>(__fmul_rn(hbw[T - t + i], gv), a.tau, a.inv_tau));
        }
        gv = gvm;
    }
    a.gv0[n] = gv;
}

// ------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------
namespace {

SingleArgs make_args(int T, long long N, float tau, float beta, float th, float sg, float h_beta,
                     float gamma1) {
    SingleArgs a{};
    a.T = T; a.N = N; a.tau = tau; a.inv_tau = 1.0f / tau; a.beta = beta; a.th = th; a.sg = sg;
    a.h_beta = h_beta; a.gamma1 = gamma1;
    return a;
}

bool aligned8_all(const void* p, const void* q, const void* r, const void* s, const void* t) {
    return ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(q) |
             reinterpret_cast<uintptr_t>(r) | reinterpret_cast<uintptr_t>(s) |
             reinterpret_cast<uintptr_t>(t)) & 7u) == 0;
}

template <int SCHEME, bool TP2>
cudaError_t fwd_dispatch(const SingleArgs& a, cudaStream_t st) {
    const int T = a.T;
    if constexpr (SCHEME == kEULER) {
        euler_lif_fwd<TP2><<<(unsigned)((a.N + 255) / 256), 256, 0, st>>>(a);
        return cudaGetLastError();
    }
    if ((T == 8 || T == 16) && (a.N % 2) == 0 && aligned8_all(a.x, a.v0, a.spike, a.v, a.bits)) {
        const unsigned grid = (unsigned)((a.N / 2 + 255) / 256);
        if (T == 8) single_fwd_x2<SCHEME, 8, TP2><<<grid, 256, 0, st>>>(a);
        else single_fwd_x2<SCHEME, 16, TP2><<<grid, 256, 0, st>>>(a);
        return cudaGetLastError();
    }
    if (T <= 32) {
        const unsigned grid = (unsigned)((a.N + 255) / 256);
        if (T <= 8) single_fwd_reg<SCHEME, 8, TP2><<<grid, 256, 0, st>>>(a);
        else if (T <= 16) single_fwd_reg<SCHEME, 16, TP2><<<grid, 256, 0, st>>>(a);
        else single_fwd_reg<SCHEME, 32, TP2><<<grid, 256, 0, st>>>(a);
        return cudaGetLastError();
    }
    if (T >= kL2MinT) {
        const unsigned grid = (unsigned)((a.N + kL2Block - 1) / kL2Block);
        const size_t smem = sizeof(float) * (size_t)(kBlkPad + 3 + T + 1);
        single_fwd_l2<SCHEME, TP2, kL2Chains><<<grid, kL2Block, smem, st>>>(a);
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned)((a.N + kLongBlock - 1) / kLongBlock);
    const size_t smem = sizeof(float) * (((kBlkPad + T + 1 + 3) & ~3) + (size_t)T * kLongBlock);
    auto k = single_fwd_blk<SCHEME, TP2, 16>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, kLongBlock, smem, st>>>(a);
    return cudaGetLastError();
}

template <int SCHEME, bool TP2>
cudaError_t bwd_dispatch(const SingleArgs& a, cudaStream_t st) {
    const int T = a.T;
    const unsigned grid = (unsigned)((a.N + 255) / 256);
    if (T <= 32) {
        if (T <= 8) single_bwd_reg<SCHEME, 8, TP2><<<grid, 256, 0, st>>>(a);
        else if (T <= 16) single_bwd_reg<SCHEME, 16, TP2><<<grid, 256, 0, st>>>(a);
        else single_bwd_reg<SCHEME, 32, TP2><<<grid, 256, 0, st>>>(a);
        return cudaGetLastError();
    }
    const size_t smem = (SCHEME == kGL1) ? sizeof(float) * (size_t)(T + 1) : 0;
    single_bwd_loop<SCHEME, TP2><<<grid, 256, smem, st>>>(a);
    return cudaGetLastError();
}

template <bool TP2>
cudaError_t fwd_scheme(int scheme, const SingleArgs& a, cudaStream_t st) {
    switch (scheme) {
        case kGL: return fwd_dispatch<kGL, TP2>(a, st);
        case kTRAP: return fwd_dispatch<kTRAP, TP2>(a, st);
        case kPRED: return fwd_dispatch<kPRED, TP2>(a, st);
        case kGL1: return fwd_dispatch<kGL1, TP2>(a, st);
        case kTRAP1: return fwd_dispatch<kTRAP1, TP2>(a, st);
        case kPRED1: return fwd_dispatch<kPRED1, TP2>(a, st);
        case kEULER: return fwd_dispatch<kEULER, TP2>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

template <bool TP2>
cudaError_t bwd_scheme(int scheme, const SingleArgs& a, cudaStream_t st) {
    switch (scheme) {
        case kGL: return bwd_dispatch<kGL, TP2>(a, st);
        case kTRAP: return bwd_dispatch<kTRAP, TP2>(a, st);
        case kPRED: return bwd_dispatch<kPRED, TP2>(a, st);
        case kGL1: return bwd_dispatch<kGL1, TP2>(a, st);
        case kEULER: return bwd_dispatch<kEULER, TP2>(a, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t single_forward_launch(int scheme, const float* x, const float* v0, const float* w,
                                  float* spike, float* v, uint32_t* bits, int T, long long N,
                                  float tau, float beta, float th, float h_beta, float gamma1,
                                  bool tau_pow2, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    SingleArgs a = make_args(T, N, tau, beta, th, 0.0f, h_beta, gamma1);
    a.x = x; a.v0 = v0; a.w = w; a.spike = spike; a.v = v; a.bits = bits;
    return tau_pow2 ? fwd_scheme<true>(scheme, a, st) : fwd_scheme<false>(scheme, a, st);
}

cudaError_t single_backward_launch(int scheme, const float* gS, const float* gV, const float* v,
                                   const uint32_t* bits, const float* w, float* gx, float* gv0,
                                   int T, long long N, float tau, float beta, float th, float sg,
                                   float h_beta, float gamma1, bool tau_pow2, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    SingleArgs a = make_args(T, N, tau, beta, th, sg, h_beta, gamma1);
    a.gS = gS; a.gV = gV; a.vs = v; a.bits_in = bits; a.w = w; a.gx = gx; a.gv0 = gv0;
    return tau_pow2 ? bwd_scheme<true>(scheme, a, st) : bwd_scheme<false>(scheme, a, st);
}

cudaError_t single1_backward_launch(int scheme, const float* gS, const float* gV, const float* x,
                                    const float* v0, const float* w, float* gx, float* gv0,
                                    int T, long long N, float tau, float th, float sg,
                                    float h_beta, bool tau_pow2, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    SingleArgs a = make_args(T, N, tau, 0.0f, th, sg, h_beta, 1.0f);
    a.x = x; a.v0 = v0; a.w = w; a.gS = gS; a.gV = gV; a.gx = gx; a.gv0 = gv0;
    const int wpad = (T + 1 + 3) & ~3;
    const int arrays = scheme == kPRED1 ? 2 : 1;
    const size_t smem = sizeof(float) * (2 * (size_t)wpad + (size_t)arrays * T * kS1Threads) +
                        sizeof(uint32_t) * 8 * kS1Threads;
    const unsigned grid = (unsigned)((N + kS1Threads - 1) / kS1Threads);
    cudaError_t e;
#define DFSNN_S1(SCH, P2)                                                                    \
    {                                                                                        \
        auto k = single1_bwd<SCH, P2>;                                                       \
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        if (e != cudaSuccess) return e;                                                      \
        k<<<grid, kS1Threads, smem, st>>>(a);                                                \
    }
    if (scheme == kTRAP1) {
        if (tau_pow2) DFSNN_S1(kTRAP1, true) else DFSNN_S1(kTRAP1, false)
    } else if (scheme == kPRED1) {
        if (tau_pow2) DFSNN_S1(kPRED1, true) else DFSNN_S1(kPRED1, false)
    } else {
        return cudaErrorInvalidValue;
    }
#undef DFSNN_S1
    return cudaGetLastError();
}

}  // namespace dfsnn
