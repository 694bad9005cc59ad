// hfam.cu -- LIF-FDE with an explicit history table and shared or per-sample parameters:
// VO-GL1, FAGL1 and VO-PREDICTOR (LIFFDEVOGL1Function, LIFFDEFAGL1Function and
// LIFFDEVOPREDICTORFunction, fde_cupy_kernels_all.py:1751-1843, :1379-1500, :1098-1198).
//
// Every neuron n belongs to sample b = n / (N/B).  With per-sample tables scale is [T, B] and
// the weights [T, B, T]; shared tables are [T] and [T, T].  Per step t, d_t = (x_t - v)/tau,
//   VO-GL1 / FAGL1:  p_t = s_t*d_t - sum_{i<t} W[t,i] v_i       (s_t = h_beta for FAGL1)
//                    spike = p_t >= th,  v_t = p_t - spike*th,  history value v_t
//   VO-PREDICTOR:    p_t = v0 + s_t*(d_t + sum_{i<t} W[t,i] d_i) + rm*(v - v0)
//                    history value d_t
// (:1594-1630, :1200-1232, :1017-1057) with the reference's rounding steps written out as
// intrinsics (NVRTC --fmad=true contracts hist += w*h to one fma, s*d - hist to
// fma(s, d, -hist), v0 + s*(d+hist) + rm*(v-v0) to two fmas).
//
// Forward: one thread per neuron; x is read once, spike, v_pre and the history sequence
// (plus the drift for VO-GL1, which its parameter gradient needs) are written once.  For
// T = 8 and 16 the history lives in registers (fully unrolled); otherwise in a shared-memory
// column per thread (T <= 256).
// Backward: the reverse sweeps of :1633-1668 (truncated: grad_v_next = -gp*(s/tau + sum_i
// W[t,i])), :1670-1709 (full history, T <= 64: an adjoint per earlier step) and :1058-1096
// (VO-PREDICTOR: grad_v_next = gp*(rm - s/tau)), writing grad_x, grad_v0 and grad_pre.  The
// parameter gradients are reductions of grad_pre against the saved history (param_long.cu)
// finished here by hfam_sum + hfam_epilogue.
#include "kernels.h"
#include "lif_common.cuh"

namespace dfsnn {

namespace {

struct HfTables {
    const float* scale;   // NULL: every s_t = hb
    float hb;
    const float* W;
    long long F;          // neurons per sample
    int B;
    int per_batch;

    __device__ __forceinline__ int sample(long long n) const { return (int)(n / F); }
    __device__ __forceinline__ float s(int t, int b) const {
        return scale ? __ldg(scale + (per_batch ? (long long)t * B + b : t)) : hb;
    }
    __device__ __forceinline__ const float* wrow(int t, int b, int T) const {
        return W + (per_batch ? ((long long)t * B + b) * T : (long long)t * T);
    }
};

struct HfFwd {
    const float* x;
    const float* v0;
    HfTables tab;
    float* spike;
    float* vpre;
    float* hsrc;    // history sequence: v after reset (GL kinds) or drift (VO-PREDICTOR)
    float* drift;   // optional drift sequence (VO-GL1)
    int T;
    long long N;
    float tau, inv_tau, th, rm;
};

template <bool PRED>
__device__ __forceinline__ float pre_value(float sv, float d, float hist, float v, float vi,
                                           float rm) {
    if constexpr (PRED) return __fmaf_rn(rm, __fsub_rn(v, vi), __fmaf_rn(sv, __fadd_rn(d, hist), vi));
    else return __fmaf_rn(sv, d, -hist);
}

// T known at compile time: history and inputs in registers
template <bool PRED, int TT, bool TAU_POW2>
__global__ void __launch_bounds__(256) hfam_fwd_r(HfFwd a) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int b = a.tab.sample(n);
    float xr[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) xr[t] = ld_stream(a.x + (long long)t * N + n);
    const float vi = a.v0[n];
    float v = vi;
    float h[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        const long long o = (long long)t * N + n;
        const float d = div_tau<TAU_POW2>(__fsub_rn(xr[t], v), a.tau, a.inv_tau);
        const float* w = a.tab.wrow(t, b, TT);
        float hist = 0.0f;
#pragma unroll
        for (int i = 0; i < t; ++i) hist = __fmaf_rn(__ldg(w + i), h[i], hist);
        const float p = pre_value<PRED>(a.tab.s(t, b), d, hist, v, vi, a.rm);
        const float sp = p >= a.th ? 1.0f : 0.0f;
        v = __fmaf_rn(-sp, a.th, p);
        h[t] = PRED ? d : v;
        st_stream(a.spike + o, sp);
        st_stream(a.vpre + o, p);
        st_stream(a.hsrc + o, h[t]);
        if (!PRED && a.drift) st_stream(a.drift + o, d);
    }
}

// any T <= 256: history in a shared-memory column per thread ([T][blockDim] floats)
template <bool PRED, bool TAU_POW2>
__global__ void __launch_bounds__(128) hfam_fwd_s(HfFwd a) {
    extern __shared__ float sh[];
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int T = a.T, stride = blockDim.x;
    float* h = sh + threadIdx.x;
    const int b = a.tab.sample(n);
    const float vi = a.v0[n];
    float v = vi;
    for (int t = 0; t < T; ++t) {
        const long long o = (long long)t * N + n;
        const float d = div_tau<TAU_POW2>(__fsub_rn(ld_stream(a.x + o), v), a.tau, a.inv_tau);
        const float* w = a.tab.wrow(t, b, T);
        float hist = 0.0f;
        for (int i = 0; i < t; ++i) hist = __fmaf_rn(__ldg(w + i), h[i * stride], hist);
        const float p = pre_value<PRED>(a.tab.s(t, b), d, hist, v, vi, a.rm);
        const float sp = p >= a.th ? 1.0f : 0.0f;
        v = __fmaf_rn(-sp, a.th, p);
        const float hv = PRED ? d : v;
        h[t * stride] = hv;
        st_stream(a.spike + o, sp);
        st_stream(a.vpre + o, p);
        st_stream(a.hsrc + o, hv);
        if (!PRED && a.drift) st_stream(a.drift + o, d);
    }
}

struct HfBwd {
    const float* gS;
    const float* vpre;
    HfTables tab;
    float* gx;
    float* gv0;
    float* gpre;
    int T;
    long long N;
    float tau, inv_tau, th, sg, rm;
};

enum HistMode { kTrunc = 0, kFull = 1, kPredMode = 2 };

template <bool FAST_SG>
__device__ __forceinline__ float surr(float z, float sg) {
    if constexpr (FAST_SG) return surrogate_fast(z, sg);
    else return surrogate_fma(z, sg);
}

// grad_v_next of the truncated sweeps
template <int HM, bool TAU_POW2>
__device__ __forceinline__ float trunc_next(const HfBwd& a, const float* w, int t, float gp,
                                            float sv) {
    const float st = div_tau<TAU_POW2>(sv, a.tau, a.inv_tau);
    if constexpr (HM == kPredMode) {
        return __fmul_rn(gp, __fsub_rn(a.rm, st));
    } else {
        float hs = 0.0f;
        for (int i = 0; i < t; ++i) hs = __fadd_rn(hs, __ldg(w + i));
        return __fmul_rn(-gp, __fadd_rn(st, hs));
    }
}

template <int HM, int TT, bool TAU_POW2, bool FAST_SG>
__global__ void __launch_bounds__(256) hfam_bwd_r(HfBwd a) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int b = a.tab.sample(n);
    float gr[TT], pr[TT];
#pragma unroll
    for (int t = 0; t < TT; ++t) {
        gr[t] = ld_stream(a.gS + (long long)t * N + n);
        pr[t] = ld_stream(a.vpre + (long long)t * N + n);
    }
    float A[HM == kFull ? TT : 1];
#pragma unroll
    for (int t = 0; t < (HM == kFull ? TT : 1); ++t) A[t] = 0.0f;
    float gvn = 0.0f, ginit = 0.0f;
#pragma unroll
    for (int t = TT - 1; t >= 0; --t) {
        const long long o = (long long)t * N + n;
        const float sur = surr<FAST_SG>(__fsub_rn(pr[t], a.th), a.sg);
        float gp;
        if constexpr (HM == kFull) gp = __fmaf_rn(gr[t], sur, A[t]);
        else gp = __fmaf_rn(gr[t], sur, gvn);
        const float sv = a.tab.s(t, b);
        const float* w = a.tab.wrow(t, b, TT);
        st_stream(a.gpre + o, gp);
        st_stream(a.gx + o, div_tau<TAU_POW2>(__fmul_rn(gp, sv), a.tau, a.inv_tau));
        if constexpr (HM == kFull) {
            const float prev = div_tau<TAU_POW2>(__fmul_rn(-gp, sv), a.tau, a.inv_tau);
            if (t == 0) ginit = __fadd_rn(ginit, prev);
            else A[t > 0 ? t - 1 : 0] = __fadd_rn(A[t > 0 ? t - 1 : 0], prev);
#pragma unroll
            for (int i = 0; i < t; ++i) A[i] = __fmaf_rn(-__ldg(w + i), gp, A[i]);
        } else {
            gvn = trunc_next<HM, TAU_POW2>(a, w, t, gp, sv);
        }
    }
    a.gv0[n] = HM == kFull ? ginit : gvn;
}

// any T; the full-history adjoints live in a shared-memory column per thread (T <= 64)
template <int HM, bool TAU_POW2, bool FAST_SG>
__global__ void __launch_bounds__(128) hfam_bwd_s(HfBwd a) {
    extern __shared__ float sA[];
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int T = a.T, stride = blockDim.x;
    const int b = a.tab.sample(n);
    float* A = sA + threadIdx.x;
    if constexpr (HM == kFull)
        for (int t = 0; t < T; ++t) A[t * stride] = 0.0f;
    float gvn = 0.0f, ginit = 0.0f;
    for (int t = T - 1; t >= 0; --t) {
        const long long o = (long long)t * N + n;
        const float sur = surr<FAST_SG>(__fsub_rn(ld_stream(a.vpre + o), a.th), a.sg);
        const float gp = __fmaf_rn(ld_stream(a.gS + o), sur, HM == kFull ? A[t * stride] : gvn);
        const float sv = a.tab.s(t, b);
        const float* w = a.tab.wrow(t, b, T);
        st_stream(a.gpre + o, gp);
        st_stream(a.gx + o, div_tau<TAU_POW2>(__fmul_rn(gp, sv), a.tau, a.inv_tau));
        if constexpr (HM == kFull) {
            const float prev = div_tau<TAU_POW2>(__fmul_rn(-gp, sv), a.tau, a.inv_tau);
            if (t == 0) ginit = __fadd_rn(ginit, prev);
            else A[(t - 1) * stride] = __fadd_rn(A[(t - 1) * stride], prev);
            for (int i = 0; i < t; ++i) A[i * stride] = __fmaf_rn(-__ldg(w + i), gp, A[i * stride]);
        } else {
            gvn = trunc_next<HM, TAU_POW2>(a, w, t, gp, sv);
        }
    }
    a.gv0[n] = HM == kFull ? ginit : gvn;
}

// msum[u][e] = sum of the rows of output unit u (sample u, or every row when shared) --
// one warp per entry, lanes over rows in a fixed stride, then a fixed butterfly
__global__ void __launch_bounds__(256) hfam_sum(const double* part, int chunks, int B,
                                                int per_batch, int R, double* msum) {
    const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x % 32;
    const long long units = per_batch ? B : 1;
    if (w >= units * R) return;
    const long long u = w / R, e = w % R;
    const long long r0 = per_batch ? u * chunks : 0;
    const long long nr = per_batch ? chunks : (long long)B * chunks;
    double s = 0.0;
    for (long long r = lane; r < nr; r += 32) s += part[(r0 + r) * R + e];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) msum[w] = s;
}

// one thread per (t, unit): grad_scale[t(,b)] and the weight-gradient row t(,b)
__global__ void __launch_bounds__(256) hfam_epilogue(int kind, const double* msum, int B,
                                                     int per_batch, int T, const float* W,
                                                     const float* scale, float* gscale,
                                                     float* gW) {
    const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long units = per_batch ? B : 1;
    if (id >= units * T) return;
    const int t = (int)(id / units), u = (int)(id % units);
    const int R = T + T * T;
    const double* m = msum + (long long)u * R;
    const double* Mt = m + T + (long long)t * T;
    const long long row = per_batch ? (long long)t * B + u : t;     // [T,B] / [T] index
    float* gw = gW ? gW + row * T : nullptr;
    if (kind == kVOPRED) {
        if (gscale) {
            const float* w = W + row * T;
            double s = Mt[t];
            for (int i = 0; i < T; ++i) s += (double)w[i] * Mt[i];
            gscale[row] = (float)s;
        }
        if (gw) {
            const double sv = (double)scale[row];
            for (int i = 0; i < T; ++i) gw[i] = (float)(sv * Mt[i]);
        }
    } else {
        if (gscale && kind == kVOGL1) gscale[row] = (float)m[t];
        if (gw) {
            const bool lower = kind == kFAGL1 && per_batch;
            for (int i = 0; i < T; ++i) gw[i] = (lower && i >= t) ? 0.0f : (float)(-Mt[i]);
        }
    }
}

HfTables tables(const float* scale, float hb, const float* W, int B, bool per_batch,
                long long N) {
    HfTables tb;
    tb.scale = scale;
    tb.hb = hb;
    tb.W = W;
    tb.B = B;
    tb.per_batch = per_batch ? 1 : 0;
    tb.F = N / B;
    return tb;
}

}  // namespace

cudaError_t hfam_forward_launch(int kind, const float* x, const float* v0, const float* scale,
                                float h_beta, const float* W, int B, bool per_batch, float* spike,
                                float* vpre, float* hsrc, float* drift, int T, long long N,
                                float tau, float th, float rm, bool tau_pow2, cudaStream_t st) {
    if (N <= 0) return cudaSuccess;
    HfFwd a;
    a.x = x;
    a.v0 = v0;
    a.tab = tables(kind == kFAGL1 ? nullptr : scale, h_beta, W, B, per_batch, N);
    a.spike = spike;
    a.vpre = vpre;
    a.hsrc = hsrc;
    a.drift = kind == kVOGL1 ? drift : nullptr;
    a.T = T;
    a.N = N;
    a.tau = tau;
    a.inv_tau = 1.0f / tau;
    a.th = th;
    a.rm = rm;
    const bool pred = kind == kVOPRED;
    if (T == 8 || T == 16) {
        const unsigned grid = (unsigned)((N + 255) / 256);
#define DFSNN_HF_FWD(TV)                                                                      \
        if (T == TV) {                                                                        \
            if (pred) {                                                                       \
                if (tau_pow2) hfam_fwd_r<true, TV, true><<<grid, 256, 0, st>>>(a);            \
                else hfam_fwd_r<true, TV, false><<<grid, 256, 0, st>>>(a);                    \
            } else {                                                                          \
                if (tau_pow2) hfam_fwd_r<false, TV, true><<<grid, 256, 0, st>>>(a);           \
                else hfam_fwd_r<false, TV, false><<<grid, 256, 0, st>>>(a);                   \
            }                                                                                 \
        }
        DFSNN_HF_FWD(8) DFSNN_HF_FWD(16)
#undef DFSNN_HF_FWD
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned)((N + 127) / 128);
    const size_t smem = (size_t)T * 128 * sizeof(float);
    auto k = pred ? (tau_pow2 ? hfam_fwd_s<true, true> : hfam_fwd_s<true, false>)
                  : (tau_pow2 ? hfam_fwd_s<false, true> : hfam_fwd_s<false, false>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, 128, smem, st>>>(a);
    return cudaGetLastError();
}

namespace {

bool fast_sg(float sg) {
    const float m = sg < 0 ? -sg : sg;
    return m >= 0x1p-60f && m <= 0x1p60f;
}

template <int HM>
cudaError_t bwd_dispatch(const HfBwd& a, bool tau_pow2, bool fsg, cudaStream_t st) {
    const int T = a.T;
    if (T == 8 || T == 16) {
        const unsigned grid = (unsigned)((a.N + 255) / 256);
#define DFSNN_HF_BWD(TV)                                                                      \
        if (T == TV) {                                                                        \
            if (tau_pow2) {                                                                   \
                if (fsg) hfam_bwd_r<HM, TV, true, true><<<grid, 256, 0, st>>>(a);             \
                else hfam_bwd_r<HM, TV, true, false><<<grid, 256, 0, st>>>(a);                \
            } else {                                                                          \
                if (fsg) hfam_bwd_r<HM, TV, false, true><<<grid, 256, 0, st>>>(a);            \
                else hfam_bwd_r<HM, TV, false, false><<<grid, 256, 0, st>>>(a);               \
            }                                                                                 \
        }
        DFSNN_HF_BWD(8) DFSNN_HF_BWD(16)
#undef DFSNN_HF_BWD
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned)((a.N + 127) / 128);
    const size_t smem = HM == kFull ? (size_t)T * 128 * sizeof(float) : 0;
    auto k = tau_pow2 ? (fsg ? hfam_bwd_s<HM, true, true> : hfam_bwd_s<HM, true, false>)
                      : (fsg ? hfam_bwd_s<HM, false, true> : hfam_bwd_s<HM, false, false>);
    if (smem > 0) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    k<<<grid, 128, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t hfam_backward_launch(int kind, bool full, const float* gS, const float* scale,
                                 float h_beta, const float* W, int B, bool per_batch,
                                 const float* vpre, float* gx, float* gv0, float* gpre, int T,
                                 long long N, float tau, float th, float sg, float rm,
                                 bool tau_pow2, cudaStream_t st) {
    if (N <= 0) return cudaSuccess;
    HfBwd a;
    a.gS = gS;
    a.vpre = vpre;
    a.tab = tables(kind == kFAGL1 ? nullptr : scale, h_beta, W, B, per_batch, N);
    a.gx = gx;
    a.gv0 = gv0;
    a.gpre = gpre;
    a.T = T;
    a.N = N;
    a.tau = tau;
    a.inv_tau = 1.0f / tau;
    a.th = th;
    a.sg = sg;
    a.rm = rm;
    const bool fsg = fast_sg(sg);
    if (kind == kVOPRED) return bwd_dispatch<kPredMode>(a, tau_pow2, fsg, st);
    if (full) return bwd_dispatch<kFull>(a, tau_pow2, fsg, st);
    return bwd_dispatch<kTrunc>(a, tau_pow2, fsg, st);
}

cudaError_t hfam_param_finalize(int kind, const double* part, int chunks, int B, bool per_batch,
                                int T, const float* W, const float* scale, double* msum,
                                float* gscale, float* gW, cudaStream_t st) {
    if (!gscale && !gW) return cudaSuccess;
    const int R = T + T * T;
    const long long units = per_batch ? B : 1;
    const long long warps = units * R;
    hfam_sum<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(part, chunks, B,
                                                                   per_batch ? 1 : 0, R, msum);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    hfam_epilogue<<<(unsigned)((units * T + 255) / 256), 256, 0, st>>>(
        kind, msum, B, per_batch ? 1 : 0, T, W, scale, gscale, gW);
    return cudaGetLastError();
}

}  // namespace dfsnn
