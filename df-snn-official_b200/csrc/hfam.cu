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
// (VO-PREDICTOR: grad_v_next = gp*(rm - s/tau)), writing grad_x and grad_v0.  The parameter
// gradients are reductions of grad_pre against the saved history: for T = 8 and 16 inside
// the sweep kernel (hfam_bwd_f, grad_pre never stored), otherwise by param_long.cu over the
// grad_pre [T, N] the sweep writes; hfam_sum + hfam_epilogue finish both.
#include "kernels.h"
#include "lif_common.cuh"
#include "mma_tf32.cuh"

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

// ---- T = 8 and 16: the reverse sweep and the parameter products in one kernel ----------
// One block per partial row s = b*chunks + c (segment c of sample b, the rows param_small
// writes), eight warps taking 32-neuron tiles of the segment in turn, one neuron per lane.
// A lane runs the reverse sweep of hfam_bwd_s on its neuron, with the inputs and (full
// history) adjoints in registers, writes grad_x and grad_v0 and keeps grad_pre in registers; when parameter gradients are wanted it writes grad_pre and
// the saved history values of its neuron as column `lane` of the warp's padded GP / V rows
// and the warp adds the tile's P[t][i] = sum_n GP[t,n] V[i,n] on the tensor pipe (3xTF32,
// as warp_tile.cuh); VO-GL1's diagonal sum_n grad_pre[t,n] drift[t,n] is a per-lane fp32
// sum.  grad_pre never goes to global memory, which saves writing and reading back
// 8 bytes per neuron-step.  Rows reduce in double in a fixed order (deterministic).
template <int TT>
struct HfFusedCfg {
    static constexpr int kWarps = 8;
    static constexpr int TN = 32;                     // neurons per warp tile
    static constexpr int RS = 40;                     // row stride: 8 banks apart
    static constexpr int NT = TT / 8;                 // mma n-tiles of 8 output columns
    static constexpr int NACC = 4 * NT;               // product accumulators per lane
    static constexpr int NRED = NACC + TT;            // doubles per thread in the reduction
    static constexpr int PER_WARP = 2 * TT * RS;      // GP rows, V rows
    static constexpr size_t kTiles = sizeof(float) * kWarps * PER_WARP;
    static constexpr size_t kRed = sizeof(double) * 32 * kWarps * NRED;
    static constexpr size_t kBytes = kTiles > kRed ? kTiles : kRed;
    static_assert(TT == 8 || TT == 16, "fused history backward covers T = 8 and T = 16");
    static_assert(RS % 32 == 8, "fragment loads are conflict-free for rows 8 banks apart");
};

// acc[4*nt + e] += sum over the tile's 32 columns of GP[t] * V[i], fragment entry e of
// n-tile nt: t = g + 8*(e >= 2), i = 8*nt + 2c + (e & 1) (g = lane / 4, c = lane % 4)
template <int TT>
__device__ __forceinline__ void hf_tile_product(const float* GP, const float* Vs, int lane,
                                                float (&acc)[HfFusedCfg<TT>::NACC]) {
    using C = HfFusedCfg<TT>;
    constexpr int RS = C::RS;
    const int g = lane >> 2, c = lane & 3;
    float d[C::NT][4];
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[nt][e] = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < C::TN; k0 += 8) {
        const float2 ar0 = *reinterpret_cast<const float2*>(GP + g * RS + k0 + 2 * c);
        uint32_t ah[4], al[4];
        split_tf32(ar0.x, ah[0], al[0]);
        split_tf32(ar0.y, ah[2], al[2]);
        if constexpr (TT == 16) {
            const float2 ar1 = *reinterpret_cast<const float2*>(GP + (g + 8) * RS + k0 + 2 * c);
            split_tf32(ar1.x, ah[1], al[1]);
            split_tf32(ar1.y, ah[3], al[3]);
        } else {
            ah[1] = al[1] = ah[3] = al[3] = 0u;
        }
#pragma unroll
        for (int nt = 0; nt < C::NT; ++nt) {
            const float2 br = *reinterpret_cast<const float2*>(Vs + (8 * nt + g) * RS + k0 + 2 * c);
            uint32_t bh0, bl0, bh1, bl1;
            split_tf32(br.x, bh0, bl0);
            split_tf32(br.y, bh1, bl1);
            mma_tf32(d[nt], al[0], al[1], al[2], al[3], bh0, bh1);
            mma_tf32(d[nt], ah[0], ah[1], ah[2], ah[3], bl0, bl1);
            mma_tf32(d[nt], ah[0], ah[1], ah[2], ah[3], bh0, bh1);
        }
    }
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[4 * nt + e] = __fadd_rn(acc[4 * nt + e], d[nt][e]);
}

struct HfFusedOut {
    const float* V;       // saved history sequence paired with grad_pre (NULL: no products)
    const float* E;       // drift for VO-GL1's grad_scale (NULL: no diagonal)
    double* part;         // partial rows [B*chunks][T + T*T]
    int chunks;
    long long per;        // neurons per segment
};

template <int HM, int TT, bool TAU_POW2, bool FAST_SG>
__global__ void __launch_bounds__(256, 3) hfam_bwd_f(HfBwd a, HfFusedOut o) {
    using C = HfFusedCfg<TT>;
    constexpr int RS = C::RS;
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float* GP = reinterpret_cast<float*>(smem) + warp * C::PER_WARP;
    float* Vs = GP + TT * RS;
    const long long N = a.N, F = a.tab.F;
    const int b = blockIdx.x / o.chunks, c = blockIdx.x % o.chunks;
    const long long nb = (long long)b * F + (long long)c * o.per;
    const long long send = (long long)b * F + F;
    const long long ne = nb + o.per < send ? nb + o.per : send;
    const bool prod = o.V != nullptr, diag = o.E != nullptr;
    float acc[C::NACC], gsd[TT];
#pragma unroll
    for (int e = 0; e < C::NACC; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int t = 0; t < TT; ++t) gsd[t] = 0.0f;
    for (long long n0 = nb + (long long)warp * C::TN; n0 < ne; n0 += (long long)C::kWarps * C::TN) {
        const long long n = n0 + lane;
        const bool on = n < ne;
        float gp[TT];
        if (on) {
            float pr[TT];
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                gp[t] = ld_stream(a.gS + (long long)t * N + n);      // grad_spike, then grad_pre
                pr[t] = ld_stream(a.vpre + (long long)t * N + n);
            }
            float A[HM == kFull ? TT : 1];
#pragma unroll
            for (int t = 0; t < (HM == kFull ? TT : 1); ++t) A[t] = 0.0f;
            float gvn = 0.0f, ginit = 0.0f;
#pragma unroll
            for (int t = TT - 1; t >= 0; --t) {
                const float sur = surr<FAST_SG>(__fsub_rn(pr[t], a.th), a.sg);
                const float g = HM == kFull ? __fmaf_rn(gp[t], sur, A[t])
                                            : __fmaf_rn(gp[t], sur, gvn);
                gp[t] = g;
                const float sv = a.tab.s(t, b);
                const float* w = a.tab.wrow(t, b, TT);
                st_stream(a.gx + (long long)t * N + n,
                          div_tau<TAU_POW2>(__fmul_rn(g, sv), a.tau, a.inv_tau));
                if constexpr (HM == kFull) {
                    const float prev = div_tau<TAU_POW2>(__fmul_rn(-g, sv), a.tau, a.inv_tau);
                    if (t == 0) ginit = __fadd_rn(ginit, prev);
                    else A[t > 0 ? t - 1 : 0] = __fadd_rn(A[t > 0 ? t - 1 : 0], prev);
#pragma unroll
                    for (int i = 0; i < t; ++i) A[i] = __fmaf_rn(-__ldg(w + i), g, A[i]);
                } else {
                    gvn = trunc_next<HM, TAU_POW2>(a, w, t, g, sv);
                }
            }
            a.gv0[n] = HM == kFull ? ginit : gvn;
        } else {
#pragma unroll
            for (int t = 0; t < TT; ++t) gp[t] = 0.0f;
        }
        if (prod) {
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                GP[t * RS + lane] = gp[t];
                Vs[t * RS + lane] = on ? ld_stream(o.V + (long long)t * N + n) : 0.0f;
            }
            if (diag && on) {
#pragma unroll
                for (int t = 0; t < TT; ++t)
                    gsd[t] = __fmaf_rn(gp[t], ld_stream(o.E + (long long)t * N + n), gsd[t]);
            }
            __syncwarp();
            hf_tile_product<TT>(GP, Vs, lane, acc);
            __syncwarp();                             // the rows are rewritten by the next tile
        }
    }
    if (!prod) return;                                // uniform: no block barrier follows
    __syncthreads();                                  // every warp is done with its rows
    double* red = reinterpret_cast<double*>(smem);
    double* mine = red + (size_t)tid * C::NRED;
#pragma unroll
    for (int e = 0; e < C::NACC; ++e) mine[e] = (double)acc[e];
#pragma unroll
    for (int t = 0; t < TT; ++t) mine[C::NACC + t] = (double)gsd[t];
    __syncthreads();
    double* row = o.part + (size_t)blockIdx.x * (TT + TT * TT);
    for (int q = tid; q < TT + TT * TT; q += blockDim.x) {
        double sum = 0.0;
        if (q < TT) {
            if (diag)
                for (int r = 0; r < C::kWarps * 32; ++r) sum += red[(size_t)r * C::NRED + C::NACC + q];
        } else {
            const int t = (q - TT) / TT, i = (q - TT) % TT;
            const int ln = 4 * (t & 7) + ((i & 7) >> 1);
            const int slot = 4 * (i >> 3) + (t >= 8 ? 2 : 0) + (i & 1);
            for (int w = 0; w < C::kWarps; ++w) sum += red[(size_t)(w * 32 + ln) * C::NRED + slot];
        }
        row[q] = sum;
    }
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
cudaError_t bwd_dispatch(const HfBwd& a, const HfFusedOut& o, int B, bool tau_pow2, bool fsg,
                         cudaStream_t st) {
    const int T = a.T;
    if (hfam_backward_fused(T)) {
        const unsigned grid = (unsigned)((long long)B * o.chunks);
#define DFSNN_HF_BWD(TV, P2, FS)                                                              \
        if (T == TV && tau_pow2 == P2 && fsg == FS) {                                         \
            auto k = hfam_bwd_f<HM, TV, P2, FS>;                                              \
            const int bytes = (int)HfFusedCfg<TV>::kBytes;                                    \
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes); \
            if (e != cudaSuccess) return e;                                                   \
            k<<<grid, 256, bytes, st>>>(a, o);                                                \
            return cudaGetLastError();                                                        \
        }
        DFSNN_HF_BWD(8, true, true) DFSNN_HF_BWD(8, true, false)
        DFSNN_HF_BWD(8, false, true) DFSNN_HF_BWD(8, false, false)
        DFSNN_HF_BWD(16, true, true) DFSNN_HF_BWD(16, true, false)
        DFSNN_HF_BWD(16, false, true) DFSNN_HF_BWD(16, false, false)
#undef DFSNN_HF_BWD
        return cudaErrorInvalidValue;
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

bool hfam_backward_fused(int T) { return T == 8 || T == 16; }

cudaError_t hfam_backward_launch(int kind, bool full, const float* gS, const float* scale,
                                 float h_beta, const float* W, int B, bool per_batch,
                                 const float* vpre, float* gx, float* gv0, float* gpre,
                                 const float* V, const float* E, double* part, int chunks, int T,
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
    HfFusedOut o;
    o.V = V;
    o.E = V ? E : nullptr;
    o.part = part;
    o.chunks = chunks < 1 ? 1 : chunks;
    const long long F = N / B;
    o.per = (F + o.chunks - 1) / o.chunks;
    const bool fsg = fast_sg(sg);
    if (kind == kVOPRED) return bwd_dispatch<kPredMode>(a, o, B, tau_pow2, fsg, st);
    if (full) return bwd_dispatch<kFull>(a, o, B, tau_pow2, fsg, st);
    return bwd_dispatch<kTrunc>(a, o, B, tau_pow2, fsg, st);
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
