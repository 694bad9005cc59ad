// glmulti.cu -- library distributed-order GL ("glmulti") LIF kernels for sm_100a.
//
// Replaces LIFFDEGLMultiFunction (spikeDE_dis/fde_cupy_kernels_all.py:1916-2011):
//   forward  = lif_fde_vo_gl1_forward_kernel with per_batch=0 (:1594-1630)
//   backward = lif_fde_glmulti_backward_kernel (:1845-1875, truncated history) or
//              lif_fde_glmulti_full_backward_kernel (:1877-1913, full history adjoint),
//              followed by grad_scale = sum(grad_pre*drift) and grad_W = -grad_pre@v_hist^T.
// Design (B200): the forward writes only the spikes (8 B per neuron-step instead of the
// reference's 20 B: spike, v_pre, v_hist, drift).  The backward re-reads x and recomputes
// the trajectory in registers (T <= 32) or shared memory (T <= 256), runs the reverse
// sweep, and reduces grad_scale / grad_W inside the same persistent kernel, so neither
// grad_pre nor v_hist nor drift ever reaches HBM.
#include "kernels.h"
#include "param_reduce.cuh"

namespace dfsnn {

struct GlmArgs {
    const float* x;       // [T, N]
    const float* v0;      // [N]
    const float* scale;   // [T]
    const float* W;       // [T, T]
    const float* gS;      // [T, N] upstream grad of the spikes (backward)
    float* spike;         // [T, N] (forward)
    float* gx;            // [T, N] (backward)
    float* gv0;           // [N]    (backward)
    double* part;         // [gridDim.x, TB + TB*TB] (backward)
    int T;
    long long N;
    float tau, inv_tau, th, sg;
};

// ------------------------------------------------------------------------------------
// forward, T <= TB <= 32: history in registers
// ------------------------------------------------------------------------------------
template <int TB, bool TP2>
__global__ void __launch_bounds__(256) glm_fwd_reg(GlmArgs a) {
    __shared__ float sW[TB * TB];
    __shared__ float sScale[TB];
    const int T = a.T;
    for (int e = threadIdx.x; e < T * T; e += blockDim.x) sW[(e / T) * TB + e % T] = a.W[e];
    for (int e = threadIdx.x; e < T; e += blockDim.x) sScale[e] = a.scale[e];
    __syncthreads();
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    float xr[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t)
        if (t < T) xr[t] = ld_stream(a.x + t * N + n);
    float v = a.v0[n];
    float vh[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        if (t < T) {
            const float d = div_tau<TP2>(__fsub_rn(xr[t], v), a.tau, a.inv_tau);
            float hist = 0.0f;
#pragma unroll
            for (int i = 0; i < t; ++i) hist = __fmaf_rn(sW[t * TB + i], vh[i], hist);
            const float p = __fmaf_rn(sScale[t], d, -hist);
            const float s = (p >= a.th) ? 1.0f : 0.0f;
            v = __fsub_rn(p, s * a.th);
            vh[t] = v;
            st_stream(a.spike + t * N + n, s);
        }
    }
}

// ------------------------------------------------------------------------------------
// forward, any T: history in shared memory [T][blockDim]
// ------------------------------------------------------------------------------------
template <bool TP2>
__global__ void __launch_bounds__(128) glm_fwd_smem(GlmArgs a) {
    extern __shared__ float sh[];
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const int T = a.T;
    float* vh = sh + threadIdx.x;
    const int st = blockDim.x;
    float v = a.v0[n];
    float xn = ld_stream(a.x + n);
    for (int t = 0; t < T; ++t) {
        const float xt = xn;
        if (t + 1 < T) xn = ld_stream(a.x + (t + 1) * N + n);
        const float d = div_tau<TP2>(__fsub_rn(xt, v), a.tau, a.inv_tau);
        const float* wrow = a.W + (size_t)t * T;
        float hist = 0.0f;
        for (int i = 0; i < t; ++i) hist = __fmaf_rn(__ldg(wrow + i), vh[i * st], hist);
        const float p = __fmaf_rn(__ldg(a.scale + t), d, -hist);
        const float s = (p >= a.th) ? 1.0f : 0.0f;
        v = __fsub_rn(p, s * a.th);
        vh[t * st] = v;
        st_stream(a.spike + t * N + n, s);
    }
}

// ------------------------------------------------------------------------------------
// backward, T <= TB <= 32: persistent, trajectory in registers, fused parameter grads
// ------------------------------------------------------------------------------------
template <int TB, bool FULL, bool TP2>
__global__ void __launch_bounds__(256) glm_bwd_reg(GlmArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* sG = reinterpret_cast<float*>(smem_raw);
    float* sV = sG + TB * kLdn;
    float* sD = sV + TB * kLdn;
    __shared__ float sW[TB * TB];
    __shared__ float sScale[TB];
    const int T = a.T;
    const long long N = a.N;
    const int tid = threadIdx.x;
    for (int e = tid; e < TB * TB; e += blockDim.x) {
        const int t = e / TB, i = e % TB;
        sW[e] = (t < T && i < T) ? a.W[t * T + i] : 0.0f;
    }
    for (int e = tid; e < TB; e += blockDim.x) sScale[e] = e < T ? a.scale[e] : 0.0f;
    TileAccumulator<TB, true> acc;
    acc.init(tid);
    const long long ntiles = (a.N + kTile - 1) / kTile;
    __syncthreads();
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long long n = tile * kTile + tid;
        const bool live = n < N;
        float xr[TB], gs[TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            xr[t] = (live && t < T) ? ld_stream(a.x + t * N + n) : 0.0f;
            gs[t] = (live && t < T) ? ld_stream(a.gS + t * N + n) : 0.0f;
        }
        // forward recompute (bit-identical to the forward kernel)
        float v = live ? a.v0[n] : 0.0f;
        float vh[TB], sur[TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            float d = 0.0f;
            if (t < T) {
                d = div_tau<TP2>(__fsub_rn(xr[t], v), a.tau, a.inv_tau);
                float hist = 0.0f;
#pragma unroll
                for (int i = 0; i < t; ++i) hist = __fmaf_rn(sW[t * TB + i], vh[i], hist);
                const float p = __fmaf_rn(sScale[t], d, -hist);
                const float s = (p >= a.th) ? 1.0f : 0.0f;
                v = __fsub_rn(p, s * a.th);
                sur[t] = surrogate_fma(__fsub_rn(p, a.th), a.sg);
            } else {
                v = 0.0f;
                sur[t] = 0.0f;
            }
            if (!live) { v = 0.0f; d = 0.0f; }
            vh[t] = v;
            sV[t * kLdn + tid] = v;
            sD[t * kLdn + tid] = d;
        }
        // reverse sweep
        if constexpr (FULL) {
            float A[TB];
#pragma unroll
            for (int t = 0; t < TB; ++t) A[t] = 0.0f;
            float ginit = 0.0f;
#pragma unroll
            for (int t = TB - 1; t >= 0; --t) {
                float gp = 0.0f;
                if (t < T) {
                    gp = __fmaf_rn(gs[t], sur[t], A[t]);
                    const float gd = __fmul_rn(gp, sScale[t]);
                    if (live) st_stream(a.gx + t * N + n, div_tau<TP2>(gd, a.tau, a.inv_tau));
                    const float prev = div_tau<TP2>(-gd, a.tau, a.inv_tau);
                    if (t == 0) ginit = __fadd_rn(ginit, prev);
                    else A[t - 1] = __fadd_rn(A[t - 1], prev);
#pragma unroll
                    for (int i = 0; i < t; ++i) A[i] = __fmaf_rn(-sW[t * TB + i], gp, A[i]);
                }
                if (!live) gp = 0.0f;
                sG[t * kLdn + tid] = gp;
            }
            if (live) a.gv0[n] = ginit;
        } else {
            float gvn = 0.0f;
#pragma unroll
            for (int t = TB - 1; t >= 0; --t) {
                float gp = 0.0f;
                if (t < T) {
                    gp = __fmaf_rn(gs[t], sur[t], gvn);
                    if (live)
                        st_stream(a.gx + t * N + n,
                                  div_tau<TP2>(__fmul_rn(gp, sScale[t]), a.tau, a.inv_tau));
                    gvn = div_tau<TP2>(__fmul_rn(-gp, sScale[t]), a.tau, a.inv_tau);
                }
                if (!live) gp = 0.0f;
                sG[t * kLdn + tid] = gp;
            }
            if (live) a.gv0[n] = gvn;
        }
        __syncthreads();
        acc.accumulate(sG, sV, sD);
        __syncthreads();
    }
    acc.finish(reinterpret_cast<double*>(smem_raw), a.part + (size_t)blockIdx.x * ProdCfg<TB>::NOUT, tid);
}

// ------------------------------------------------------------------------------------
// sum the per-block partials in a fixed order: gs (T) and gW (T x T, negated)
// ------------------------------------------------------------------------------------
__global__ void param_finalize(const double* part, int nblocks, int TB, int T, float* gscale,
                               float* gW, int lower_only) {
    const int nout = TB + TB * TB;
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= T + T * T) return;
    int src;
    if (o < T) src = o;
    else {
        const int t = (o - T) / T, i = (o - T) % T;
        src = TB + t * TB + i;
    }
    double s = 0.0;
    for (int b = 0; b < nblocks; ++b) s += part[(size_t)b * nout + src];
    if (o < T) {
        if (gscale) gscale[o] = (float)s;
    } else if (gW) {
        const int t = (o - T) / T, i = (o - T) % T;
        gW[o - T] = (lower_only && i >= t) ? 0.0f : (float)(-s);
    }
}

// ------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------
namespace {

int tb_bucket(int T) { return T <= 8 ? 8 : (T <= 16 ? 16 : 32); }

template <int TB, bool FULL, bool TP2>
size_t bwd_reg_smem() {
    const size_t stage = ProdCfg<TB>::SMEM_BYTES;
    const size_t red = size_t(kTile) * 20 * sizeof(double);
    return stage > red ? stage : red;
}

template <int TB, bool FULL, bool TP2>
cudaError_t launch_bwd_reg(const GlmArgs& a, int grid, cudaStream_t st) {
    const size_t smem = bwd_reg_smem<TB, FULL, TP2>();
    auto k = glm_bwd_reg<TB, FULL, TP2>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<grid, kTile, smem, st>>>(a);
    return cudaGetLastError();
}

template <int TB, bool TP2>
int bwd_reg_grid_t(long long N, bool full) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = bwd_reg_smem<TB, true, TP2>();
    if (full) {
        cudaFuncSetAttribute(glm_bwd_reg<TB, true, TP2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, glm_bwd_reg<TB, true, TP2>, kTile, smem);
    } else {
        cudaFuncSetAttribute(glm_bwd_reg<TB, false, TP2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, glm_bwd_reg<TB, false, TP2>, kTile, smem);
    }
    if (per < 1) per = 1;
    const long long ntiles = (N + kTile - 1) / kTile;
    long long g = (long long)sms * per;
    if (g > ntiles) g = ntiles;
    return g < 1 ? 1 : (int)g;
}

}  // namespace

int glmulti_bwd_blocks(int T, long long N, bool full, bool tau_pow2) {
    const int TB = tb_bucket(T);
    if (TB == 8) return tau_pow2 ? bwd_reg_grid_t<8, true>(N, full) : bwd_reg_grid_t<8, false>(N, full);
    if (TB == 16) return tau_pow2 ? bwd_reg_grid_t<16, true>(N, full) : bwd_reg_grid_t<16, false>(N, full);
    return tau_pow2 ? bwd_reg_grid_t<32, true>(N, full) : bwd_reg_grid_t<32, false>(N, full);
}

int glmulti_part_stride(int T) {
    const int TB = tb_bucket(T);
    return TB + TB * TB;
}

cudaError_t glmulti_forward_launch(const float* x, const float* v0, const float* scale,
                                   const float* W, float* spike, int T, long long N, float tau,
                                   float th, bool tau_pow2, cudaStream_t st) {
    GlmArgs a{};
    a.x = x; a.v0 = v0; a.scale = scale; a.W = W; a.spike = spike;
    a.T = T; a.N = N; a.tau = tau; a.inv_tau = 1.0f / tau; a.th = th;
    if (N == 0) return cudaSuccess;
    if (T <= 32) {
        const unsigned grid = (unsigned)((N + 255) / 256);
        const int TB = tb_bucket(T);
#define DFSNN_FWD(TBV)                                                        \
    if (TB == TBV) {                                                          \
        if (tau_pow2) glm_fwd_reg<TBV, true><<<grid, 256, 0, st>>>(a);        \
        else glm_fwd_reg<TBV, false><<<grid, 256, 0, st>>>(a);                \
    }
        DFSNN_FWD(8) DFSNN_FWD(16) DFSNN_FWD(32)
#undef DFSNN_FWD
        return cudaGetLastError();
    }
    const unsigned grid = (unsigned)((N + 127) / 128);
    const size_t smem = sizeof(float) * (size_t)T * 128;
    cudaError_t e;
    if (tau_pow2) {
        e = cudaFuncSetAttribute(glm_fwd_smem<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        glm_fwd_smem<true><<<grid, 128, smem, st>>>(a);
    } else {
        e = cudaFuncSetAttribute(glm_fwd_smem<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        glm_fwd_smem<false><<<grid, 128, smem, st>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t glmulti_backward_launch(const float* gS, const float* x, const float* v0,
                                    const float* scale, const float* W, float* gx, float* gv0,
                                    float* gscale, float* gW, int T, long long N, float tau,
                                    float th, float sg, bool full, bool tau_pow2, double* part,
                                    int nblocks, cudaStream_t st) {
    GlmArgs a{};
    a.x = x; a.v0 = v0; a.scale = scale; a.W = W; a.gS = gS; a.gx = gx; a.gv0 = gv0;
    a.part = part; a.T = T; a.N = N; a.tau = tau; a.inv_tau = 1.0f / tau; a.th = th; a.sg = sg;
    cudaError_t e = cudaSuccess;
    const int TB = tb_bucket(T);
#define DFSNN_BWD(TBV)                                                                       \
    if (TB == TBV) {                                                                         \
        if (full) e = tau_pow2 ? launch_bwd_reg<TBV, true, true>(a, nblocks, st)             \
                               : launch_bwd_reg<TBV, true, false>(a, nblocks, st);           \
        else e = tau_pow2 ? launch_bwd_reg<TBV, false, true>(a, nblocks, st)                 \
                          : launch_bwd_reg<TBV, false, false>(a, nblocks, st);               \
    }
    DFSNN_BWD(8) DFSNN_BWD(16) DFSNN_BWD(32)
#undef DFSNN_BWD
    if (e != cudaSuccess) return e;
    if (gscale || gW) {
        const int nout = T + T * T;
        param_finalize<<<(nout + 127) / 128, 128, 0, st>>>(part, nblocks, TB, T, gscale, gW, 0);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace dfsnn
