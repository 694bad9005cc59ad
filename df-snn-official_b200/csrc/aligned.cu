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
// per neuron-step); the backward recomputes them and reduces grad a / grad W in-kernel.
#include "kernels.h"
#include "param_reduce.cuh"

namespace dfsnn {

struct AlnArgs {
    const float* x;
    const float* v0;
    const float* a;      // [T] per-step gain (the schedule's scale)
    const float* W;      // [T, T]
    const float* g;      // [T, N] upstream grad of the spikes
    float* spike;
    float* gx;
    float* gv0;
    double* part;
    int T;
    long long N;
    float tau, inv_tau, th, sg, rho;
};

// One forward step of aligned_forward.  Returns v_t; h is the history sum.
template <int TB, bool TP2>
__device__ __forceinline__ float aligned_step(float x, float v, const float* sW, const float* sA,
                                              const float (&vh)[TB], int t, float tau, float inv_tau,
                                              float th, float& pred, bool& fire, float& h) {
    const float d = div_tau<TP2>(__fsub_rn(x, v), tau, inv_tau);
    pred = __fadd_rn(v, d);
    fire = pred >= th;
    const float spike = fire ? 1.0f : 0.0f;
    h = 0.0f;
#pragma unroll
    for (int j = 0; j < t; ++j) h = __fadd_rn(h, __fmul_rn(sW[t * TB + j], vh[j]));
    const float f = __fsub_rn(d, div_tau<TP2>(__fmul_rn(spike, th), tau, inv_tau));
    return __fsub_rn(__fmul_rn(sA[t], f), h);
}

template <int TB, bool TP2>
__global__ void __launch_bounds__(256) aln_fwd_reg(AlnArgs a) {
    __shared__ float sW[TB * TB];
    __shared__ float sA[TB];
    const int T = a.T;
    for (int e = threadIdx.x; e < T * T; e += blockDim.x) sW[(e / T) * TB + e % T] = a.W[e];
    for (int e = threadIdx.x; e < T; e += blockDim.x) sA[e] = a.a[e];
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
            float pred, h;
            bool fire;
            v = aligned_step<TB, TP2>(xr[t], v, sW, sA, vh, t, a.tau, a.inv_tau, a.th, pred, fire, h);
            vh[t] = v;
            st_stream(a.spike + t * N + n, fire ? 1.0f : 0.0f);
        }
    }
}

template <int TB, bool TP2>
__global__ void __launch_bounds__(256) aln_bwd_reg(AlnArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* sG = reinterpret_cast<float*>(smem_raw);   // adjoint r_t
    float* sV = sG + TB * kLdn;                        // v_t
    float* sE = sV + TB * kLdn;                        // r_t*(v_t+h_t)/a_t
    __shared__ float sW[TB * TB];
    __shared__ float sA[TB];
    const int T = a.T;
    const long long N = a.N;
    const int tid = threadIdx.x;
    for (int e = tid; e < TB * TB; e += blockDim.x) {
        const int t = e / TB, i = e % TB;
        sW[e] = (t < T && i < T) ? a.W[t * T + i] : 0.0f;
    }
    for (int e = tid; e < TB; e += blockDim.x) sA[e] = e < T ? a.a[e] : 1.0f;
    TileAccumulator<TB, false> acc;
    acc.init(tid);
    const long long ntiles = (N + kTile - 1) / kTile;
    const float zc = __fmul_rn(kAlignedPiHalf, a.sg);
    const float one_m = __fsub_rn(1.0f, __fdiv_rn(1.0f, a.tau));      // 1 - 1/tau
    __syncthreads();
    for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long long n = tile * kTile + tid;
        const bool live = n < N;
        float xr[TB], gr[TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            xr[t] = (live && t < T) ? ld_stream(a.x + t * N + n) : 0.0f;
            gr[t] = (live && t < T) ? ld_stream(a.g + t * N + n) : 0.0f;
        }
        float v = live ? a.v0[n] : 0.0f;
        float vh[TB], q[TB], vph[TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            if (t < T) {
                float pred, h;
                bool fire;
                v = aligned_step<TB, TP2>(xr[t], v, sW, sA, vh, t, a.tau, a.inv_tau, a.th, pred, fire, h);
                const float z = __fmul_rn(zc, __fsub_rn(pred, a.th));
                const float den = __fmul_rn(2.0f, __fadd_rn(1.0f, __fmul_rn(z, z)));
                q[t] = __fdiv_rn(__fmul_rn(gr[t], a.sg), den);
                vph[t] = __fadd_rn(v, h);
            } else {
                v = 0.0f;
                q[t] = 0.0f;
                vph[t] = 0.0f;
            }
            if (!live) v = 0.0f;
            vh[t] = v;
            sV[t * kLdn + tid] = v;
        }
        float A[TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) A[t] = 0.0f;
#pragma unroll
        for (int t = TB - 1; t >= 0; --t) {
            float r = 0.0f, e = 0.0f;
            if (t < T) {
                r = A[t];
                const float ra = __fmul_rn(r, sA[t]);
                if (live) st_stream(a.gx + t * N + n, div_tau<TP2>(__fadd_rn(q[t], ra), a.tau, a.inv_tau));
                const float prev = __fsub_rn(__fmul_rn(q[t], one_m), div_tau<TP2>(ra, a.tau, a.inv_tau));
                if (t) A[t - 1] = __fadd_rn(A[t - 1], prev);
                else if (live) a.gv0[n] = prev;
#pragma unroll
                for (int j = 0; j < t; ++j) A[j] = __fsub_rn(A[j], __fmul_rn(__fmul_rn(a.rho, sW[t * TB + j]), r));
                e = __fdiv_rn(__fmul_rn(r, vph[t]), sA[t]);
            }
            if (!live) { r = 0.0f; e = 0.0f; }
            sG[t * kLdn + tid] = r;
            sE[t * kLdn + tid] = e;
        }
        __syncthreads();
        acc.accumulate(sG, sV, sE);
        __syncthreads();
    }
    acc.finish(reinterpret_cast<double*>(smem_raw), a.part + (size_t)blockIdx.x * ProdCfg<TB>::NOUT, tid);
}

namespace {

template <int TB>
size_t aln_smem() {
    const size_t stage = ProdCfg<TB>::SMEM_BYTES;
    const size_t red = size_t(kTile) * 20 * sizeof(double);
    return stage > red ? stage : red;
}

template <int TB, bool TP2>
int aln_grid_t(long long N) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = aln_smem<TB>();
    cudaFuncSetAttribute(aln_bwd_reg<TB, TP2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, aln_bwd_reg<TB, TP2>, kTile, smem);
    if (per < 1) per = 1;
    const long long ntiles = (N + kTile - 1) / kTile;
    long long g = (long long)sms * per;
    if (g > ntiles) g = ntiles;
    return g < 1 ? 1 : (int)g;
}

template <int TB, bool TP2>
cudaError_t aln_bwd_launch_t(const AlnArgs& a, int grid, cudaStream_t st) {
    const size_t smem = aln_smem<TB>();
    cudaError_t e = cudaFuncSetAttribute(aln_bwd_reg<TB, TP2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    aln_bwd_reg<TB, TP2><<<grid, kTile, smem, st>>>(a);
    return cudaGetLastError();
}

int tb_of(int T) { return T <= 8 ? 8 : (T <= 16 ? 16 : 32); }

}  // namespace

int aligned_bwd_blocks(int T, long long N, bool tau_pow2) {
    const int TB = tb_of(T);
    if (TB == 8) return tau_pow2 ? aln_grid_t<8, true>(N) : aln_grid_t<8, false>(N);
    if (TB == 16) return tau_pow2 ? aln_grid_t<16, true>(N) : aln_grid_t<16, false>(N);
    return tau_pow2 ? aln_grid_t<32, true>(N) : aln_grid_t<32, false>(N);
}

int aligned_part_stride(int T) {
    const int TB = tb_of(T);
    return TB + TB * TB;
}

cudaError_t aligned_forward_launch(const float* x, const float* v0, const float* a_,
                                   const float* W, float* spike, int T, long long N, float tau,
                                   float th, bool tau_pow2, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    AlnArgs a{};
    a.x = x; a.v0 = v0; a.a = a_; a.W = W; a.spike = spike; a.T = T; a.N = N; a.tau = tau;
    a.inv_tau = 1.0f / tau; a.th = th;
    const unsigned grid = (unsigned)((N + 255) / 256);
    const int TB = tb_of(T);
#define DFSNN_AF(TBV)                                                    \
    if (TB == TBV) {                                                     \
        if (tau_pow2) aln_fwd_reg<TBV, true><<<grid, 256, 0, st>>>(a);   \
        else aln_fwd_reg<TBV, false><<<grid, 256, 0, st>>>(a);           \
    }
    DFSNN_AF(8) DFSNN_AF(16) DFSNN_AF(32)
#undef DFSNN_AF
    return cudaGetLastError();
}

cudaError_t aligned_backward_launch(const float* g, const float* x, const float* v0,
                                    const float* a_, const float* W, float* gx, float* gv0,
                                    float* ga, float* gW, int T, long long N, float tau, float th,
                                    float sg, float rho, bool tau_pow2, double* part, int nblocks,
                                    cudaStream_t st) {
    AlnArgs a{};
    a.x = x; a.v0 = v0; a.a = a_; a.W = W; a.g = g; a.gx = gx; a.gv0 = gv0; a.part = part;
    a.T = T; a.N = N; a.tau = tau; a.inv_tau = 1.0f / tau; a.th = th; a.sg = sg; a.rho = rho;
    const int TB = tb_of(T);
    cudaError_t e = cudaSuccess;
#define DFSNN_AB(TBV)                                                                         \
    if (TB == TBV) e = tau_pow2 ? aln_bwd_launch_t<TBV, true>(a, nblocks, st)                 \
                                : aln_bwd_launch_t<TBV, false>(a, nblocks, st);
    DFSNN_AB(8) DFSNN_AB(16) DFSNN_AB(32)
#undef DFSNN_AB
    if (e != cudaSuccess) return e;
    if (ga || gW) {
        const int nout = T + T * T;
        param_finalize<<<(nout + 127) / 128, 128, 0, st>>>(part, nblocks, TB, T, ga, gW, 1);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace dfsnn
