// direct_euler.cu -- LIF-like direct Euler neuron kernels for sm_100a.
//
// Replaces DirectLIFLikeEulerCuPyFunction (spikeDE_dis/direct_euler_cupy.py:140-253):
//   forward  direct_lif_euler_forward  (:22-58)
//   backward direct_lif_euler_backward (:66-131)
// Differences by design:
//   * the forward writes only spike and z_final; the backward recomputes z_pre and the
//     spike input from x (the reference stores both, 8 extra bytes per neuron-step), using
//     one checkpoint of z per 32-step segment;
//   * the three scalar gradients (input scale, spike gain, spike bias) are reduced per
//     block and then summed in a fixed order, instead of three atomicAdds per thread;
//   * the learnable scalars are read from device memory, so no host synchronisation.
#include "kernels.h"
#include "lif_common.cuh"

namespace dfsnn {

struct EulerArgs {
    const float* x;
    const float* z0;
    const float* in_scale;   // device scalars
    const float* gain;
    const float* bias;
    float* spike;
    float* zfinal;
    const float* gS;
    const float* gzf;        // may be null
    float* gx;
    float* gz0;
    double* part;            // [gridDim.x, 3]
    int T;
    long long N;
    float tau, th, step, reset_strength, sg, sdt;
};

struct EulerStep {
    float z, si;
};

// One forward step (direct_euler_cupy.py:47-55).  Returns the next z; z_pre = z, s_in.
__device__ __forceinline__ float euler_step(float z, float cur, float sc, float gain, float bias,
                                            const EulerArgs& a, float& si, float& s) {
    const float dz = __fdiv_rn(__fmaf_rn(cur, sc, -z), a.tau);         // (-z + cur*scale)/tau
    const float sv = __fmaf_rn(a.sdt, dz, z);                          // z + dt*dz
    si = __fsub_rn(__fmaf_rn(sv, gain, bias), a.th);                   // sv*gain + bias - th
    s = si >= 0.0f ? 1.0f : 0.0f;
    const float rs = __fdiv_rn(__fmul_rn(__fmul_rn(a.reset_strength, s), a.th), a.tau);
    return __fmaf_rn(a.step, __fsub_rn(dz, rs), z);                    // z + step*(dz - rs)
}

__global__ void __launch_bounds__(256) euler_fwd(EulerArgs a) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.N) return;
    const long long N = a.N;
    const float sc = __ldg(a.in_scale), gain = __ldg(a.gain), bias = __ldg(a.bias);
    float z = a.z0[n];
    float xn = ld_stream(a.x + n);
    for (int t = 0; t < a.T; ++t) {
        const float cur = xn;
        if (t + 1 < a.T) xn = ld_stream(a.x + (t + 1) * N + n);
        float si, s;
        z = euler_step(z, cur, sc, gain, bias, a, si, s);
        st_stream(a.spike + t * N + n, s);
    }
    a.zfinal[n] = z;
}

constexpr int kSeg = 32;
constexpr int kMaxSeg = 32;   // T <= 1024

__global__ void __launch_bounds__(256) euler_bwd(EulerArgs a) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = n < a.N;
    const long long N = a.N;
    const int T = a.T;
    const float sc = __ldg(a.in_scale), gain = __ldg(a.gain);
    const float bias = __ldg(a.bias);
    float ls = 0.0f, lg = 0.0f, lb = 0.0f;
    if (live) {
        const int nseg = (T + kSeg - 1) / kSeg;
        float ck[kMaxSeg];
        float z = a.z0[n];
        for (int sgi = 0; sgi < nseg; ++sgi) {
            ck[sgi] = z;
            const int t1 = min(T, (sgi + 1) * kSeg);
            for (int t = sgi * kSeg; t < t1; ++t) {
                float si, s;
                z = euler_step(z, ld_stream(a.x + t * N + n), sc, gain, bias, a, si, s);
            }
        }
        // reverse sweep (direct_euler_cupy.py:94-124)
        const float dz_dz = __fdiv_rn(-1.0f, a.tau);
        const float dz_dx = __fdiv_rn(sc, a.tau);
        const float sv_dz = __fmaf_rn(a.sdt, dz_dz, 1.0f);
        const float sv_dx = __fmul_rn(a.sdt, dz_dx);
        const float one_m = __fsub_rn(1.0f, __fdiv_rn(a.step, a.tau));
        const float step_dx = __fmul_rn(a.step, dz_dx);
        float gzn = a.gzf ? a.gzf[n] : 0.0f;
        for (int sgi = nseg - 1; sgi >= 0; --sgi) {
            const int t0 = sgi * kSeg;
            const int len = min(kSeg, T - t0);
            float zp[kSeg], sin_[kSeg], xs[kSeg];
            float zz = ck[sgi];
#pragma unroll
            for (int j = 0; j < kSeg; ++j) {
                if (j < len) {
                    xs[j] = ld_stream(a.x + (t0 + j) * N + n);
                    zp[j] = zz;
                    float s;
                    zz = euler_step(zz, xs[j], sc, gain, bias, a, sin_[j], s);
                }
            }
#pragma unroll
            for (int j = kSeg - 1; j >= 0; --j) {
                if (j < len) {
                    const int t = t0 + j;
                    const float cur = xs[j];
                    const float dz_ds = __fdiv_rn(cur, a.tau);
                    const float sv_ds = __fmul_rn(a.sdt, dz_ds);
                    const float sv = __fmaf_rn(zp[j], sv_dz, __fmul_rn(cur, sv_dx));
                    const float surr = surrogate_fma(sin_[j], a.sg);
                    const float gsi = __fmul_rn(ld_stream(a.gS + t * N + n), surr);
                    lg = __fmaf_rn(gsi, sv, lg);
                    lb = __fadd_rn(lb, gsi);
                    const float gsv = __fmul_rn(gsi, gain);
                    const float gz = __fmaf_rn(gzn, one_m, __fmul_rn(gsv, sv_dz));
                    st_stream(a.gx + t * N + n, __fmaf_rn(gzn, step_dx, __fmul_rn(gsv, sv_dx)));
                    ls = __fadd_rn(ls, __fmaf_rn(gzn, __fmul_rn(a.step, dz_ds), __fmul_rn(gsv, sv_ds)));
                    gzn = gz;
                }
            }
        }
        a.gz0[n] = gzn;
    }
    // block reduction of the three scalars (double), fixed order
    __shared__ double red[3][256 / 32];
    double d0 = ls, d1 = lg, d2 = lb;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        d0 += __shfl_down_sync(0xffffffffu, d0, off);
        d1 += __shfl_down_sync(0xffffffffu, d1, off);
        d2 += __shfl_down_sync(0xffffffffu, d2, off);
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) { red[0][warp] = d0; red[1][warp] = d1; red[2][warp] = d2; }
    __syncthreads();
    if (threadIdx.x < 3) {
        double s = 0.0;
        for (int w = 0; w < (int)(blockDim.x / 32); ++w) s += red[threadIdx.x][w];
        a.part[(size_t)blockIdx.x * 3 + threadIdx.x] = s;
    }
}

__global__ void euler_finalize(const double* part, int nblocks, float* g3) {
    const int k = threadIdx.x;
    if (k >= 3) return;
    double s = 0.0;
    for (int b = 0; b < nblocks; ++b) s += part[(size_t)b * 3 + k];
    g3[k] = (float)s;
}

int euler_bwd_blocks(long long N) { return (int)((N + 255) / 256); }

cudaError_t euler_forward_launch(const float* x, const float* z0, const float* in_scale,
                                 const float* gain, const float* bias, float* spike, float* zfinal,
                                 int T, long long N, float tau, float th, float step,
                                 float reset_strength, float sdt, cudaStream_t st) {
    if (N == 0) return cudaSuccess;
    EulerArgs a{};
    a.x = x; a.z0 = z0; a.in_scale = in_scale; a.gain = gain; a.bias = bias; a.spike = spike;
    a.zfinal = zfinal; a.T = T; a.N = N; a.tau = tau; a.th = th; a.step = step;
    a.reset_strength = reset_strength; a.sdt = sdt;
    euler_fwd<<<(unsigned)((N + 255) / 256), 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t euler_backward_launch(const float* gS, const float* gzf, const float* x,
                                  const float* z0, const float* in_scale, const float* gain,
                                  const float* bias, float* gx, float* gz0, float* g3, int T,
                                  long long N, float tau, float th, float step,
                                  float reset_strength, float sg, float sdt, double* part,
                                  cudaStream_t st) {
    EulerArgs a{};
    a.x = x; a.z0 = z0; a.in_scale = in_scale; a.gain = gain; a.bias = bias; a.gS = gS;
    a.gzf = gzf; a.gx = gx; a.gz0 = gz0; a.part = part; a.T = T; a.N = N; a.tau = tau;
    a.th = th; a.step = step; a.reset_strength = reset_strength; a.sg = sg; a.sdt = sdt;
    const int nb = euler_bwd_blocks(N);
    if (nb > 0) {
        euler_bwd<<<nb, 256, 0, st>>>(a);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    euler_finalize<<<1, 32, 0, st>>>(part, nb, g3);
    return cudaGetLastError();
}

}  // namespace dfsnn
