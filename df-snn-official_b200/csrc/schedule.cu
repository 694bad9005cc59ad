// schedule.cu -- the glmulti schedule of LIFNeuronFDE in one kernel per direction.
//
// Forward (spikeDE_dis/neuron.py:1461-1514, _get_glmulti_weights + _build_glmulti_schedule):
//   m_j    = softplus(raw_j) (constraint 1) or raw_j (constraint 0)           (:1488-1489)
//   c~[k]  = sum_j (m_j * h^-beta_j) * c_k^(beta_j),  k = 0..T                 (:1477-1479)
//   scale  = 1/c~[0] for every t;  W[t,i] = c~[t-i] * (1/c~[0]) for i < t, 0 otherwise
// with PyTorch's own fp32 operations (softplus = log1pf(expf(x)) below its threshold of 20,
// products, the J-term sum in index order, an IEEE reciprocal), so scale and W are the values
// the reference's chain of small PyTorch kernels produces -- the reference launches about
// 2T+10 of them per forward and as many in the autograd backward.
// Backward: grad_raw from grad_scale and grad_W through the same chain, accumulated in double
// in a fixed order (the reference's autograd sums in fp32; results agree to ~1e-7).
#include "../../include/dfsnn_b200.h"
#include "kernels.h"

namespace dfsnn {
namespace {

constexpr int kMaxJ = 16;

__device__ __forceinline__ float softplus_ref(float x) {
    return x > 20.0f ? x : log1pf(expf(x));       // torch softplus, beta 1, threshold 20
}

__global__ void __launch_bounds__(256) schedule_fwd(const float* raw, const float* basis,
                                                    const float* hpow, int J, int T,
                                                    int constraint, float* scale, float* W,
                                                    float* c_tilde) {
    __shared__ float wh[kMaxJ];
    __shared__ float ct[DFSNN_MAX_T + 1];
    __shared__ float c0_inv;
    const int tid = threadIdx.x;
    if (tid < J) {
        const float m = constraint == 1 ? softplus_ref(raw[tid]) : raw[tid];
        wh[tid] = __fmul_rn(m, hpow[tid]);
    }
    __syncthreads();
    for (int k = tid; k <= T; k += blockDim.x) {
        float s = 0.0f;
        for (int j = 0; j < J; ++j) s = __fadd_rn(s, __fmul_rn(wh[j], basis[j * (T + 1) + k]));
        ct[k] = s;
        c_tilde[k] = s;
    }
    __syncthreads();
    if (tid == 0) c0_inv = __fdiv_rn(1.0f, ct[0]);
    __syncthreads();
    const float ci = c0_inv;
    for (int t = tid; t < T; t += blockDim.x) scale[t] = ci;
    for (int e = tid; e < T * T; e += blockDim.x) {
        const int t = e / T, i = e % T;
        W[e] = i < t ? __fmul_rn(ct[t - i], ci) : 0.0f;
    }
}

__global__ void __launch_bounds__(256) schedule_bwd(const float* raw, const float* basis,
                                                    const float* hpow, const float* c_tilde,
                                                    const float* gscale, const float* gW, int J,
                                                    int T, int constraint, float* grad_raw) {
    __shared__ double diag[DFSNN_MAX_T + 1];     // D[k] = sum_t gW[t][t-k]
    __shared__ double gct[DFSNN_MAX_T + 1];      // grad of c~
    const int tid = threadIdx.x;
    for (int k = tid; k <= T; k += blockDim.x) {
        double d = 0.0;
        if (k >= 1 && gW)
            for (int t = k; t < T; ++t) d += (double)gW[t * T + (t - k)];
        diag[k] = d;
    }
    __syncthreads();
    if (tid == 0) {
        const double ci = 1.0 / (double)c_tilde[0];
        double gci = 0.0;                        // grad of 1/c~[0]
        if (gscale)
            for (int t = 0; t < T; ++t) gci += (double)gscale[t];
        for (int k = 1; k < T; ++k) gci += diag[k] * (double)c_tilde[k];
        gct[0] = -gci * ci * ci;
        for (int k = 1; k <= T; ++k) gct[k] = diag[k] * ci;
    }
    __syncthreads();
    if (tid < J) {
        double g = 0.0;
        for (int k = 0; k <= T; ++k) g += gct[k] * (double)basis[tid * (T + 1) + k];
        g *= (double)hpow[tid];                  // d c~ / d m_j
        if (constraint == 1) {                   // softplus'(x) = sigmoid(x), identity above 20
            const double x = (double)raw[tid];
            if (x <= 20.0) g *= 1.0 / (1.0 + exp(-x));
        }
        grad_raw[tid] = (float)g;
    }
}

}  // namespace
}  // namespace dfsnn

extern "C" int dfsnn_glmulti_schedule_forward(const float* raw, const float* basis,
                                              const float* h_pow, int J, int T, int constraint,
                                              float* scale, float* weights, float* c_tilde,
                                              void* stream) {
    if (!raw || !basis || !h_pow || !scale || !weights || !c_tilde) return DFSNN_ERR_NULL;
    if (J < 1 || J > dfsnn::kMaxJ || T < 1) return DFSNN_ERR_SHAPE;
    if (T > DFSNN_MAX_T) return DFSNN_ERR_T_LIMIT;
    if (constraint != 0 && constraint != 1) return DFSNN_ERR_PARAM;
    dfsnn::schedule_fwd<<<1, 256, 0, (cudaStream_t)stream>>>(raw, basis, h_pow, J, T, constraint,
                                                            scale, weights, c_tilde);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DFSNN_OK : dfsnn::record_cuda_error(e);
}

extern "C" int dfsnn_glmulti_schedule_backward(const float* raw, const float* basis,
                                               const float* h_pow, const float* c_tilde,
                                               const float* grad_scale, const float* grad_weights,
                                               int J, int T, int constraint, float* grad_raw,
                                               void* stream) {
    if (!raw || !basis || !h_pow || !c_tilde || !grad_raw) return DFSNN_ERR_NULL;
    if (J < 1 || J > dfsnn::kMaxJ || T < 1) return DFSNN_ERR_SHAPE;
    if (T > DFSNN_MAX_T) return DFSNN_ERR_T_LIMIT;
    if (constraint != 0 && constraint != 1) return DFSNN_ERR_PARAM;
    dfsnn::schedule_bwd<<<1, 256, 0, (cudaStream_t)stream>>>(raw, basis, h_pow, c_tilde,
                                                            grad_scale, grad_weights, J, T,
                                                            constraint, grad_raw);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? DFSNN_OK : dfsnn::record_cuda_error(e);
}
