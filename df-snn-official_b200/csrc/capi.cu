// capi.cu -- extern "C" entry points declared in include/dfsnn_b200.h.
// Validates arguments (nothing is launched on a bad call), picks the kernel variant
// (T bucket, tau a power of two or not) and launches on the caller's stream.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/dfsnn_b200.h"
#include "kernels.h"

namespace {

thread_local int g_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return DFSNN_OK;
    g_last_cuda_error = (int)e;
    return DFSNN_ERR_CUDA;
}

bool finite(float v) { return std::isfinite(v); }

bool valid_tau(float tau) { return finite(tau) && tau != 0.0f; }

// 1/tau is exact and x/tau == x*(1/tau) for every x iff |tau| is a power of two
// whose reciprocal is a normal float.
bool tau_is_pow2(float tau) {
    if (!finite(tau) || tau == 0.0f) return false;
    int ex = 0;
    const float m = std::frexp(std::fabs(tau), &ex);
    return m == 0.5f && ex > -125 && ex < 126;
}

int check_seq(int T, long long N, int tmax) {
    if (T < 1 || N < 0) return DFSNN_ERR_SHAPE;
    if (T > tmax) return DFSNN_ERR_T_LIMIT;
    return DFSNN_OK;
}

bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// Workspace of the persistent backward kernels: a 16-byte header holding the device error
// word (set when a bounded wait in the kernel gives up; the reduced outputs are then NaN),
// followed by one row of double partials per block.
constexpr size_t kWsHeader = 16;

}  // namespace

namespace dfsnn {
int record_cuda_error(cudaError_t e) { return cuda_status(e); }
}  // namespace dfsnn

extern "C" {

const char* dfsnn_status_string(int status) {
    switch (status) {
        case DFSNN_OK: return "ok";
        case DFSNN_ERR_NULL: return "a required pointer is NULL";
        case DFSNN_ERR_SHAPE: return "invalid shape (T < 1 or N < 0)";
        case DFSNN_ERR_T_LIMIT: return "T exceeds the limit of this entry point";
        case DFSNN_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
        case DFSNN_ERR_CUDA: return "CUDA error (see dfsnn_last_cuda_error)";
        case DFSNN_ERR_SCHEME: return "unknown scheme id";
        case DFSNN_ERR_PARAM: return "invalid scalar parameter (tau == 0 or non-finite)";
        default: return "unknown status";
    }
}

int dfsnn_last_cuda_error(void) { return g_last_cuda_error; }

const char* dfsnn_version(void) { return "dfsnn_b200 0.1 sm_100a"; }

// ---------------------------------------------------------------------------------------
// library glmulti
// ---------------------------------------------------------------------------------------
int dfsnn_glmulti_forward(const float* x, const float* v0, const float* scale,
                          const float* weights, float* spike, int T, long long N, float tau,
                          float threshold, void* stream) {
    if (int s = check_seq(T, N, DFSNN_MAX_T)) return s;
    if (N > 0 && (!x || !v0 || !scale || !weights || !spike)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold)) return DFSNN_ERR_PARAM;
    return cuda_status(dfsnn::glmulti_forward_launch(x, v0, scale, weights, spike, T, N, tau,
                                                     threshold, tau_is_pow2(tau),
                                                     (cudaStream_t)stream));
}

}  // extern "C"

namespace {

// Long-history layout (T > 32): header, `slices` partial rows of T + T*T doubles, then three
// [T, N] float scratch arrays, each starting on a 256-byte boundary.
size_t long_part_bytes(int T, long long N) {
    return (size_t)dfsnn::param_long_slices(T, N) * (size_t)(T + T * T) * sizeof(double);
}
size_t round256(size_t b) { return (b + 255) & ~size_t(255); }
size_t long_workspace_bytes(int T, long long N) {
    return round256(kWsHeader + long_part_bytes(T, N)) + 3 * round256((size_t)T * N * sizeof(float));
}

int glmulti_backward_limit(int full_history) {
    return full_history ? DFSNN_MAX_T_FULL : DFSNN_MAX_T;
}

}  // namespace

extern "C" {

size_t dfsnn_glmulti_backward_workspace_size(int T, long long N, int full_history) {
    if (T < 1 || T > glmulti_backward_limit(full_history) || N < 0) return 0;
    if (T > 32) return long_workspace_bytes(T, N);
    const int b1 = dfsnn::glmulti_bwd_blocks(T, N, full_history != 0, true);
    const int b2 = dfsnn::glmulti_bwd_blocks(T, N, full_history != 0, false);
    const int b = b1 > b2 ? b1 : b2;
    return kWsHeader + (size_t)b * (size_t)dfsnn::glmulti_part_stride(T) * sizeof(double);
}

int dfsnn_glmulti_backward(const float* grad_spike, const float* x, const float* v0,
                           const float* scale, const float* weights, float* grad_x,
                           float* grad_v0, float* grad_scale, float* grad_weights, int T,
                           long long N, float tau, float threshold, float surrogate_scale,
                           int full_history, void* workspace, size_t workspace_bytes,
                           void* stream) {
    if (int s = check_seq(T, N, glmulti_backward_limit(full_history))) return s;
    if (!scale || !weights) return DFSNN_ERR_NULL;
    if (N > 0 && (!grad_spike || !x || !v0 || !grad_x || !grad_v0)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold) || !finite(surrogate_scale)) return DFSNN_ERR_PARAM;
    if (!workspace || !aligned8(workspace)) return DFSNN_ERR_WORKSPACE;
    const bool p2 = tau_is_pow2(tau);
    char* ws = static_cast<char*>(workspace);
    if (T > 32) {
        if (workspace_bytes < long_workspace_bytes(T, N)) return DFSNN_ERR_WORKSPACE;
        const size_t scratch_off = round256(kWsHeader + long_part_bytes(T, N));
        return cuda_status(dfsnn::glmulti_backward_long_launch(
            grad_spike, x, v0, scale, weights, grad_x, grad_v0, grad_scale, grad_weights, T, N,
            tau, threshold, surrogate_scale, full_history != 0, p2,
            reinterpret_cast<double*>(ws + kWsHeader), dfsnn::param_long_slices(T, N),
            reinterpret_cast<float*>(ws + scratch_off), reinterpret_cast<unsigned int*>(ws),
            (cudaStream_t)stream));
    }
    const size_t stride = (size_t)dfsnn::glmulti_part_stride(T) * sizeof(double);
    long long nb = dfsnn::glmulti_bwd_blocks(T, N, full_history != 0, p2);
    const long long cap =
        workspace_bytes > kWsHeader ? (long long)((workspace_bytes - kWsHeader) / stride) : 0;
    if (cap < 1) return DFSNN_ERR_WORKSPACE;
    if (nb > cap) nb = cap;
    return cuda_status(dfsnn::glmulti_backward_launch(
        grad_spike, x, v0, scale, weights, grad_x, grad_v0, grad_scale, grad_weights, T, N, tau,
        threshold, surrogate_scale, full_history != 0, p2,
        reinterpret_cast<double*>(ws + kWsHeader), reinterpret_cast<unsigned int*>(ws), (int)nb,
        (cudaStream_t)stream));
}

// ---------------------------------------------------------------------------------------
// aligned glmulti
// ---------------------------------------------------------------------------------------
int dfsnn_aligned_forward(const float* x, const float* v0, const float* a,
                          const float* weights, float* spike, int T, long long N, float tau,
                          float threshold, void* stream) {
    if (int s = check_seq(T, N, DFSNN_MAX_T_FULL)) return s;
    if (N > 0 && (!x || !v0 || !a || !weights || !spike)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold)) return DFSNN_ERR_PARAM;
    return cuda_status(dfsnn::aligned_forward_launch(x, v0, a, weights, spike, T, N, tau,
                                                     threshold, tau_is_pow2(tau),
                                                     (cudaStream_t)stream));
}

int dfsnn_aligned_forward_typed(const void* x, const float* v0, const float* a,
                                const float* weights, void* spike, int dtype, int T, long long N,
                                float tau, float threshold, void* stream) {
    if (int s = check_seq(T, N, DFSNN_MAX_T_FULL)) return s;
    if (dtype != DFSNN_DTYPE_F32 && dtype != DFSNN_DTYPE_F16 && dtype != DFSNN_DTYPE_BF16)
        return DFSNN_ERR_PARAM;
    if (N > 0 && (!x || !v0 || !a || !weights || !spike)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold)) return DFSNN_ERR_PARAM;
    const int io = dtype == DFSNN_DTYPE_F16 ? dfsnn::kIoF16
                                            : (dtype == DFSNN_DTYPE_BF16 ? dfsnn::kIoBF16 : dfsnn::kIoF32);
    return cuda_status(dfsnn::aligned_forward_launch_io(x, io, v0, a, weights, spike, T, N, tau,
                                                        threshold, tau_is_pow2(tau),
                                                        (cudaStream_t)stream));
}

size_t dfsnn_aligned_backward_workspace_size(int T, long long N) {
    if (T < 1 || T > DFSNN_MAX_T_FULL || N < 0) return 0;
    if (T > 32) return long_workspace_bytes(T, N);
    const int b1 = dfsnn::aligned_bwd_blocks(T, N, true);
    const int b2 = dfsnn::aligned_bwd_blocks(T, N, false);
    const int b = b1 > b2 ? b1 : b2;
    return kWsHeader + (size_t)b * (size_t)dfsnn::aligned_part_stride(T) * sizeof(double);
}

int dfsnn_aligned_backward(const float* grad_spike, const float* x, const float* v0,
                           const float* a, const float* weights, float* grad_x,
                           float* grad_v0, float* grad_a, float* grad_weights, int T,
                           long long N, float tau, float threshold, float surrogate_scale,
                           float rho, void* workspace, size_t workspace_bytes, void* stream) {
    if (int s = check_seq(T, N, DFSNN_MAX_T_FULL)) return s;
    if (!a || !weights) return DFSNN_ERR_NULL;
    if (N > 0 && (!grad_spike || !x || !v0 || !grad_x || !grad_v0)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold) || !finite(surrogate_scale) || !finite(rho))
        return DFSNN_ERR_PARAM;
    if (!workspace || !aligned8(workspace)) return DFSNN_ERR_WORKSPACE;
    const bool p2 = tau_is_pow2(tau);
    char* ws = static_cast<char*>(workspace);
    if (T > 32) {
        if (workspace_bytes < long_workspace_bytes(T, N)) return DFSNN_ERR_WORKSPACE;
        const size_t scratch_off = round256(kWsHeader + long_part_bytes(T, N));
        return cuda_status(dfsnn::aligned_backward_long_launch(
            grad_spike, x, v0, a, weights, grad_x, grad_v0, grad_a, grad_weights, T, N, tau,
            threshold, surrogate_scale, rho, p2, reinterpret_cast<double*>(ws + kWsHeader),
            dfsnn::param_long_slices(T, N), reinterpret_cast<float*>(ws + scratch_off),
            reinterpret_cast<unsigned int*>(ws), (cudaStream_t)stream));
    }
    const size_t stride = (size_t)dfsnn::aligned_part_stride(T) * sizeof(double);
    long long nb = dfsnn::aligned_bwd_blocks(T, N, p2);
    const long long cap =
        workspace_bytes > kWsHeader ? (long long)((workspace_bytes - kWsHeader) / stride) : 0;
    if (cap < 1) return DFSNN_ERR_WORKSPACE;
    if (nb > cap) nb = cap;
    return cuda_status(dfsnn::aligned_backward_launch(
        grad_spike, x, v0, a, weights, grad_x, grad_v0, grad_a, grad_weights, T, N, tau,
        threshold, surrogate_scale, rho, p2, reinterpret_cast<double*>(ws + kWsHeader),
        reinterpret_cast<unsigned int*>(ws), (int)nb, (cudaStream_t)stream));
}

// ---------------------------------------------------------------------------------------
// single-order schemes
// ---------------------------------------------------------------------------------------
size_t dfsnn_spike_bits_words(int T, long long N) {
    if (T < 1 || N < 0) return 0;
    return (size_t)((T + 31) / 32) * (size_t)N;
}

int dfsnn_single_forward(int scheme, const float* x, const float* v0, const float* weights,
                         float* spike, float* v_seq, unsigned int* spike_bits, int T,
                         long long N, float tau, float beta, float threshold, float h_beta,
                         float gamma_beta_plus_1, void* stream) {
    if (scheme < DFSNN_GL || scheme > DFSNN_EULER_LIF) return DFSNN_ERR_SCHEME;
    if (int s = check_seq(T, N, DFSNN_MAX_T)) return s;
    if (!weights && scheme != DFSNN_EULER_LIF) return DFSNN_ERR_NULL;
    if (N > 0 && (!x || !v0 || !spike || !v_seq || !spike_bits)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(beta) || !finite(threshold) || !finite(h_beta) ||
        !finite(gamma_beta_plus_1))
        return DFSNN_ERR_PARAM;
    return cuda_status(dfsnn::single_forward_launch(scheme, x, v0, weights, spike, v_seq,
                                                    reinterpret_cast<uint32_t*>(spike_bits), T, N,
                                                    tau, beta, threshold, h_beta,
                                                    gamma_beta_plus_1, tau_is_pow2(tau),
                                                    (cudaStream_t)stream));
}

int dfsnn_single_backward(int scheme, const float* grad_spike, const float* grad_v,
                          const float* v_seq, const unsigned int* spike_bits,
                          const float* weights, float* grad_x, float* grad_v0, int T,
                          long long N, float tau, float beta, float threshold,
                          float surrogate_scale, float h_beta, float gamma_beta_plus_1,
                          void* stream) {
    if ((scheme < DFSNN_GL || scheme > DFSNN_GL1) && scheme != DFSNN_EULER_LIF)
        return DFSNN_ERR_SCHEME;                  // TRAP1 / PREDICTOR1: recompute backward
    if (int s = check_seq(T, N, DFSNN_MAX_T)) return s;
    if (!weights && scheme != DFSNN_EULER_LIF) return DFSNN_ERR_NULL;
    if (N > 0 && (!grad_spike || !grad_v || !v_seq || !spike_bits || !grad_x || !grad_v0))
        return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(beta) || !finite(threshold) || !finite(surrogate_scale) ||
        !finite(h_beta) || !finite(gamma_beta_plus_1))
        return DFSNN_ERR_PARAM;
    return cuda_status(dfsnn::single_backward_launch(
        scheme, grad_spike, grad_v, v_seq, reinterpret_cast<const uint32_t*>(spike_bits), weights,
        grad_x, grad_v0, T, N, tau, beta, threshold, surrogate_scale, h_beta, gamma_beta_plus_1,
        tau_is_pow2(tau), (cudaStream_t)stream));
}

int dfsnn_single_recompute_backward(int scheme, const float* grad_spike, const float* grad_v,
                                    const float* x, const float* v0, const float* weights,
                                    float* grad_x, float* grad_v0, int T, long long N, float tau,
                                    float threshold, float surrogate_scale, float h_beta,
                                    void* stream) {
    if (scheme != DFSNN_TRAP1 && scheme != DFSNN_PREDICTOR1) return DFSNN_ERR_SCHEME;
    if (int s = check_seq(T, N, DFSNN_MAX_T)) return s;
    if (!weights) return DFSNN_ERR_NULL;
    if (N > 0 && (!grad_spike || !grad_v || !x || !v0 || !grad_x || !grad_v0))
        return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold) || !finite(surrogate_scale) || !finite(h_beta))
        return DFSNN_ERR_PARAM;
    return cuda_status(dfsnn::single1_backward_launch(scheme, grad_spike, grad_v, x, v0, weights,
                                                      grad_x, grad_v0, T, N, tau, threshold,
                                                      surrogate_scale, h_beta, tau_is_pow2(tau),
                                                      (cudaStream_t)stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// VO-GL1 / FAGL1 / VO-PREDICTOR
// ---------------------------------------------------------------------------------------
namespace {

// Workspace: grad_pre [T, N] floats (not for T = 8 and 16, whose sweep kernel forms the
// parameter rows itself), then the partial rows (B*chunks rows of T + T*T doubles), then the
// summed rows ((per_batch ? B : 1) of them), each on a 256-byte boundary.
struct HistWs {
    size_t gpre, part, msum, total;
    int chunks;
};

HistWs hist_ws(int T, long long N, int B, int per_batch) {
    HistWs w;
    const size_t R = (size_t)T + (size_t)T * T;
    const bool fused = dfsnn::hfam_backward_fused(T);
    w.chunks = dfsnn::param_rows_chunks(T, N, B);
    w.gpre = 0;
    w.part = fused ? 0 : round256((size_t)T * (size_t)N * sizeof(float));
    w.msum = w.part + round256((size_t)B * w.chunks * R * sizeof(double));
    w.total = w.msum + round256((size_t)(per_batch ? B : 1) * R * sizeof(double));
    return w;
}

int check_hist(int T, long long N, int B, int per_batch, int tmax) {
    if (int s = check_seq(T, N, tmax)) return s;
    if (B < 1 || N % B != 0) return DFSNN_ERR_SHAPE;
    if (per_batch != 0 && per_batch != 1) return DFSNN_ERR_PARAM;
    return DFSNN_OK;
}

int hist_forward(int kind, const float* x, const float* v0, const float* scale,
                 const float* weights, int batch, int per_batch, float* spike, float* v_pre,
                 float* hsrc, float* drift, int T, long long N, float tau, float threshold,
                 float h_beta, float residual_mix, int tmax, void* stream) {
    if (int s = check_hist(T, N, batch, per_batch, tmax)) return s;
    if (!weights || (kind != dfsnn::kFAGL1 && !scale)) return DFSNN_ERR_NULL;
    if (N > 0 && (!x || !v0 || !spike || !v_pre || !hsrc || (kind == dfsnn::kVOGL1 && !drift)))
        return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold) || !finite(h_beta) || !finite(residual_mix))
        return DFSNN_ERR_PARAM;
    return cuda_status(dfsnn::hfam_forward_launch(kind, x, v0, scale, h_beta, weights, batch,
                                                  per_batch != 0, spike, v_pre, hsrc, drift, T,
                                                  N, tau, threshold, residual_mix,
                                                  tau_is_pow2(tau), (cudaStream_t)stream));
}

// V: the saved sequence the weight gradient pairs with grad_pre; E: the drift (VO-GL1's
// grad_scale), NULL otherwise
int hist_backward(int kind, int full, const float* grad_spike, const float* scale,
                  const float* weights, const float* v_pre, const float* V, const float* E,
                  int batch, int per_batch, float* grad_x, float* grad_v0, float* grad_scale,
                  float* grad_weights, int T, long long N, float tau, float threshold,
                  float surrogate_scale, float h_beta, float residual_mix, int tmax,
                  void* workspace, size_t workspace_bytes, void* stream) {
    if (full != 0 && full != 1) return DFSNN_ERR_PARAM;
    if (int s = check_hist(T, N, batch, per_batch, full ? DFSNN_MAX_T_FULL : tmax)) return s;
    if (!weights || (kind != dfsnn::kFAGL1 && !scale)) return DFSNN_ERR_NULL;
    const bool params = grad_scale || grad_weights;
    if (N > 0 && (!grad_spike || !v_pre || !grad_x || !grad_v0)) return DFSNN_ERR_NULL;
    if (N > 0 && params && (!V || (grad_scale && kind == dfsnn::kVOGL1 && !E)))
        return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold) || !finite(surrogate_scale) || !finite(h_beta) ||
        !finite(residual_mix))
        return DFSNN_ERR_PARAM;
    const HistWs w = hist_ws(T, N, batch, per_batch);
    if (!workspace || !aligned8(workspace) || workspace_bytes < w.total) return DFSNN_ERR_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    const bool fused = dfsnn::hfam_backward_fused(T);
    float* gpre = fused ? nullptr : reinterpret_cast<float*>(ws + w.gpre);
    double* part = reinterpret_cast<double*>(ws + w.part);
    double* msum = reinterpret_cast<double*>(ws + w.msum);
    cudaStream_t st = (cudaStream_t)stream;
    const bool p2 = tau_is_pow2(tau);
    const float* Ediag = (kind == dfsnn::kVOGL1 && grad_scale) ? E : nullptr;
    cudaError_t e = dfsnn::hfam_backward_launch(kind, full != 0, grad_spike, scale, h_beta,
                                                weights, batch, per_batch != 0, v_pre, grad_x,
                                                grad_v0, gpre, params ? V : nullptr, Ediag, part,
                                                w.chunks, T, N, tau, threshold, surrogate_scale,
                                                residual_mix, p2, st);
    if (e != cudaSuccess || !params) return cuda_status(e);
    if (N == 0) {
        e = cudaMemsetAsync(part, 0, (size_t)batch * w.chunks * (T + (size_t)T * T) * sizeof(double), st);
    } else if (!fused) {                  // T = 8 and 16: the sweep kernel wrote the rows
        const int diag = (kind == dfsnn::kVOGL1 && grad_scale) ? dfsnn::kDiagProduct
                                                               : dfsnn::kDiagNone;
        e = dfsnn::param_rows_launch(gpre, V, E, T, N, batch, diag, part, w.chunks, true, st);
    }
    if (e != cudaSuccess) return cuda_status(e);
    return cuda_status(dfsnn::hfam_param_finalize(kind, part, w.chunks, batch, per_batch != 0, T,
                                                  weights, scale, msum, grad_scale, grad_weights,
                                                  st));
}

}  // namespace

extern "C" {

size_t dfsnn_history_backward_workspace_size(int T, long long N, int batch, int per_batch) {
    if (T < 1 || T > DFSNN_MAX_T || N < 0 || batch < 1 || N % batch != 0) return 0;
    if (per_batch != 0 && per_batch != 1) return 0;
    return hist_ws(T, N, batch, per_batch).total;
}

int dfsnn_vo_gl1_forward(const float* x, const float* v0, const float* scale,
                         const float* weights, int batch, int per_batch, float* spike,
                         float* v_pre, float* v_hist, float* drift, int T, long long N, float tau,
                         float threshold, void* stream) {
    return hist_forward(dfsnn::kVOGL1, x, v0, scale, weights, batch, per_batch, spike, v_pre,
                        v_hist, drift, T, N, tau, threshold, 1.0f, 0.0f, DFSNN_MAX_T, stream);
}

int dfsnn_fa_gl1_forward(const float* x, const float* v0, const float* weights, int batch,
                         int per_batch, float* spike, float* v_pre, float* v_hist, int T,
                         long long N, float tau, float h_beta, float threshold, void* stream) {
    return hist_forward(dfsnn::kFAGL1, x, v0, nullptr, weights, batch, per_batch, spike, v_pre,
                        v_hist, nullptr, T, N, tau, threshold, h_beta, 0.0f, DFSNN_MAX_T_FULL,
                        stream);
}

int dfsnn_vo_predictor_forward(const float* x, const float* v0, const float* scale,
                               const float* weights, int batch, int per_batch, float* spike,
                               float* v_pre, float* drift, int T, long long N, float tau,
                               float threshold, float residual_mix, void* stream) {
    return hist_forward(dfsnn::kVOPRED, x, v0, scale, weights, batch, per_batch, spike, v_pre,
                        drift, nullptr, T, N, tau, threshold, 1.0f, residual_mix, DFSNN_MAX_T,
                        stream);
}

int dfsnn_vo_gl1_backward(const float* grad_spike, const float* scale, const float* weights,
                          const float* v_pre, const float* v_hist, const float* drift, int batch,
                          int per_batch, float* grad_x, float* grad_v0, float* grad_scale,
                          float* grad_weights, int T, long long N, float tau, float threshold,
                          float surrogate_scale, int full_history, void* workspace,
                          size_t workspace_bytes, void* stream) {
    return hist_backward(dfsnn::kVOGL1, full_history, grad_spike, scale, weights, v_pre, v_hist,
                         drift, batch, per_batch, grad_x, grad_v0, grad_scale, grad_weights, T, N,
                         tau, threshold, surrogate_scale, 1.0f, 0.0f, DFSNN_MAX_T, workspace,
                         workspace_bytes, stream);
}

int dfsnn_fa_gl1_backward(const float* grad_spike, const float* weights, const float* v_pre,
                          const float* v_hist, int batch, int per_batch, float* grad_x,
                          float* grad_v0, float* grad_weights, int T, long long N, float tau,
                          float h_beta, float threshold, float surrogate_scale, int full_history,
                          void* workspace, size_t workspace_bytes, void* stream) {
    return hist_backward(dfsnn::kFAGL1, full_history, grad_spike, nullptr, weights, v_pre, v_hist,
                         nullptr, batch, per_batch, grad_x, grad_v0, nullptr, grad_weights, T, N,
                         tau, threshold, surrogate_scale, h_beta, 0.0f, DFSNN_MAX_T_FULL,
                         workspace, workspace_bytes, stream);
}

int dfsnn_vo_predictor_backward(const float* grad_spike, const float* scale,
                                const float* weights, const float* v_pre, const float* drift,
                                int batch, int per_batch, float* grad_x, float* grad_v0,
                                float* grad_scale, float* grad_weights, int T, long long N,
                                float tau, float threshold, float surrogate_scale,
                                float residual_mix, void* workspace, size_t workspace_bytes,
                                void* stream) {
    return hist_backward(dfsnn::kVOPRED, 0, grad_spike, scale, weights, v_pre, drift, nullptr,
                         batch, per_batch, grad_x, grad_v0, grad_scale, grad_weights, T, N, tau,
                         threshold, surrogate_scale, 1.0f, residual_mix, DFSNN_MAX_T, workspace,
                         workspace_bytes, stream);
}

// ---------------------------------------------------------------------------------------
// direct LIF-like Euler
// ---------------------------------------------------------------------------------------
int dfsnn_direct_euler_forward(const float* x, const float* z0, const float* input_scale,
                               const float* spike_gain, const float* spike_bias, float* spike,
                               float* z_final, int T, long long N, float tau, float threshold,
                               float step_size, float reset_strength, float spike_update_dt,
                               void* stream) {
    if (int s = check_seq(T, N, 1024)) return s;
    if (!input_scale || !spike_gain || !spike_bias) return DFSNN_ERR_NULL;
    if (N > 0 && (!x || !z0 || !spike || !z_final)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold) || !finite(step_size) || !finite(reset_strength) ||
        !finite(spike_update_dt))
        return DFSNN_ERR_PARAM;
    return cuda_status(dfsnn::euler_forward_launch(x, z0, input_scale, spike_gain, spike_bias,
                                                   spike, z_final, T, N, tau, threshold,
                                                   step_size, reset_strength, spike_update_dt,
                                                   (cudaStream_t)stream));
}

size_t dfsnn_direct_euler_backward_workspace_size(long long N) {
    if (N < 0) return 0;
    const long long nb = dfsnn::euler_bwd_blocks(N);
    return (size_t)(nb > 0 ? nb : 1) * 3 * sizeof(double);
}

int dfsnn_direct_euler_backward(const float* grad_spike, const float* grad_z_final,
                                const float* x, const float* z0, const float* input_scale,
                                const float* spike_gain, const float* spike_bias,
                                float* grad_x, float* grad_z0, float* grad3, int T, long long N,
                                float tau, float threshold, float step_size,
                                float reset_strength, float surrogate_scale,
                                float spike_update_dt, void* workspace, size_t workspace_bytes,
                                void* stream) {
    if (int s = check_seq(T, N, 1024)) return s;
    if (!input_scale || !spike_gain || !spike_bias || !grad3) return DFSNN_ERR_NULL;
    if (N > 0 && (!grad_spike || !x || !z0 || !grad_x || !grad_z0)) return DFSNN_ERR_NULL;
    if (!valid_tau(tau) || !finite(threshold) || !finite(step_size) || !finite(reset_strength) ||
        !finite(surrogate_scale) || !finite(spike_update_dt))
        return DFSNN_ERR_PARAM;
    if (!workspace || !aligned8(workspace) ||
        workspace_bytes < dfsnn_direct_euler_backward_workspace_size(N))
        return DFSNN_ERR_WORKSPACE;
    return cuda_status(dfsnn::euler_backward_launch(
        grad_spike, grad_z_final, x, z0, input_scale, spike_gain, spike_bias, grad_x, grad_z0,
        grad3, T, N, tau, threshold, step_size, reset_strength, surrogate_scale, spike_update_dt,
        static_cast<double*>(workspace), (cudaStream_t)stream));
}

}  // extern "C"
