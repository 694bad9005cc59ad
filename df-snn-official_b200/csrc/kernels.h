// kernels.h -- internal host launchers of the LIF-FDE kernels (not part of the C-ABI;
// include/dfsnn_b200.h is the public interface, implemented in capi.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace dfsnn {

enum Scheme { kGL = 0, kTRAP = 1, kPRED = 2, kGL1 = 3, kTRAP1 = 4, kPRED1 = 5, kEULER = 6 };

// library glmulti
cudaError_t glmulti_forward_launch(const float* x, const float* v0, const float* scale,
                                   const float* W, float* spike, int T, long long N, float tau,
                                   float th, bool tau_pow2, cudaStream_t st);
int glmulti_bwd_blocks(int T, long long N, bool full, bool tau_pow2);
int glmulti_part_stride(int T);
cudaError_t glmulti_backward_launch(const float* gS, const float* x, const float* v0,
                                    const float* scale, const float* W, float* gx, float* gv0,
                                    float* gscale, float* gW, int T, long long N, float tau,
                                    float th, float sg, bool full, bool tau_pow2, double* part,
                                    unsigned int* err, int nblocks, cudaStream_t st);
cudaError_t launch_param_finalize(const double* part, int nblocks, int TB, int T, float* gscale,
                                  float* gW, int lower_only, const unsigned int* err,
                                  cudaStream_t st);
// long-history backward (32 < T <= 256; full history T <= 64): scratch holds three [T, N]
// float arrays (v, drift, grad_pre); part holds `slices` rows of T + T*T doubles
cudaError_t glmulti_backward_long_launch(const float* gS, const float* x, const float* v0,
                                         const float* scale, const float* W, float* gx,
                                         float* gv0, float* gscale, float* gW, int T, long long N,
                                         float tau, float th, float sg, bool full, bool tau_pow2,
                                         double* part, int slices, float* scratch,
                                         unsigned int* err, cudaStream_t st);
cudaError_t aligned_backward_long_launch(const float* g, const float* x, const float* v0,
                                         const float* a_, const float* W, float* gx, float* gv0,
                                         float* ga, float* gW, int T, long long N, float tau,
                                         float th, float sg, float rho, bool tau_pow2,
                                         double* part, int slices, float* scratch,
                                         unsigned int* err, cudaStream_t st);
// gs / gW partial rows from [T, N] scratch (param_long.cu)
int param_long_slices(int T, long long N);
cudaError_t param_long_launch(const float* G, const float* V, const float* E, int T, long long N,
                              bool diag_product, double* part, int slices, cudaStream_t st);
// Per-sample rows: B samples of N/B neurons, `chunks` rows per sample (row b*chunks + c),
// each [T + T*T] doubles = {d[t], M[t][i]}.  diag: what d holds.
enum DiagMode { kDiagNone = 0, kDiagSum = 1, kDiagProduct = 2 };
int param_rows_chunks(int T, long long N, int B);
cudaError_t param_rows_launch(const float* G, const float* V, const float* E, int T, long long N,
                              int B, int diag, double* part, int chunks, bool small_ok,
                              cudaStream_t st);

// VO-GL1 / FAGL1 / VO-PREDICTOR (hfam.cu): per-neuron history kernels with shared or
// per-sample (scale, weights) tables
enum HistKind { kVOGL1 = 0, kFAGL1 = 1, kVOPRED = 2 };
cudaError_t hfam_forward_launch(int kind, const float* x, const float* v0, const float* scale,
                                float h_beta, const float* W, int B, bool per_batch, float* spike,
                                float* vpre, float* hsrc, float* drift, int T, long long N,
                                float tau, float th, float rm, bool tau_pow2, cudaStream_t st);
// T = 8 and 16: one kernel runs the reverse sweep and writes the parameter rows (part, the
// layout of param_rows_launch with B*chunks rows) from V (and E, VO-GL1's drift) itself, when
// V is non-NULL; grad_pre is never stored.  Other T: the sweep writes grad_pre [T, N] and the
// caller reduces it with param_rows_launch.
bool hfam_backward_fused(int T);
cudaError_t hfam_backward_launch(int kind, bool full, const float* gS, const float* scale,
                                 float h_beta, const float* W, int B, bool per_batch,
                                 const float* vpre, float* gx, float* gv0, float* gpre,
                                 const float* V, const float* E, double* part, int chunks, int T,
                                 long long N, float tau, float th, float sg, float rm,
                                 bool tau_pow2, cudaStream_t st);
// gscale / gW from the summed rows (either may be NULL); msum holds (per_batch ? B : 1) rows
cudaError_t hfam_param_finalize(int kind, const double* part, int chunks, int B, bool per_batch,
                                int T, const float* W, const float* scale, double* msum,
                                float* gscale, float* gW, cudaStream_t st);
// true when the x / grad / v0 tiles can be staged with cp.async.bulk (16-byte rows)
bool bulk_eligible(const void* p, const void* q, const void* r, long long N);

// aligned glmulti
cudaError_t aligned_forward_launch(const float* x, const float* v0, const float* a,
                                   const float* W, float* spike, int T, long long N, float tau,
                                   float th, bool tau_pow2, cudaStream_t st);
// element types of x / spike for the typed forward
constexpr int kIoF32 = 0, kIoF16 = 1, kIoBF16 = 2;
cudaError_t aligned_forward_launch_io(const void* x, int dtype, const float* v0, const float* a,
                                      const float* W, void* spike, int T, long long N, float tau,
                                      float th, bool tau_pow2, cudaStream_t st);
int aligned_bwd_blocks(int T, long long N, bool tau_pow2);
int aligned_part_stride(int T);
cudaError_t aligned_backward_launch(const float* g, const float* x, const float* v0,
                                    const float* a, const float* W, float* gx, float* gv0,
                                    float* ga, float* gW, int T, long long N, float tau, float th,
                                    float sg, float rho, bool tau_pow2, double* part,
                                    unsigned int* err, int nblocks, cudaStream_t st);

// single-order schemes
cudaError_t single_forward_launch(int scheme, const float* x, const float* v0, const float* w,
                                  float* spike, float* v, uint32_t* bits, int T, long long N,
                                  float tau, float beta, float th, float h_beta, float gamma1,
                                  bool tau_pow2, cudaStream_t st);
cudaError_t single_backward_launch(int scheme, const float* gS, const float* gV, const float* v,
                                   const uint32_t* bits, const float* w, float* gx, float* gv0,
                                   int T, long long N, float tau, float beta, float th, float sg,
                                   float h_beta, float gamma1, bool tau_pow2, cudaStream_t st);

// TRAP1 / PREDICTOR1 backward: recomputes the trajectory from x and v0 as the reference does
cudaError_t single1_backward_launch(int scheme, const float* gS, const float* gV, const float* x,
                                    const float* v0, const float* w, float* gx, float* gv0,
                                    int T, long long N, float tau, float th, float sg,
                                    float h_beta, bool tau_pow2, cudaStream_t st);

// Store e as the calling thread's dfsnn_last_cuda_error() value; returns DFSNN_ERR_CUDA.
int record_cuda_error(cudaError_t e);

// direct LIF-like Euler
int euler_bwd_blocks(long long N);
cudaError_t euler_forward_launch(const float* x, const float* z0, const float* in_scale,
                                 const float* gain, const float* bias, float* spike, float* zfinal,
                                 int T, long long N, float tau, float th, float step,
                                 float reset_strength, float sdt, cudaStream_t st);
cudaError_t euler_backward_launch(const float* gS, const float* gzf, const float* x,
                                  const float* z0, const float* in_scale, const float* gain,
                                  const float* bias, float* gx, float* gz0, float* g3, int T,
                                  long long N, float tau, float th, float step,
                                  float reset_strength, float sg, float sdt, double* part,
                                  cudaStream_t st);

}  // namespace dfsnn
