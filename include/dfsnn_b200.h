/*
 * dfsnn_b200.h -- C ABI of the B200 (sm_100a) LIF-FDE kernels.
 *
 * Drop-in boundary for the hot path of DF-SNN's LIFNeuronFDE
 * (cjge-ustc/DF-SNN-official, spikeDE_dis/neuron.py:1058).  In the reference, every
 * entry below is a CuPy RawKernel launch made from a torch.autograd.Function in
 * spikeDE_dis/fde_cupy_kernels_all.py, examples/cnn128/aligned_glmulti.py or
 * spikeDE_dis/direct_euler_cupy.py; each declaration names the launch(es) it replaces.
 *
 * Conventions
 *   - Every pointer is a device pointer (cudaMalloc / torch CUDA memory) unless stated;
 *     the library never allocates, frees or retains them.
 *   - Sequences are time-major float32 [T, N], row-major (element (t, n) at t*N + n),
 *     exactly the [T, N] layout the reference Functions pass to their kernels.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 *     asynchronous on that stream and launches on the calling thread's current device.
 *   - Return value: DFSNN_OK or one of the DFSNN_ERR_* codes; nothing is launched when
 *     argument validation fails.  dfsnn_status_string() names a code,
 *     dfsnn_last_cuda_error() gives the cudaError_t behind DFSNN_ERR_CUDA.
 *   - Arithmetic reproduces the reference kernels' fp32 operation order (including the
 *     fused multiply-adds NVRTC forms under --fmad=true, and none for the aligned kernels
 *     compiled with --fmad=false), so spikes, membranes and per-neuron gradients match the
 *     reference bit for bit; reductions over neurons are accumulated in a fixed order
 *     (deterministic) with compensated fp32 and double partials.
 */
#ifndef DFSNN_B200_H
#define DFSNN_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DFSNN_OK 0
#define DFSNN_ERR_NULL 1        /* a required pointer is NULL */
#define DFSNN_ERR_SHAPE 2       /* T < 1 or N < 0 */
#define DFSNN_ERR_T_LIMIT 3     /* T above this entry point's limit */
#define DFSNN_ERR_WORKSPACE 4   /* workspace NULL, misaligned or too small */
#define DFSNN_ERR_CUDA 5        /* a CUDA call or kernel launch failed */
#define DFSNN_ERR_SCHEME 6      /* unknown scheme id */
#define DFSNN_ERR_PARAM 7       /* tau == 0 or a non-finite scalar parameter */

#define DFSNN_MAX_T 256         /* forward / truncated limit (reference: 256-entry locals) */
#define DFSNN_MAX_T_FULL 64     /* full-history glmulti backward and aligned glmulti (as the reference) */

/* scheme ids of the single-order family */
#define DFSNN_GL 0
#define DFSNN_TRAP 1
#define DFSNN_PREDICTOR 2
#define DFSNN_GL1 3
#define DFSNN_TRAP1 4        /* LIFFDETRAP1Function (fde_cupy_kernels_all.py:2018-2276) */
#define DFSNN_PREDICTOR1 5   /* LIFFDEPREDICTOR1Function (:2278-2545) */
#define DFSNN_EULER_LIF 6    /* LIFEulerFunction (:2546-2756): no history; weights may be NULL */

const char* dfsnn_status_string(int status);
int dfsnn_last_cuda_error(void);
const char* dfsnn_version(void);

/* ---------------------------------------------------------------------------------
 * Library distributed-order GL (LIFFDEGLMultiFunction, fde_cupy_kernels_all.py:1916-2011)
 * ------------------------------------------------------------------------------- */

/* Replaces the lif_fde_vo_gl1_forward_kernel launch with per_batch=0
 * (fde_cupy_kernels_all.py:1938-1971 launching :1594-1630).
 * p_t = scale[t]*d_t - sum_{i<t} W[t,i] v_i, d_t = (x_t - v_{t-1})/tau, spike = p_t >= th,
 * v_t = p_t - spike*th.  Writes spike[T,N] only (the backward recomputes the rest). */
int dfsnn_glmulti_forward(const float* x, const float* v0, const float* scale,
                          const float* weights, float* spike, int T, long long N, float tau,
                          float threshold, void* stream);

/* glmulti schedule (LIFNeuronFDE._get_glmulti_weights + _build_glmulti_schedule,
 * neuron.py:1461-1514) in one launch: masses m = softplus(raw) (constraint 1) or raw
 * (constraint 0), c~[k] = sum_j m_j h_pow[j] basis[j][k] (k = 0..T), scale[t] = 1/c~[0],
 * weights[t][i] = c~[t-i]/c~[0] for i < t, else 0.  Same fp32 operations as the reference's
 * PyTorch chain, so scale and weights are bit-identical to it.  basis is [J][T+1], c_tilde
 * (T+1 floats) is kept for the backward.  J <= 16, T <= DFSNN_MAX_T. */
int dfsnn_glmulti_schedule_forward(const float* raw, const float* basis, const float* h_pow,
                                   int J, int T, int constraint, float* scale, float* weights,
                                   float* c_tilde, void* stream);

/* Gradient of the schedule with respect to raw (J floats) given grad_scale [T] and
 * grad_weights [T][T] (either may be NULL = zero); upper-triangle entries of grad_weights
 * are ignored (the reference's torch.where discards them).  Accumulated in double. */
int dfsnn_glmulti_schedule_backward(const float* raw, const float* basis, const float* h_pow,
                                    const float* c_tilde, const float* grad_scale,
                                    const float* grad_weights, int J, int T, int constraint,
                                    float* grad_raw, void* stream);

/* Bytes of device workspace dfsnn_glmulti_backward needs (8-byte aligned); 0 when T is
 * outside the limit for this history mode. */
size_t dfsnn_glmulti_backward_workspace_size(int T, long long N, int full_history);

/* Replaces LIFFDEGLMultiFunction.backward (fde_cupy_kernels_all.py:1973-2011): the
 * lif_fde_glmulti_backward_kernel (:1845-1875, full_history=0) or
 * lif_fde_glmulti_full_backward_kernel (:1877-1913, full_history=1) launch, then
 * grad_scale[t] = sum_n grad_pre*drift and grad_weights = -grad_pre @ v_hist^T (full T x T).
 * grad_scale / grad_weights may be NULL (not needed).  T <= DFSNN_MAX_T_FULL with
 * full_history (the reference's limit), T <= DFSNN_MAX_T without.  For T > 32 the workspace
 * also holds three [T, N] float arrays (v, drift, grad_pre) for the parameter reduction. */
int dfsnn_glmulti_backward(const float* grad_spike, const float* x, const float* v0,
                           const float* scale, const float* weights, float* grad_x,
                           float* grad_v0, float* grad_scale, float* grad_weights, int T,
                           long long N, float tau, float threshold, float surrogate_scale,
                           int full_history, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Same computation and results as dfsnn_glmulti_backward, for callers that cannot allocate
 * device memory when the backward runs (a host callback, a runtime that owns all device
 * memory, an allocation-free serving loop).  No counterpart in the reference: it has no
 * workspace argument; its scratch (error word + per-block partial sums) is a 1.1 MB
 * file-scope device array that every device loading the library keeps until exit.
 * Limit: T <= 16 (DFSNN_ERR_T_LIMIT above).  All calls share that array: calls whose work
 * overlaps on the GPU (other streams or host threads) race.  The first call on a device
 * looks up the array's address; make it before any stream capture, and make no call on a
 * device after cudaDeviceReset of that device (the looked-up address is kept for the life
 * of the process).  The array holds 512 rows of partial sums: while the regular entry point
 * would use at most 512 (a 148-SM B200 uses 148 or 296), grad_scale / grad_weights equal its
 * results bit for bit; beyond that the blocks are capped at 512 and the sums agree within
 * the reduction tolerance.  A bounded device wait that times out shows only as NaN in
 * grad_scale / grad_weights (there is no workspace to read the error word from), so a
 * caller that passes both as NULL gets no timeout report.  Allocates nothing. */
int dfsnn_glmulti_backward_noalloc(const float* grad_spike, const float* x, const float* v0,
                                   const float* scale, const float* weights, float* grad_x,
                                   float* grad_v0, float* grad_scale, float* grad_weights, int T,
                                   long long N, float tau, float threshold,
                                   float surrogate_scale, int full_history, void* stream);

/* ---------------------------------------------------------------------------------
 * Aligned distributed-order GL (AlignedGLMulti, examples/cnn128/aligned_glmulti.py)
 * ------------------------------------------------------------------------------- */

/* Replaces the aligned_forward launch (aligned_glmulti.py:106-121 launching :7-17). */
int dfsnn_aligned_forward(const float* x, const float* v0, const float* a,
                          const float* weights, float* spike, int T, long long N, float tau,
                          float threshold, void* stream);

/* Element types of dfsnn_aligned_forward_typed's x and spike arrays. */
#define DFSNN_DTYPE_F32 0
#define DFSNN_DTYPE_F16 1
#define DFSNN_DTYPE_BF16 2

/* Replaces AlignedGLMulti.forward for the half-precision activations it receives under
 * autocast (aligned_glmulti.py:112-121: x.float(), the aligned_forward launch, s.to(x.dtype)):
 * x and spike are float16 (DFSNN_DTYPE_F16) or bfloat16 (DFSNN_DTYPE_BF16) [T, N] arrays read
 * and written in that type, the arithmetic is dfsnn_aligned_forward's fp32, so the spikes are
 * the reference's.  DFSNN_DTYPE_F32 is dfsnn_aligned_forward. */
int dfsnn_aligned_forward_typed(const void* x, const float* v0, const float* a,
                                const float* weights, void* spike, int dtype, int T, long long N,
                                float tau, float threshold, void* stream);

size_t dfsnn_aligned_backward_workspace_size(int T, long long N);

/* Replaces AlignedGLMulti.backward (aligned_glmulti.py:123-145): aligned_backward (:20-32)
 * with HISTORY_RHO = rho, aligned_scale (:33-41) + sum, and -(ga@h^T)*tril(-1).
 * grad_a / grad_weights may be NULL.  T <= DFSNN_MAX_T_FULL. */
int dfsnn_aligned_backward(const float* grad_spike, const float* x, const float* v0,
                           const float* a, const float* weights, float* grad_x,
                           float* grad_v0, float* grad_a, float* grad_weights, int T,
                           long long N, float tau, float threshold, float surrogate_scale,
                           float rho, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Single-order schemes: GL, TRAP, PREDICTOR, GL1 (LIFFDEGLFunction, LIFFDETRAPFunction,
 * LIFFDEPREDICTORFunction, LIFFDEGL1Function)
 * ------------------------------------------------------------------------------- */

/* Number of uint32 words of the spike bitmask for (T, N): ceil(T/32) * N. */
size_t dfsnn_spike_bits_words(int T, long long N);

/* Replaces the lif_fde_{gl,trap,predictor,gl1}_forward_kernel launches
 * (fde_cupy_kernels_all.py:24-75, :327-381, :479-539, :170-260; launched from the Functions'
 * forward at :658-698, :843-882, :933-975, :749-793).  weights = the reversed table of T+1 entries.
 * Writes spike[T,N], v_seq[T,N] and the spike bitmask the backward consumes.
 * h_beta / gamma_beta_plus_1 are used by PREDICTOR (both) and GL1 (h_beta).  Schemes
 * DFSNN_TRAP1 / DFSNN_PREDICTOR1 replace lif_fde_trap1_forward_kernel (:2018-2070) and
 * lif_fde_predictor1_forward_kernel (:2278-2335) (h_beta used by both; TRAP1's Function
 * passes h_beta = 1).  Their spike_bits output is written but their backward does not use it.
 * DFSNN_EULER_LIF replaces lif_euler_forward_kernel (:2546-2584); weights may be NULL. */
int dfsnn_single_forward(int scheme, const float* x, const float* v0, const float* weights,
                         float* spike, float* v_seq, unsigned int* spike_bits, int T,
                         long long N, float tau, float beta, float threshold, float h_beta,
                         float gamma_beta_plus_1, void* stream);

/* Replaces lif_fde_trap1_backward_kernel (:2072-2161, launched :2225-2276) and
 * lif_fde_predictor1_backward_kernel (:2337-2432, launched :2497-2545) (scheme DFSNN_TRAP1 or
 * DFSNN_PREDICTOR1): like the reference, recomputes the trajectory from x and v0 with a plain
 * fused multiply-add history sum (not the forward's Kahan sum) before the reverse sweep.
 * grad_v is the upstream gradient of v_seq.  T <= DFSNN_MAX_T. */
int dfsnn_single_recompute_backward(int scheme, const float* grad_spike, const float* grad_v,
                                    const float* x, const float* v0, const float* weights,
                                    float* grad_x, float* grad_v0, int T, long long N, float tau,
                                    float threshold, float surrogate_scale, float h_beta,
                                    void* stream);

/* Replaces the lif_fde_{gl,trap,predictor,gl1}_backward_kernel and lif_euler_backward_kernel
 * (:2586-2654) launches (:77-163,
 * :383-472, :541-637, :262-320; launched from :700-732, :884-916, :977-1010, :795-827):
 * truncated reverse sweep, from the saved v_seq and
 * spike bitmask instead of a recompute. */
int dfsnn_single_backward(int scheme, const float* grad_spike, const float* grad_v,
                          const float* v_seq, const unsigned int* spike_bits,
                          const float* weights, float* grad_x, float* grad_v0, int T,
                          long long N, float tau, float beta, float threshold,
                          float surrogate_scale, float h_beta, float gamma_beta_plus_1,
                          void* stream);

/* ---------------------------------------------------------------------------------
 * Direct LIF-like Euler (DirectLIFLikeEulerCuPyFunction, spikeDE_dis/direct_euler_cupy.py)
 * ------------------------------------------------------------------------------- */

/* Replaces direct_lif_euler_forward (direct_euler_cupy.py:22-58, launched :157-182).
 * input_scale / spike_gain / spike_bias are device scalars. */
int dfsnn_direct_euler_forward(const float* x, const float* z0, const float* input_scale,
                               const float* spike_gain, const float* spike_bias, float* spike,
                               float* z_final, int T, long long N, float tau, float threshold,
                               float step_size, float reset_strength, float spike_update_dt,
                               void* stream);

size_t dfsnn_direct_euler_backward_workspace_size(long long N);

/* Replaces direct_lif_euler_backward (direct_euler_cupy.py:66-131, launched :200-236).
 * grad_z_final may be NULL (zeros).  grad3 receives {grad_input_scale, grad_spike_gain,
 * grad_spike_bias} (3 device floats), reduced without atomics.  T <= 1024. */
int dfsnn_direct_euler_backward(const float* grad_spike, const float* grad_z_final,
                                const float* x, const float* z0, const float* input_scale,
                                const float* spike_gain, const float* spike_bias,
                                float* grad_x, float* grad_z0, float* grad3, int T, long long N,
                                float tau, float threshold, float step_size,
                                float reset_strength, float surrogate_scale,
                                float spike_update_dt, void* workspace, size_t workspace_bytes,
                                void* stream);

/* ---------------------------------------------------------------------------------
 * History-table Functions with shared or per-sample parameters: VO-GL1, FAGL1,
 * VO-PREDICTOR (LIFFDEVOGL1Function, LIFFDEFAGL1Function, LIFFDEVOPREDICTORFunction)
 *
 * batch = B: neuron n belongs to sample n / (N/B); N % B must be 0.  per_batch = 0: scale is
 * [T] and weights [T][T]; per_batch = 1: scale is [T][B] and weights [T][B][T].  T <= 256
 * (DFSNN_MAX_T); FAGL1 and every full-history backward T <= 64 (the reference's limits).
 * ------------------------------------------------------------------------------- */

/* Replaces the lif_fde_vo_gl1_forward_kernel launch of LIFFDEVOGL1Function.forward
 * (fde_cupy_kernels_all.py:1786-1809 launching :1594-1630): writes spike, v_pre, v_hist (v
 * after reset) and drift, all [T, N]. */
int dfsnn_vo_gl1_forward(const float* x, const float* v0, const float* scale,
                         const float* weights, int batch, int per_batch, float* spike,
                         float* v_pre, float* v_hist, float* drift, int T, long long N, float tau,
                         float threshold, void* stream);

/* Replaces the lif_fde_fa_gl1_forward_kernel launch of LIFFDEFAGL1Function.forward
 * (:1413-1455 launching :1200-1232); the per-step scale is h_beta.  per_batch follows the
 * weights' rank ([T][B][T] or [T][T]). */
int dfsnn_fa_gl1_forward(const float* x, const float* v0, const float* weights, int batch,
                         int per_batch, float* spike, float* v_pre, float* v_hist, int T,
                         long long N, float tau, float h_beta, float threshold, void* stream);

/* Replaces the lif_fde_vo_predictor_forward_kernel launch of LIFFDEVOPREDICTORFunction.forward
 * (:1121-1156 launching :1017-1057): writes spike, v_pre and drift. */
int dfsnn_vo_predictor_forward(const float* x, const float* v0, const float* scale,
                               const float* weights, int batch, int per_batch, float* spike,
                               float* v_pre, float* drift, int T, long long N, float tau,
                               float threshold, float residual_mix, void* stream);

/* Bytes of device workspace the three backward entry points need (8-byte aligned): grad_pre
 * plus the partial sums of the parameter reduction.  0 for invalid arguments. */
size_t dfsnn_history_backward_workspace_size(int T, long long N, int batch, int per_batch);

/* Replaces LIFFDEVOGL1Function.backward (:1811-1840): the lif_fde_vo_gl1_backward_kernel
 * (:1633-1668) or lif_fde_vo_gl1_full_backward_kernel (:1670-1709, full_history = 1) launch,
 * then grad_scale = sum grad_pre*drift and grad_weights = -grad_pre @ v_hist^T over each
 * sample (per_batch) or all neurons -- every entry, upper triangle included, as the
 * reference's einsum / matmul.  Sums in double.  grad_scale / grad_weights may be NULL
 * (v_hist / drift are then not read). */
int dfsnn_vo_gl1_backward(const float* grad_spike, const float* scale, const float* weights,
                          const float* v_pre, const float* v_hist, const float* drift, int batch,
                          int per_batch, float* grad_x, float* grad_v0, float* grad_scale,
                          float* grad_weights, int T, long long N, float tau, float threshold,
                          float surrogate_scale, int full_history, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Replaces LIFFDEFAGL1Function.backward (:1457-1497): the lif_fde_fa_gl1_backward_kernel
 * (:1235-1272) or lif_fde_fa_gl1_full_backward_kernel (:1274-1312) launch, then
 * grad_weights = -grad_pre @ v_hist^T: per sample with zeros on and above the diagonal
 * (lif_fde_fa_gl1_weight_grad_kernel, :1314-1344), or over all neurons with every entry (the
 * reference's matmul, which it runs in TF32; here fp32 products summed in double). */
int dfsnn_fa_gl1_backward(const float* grad_spike, const float* weights, const float* v_pre,
                          const float* v_hist, int batch, int per_batch, float* grad_x,
                          float* grad_v0, float* grad_weights, int T, long long N, float tau,
                          float h_beta, float threshold, float surrogate_scale, int full_history,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Replaces LIFFDEVOPREDICTORFunction.backward (:1158-1191): the
 * lif_fde_vo_predictor_backward_kernel launch (:1058-1096), then
 * grad_scale = sum grad_pre*(drift + weights @ drift) and
 * grad_weights = (grad_pre*scale) @ drift^T per sample or over all neurons (full matrices). */
int dfsnn_vo_predictor_backward(const float* grad_spike, const float* scale,
                                const float* weights, const float* v_pre, const float* drift,
                                int batch, int per_batch, float* grad_x, float* grad_v0,
                                float* grad_scale, float* grad_weights, int T, long long N,
                                float tau, float threshold, float surrogate_scale,
                                float residual_mix, void* workspace, size_t workspace_bytes,
                                void* stream);

/* ---------------------------------------------------------------------------------
 * Multi-term GL integrator of the SNN wrapper path (spikeDE_dis/solver.py)
 * ------------------------------------------------------------------------------- */

#define DFSNN_F32 0
#define DFSNN_F64 1

/* One integrator step for one state component, replacing the per-step body of
 * forward_glmulti_cupy (solver.py:3310-3362: torch.stack of the history, weighted_sum
 * kernels :90-104 per 96-row chunk, the chunk sum, f - conv and the c~_0^-1 scale) and of
 * backward_glmulti_cupy (:2959-2995: the coefficient dot product and the same update):
 *   out = c0_inv[0] * (f - conv),  conv = sum_{row_begin <= j < row_end} c_tilde[coeff_base - j]
 *                                         * rows[j][n]
 * rows is a device table of row pointers (state_size elements each, dtype DFSNN_F32 or
 * DFSNN_F64).  chunk > 0: fused multiply-add chains over chunks of `chunk` rows whose results
 * are added in order (the forward's weighted_sum kernels); chunk == 0: one chain (the
 * adjoint's dot product); chunk < 0: multiply, then add, term by term (the forward's PyTorch
 * loop for history_chunk_size <= 0).  diff (optional) receives f - conv.  If table is not
 * NULL, table[out_slot] = out is stored by the kernel (out_slot >= row_end), so later steps
 * find this step's output; c_tilde and c0_inv are device arrays. */
int dfsnn_gl_history_step(int dtype, const void* f, const void* const* rows, int row_begin,
                          int row_end, const void* c_tilde, int coeff_base, const void* c0_inv,
                          int chunk, void* out, void* diff, long long state_size, void** table,
                          int out_slot, void* stream);

/* Bytes of workspace dfsnn_gl_history_step_backward needs for `rows` history rows. */
size_t dfsnn_gl_history_step_workspace_size(int rows, long long state_size);

/* Gradients of one step given grad_out: grad_f = c0_inv*grad_out; if grad_rows is not NULL,
 * grad_rows[j - row_begin][n] = c_tilde[coeff_base - j] * (-grad_f[n]) ([rows, state_size]);
 * grad_coeff[j - row_begin] = sum_n rows[j][n] * (-grad_f[n]) and grad_c0_inv[0] =
 * sum_n grad_out[n] * diff[n], both summed in double (either may be NULL).  The autograd of
 * the reference's step with an attached history sum (_CupyWeightedHistorySum.backward,
 * solver.py:136-146, and the PyTorch ops around it). */
int dfsnn_gl_history_step_backward(int dtype, const void* grad_out, const void* c0_inv,
                                   const void* const* rows, int row_begin, int row_end,
                                   const void* c_tilde, int coeff_base, const void* diff,
                                   void* grad_f, void* grad_rows, void* grad_coeff,
                                   void* grad_c0_inv, long long state_size, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ---- self-check (no reference counterpart) ----------------------------------------
 * The backward kernels divide the arctan surrogate's numerator by its denominator with an
 * FMA-corrected reciprocal (Markstein) instead of the IEEE division sequence.  This entry
 * point compares that quotient bit for bit with __fdiv_rn on the device: for each of the
 * n_numerators numerators a[k] (device array) and every float denominator b with biased
 * exponent in [exp_lo, exp_hi] (all 2^23 mantissas per exponent; b = 2 has exponent 128),
 * plus the refined reciprocal against __frcp_rn for every mantissa.  mismatches (device,
 * 2 x unsigned long long) receives {quotient mismatches, reciprocal mismatches}; it is
 * zeroed by the call.  Exponents outside [128, 191] (b < 2 or b > 2^64, where the kernels
 * take the IEEE division) are rejected with DFSNN_ERR_PARAM. */
int dfsnn_check_surrogate_quotient(const float* a, int n_numerators, int exp_lo, int exp_hi,
                                   unsigned long long* mismatches, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DFSNN_B200_H */
