/*
 * lif_fde_oracle.c -- CPU restatement of the DF-SNN LIFNeuronFDE hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle: tests/, __graft_entry__.smoke()
 * and the cpu_baseline / reference legs of bench.py may call it, as the checker or as
 * the timed CPU baseline.  Nothing in the CUDA product path links or calls it.
 *
 * Every function restates one reference CUDA kernel (CuPy RawKernel strings in
 * spikeDE_dis/fde_cupy_kernels_all.py, examples/cnn128/aligned_glmulti.py and
 * spikeDE_dis/direct_euler_cupy.py) operation by operation in IEEE fp32, so that the
 * CUDA kernels of this repository can be checked bit for bit:
 *   - the reference kernels are compiled by NVRTC with its default --fmad=true, which
 *     contracts a*b+c into one fused multiply-add; every such contraction is written
 *     here as an explicit fmaf() and the file is compiled with -ffp-contract=off;
 *   - the aligned kernels are compiled by the reference with --fmad=false, so their
 *     restatement uses no fmaf() at all;
 *   - divisions are IEEE round-to-nearest in both places.
 * Parameter-gradient reductions over neurons (torch.sum / torch.matmul in the
 * reference) are accumulated in double here: they are the precise value that both
 * the reference's fp32 reductions and the CUDA reductions approximate.
 *
 * Pinning: tests/test_oracle_golden.py checks this oracle against fixtures made by
 * running the reference's own torch code and the reference's own kernel sources
 * compiled for the host (oracle/build_ref.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define PI_HALF_F 1.57079632679489661923f
#define ALIGNED_PI_HALF_F 1.5707963267948966f

/* Arctan surrogate derivative as the fmad=true kernels compute it
 * (fde_cupy_kernels_all.py:143-146, :1862-1864): u = (pi/2*a)*z, a / (2*(1+u*u)). */
static inline float surr_fma(float z, float sg) {
    const float u = (PI_HALF_F * sg) * z;
    return sg / (2.0f * fmaf(u, u, 1.0f));
}

/* ------------------------------------------------------------------------------------
 * Single-order schemes: GL (fde_cupy_kernels_all.py:24-75, 77-163), TRAP (:327-381,
 * 383-472), PREDICTOR (:479-539, 541-637), GL1 (:170-260, 262-320).
 * w is the reversed weight table of T+1 entries (c_rev / trap_w / pred_w); at step k
 * the history term i<k uses w[T-k+i].
 * ---------------------------------------------------------------------------------- */
enum { ORC_GL = 0, ORC_TRAP = 1, ORC_PRED = 2, ORC_GL1 = 3, ORC_TRAP1 = 4, ORC_PRED1 = 5,
       ORC_EULER = 6 };
/* EULER = LIFEulerFunction (fde_cupy_kernels_all.py:2546-2756): v + dv, no history term. */
/* TRAP1 (fde_cupy_kernels_all.py:2018-2070) and PREDICTOR1 (:2278-2335) share the Kahan
 * forward; their updates are v + h_beta*dv - hist and v + h_beta*(w_T*dv + hist). */

static void single_forward_one(int scheme, const float* x, float v, const float* w,
                               float* spike, float* vseq, float* hv, int T, int64_t N, int64_t n,
                               float tau, float beta, float th, float h_beta, float gamma1) {
    const float trap_factor = fmaf(1.5f, beta, 0.5f);          /* :346 */
    const float pred_scale = h_beta / gamma1;                   /* :528 */
    for (int k = 0; k < T; ++k) {
        const float dv = (x[(int64_t)k * N + n] - v) / tau;    /* (-v + x)/tau */
        float hist = 0.0f;
        if (k > 0 && scheme != ORC_EULER) {                     /* Kahan, :52-63 */
            float sum = 0.0f, c = 0.0f;
            for (int i = 0; i < k; ++i) {
                const float y = fmaf(w[T - k + i], hv[i], -c);
                const float t = sum + y;
                c = (t - sum) - y;
                sum = t;
            }
            hist = sum;
        }
        float p;
        if (scheme == ORC_GL)        p = dv - hist;                              /* :66 */
        else if (scheme == ORC_GL1)  p = fmaf(h_beta, dv, -hist);                /* gl1 :213 */
        else if (scheme == ORC_TRAP) p = v + fmaf(trap_factor, dv, -hist);       /* :372 */
        else if (scheme == ORC_TRAP1) p = fmaf(h_beta, dv, v) - hist;            /* :2059 */
        else if (scheme == ORC_PRED1) p = fmaf(h_beta, fmaf(w[T], dv, hist), v); /* :2326 */
        else if (scheme == ORC_EULER) p = v + dv;                                 /* :2571 */
        else                         p = fmaf(pred_scale, fmaf(w[T], dv, hist), v); /* :528 */
        const float s = (p >= th) ? 1.0f : 0.0f;
        const float vn = p - s * th;
        spike[(int64_t)k * N + n] = s;
        vseq[(int64_t)k * N + n] = vn;
        hv[k] = (scheme == ORC_PRED || scheme == ORC_PRED1) ? (-vn) / tau : vn;   /* -v/tau */
        v = vn;
    }
}

void orc_single_forward(int scheme, const float* x, const float* v0, const float* w,
                        float* spike, float* vseq, int T, int64_t N, float tau, float beta,
                        float th, float h_beta, float gamma1) {
    #pragma omp parallel
    {
        float* hv = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n)
            single_forward_one(scheme, x, v0[n], w, spike, vseq, hv, T, N, n, tau, beta, th,
                               h_beta, gamma1);
        free(hv);
    }
}

/* Backward of the single-order schemes: the reference recomputes the forward and runs a
 * truncated reverse sweep (history detached).  The surrogate is evaluated at
 * v + spike*theta, rebuilt from the post-reset voltage (:137-146). */
void orc_single_backward(int scheme, const float* gS, const float* gV, const float* spike,
                         const float* vseq, const float* w, float* gx, float* gv0, int T,
                         int64_t N, float tau, float beta, float th, float sg, float h_beta,
                         float gamma1) {
    const float trap_factor = fmaf(1.5f, beta, 0.5f);
    const float pred_scale = h_beta / gamma1;
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        float gv = 0.0f;
        for (int t = T - 1; t >= 0; --t) {
            const int64_t o = (int64_t)t * N + n;
            gv = gv + gV[o];
            const float p = fmaf(spike[o], th, vseq[o]);
            const float surr = surr_fma(p - th, sg);
            gv = fmaf(gS[o], surr, gv);
            float gvm;
            if (scheme == ORC_GL) {                              /* :150-154 */
                gx[o] = gv / tau;
                gvm = (-gv) / tau;
            } else if (scheme == ORC_TRAP) {                     /* :459-463 */
                const float gsd = gv * trap_factor;
                gx[o] = gsd / tau;
                gvm = gv - gsd / tau;
            } else if (scheme == ORC_PRED) {                     /* :621-629 */
                const float gdc = (gv * pred_scale) * w[T];
                gx[o] = gdc / tau;
                gvm = gv - gdc / tau;
            } else if (scheme == ORC_EULER) {                    /* :2645-2647 */
                gx[o] = gv / tau;
                gvm = gv * (1.0f - 1.0f / tau);
            } else {                                             /* GL1 :296-312 */
                const float gd = h_beta * gv;
                gx[o] = gd / tau;
                gvm = (-gd) / tau;
                for (int i = 0; i < t; ++i) gvm = fmaf(-w[T - t + i], gv, gvm);
            }
            if (t > 0) gv = gvm; else gv0[n] = gvm;
        }
    }
}

/* TRAP1 / PREDICTOR1 backward (fde_cupy_kernels_all.py:2072-2161, :2337-2432): the reference
 * recomputes the trajectory with a plain fused multiply-add history sum (not the forward's
 * Kahan sum), then runs a reverse sweep whose history term touches only the current step's
 * gradient.  Restated operation by operation. */
void orc_single1_backward(int scheme, const float* gS, const float* gV, const float* x,
                          const float* v0, const float* w, float* gx, float* gv0, int T,
                          int64_t N, float tau, float th, float sg, float h_beta) {
    #pragma omp parallel
    {
        float* vl = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
        float* hv = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
        float* sp = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            float v = v0[n];
            for (int k = 0; k < T; ++k) {                        /* :2103-2124, :2371-2395 */
                const float dv = (x[(int64_t)k * N + n] - v) / tau;
                float hist = 0.0f;
                for (int i = 0; i < k; ++i) hist = fmaf(w[T - k + i], hv[i], hist);
                const float p = (scheme == ORC_TRAP1) ? fmaf(h_beta, dv, v) - hist
                                                      : fmaf(h_beta, fmaf(w[T], dv, hist), v);
                const float s = (p >= th) ? 1.0f : 0.0f;
                const float vn = p - s * th;
                vl[k] = vn;
                sp[k] = s;
                hv[k] = (scheme == ORC_TRAP1) ? vn : (-vn) / tau;
                v = vn;
            }
            float gv = 0.0f;
            for (int t = T - 1; t >= 0; --t) {                   /* :2128-2157, :2399-2428 */
                const int64_t o = (int64_t)t * N + n;
                gv = gv + gV[o];
                const float pp = fmaf(sp[t], th, vl[t]);
                gv = fmaf(gS[o], surr_fma(pp - th, sg), gv);
                float gvm;
                if (scheme == ORC_TRAP1) {
                    gx[o] = (h_beta * gv) / tau;
                    gvm = gv * (1.0f - h_beta / tau);
                    for (int i = 0; i < t; ++i) gvm = fmaf(-w[T - t + i], gv, gvm);
                } else {
                    const float hw = h_beta * w[T];
                    gx[o] = (hw * gv) / tau;
                    gvm = gv * (1.0f - hw / tau);
                    for (int i = 0; i < t; ++i) gvm = gvm - ((h_beta * w[T - t + i]) * gv) / tau;
                }
                gv = gvm;
            }
            gv0[n] = gv;
        }
        free(vl);
        free(hv);
        free(sp);
    }
}

/* ------------------------------------------------------------------------------------
 * History family with optional per-sample tables (neuron n belongs to sample n / (N/B);
 * per_batch: scale [T][B], W [T][B][T]; else scale [T], W [T][T]):
 *   mode 0 "GLX": VO-GL1 (fde_cupy_kernels_all.py:1594-1630) and FAGL1 (:1200-1233, scale
 *          = h_beta everywhere, scale == NULL): v_pre = s*drift - sum_i W v_hist_i
 *   mode 1 "VOPRED": VO-PREDICTOR (:1017-1056): history over the drift,
 *          v_pre = v0 + s*(drift + hist) + rm*(v - v0)
 * Outputs spike, v_pre and the history source (v_hist or drift); for VOPRED also the
 * drift-plus-history the parameter gradient needs (the reference recomputes it with a
 * torch.matmul; a reduction input, compared within tolerance).
 * ---------------------------------------------------------------------------------- */
static inline int64_t hf_w(int per_batch, int B, int T, int t, int b, int i) {
    return per_batch ? ((int64_t)(t * B + b) * T + i) : ((int64_t)t * T + i);
}
static inline float hf_s(const float* scale, float hb, int per_batch, int B, int t, int b) {
    return scale ? scale[per_batch ? (t * B + b) : t] : hb;
}

void orc_hfam_forward(int mode, const float* x, const float* v0, const float* scale, float hb,
                      const float* W, int per_batch, int B, float* spike, float* vpre,
                      float* hsrc, float* aux, int T, int64_t N, float tau, float th, float rm) {
    const int64_t F = N / B;
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const int b = (int)(n / F);
        float v = v0[n];
        for (int t = 0; t < T; ++t) {
            const int64_t o = (int64_t)t * N + n;
            const float drift = (x[o] - v) / tau;                        /* (-v + x)/tau */
            float hist = 0.0f;
            for (int i = 0; i < t; ++i)
                hist = fmaf(W[hf_w(per_batch, B, T, t, b, i)], hsrc[(int64_t)i * N + n], hist);
            const float sv = hf_s(scale, hb, per_batch, B, t, b);
            float p;
            if (mode == 0) {
                p = fmaf(sv, drift, -hist);                               /* :1624 / :1226 */
                if (aux) aux[o] = drift;
            } else {
                p = fmaf(rm, v - v0[n], fmaf(sv, drift + hist, v0[n]));  /* :1047 */
                hsrc[o] = drift;
                if (aux) aux[o] = drift + hist;
            }
            const float sp = (p >= th) ? 1.0f : 0.0f;
            spike[o] = sp;
            vpre[o] = p;
            v = p - sp * th;
            if (mode == 0) hsrc[o] = v;
        }
    }
}

/* hist_mode 0: VO-GL1 / FAGL1 truncated (:1632-1668, :1235-1272): grad_v_next =
 *   -gp * (s/tau + sum_i W[t,i]); 1: full history (:1670-1709, :1274-1312); 2: VO-PREDICTOR
 *   truncated (:1058-1096): grad_v_next = gp * (rm - s/tau). */
void orc_hfam_backward(int hist_mode, const float* gS, const float* scale, float hb,
                       const float* W, int per_batch, int B, const float* vpre, float* gx,
                       float* gv0, float* gpre, int T, int64_t N, float tau, float th, float sg,
                       float rm) {
    const int64_t F = N / B;
    #pragma omp parallel
    {
        float* A = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            const int b = (int)(n / F);
            for (int t = 0; t < T; ++t) A[t] = 0.0f;
            float gvn = 0.0f, ginit = 0.0f;
            for (int t = T - 1; t >= 0; --t) {
                const int64_t o = (int64_t)t * N + n;
                const float sur = surr_fma(vpre[o] - th, sg);
                const float sv = hf_s(scale, hb, per_batch, B, t, b);
                const float gp = fmaf(gS[o], sur, hist_mode == 1 ? A[t] : gvn);
                gpre[o] = gp;
                gx[o] = (gp * sv) / tau;
                if (hist_mode == 0) {
                    float hsum = 0.0f;
                    for (int i = 0; i < t; ++i) hsum = hsum + W[hf_w(per_batch, B, T, t, b, i)];
                    gvn = (-gp) * (sv / tau + hsum);
                } else if (hist_mode == 2) {
                    gvn = gp * (rm - sv / tau);
                } else {
                    const float prev = ((-gp) * sv) / tau;
                    if (t == 0) ginit = ginit + prev; else A[t - 1] = A[t - 1] + prev;
                    for (int i = 0; i < t; ++i)
                        A[i] = fmaf(-W[hf_w(per_batch, B, T, t, b, i)], gp, A[i]);
                }
            }
            gv0[n] = hist_mode == 1 ? ginit : gvn;
        }
        free(A);
    }
}

/* Per-sample parameter gradients in double: gs[t][b] = sum_{n in b} G[t,n] E[t,n] (gs may be
 * NULL) and gW[t][b][i] = sign * sum_{n in b} G[t,n] * (scale ? scale[t][b] : 1) * V[i,n],
 * zero for i >= t when lower_only (torch.sum / einsum / matmul of the reference Functions:
 * :1829-1838, :1167-1181, :1478-1497). */
void orc_hfam_param_grads(const float* G, const float* V, const float* E, const float* scale,
                          int per_batch, int B, int T, int64_t N, double sign, int lower_only,
                          double* gs, double* gW) {
    const int64_t F = N / B;
    #pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)T * B; ++row) {
        const int t = (int)(row / B), b = (int)(row % B);
        const int ob = per_batch ? b : 0;
        const double sv = scale ? (double)scale[per_batch ? (t * B + b) : t] : 1.0;
        double s = 0.0;
        for (int64_t f = 0; f < F; ++f) {
            const int64_t n = (int64_t)b * F + f;
            if (E) s += (double)G[(int64_t)t * N + n] * (double)E[(int64_t)t * N + n];
        }
        if (gs) {
            if (per_batch) gs[t * B + b] = s;
            else {
                #pragma omp atomic
                gs[t] += s;
            }
        }
        for (int i = 0; i < T; ++i) {
            double acc = 0.0;
            if (!(lower_only && i >= t))
                for (int64_t f = 0; f < F; ++f) {
                    const int64_t n = (int64_t)b * F + f;
                    acc += (double)G[(int64_t)t * N + n] * sv * (double)V[(int64_t)i * N + n];
                }
            const int64_t o = per_batch ? ((int64_t)(t * B + ob) * T + i) : ((int64_t)t * T + i);
            if (per_batch) gW[o] = sign * acc;
            else {
                #pragma omp atomic
                gW[o] += sign * acc;
            }
        }
    }
}

/* ------------------------------------------------------------------------------------
 * Library glmulti: forward = lif_fde_vo_gl1_forward_kernel with per_batch=0
 * (fde_cupy_kernels_all.py:1594-1630); backward = lif_fde_glmulti_backward_kernel
 * (:1845-1875, truncated) or lif_fde_glmulti_full_backward_kernel (:1877-1913, full);
 * parameter gradients = torch.sum(grad_pre*drift,1) and -grad_pre @ v_hist^T
 * (:1999-2009).
 * ---------------------------------------------------------------------------------- */
void orc_glmulti_forward(const float* x, const float* v0, const float* scale, const float* W,
                         float* spike, float* vpre, float* vhist, float* drift, int T, int64_t N,
                         float tau, float th) {
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        float v = v0[n];
        for (int t = 0; t < T; ++t) {
            const int64_t o = (int64_t)t * N + n;
            const float d = (x[o] - v) / tau;
            float hist = 0.0f;
            for (int i = 0; i < t; ++i) hist = fmaf(W[t * T + i], vhist[(int64_t)i * N + n], hist);
            const float p = fmaf(scale[t], d, -hist);
            const float s = (p >= th) ? 1.0f : 0.0f;
            vpre[o] = p;
            drift[o] = d;
            spike[o] = s;
            v = p - s * th;
            vhist[o] = v;
        }
    }
}

void orc_glmulti_backward(int full, const float* gS, const float* scale, const float* W,
                          const float* vpre, float* gx, float* gv0, float* gpre, int T, int64_t N,
                          float tau, float th, float sg) {
    #pragma omp parallel
    {
        float* A = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            if (!full) {
                float gvn = 0.0f;
                for (int t = T - 1; t >= 0; --t) {
                    const int64_t o = (int64_t)t * N + n;
                    const float surr = surr_fma(vpre[o] - th, sg);
                    const float gp = fmaf(gS[o], surr, gvn);
                    gpre[o] = gp;
                    gx[o] = (gp * scale[t]) / tau;
                    gvn = ((-gp) * scale[t]) / tau;
                }
                gv0[n] = gvn;
            } else {
                for (int t = 0; t < T; ++t) A[t] = 0.0f;
                float ginit = 0.0f;
                for (int t = T - 1; t >= 0; --t) {
                    const int64_t o = (int64_t)t * N + n;
                    const float surr = surr_fma(vpre[o] - th, sg);
                    const float gp = fmaf(gS[o], surr, A[t]);
                    gpre[o] = gp;
                    const float gd = gp * scale[t];
                    gx[o] = gd / tau;
                    const float prev = (-gd) / tau;
                    if (t == 0) ginit = ginit + prev; else A[t - 1] = A[t - 1] + prev;
                    for (int i = 0; i < t; ++i) A[i] = fmaf(-W[t * T + i], gp, A[i]);
                }
                gv0[n] = ginit;
            }
        }
        free(A);
    }
}

/* Reductions over neurons in a fixed chunk order, independent of the thread count. */
#define ORC_CHUNK 4096

void orc_glmulti_param_grads(const float* gpre, const float* drift, const float* vhist,
                             double* gs, double* gW, int T, int64_t N) {
    const int64_t nchunks = (N + ORC_CHUNK - 1) / ORC_CHUNK;
    const int P = T + T * T;
    double* part = (double*)calloc((size_t)(nchunks > 0 ? nchunks : 1) * (size_t)P, sizeof(double));
    #pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < nchunks; ++c) {
        double* acc = part + (size_t)c * P;
        const int64_t n1 = (c + 1) * ORC_CHUNK < N ? (c + 1) * ORC_CHUNK : N;
        for (int t = 0; t < T; ++t) {
            const float* g = gpre + (int64_t)t * N;
            const float* d = drift + (int64_t)t * N;
            double s = 0.0;
            for (int64_t n = c * ORC_CHUNK; n < n1; ++n) s += (double)g[n] * (double)d[n];
            acc[t] = s;
            for (int i = 0; i < T; ++i) {
                const float* h = vhist + (int64_t)i * N;
                double w = 0.0;
                for (int64_t n = c * ORC_CHUNK; n < n1; ++n) w += (double)g[n] * (double)h[n];
                acc[T + t * T + i] = -w;
            }
        }
    }
    for (int k = 0; k < P; ++k) {
        double s = 0.0;
        for (int64_t c = 0; c < nchunks; ++c) s += part[(size_t)c * P + k];
        if (k < T) gs[k] = s; else gW[k - T] = s;
    }
    free(part);
}

/* ------------------------------------------------------------------------------------
 * Aligned glmulti (examples/cnn128/aligned_glmulti.py): aligned_forward (:7-17),
 * aligned_backward (:20-32) and the parameter gradients of AlignedGLMulti.backward
 * (aligned_scale :33-41 summed over chunks, and -(ga@h^T)*tril(-1), :141-144).
 * Compiled by the reference with --fmad=false: no fused multiply-adds here.
 * ---------------------------------------------------------------------------------- */
void orc_aligned_forward(const float* x, const float* v0, const float* a, const float* w,
                         float* s, float* p, float* hist, int T, int64_t N, float tau, float th) {
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        float v = v0[n];
        for (int t = 0; t < T; ++t) {
            const int64_t o = (int64_t)t * N + n;
            const float d = (x[o] - v) / tau;
            const float pred = v + d;
            const float spike = pred >= th ? 1.0f : 0.0f;
            float h = 0.0f;
            for (int j = 0; j < t; ++j) {
                const float prod = w[t * T + j] * hist[(int64_t)j * N + n];
                h = h + prod;
            }
            const float f = d - (spike * th) / tau;
            const float af = a[t] * f;
            v = af - h;
            s[o] = spike;
            p[o] = pred;
            hist[o] = v;
        }
    }
}

void orc_aligned_backward(const float* g, const float* a, const float* w, const float* p,
                          float* gx, float* gv, float* ga, int T, int64_t N, float tau, float th,
                          float sg, float rho) {
    #pragma omp parallel
    {
        float* adj = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
        #pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            for (int t = 0; t < T; ++t) adj[t] = 0.0f;
            for (int t = T - 1; t >= 0; --t) {
                const int64_t o = (int64_t)t * N + n;
                const float zc = ALIGNED_PI_HALF_F * sg;
                const float z = zc * (p[o] - th);
                const float zz = z * z;
                const float den = 2.0f * (1.0f + zz);
                const float gsg = g[o] * sg;
                const float q = gsg / den;
                const float r = adj[t];
                ga[o] = r;
                const float ra = r * a[t];
                gx[o] = (q + ra) / tau;
                const float inv = 1.0f / tau;
                const float qd = q * (1.0f - inv);
                const float prev = qd - ra / tau;
                if (t) adj[t - 1] = adj[t - 1] + prev; else gv[n] = prev;
                for (int j = 0; j < t; ++j) {
                    const float rw = rho * w[t * T + j];
                    const float m = rw * r;
                    adj[j] = adj[j] - m;
                }
            }
        }
        free(adj);
    }
}

void orc_aligned_param_grads(const float* ga, const float* hist, const float* w, const float* a,
                             double* gs, double* gw, int T, int64_t N) {
    const int64_t nchunks = (N + ORC_CHUNK - 1) / ORC_CHUNK;
    const int P = T + T * T;
    double* part = (double*)calloc((size_t)(nchunks > 0 ? nchunks : 1) * (size_t)P, sizeof(double));
    #pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < nchunks; ++c) {
        double* acc = part + (size_t)c * P;
        const int64_t n1 = (c + 1) * ORC_CHUNK < N ? (c + 1) * ORC_CHUNK : N;
        for (int64_t n = c * ORC_CHUNK; n < n1; ++n) {
            for (int t = 0; t < T; ++t) {
                float h = 0.0f;
                for (int j = 0; j < t; ++j) {
                    const float prod = w[t * T + j] * hist[(int64_t)j * N + n];
                    h = h + prod;
                }
                const float r = ga[(int64_t)t * N + n];
                const float term = (r * (hist[(int64_t)t * N + n] + h)) / a[t];
                acc[t] += (double)term;
                for (int j = 0; j < t; ++j)
                    acc[T + t * T + j] -= (double)r * (double)hist[(int64_t)j * N + n];
            }
        }
    }
    for (int k = 0; k < P; ++k) {
        double s = 0.0;
        for (int64_t c = 0; c < nchunks; ++c) s += part[(size_t)c * P + k];
        if (k < T) gs[k] = s; else gw[k - T] = s;
    }
    free(part);
}

/* ------------------------------------------------------------------------------------
 * Direct LIF-like Euler (spikeDE_dis/direct_euler_cupy.py:22-58 forward, :66-131
 * backward).  The reference accumulates the three scalar gradients with one atomicAdd
 * per thread; here they are summed in double.
 * ---------------------------------------------------------------------------------- */
void orc_euler_forward(const float* x, const float* z0, float* spike, float* zpre, float* sin_,
                       float* zfinal, int T, int64_t N, float in_scale, float gain, float bias,
                       float tau, float th, float step, float reset_strength, float sdt) {
    #pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        float z = z0[n];
        for (int t = 0; t < T; ++t) {
            const int64_t o = (int64_t)t * N + n;
            const float cur = x[o];
            const float dz = fmaf(cur, in_scale, -z) / tau;          /* (-z + cur*scale)/tau */
            const float sv = fmaf(sdt, dz, z);                       /* z + dt*dz */
            const float si = fmaf(sv, gain, bias) - th;              /* sv*gain + bias - th */
            const float s = si >= 0.0f ? 1.0f : 0.0f;
            zpre[o] = z;
            sin_[o] = si;
            spike[o] = s;
            const float rs = ((reset_strength * s) * th) / tau;
            z = fmaf(step, dz - rs, z);                              /* z + step*(dz - ...) */
        }
        zfinal[n] = z;
    }
}

void orc_euler_backward(const float* gS, const float* gzf, const float* x, const float* zpre,
                        const float* sin_, float* gx, float* gz0, double* g3, int T, int64_t N,
                        float in_scale, float gain, float tau, float step, float sg, float sdt) {
    const int64_t nchunks = (N + ORC_CHUNK - 1) / ORC_CHUNK;
    double* part = (double*)calloc((size_t)(nchunks > 0 ? nchunks : 1) * 3, sizeof(double));
    #pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < nchunks; ++c) {
        const int64_t n1 = (c + 1) * ORC_CHUNK < N ? (c + 1) * ORC_CHUNK : N;
        double a0 = 0.0, a1 = 0.0, a2 = 0.0;
        for (int64_t n = c * ORC_CHUNK; n < n1; ++n) {
            float gzn = gzf ? gzf[n] : 0.0f;
            float ls = 0.0f, lg = 0.0f, lb = 0.0f;
            for (int t = T - 1; t >= 0; --t) {
                const int64_t o = (int64_t)t * N + n;
                const float z = zpre[o];
                const float cur = x[o];
                const float si = sin_[o];
                const float dz_dz = -1.0f / tau;
                const float dz_dx = in_scale / tau;
                const float dz_ds = cur / tau;
                const float sv_dz = fmaf(sdt, dz_dz, 1.0f);
                const float sv_dx = sdt * dz_dx;
                const float sv_ds = sdt * dz_ds;
                const float sv = fmaf(z, sv_dz, cur * sv_dx);
                const float surr = surr_fma(si, sg);
                const float gsi = gS[o] * surr;
                lg = fmaf(gsi, sv, lg);
                lb = lb + gsi;
                const float gsv = gsi * gain;
                const float one_m = 1.0f - step / tau;
                const float gz = fmaf(gzn, one_m, gsv * sv_dz);
                gx[o] = fmaf(gzn, step * dz_dx, gsv * sv_dx);
                ls = ls + fmaf(gzn, step * dz_ds, gsv * sv_ds);
                gzn = gz;
            }
            gz0[n] = gzn;
            a0 += ls; a1 += lg; a2 += lb;
        }
        part[c * 3 + 0] = a0; part[c * 3 + 1] = a1; part[c * 3 + 2] = a2;
    }
    g3[0] = g3[1] = g3[2] = 0.0;
    for (int64_t c = 0; c < nchunks; ++c) {
        g3[0] += part[c * 3 + 0]; g3[1] += part[c * 3 + 1]; g3[2] += part[c * 3 + 2];
    }
    free(part);
}

/* Set the OpenMP thread count of the calling thread's later parallel regions (the oracle's and
 * those of any library sharing this OpenMP runtime, e.g. the host build of the reference
 * kernels).  Launchers such as torchrun export OMP_NUM_THREADS=1; the CPU baseline overrides it
 * with every host thread it may use. */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
    extern void omp_set_num_threads(int);
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* Number of OpenMP threads the oracle runs with (for the cpu_baseline "cores" field). */
int orc_num_threads(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------------------------------
 * Multi-term GL integrator step of the SNN wrapper path (spikeDE_dis/solver.py):
 *   out[n] = c0_inv * (f[n] - conv[n]),  conv[n] = sum_{r < L} coef[r] * hist[r*S + n]
 * chunk > 0: forward_glmulti_cupy (:3331-3358) -- per chunk of `chunk` rows the weighted_sum
 *            kernel (:90-104, acc += coeff[j]*history[...], one fma per term under NVRTC
 *            --fmad=true), chunk results summed left to right by PyTorch adds;
 * chunk == 0: one fma chain over all rows (the adjoint's dot product, :2976-2987, whose
 *            cuBLAS summation order is unspecified; this is the order the kernels use);
 * chunk < 0: the forward's PyTorch loop for history_chunk_size <= 0 (:3323-3330),
 *            conv = conv + coef*row with both operations rounded.
 * ------------------------------------------------------------------------------------- */
#define ORC_GL_STEP(NAME, F, FMA)                                                          \
void NAME(const F* f, const F* hist, const F* coef, int L, int64_t S, F c0_inv, int chunk,  \
          F* out) {                                                                        \
    _Pragma("omp parallel for schedule(static)")                                           \
    for (int64_t n = 0; n < S; ++n) {                                                      \
        F conv = (F)0;                                                                     \
        if (chunk < 0) {                                                                   \
            for (int r = 0; r < L; ++r) {                                                  \
                const F p = coef[r] * hist[(int64_t)r * S + n];                            \
                conv = conv + p;                                                           \
            }                                                                              \
        } else {                                                                           \
            const int step = chunk > 0 ? chunk : (L > 0 ? L : 1);                          \
            for (int c0 = 0; c0 < L; c0 += step) {                                         \
                const int c1 = c0 + step < L ? c0 + step : L;                              \
                F acc = (F)0;                                                              \
                for (int r = c0; r < c1; ++r) acc = FMA(coef[r], hist[(int64_t)r * S + n], acc); \
                conv = c0 == 0 ? acc : conv + acc;                                         \
            }                                                                              \
        }                                                                                  \
        out[n] = c0_inv * (f[n] - conv);                                                   \
    }                                                                                      \
}
ORC_GL_STEP(orc_gl_step_f32, float, fmaf)
ORC_GL_STEP(orc_gl_step_f64, double, fma)
