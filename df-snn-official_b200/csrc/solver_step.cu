// solver_step.cu -- one step of the multi-term Grünwald–Letnikov integrator of the SNN wrapper
// path (spikeDE_dis/solver.py: forward_glmulti_cupy :3270-3369, backward_glmulti_cupy
// :2905-3002), fused into one kernel per state component:
//
//   y = c0_inv * (f - conv),   conv = sum_{j = row_begin}^{row_end - 1} c~[coeff_base - j] * row_j
//
// The reference stacks the history rows into a new tensor every step (O(k) copies per step),
// launches weighted_sum (:90-104) per 96-row chunk, adds the chunk results and then subtracts
// and scales with two more PyTorch kernels.  Here the rows are read in place through a device
// table of row pointers (each step's kernel registers its own output in the table), and the
// arithmetic keeps the reference's rounding steps:
//   chunk > 0  : per chunk of `chunk` rows one fused multiply-add chain from 0 (the weighted_sum
//                kernel, NVRTC --fmad=true), chunk results added left to right (the first one
//                is the running sum itself);
//   chunk == 0 : one chain over all rows (the adjoint's coefficient dot product);
//   chunk < 0  : conv = conv + RN(c*row) term by term from +0 (the PyTorch loop of :3323-3330).
//
// The backward (autograd of the step when the history sum is not detached) gives
// grad_f = c0_inv*g, grad_row_j = c~_j * (-grad_f) (the CuPy Function's double product rounded
// to the state type equals the single rounding of this product) and the reductions
// grad_coeff_j = sum_n row_j[n] * (-grad_f[n]) and grad_c0_inv = sum_n g[n] * diff[n] in double.
#include "../../include/dfsnn_b200.h"
#include "kernels.h"

namespace dfsnn {
namespace {

template <typename F>
__device__ __forceinline__ F fma_t(F a, F b, F c);
template <>
__device__ __forceinline__ float fma_t(float a, float b, float c) { return __fmaf_rn(a, b, c); }
template <>
__device__ __forceinline__ double fma_t(double a, double b, double c) { return __fma_rn(a, b, c); }

template <typename F>
__device__ __forceinline__ F add_t(F a, F b);
template <>
__device__ __forceinline__ float add_t(float a, float b) { return __fadd_rn(a, b); }
template <>
__device__ __forceinline__ double add_t(double a, double b) { return __dadd_rn(a, b); }

template <typename F>
__device__ __forceinline__ F sub_t(F a, F b);
template <>
__device__ __forceinline__ float sub_t(float a, float b) { return __fsub_rn(a, b); }
template <>
__device__ __forceinline__ double sub_t(double a, double b) { return __dsub_rn(a, b); }

template <typename F>
__device__ __forceinline__ F mul_t(F a, F b);
template <>
__device__ __forceinline__ float mul_t(float a, float b) { return __fmul_rn(a, b); }
template <>
__device__ __forceinline__ double mul_t(double a, double b) { return __dmul_rn(a, b); }

template <typename F>
struct StepArgs {
    const F* f;
    const F* const* rows;   // device table of row pointers
    F** table_out;          // same table, written at out_slot (NULL: no registration)
    int row_begin, row_end, coeff_base, chunk, out_slot;
    const F* c_tilde;
    const F* c0_inv;
    F* out;
    F* diff;                // optional f - conv
    long long S;
};

template <typename F>
__global__ void __launch_bounds__(256) gl_step(StepArgs<F> a) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (a.table_out && n == 0) a.table_out[a.out_slot] = a.out;
    if (n >= a.S) return;
    F conv = F(0);
    if (a.chunk < 0) {
        for (int j = a.row_begin; j < a.row_end; ++j)
            conv = add_t(conv, mul_t(a.c_tilde[a.coeff_base - j], a.rows[j][n]));
    } else {
        const int step = a.chunk > 0 ? a.chunk : (a.row_end - a.row_begin);
        bool first = true;
        for (int c0 = a.row_begin; c0 < a.row_end; c0 += step) {
            const int c1 = (c0 + step) < a.row_end ? (c0 + step) : a.row_end;
            F acc = F(0);
            for (int j = c0; j < c1; ++j) acc = fma_t(a.c_tilde[a.coeff_base - j], a.rows[j][n], acc);
            conv = first ? acc : add_t(conv, acc);
            first = false;
        }
    }
    const F d = sub_t(a.f[n], conv);
    a.out[n] = mul_t(*a.c0_inv, d);
    if (a.diff) a.diff[n] = d;
}

// Four consecutive elements per thread (S % 4 == 0, f / out / diff 16-byte aligned): every
// history row is read with 16-byte loads when its pointer is aligned (a uniform test: all
// threads see the same row), else with four scalar loads; the arithmetic per element is the
// scalar kernel's.
template <typename F>
struct Vec4;
template <>
struct Vec4<float> {
    using T = float4;
};
template <>
struct Vec4<double> {
    using T = double4;
};

template <typename F>
__device__ __forceinline__ void load4(const F* p, long long n, F (&v)[4]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0 && (sizeof(F) == 4 ||
                                                       (reinterpret_cast<uintptr_t>(p) & 31) == 0)) {
        const typename Vec4<F>::T q = *reinterpret_cast<const typename Vec4<F>::T*>(p + n);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = p[n + u];
    }
}

template <typename F>
__global__ void __launch_bounds__(256) gl_step4(StepArgs<F> a) {
    const long long n = 4 * ((long long)blockIdx.x * blockDim.x + threadIdx.x);
    if (a.table_out && n == 0) a.table_out[a.out_slot] = a.out;
    if (n >= a.S) return;
    F conv[4] = {F(0), F(0), F(0), F(0)};
    if (a.chunk < 0) {
        for (int j = a.row_begin; j < a.row_end; ++j) {
            const F c = a.c_tilde[a.coeff_base - j];
            F r[4];
            load4(a.rows[j], n, r);
#pragma unroll
            for (int u = 0; u < 4; ++u) conv[u] = add_t(conv[u], mul_t(c, r[u]));
        }
    } else {
        const int step = a.chunk > 0 ? a.chunk : (a.row_end - a.row_begin);
        bool first = true;
        for (int c0 = a.row_begin; c0 < a.row_end; c0 += step) {
            const int c1 = (c0 + step) < a.row_end ? (c0 + step) : a.row_end;
            F acc[4] = {F(0), F(0), F(0), F(0)};
#pragma unroll 4
            for (int j = c0; j < c1; ++j) {
                const F c = a.c_tilde[a.coeff_base - j];
                F r[4];
                load4(a.rows[j], n, r);
#pragma unroll
                for (int u = 0; u < 4; ++u) acc[u] = fma_t(c, r[u], acc[u]);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) conv[u] = first ? acc[u] : add_t(conv[u], acc[u]);
            first = false;
        }
    }
    const F c0 = *a.c0_inv;
    F fv[4];
    load4(a.f, n, fv);
    F y[4], d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        d[u] = sub_t(fv[u], conv[u]);
        y[u] = mul_t(c0, d[u]);
    }
    *reinterpret_cast<typename Vec4<F>::T*>(a.out + n) = {y[0], y[1], y[2], y[3]};
    if (a.diff) *reinterpret_cast<typename Vec4<F>::T*>(a.diff + n) = {d[0], d[1], d[2], d[3]};
}

template <typename F>
struct StepBwdArgs {
    const F* g;
    const F* c0_inv;
    const F* const* rows;
    int row_begin, row_end, coeff_base;
    const F* c_tilde;
    F* grad_f;
    F* grad_rows;       // [L, S] (NULL: not needed)
    long long S;
};

template <typename F>
__global__ void __launch_bounds__(256) gl_step_bwd(StepBwdArgs<F> a) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= a.S) return;
    const F gf = mul_t(*a.c0_inv, a.g[n]);
    a.grad_f[n] = gf;
    if (a.grad_rows) {
        const F gc = -gf;
        for (int j = a.row_begin; j < a.row_end; ++j)
            a.grad_rows[(long long)(j - a.row_begin) * a.S + n] = mul_t(a.c_tilde[a.coeff_base - j], gc);
    }
}

// part[(q) * slices + s] for q < L: sum over slice s of row_q[n] * (-c0_inv*g[n]);
// q == L: sum over slice s of g[n] * diff[n]
template <typename F>
__global__ void __launch_bounds__(256) gl_step_reduce(const F* g, const F* c0_inv,
                                                      const F* const* rows, int row_begin, int L,
                                                      const F* diff, long long S,
                                                      long long per, double* part) {
    __shared__ double red[256];
    const int q = blockIdx.y, s = blockIdx.x;
    const long long n0 = (long long)s * per;
    const long long n1 = (n0 + per) < S ? (n0 + per) : S;
    const F c0 = *c0_inv;
    double acc = 0.0;
    if (q < L) {
        const F* row = rows[row_begin + q];
        for (long long n = n0 + threadIdx.x; n < n1; n += blockDim.x)
            acc += (double)row[n] * (double)(-mul_t(c0, g[n]));
    } else if (diff) {
        for (long long n = n0 + threadIdx.x; n < n1; n += blockDim.x)
            acc += (double)g[n] * (double)diff[n];
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) part[(long long)q * gridDim.x + s] = red[0];
}

template <typename F>
__global__ void gl_step_finalize(const double* part, int slices, int rows, F* out) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= rows) return;
    double s = 0.0;
    for (int i = 0; i < slices; ++i) s += part[(long long)q * slices + i];
    out[q] = (F)s;
}

int reduce_slices(long long S) {
    long long s = (S + 65535) / 65536;
    if (s > 64) s = 64;
    return s < 1 ? 1 : (int)s;
}

template <typename F>
cudaError_t step_launch(const void* f, const void* const* rows, int row_begin, int row_end,
                        const void* c_tilde, int coeff_base, const void* c0_inv, int chunk,
                        void* out, void* diff, long long S, void** table, int out_slot,
                        cudaStream_t st) {
    StepArgs<F> a;
    a.f = static_cast<const F*>(f);
    a.rows = reinterpret_cast<const F* const*>(rows);
    a.table_out = reinterpret_cast<F**>(table);
    a.row_begin = row_begin;
    a.row_end = row_end;
    a.coeff_base = coeff_base;
    a.chunk = chunk;
    a.out_slot = out_slot;
    a.c_tilde = static_cast<const F*>(c_tilde);
    a.c0_inv = static_cast<const F*>(c0_inv);
    a.out = static_cast<F*>(out);
    a.diff = static_cast<F*>(diff);
    a.S = S;
    constexpr uintptr_t kAlign = sizeof(F) == 4 ? 15 : 31;
    const bool vec = S % 4 == 0 && ((reinterpret_cast<uintptr_t>(f) | reinterpret_cast<uintptr_t>(out) |
                                     reinterpret_cast<uintptr_t>(diff)) & kAlign) == 0;
    if (vec) {
        const long long blocks = S > 0 ? (S / 4 + 255) / 256 : 1;
        gl_step4<F><<<(unsigned)blocks, 256, 0, st>>>(a);
    } else {
        const long long blocks = S > 0 ? (S + 255) / 256 : 1;
        gl_step<F><<<(unsigned)blocks, 256, 0, st>>>(a);
    }
    return cudaGetLastError();
}

template <typename F>
cudaError_t step_bwd_launch(const void* g, const void* c0_inv, const void* const* rows,
                            int row_begin, int row_end, const void* c_tilde, int coeff_base,
                            const void* diff, void* grad_f, void* grad_rows, void* grad_coeff,
                            void* grad_c0_inv, double* part, long long S, cudaStream_t st) {
    StepBwdArgs<F> a;
    a.g = static_cast<const F*>(g);
    a.c0_inv = static_cast<const F*>(c0_inv);
    a.rows = reinterpret_cast<const F* const*>(rows);
    a.row_begin = row_begin;
    a.row_end = row_end;
    a.coeff_base = coeff_base;
    a.c_tilde = static_cast<const F*>(c_tilde);
    a.grad_f = static_cast<F*>(grad_f);
    a.grad_rows = static_cast<F*>(grad_rows);
    a.S = S;
    if (S > 0) {
        gl_step_bwd<F><<<(unsigned)((S + 255) / 256), 256, 0, st>>>(a);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const int L = row_end - row_begin;
    if (!grad_coeff && !grad_c0_inv) return cudaSuccess;
    const int slices = reduce_slices(S);
    const long long per = (S + slices - 1) / slices;
    // rows q < L reduce grad_coeff; q == L (the last grid row) reduces grad_c0_inv
    const dim3 grid((unsigned)slices, (unsigned)(L + 1));
    gl_step_reduce<F><<<grid, 256, 0, st>>>(a.g, a.c0_inv, a.rows, row_begin, L,
                                            static_cast<const F*>(grad_c0_inv ? diff : nullptr),
                                            S, per, part);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (grad_coeff) {
        gl_step_finalize<F><<<(L + 127) / 128 > 0 ? (L + 127) / 128 : 1, 128, 0, st>>>(
            part, slices, L, static_cast<F*>(grad_coeff));
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (grad_c0_inv) {
        gl_step_finalize<F><<<1, 32, 0, st>>>(part + (long long)L * slices, slices, 1,
                                              static_cast<F*>(grad_c0_inv));
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace

size_t gl_step_reduce_bytes(int L, long long S) {
    return (size_t)(L + 1) * (size_t)reduce_slices(S) * sizeof(double);
}

}  // namespace dfsnn

extern "C" size_t dfsnn_gl_history_step_workspace_size(int rows, long long state_size) {
    if (rows < 0 || state_size < 0) return 0;
    return dfsnn::gl_step_reduce_bytes(rows, state_size);
}

extern "C" int dfsnn_gl_history_step(int dtype, const void* f, const void* const* rows,
                                     int row_begin, int row_end, const void* c_tilde,
                                     int coeff_base, const void* c0_inv, int chunk, void* out,
                                     void* diff, long long state_size, void** table, int out_slot,
                                     void* stream) {
    if (dtype != DFSNN_F32 && dtype != DFSNN_F64) return DFSNN_ERR_PARAM;
    if (state_size < 0 || row_begin < 0 || row_end < row_begin) return DFSNN_ERR_SHAPE;
    if (!c0_inv || (row_end > row_begin && (!rows || !c_tilde))) return DFSNN_ERR_NULL;
    if (row_end > row_begin && coeff_base - (row_end - 1) < 0) return DFSNN_ERR_SHAPE;
    if (state_size > 0 && (!f || !out)) return DFSNN_ERR_NULL;
    if (table && out_slot < row_end) return DFSNN_ERR_SHAPE;   // never a row being read
    cudaError_t e = dtype == DFSNN_F32
        ? dfsnn::step_launch<float>(f, rows, row_begin, row_end, c_tilde, coeff_base, c0_inv,
                                    chunk, out, diff, state_size, table, out_slot,
                                    (cudaStream_t)stream)
        : dfsnn::step_launch<double>(f, rows, row_begin, row_end, c_tilde, coeff_base, c0_inv,
                                     chunk, out, diff, state_size, table, out_slot,
                                     (cudaStream_t)stream);
    return e == cudaSuccess ? DFSNN_OK : dfsnn::record_cuda_error(e);
}

extern "C" int dfsnn_gl_history_step_backward(int dtype, const void* grad_out, const void* c0_inv,
                                              const void* const* rows, int row_begin, int row_end,
                                              const void* c_tilde, int coeff_base,
                                              const void* diff, void* grad_f, void* grad_rows,
                                              void* grad_coeff, void* grad_c0_inv,
                                              long long state_size, void* workspace,
                                              size_t workspace_bytes, void* stream) {
    if (dtype != DFSNN_F32 && dtype != DFSNN_F64) return DFSNN_ERR_PARAM;
    if (state_size < 0 || row_begin < 0 || row_end < row_begin) return DFSNN_ERR_SHAPE;
    if (!c0_inv || (state_size > 0 && (!grad_out || !grad_f))) return DFSNN_ERR_NULL;
    const bool need_rows = grad_rows || grad_coeff;
    if (need_rows && row_end > row_begin && (!rows || !c_tilde)) return DFSNN_ERR_NULL;
    if (row_end > row_begin && coeff_base - (row_end - 1) < 0) return DFSNN_ERR_SHAPE;
    if (grad_c0_inv && state_size > 0 && !diff) return DFSNN_ERR_NULL;
    if ((grad_coeff || grad_c0_inv) &&
        (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 7u) != 0 ||
         workspace_bytes < dfsnn::gl_step_reduce_bytes(row_end - row_begin, state_size)))
        return DFSNN_ERR_WORKSPACE;
    cudaError_t e = dtype == DFSNN_F32
        ? dfsnn::step_bwd_launch<float>(grad_out, c0_inv, rows, row_begin, row_end, c_tilde,
                                        coeff_base, diff, grad_f, grad_rows, grad_coeff,
                                        grad_c0_inv, static_cast<double*>(workspace), state_size,
                                        (cudaStream_t)stream)
        : dfsnn::step_bwd_launch<double>(grad_out, c0_inv, rows, row_begin, row_end, c_tilde,
                                         coeff_base, diff, grad_f, grad_rows, grad_coeff,
                                         grad_c0_inv, static_cast<double*>(workspace),
                                         state_size, (cudaStream_t)stream);
    return e == cudaSuccess ? DFSNN_OK : dfsnn::record_cuda_error(e);
}
