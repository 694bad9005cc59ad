// param_long.cu -- parameter-gradient reductions over [T, N] scratch arrays written by a
// backward sweep:
//   d[t]    = sum_n G[t,n] * E[t,n]   (kDiagProduct)   or   sum_n E[t,n]   (kDiagSum)
//   M[t,i]  = sum_n G[t,n] * V[i,n]
// i.e. the reference's torch.sum(grad_pre*drift) + torch.matmul(grad_pre, v_hist^T)
// (fde_cupy_kernels_all.py:1999-2009), aligned_scale + ga@h^T (aligned_glmulti.py:33-41,
// :141-144), and the per-sample sums / einsums of the VO-GL1, FAGL1 and VO-PREDICTOR
// Functions (fde_cupy_kernels_all.py:1829-1838, :1478-1497, :1167-1181).
//
// Neurons are split into B samples of F consecutive neurons and each sample into `chunks`
// segments; block row s = b*chunks + c reduces segment c of sample b and writes partial row
// s of [T + T*T] doubles (d, then M row-major).  Nothing crosses a sample boundary, so a
// caller sums the rows of one sample for per-sample results or all rows for shared ones,
// in a fixed order -- deterministic, no atomics.
//
// Two kernels:
//  * param_long: any T.  Grid (rows, tiles, tiles); block (s, bt, bi) computes the 64 x 64
//    output tile (bt, bi), each of its 256 threads a 4 x 4 block, from chunks of 32 neurons
//    staged through shared memory, multiplied in fp32 and folded into doubles per chunk.
//  * param_small<TB> (T <= TB, TB = 8, 16, 32, 64): one block per row computes all T x T
//    outputs.  Chunks of
//    2048/T neurons stream into padded shared-memory rows by 4-byte cp.async (any alignment,
//    zero-filled past the segment) through a 4-stage pipeline, three chunks ahead of the
//    products (one ahead left the kernel waiting on DRAM latency at ~2 TB/s).  Threads form groups of (T/4)^2, each thread a 4 x 4 block of M; the
//    groups split a chunk by 4-neuron quads (LDS.128 of each G and V row), and the group
//    results are summed in a fixed order at the end.  About one shared-memory wavefront per
//    neuron, so the kernel runs at the speed of its global loads.
#include "kernels.h"
#include "lif_common.cuh"

namespace dfsnn {

namespace {

constexpr int kLT = 64;      // output tile edge (param_long)
constexpr int kLK = 32;      // neurons per chunk (param_long)

struct Segment {
    long long nb, ne;        // neuron range [nb, ne) of this block row
};

__device__ __forceinline__ Segment row_segment(long long F, int chunks, long long per) {
    const long long b = blockIdx.x / chunks, c = blockIdx.x % chunks;
    const long long s0 = b * F + c * per;
    const long long send = b * F + F;
    return {s0, (s0 + per) < send ? (s0 + per) : send};
}

template <int DIAG>
__global__ void __launch_bounds__(256) param_long(const float* G, const float* V, const float* E,
                                                  int T, long long N, long long F, int chunks,
                                                  long long per, double* part) {
    __shared__ float sG[kLT][kLK + 1];
    __shared__ float sV[kLT][kLK + 1];
    __shared__ float sE[kLT][kLK + 1];
    const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
    const int t0 = blockIdx.y * kLT, i0 = blockIdx.z * kLT;
    const bool diag = DIAG != kDiagNone && blockIdx.y == blockIdx.z;
    const Segment sg = row_segment(F, chunks, per);
    double acc[4][4], accs = 0.0;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.0;
    for (long long k0 = sg.nb; k0 < sg.ne; k0 += kLK) {
        // stage rows t0.. of G (and E on the diagonal) and rows i0.. of V, zeros outside
        for (int e = tid; e < kLT * kLK; e += 256) {
            const int row = e / kLK, k = e % kLK;
            const long long n = k0 + k;
            const bool okn = n < sg.ne;
            sG[row][k] = (okn && t0 + row < T) ? G[(long long)(t0 + row) * N + n] : 0.0f;
            sV[row][k] = (okn && i0 + row < T) ? V[(long long)(i0 + row) * N + n] : 0.0f;
            if (diag) sE[row][k] = (okn && t0 + row < T) ? E[(long long)(t0 + row) * N + n] : 0.0f;
        }
        __syncthreads();
        float pc[4][4], ps = 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) pc[r][c] = 0.0f;
#pragma unroll 8
        for (int k = 0; k < kLK; ++k) {
            float g[4], v[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) g[r] = sG[4 * ty + r][k];
#pragma unroll
            for (int c = 0; c < 4; ++c) v[c] = sV[4 * tx + c][k];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) pc[r][c] = __fmaf_rn(g[r], v[c], pc[r][c]);
        }
        if (diag && tx < 4) {
            const int row = 4 * ty + tx;
#pragma unroll 8
            for (int k = 0; k < kLK; ++k)
                ps = DIAG == kDiagProduct ? __fmaf_rn(sG[row][k], sE[row][k], ps)
                                          : __fadd_rn(ps, sE[row][k]);
            accs += (double)ps;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] += (double)pc[r][c];
        __syncthreads();
    }
    double* row = part + (size_t)blockIdx.x * (size_t)(T + T * T);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int t = t0 + 4 * ty + r;
        if (t >= T) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int i = i0 + 4 * tx + c;
            if (i < T) row[T + t * T + i] = acc[r][c];
        }
    }
    if (blockIdx.y == blockIdx.z && tx < 4 && t0 + 4 * ty + tx < T)
        row[t0 + 4 * ty + tx] = diag ? accs : 0.0;
}

// ---- T <= 64 -------------------------------------------------------------------------
// Template bucket TB in {8, 16, 32, 64}, runtime T <= TB (rows T..TB-1 are staged as zeros).
template <int TB, int DIAG>
struct SmallCfg {
    static constexpr int kK = 2048 / TB;            // neurons per chunk: 2048 words per array
    // padded row: with thread (ty, tx) reading rows ty + kSt*r / tx + kSt*c, the rows of one
    // 16-byte load are consecutive; 8 banks per row (TB <= 16, two quads per warp) or 4 banks
    // per row (TB >= 32, up to 8 rows per warp) put them in distinct bank groups
    static constexpr int kRS = kK + (TB >= 32 ? 4 : 8);
    static constexpr int kNA = DIAG == kDiagNone ? 2 : 3;   // staged arrays: G, V (, E)
    static constexpr int kSt = TB / 4;
    static constexpr int kGS = kSt * kSt;           // threads per group
    static constexpr int kNG = 256 / kGS;           // groups per block
    static constexpr int kQ = kK / 4;               // quads per chunk
    static constexpr int kStages = 4;               // chunks in flight: kStages - 1 ahead
    static constexpr int kStageFloats = kNA * TB * kRS;
    static constexpr int kStage = kStages * kStageFloats * 4;
    static constexpr int kReduce = kNG * (TB * TB + TB) * 8;
    static constexpr int kBytes = kStage > kReduce ? kStage : kReduce;
    static_assert(kQ % kNG == 0, "every group takes the same number of quads");
};

// 4-byte asynchronous copy global -> shared (LDGSTS); src_bytes 0 fills the word with zero
__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int PENDING>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(PENDING) : "memory");
}

// stage the chunk starting at neuron k0: word e = tid + 256 j of each array is row e / kK,
// column e % kK (a warp covers consecutive neurons of one row); rows >= T read as zeros
template <int TB, int DIAG>
__device__ __forceinline__ void small_stage(float* st, const float* G, const float* V,
                                            const float* E, int T, long long N, long long k0,
                                            long long ne) {
    using C = SmallCfg<TB, DIAG>;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int e = threadIdx.x + 256 * j;
        const int row = e / C::kK, col = e % C::kK;
        const long long n = k0 + col;
        const bool ok = n < ne && row < T;
        const long long off = ok ? (long long)row * N + n : 0;   // a valid address always
        cp_async4(st + row * C::kRS + col, G + off, ok);
        cp_async4(st + (TB + row) * C::kRS + col, V + off, ok);
        if (DIAG != kDiagNone) cp_async4(st + (2 * TB + row) * C::kRS + col, E + off, ok);
    }
}

template <int TB, int DIAG>
__global__ void __launch_bounds__(256) param_small(const float* __restrict__ G,
                                                   const float* __restrict__ V,
                                                   const float* __restrict__ E, int T,
                                                   long long N, long long F, int chunks,
                                                   long long per, double* part) {
    using C = SmallCfg<TB, DIAG>;
    constexpr int kSt = C::kSt;
    extern __shared__ __align__(16) unsigned char smem[];
    float* stages = reinterpret_cast<float*>(smem);
    const int tid = threadIdx.x;
    const int grp = tid / C::kGS, lt = tid % C::kGS;
    const int ty = lt / kSt, tx = lt % kSt;
    // Thread (ty, tx) owns M[ty + kSt r][tx + kSt c], r, c < 4.  Diagonal d[t]: for kSt <= 4
    // row t = ty + kSt r is taken by the thread with tx = r mod kSt (kDR rows each); for
    // kSt > 4 by the thread with tx == ty (all four of its rows).
    constexpr int kDR = kSt <= 4 ? 4 / kSt : 4;
    const bool dthread = kSt <= 4 || tx == ty;
    const Segment sg = row_segment(F, chunks, per);
    const long long nchunks = sg.ne > sg.nb ? (sg.ne - sg.nb + C::kK - 1) / C::kK : 0;
    double acc[4][4], dacc[kDR];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.0;
#pragma unroll
    for (int k = 0; k < kDR; ++k) dacc[k] = 0.0;
    // prologue: kStages - 1 chunks in flight (one commit group each, empty past the end)
#pragma unroll
    for (int s = 0; s < C::kStages - 1; ++s) {
        if (s < nchunks)
            small_stage<TB, DIAG>(stages + s * C::kStageFloats, G, V, E, T, N,
                                  sg.nb + s * C::kK, sg.ne);
        cp_async_commit();
    }
    for (long long it = 0; it < nchunks; ++it) {
        cp_async_wait<C::kStages - 2>();      // chunk `it` has landed
        __syncthreads();                      // ... for every thread; stage it-1 is free
        {
            const long long nx = it + C::kStages - 1;
            if (nx < nchunks)
                small_stage<TB, DIAG>(stages + (int)(nx % C::kStages) * C::kStageFloats, G, V,
                                      E, T, N, sg.nb + nx * C::kK, sg.ne);
            cp_async_commit();
        }
        const float* sG = stages + (int)(it % C::kStages) * C::kStageFloats;
        const float* sV = sG + TB * C::kRS;
        const float* sE = sV + TB * C::kRS;
        float pc[4][4], pd[kDR];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) pc[r][c] = 0.0f;
#pragma unroll
        for (int k = 0; k < kDR; ++k) pd[k] = 0.0f;
#pragma unroll
        for (int qi = 0; qi < C::kQ / C::kNG; ++qi) {
            const int q = grp + qi * C::kNG;
            float4 g[4], v[4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
                g[r] = *reinterpret_cast<const float4*>(sG + (ty + kSt * r) * C::kRS + 4 * q);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                v[c] = *reinterpret_cast<const float4*>(sV + (tx + kSt * c) * C::kRS + 4 * q);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    pc[r][c] = __fmaf_rn(g[r].x, v[c].x, pc[r][c]);
                    pc[r][c] = __fmaf_rn(g[r].y, v[c].y, pc[r][c]);
                    pc[r][c] = __fmaf_rn(g[r].z, v[c].z, pc[r][c]);
                    pc[r][c] = __fmaf_rn(g[r].w, v[c].w, pc[r][c]);
                }
            if (DIAG != kDiagNone && dthread) {
#pragma unroll
                for (int k = 0; k < kDR; ++k) {
                    const int r = kSt <= 4 ? tx + kSt * k : k;   // this thread's diagonal row
                    const float4 e = *reinterpret_cast<const float4*>(
                        sE + (ty + kSt * r) * C::kRS + 4 * q);
                    if (DIAG == kDiagProduct) {
                        float4 gg = g[0];                        // g[r] without a dynamic index
#pragma unroll
                        for (int rr = 1; rr < 4; ++rr)
                            if (r == rr) gg = g[rr];
                        pd[k] = __fmaf_rn(gg.x, e.x, pd[k]);
                        pd[k] = __fmaf_rn(gg.y, e.y, pd[k]);
                        pd[k] = __fmaf_rn(gg.z, e.z, pd[k]);
                        pd[k] = __fmaf_rn(gg.w, e.w, pd[k]);
                    } else {
                        pd[k] = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(pd[k], e.x), e.y), e.z), e.w);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] += (double)pc[r][c];
#pragma unroll
        for (int k = 0; k < kDR; ++k) dacc[k] += (double)pd[k];
    }
    cp_async_wait<0>();
    __syncthreads();          // all stages idle: the reduction area may overwrite them
    // fixed-order sum over the groups: red[g][0..TB) = d, red[g][TB..) = M (TB-strided)
    double* red = reinterpret_cast<double*>(smem);
    constexpr int kRow = TB * TB + TB;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c)
            red[grp * kRow + TB + (ty + kSt * r) * TB + tx + kSt * c] = acc[r][c];
    if (dthread) {            // covers every diagonal row (zeros without DIAG)
#pragma unroll
        for (int k = 0; k < kDR; ++k) {
            const int r = kSt <= 4 ? tx + kSt * k : k;
            red[grp * kRow + ty + kSt * r] = dacc[k];
        }
    }
    __syncthreads();
    const int R = T + T * T;                  // output row [T + T*T] of the runtime T
    double* out = part + (size_t)blockIdx.x * R;
    for (int e = tid; e < R; e += 256) {
        const int src = e < T ? e : TB + ((e - T) / T) * TB + (e - T) % T;
        double s = 0.0;
        for (int g = 0; g < C::kNG; ++g) s += red[g * kRow + src];
        out[e] = s;
    }
}

}  // namespace

int param_long_slices(int T, long long N) {
    const int tiles = (T + kLT - 1) / kLT;
    long long s = (N + 8191) / 8192;
    const long long cap = 2368 / (tiles * tiles);     // ~16 blocks per SM in total
    if (s > cap) s = cap;
    return s < 1 ? 1 : (int)s;
}

cudaError_t param_long_launch(const float* G, const float* V, const float* E, int T, long long N,
                              bool diag_product, double* part, int slices, cudaStream_t st) {
    return param_rows_launch(G, V, E, T, N, 1, diag_product ? kDiagProduct : kDiagSum, part,
                             slices, true, st);
}

int param_rows_chunks(int T, long long N, int B) {
    const long long F = N / (B < 1 ? 1 : B);
    long long target, cap;
    if (T <= 64) {
        target = 148 * 8;
        cap = (F + 127) / 128;
    } else {
        const int tiles = (T + kLT - 1) / kLT;
        target = 2368 / (tiles * tiles);
        cap = (F + 8191) / 8192;
    }
    long long c = (target + B - 1) / B;
    if (c > cap) c = cap;
    return c < 1 ? 1 : (int)c;
}

cudaError_t param_rows_launch(const float* G, const float* V, const float* E, int T, long long N,
                              int B, int diag, double* part, int chunks, bool small_ok,
                              cudaStream_t st) {
    if (N <= 0 || B < 1) return cudaSuccess;
    const long long F = N / B;
    long long per = (F + chunks - 1) / chunks;
    const dim3 rows((unsigned)((long long)B * chunks));
    if (small_ok && T <= 64) {
        per = (per + 3) / 4 * 4;                 // segments start on whole quads
        const int TB = T <= 8 ? 8 : T <= 16 ? 16 : T <= 32 ? 32 : 64;
#define DFSNN_SMALL(TV, DV)                                                                   \
        if (TB == TV && diag == DV) {                                                         \
            auto k = param_small<TV, DV>;                                                     \
            const int bytes = SmallCfg<TV, DV>::kBytes;                                       \
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes); \
            if (e != cudaSuccess) return e;                                                   \
            k<<<rows, 256, bytes, st>>>(G, V, E, T, N, F, chunks, per, part);                 \
            return cudaGetLastError();                                                        \
        }
        DFSNN_SMALL(8, kDiagNone) DFSNN_SMALL(8, kDiagSum) DFSNN_SMALL(8, kDiagProduct)
        DFSNN_SMALL(16, kDiagNone) DFSNN_SMALL(16, kDiagSum) DFSNN_SMALL(16, kDiagProduct)
        DFSNN_SMALL(32, kDiagNone) DFSNN_SMALL(32, kDiagSum) DFSNN_SMALL(32, kDiagProduct)
        DFSNN_SMALL(64, kDiagNone) DFSNN_SMALL(64, kDiagSum) DFSNN_SMALL(64, kDiagProduct)
#undef DFSNN_SMALL
    }
    per = (per + kLK - 1) / kLK * kLK;
    if (per < kLK) per = kLK;
    const int tiles = (T + kLT - 1) / kLT;
    const dim3 grid(rows.x, (unsigned)tiles, (unsigned)tiles);
    if (diag == kDiagProduct) param_long<kDiagProduct><<<grid, 256, 0, st>>>(G, V, E, T, N, F, chunks, per, part);
    else if (diag == kDiagSum) param_long<kDiagSum><<<grid, 256, 0, st>>>(G, V, E, T, N, F, chunks, per, part);
    else param_long<kDiagNone><<<grid, 256, 0, st>>>(G, V, E, T, N, F, chunks, per, part);
    return cudaGetLastError();
}

}  // namespace dfsnn
