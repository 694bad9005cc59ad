// param_long.cu -- shared-parameter gradients of the long-history backward kernels (T > 32):
//   gs[t]   = sum_n G[t,n] * E[t,n]   (DIAG_PRODUCT)   or   sum_n E[t,n]
//   gW[t,i] = sum_n G[t,n] * V[i,n]
// from [T, N] scratch arrays written by the backward sweep, i.e. the reference's
// torch.sum(grad_pre*drift) + torch.matmul(grad_pre, v_hist^T) (fde_cupy_kernels_all.py:
// 1999-2009) and aligned_scale + ga@h^T (aligned_glmulti.py:33-41, :141-144).
//
// Grid (slices, tiles, tiles): block (s, bt, bi) reduces neuron slice s into the 64 x 64
// output tile (bt, bi); each of its 256 threads owns a 4 x 4 block of the tile.  Chunks of
// 32 neurons are staged through shared memory, multiplied in fp32 and folded into double
// accumulators per chunk.  Every block writes its part of the slice's partial row
// [T + T*T] (double); param_finalize sums the rows in a fixed order -- deterministic, no
// atomics.
#include "kernels.h"
#include "lif_common.cuh"

namespace dfsnn {

namespace {

constexpr int kLT = 64;      // output tile edge
constexpr int kLK = 32;      // neurons per chunk

template <bool DIAG_PRODUCT>
__global__ void __launch_bounds__(256) param_long(const float* G, const float* V, const float* E,
                                                  int T, long long N, long long per_slice,
                                                  double* part) {
    __shared__ float sG[kLT][kLK + 1];
    __shared__ float sV[kLT][kLK + 1];
    __shared__ float sE[kLT][kLK + 1];
    const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
    const int t0 = blockIdx.y * kLT, i0 = blockIdx.z * kLT;
    const bool diag = blockIdx.y == blockIdx.z;
    const long long nb = (long long)blockIdx.x * per_slice;
    const long long ne = (nb + per_slice) < N ? (nb + per_slice) : N;
    double acc[4][4], accs = 0.0;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.0;
    for (long long k0 = nb; k0 < ne; k0 += kLK) {
        // stage rows t0.. of G (and E on the diagonal) and rows i0.. of V, zeros outside
        for (int e = tid; e < kLT * kLK; e += 256) {
            const int row = e / kLK, k = e % kLK;
            const long long n = k0 + k;
            const bool okn = n < ne;
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
                ps = DIAG_PRODUCT ? __fmaf_rn(sG[row][k], sE[row][k], ps) : __fadd_rn(ps, sE[row][k]);
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
    if (diag && tx < 4 && t0 + 4 * ty + tx < T) row[t0 + 4 * ty + tx] = accs;
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
    const int tiles = (T + kLT - 1) / kLT;
    long long per = (N + slices - 1) / slices;
    per = (per + kLK - 1) / kLK * kLK;
    if (per < kLK) per = kLK;
    const dim3 grid((unsigned)slices, (unsigned)tiles, (unsigned)tiles);
    if (diag_product) param_long<true><<<grid, 256, 0, st>>>(G, V, E, T, N, per, part);
    else param_long<false><<<grid, 256, 0, st>>>(G, V, E, T, N, per, part);
    return cudaGetLastError();
}

}  // namespace dfsnn
