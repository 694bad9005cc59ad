// param_reduce.cuh -- block-level accumulation of the shared-parameter gradients
//   gs[t]   = sum_n g[t,n]*e[t,n]   (DIAG_PRODUCT)   or   sum_n e[t,n]
//   gW[t,i] = sum_n g[t,n] * v[i,n]                 (all t, i < TB)
// for the persistent glmulti / aligned backward kernels.  It replaces the reference's
// torch.sum(grad_pre*drift) + torch.matmul(grad_pre, v_hist^T)
// (fde_cupy_kernels_all.py:1999-2009) and aligned_scale + the ga@h^T GEMM
// (aligned_glmulti.py:33-41, :141-144): the operands never leave shared memory.
//
// Operands are time-major [TB][256] tiles in shared memory.  Each thread owns a 4x4 block
// of the TB x TB product for a fixed slice of the tile's neurons, read as float4 along the
// neuron axis (lanes of a warp share the t-rows, so the g loads broadcast); diagonal blocks
// also accumulate gs.  Per-tile fp32 partials are added to per-thread fp32 accumulators;
// at the end the block reduces its slices in double, in a fixed order (deterministic, no
// atomics), into one row [TB + TB*TB] of a per-block partials array.
#pragma once
#include "lif_common.cuh"
#include "pack2.cuh"

namespace dfsnn {

constexpr int kTile = 256;   // neurons per tile = threads per block

template <int TB>
struct ProdCfg {
    static constexpr int NTR = TB / 4;                  // 4-row blocks along t (and along i)
    static constexpr int NSLICE = kTile / (NTR * NTR);  // neuron slices
    static constexpr int NG = kTile / (4 * NSLICE);     // float4 neuron groups per slice
    static constexpr int LANES_PER_SLICE = NTR;
    static constexpr int SLICES_PER_WARP = 32 / NTR;
    static constexpr int NOUT = TB + TB * TB;           // gs then gW, row-major
    static_assert(TB % 4 == 0 && TB <= 32 && TB >= 8, "TB must be 8, 16 or 32");
};

template <int TB, bool DIAG_PRODUCT>
struct TileProduct {
    using C = ProdCfg<TB>;
    float acc[4][4];
    float accs[4];
    int tr, tc, slice;

    __device__ __forceinline__ void init(int tid) {
        const int lane = tid & 31, w = tid >> 5;
        tc = lane % C::NTR;
        tr = w % C::NTR;
        slice = (w / C::NTR) * C::SLICES_PER_WARP + lane / C::NTR;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            accs[r] = 0.0f;
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
        }
    }

    // G, V, E: [TB][kTile] time-major tiles (rows t >= T and dead neurons hold zeros).
    // Each float4 group of neurons is reduced as two packed lanes (FFMA2): this is a sum
    // over neurons whose order is free (the reference's torch.sum / cuBLAS fix none either).
    __device__ __forceinline__ void accumulate(const float* G, const float* V, const float* E) {
        float2 pw[4][4], ps[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            ps[r] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int c = 0; c < 4; ++c) pw[r][c] = make_float2(0.0f, 0.0f);
        }
        const bool diag = tr == tc;
#pragma unroll 2
        for (int jj = 0; jj < C::NG; ++jj) {
            const int kb = 4 * (jj * C::NSLICE + slice);
            float4 g[4], v[4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
                g[r] = *reinterpret_cast<const float4*>(G + (4 * tr + r) * kTile + kb);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                v[c] = *reinterpret_cast<const float4*>(V + (4 * tc + c) * kTile + kb);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float2 g01 = make_float2(g[r].x, g[r].y), g23 = make_float2(g[r].z, g[r].w);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    pw[r][c] = fma2(g01, make_float2(v[c].x, v[c].y), pw[r][c]);
                    pw[r][c] = fma2(g23, make_float2(v[c].z, v[c].w), pw[r][c]);
                }
            }
            if (diag) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float4 e = *reinterpret_cast<const float4*>(E + (4 * tr + r) * kTile + kb);
                    if constexpr (DIAG_PRODUCT) {
                        ps[r] = fma2(make_float2(g[r].x, g[r].y), make_float2(e.x, e.y), ps[r]);
                        ps[r] = fma2(make_float2(g[r].z, g[r].w), make_float2(e.z, e.w), ps[r]);
                    } else {
                        ps[r] = add2(ps[r], make_float2(e.x, e.y));
                        ps[r] = add2(ps[r], make_float2(e.z, e.w));
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            accs[r] = __fadd_rn(accs[r], __fadd_rn(ps[r].x, ps[r].y));
#pragma unroll
            for (int c = 0; c < 4; ++c)
                acc[r][c] = __fadd_rn(acc[r][c], __fadd_rn(pw[r][c].x, pw[r][c].y));
        }
    }

    static __device__ __forceinline__ int owner(int otr, int otc, int sl) {
        const int w = (sl / C::SLICES_PER_WARP) * C::NTR + otr;
        const int lane = (sl % C::SLICES_PER_WARP) * C::NTR + otc;
        return w * 32 + lane;
    }

    // Reduce all slices of the block in double, fixed order; write the block's partial row.
    // red: kTile*20 doubles of shared memory (callers reuse their staging buffers).
    __device__ __forceinline__ void finish(double* red, double* part, int tid) {
        double* mine = red + (size_t)tid * 20;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
#pragma unroll
            for (int c = 0; c < 4; ++c) mine[r * 4 + c] = (double)acc[r][c];
            mine[16 + r] = (double)accs[r];
        }
        __syncthreads();
        for (int o = tid; o < C::NOUT; o += blockDim.x) {
            const bool is_s = o < TB;
            const int t = is_s ? o : (o - TB) / TB;
            const int i = is_s ? o : (o - TB) % TB;
            const int otr = t / 4, otc = is_s ? otr : i / 4, r = t % 4, c = i % 4;
            double sum = 0.0;
            for (int sl = 0; sl < C::NSLICE; ++sl)
                sum += red[(size_t)owner(otr, otc, sl) * 20 + (is_s ? 16 + r : r * 4 + c)];
            part[o] = sum;
        }
    }
};

// Sum per-block partial rows [nblocks][TB + TB*TB] in a fixed order: one warp per output,
// lanes stride over blocks, then a fixed shuffle tree.  gs -> gscale[T], -gW -> gW[T,T]
// (strictly lower triangle only when lower_only).  A set error word poisons the outputs.
__global__ void param_finalize(const double* part, int nblocks, int TB, int T, float* gscale,
                               float* gW, int lower_only, const unsigned int* err);

}  // namespace dfsnn
