// param_reduce.cuh -- block-level accumulation of the shared-parameter gradients
//   gs[t]   = sum_n e[t,n]              (or sum_n g[t,n]*d[t,n])
//   gW[t,i] = sum_n g[t,n] * v[i,n]     (all t, i < TB)
// for the persistent glmulti / aligned backward kernels, replacing the reference's
// torch.sum(grad_pre*drift) + torch.matmul(grad_pre, v_hist^T)
// (fde_cupy_kernels_all.py:1999-2009) and aligned_scale + the ga@h^T GEMM
// (aligned_glmulti.py:33-41, :141-144).  No atomics: each thread owns a 4x4 tile of the
// TB x TB product (plus 4 gs entries on diagonal tiles) for a fixed slice of the 256
// neurons of every tile; per-tile fp32 partials are folded into Kahan-compensated fp32
// accumulators, and the block reduces its slices once at the end in double, in a fixed
// order, writing one row of a [gridDim.x, TB + TB*TB] double partials array.
#pragma once
#include "lif_common.cuh"

namespace dfsnn {

constexpr int kTile = 256;           // neurons per tile = threads per block
constexpr int kLdn = kTile + 1;      // row stride of the time-major staging arrays

template <int TB>
struct ProdCfg {
    static constexpr int NTR = TB / 4;             // 4-row tiles along t (and along i)
    static constexpr int NTILE = NTR * NTR;        // 4x4 output tiles
    static constexpr int NSLICE = kTile / NTILE;   // neuron slices per tile
    static constexpr int NPER = kTile / NSLICE;    // neurons per slice
    static constexpr int NOUT = TB + TB * TB;      // gs then gW, row-major
    static_assert(TB % 4 == 0 && NTILE <= kTile, "TB must be a multiple of 4, at most 32");
    // staging arrays: g, v, d (or e), each [TB][kLdn] floats
    static constexpr size_t SMEM_BYTES = size_t(3) * TB * kLdn * sizeof(float);
};

// Kahan-compensated running sum of per-tile partials.
struct KahanAcc {
    float hi = 0.0f, lo = 0.0f;
    __device__ __forceinline__ void add(float p) {
        const float y = __fsub_rn(p, lo);
        const float t = __fadd_rn(hi, y);
        lo = __fsub_rn(__fsub_rn(t, hi), y);
        hi = t;
    }
};

// Per-thread accumulator of one 4x4 tile (+4 diagonal gs entries).
template <int TB, bool DIAG_PRODUCT>
struct TileAccumulator {
    using C = ProdCfg<TB>;
    KahanAcc w[4][4];
    KahanAcc s[4];
    int tr, tc, slice;

    __device__ __forceinline__ void init(int tid) {
        const int tile = tid % C::NTILE;
        slice = tid / C::NTILE;
        tr = tile / C::NTR;
        tc = tile % C::NTR;
    }

    // sG/sV/sE: time-major staging [TB][kLdn]; neurons of this tile are columns 0..255.
    __device__ __forceinline__ void accumulate(const float* sG, const float* sV, const float* sE) {
        float pw[4][4];
        float ps[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            ps[r] = 0.0f;
#pragma unroll
            for (int c = 0; c < 4; ++c) pw[r][c] = 0.0f;
        }
        const bool diag = (tr == tc);
#pragma unroll 4
        for (int j = 0; j < C::NPER; ++j) {
            const int k = j * C::NSLICE + slice;
            float g[4], v[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) g[r] = sG[(4 * tr + r) * kLdn + k];
#pragma unroll
            for (int c = 0; c < 4; ++c) v[c] = sV[(4 * tc + c) * kLdn + k];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) pw[r][c] = __fmaf_rn(g[r], v[c], pw[r][c]);
            if (diag) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float e = sE[(4 * tr + r) * kLdn + k];
                    if constexpr (DIAG_PRODUCT) ps[r] = __fmaf_rn(g[r], e, ps[r]);
                    else ps[r] = __fadd_rn(ps[r], e);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            if (diag) s[r].add(ps[r]);
#pragma unroll
            for (int c = 0; c < 4; ++c) w[r][c].add(pw[r][c]);
        }
    }

    // Reduce all slices of the block in double, fixed order; write this block's partial
    // row (NOUT doubles) to part.  red must hold NSLICE*NTILE*20 doubles of shared memory.
    __device__ __forceinline__ void finish(double* red, double* part, int tid) {
        double* mine = red + (size_t)tid * 20;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                mine[r * 4 + c] = (double)w[r][c].hi + (double)(-w[r][c].lo);
            mine[16 + r] = (double)s[r].hi + (double)(-s[r].lo);
        }
        __syncthreads();
        for (int o = tid; o < C::NOUT; o += blockDim.x) {
            int t, i;
            bool is_s = o < TB;
            if (is_s) { t = o; i = o; } else { t = (o - TB) / TB; i = (o - TB) % TB; }
            const int otr = t / 4, otc = i / 4, r = t % 4, c = i % 4;
            double sum = 0.0;
            for (int sl = 0; sl < C::NSLICE; ++sl) {
                const int th = sl * C::NTILE + (is_s ? (otr * C::NTR + otr) : (otr * C::NTR + otc));
                sum += red[(size_t)th * 20 + (is_s ? 16 + r : r * 4 + c)];
            }
            part[o] = sum;
        }
    }
};

}  // namespace dfsnn
