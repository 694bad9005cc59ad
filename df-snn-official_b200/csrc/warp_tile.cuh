// warp_tile.cuh -- building blocks of the warp-tiled persistent backward kernels (glmulti and
// aligned, T in {8, 16}): each warp owns a fixed, strided set of 64-neuron tiles, stages them
// itself with three TMA box copies per tile (x and grad_spike as [T x 64] boxes, v0 as a
// [1 x 64] box; neurons past N read as zeros) into its own two shared-memory stages with one
// mbarrier each, and writes grad_x / grad_v0 back with TMA stores that clip at N -- no block
// barrier in the tile loop.  Lane l carries neurons 2l and 2l+1 as the halves of float2
// values.  The shared-parameter product sum_n G[t,n] V[i,n] is accumulated per lane as a 4x4
// block over one slice of each tile's neurons, from padded GP / V rows (the product's float4
// reads are then free of bank conflicts), and reduced per block in double in a fixed order
// at the end.
#pragma once
#include <cstdint>

#include "bulk_pipe.cuh"
#include "pack2.cuh"
#include "lif_common.cuh"
#include "tma.cuh"

namespace dfsnn {

struct alignas(64) TileMaps {
    CUtensorMap x;    // [T, N], boxes T x 64 (loads)
    CUtensorMap g;    // [T, N] grad_spike
    CUtensorMap v0;   // [1, N], boxes 1 x 64
    CUtensorMap gx;   // [T, N] grad_x (stores)
    CUtensorMap gv0;  // [1, N] grad_v0
};

template <int T>
struct WarpBwdCfg {
    static constexpr int kWarps = 8;
    static constexpr int TN = 64;                        // neurons per warp tile
    // padded GP / V row stride (floats): rows start 32 B (T = 16) or 64 B (T = 8) apart
    // modulo 128 B, so the product's float4 reads hit distinct banks
    static constexpr int RS = T <= 8 ? 80 : 72;
    static constexpr int STAGE = 2 * T * TN + TN;        // dense X rows, G rows, v0 row
    static constexpr int PER_WARP = 2 * STAGE + 2 * T * RS;   // two stages + GP + V rows
    static constexpr size_t kBytes = sizeof(float) * kWarps * PER_WARP + 128;  // + alignment
    static constexpr uint32_t kTxBytes = sizeof(float) * STAGE;
    static constexpr int kMinBlocks = T <= 8 ? 2 : 1;    // blocks per SM the registers allow
    static constexpr int NRED = 16 + T;                  // doubles per thread in the reduction
    static constexpr int TBLK = T / 4;                   // 4-row blocks along t (and along i)
    static constexpr int LANES_PER_SLICE = TBLK * TBLK;
    static constexpr int NSLICES = 32 / LANES_PER_SLICE;
    static constexpr int GROUPS = TN / (4 * NSLICES);    // float4 neuron groups per lane
    static_assert(T == 8 || T == 16, "warp-tiled backward covers T = 8 and T = 16");
    static_assert((sizeof(float) * STAGE) % 128 == 0 && (sizeof(float) * PER_WARP) % 128 == 0,
                  "TMA destinations must stay 128-byte aligned");
    static_assert(sizeof(double) * 32 * kWarps * NRED <= kBytes - 128, "reduction scratch");
};

// Arm stage X of this warp and copy its tile (lane 0).  The stage's previous contents
// were fenced against the async proxy when its grad_x / grad_v0 store was issued; the
// store must have finished reading the stage before the new copies land.
template <int T>
__device__ __forceinline__ void warp_load(float* X, uint64_t* bar, const TileMaps& m,
                                          long long n0) {
    constexpr int TN = WarpBwdCfg<T>::TN;
    bulk_wait_read_all();
    mbar_arrive_expect_tx(bar, WarpBwdCfg<T>::kTxBytes);
    tma_load_rows(X, &m.x, (int)n0, bar);
    tma_load_rows(X + T * TN, &m.g, (int)n0, bar);
    tma_load_rows(X + 2 * T * TN, &m.v0, (int)n0, bar);
}

// Store the tile's grad_x rows (in G) and grad_v0 row (in V0) with TMA (columns past N
// are clipped by the tensor maps).  All lanes fence their generic writes of the stage.
template <int T>
__device__ __forceinline__ void warp_store(float* X, const TileMaps& m, long long n0, int lane) {
    constexpr int TN = WarpBwdCfg<T>::TN;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_rows(&m.gx, X + T * TN, (int)n0);
        tma_store_rows(&m.gv0, X + 2 * T * TN, (int)n0);
        bulk_commit();
    }
}

// pw[r][c] += sum over this lane's neurons of GP[t] * V[i], t = tr + TBLK*r,
// i = tc + TBLK*c; each float4 group of neurons enters as two packed halves.
template <int T>
__device__ __forceinline__ void warp_product(const float* GP, const float* Vs, int lane,
                                             float2 (&pw)[4][4]) {
    using C = WarpBwdCfg<T>;
    constexpr int RS = C::RS;
    const int tr = lane % C::TBLK, tc = (lane / C::TBLK) % C::TBLK, sl = lane / C::LANES_PER_SLICE;
#pragma unroll
    for (int jj = 0; jj < C::GROUPS; ++jj) {
        const int kb = 4 * (sl * C::GROUPS + jj);
        float4 g[4], v[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            g[r] = *reinterpret_cast<const float4*>(GP + (tr + C::TBLK * r) * RS + kb);
#pragma unroll
        for (int c = 0; c < 4; ++c)
            v[c] = *reinterpret_cast<const float4*>(Vs + (tc + C::TBLK * c) * RS + kb);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float2 g01 = make_float2(g[r].x, g[r].y), g23 = make_float2(g[r].z, g[r].w);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                pw[r][c] = fma2(g01, make_float2(v[c].x, v[c].y), pw[r][c]);
                pw[r][c] = fma2(g23, make_float2(v[c].z, v[c].w), pw[r][c]);
            }
        }
    }
}

// num / b per half: div_markstein in packed form, or the IEEE division (SLOW).  The fast form
// is exact for 2 <= b <= 2^64 and |num| in [2^-60, 2^60] (callers check and take SLOW for
// the whole warp otherwise); a zero numerator gives +0 (IEEE: the numerator's sign).
template <bool SLOW>
__device__ __forceinline__ float2 quot2(float2 num, float2 b) {
    if constexpr (SLOW) {
        return make_float2(__fdiv_rn(num.x, b.x), __fdiv_rn(num.y, b.y));
    } else {
        const float2 nb = pmul2(b, f2(-1.0f));
        const float2 y0 = make_float2(rcp_approx(b.x), rcp_approx(b.y));
        const float2 y = pfma2(pfma2(nb, y0, f2(1.0f)), y0, y0);
        const float2 q0 = pmul2(num, y);
        return pfma2(pfma2(nb, q0, num), y, q0);
    }
}

// |v| in the numerator range of quot2 (or zero)
__device__ __forceinline__ bool quot_num_ok(float v) {
    const float m = fabsf(v);
    return m <= 0x1p60f && (m >= 0x1p-60f || m == 0.0f);
}

// Block reduction in double, fixed order, into this block's partial row [T + T*T]:
// gs (per-lane sums gsa over all lanes) then the T x T product (pw).  Uses the stages as
// scratch: every warp must have finished its tiles and its stores.
template <int T>
__device__ __forceinline__ void warp_tiles_finish(const float2 (&pw)[4][4], const float2 (&gsa)[T],
                                                  unsigned char* aligned_smem, double* part_base,
                                                  int tid) {
    using C = WarpBwdCfg<T>;
    __syncthreads();
    double* red = reinterpret_cast<double*>(aligned_smem);
    double* mine = red + (size_t)tid * C::NRED;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) mine[r * 4 + c] = (double)pw[r][c].x + (double)pw[r][c].y;
#pragma unroll
    for (int t = 0; t < T; ++t) mine[16 + t] = (double)gsa[t].x + (double)gsa[t].y;
    __syncthreads();
    double* part = part_base + (size_t)blockIdx.x * (T + T * T);
    for (int o = tid; o < T + T * T; o += blockDim.x) {
        double sum = 0.0;
        if (o < T) {
            for (int q = 0; q < C::kWarps * 32; ++q) sum += red[(size_t)q * C::NRED + 16 + o];
        } else {
            const int t = (o - T) / T, i = (o - T) % T;
            const int r = t / C::TBLK, c = i / C::TBLK;
            const int l0 = (t % C::TBLK) + C::TBLK * (i % C::TBLK);
            for (int w = 0; w < C::kWarps; ++w)
                for (int sl = 0; sl < C::NSLICES; ++sl)
                    sum += red[(size_t)(w * 32 + sl * C::LANES_PER_SLICE + l0) * C::NRED + r * 4 + c];
        }
        part[o] = sum;
    }
}

// Tensor maps of a warp-tiled backward; false when the arrays do not meet the TMA rules.
inline bool encode_tile_maps(TileMaps* m, const float* x, const float* g, const float* v0,
                             float* gx, float* gv0, int T, long long N) {
    const int bn = 64;   // WarpBwdCfg<T>::TN
    return encode_rows_map(&m->x, x, N, T, bn) && encode_rows_map(&m->g, g, N, T, bn) &&
           encode_rows_map(&m->v0, v0, N, 1, bn) && encode_rows_map(&m->gx, gx, N, T, bn) &&
           encode_rows_map(&m->gv0, gv0, N, 1, bn);
}

}  // namespace dfsnn
