// warp_tile.cuh -- building blocks of the warp-tiled persistent backward kernels (glmulti and
// aligned, T in {8, 16}): each warp owns a fixed, strided set of 64-neuron tiles, stages them
// itself with three TMA box copies per tile (x and grad_spike as [T x 64] boxes, v0 as a
// [1 x 64] box; neurons past N read as zeros) into its own two shared-memory stages with one
// mbarrier each, and writes grad_x / grad_v0 back with TMA stores that clip at N -- no block
// barrier in the tile loop.  Lane l carries neurons 2l and 2l+1 as the halves of float2
// values.
//
// The shared-parameter product P[t][i] = sum_n GP[t,n] V[i,n] runs on the tensor pipe:
// mma.sync m16n8k8 (tf32 inputs, fp32 accumulation) with every fp32 operand split into a
// tf32 head and a tail (x = hi + lo, hi = x with its 13 low mantissa bits cleared, lo =
// x - hi exactly) and three products per pair (lo*hi + hi*lo + hi*hi; the dropped lo*lo
// and the tail's own truncation are ~2^-21 of each product).  Each tile's products start
// from a zero accumulator and are added to the lane's running fp32 sums with
// round-to-nearest adds; blocks then reduce in double in a fixed order (deterministic).
// Fragment mapping (PTX m16n8k8 .tf32, groupID g = lane / 4, thread-in-group c = lane % 4):
// A[m][k] = GP[t = m][neuron], B[k][n] = V[i = n][neuron], with the reduction index k
// permuted -- k = c holds neuron 2c and k = c + 4 holds neuron 2c + 1 of each 8-neuron
// step -- so that each lane's (a0, a2), (a1, a3) and (b0, b1) pairs are adjacent floats,
// one 64-bit shared load each; rows RS = 72 floats apart (8 mod 32 banks) make the loads
// of a warp free of bank conflicts.
#pragma once
#include <cstdint>

#include "bulk_pipe.cuh"
#include "mma_tf32.cuh"
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
    static constexpr int RS = 72;                        // padded GP / V row stride (floats)
    static constexpr int STAGE = 2 * T * TN + TN;        // dense X rows, G rows, v0 row
    static constexpr int PER_WARP = 2 * STAGE + 2 * T * RS;   // two stages + GP + V rows
    static constexpr size_t kBytes = sizeof(float) * kWarps * PER_WARP + 128;  // + alignment
    static constexpr uint32_t kTxBytes = sizeof(float) * STAGE;
    static constexpr int kMinBlocks = T <= 8 ? 2 : 1;    // blocks per SM the registers allow
    static constexpr int NT = T / 8;                     // mma n-tiles of 8 output columns
    static constexpr int NACC = 4 * NT;                  // product accumulators per lane
    static constexpr int NRED = NACC + T;                // doubles per thread in the reduction
    static_assert(T == 8 || T == 16, "warp-tiled backward covers T = 8 and T = 16");
    static_assert((sizeof(float) * STAGE) % 128 == 0 && (sizeof(float) * PER_WARP) % 128 == 0,
                  "TMA destinations must stay 128-byte aligned");
    static_assert(RS % 32 == 8, "fragment loads are conflict-free for rows 8 banks apart");
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

// acc[4*nt + e] += this tile's sum over its 64 neurons of GP[t] * V[i] for the lane's
// fragment entries e of n-tile nt: t = g + 8*(e >= 2), i = 8*nt + 2c + (e & 1).  For
// T = 8 the A rows 8..15 are zero and their entries are never read.
template <int T>
__device__ __forceinline__ void warp_product(const float* GP, const float* Vs, int lane,
                                             float (&acc)[WarpBwdCfg<T>::NACC]) {
    using C = WarpBwdCfg<T>;
    constexpr int RS = C::RS;
    const int g = lane >> 2, c = lane & 3;
    float d[C::NT][4];
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[nt][e] = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < C::TN; k0 += 8) {
        const float2 ar0 = *reinterpret_cast<const float2*>(GP + g * RS + k0 + 2 * c);
        uint32_t ah[4], al[4];
        split_tf32(ar0.x, ah[0], al[0]);
        split_tf32(ar0.y, ah[2], al[2]);
        if constexpr (T == 16) {
            const float2 ar1 = *reinterpret_cast<const float2*>(GP + (g + 8) * RS + k0 + 2 * c);
            split_tf32(ar1.x, ah[1], al[1]);
            split_tf32(ar1.y, ah[3], al[3]);
        } else {
            ah[1] = al[1] = ah[3] = al[3] = 0u;
        }
#pragma unroll
        for (int nt = 0; nt < C::NT; ++nt) {
            const float2 br = *reinterpret_cast<const float2*>(Vs + (8 * nt + g) * RS + k0 + 2 * c);
            uint32_t bh0, bl0, bh1, bl1;
            split_tf32(br.x, bh0, bl0);
            split_tf32(br.y, bh1, bl1);
            mma_tf32(d[nt], al[0], al[1], al[2], al[3], bh0, bh1);
            mma_tf32(d[nt], ah[0], ah[1], ah[2], ah[3], bl0, bl1);
            mma_tf32(d[nt], ah[0], ah[1], ah[2], ah[3], bh0, bh1);
        }
    }
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[4 * nt + e] = __fadd_rn(acc[4 * nt + e], d[nt][e]);
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

// Block reduction in double, fixed order, into this block's partial row [T + T*T]: the
// per-lane sums gsa over all threads, then P[t][i] from the one lane of each warp that
// holds it.  Uses the stages as scratch: every warp must have finished its tiles and its
// stores.
template <int T>
__device__ __forceinline__ void warp_tiles_finish(const float (&acc)[WarpBwdCfg<T>::NACC],
                                                  const float2 (&gsa)[T],
                                                  unsigned char* aligned_smem, double* part_base,
                                                  int tid) {
    using C = WarpBwdCfg<T>;
    __syncthreads();
    double* red = reinterpret_cast<double*>(aligned_smem);
    double* mine = red + (size_t)tid * C::NRED;
#pragma unroll
    for (int e = 0; e < C::NACC; ++e) mine[e] = (double)acc[e];
#pragma unroll
    for (int t = 0; t < T; ++t) mine[C::NACC + t] = (double)gsa[t].x + (double)gsa[t].y;
    __syncthreads();
    double* part = part_base + (size_t)blockIdx.x * (T + T * T);
    for (int o = tid; o < T + T * T; o += blockDim.x) {
        double sum = 0.0;
        if (o < T) {
            for (int q = 0; q < C::kWarps * 32; ++q) sum += red[(size_t)q * C::NRED + C::NACC + o];
        } else {
            const int t = (o - T) / T, i = (o - T) % T;
            const int lane = 4 * (t & 7) + ((i & 7) >> 1);
            const int slot = 4 * (i >> 3) + ((t >= 8) ? 2 : 0) + (i & 1);
            for (int w = 0; w < C::kWarps; ++w) sum += red[(size_t)(w * 32 + lane) * C::NRED + slot];
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
