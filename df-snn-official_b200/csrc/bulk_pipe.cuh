// bulk_pipe.cuh -- double-buffered staging of [T, 256]-neuron input tiles in shared memory
// with cp.async.bulk (global -> shared, no multicast) and mbarrier transaction counts.
//
// One elected thread issues, per tile and per input array, T row copies of 256 neurons
// (1 KB each, 16-byte aligned: requires N % 4 == 0 and 16-byte aligned base pointers) and
// arms the stage's mbarrier with the expected byte count.  Every wait is bounded: after
// kMaxWaitIters failed try_waits the caller reports a timeout, sets the kernel's error word
// and leaves the loop together with the whole block (see BulkPipe::wait).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dfsnn {

constexpr uint32_t kMaxWaitIters = 1u << 22;   // x ~1 us per try_wait: a few seconds at most

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMaxWaitIters; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Two-stage pipeline of NARR input arrays (each staged as [T][kTileN] floats per stage)
// plus one optional single-row array (e.g. the initial membrane v0[N], staged as [kTileN]).
template <int NARR>
struct BulkPipe {
    static constexpr int kTileN = 256;
    uint64_t* bar;              // [2] mbarriers in shared memory
    float* stage[2][NARR];      // stage buffers
    float* row_stage[2];        // single-row stage buffers (used when row_src != nullptr)
    const float* src[NARR];     // [T, N] global arrays
    const float* row_src;       // [N] global array or nullptr
    int T;
    long long N;

    // thread 0 only: arm stage s and issue the row copies of tile `tile`
    __device__ __forceinline__ void issue(int s, long long tile) const {
        const long long n0 = tile * kTileN;
        const long long len = (N - n0) < kTileN ? (N - n0) : kTileN;
        const uint32_t row_bytes = (uint32_t)(len * sizeof(float));
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&bar[s], row_bytes * ((uint32_t)T * NARR + (row_src ? 1u : 0u)));
        for (int a = 0; a < NARR; ++a)
            for (int t = 0; t < T; ++t)
                bulk_copy_g2s(stage[s][a] + t * kTileN, src[a] + (long long)t * N + n0, row_bytes,
                              &bar[s]);
        if (row_src) bulk_copy_g2s(row_stage[s], row_src + n0, row_bytes, &bar[s]);
    }
};

}  // namespace dfsnn
