// tma.cuh -- tensor-map (TMA) staging of time-major [T, N] fp32 arrays for sm_100a.
//
// One cp.async.bulk.tensor copy moves a box of `rows` time steps x `box_n` neurons into
// shared memory (dense rows of box_n floats) and signals an mbarrier with the box's byte
// count; neurons past N read as zeros.  No multicast: every copy lands in the issuing
// CTA's own shared memory.  Host requirements (checked by encode_rows_map): base address
// 16-byte aligned, N % 4 == 0 (row stride a multiple of 16 bytes), box_n * 4 a multiple of
// 16 bytes, rows and box_n <= 256; the neuron coordinate of every copy is a multiple of
// box_n, hence of 4 (16 bytes).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "bulk_pipe.cuh"

namespace dfsnn {

// box (rows x box_n) of a [rows, N] map at neuron n0 -> dst (128-byte aligned)
__device__ __forceinline__ void tma_load_rows(void* dst, const CUtensorMap* map, int n0,
                                              uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(n0), "r"(0), "r"(smem_u32(bar))
        : "memory");
}

// rows x box_n box at neuron n0 of a [rows, N] map <- src (shared, 128-byte aligned); part of
// the calling thread's current bulk group.  Columns past N are not written.
__device__ __forceinline__ void tma_store_rows(const CUtensorMap* map, const void* src, int n0) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::
                     "l"(reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(n0), "r"(0)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// wait until every bulk group of the calling thread has finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// wait until every bulk group of the calling thread has completed
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Encode a map over the time-major array base[rows][N] with boxes of rows x box_n floats.
// Returns false when the layout does not meet the TMA rules or the driver call fails.
bool encode_rows_map(CUtensorMap* map, const float* base, long long N, int rows, int box_n);

}  // namespace dfsnn
