// mma_tf32.cuh -- the 3xTF32 building blocks of the parameter products on the tensor pipe:
// every fp32 operand split into a tf32 head and its exact tail, and one m16n8k8 tf32
// mma.sync with fp32 accumulation (PTX ISA, warp-level matrix multiply-accumulate).
#pragma once
#include <cstdint>

namespace dfsnn {

// tf32 head of x (13 low mantissa bits cleared) and the exact tail x - head
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    const uint32_t h = __float_as_uint(x) & 0xffffe000u;
    hi = h;
    lo = __float_as_uint(__fsub_rn(x, __uint_as_float(h)));
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

}  // namespace dfsnn
