/*
 * ref_shim.h -- lets the reference's one-thread-per-element CUDA kernel sources compile
 * as host C++ so that oracle/build_ref.py can run the reference's own arithmetic on the
 * CPU (TEST INFRASTRUCTURE ONLY: used to pin the oracle and as the timed reference arm).
 *
 * A "launch" is a loop over global thread indices; each iteration sets the thread-local
 * blockIdx/threadIdx/blockDim the kernel reads.  Only kernels without inter-thread
 * communication are ever called through it; __shared__/__syncthreads exist only so that
 * the other kernels in the same source strings compile.
 */
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>

struct dfsnn_ref_dim3 { unsigned int x, y, z; };
static thread_local dfsnn_ref_dim3 blockIdx = {0, 0, 0};
static thread_local dfsnn_ref_dim3 threadIdx = {0, 0, 0};
static thread_local dfsnn_ref_dim3 blockDim = {256, 1, 1};
static thread_local dfsnn_ref_dim3 gridDim = {1, 1, 1};

#define __global__
#define __device__
#define __forceinline__ inline
#define __shared__ static thread_local
static inline void __syncthreads() {}
using std::max;
using std::min;

/* Reference kernels accumulate scalar gradients with atomicAdd. */
static inline float atomicAdd(float* address, float value) {
    float old;
#pragma omp atomic capture
    { old = *address; *address += value; }
    return old;
}

/* Set the thread-local indices of global thread g for a 1-D launch of 256-thread blocks. */
static inline void dfsnn_ref_set_thread(long long g) {
    blockDim.x = 256;
    blockIdx.x = (unsigned int)(g / 256);
    threadIdx.x = (unsigned int)(g % 256);
}
