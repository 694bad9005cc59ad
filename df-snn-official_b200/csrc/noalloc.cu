// noalloc.cu -- glmulti backward for callers that cannot allocate device memory.
//
// dfsnn_glmulti_backward needs a caller-provided workspace (a 16-byte device error word plus
// one row of double partial sums per block).  Some callers of this library cannot call
// cudaMalloc or any allocating routine at the point where they run the backward -- for
// example code that runs inside a host callback, under a memory-budget policy that forbids
// allocation after start-up, or from a runtime that owns all device memory itself.  For
// them, dfsnn_glmulti_backward_noalloc keeps that scratch in a file-scope device array of
// fixed size instead.
//
// Limits and sharing rules (also in include/dfsnn_b200.h):
//   * T <= 16: the array holds kNoAllocRows rows of (16 + 16*16) doubles; larger T is
//     rejected with DFSNN_ERR_T_LIMIT;
//   * the array exists once per device for the life of the process, and every call uses it:
//     calls whose work overlaps on the GPU (two streams, or two host threads) race on it;
//   * the first call on a device looks up the array's device address (once per device, with
//     that device current); make that first call before any stream capture, and no call on a
//     device after cudaDeviceReset of it (the address is kept for the life of the process);
//   * at most kNoAllocRows blocks write partial rows: below that the reduced outputs equal
//     dfsnn_glmulti_backward's bit for bit (a 148-SM B200 uses 148 or 296 blocks);
//   * a bounded wait that times out is reported only as NaN in grad_scale / grad_weights.
#include <cmath>
#include <cstdint>
#include <mutex>

#include "../../include/dfsnn_b200.h"
#include "kernels.h"

namespace {

constexpr int kNoAllocMaxT = 16;
constexpr int kNoAllocStride = kNoAllocMaxT + kNoAllocMaxT * kNoAllocMaxT;   // doubles per row
constexpr int kNoAllocRows = 512;                                          // partial rows
constexpr size_t kHeaderDoubles = 2;                                       // 16-byte error word

// [16-byte error header][kNoAllocRows rows of partial sums]: 1.1 MB per device.
static __device__ __align__(256) double g_noalloc_scratch[kHeaderDoubles + (size_t)kNoAllocRows * kNoAllocStride];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array for the current device (looked up once per device).
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int dfsnn_glmulti_backward_noalloc(const float* grad_spike, const float* x,
                                              const float* v0, const float* scale,
                                              const float* weights, float* grad_x,
                                              float* grad_v0, float* grad_scale,
                                              float* grad_weights, int T, long long N,
                                              float tau, float threshold, float surrogate_scale,
                                              int full_history, void* stream) {
    if (T < 1 || N < 0) return DFSNN_ERR_SHAPE;
    if (T > kNoAllocMaxT) return DFSNN_ERR_T_LIMIT;
    if (!scale || !weights) return DFSNN_ERR_NULL;
    if (N > 0 && (!grad_spike || !x || !v0 || !grad_x || !grad_v0)) return DFSNN_ERR_NULL;
    if (!std::isfinite(tau) || tau == 0.0f || !std::isfinite(threshold) ||
        !std::isfinite(surrogate_scale))
        return DFSNN_ERR_PARAM;
    void* base = nullptr;
    cudaError_t e = scratch_address(&base);
    if (e != cudaSuccess) return dfsnn::record_cuda_error(e);
    int ex = 0;
    const bool p2 = std::frexp(std::fabs(tau), &ex) == 0.5f && ex > -125 && ex < 126;
    long long nb = dfsnn::glmulti_bwd_blocks(T, N, full_history != 0, p2);
    if (nb > kNoAllocRows) nb = kNoAllocRows;
    double* scratch = static_cast<double*>(base);
    // glmulti_backward_launch clears the error word itself; every block overwrites its own
    // partial row, so nothing else of the shared array needs clearing between calls.
    e = dfsnn::glmulti_backward_launch(
        grad_spike, x, v0, scale, weights, grad_x, grad_v0, grad_scale, grad_weights, T, N, tau,
        threshold, surrogate_scale, full_history != 0, p2, scratch + kHeaderDoubles,
        reinterpret_cast<unsigned int*>(scratch), (int)nb, (cudaStream_t)stream);
    if (e != cudaSuccess) return dfsnn::record_cuda_error(e);
    return DFSNN_OK;
}
