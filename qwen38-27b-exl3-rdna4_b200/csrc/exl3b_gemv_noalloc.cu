// exl3b_linear_noalloc: the m <= 16 EXL3 linear with its scratch in a static device array, for
// callers that cannot allocate device memory (see include/exl3b.h).  It runs the same launches
// as exl3b_linear; only the workspace comes from here instead of from the caller.
#include <mutex>

#include "exl3b_common.cuh"

namespace exl3b {

int linear_impl(const uint16_t* x, int m, int k, int groups, const uint16_t* const* trellis, const int* n, int K,
                int codebook, const uint16_t* const* suh, const uint16_t* const* svh, uint16_t* const* y,
                int64_t ldy, void* workspace, size_t ws_bytes, void* stream, const exl3b_tp_comm* comm,
                const uint16_t* norm_w, float norm_eps);
size_t linear_workspace_exact(int m, int k, int n, int K);

// The scratch: held by every device that loads the library, shared by all calls on that device.
// Static device memory starts zeroed.  In host code `g_noalloc_scratch` names a host-side stand-in,
// never the device memory; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[EXL3B_NOALLOC_SCRATCH_BYTES];

// Bytes at the start of a linear workspace that must be zero when a call starts (error word +
// column-block counters; matches the layout in exl3b_gemv.cu).
constexpr size_t kZeroBytes = EXL3B_WS_ZERO_BYTES;

constexpr int kMaxDevices = 64;
static std::mutex g_setup_mu;
static void* g_scratch_ptr[kMaxDevices];  // set once a device's set-up has succeeded

// The array's device address on the current device.  The first call on a device resolves it with
// that device current; a failed set-up is not remembered, so the next call tries again.
static int scratch_for_current_device(void** out, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e);
    if (dev < 0 || dev >= kMaxDevices) return EXL3B_BAD_ARG;
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        // the set-up belongs before any capture: refuse it (without touching any stream) when the
        // stream is being captured
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        e = cudaStreamIsCapturing(stream, &cap);
        if (e != cudaSuccess) return cuda_status(e);
        if (cap != cudaStreamCaptureStatusNone) return EXL3B_BAD_ARG;
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e);
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return EXL3B_OK;
}

}  // namespace exl3b

using namespace exl3b;

extern "C" int exl3b_linear_noalloc(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K,
                                    int codebook, const uint16_t* suh, const uint16_t* svh, uint16_t* y,
                                    int64_t ldy, void* stream) {
    if (m < 1 || m > EXL3B_GEMV_MAX_ROWS || k < 128 || n < 128 || k % 128 || n % 128 || K < 1 || K > 8)
        return EXL3B_DECLINED;
    // the exact bytes this call's partition uses, the same layout exl3b_linear checks
    if (linear_workspace_exact(m, k, n, K) > EXL3B_NOALLOC_SCRATCH_BYTES) return EXL3B_TOO_LARGE;
    void* scratch = nullptr;
    int st = scratch_for_current_device(&scratch, (cudaStream_t)stream);
    if (st != EXL3B_OK) return st;
    // the counters and the error word must start at zero; a failed earlier call may have left
    // them otherwise, so clear them in stream order before this call's kernels
    cudaError_t e = cudaMemsetAsync(scratch, 0, kZeroBytes, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_status(e);
    const uint16_t* tr[1] = {trellis};
    const uint16_t* su[1] = {suh};
    const uint16_t* sv[1] = {svh};
    uint16_t* yy[1] = {y};
    int nn[1] = {n};
    return linear_impl(x, m, k, 1, tr, nn, K, codebook, su, sv, yy, ldy, scratch, EXL3B_NOALLOC_SCRATCH_BYTES,
                       stream, nullptr, nullptr, 0.f);
}

extern "C" int exl3b_linear_noalloc_error(int* out, void* stream) {
    if (!out) return EXL3B_BAD_ARG;
    void* scratch = nullptr;
    int st = scratch_for_current_device(&scratch, (cudaStream_t)stream);
    if (st != EXL3B_OK) return st;
    return exl3b_linear_workspace_error(scratch, out, stream);
}
