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

// The scratch: held by every device that loads the library, shared by all calls on that device.
// In host code `g_noalloc_scratch` names a host-side stand-in, never the device memory; the
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[EXL3B_NOALLOC_SCRATCH_BYTES];

// Bytes at the start of a linear workspace that must be zero when a call starts (error word +
// column-block counters; matches the layout in exl3b_gemv.cu).
constexpr size_t kZeroBytes = EXL3B_WS_ZERO_BYTES;

constexpr int kMaxDevices = 64;
static std::once_flag g_setup_once[kMaxDevices];
static void* g_scratch_ptr[kMaxDevices];
static cudaError_t g_setup_err[kMaxDevices];

// Once per device, with that device current: resolve the device address of the array and zero it.
static int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e);
    if (dev < 0 || dev >= kMaxDevices) return EXL3B_BAD_ARG;
    std::call_once(g_setup_once[dev], [dev] {
        void* p = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err == cudaSuccess) err = cudaMemset(p, 0, kZeroBytes);
        g_scratch_ptr[dev] = (err == cudaSuccess) ? p : nullptr;
        g_setup_err[dev] = err;
    });
    if (g_setup_err[dev] != cudaSuccess) return cuda_status(g_setup_err[dev]);
    *out = g_scratch_ptr[dev];
    return EXL3B_OK;
}

}  // namespace exl3b

using namespace exl3b;

extern "C" int exl3b_linear_noalloc(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K,
                                    int codebook, const uint16_t* suh, const uint16_t* svh, uint16_t* y,
                                    int64_t ldy, void* stream) {
    if (m < 1 || m > EXL3B_GEMV_MAX_ROWS || k < 128 || n < 128) return EXL3B_DECLINED;
    const size_t need = exl3b_linear_workspace_bytes(m, k, 1, n);
    if (need == 0) return EXL3B_DECLINED;
    if (need > EXL3B_NOALLOC_SCRATCH_BYTES) return EXL3B_TOO_LARGE;
    void* scratch = nullptr;
    int st = scratch_for_current_device(&scratch);
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
