// The elementwise steps a decoder layer runs between the EXL3 linears and the paged attention:
// RMSNorm (optionally with the residual add before it), neox rotary embedding of q and k, and
// SiluAndMul for the M > 16 route (the M <= 16 route fuses it into the gate/up GEMV epilogue).
// The reference leaves these to vLLM's own kernels (its plugin replaces only the linears and the
// KV cache); their semantics follow vLLM's rms_norm / fused_add_rms_norm, rotary_embedding
// (is_neox_style) and SiluAndMul, with the rounding points stated at each kernel.
//
// Every kernel is a programmatic dependent launch: it lets the next kernel start at once (the
// next EXL3 linear then streams its first weights while this one runs) and waits for the previous
// kernel's results before its first read.
#include <algorithm>

#include <cuda_fp8.h>

#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 8;  // 8-half vectors per thread: cols <= 8 * 8 * 256 = 16384

// One CTA per row.  With a residual: r = fp16(x + r) is stored back and normalised (vLLM
// fused_add_rms_norm); without: x is normalised (rms_norm).  out = fp16( fp16(v * s) * w ) with
// s = rsqrt(mean(v^2) + eps) over the fp16 values v, the mean summed in fp32.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const __half* x, int64_t ldx, __half* res, int64_t ldr,
                                                               const __half* w, __half* out, int64_t ldo, int cols,
                                                               float eps) {
    griddep_launch();
    griddep_wait();
    const int row = blockIdx.x, nv = cols / 8;
    const __half* xr = x + row * ldx;
    __half* rr = res ? res + row * ldr : nullptr;
    uint4 v[kNormMaxVec];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNormMaxVec; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i >= nv) break;
        uint4 a = *reinterpret_cast<const uint4*>(xr + 8 * i);
        if (rr) {
            const uint4 b = *reinterpret_cast<const uint4*>(rr + 8 * i);
            a.x = h2_as_u32(__hadd2(u32_as_h2(a.x), u32_as_h2(b.x)));
            a.y = h2_as_u32(__hadd2(u32_as_h2(a.y), u32_as_h2(b.y)));
            a.z = h2_as_u32(__hadd2(u32_as_h2(a.z), u32_as_h2(b.z)));
            a.w = h2_as_u32(__hadd2(u32_as_h2(a.w), u32_as_h2(b.w)));
            *reinterpret_cast<uint4*>(rr + 8 * i) = a;
        }
        v[j] = a;
        const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(u32_as_h2(u[e]));
            ss = fmaf(f.x, f.x, ss);
            ss = fmaf(f.y, f.y, ss);
        }
    }
    __shared__ float red[kNormThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
    const float s = rsqrtf(tot / (float)cols + eps);
    __half* orow = out + row * ldo;
#pragma unroll
    for (int j = 0; j < kNormMaxVec; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i >= nv) break;
        const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * i);
        const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(u32_as_h2(u[e]));
            o[e] = h2_as_u32(__hmul2(__floats2half2_rn(f.x * s, f.y * s), u32_as_h2(ww[e])));
        }
        *reinterpret_cast<uint4*>(orow + 8 * i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Neox rotary embedding over heads of 128: for i < 64, with (c, s) = cos_sin[pos][i], [64 + i],
//   o[i] = x[i] c - x[i + 64] s,   o[i + 64] = x[i + 64] c + x[i] s   (fp32, one rounding each).
// Row t of qkv holds num_q heads of q then num_k heads of k; q goes to q_out (contiguous rows for
// the attention), k is rotated in place.  A position outside [0, max_pos) leaves k untouched and
// writes zeros to the token's q rows.
__global__ void __launch_bounds__(256) rope_kernel(__half* qkv, int64_t ld, __half* q_out, int64_t ldq, int nq,
                                                   int nk, const int64_t* pos, const float* cos_sin, int64_t max_pos) {
    griddep_launch();
    griddep_wait();
    const int t = blockIdx.x;
    const int64_t p = pos[t];
    const bool ok = p >= 0 && p < max_pos;
    const float* cs = cos_sin + (ok ? p : 0) * 128;
    for (int idx = threadIdx.x; idx < (nq + nk) * 32; idx += blockDim.x) {
        const int h = idx >> 5, i = 2 * (idx & 31);
        __half* src = qkv + t * ld + h * 128;
        __half* dst = h < nq ? q_out + t * ldq + h * 128 : src;
        if (!ok) {
            if (h < nq) {
                *reinterpret_cast<uint32_t*>(dst + i) = 0u;
                *reinterpret_cast<uint32_t*>(dst + i + 64) = 0u;
            }
            continue;
        }
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(src + i));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(src + i + 64));
        const float2 c = *reinterpret_cast<const float2*>(cs + i);
        const float2 s = *reinterpret_cast<const float2*>(cs + 64 + i);
        // o = fma(x, c, -(partner * s)) with the product rounded first: one fixed rounding sequence
        *reinterpret_cast<__half2*>(dst + i) = __floats2half2_rn(__fmaf_rn(a.x, c.x, -__fmul_rn(b.x, s.x)),
                                                                 __fmaf_rn(a.y, c.y, -__fmul_rn(b.y, s.y)));
        *reinterpret_cast<__half2*>(dst + i + 64) = __floats2half2_rn(__fmaf_rn(b.x, c.x, __fmul_rn(a.x, s.x)),
                                                                      __fmaf_rn(b.y, c.y, __fmul_rn(a.y, s.y)));
    }
}

// out[r][c] = fp16( fp16(silu(g)) * u ), g = in[r][c], u = in[r][n + c]  (8 columns per thread)
__global__ void __launch_bounds__(256) silu_mul_kernel(const __half* in, int64_t ldi, __half* out, int64_t ldo,
                                                       int rows, int n) {
    griddep_launch();
    griddep_wait();
    const int nv = n / 8;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < (int64_t)rows * nv;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / nv;
        const int c = (int)(idx % nv) * 8;
        const uint4 g = *reinterpret_cast<const uint4*>(in + r * ldi + c);
        const uint4 u = *reinterpret_cast<const uint4*>(in + r * ldi + n + c);
        uint4 o;
        o.x = h2_as_u32(silu_mul2(u32_as_h2(g.x), u32_as_h2(u.x)));
        o.y = h2_as_u32(silu_mul2(u32_as_h2(g.y), u32_as_h2(u.y)));
        o.z = h2_as_u32(silu_mul2(u32_as_h2(g.z), u32_as_h2(u.z)));
        o.w = h2_as_u32(silu_mul2(u32_as_h2(g.w), u32_as_h2(u.w)));
        *reinterpret_cast<uint4*>(out + r * ldo + c) = o;
    }
}

template <typename... Args>
static cudaError_t launch_pdl(void (*kern)(Args...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

static int glue_sms() {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
}

// ---------------------------------------------------------------------------------------------
// fp8 (e4m3) input embedding: out[t][:] = fp16(table[ids[t]][:]).  One warp per token, 16 bytes
// of the row per lane and step; every e4m3 value is exact in fp16 (the cast of torch's
// .to(float16)).  An id outside [0, rows) writes a zero row.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fp8_embedding_kernel(const uint8_t* table, int64_t rows, int64_t dim,
                                                           const void* ids, int ids_64, int64_t n, __half* out) {
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= n) return;
    const int lane = threadIdx.x & 31;
    const int64_t id = ids_64 ? static_cast<const int64_t*>(ids)[t] : (int64_t)static_cast<const int32_t*>(ids)[t];
    const bool ok = id >= 0 && id < rows;
    const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * dim);
    uint4* dst = reinterpret_cast<uint4*>(out + t * dim);
    for (int64_t c = lane; c < dim / 16; c += 32) {
        const uint4 v = ok ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t h[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xFFFFu), __NV_E4M3);
            const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
            h[2 * i] = (uint32_t)lo.x | ((uint32_t)lo.y << 16);
            h[2 * i + 1] = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
        }
        dst[2 * c] = make_uint4(h[0], h[1], h[2], h[3]);
        dst[2 * c + 1] = make_uint4(h[4], h[5], h[6], h[7]);
    }
}

}  // namespace exl3b

using namespace exl3b;

extern "C" int exl3b_rmsnorm(const uint16_t* x, int64_t ldx, uint16_t* residual, int64_t ldr, const uint16_t* weight,
                             uint16_t* out, int64_t ldo, int rows, int cols, float eps, void* stream) {
    if (rows < 0 || cols <= 0 || cols % 8 || cols > 8 * kNormMaxVec * kNormThreads) return EXL3B_DECLINED;
    if (!x || !weight || !out) return EXL3B_BAD_ARG;
    if (ldx < cols || ldo < cols || ldx % 8 || ldo % 8 || (residual && (ldr < cols || ldr % 8))) return EXL3B_BAD_ARG;
    if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(out, 16) || (residual && !aligned(residual, 16)))
        return EXL3B_BAD_ARG;
    if (rows == 0) return EXL3B_OK;
    return cuda_status(launch_pdl(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), (cudaStream_t)stream,
                                  reinterpret_cast<const __half*>(x), ldx, reinterpret_cast<__half*>(residual), ldr,
                                  reinterpret_cast<const __half*>(weight), reinterpret_cast<__half*>(out), ldo, cols,
                                  eps));
}

extern "C" int exl3b_rope_neox(uint16_t* qkv, int64_t ld, uint16_t* q_out, int64_t ld_q, int tokens, int num_q_heads,
                               int num_k_heads, const int64_t* positions, const float* cos_sin, int64_t max_position,
                               void* stream) {
    if (tokens < 0 || num_q_heads < 0 || num_k_heads < 0 || max_position < 1) return EXL3B_BAD_ARG;
    if (!qkv || !positions || !cos_sin || (num_q_heads && !q_out)) return EXL3B_BAD_ARG;
    if (ld < (int64_t)(num_q_heads + num_k_heads) * 128 || ld % 2 || (num_q_heads && (ld_q < num_q_heads * 128 || ld_q % 2)))
        return EXL3B_BAD_ARG;
    if (!aligned(qkv, 4) || (q_out && !aligned(q_out, 4)) || !aligned(cos_sin, 8) || !aligned(positions, 8))
        return EXL3B_BAD_ARG;
    if (tokens == 0 || num_q_heads + num_k_heads == 0) return EXL3B_OK;
    return cuda_status(launch_pdl(rope_kernel, dim3(tokens), dim3(256), (cudaStream_t)stream,
                                  reinterpret_cast<__half*>(qkv), ld, reinterpret_cast<__half*>(q_out), ld_q,
                                  num_q_heads, num_k_heads, positions, cos_sin, max_position));
}

extern "C" int exl3b_silu_mul(const uint16_t* in, int64_t ld_in, uint16_t* out, int64_t ld_out, int rows, int n,
                              void* stream) {
    if (rows < 0 || n <= 0 || n % 8) return EXL3B_DECLINED;
    if (!in || !out || ld_in < 2 * (int64_t)n || ld_out < n || ld_in % 8 || ld_out % 8) return EXL3B_BAD_ARG;
    if (!aligned(in, 16) || !aligned(out, 16)) return EXL3B_BAD_ARG;
    if (rows == 0) return EXL3B_OK;
    const int64_t work = (int64_t)rows * (n / 8);
    const int blocks = (int)std::min<int64_t>((work + 255) / 256, 8LL * glue_sms());
    return cuda_status(launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), (cudaStream_t)stream,
                                  reinterpret_cast<const __half*>(in), ld_in, reinterpret_cast<__half*>(out), ld_out,
                                  rows, n));
}

extern "C" int exl3b_fp8_embedding(const uint8_t* table, int64_t rows, int64_t dim, const void* ids, int ids_64,
                                   int64_t n, uint16_t* out, void* stream) {
    if (rows <= 0 || dim <= 0 || n < 0) return EXL3B_BAD_ARG;
    if (dim % 16) return EXL3B_DECLINED;
    if (n == 0) return EXL3B_OK;
    if (!table || !ids || !out || !aligned(table, 16) || !aligned(out, 16)) return EXL3B_BAD_ARG;
    const unsigned grid = (unsigned)((n + 7) / 8);
    fp8_embedding_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(table, rows, dim, ids, ids_64 ? 1 : 0, n,
                                                                 reinterpret_cast<__half*>(out));
    return cuda_status(cudaGetLastError());
}
