// Codebook decode, trellis dequantisation ("reconstruct") and the standalone 128-point Hadamard.
//
// dequant: reference exllamav3_ext.reconstruct / reconstruct_slice (vllm_plugin/exl3rocm/ops.py:92-95),
// semantics reference/exl3_oracle.py:156-219.  had128: exllamav3_ext.had_r_128 (ops.py:88,97),
// semantics reference/exl3_oracle.py:264-301.
#include "exl3b_common.cuh"

namespace exl3b {

template <int CB>
__global__ void decode_states_kernel(const uint16_t* __restrict__ states, float* __restrict__ out, int64_t count) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) out[i] = __half2float(decode_one<CB>(states[i]));
}

// One warp per 16x16 tile, eight warps per block.  Lane L decodes positions 8L..8L+7 into a
// per-warp shared tile, then the warp writes the tile's 16 rows with 16-byte stores.
template <int K, int CB>
__global__ void __launch_bounds__(256) dequant_kernel(const uint16_t* __restrict__ trellis, int k_tiles, int n_tiles,
                                                      int nt0, int nt1, __half* __restrict__ W, int64_t ldw) {
    __shared__ __align__(16) __half tile_s[8][16][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int width = nt1 - nt0;
    const int64_t tile = (int64_t)blockIdx.x * 8 + warp;
    if (tile >= (int64_t)k_tiles * width) return;
    const int kt = (int)(tile / width), nt = nt0 + (int)(tile % width);

    LaneGeom<K> g;
    g.init(lane);
    const uint8_t* base = reinterpret_cast<const uint8_t*>(trellis + ((int64_t)kt * n_tiles + nt) * 16 * K);
    uint32_t Wd[LaneGeom<K>::kNW];
#pragma unroll
    for (int j = 0; j < LaneGeom<K>::kNW; ++j) Wd[j] = __ldg(reinterpret_cast<const uint32_t*>(base + g.off[j]));
    uint32_t w[8];
    lane_windows<K>(Wd, g.phi, w);
    const int r0 = 2 * (lane & 3), cA = lane >> 2;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const __half2 v = u32_as_h2(decode_pair<CB>(w[i], w[i + 1]));
        const int row = r0 + 8 * ((i >> 1) & 1), col = cA + 8 * (i >> 2);
        tile_s[warp][row][col] = __low2half(v);
        tile_s[warp][row + 1][col] = __high2half(v);
    }
    __syncwarp();
    const int row = lane >> 1, half8 = (lane & 1) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(&tile_s[warp][row][half8]);
    __half* dst = W + (int64_t)(kt * 16 + row) * ldw + (int64_t)(nt - nt0) * 16 + half8;
    *reinterpret_cast<uint4*>(dst) = v;
}

// One warp per (row, 128-column block).
__global__ void had128_kernel(const __half* in, int64_t ld_in, __half* out, int64_t ld_out, int64_t rows,
                              int64_t blocks, const __half* __restrict__ pre, const __half* __restrict__ post,
                              float scale) {
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= rows * blocks) return;
    const int lane = threadIdx.x & 31;
    const int64_t r = item / blocks, b = item % blocks;
    const int64_t c = b * 128 + 4 * lane;
    const uint2 raw = *reinterpret_cast<const uint2*>(in + r * ld_in + c);
    __half2 h01 = u32_as_h2(raw.x), h23 = u32_as_h2(raw.y);
    if (pre) {
        const uint2 p = *reinterpret_cast<const uint2*>(pre + c);
        h01 = __hmul2(h01, u32_as_h2(p.x));
        h23 = __hmul2(h23, u32_as_h2(p.y));
    }
    float v[4] = {__low2float(h01), __high2float(h01), __low2float(h23), __high2float(h23)};
    had128_warp(v);
    const float s = kRScale * scale;
    h01 = __floats2half2_rn(v[0] * s, v[1] * s);
    h23 = __floats2half2_rn(v[2] * s, v[3] * s);
    if (post) {
        const uint2 q = *reinterpret_cast<const uint2*>(post + c);
        h01 = __hmul2(h01, u32_as_h2(q.x));
        h23 = __hmul2(h23, u32_as_h2(q.y));
    }
    *reinterpret_cast<uint2*>(out + r * ld_out + c) = make_uint2(h2_as_u32(h01), h2_as_u32(h23));
}

template <int CB>
static cudaError_t launch_dequant_cb(int K, const uint16_t* tr, int kt, int ntl, int nt0, int nt1, __half* W,
                                     int64_t ldw, cudaStream_t st) {
    const int64_t tiles = (int64_t)kt * (nt1 - nt0);
    const dim3 grid((unsigned)((tiles + 7) / 8)), block(256);
    switch (K) {
        case 1: dequant_kernel<1, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
        case 2: dequant_kernel<2, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
        case 3: dequant_kernel<3, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
        case 4: dequant_kernel<4, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
        case 5: dequant_kernel<5, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
        case 6: dequant_kernel<6, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
        case 7: dequant_kernel<7, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
        default: dequant_kernel<8, CB><<<grid, block, 0, st>>>(tr, kt, ntl, nt0, nt1, W, ldw); break;
    }
    return cudaGetLastError();
}

}  // namespace exl3b

using namespace exl3b;

extern "C" int exl3b_decode_states(const uint16_t* states, float* out, int64_t count, int codebook, void* stream) {
    if (count < 0 || codebook < 0 || codebook > 2) return EXL3B_BAD_ARG;
    if (count == 0) return EXL3B_OK;
    if (!states || !out) return EXL3B_BAD_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const unsigned grid = (unsigned)((count + 255) / 256);
    switch (codebook) {
        case 0: decode_states_kernel<0><<<grid, 256, 0, st>>>(states, out, count); break;
        case 1: decode_states_kernel<1><<<grid, 256, 0, st>>>(states, out, count); break;
        default: decode_states_kernel<2><<<grid, 256, 0, st>>>(states, out, count); break;
    }
    return cuda_status(cudaGetLastError());
}

extern "C" int exl3b_dequant(const uint16_t* trellis, int k, int n, int K, int codebook, int n0, int n1,
                             uint16_t* W, int64_t ldw, void* stream) {
    if (K < 1 || K > 8 || codebook < 0 || codebook > 2) return EXL3B_DECLINED;
    if (k <= 0 || n <= 0 || k % 16 || n % 16 || n0 < 0 || n1 > n || n0 >= n1 || n0 % 16 || n1 % 16)
        return EXL3B_BAD_ARG;
    if (!trellis || !W || ldw < n1 - n0 || ldw % 8 || !aligned(W, 16) || !aligned(trellis, 4)) return EXL3B_BAD_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    __half* Wh = reinterpret_cast<__half*>(W);
    cudaError_t e;
    switch (codebook) {
        case 0: e = launch_dequant_cb<0>(K, trellis, k / 16, n / 16, n0 / 16, n1 / 16, Wh, ldw, st); break;
        case 1: e = launch_dequant_cb<1>(K, trellis, k / 16, n / 16, n0 / 16, n1 / 16, Wh, ldw, st); break;
        default: e = launch_dequant_cb<2>(K, trellis, k / 16, n / 16, n0 / 16, n1 / 16, Wh, ldw, st); break;
    }
    return cuda_status(e);
}

extern "C" int exl3b_had128(const uint16_t* in, int64_t ld_in, uint16_t* out, int64_t ld_out, int64_t rows,
                            int64_t cols, const uint16_t* pre, const uint16_t* post, float scale, void* stream) {
    if (rows < 0 || cols < 0 || cols % 128) return EXL3B_BAD_ARG;
    if (rows == 0 || cols == 0) return EXL3B_OK;
    if (!in || !out || ld_in < cols || ld_out < cols || ld_in % 4 || ld_out % 4) return EXL3B_BAD_ARG;
    if (!aligned(in, 8) || !aligned(out, 8) || (pre && !aligned(pre, 8)) || (post && !aligned(post, 8)))
        return EXL3B_BAD_ARG;
    const int64_t items = rows * (cols / 128);
    const unsigned grid = (unsigned)((items + 7) / 8);
    had128_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const __half*>(in), ld_in, reinterpret_cast<__half*>(out), ld_out, rows, cols / 128,
        reinterpret_cast<const __half*>(pre), reinterpret_cast<const __half*>(post), scale);
    return cuda_status(cudaGetLastError());
}

extern "C" int exl3b_version(void) { return (0 << 16) | (1 << 8) | 0; }

extern "C" const char* exl3b_status_string(int status) {
    switch (status) {
        case EXL3B_OK: return "ok";
        case EXL3B_DECLINED: return "declined: shape or flags not implemented by the kernels";
        case EXL3B_BAD_ARG: return "bad argument: null or misaligned pointer, or bad size";
        case EXL3B_WORKSPACE: return "workspace too small";
        case EXL3B_TOO_LARGE: return "call needs more scratch than the static scratch array of exl3b_linear_noalloc holds";
        default: break;
    }
    if (status < 0) return cudaGetErrorString((cudaError_t)(-status));
    return "unknown status";
}
