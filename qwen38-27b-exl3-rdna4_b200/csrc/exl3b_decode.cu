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

// Four lanes per (row, 128-column block), eight blocks per warp.  Lane j of a block holds its
// 4-element chunks l = j + 4i (i = 0..7): H4 inside a chunk, then chunk distances 1 and 2 between the
// block's lanes and 4, 8, 16 inside a lane, the operations and order of had128_warp (a warp holding
// chunk l in lane l), so the results are the same bit for bit with two shuffle stages instead of five
// (one warp per block ran 77 us for 213 MB, issue-bound on its shuffles).
constexpr int kHadBlocksPerWarp = 8;
__global__ void __launch_bounds__(256) had128_kernel(const __half* in, int64_t ld_in, __half* out, int64_t ld_out,
                                                     int64_t rows, int64_t blocks, const __half* __restrict__ pre,
                                                     const __half* __restrict__ post, float scale) {
    const int lane = threadIdx.x & 31, j = lane & 3;
    const int64_t item = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kHadBlocksPerWarp +
                         (lane >> 2);
    const bool live = item < rows * blocks;  // dead lanes run along (they take part in the shuffles)
    const int64_t r = live ? item / blocks : 0, b = live ? item % blocks : 0;
    float v[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t c = b * 128 + 16 * i + 4 * j;
        uint2 raw = live ? *reinterpret_cast<const uint2*>(in + r * ld_in + c) : make_uint2(0u, 0u);
        __half2 h01 = u32_as_h2(raw.x), h23 = u32_as_h2(raw.y);
        if (pre && live) {
            const uint2 p = *reinterpret_cast<const uint2*>(pre + c);
            h01 = __hmul2(h01, u32_as_h2(p.x));
            h23 = __hmul2(h23, u32_as_h2(p.y));
        }
        const float x0 = __low2float(h01), x1 = __high2float(h01), x2 = __low2float(h23), x3 = __high2float(h23);
        const float s0 = x0 + x1, d0 = x0 - x1, s1 = x2 + x3, d1 = x2 - x3;
        v[i][0] = s0 + s1; v[i][1] = d0 + d1; v[i][2] = s0 - s1; v[i][3] = d0 - d1;
    }
#pragma unroll
    for (int d = 1; d <= 2; d <<= 1) {
        const bool upper = (j & d) != 0;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float o = __shfl_xor_sync(0xFFFFFFFFu, v[i][e], d);
                v[i][e] = upper ? (o - v[i][e]) : (v[i][e] + o);
            }
    }
#pragma unroll
    for (int d = 1; d <= 4; d <<= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (!(i & d))
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float lo = v[i][e], hi = v[i | d][e];
                    v[i][e] = lo + hi;
                    v[i | d][e] = lo - hi;
                }
    if (!live) return;
    const float s = kRScale * scale;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t c = b * 128 + 16 * i + 4 * j;
        __half2 h01 = __floats2half2_rn(v[i][0] * s, v[i][1] * s);
        __half2 h23 = __floats2half2_rn(v[i][2] * s, v[i][3] * s);
        if (post) {
            const uint2 q = *reinterpret_cast<const uint2*>(post + c);
            h01 = __hmul2(h01, u32_as_h2(q.x));
            h23 = __hmul2(h23, u32_as_h2(q.y));
        }
        *reinterpret_cast<uint2*>(out + r * ld_out + c) = make_uint2(h2_as_u32(h01), h2_as_u32(h23));
    }
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
    const int64_t per_block = 8 * kHadBlocksPerWarp;  // 8 warps per CTA
    const unsigned grid = (unsigned)((items + per_block - 1) / per_block);
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
