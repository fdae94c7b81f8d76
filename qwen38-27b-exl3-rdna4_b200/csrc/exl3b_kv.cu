// Paged KV cache on B200: int8 and int4 per-token-head quantize-on-write and split-KV decode /
// speculative-verify attention.
//
// Cache formats (bytes identical to the formats the reference serves):
//   int8  key/value [blocks][block_size][Hkv][128] int8, scales [blocks][block_size][Hkv] fp32
//         (vLLM int8_per_token_head, written by vllm/v1/attention/ops/triton_reshape_and_cache_flash.py
//         :139-238; read by triton_unified_attention.py:473-545)
//   int4  key/value [blocks][block_size][Hkv][64] uint8, element 2i in the low nibble of byte i,
//         scales [blocks][block_size][Hkv] fp32 whose low 4 mantissa bits hold the zero point;
//         values live in the randomised-Hadamard (RHT) domain, unnormalised (reference
//         vllm_plugin/exl3rocm/kv_int4.py:161-173, 272-342)
//   int4 exact rows: per request slot [SINKS + TAIL][Hkv][128] fp16 for K and V plus int32 tags
//         [SINKS + TAIL]; position p < SINKS lives in row p, other positions in row
//         SINKS + p % TAIL; a row is used only when its tag equals the position (kv_int4.py:92-118).
//
// Attention works on one (sequence, KV head, split of the context) per CTA; each warp owns 16 query
// rows (query token x GQA head) and walks the split in 32-token tiles with mma.m16n8k16: S = Q K^T
// then O += P V with fp32 accumulation and an online softmax.  The head dimension is permuted
// consistently in Q, K and V so that every lane reads its cache bytes as 16-byte contiguous loads;
// the permutation is undone when the partial outputs are written.  A second kernel combines the
// splits (vLLM reduce_segments) and, for int4, undoes the rotation.
#include <mutex>

#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kHD = 128;        // head dimension
constexpr int kSinks = 4;       // exact rows at the start of a sequence (kv_int4.py:47)
constexpr int kTail = 128;      // exact rows at the end of a sequence (kv_int4.py:48)
constexpr int kExactRows = kSinks + kTail;
constexpr float kClipStep = 0.075f;  // kv_int4.py:213
constexpr int kClipSteps = 3;
constexpr int kMaxSplits = 64;  // kv_int4.py:43
// one split's partial for one (token, query head): acc[128], m, l, padded to 132 floats so that
// every record starts on a 16-byte boundary (the kernels move it as float4)
constexpr int kPartialStride = kHD + 4;

EXL3B_DEV float load_in(const void* p, int64_t i, int dtype) {
    return dtype == 0 ? __half2float(reinterpret_cast<const __half*>(p)[i])
                      : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

EXL3B_DEV float warp_max(float v) {
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, d));
    return v;
}
EXL3B_DEV float warp_min(float v) {
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) v = fminf(v, __shfl_xor_sync(0xFFFFFFFFu, v, d));
    return v;
}
// xor butterfly with distances 16, 8, 4, 2, 1 (the oracle's order); every lane ends with the sum
EXL3B_DEV float warp_sum(float v) {
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, d));
    return v;
}

// ---------------------------------------------------------------------------------------------
// int8 write: one warp per (token, KV head); lane l owns elements 4l..4l+3
// ---------------------------------------------------------------------------------------------
struct KvWriteArgs {
    const void* key; const void* value; int dtype;    // [T][H][128], row strides in elements
    int64_t k_stride_tok, k_stride_head, v_stride_tok, v_stride_head;
    void* key_cache; void* value_cache; float* k_scale; float* v_scale;
    const int64_t* slot_mapping;
    int num_tokens, num_heads, block_size;
};

EXL3B_DEV void int8_quant_store(const float (&x)[4], int8_t* dst, float* scale_dst, int lane) {
    const float amax = warp_max(fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3]))));
    const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-6f);
    const float inv = __fdiv_rn(1.f, scale);
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float q = fminf(fmaxf(__fmul_rn(x[i], inv), -128.f), 127.f);
        packed |= ((uint32_t)(__float2int_rz(q) & 0xFF)) << (8 * i);
    }
    reinterpret_cast<uint32_t*>(dst)[lane] = packed;
    if (lane == 0) *scale_dst = scale;
}

__global__ void kv_int8_write_kernel(const KvWriteArgs a) {
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= (int64_t)a.num_tokens * a.num_heads) return;
    const int lane = threadIdx.x & 31;
    const int t = (int)(item / a.num_heads), h = (int)(item % a.num_heads);
    const int64_t slot = a.slot_mapping[t];
    if (slot < 0) return;
    const int64_t blk = slot / a.block_size, off = slot % a.block_size;
    const int64_t row = (blk * a.block_size + off) * a.num_heads + h;
    float xk[4], xv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        xk[i] = load_in(a.key, t * a.k_stride_tok + h * a.k_stride_head + 4 * lane + i, a.dtype);
        xv[i] = load_in(a.value, t * a.v_stride_tok + h * a.v_stride_head + 4 * lane + i, a.dtype);
    }
    int8_quant_store(xk, reinterpret_cast<int8_t*>(a.key_cache) + row * kHD, a.k_scale + row, lane);
    int8_quant_store(xv, reinterpret_cast<int8_t*>(a.value_cache) + row * kHD, a.v_scale + row, lane);
}

// ---------------------------------------------------------------------------------------------
// int4 write: one warp per (token, KV head, side); RHT in registers, clip search, pack, exact rows
// ---------------------------------------------------------------------------------------------
struct KvInt4Extra {
    const float* signs;             // [128] +-1 of the RHT
    const float* bias_k; const float* bias_v;  // optional [H][128] rotated-domain biases, or null
    const int32_t* query_start_loc; const int32_t* seq_lens; const int32_t* seq_slots;  // [num_seqs(+1)]
    int num_seqs;
    __half* exact_k; __half* exact_v; int32_t* exact_tag;  // per slot [kExactRows][H][128], [kExactRows]
};

EXL3B_DEV int round_half_away(float v) { return __float2int_rz(v >= 0.f ? __fadd_rn(v, 0.5f) : __fsub_rn(v, 0.5f)); }

// codes c[4] (0..15) for this lane's 4 elements and the row's scale bits
EXL3B_DEV void int4_quant_row(const float (&y)[4], int (&code)[4], uint32_t& sbits) {
    const float lo0 = warp_min(fminf(fminf(y[0], y[1]), fminf(y[2], y[3])));
    const float hi0 = warp_max(fmaxf(fmaxf(y[0], y[1]), fmaxf(y[2], y[3])));
    const float mu = __fmul_rn(warp_sum(__fadd_rn(__fadd_rn(__fadd_rn(y[0], y[1]), y[2]), y[3])), 1.f / 128.f);
    float best_err = __int_as_float(0x7F800000), best_sc = 0.f;
    int best_zp = 0;
#pragma unroll 1
    for (int c = 0; c < kClipSteps * kClipSteps; ++c) {
        const float flo = __fmaf_rn(-kClipStep, (float)(c / kClipSteps), 1.f);
        const float fhi = __fmaf_rn(-kClipStep, (float)(c % kClipSteps), 1.f);
        const float lo = __fmaf_rn(__fsub_rn(lo0, mu), flo, mu);
        const float hi = __fmaf_rn(__fsub_rn(hi0, mu), fhi, mu);
        const float sc = fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 15.f), 1e-6f);
        const int zp = min(max(round_half_away(__fdiv_rn(-lo, sc)), 0), 15);
        const float inv = __fdiv_rn(1.f, sc);
        float e[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int qn = min(max(round_half_away(__fmaf_rn(y[i], inv, (float)zp)), 0), 15);
            e[i] = __fmaf_rn((float)(qn - zp), sc, -y[i]);
        }
        float s = __fmul_rn(e[0], e[0]);
        s = __fmaf_rn(e[1], e[1], s);
        s = __fmaf_rn(e[2], e[2], s);
        s = __fmaf_rn(e[3], e[3], s);
        const float err = warp_sum(s);
        if (err < best_err) { best_err = err; best_sc = sc; best_zp = zp; }
    }
    const float inv = __fdiv_rn(1.f, best_sc);
#pragma unroll
    for (int i = 0; i < 4; ++i) code[i] = min(max(round_half_away(__fmaf_rn(y[i], inv, (float)best_zp)), 0), 15);
    sbits = ((uint32_t)__float_as_uint(best_sc) & 0xFFFFFFF0u) | (uint32_t)best_zp;
}

// sequence of token t from query_start_loc (binary search, as vLLM's find_seq_idx)
EXL3B_DEV int seq_of_token(const int32_t* qsl, int num_seqs, int t) {
    int lo = 0, hi = num_seqs;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (qsl[mid] <= t) lo = mid; else hi = mid - 1;
    }
    return min(lo, num_seqs - 1);
}

EXL3B_DEV int exact_row(int pos) { return pos < kSinks ? pos : kSinks + pos % kTail; }

__global__ void kv_int4_write_kernel(const KvWriteArgs a, const KvInt4Extra x) {
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= (int64_t)a.num_tokens * a.num_heads * 2) return;
    const int lane = threadIdx.x & 31;
    const int side = (int)(item & 1);
    const int t = (int)((item >> 1) / a.num_heads), h = (int)((item >> 1) % a.num_heads);
    const int64_t slot = a.slot_mapping[t];
    if (slot < 0) return;
    const void* src = side ? a.value : a.key;
    const int64_t base = side ? t * a.v_stride_tok + h * a.v_stride_head : t * a.k_stride_tok + h * a.k_stride_head;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = load_in(src, base + 4 * lane + i, a.dtype) * x.signs[4 * lane + i];
    // unnormalised Hadamard, fp32, H4 in lane then xor butterflies 1..16 (same order as had128_warp)
    had128_warp(v);
    const float* bias = side ? x.bias_v : x.bias_k;
    if (bias) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fadd_rn(v[i], bias[h * kHD + 4 * lane + i]);
    }
    int code[4];
    uint32_t sbits;
    int4_quant_row(v, code, sbits);
    const int64_t blk = slot / a.block_size, off = slot % a.block_size;
    const int64_t row = (blk * a.block_size + off) * a.num_heads + h;
    uint8_t* cache = reinterpret_cast<uint8_t*>(side ? a.value_cache : a.key_cache) + row * (kHD / 2);
    const uint16_t packed = (uint16_t)((code[0] | (code[1] << 4)) | ((code[2] | (code[3] << 4)) << 8));
    reinterpret_cast<uint16_t*>(cache)[lane] = packed;
    if (lane == 0) (side ? a.v_scale : a.k_scale)[row] = __uint_as_float(sbits);
    // exact rows
    if (x.exact_tag && x.seq_slots) {
        const int s = seq_of_token(x.query_start_loc, x.num_seqs, t);
        const int rs = x.seq_slots[s];
        const int q0 = x.query_start_loc[s], q1 = x.query_start_loc[s + 1];
        const int L = x.seq_lens[s];
        const int pos = L - (q1 - q0) + (t - q0);
        if (rs >= 0 && pos >= 0 && (pos < kSinks || pos >= L - kTail)) {
            const int e = exact_row(pos);
            __half* ex = (side ? x.exact_v : x.exact_k) + (((int64_t)rs * kExactRows + e) * a.num_heads + h) * kHD;
            reinterpret_cast<uint2*>(ex)[lane] = make_uint2(h2_as_u32(__floats2half2_rn(v[0], v[1])),
                                                           h2_as_u32(__floats2half2_rn(v[2], v[3])));
            if (side == 0 && h == 0 && lane == 0) x.exact_tag[(int64_t)rs * kExactRows + e] = pos;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// rotation kernel: out = fp16( H (in * pre) ) * post_scale (* post) per 128-row, one warp per row
// ---------------------------------------------------------------------------------------------
__global__ void kv_rotate_kernel(const __half* in, __half* out, int64_t rows, const float* pre, const float* post,
                                 float scale) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int lane = threadIdx.x & 31;
    const uint2 raw = reinterpret_cast<const uint2*>(in + r * kHD)[lane];
    float v[4] = {__low2float(u32_as_h2(raw.x)), __high2float(u32_as_h2(raw.x)), __low2float(u32_as_h2(raw.y)),
                  __high2float(u32_as_h2(raw.y))};
    if (pre) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] *= pre[4 * lane + i];
    }
    had128_warp(v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i] *= scale;
        if (post) v[i] *= post[4 * lane + i];
    }
    reinterpret_cast<uint2*>(out + r * kHD)[lane] =
        make_uint2(h2_as_u32(__floats2half2_rn(v[0], v[1])), h2_as_u32(__floats2half2_rn(v[2], v[3])));
}

// ---------------------------------------------------------------------------------------------
// split-KV attention
// ---------------------------------------------------------------------------------------------
struct KvAttnArgs {
    const __half* q;             // [T][Hq][128] (int4: already rotated)
    const void* key_cache; const void* value_cache;
    const float* k_scale; const float* v_scale;
    const int32_t* block_table; int64_t bt_stride;
    const int32_t* seq_lens; const int32_t* query_start_loc;
    int num_seqs, num_q_heads, num_kv_heads, block_size_log2, num_splits;
    float score_scale;           // softmax scale (int4: / d)
    float* partial;              // [T][Hq][splits][kPartialStride]: acc, m, l
    // int4 exact rows
    const __half* exact_k; const __half* exact_v; const int32_t* exact_tag; const int32_t* seq_slots;
};

// int8 word (4 signed bytes) -> two half2 (bytes 0,1) and (bytes 2,3), exact
EXL3B_DEV void i8x4_to_h2(uint32_t w, uint32_t& h01, uint32_t& h23) {
    const uint32_t u = w ^ 0x80808080u;                           // b + 128
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x5140);        // [u0, 0x64, u1, 0x64]
    const uint32_t b = __byte_perm(u, 0x64646464u, 0x7362);        // [u2, 0x64, u3, 0x64]
    const __half2 off = u32_as_h2(0x64806480u);                    // 1152
    h01 = h2_as_u32(__hsub2(u32_as_h2(a), off));
    h23 = h2_as_u32(__hsub2(u32_as_h2(b), off));
}

// nibbles i and i+4 of an 8-nibble word, minus the zero point, as half2 (exact)
EXL3B_DEV uint32_t nib_pair(uint32_t w, int s, uint32_t zp_h2) {
    const uint32_t v = ((w >> (4 * s)) & 0x000F000Fu) | 0x64006400u;  // (1024 + n_s, 1024 + n_{s+4})
    return h2_as_u32(__hsub2(u32_as_h2(v), u32_as_h2(zp_h2)));
}

EXL3B_DEV float exp_f(float x) { return exp2f(x * 1.4426950408889634f); }

template <int KV>
struct KvTraits;

// The d permutation of the QK^T product, per MMA k-chunk c (0..7) and lane q:
//   int8: k-slots (2q, 2q+1, 2q+8, 2q+9) <- d = 32q + 4c + (0, 1, 2, 3)
//   int4: k-slots (2q, 2q+1, 2q+8, 2q+9) <- d = 32q + 8(c/2) + 2(c%2) + (0, 4, 1, 5)
// and of P V, per lane g: output column n of n-tile j is d = 16n + j, so lane g reads every token's
// values at d = 16g .. 16g+15.  In the V half2 pairs p = 0..7 cover (jA(p), jB(p)):
//   int8: (2p, 2p+1);   int4: (8(p/4) + p%4, 8(p/4) + p%4 + 4)
template <>
struct KvTraits<8> {
    EXL3B_DEV static int dmap(int q, int c, int slot) { return 32 * q + 4 * c + slot; }
    EXL3B_DEV static int jA(int p) { return 2 * p; }
    EXL3B_DEV static int jB(int p) { return 2 * p + 1; }
};
template <>
struct KvTraits<4> {
    EXL3B_DEV static int dmap(int q, int c, int slot) {
        const int add = (slot == 0) ? 0 : (slot == 1) ? 4 : (slot == 2) ? 1 : 5;
        return 32 * q + 8 * (c / 2) + 2 * (c % 2) + add;
    }
    EXL3B_DEV static int jA(int p) { return 8 * (p / 4) + p % 4; }
    EXL3B_DEV static int jB(int p) { return 8 * (p / 4) + p % 4 + 4; }
};

// Per-warp shared memory: a ring of kRing tiles (32 tokens: K rows, V rows, k scales, v scales)
// filled with cp.async one tile ahead of the math, and a window of the split's block ids.
template <int KV>
struct AttnSmem {
    static constexpr int kRowBytes = KV == 8 ? kHD : kHD / 2;
    static constexpr int kRows = 32 * kRowBytes;                  // K (or V) bytes of one tile
    static constexpr int kTile = 2 * kRows + 2 * 32 * 4;          // K, V, k scales, v scales
    static constexpr int kRing = KV == 8 ? 2 : 3;
    static constexpr int kBtWindow = 256;                          // block ids kept per warp
    static constexpr int kWarpBytes = kRing * kTile + kBtWindow * 4;
};

EXL3B_DEV void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" :: "r"(dst), "l"(src) : "memory");
}
EXL3B_DEV void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" :: "r"(dst), "l"(src) : "memory");
}
EXL3B_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
EXL3B_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" :: "n"(N) : "memory"); }

template <int KV, int MT>
__global__ void __launch_bounds__(32 * MT) kv_attn_kernel(const KvAttnArgs a) {
    using Tr = KvTraits<KV>;
    using SM = AttnSmem<KV>;
    constexpr int RB = SM::kRowBytes;
    constexpr int C16 = RB / 16;  // 16-byte chunks per row (8 or 4)
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int seq = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const int L = a.seq_lens[seq];
    const int q0 = a.query_start_loc[seq], qlen = a.query_start_loc[seq + 1] - q0;
    if (qlen <= 0 || L <= 0) return;
    const int G = a.num_q_heads / a.num_kv_heads;
    const int rows = qlen * G;
    const int per = ((L + a.num_splits - 1) / a.num_splits + 31) & ~31;  // tokens per split, x32
    const int t_lo = split * per, t_hi = min(L, t_lo + per);
    if (t_lo >= t_hi) return;  // empty split: the reduce kernel skips it
    // row r of the sequence = query (r / G), head kvh*G + r % G; this warp owns rows 16w .. 16w+15
    const int rbase = 16 * warp;
    if (rbase >= rows) return;  // no CTA-wide barrier below: warps run independently
    const int r_lo = rbase + gq, r_hi = rbase + gq + 8;

    uint8_t* wsm = smem_raw + warp * SM::kWarpBytes;
    const uint32_t wsm_u = smem_u32(wsm);
    int32_t* bt_win = reinterpret_cast<int32_t*>(wsm + SM::kRing * SM::kTile);
    const int32_t* bt = a.block_table + (int64_t)seq * a.bt_stride;
    const int lg = a.block_size_log2, bs_mask = (1 << lg) - 1;
    int win_base = -1;  // first block index held in bt_win

    // ---- Q fragments: A[r][k-slot] = Q[row r][dmap] ----
    uint32_t qa[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
            const int r = hrow ? r_hi : r_lo;
            __half v4[4] = {__float2half(0.f), __float2half(0.f), __float2half(0.f), __float2half(0.f)};
            if (r < rows) {
                const __half* qrow = a.q + ((int64_t)(q0 + r / G) * a.num_q_heads + kvh * G + r % G) * kHD;
#pragma unroll
                for (int s = 0; s < 4; ++s) v4[s] = qrow[Tr::dmap(tq, c, s)];
            }
            qa[c][hrow] = h2_as_u32(__halves2half2(v4[0], v4[1]));      // k-slots 2q, 2q+1
            qa[c][hrow + 2] = h2_as_u32(__halves2half2(v4[2], v4[3]));  // k-slots 2q+8, 2q+9
        }
    }

    // ---- tile loader: all of a 32-token tile's rows and scales, one cp.async group ----
    // Row r of a tile is stored with its 16-byte chunks XOR-swizzled by (r & (C16 - 1)), so that
    // the lanes reading the same chunk index of different rows hit different banks.
    const int ntiles = (t_hi - t_lo + 31) >> 5;
    auto issue_tile = [&](int ti) {
        const int t0 = t_lo + 32 * ti;
        // block-id window: refill when the tile leaves it (the window is private to this warp)
        const int b_first = t0 >> lg, b_last = min(t0 + 31, t_hi - 1) >> lg;
        if (win_base < 0 || b_first < win_base || b_last >= win_base + SM::kBtWindow) {
            __syncwarp();
            win_base = b_first;
            const int nb = min(SM::kBtWindow, ((t_hi - 1) >> lg) - b_first + 1);
            for (int i = lane; i < nb; i += 32) bt_win[i] = bt[b_first + i];
            __syncwarp();
        }
        const uint32_t tb = wsm_u + (ti % SM::kRing) * SM::kTile;
#pragma unroll
        for (int j = 0; j < C16; ++j) {  // 32 rows x C16 chunks, C16 per lane per side
            const int cidx = lane + 32 * j;
            const int r = cidx / C16, ch = cidx % C16;
            const int t = t0 + r;
            if (t < t_hi) {
                const int64_t blk = bt_win[(t >> lg) - win_base];
                const int64_t row = ((blk << lg) + (t & bs_mask)) * a.num_kv_heads + kvh;
                const uint32_t soff = r * RB + ((ch ^ (r & (C16 - 1))) * 16);
                cp_async16(tb + soff, reinterpret_cast<const uint8_t*>(a.key_cache) + row * RB + ch * 16);
                cp_async16(tb + SM::kRows + soff, reinterpret_cast<const uint8_t*>(a.value_cache) + row * RB + ch * 16);
            }
        }
        {
            const int t = t0 + lane;
            if (t < t_hi) {
                const int64_t blk = bt_win[(t >> lg) - win_base];
                const int64_t row = ((blk << lg) + (t & bs_mask)) * a.num_kv_heads + kvh;
                cp_async4(tb + 2 * SM::kRows + lane * 4, a.k_scale + row);
                cp_async4(tb + 2 * SM::kRows + 128 + lane * 4, a.v_scale + row);
            }
        }
        cp_async_commit();
    };

    float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
    float acc[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
    // causal limit of rows g and g+8: key t allowed if t <= L - qlen + query index
    const int lim0 = (r_lo < rows) ? L - qlen + r_lo / G : -1;
    const int lim1 = (r_hi < rows) ? L - qlen + r_hi / G : -1;
    const int rs = (KV == 4 && a.seq_slots) ? a.seq_slots[seq] : -1;
    auto exact_of = [&](int t) -> int {  // exact row of position t, or -1 (int4 only)
        if (KV != 4 || rs < 0 || a.exact_tag == nullptr) return -1;
        if (!(t < kSinks || t >= L - kTail)) return -1;
        const int e = exact_row(t);
        return a.exact_tag[(int64_t)rs * kExactRows + e] == t ? e : -1;
    };

    for (int ti = 0; ti < SM::kRing - 1 && ti < ntiles; ++ti) issue_tile(ti);

    for (int ti = 0; ti < ntiles; ++ti) {
        if (ti + SM::kRing - 1 < ntiles) issue_tile(ti + SM::kRing - 1);
        else cp_async_commit();  // keep the group count in step
        cp_async_wait<SM::kRing - 1>();
        __syncwarp();
        const int t0 = t_lo + 32 * ti;
        const uint8_t* tile = wsm + (ti % SM::kRing) * SM::kTile;
        const float* ksc_s = reinterpret_cast<const float*>(tile + 2 * SM::kRows);
        const float* vsc_s = ksc_s + 32;
        auto chunk_at = [&](int side, int r, int ch) -> uint4 {
            return *reinterpret_cast<const uint4*>(tile + side * SM::kRows + r * RB + ((ch ^ (r & (C16 - 1))) * 16));
        };

        // ---------------- S = Q K^T for 4 n-tiles of 8 tokens ----------------
        float s[4][4];
        float ksc_tok[4];
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            const int r = 8 * n + gq, t = t0 + r;
            uint32_t b[8][2];
            float ksc = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) b[c][0] = b[c][1] = 0u;
            if (t < t_hi) {
                const int e = exact_of(t);
                if (e >= 0) {
                    const __half* ex = a.exact_k + (((int64_t)rs * kExactRows + e) * a.num_kv_heads + kvh) * kHD;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        b[c][0] = h2_as_u32(__halves2half2(ex[Tr::dmap(tq, c, 0)], ex[Tr::dmap(tq, c, 1)]));
                        b[c][1] = h2_as_u32(__halves2half2(ex[Tr::dmap(tq, c, 2)], ex[Tr::dmap(tq, c, 3)]));
                    }
                    ksc = 1.f;
                } else if constexpr (KV == 8) {
                    const uint4 w0 = chunk_at(0, r, 2 * tq), w1 = chunk_at(0, r, 2 * tq + 1);
                    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int c = 0; c < 8; ++c) i8x4_to_h2(w[c], b[c][0], b[c][1]);
                    ksc = ksc_s[r];
                } else {
                    const uint4 w4 = chunk_at(0, r, tq);
                    const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
                    const uint32_t sb = __float_as_uint(ksc_s[r]);
                    const uint32_t zp = 0x6400u | (sb & 0xFu);
                    const uint32_t zp2 = zp | (zp << 16);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        b[c][0] = nib_pair(w[c / 2], 2 * (c % 2), zp2);
                        b[c][1] = nib_pair(w[c / 2], 2 * (c % 2) + 1, zp2);
                    }
                    ksc = __uint_as_float(sb & 0xFFFFFFF0u);
                }
            }
            ksc_tok[n] = ksc;
            float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 8; ++c) mma_16816(d4, qa[c], b[c][0], b[c][1]);
#pragma unroll
            for (int e = 0; e < 4; ++e) s[n][e] = d4[e];
        }
        // scale and mask: this lane holds S[row g (e<2) / g+8 (e>=2)][token 8n + 2tq + (e&1)]
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 4; ++n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int t = t0 + 8 * n + 2 * tq + (e & 1);
                const float ks = __shfl_sync(0xFFFFFFFFu, ksc_tok[n], (2 * tq + (e & 1)) * 4);
                const bool ok = t < t_hi && t <= ((e < 2) ? lim0 : lim1);
                s[n][e] = ok ? s[n][e] * (a.score_scale * ks) : -INFINITY;
                mx[e >> 1] = fmaxf(mx[e >> 1], s[n][e]);
            }
        }
        float corr[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 2));
            const float mnew = fmaxf(m_i[h], mx[h]);
            corr[h] = (mnew == -INFINITY) ? 1.f : exp_f(m_i[h] - mnew);
            m_i[h] = mnew;
        }
        float rowsum[2] = {0.f, 0.f};
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mm = m_i[e >> 1];
                const float p = (mm == -INFINITY) ? 0.f : exp_f(s[n][e] - mm);
                s[n][e] = p;
                rowsum[e >> 1] += p;
            }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            rowsum[h] += __shfl_xor_sync(0xFFFFFFFFu, rowsum[h], 1);
            rowsum[h] += __shfl_xor_sync(0xFFFFFFFFu, rowsum[h], 2);
            l_i[h] = l_i[h] * corr[h] + rowsum[h];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            acc[j][0] *= corr[0]; acc[j][1] *= corr[0];
            acc[j][2] *= corr[1]; acc[j][3] *= corr[1];
        }
        // ---------------- O += (P * v_scale) V, two k-chunks of 16 tokens ----------------
#pragma unroll
        for (int kc = 0; kc < 2; ++kc) {
            float vs4[4];
            uint32_t vh[4][8];  // half2 pairs (jA(p), jB(p)) of d = 16 gq + j, for the lane's 4 tokens
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = 16 * kc + 2 * tq + (i & 1) + 8 * (i >> 1);
                const int t = t0 + r;
                vs4[i] = 0.f;
#pragma unroll
                for (int p = 0; p < 8; ++p) vh[i][p] = 0u;
                if (t < t_hi) {
                    const int e = exact_of(t);
                    if (e >= 0) {
                        const uint4* ep = reinterpret_cast<const uint4*>(
                            a.exact_v + (((int64_t)rs * kExactRows + e) * a.num_kv_heads + kvh) * kHD + 16 * gq);
                        const uint4 h0 = ep[0], h1 = ep[1];
                        const uint32_t nat[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};  // (2p, 2p+1)
                        // re-pair into the int4 layout (j, j+4), j = 8(p/4) + p%4: v[j] and v[j+4]
                        // sit in the same half of nat[j/2] and nat[j/2 + 2]
#pragma unroll
                        for (int p = 0; p < 8; ++p) {
                            const int j = 8 * (p / 4) + p % 4;
                            vh[i][p] = __byte_perm(nat[j / 2], nat[j / 2 + 2], (j & 1) ? 0x7632u : 0x5410u);
                        }
                        vs4[i] = 1.f;
                    } else if constexpr (KV == 8) {
                        const uint4 w4 = chunk_at(1, r, gq);
                        const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                        for (int c = 0; c < 4; ++c) i8x4_to_h2(w[c], vh[i][2 * c], vh[i][2 * c + 1]);
                        vs4[i] = vsc_s[r];
                    } else {
                        // this lane's 8 bytes (d = 16 gq .. 16 gq + 15) are the half gq & 1 of chunk gq / 2
                        const uint4 w4 = chunk_at(1, r, gq >> 1);
                        const uint32_t w[2] = {(gq & 1) ? w4.z : w4.x, (gq & 1) ? w4.w : w4.y};
                        const uint32_t sb = __float_as_uint(vsc_s[r]);
                        const uint32_t zp = 0x6400u | (sb & 0xFu);
                        const uint32_t zp2 = zp | (zp << 16);
#pragma unroll
                        for (int p = 0; p < 8; ++p) vh[i][p] = nib_pair(w[p / 4], p % 4, zp2);
                        vs4[i] = __uint_as_float(sb & 0xFFFFFFF0u);
                    }
                }
            }
            uint32_t pa[4];
            pa[0] = h2_as_u32(__floats2half2_rn(s[2 * kc][0] * vs4[0], s[2 * kc][1] * vs4[1]));
            pa[1] = h2_as_u32(__floats2half2_rn(s[2 * kc][2] * vs4[0], s[2 * kc][3] * vs4[1]));
            pa[2] = h2_as_u32(__floats2half2_rn(s[2 * kc + 1][0] * vs4[2], s[2 * kc + 1][1] * vs4[3]));
            pa[3] = h2_as_u32(__floats2half2_rn(s[2 * kc + 1][2] * vs4[2], s[2 * kc + 1][3] * vs4[3]));
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                // b0 of n-tile j = (token 2tq, token 2tq+1) at j; b1 = (2tq+8, 2tq+9)
                const uint32_t bA0 = __byte_perm(vh[0][p], vh[1][p], 0x5410);  // jA
                const uint32_t bB0 = __byte_perm(vh[0][p], vh[1][p], 0x7632);  // jB
                const uint32_t bA1 = __byte_perm(vh[2][p], vh[3][p], 0x5410);
                const uint32_t bB1 = __byte_perm(vh[2][p], vh[3][p], 0x7632);
                mma_16816(acc[Tr::jA(p)], pa, bA0, bA1);
                mma_16816(acc[Tr::jB(p)], pa, bB0, bB1);
            }
        }
        __syncwarp();  // the ring slot of this tile is refilled next iteration
    }
    cp_async_wait<0>();

    // ---- partial of this split: acc (d order restored), m, l ----
    // lane (g, q) holds for row g: d = 32q + j (acc[j][0]) and 32q + 16 + j (acc[j][1]); row g+8: [2], [3]
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
        const int r = hrow ? r_hi : r_lo;
        if (r >= rows) continue;
        const int64_t tok = q0 + r / G;
        const int hq = kvh * G + r % G;
        float* dst = a.partial + ((tok * a.num_q_heads + hq) * a.num_splits + split) * kPartialStride;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            float4* d4 = reinterpret_cast<float4*>(dst + 32 * tq + 16 * half);
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4)
                d4[j4] = make_float4(acc[4 * j4][2 * hrow + half], acc[4 * j4 + 1][2 * hrow + half],
                                     acc[4 * j4 + 2][2 * hrow + half], acc[4 * j4 + 3][2 * hrow + half]);
        }
        if (tq == 0) {
            dst[kHD] = m_i[hrow];
            dst[kHD + 1] = l_i[hrow];
        }
    }
}

// ---------------------------------------------------------------------------------------------

// ---------------------------------------------------------------------------------------------
// split reduce (vLLM reduce_segments), + for int4 the un-rotation out = H(rot) * s / d
// ---------------------------------------------------------------------------------------------
struct KvReduceArgs {
    const float* partial; __half* out;
    const int32_t* seq_lens; const int32_t* query_start_loc;
    int num_seqs, num_tokens, num_q_heads, num_splits;
    const float* unrot_signs;  // int4: RHT signs, else null
};

__global__ void kv_reduce_kernel(const KvReduceArgs a) {
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= (int64_t)a.num_tokens * a.num_q_heads) return;
    const int lane = threadIdx.x & 31;
    const int t = (int)(item / a.num_q_heads);
    const int s = seq_of_token(a.query_start_loc, a.num_seqs, t);
    const int L = a.seq_lens[s];
    const int per = ((L + a.num_splits - 1) / a.num_splits + 31) & ~31;
    const int nsp = (L + per - 1) / per;  // splits that held tokens
    const float* base = a.partial + item * a.num_splits * kPartialStride;
    float M = -INFINITY;
    for (int sp = 0; sp < nsp; ++sp) M = fmaxf(M, base[sp * kPartialStride + kHD]);
    float v[4] = {0.f, 0.f, 0.f, 0.f}, lsum = 0.f;
    if (M != -INFINITY) {
        for (int sp = 0; sp < nsp; ++sp) {
            const float* p = base + sp * kPartialStride;
            const float ms = p[kHD];
            if (ms == -INFINITY) continue;
            const float w = exp_f(ms - M);
            lsum += w * p[kHD + 1];
            const float4 x = reinterpret_cast<const float4*>(p)[lane];
            v[0] += w * x.x; v[1] += w * x.y; v[2] += w * x.z; v[3] += w * x.w;
        }
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] *= inv;
    if (a.unrot_signs) {
        // the reference stores the rotated output as fp16 before un-rotating (kv_int4.py:539-563)
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __half2float(__float2half_rn(v[i]));
        had128_warp(v);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = v[i] * a.unrot_signs[4 * lane + i] * (1.f / kHD);
    }
    reinterpret_cast<uint2*>(a.out + item * kHD)[lane] =
        make_uint2(h2_as_u32(__floats2half2_rn(v[0], v[1])), h2_as_u32(__floats2half2_rn(v[2], v[3])));
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
static int kv_num_sms() {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
}

static int kv_splits(int num_seqs, int num_kv_heads, int max_seq_len) {
    const int want = (8 * kv_num_sms() + num_seqs * num_kv_heads - 1) / (num_seqs * num_kv_heads);
    const int by_len = (max_seq_len + 63) / 64;
    return std::max(1, std::min(kMaxSplits, std::min(want, by_len)));
}

template <int KV, int MT>
static cudaError_t launch_attn(dim3 grid, const KvAttnArgs& a, cudaStream_t st) {
    const int smem = MT * AttnSmem<KV>::kWarpBytes;
    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [&] {
        attr_err[dev & 63] = cudaFuncSetAttribute(kv_attn_kernel<KV, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
    kv_attn_kernel<KV, MT><<<grid, 32 * MT, smem, st>>>(a);
    return cudaGetLastError();
}

static bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }
static int ilog2(int v) { int l = 0; while ((1 << l) < v) ++l; return l; }

}  // namespace exl3b

using namespace exl3b;

static int kv_write_common(KvWriteArgs& a, const void* key, const void* value, int dtype, int64_t num_tokens,
                           int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                           int64_t v_stride_tok, int64_t v_stride_head, void* key_cache, void* value_cache,
                           float* k_scale, float* v_scale, const int64_t* slot_mapping, int block_size) {
    if (head_size != kHD || (dtype != 0 && dtype != 1) || block_size <= 0) return EXL3B_DECLINED;
    if (num_tokens < 0 || num_kv_heads <= 0) return EXL3B_BAD_ARG;
    if (num_tokens > 0 && (!key || !value || !key_cache || !value_cache || !k_scale || !v_scale || !slot_mapping))
        return EXL3B_BAD_ARG;
    a.key = key; a.value = value; a.dtype = dtype;
    a.k_stride_tok = k_stride_tok; a.k_stride_head = k_stride_head;
    a.v_stride_tok = v_stride_tok; a.v_stride_head = v_stride_head;
    a.key_cache = key_cache; a.value_cache = value_cache; a.k_scale = k_scale; a.v_scale = v_scale;
    a.slot_mapping = slot_mapping; a.num_tokens = (int)num_tokens; a.num_heads = num_kv_heads;
    a.block_size = block_size;
    return EXL3B_OK;
}

extern "C" int exl3b_kv_int8_write(const void* key, const void* value, int dtype, int64_t num_tokens,
                                   int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                                   int64_t v_stride_tok, int64_t v_stride_head, int8_t* key_cache,
                                   int8_t* value_cache, float* k_scale, float* v_scale, const int64_t* slot_mapping,
                                   int block_size, void* stream) {
    KvWriteArgs a = {};
    int st = kv_write_common(a, key, value, dtype, num_tokens, num_kv_heads, head_size, k_stride_tok, k_stride_head,
                             v_stride_tok, v_stride_head, key_cache, value_cache, k_scale, v_scale, slot_mapping,
                             block_size);
    if (st != EXL3B_OK || num_tokens == 0) return st;
    const int64_t items = num_tokens * num_kv_heads;
    kv_int8_write_kernel<<<(unsigned)((items + 7) / 8), 256, 0, (cudaStream_t)stream>>>(a);
    return cuda_status(cudaGetLastError());
}

extern "C" int exl3b_kv_int4_write(const void* key, const void* value, int dtype, int64_t num_tokens,
                                   int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                                   int64_t v_stride_tok, int64_t v_stride_head, uint8_t* key_cache,
                                   uint8_t* value_cache, float* k_scale, float* v_scale, const int64_t* slot_mapping,
                                   int block_size, const float* rht_signs, const float* bias_k, const float* bias_v,
                                   const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* seq_slots,
                                   int num_seqs, uint16_t* exact_k, uint16_t* exact_v, int32_t* exact_tag,
                                   void* stream) {
    KvWriteArgs a = {};
    int st = kv_write_common(a, key, value, dtype, num_tokens, num_kv_heads, head_size, k_stride_tok, k_stride_head,
                             v_stride_tok, v_stride_head, key_cache, value_cache, k_scale, v_scale, slot_mapping,
                             block_size);
    if (st != EXL3B_OK || num_tokens == 0) return st;
    if (!rht_signs) return EXL3B_BAD_ARG;
    const bool exact = exact_tag != nullptr;
    if (exact && (!exact_k || !exact_v || !query_start_loc || !seq_lens || !seq_slots || num_seqs <= 0))
        return EXL3B_BAD_ARG;
    KvInt4Extra x = {};
    x.signs = rht_signs; x.bias_k = bias_k; x.bias_v = bias_v;
    x.query_start_loc = query_start_loc; x.seq_lens = seq_lens; x.seq_slots = exact ? seq_slots : nullptr;
    x.num_seqs = num_seqs;
    x.exact_k = reinterpret_cast<__half*>(exact_k); x.exact_v = reinterpret_cast<__half*>(exact_v);
    x.exact_tag = exact_tag;
    const int64_t items = num_tokens * num_kv_heads * 2;
    kv_int4_write_kernel<<<(unsigned)((items + 7) / 8), 256, 0, (cudaStream_t)stream>>>(a, x);
    return cuda_status(cudaGetLastError());
}

extern "C" size_t exl3b_kv_attn_workspace_bytes(int num_tokens, int num_q_heads, int num_seqs, int num_kv_heads,
                                                int max_seq_len) {
    if (num_tokens <= 0 || num_q_heads <= 0 || num_seqs <= 0 || num_kv_heads <= 0) return 0;
    const int S = kv_splits(num_seqs, num_kv_heads, std::max(1, max_seq_len));
    const size_t qr = (size_t)num_tokens * num_q_heads * kHD * 2;
    return (qr + 255) / 256 * 256 + (size_t)num_tokens * num_q_heads * S * kPartialStride * 4;
}

static int kv_attn_common(int kv, const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                          int num_kv_heads, int head_size, const void* key_cache, const void* value_cache,
                          const float* k_scale, const float* v_scale, int block_size, const int32_t* block_table,
                          int64_t bt_stride, const int32_t* seq_lens, const int32_t* query_start_loc, int num_seqs,
                          int max_q_len, int max_seq_len, float softmax_scale, const float* rht_signs,
                          const uint16_t* exact_k, const uint16_t* exact_v, const int32_t* exact_tag,
                          const int32_t* seq_slots, void* workspace, size_t ws_bytes, void* stream) {
    if (head_size != kHD || !pow2(block_size)) return EXL3B_DECLINED;
    if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads) return EXL3B_DECLINED;
    if (num_tokens == 0) return EXL3B_OK;
    const int G = num_q_heads / num_kv_heads;
    if (max_q_len <= 0 || max_q_len * G > 32) return EXL3B_DECLINED;
    if (!q || !out || !key_cache || !value_cache || !k_scale || !v_scale || !block_table || !seq_lens ||
        !query_start_loc || num_seqs <= 0 || !workspace)
        return EXL3B_BAD_ARG;
    if (kv == 4 && !rht_signs) return EXL3B_BAD_ARG;
    if (ws_bytes < exl3b_kv_attn_workspace_bytes(num_tokens, num_q_heads, num_seqs, num_kv_heads, max_seq_len))
        return EXL3B_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    const int S = kv_splits(num_seqs, num_kv_heads, std::max(1, max_seq_len));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const size_t qr_bytes = ((size_t)num_tokens * num_q_heads * kHD * 2 + 255) / 256 * 256;
    const __half* qin = reinterpret_cast<const __half*>(q);
    if (kv == 4) {  // rotate q into the workspace: qr = fp16(H (q * s)), unnormalised (kv_int4.py:526)
        __half* qr = reinterpret_cast<__half*>(ws);
        const int64_t rows = (int64_t)num_tokens * num_q_heads;
        kv_rotate_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(qin, qr, rows, rht_signs, nullptr, 1.f);
        qin = qr;
    }
    KvAttnArgs a = {};
    a.q = qin; a.key_cache = key_cache; a.value_cache = value_cache; a.k_scale = k_scale; a.v_scale = v_scale;
    a.block_table = block_table; a.bt_stride = bt_stride; a.seq_lens = seq_lens; a.query_start_loc = query_start_loc;
    a.num_seqs = num_seqs; a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads;
    a.block_size_log2 = ilog2(block_size); a.num_splits = S;
    a.score_scale = kv == 4 ? softmax_scale / kHD : softmax_scale;
    a.partial = reinterpret_cast<float*>(ws + qr_bytes);
    a.exact_k = reinterpret_cast<const __half*>(exact_k); a.exact_v = reinterpret_cast<const __half*>(exact_v);
    a.exact_tag = exact_tag; a.seq_slots = seq_slots;
    const dim3 grid(num_seqs, num_kv_heads, S);
    const bool two = max_q_len * G > 16;
    cudaError_t e;
    if (kv == 8) e = two ? launch_attn<8, 2>(grid, a, st) : launch_attn<8, 1>(grid, a, st);
    else e = two ? launch_attn<4, 2>(grid, a, st) : launch_attn<4, 1>(grid, a, st);
    if (e != cudaSuccess) return cuda_status(e);
    KvReduceArgs r = {};
    r.partial = a.partial; r.out = reinterpret_cast<__half*>(out); r.seq_lens = seq_lens;
    r.query_start_loc = query_start_loc; r.num_seqs = num_seqs; r.num_tokens = num_tokens;
    r.num_q_heads = num_q_heads; r.num_splits = S; r.unrot_signs = kv == 4 ? rht_signs : nullptr;
    const int64_t items = (int64_t)num_tokens * num_q_heads;
    kv_reduce_kernel<<<(unsigned)((items + 7) / 8), 256, 0, st>>>(r);
    return cuda_status(cudaGetLastError());
}

extern "C" int exl3b_kv_int8_attn(const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                                  int num_kv_heads, int head_size, const int8_t* key_cache,
                                  const int8_t* value_cache, const float* k_scale, const float* v_scale,
                                  int block_size, const int32_t* block_table, int64_t bt_stride,
                                  const int32_t* seq_lens, const int32_t* query_start_loc, int num_seqs,
                                  int max_q_len, int max_seq_len, float softmax_scale, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    return kv_attn_common(8, q, out, num_tokens, num_q_heads, num_kv_heads, head_size, key_cache, value_cache,
                          k_scale, v_scale, block_size, block_table, bt_stride, seq_lens, query_start_loc, num_seqs,
                          max_q_len, max_seq_len, softmax_scale, nullptr, nullptr, nullptr, nullptr, nullptr,
                          workspace, workspace_bytes, stream);
}

extern "C" int exl3b_kv_int4_attn(const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                                  int num_kv_heads, int head_size, const uint8_t* key_cache,
                                  const uint8_t* value_cache, const float* k_scale, const float* v_scale,
                                  int block_size, const int32_t* block_table, int64_t bt_stride,
                                  const int32_t* seq_lens, const int32_t* query_start_loc, int num_seqs,
                                  int max_q_len, int max_seq_len, float softmax_scale, const float* rht_signs,
                                  const uint16_t* exact_k, const uint16_t* exact_v, const int32_t* exact_tag,
                                  const int32_t* seq_slots, void* workspace, size_t workspace_bytes, void* stream) {
    return kv_attn_common(4, q, out, num_tokens, num_q_heads, num_kv_heads, head_size, key_cache, value_cache,
                          k_scale, v_scale, block_size, block_table, bt_stride, seq_lens, query_start_loc, num_seqs,
                          max_q_len, max_seq_len, softmax_scale, rht_signs, exact_k, exact_v, exact_tag, seq_slots,
                          workspace, workspace_bytes, stream);
}
