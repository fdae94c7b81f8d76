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
constexpr int kMaxSplits = 256;  // the reference segments at most 64 ways (kv_int4.py:43); B200 fills with more
// one split's partial for one (token, query head): acc[128], m, l, padded to 132 floats so that
// every record starts on a 16-byte boundary (the kernels move it as float4)
constexpr int kPartialStride = kHD + 4;

// Where the (block, slot, head) row of a paged cache and its fp32 scale live.  Dense caches hold rows
// of R bytes at [blocks][block_size][H] and scales at [blocks][block_size][H]; vLLM's per-token-head
// caches keep each row's scale inline after it and interleave the K and V halves of every block, so
// the host passes their strides.
struct KvLayout {
    int64_t blk, slot, head;     // cache strides in bytes
    int64_t sblk, sslot, shead;  // scale strides in floats
    EXL3B_DEV int64_t row(int64_t b, int64_t o, int h) const { return b * blk + o * slot + (int64_t)h * head; }
    EXL3B_DEV int64_t srow(int64_t b, int64_t o, int h) const { return b * sblk + o * sslot + (int64_t)h * shead; }
};

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
    KvLayout lay;
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
    const int64_t row = a.lay.row(blk, off, h), srow = a.lay.srow(blk, off, h);
    float xk[4], xv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        xk[i] = load_in(a.key, t * a.k_stride_tok + h * a.k_stride_head + 4 * lane + i, a.dtype);
        xv[i] = load_in(a.value, t * a.v_stride_tok + h * a.v_stride_head + 4 * lane + i, a.dtype);
    }
    int8_quant_store(xk, reinterpret_cast<int8_t*>(a.key_cache) + row, a.k_scale + srow, lane);
    int8_quant_store(xv, reinterpret_cast<int8_t*>(a.value_cache) + row, a.v_scale + srow, lane);
}

// The same write fused with the neox rotary embedding of the token's q and k (a decode step's qkv
// projection output goes straight to the cache): one warp per (token, head slot); slots [0, nq)
// rotate q head j into q_out, slots [nq, nq + H) rotate k head h, round it to fp16 (the value the
// unfused route stores), quantise it and v.  Lane l owns elements 4l..4l+3, so the rotation
// partner of element i (i +- 64) sits in lane l ^ 16.  Rotation arithmetic as exl3b_rope_neox.
struct KvRopeArgs {
    const __half* qkv; int64_t ld;      // row t: q heads, k heads, v heads of 128
    __half* q_out; int64_t ld_q;
    int nq;
    const int64_t* positions; const float* cos_sin; int64_t max_pos;
};

EXL3B_DEV void rope4(float (&x)[4], const float* cs, int lane) {
    const bool hi = lane >= 16;  // elements 64.. : o = x c + partner s; below: o = x c - partner s
    const int i0 = (4 * lane) & 63;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float y = __shfl_xor_sync(0xFFFFFFFFu, x[e], 16);
        const float c = cs[i0 + e], sn = cs[64 + i0 + e];
        x[e] = hi ? __fmaf_rn(x[e], c, __fmul_rn(y, sn)) : __fmaf_rn(x[e], c, -__fmul_rn(y, sn));
    }
}

__global__ void kv_int8_write_rope_kernel(const KvWriteArgs a, const KvRopeArgs r) {
    // a programmatic dependent launch: the attention after it may be scheduled now; qkv comes from
    // the previous kernel
    griddep_launch();
    griddep_wait();
    const int slots = r.nq + a.num_heads;
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= (int64_t)a.num_tokens * slots) return;
    const int lane = threadIdx.x & 31;
    const int t = (int)(item / slots), j = (int)(item % slots);
    const int64_t p = r.positions[t];
    const bool ok = p >= 0 && p < r.max_pos;
    const float* cs = r.cos_sin + (ok ? p : 0) * 128;
    const __half* row_in = r.qkv + t * r.ld;
    if (j < r.nq) {
        const uint2 w = *reinterpret_cast<const uint2*>(row_in + j * kHD + 4 * lane);
        float x[4] = {__low2float(u32_as_h2(w.x)), __high2float(u32_as_h2(w.x)), __low2float(u32_as_h2(w.y)),
                      __high2float(u32_as_h2(w.y))};
        rope4(x, cs, lane);
        uint2 o = make_uint2(h2_as_u32(__floats2half2_rn(x[0], x[1])), h2_as_u32(__floats2half2_rn(x[2], x[3])));
        if (!ok) o = make_uint2(0u, 0u);
        *reinterpret_cast<uint2*>(r.q_out + t * r.ld_q + j * kHD + 4 * lane) = o;
        return;
    }
    const int h = j - r.nq;
    const int64_t slot = a.slot_mapping[t];
    if (slot < 0) return;
    const int64_t blk = slot / a.block_size, off = slot % a.block_size;
    const int64_t row = a.lay.row(blk, off, h), srow = a.lay.srow(blk, off, h);
    const uint2 wk = *reinterpret_cast<const uint2*>(row_in + (r.nq + h) * kHD + 4 * lane);
    const uint2 wv = *reinterpret_cast<const uint2*>(row_in + (r.nq + a.num_heads + h) * kHD + 4 * lane);
    float xk[4] = {__low2float(u32_as_h2(wk.x)), __high2float(u32_as_h2(wk.x)), __low2float(u32_as_h2(wk.y)),
                   __high2float(u32_as_h2(wk.y))};
    const float xv[4] = {__low2float(u32_as_h2(wv.x)), __high2float(u32_as_h2(wv.x)), __low2float(u32_as_h2(wv.y)),
                         __high2float(u32_as_h2(wv.y))};
    if (ok) {
        rope4(xk, cs, lane);
#pragma unroll
        for (int e = 0; e < 4; ++e) xk[e] = __half2float(__float2half_rn(xk[e]));
    }
    int8_quant_store(xk, reinterpret_cast<int8_t*>(a.key_cache) + row, a.k_scale + srow, lane);
    int8_quant_store(xv, reinterpret_cast<int8_t*>(a.value_cache) + row, a.v_scale + srow, lane);
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

// One warp per eight rows (token, KV head, side), four lanes per row.  Lane j of a row holds the
// 4-element chunks l = j + 4i (i = 0..7) of its 128 elements: the unnormalised Hadamard (H4 inside a
// chunk, then butterflies over chunk distances 1, 2, 4, 8, 16), the row sums and the clip search's
// error sums then run in exactly the order of a warp holding chunk l in lane l (distances 16, 8 and
// 4 fall inside a lane, 2 and 1 between the row's lanes), so the codes and scales are bit for bit
// those of the oracle, while a warp shuffles twice per sum instead of five times and keeps all of
// its lanes on useful work (a warp per row issued ~1500 instructions per row).
constexpr int kW4Rows = 8;  // rows per warp
EXL3B_DEV float sum_chunks(const float (&c)[8]) {  // the xor-16/8/4 levels over this lane's chunks
    const float t0 = __fadd_rn(c[0], c[4]), t1 = __fadd_rn(c[1], c[5]), t2 = __fadd_rn(c[2], c[6]),
                t3 = __fadd_rn(c[3], c[7]);
    return __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
}
EXL3B_DEV float row_sum4(float v) {  // the xor-2/1 levels between the row's four lanes
    v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
    return __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
}
// round_half_away(v) clamped to [0, 15], as a float: for v >= 0 it is floor(v + 0.5), and negative v
// (whose rounding is <= 0) clamps to 0 either way
EXL3B_DEV float code_of(float v) { return fminf(fmaxf(floorf(__fadd_rn(v, 0.5f)), 0.f), 15.f); }

// Two fp32 lanes in one 64-bit register pair (low = first) and the sm_100 packed fp32 arithmetic on
// them (add / mul / fma .rn.f32x2): each lane is rounded exactly as the scalar .rn instruction.
EXL3B_DEV uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
EXL3B_DEV void f2_unpack(uint64_t r, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r)); }
EXL3B_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
EXL3B_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
EXL3B_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__global__ void __launch_bounds__(256) kv_int4_write_kernel(const KvWriteArgs a, const KvInt4Extra x) {
    const int lane = threadIdx.x & 31, j = lane & 3;
    const int64_t item = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kW4Rows + (lane >> 2);
    const int64_t items = (int64_t)a.num_tokens * a.num_heads * 2;
    // rows outside the call or without a slot run along on zeros (every lane takes part in the shuffles)
    bool live = item < items;
    const int side = (int)(item & 1);
    const int t = live ? (int)((item >> 1) / a.num_heads) : 0, h = live ? (int)((item >> 1) % a.num_heads) : 0;
    const int64_t slot = live ? a.slot_mapping[t] : -1;
    live = live && slot >= 0;
    const void* src = side ? a.value : a.key;
    const int64_t base = side ? t * a.v_stride_tok + h * a.v_stride_head : t * a.k_stride_tok + h * a.k_stride_head;
    const bool vec = ((base & 3) == 0) && ((reinterpret_cast<uintptr_t>(src) & 7) == 0);
    float y[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e0 = 16 * i + 4 * j;
        const float4 sg = *reinterpret_cast<const float4*>(x.signs + e0);
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) {
            if (vec) {
                const uint2 w = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(src) + base + e0);
                if (a.dtype == 0) {
                    v[0] = __low2float(u32_as_h2(w.x)); v[1] = __high2float(u32_as_h2(w.x));
                    v[2] = __low2float(u32_as_h2(w.y)); v[3] = __high2float(u32_as_h2(w.y));
                } else {
                    v[0] = __uint_as_float(w.x << 16); v[1] = __uint_as_float(w.x & 0xFFFF0000u);
                    v[2] = __uint_as_float(w.y << 16); v[3] = __uint_as_float(w.y & 0xFFFF0000u);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) v[c] = load_in(src, base + e0 + c, a.dtype);
            }
        }
        y[i][0] = v[0] * sg.x; y[i][1] = v[1] * sg.y; y[i][2] = v[2] * sg.z; y[i][3] = v[3] * sg.w;
        // H4 inside the chunk
        const float s0 = y[i][0] + y[i][1], d0 = y[i][0] - y[i][1];
        const float s1 = y[i][2] + y[i][3], d1 = y[i][2] - y[i][3];
        y[i][0] = s0 + s1; y[i][1] = d0 + d1; y[i][2] = s0 - s1; y[i][3] = d0 - d1;
    }
    // chunk distances 1 and 2: the partner chunk is in lane j ^ 1 / j ^ 2 (lower chunk: own + partner,
    // upper chunk: partner - own)
#pragma unroll
    for (int d = 1; d <= 2; d <<= 1) {
        const bool upper = (j & d) != 0;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float o = __shfl_xor_sync(0xFFFFFFFFu, y[i][c], d);
                y[i][c] = upper ? (o - y[i][c]) : (y[i][c] + o);
            }
    }
    // chunk distances 4, 8, 16: i ^ 1, i ^ 2, i ^ 4 inside the lane
#pragma unroll
    for (int d = 1; d <= 4; d <<= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (!(i & d))
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float lo = y[i][c], hi = y[i | d][c];
                    y[i][c] = lo + hi;
                    y[i | d][c] = lo - hi;
                }
    const float* bias = side ? x.bias_v : x.bias_k;
    if (bias) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 b = *reinterpret_cast<const float4*>(bias + h * kHD + 16 * i + 4 * j);
            y[i][0] = __fadd_rn(y[i][0], b.x); y[i][1] = __fadd_rn(y[i][1], b.y);
            y[i][2] = __fadd_rn(y[i][2], b.z); y[i][3] = __fadd_rn(y[i][3], b.w);
        }
    }
    // ---- 3x3 clip search (kv_int4.py:198-213), the row-wide sums in the order described above ----
    float lo0 = y[0][0], hi0 = y[0][0];
    float cs[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        lo0 = fminf(lo0, fminf(fminf(y[i][0], y[i][1]), fminf(y[i][2], y[i][3])));
        hi0 = fmaxf(hi0, fmaxf(fmaxf(y[i][0], y[i][1]), fmaxf(y[i][2], y[i][3])));
        cs[i] = __fadd_rn(__fadd_rn(__fadd_rn(y[i][0], y[i][1]), y[i][2]), y[i][3]);
    }
#pragma unroll
    for (int d = 2; d >= 1; d >>= 1) {
        lo0 = fminf(lo0, __shfl_xor_sync(0xFFFFFFFFu, lo0, d));
        hi0 = fmaxf(hi0, __shfl_xor_sync(0xFFFFFFFFu, hi0, d));
    }
    const float mu = __fmul_rn(row_sum4(sum_chunks(cs)), 1.f / 128.f);
    // chunks i and i + 1 side by side in one 64-bit register pair for the packed fp32 (f32x2)
    // arithmetic of the search: each half rounds exactly as the scalar instruction would
    uint64_t y2[4][4], ny2[4][4];  // y and -y (the addend of every candidate's error)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            y2[i][c] = f2_pack(y[2 * i][c], y[2 * i + 1][c]);
            ny2[i][c] = f2_pack(-y[2 * i][c], -y[2 * i + 1][c]);
        }
    float best_err = __int_as_float(0x7F800000), best_sc = 0.f, best_zp = 0.f;
#pragma unroll 1
    for (int cand = 0; cand < kClipSteps * kClipSteps; ++cand) {
        const float flo = __fmaf_rn(-kClipStep, (float)(cand / kClipSteps), 1.f);
        const float fhi = __fmaf_rn(-kClipStep, (float)(cand % kClipSteps), 1.f);
        const float lo = __fmaf_rn(__fsub_rn(lo0, mu), flo, mu);
        const float hi = __fmaf_rn(__fsub_rn(hi0, mu), fhi, mu);
        const float sc = fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 15.f), 1e-6f);
        const float zp = code_of(__fdiv_rn(-lo, sc));
        const float inv = __fdiv_rn(1.f, sc);
        const uint64_t inv2 = f2_pack(inv, inv), zp2 = f2_pack(zp, zp), nzp2 = f2_pack(-zp, -zp);
        const uint64_t sc2 = f2_pack(sc, sc), half2 = f2_pack(0.5f, 0.5f);
        // per element, as the scalar code_of / error: e = (code_of(y * inv + zp) - zp) * sc - y, and
        // the chunk's sum of e^2 in element order; code_of's floor and clamp stay scalar
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint64_t q2 = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float u0, u1;
                f2_unpack(f2_add(f2_fma(y2[i][c], inv2, zp2), half2), u0, u1);
                u0 = fminf(fmaxf(floorf(u0), 0.f), 15.f);
                u1 = fminf(fmaxf(floorf(u1), 0.f), 15.f);
                const uint64_t e2 = f2_fma(f2_add(f2_pack(u0, u1), nzp2), sc2, ny2[i][c]);
                q2 = c == 0 ? f2_mul(e2, e2) : f2_fma(e2, e2, q2);
            }
            f2_unpack(q2, cs[2 * i], cs[2 * i + 1]);
        }
        const float err = row_sum4(sum_chunks(cs));
        if (err < best_err) { best_err = err; best_sc = sc; best_zp = zp; }
    }
    if (!live) return;  // no shuffles below
    const float inv = __fdiv_rn(1.f, best_sc);
    const int64_t blk = slot / a.block_size, off = slot % a.block_size;
    uint16_t* cache = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(side ? a.value_cache : a.key_cache) +
                                                  a.lay.row(blk, off, h));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int code[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) code[c] = (int)code_of(__fmaf_rn(y[i][c], inv, best_zp));
        cache[j + 4 * i] = (uint16_t)((code[0] | (code[1] << 4)) | ((code[2] | (code[3] << 4)) << 8));
    }
    if (j == 0) {
        const uint32_t sbits = ((uint32_t)__float_as_uint(best_sc) & 0xFFFFFFF0u) | (uint32_t)best_zp;
        (side ? a.v_scale : a.k_scale)[a.lay.srow(blk, off, h)] = __uint_as_float(sbits);
    }
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
#pragma unroll
            for (int i = 0; i < 8; ++i)
                *reinterpret_cast<uint2*>(ex + 16 * i + 4 * j) =
                    make_uint2(h2_as_u32(__floats2half2_rn(y[i][0], y[i][1])),
                               h2_as_u32(__floats2half2_rn(y[i][2], y[i][3])));
            if (side == 0 && h == 0 && j == 0) x.exact_tag[(int64_t)rs * kExactRows + e] = pos;
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
    int tsplit;                  // > 1: that many warps share the split's keys (one warp holds all rows)
    KvLayout lay;
    int al16;                    // every cache row starts on a 16-byte boundary: 16-byte copies
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

// The d permutation of the QK^T product, per MMA k-chunk c (0..7) and lane q (= lane & 3):
//   int8: k-slots (2q, 2q+1, 2q+8, 2q+9) <- d = 32q + 4c + (0, 1, 2, 3)
//   int4: k-slots (2q, 2q+1, 2q+8, 2q+9) <- d = 32q + 8(c/2) + 2(c%2) + (0, 4, 1, 5)
// so that one lane's K bytes of a token are contiguous (32 bytes int8, 16 bytes int4).
template <>
struct KvTraits<8> {
    EXL3B_DEV static int dmap(int q, int c, int slot) { return 32 * q + 4 * c + slot; }
};
template <>
struct KvTraits<4> {
    EXL3B_DEV static int dmap(int q, int c, int slot) {
        const int add = (slot == 0) ? 0 : (slot == 1) ? 4 : (slot == 2) ? 1 : 5;
        return 32 * q + 8 * (c / 2) + 2 * (c % 2) + add;
    }
};

// Per-warp shared memory: a ring of kRing tiles (32 tokens: K rows, V rows, k scales, v scales)
// filled with cp.async one tile ahead of the math, and a window of the split's block ids.
// Occupancy of the split-KV kernels (one warp per CTA for decode).  int8: a two-tile ring (17.9 KB a
// warp) lets a B200 SM hold 12 CTAs, and the one-n-tile kernel is held to 168 registers so that 12 fit
// (187 unbounded measured 3277 against 4257 GB/s at 32k x 8: 10 resident warps and a second wave).
// int4: a two-tile ring (9.7 KB a warp) and 128 registers make 16 resident warps per SM; against
// three tiles and 12 warps, 32k x 8 went 1639 -> 1948 GB/s and 64k x 8 1901 -> 2136 GB/s.
constexpr int kRing4 = 2;
constexpr int kWarpsPerSm8 = 12, kWarpsPerSm4 = 16;
template <int KV, int NT>
constexpr int attn_min_blocks() { return NT > 1 ? 1 : KV == 4 ? 4 : 3; }
template <int KV>
struct AttnSmem {
    static constexpr int kRowBytes = KV == 8 ? kHD : kHD / 2;
    static constexpr int kRows = 32 * kRowBytes;                  // K (or V) bytes of one tile
    static constexpr int kTile = 2 * kRows + 2 * 32 * 4;          // K, V, k scales, v scales
    static constexpr int kRing = KV == 8 ? 2 : kRing4;
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

// mma.m16n8k16 f16 -> f32 without the volatile qualifier, so that it schedules with the rest
EXL3B_DEV void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// 8x8 b16 transpose across the warp: lane l holds row l/4, columns 2(l%4), 2(l%4)+1, before and after
EXL3B_DEV uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}
EXL3B_DEV float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}
EXL3B_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }

// Attention of one (sequence, KV head, split), transposed: tokens are the MMA's M dimension and
// query rows its N dimension (8 per n-tile), so that a decode step's GQA group of 5 rows fills 5/8
// of an n-tile instead of 5/16 of an m-tile.
//   S^T[token][row] = K[token][:] . Q[row][:]      A = K tile (16 tokens x 16 d), B = Q^T (resident)
//   O^T[d][row]    += V^T[d][:] . P'^T[:][row]     A = V^T (16 d x 16 tokens), B = P'^T
// P' = p * v_scale[token] in fp16 leaves the S^T accumulator as (token g, rows 2q, 2q+1) and
// movmatrix.trans turns each 8x8 block into the B fragment (rows g, tokens 2q, 2q+1).  In PV lane
// g covers d = 16g .. 16g+15: m-tile j's rows g and g+8 are d = 16g + 2j and 16g + 2j + 1, so a lane
// reads 16 contiguous bytes (int8) or 8 (int4) of each of its 4 tokens per 16-token chunk.
// Each warp owns 8 * NT query rows; the CTA's warps share nothing and never wait on one another.
template <int KV, int NT>
__global__ void __launch_bounds__(32 * 4, attn_min_blocks<KV, NT>()) kv_attn_kernel(const KvAttnArgs a) {
    griddep_launch();  // the split combine may be scheduled now; it waits for this grid's partials
    griddep_wait();    // a programmatic dependent launch: q and the cache rows come from earlier kernels
    using Tr = KvTraits<KV>;
    using SM = AttnSmem<KV>;
    constexpr int RB = SM::kRowBytes;
    constexpr int C16 = RB / 16;  // 16-byte chunks per row (8 or 4)
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int seq = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int L = a.seq_lens[seq];
    const int q0 = a.query_start_loc[seq], qlen = a.query_start_loc[seq + 1] - q0;
    if (qlen <= 0 || L <= 0) return;
    const int G = a.num_q_heads / a.num_kv_heads;
    const int rows = qlen * G;
    const int per = ((L + a.num_splits - 1) / a.num_splits + 31) & ~31;  // tokens per split, x32
    const int t_lo = split * per, t_hi = min(L, t_lo + per);
    if (t_lo >= t_hi) return;  // empty split: the reduce kernel skips it
    // row r of the sequence = query (r / G), head kvh*G + r % G; this warp owns rows rbase + 0 .. 8NT-1.
    // With tsplit > 1 every warp owns all rows (rows <= 8 NT) and takes every tsplit-th tile of the
    // split; the warps' results are merged at the end (the only CTA-wide barrier).  Otherwise warps
    // split the rows and run independently.
    const int ts = a.tsplit;
    const int rbase = ts > 1 ? 0 : 8 * NT * warp;
    if (rbase >= rows) return;

    uint8_t* wsm = smem_raw + warp * SM::kWarpBytes;
    const uint32_t wsm_u = smem_u32(wsm);
    int32_t* bt_win = reinterpret_cast<int32_t*>(wsm + SM::kRing * SM::kTile);
    const int32_t* bt = a.block_table + (int64_t)seq * a.bt_stride;
    const int lg = a.block_size_log2, bs_mask = (1 << lg) - 1;
    int win_base = -1;  // first block index held in bt_win

    // ---- Q^T fragments, resident: B[k-slot][n] = Q[row rbase + 8nt + n][dmap], lane (n = g, slots q) ----
    // The K side of the MMAs takes the cache values with a bias (int8: 1152 + k, int4: 1024 + nibble),
    // one instruction cheaper to build than the true values: S^T then carries bias * (sum of the row's
    // q), removed per score (a score sums only 128 products).  The V side takes the true values: its
    // accumulator runs over the whole split, and a bias there would make it carry ~1000 x the signal
    // and lose the signal's low bits to the accumulation rounding as the split grows.
    uint32_t qb[NT][8][2];
    float qsum[NT][2];  // sum of the fp16 q of rows 2q and 2q+1 of each n-tile
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = rbase + 8 * nt + g;
        const __half* qrow = a.q + ((int64_t)(q0 + r / G) * a.num_q_heads + kvh * G + r % G) * kHD;
        float part = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            __half v4[4];
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                v4[s] = r < rows ? qrow[Tr::dmap(q, c, s)] : __float2half(0.f);
                part += __half2float(v4[s]);
            }
            qb[nt][c][0] = h2_as_u32(__halves2half2(v4[0], v4[1]));
            qb[nt][c][1] = h2_as_u32(__halves2half2(v4[2], v4[3]));
        }
        part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
        part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);  // row g's sum in the four lanes of group g
        qsum[nt][0] = __shfl_sync(0xFFFFFFFFu, part, 4 * (2 * q));
        qsum[nt][1] = __shfl_sync(0xFFFFFFFFu, part, 4 * (2 * q + 1));
    }

    // ---- tile loader: all of a 32-token tile's rows and scales, one cp.async group ----
    // Row r of a tile is stored with its 16-byte chunks XOR-swizzled by (r & (C16 - 1)), so that
    // the lanes reading the same chunk index of different rows hit different banks.
    const int ntiles_all = (t_hi - t_lo + 31) >> 5;
    const int tw = ts > 1 ? warp : 0;  // this warp's first tile; its j-th is tw + j * tstep
    const int tstep = ts > 1 ? ts : 1;
    const int ntiles = ntiles_all > tw ? (ntiles_all - tw + tstep - 1) / tstep : 0;
    auto issue_tile = [&](int ti) {
        const int t0 = t_lo + 32 * (tw + ti * tstep);
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
        // Lane l looks up token t0 + l once (block table, row index) and copies its two scales; the
        // 16-byte chunks then go out coalesced (eight lanes per row) with each row index taken from
        // the lane that looked it up.
        const int t = t0 + lane;
        uint32_t my_slot = 0xFFFFFFFFu;  // block * block_size + slot of token t: fits 32 bits for any cache
        if (t < t_hi) {
            my_slot = ((uint32_t)bt_win[(t >> lg) - win_base] << lg) + (uint32_t)(t & bs_mask);
            const int64_t srow = a.lay.srow(my_slot >> lg, my_slot & (uint32_t)bs_mask, kvh);
            cp_async4(tb + 2 * SM::kRows + lane * 4, a.k_scale + srow);
            cp_async4(tb + 2 * SM::kRows + 128 + lane * 4, a.v_scale + srow);
        }
        const int ch = lane % C16;
#pragma unroll
        for (int j = 0; j < C16; ++j) {  // rows lane / C16 + (32 / C16) j, chunk lane % C16
            const int r = lane / C16 + (32 / C16) * j;
            const uint32_t sl = __shfl_sync(0xFFFFFFFFu, my_slot, r);
            if (sl != 0xFFFFFFFFu) {
                const int64_t off = a.lay.row(sl >> lg, sl & (uint32_t)bs_mask, kvh) + ch * 16;
                const uint32_t soff = r * RB + ((ch ^ (r & (C16 - 1))) * 16);
                const uint8_t* ks = reinterpret_cast<const uint8_t*>(a.key_cache) + off;
                const uint8_t* vs = reinterpret_cast<const uint8_t*>(a.value_cache) + off;
                if (a.al16) {
                    cp_async16(tb + soff, ks);
                    cp_async16(tb + SM::kRows + soff, vs);
                } else {  // rows on 4-byte boundaries (scales inline): four 4-byte copies per chunk
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        cp_async4(tb + soff + 4 * w, ks + 4 * w);
                        cp_async4(tb + SM::kRows + soff + 4 * w, vs + 4 * w);
                    }
                }
            }
        }
        cp_async_commit();
    };

    const float sl2 = a.score_scale * 1.4426950408889634f;  // scores in the log2 domain
    // l_i holds this lane's share (its tokens); it is summed over the lane group at the end
    float m_i[NT][2], l_i[NT][2], lim[NT][2];
    float acc[NT][8][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            m_i[nt][h] = -INFINITY;
            l_i[nt][h] = 0.f;
            // causal limit of row 2q + h: key t allowed if t <= L - qlen + query index
            const int r = rbase + 8 * nt + 2 * q + h;
            lim[nt][h] = (r < rows) ? (float)(L - qlen + r / G) : -1.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[nt][j][e] = 0.f;
    }
    // the warp's smallest causal limit over its real rows (rows past `rows` are never written)
    const int lim_lo = L - qlen + rbase / G;
    const int rs = (KV == 4 && a.seq_slots) ? a.seq_slots[seq] : -1;
    const bool has_exact = KV == 4 && rs >= 0 && a.exact_tag != nullptr;
    auto exact_of = [&](int t) -> int {  // exact row of position t, or -1 (int4 only)
        if (KV != 4 || !has_exact) return -1;
        if (!(t < kSinks || t >= L - kTail)) return -1;
        const int e = exact_row(t);
        return a.exact_tag[(int64_t)rs * kExactRows + e] == t ? e : -1;
    };

    // exactly kRing - 1 groups ahead of the loop (empty ones for splits shorter than that), so that
    // wait_group<kRing - 1> in the loop always means "tile ti has landed"
    for (int ti = 0; ti < SM::kRing - 1; ++ti) {
        if (ti < ntiles) issue_tile(ti);
        else cp_async_commit();
    }

    for (int ti = 0; ti < ntiles; ++ti) {
        if (ti + SM::kRing - 1 < ntiles) issue_tile(ti + SM::kRing - 1);
        else cp_async_commit();  // keep the group count in step
        cp_async_wait<SM::kRing - 1>();
        __syncwarp();
        const int t0 = t_lo + 32 * (tw + ti * tstep);
        const uint8_t* tile = wsm + (ti % SM::kRing) * SM::kTile;
        const float* ksc_s = reinterpret_cast<const float*>(tile + 2 * SM::kRows);
        const float* vsc_s = ksc_s + 32;
        auto chunk_at = [&](int side, int r, int ch) -> uint4 {
            return *reinterpret_cast<const uint4*>(tile + side * SM::kRows + r * RB + ((ch ^ (r & (C16 - 1))) * 16));
        };
        // this tile holds exact rows only if it meets the first kSinks or the last kTail positions
        const bool ex_tile = has_exact && (t0 < kSinks || t0 + 31 >= L - kTail);

        // K of tiles without exact rows runs on biased values (see qsum); the others on true values
        const bool biased = !ex_tile;
        // K fragments of token r of the tile: k-slot pairs (2q, 2q+1) -> kf[c][0], (2q+8, 2q+9) -> kf[c][1];
        // returns the token's k scale, and its bias in kb
        auto k_frag = [&](int r, uint32_t (&kf)[8][2], float& kb) -> float {
            const int t = t0 + r;
            kb = 0.f;
            if (t >= t_hi) {
#pragma unroll
                for (int c = 0; c < 8; ++c) kf[c][0] = kf[c][1] = 0u;
                return 0.f;
            }
            if (KV == 4 && ex_tile) {
                const int e = exact_of(t);
                if (e >= 0) {
                    const __half* ex = a.exact_k + (((int64_t)rs * kExactRows + e) * a.num_kv_heads + kvh) * kHD;
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        kf[c][0] = h2_as_u32(__halves2half2(ex[Tr::dmap(q, c, 0)], ex[Tr::dmap(q, c, 1)]));
                        kf[c][1] = h2_as_u32(__halves2half2(ex[Tr::dmap(q, c, 2)], ex[Tr::dmap(q, c, 3)]));
                    }
                    return 1.f;
                }
            }
            if constexpr (KV == 8) {
                const uint4 w0 = chunk_at(0, r, 2 * q), w1 = chunk_at(0, r, 2 * q + 1);
                const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int c = 0; c < 8; ++c) {  // 1152 + k, exact in fp16
                    const uint32_t u = w[c] ^ 0x80808080u;
                    kf[c][0] = prmt(u, 0x64646464u, 0x5140u);
                    kf[c][1] = prmt(u, 0x64646464u, 0x7362u);
                }
                kb = 1152.f;
                return ksc_s[r];
            } else {
                const uint4 w4 = chunk_at(0, r, q);
                const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
                const uint32_t sb = __float_as_uint(ksc_s[r]);
                if (biased) {
#pragma unroll
                    for (int c = 0; c < 8; ++c) {  // 1024 + nibble
                        kf[c][0] = ((w[c / 2] >> (4 * (2 * (c % 2)))) & 0x000F000Fu) | 0x64006400u;
                        kf[c][1] = ((w[c / 2] >> (4 * (2 * (c % 2) + 1))) & 0x000F000Fu) | 0x64006400u;
                    }
                    kb = 1024.f + (float)(sb & 0xFu);
                } else {
                    const uint32_t zp = 0x6400u | (sb & 0xFu);
                    const uint32_t zp2 = zp | (zp << 16);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        kf[c][0] = nib_pair(w[c / 2], 2 * (c % 2), zp2);
                        kf[c][1] = nib_pair(w[c / 2], 2 * (c % 2) + 1, zp2);
                    }
                }
                return __uint_as_float(sb & 0xFFFFFFF0u);
            }
        };

        // ---------------- S^T = K Q^T: two m-tiles of 16 tokens ----------------
        // s[nt][mt][e]: token 16mt + g + 8(e >> 1), row 2q + (e & 1) of n-tile nt
        float s[NT][2][4];
        float ksc[2][2], kbias[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            uint32_t kA[8][2], kB[8][2];
            ksc[mt][0] = k_frag(16 * mt + g, kA, kbias[mt][0]);
            ksc[mt][1] = k_frag(16 * mt + g + 8, kB, kbias[mt][1]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c = 0; c < 8; ++c) mma_f16(d4, kA[c][0], kB[c][0], kA[c][1], kB[c][1], qb[nt][c][0], qb[nt][c][1]);
#pragma unroll
                for (int e = 0; e < 4; ++e) s[nt][mt][e] = d4[e];
            }
        }
        // scale (log2 domain) and mask; a tile needs the mask only at the split's end or the causal edge
        const bool masked = !(t0 + 32 <= t_hi && t0 + 31 <= lim_lo);
        float mx[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            mx[nt][0] = mx[nt][1] = -INFINITY;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = fmaf(-kbias[mt][e >> 1], qsum[nt][e & 1], s[nt][mt][e]) * (sl2 * ksc[mt][e >> 1]);
                    if (masked) {
                        const int t = t0 + 16 * mt + g + 8 * (e >> 1);
                        v = (t < t_hi && (float)t <= lim[nt][e & 1]) ? v : -INFINITY;
                    }
                    s[nt][mt][e] = v;
                    mx[nt][e & 1] = fmaxf(mx[nt][e & 1], v);
                }
        }
        float corr[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v = mx[nt][h];
                v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
                v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, 8));
                v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, 16));
                const float mnew = fmaxf(m_i[nt][h], v);
                corr[nt][h] = (mnew == -INFINITY) ? 1.f : ex2(m_i[nt][h] - mnew);
                m_i[nt][h] = mnew;
            }
        float rsum[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            rsum[nt][0] = rsum[nt][1] = 0.f;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float mm = m_i[nt][e & 1];
                    const float p = (mm == -INFINITY) ? 0.f : ex2(s[nt][mt][e] - mm);
                    s[nt][mt][e] = p;
                    rsum[nt][e & 1] += p;
                }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                l_i[nt][h] = l_i[nt][h] * corr[nt][h] + rsum[nt][h];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    acc[nt][j][h] *= corr[nt][h];
                    acc[nt][j][2 + h] *= corr[nt][h];
                }
            }

        // ---------------- O^T += V^T P'^T, two k-chunks of 16 tokens ----------------
#pragma unroll
        for (int kc = 0; kc < 2; ++kc) {
            // P'^T B fragments: (row g, tokens 16kc + 2q, +1) and (+8)
            float vsA = 0.f, vsB = 0.f;
            {
                const int rA = 16 * kc + g, rB = rA + 8;
                if (t0 + rA < t_hi) vsA = vsc_s[rA];
                if (t0 + rB < t_hi) vsB = vsc_s[rB];
                if constexpr (KV == 4) {
                    vsA = __uint_as_float(__float_as_uint(vsA) & 0xFFFFFFF0u);
                    vsB = __uint_as_float(__float_as_uint(vsB) & 0xFFFFFFF0u);
                    if (ex_tile) {
                        if (t0 + rA < t_hi && exact_of(t0 + rA) >= 0) vsA = 1.f;
                        if (t0 + rB < t_hi && exact_of(t0 + rB) >= 0) vsB = 1.f;
                    }
                }
            }
            uint32_t pb[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const __half2 lo = __floats2half2_rn(s[nt][kc][0] * vsA, s[nt][kc][1] * vsA);
                const __half2 hi = __floats2half2_rn(s[nt][kc][2] * vsB, s[nt][kc][3] * vsB);
                pb[nt][0] = movm_t(h2_as_u32(lo));
                pb[nt][1] = movm_t(h2_as_u32(hi));
            }
            // V^T A fragments: tokens T0..T3 = 16kc + (2q, 2q+1, 2q+8, 2q+9); m-tile j rows g / g+8 are
            // d = 16g + 2j / 16g + 2j + 1.  va[j][0..3] = (a0, a1, a2, a3)
            uint32_t va[8][4];
            const int rT[4] = {16 * kc + 2 * q, 16 * kc + 2 * q + 1, 16 * kc + 2 * q + 8, 16 * kc + 2 * q + 9};
            bool slow = false;
            if constexpr (KV == 4) slow = ex_tile;
            if (!slow) {
                if constexpr (KV == 8) {
                    uint32_t w[4][4];
#pragma unroll
                    for (int T = 0; T < 4; ++T) {
                        uint4 v4 = make_uint4(0u, 0u, 0u, 0u);
                        if (t0 + rT[T] < t_hi) v4 = chunk_at(1, rT[T], g);
                        w[T][0] = v4.x ^ 0x80808080u; w[T][1] = v4.y ^ 0x80808080u;
                        w[T][2] = v4.z ^ 0x80808080u; w[T][3] = v4.w ^ 0x80808080u;
                    }
                    const __half2 bias = u32_as_h2(0x64806480u);  // 1152
#pragma unroll
                    for (int j = 0; j < 8; ++j) {  // (1152 + v) - 1152 = v, exact in fp16
                        const uint32_t sel = (j & 1) ? 0x7362u : 0x5140u;
#pragma unroll
                        for (int pr = 0; pr < 2; ++pr) {  // token pairs (T0, T1) and (T2, T3)
                            const uint32_t x = prmt(w[2 * pr][j >> 1], w[2 * pr + 1][j >> 1], sel);
                            va[j][2 * pr] = h2_as_u32(__hsub2(u32_as_h2(prmt(x, 0x64646464u, 0x5140u)), bias));
                            va[j][2 * pr + 1] = h2_as_u32(__hsub2(u32_as_h2(prmt(x, 0x64646464u, 0x7362u)), bias));
                        }
                    }
                } else {
                    uint32_t w[4][2], zp[4];
#pragma unroll
                    for (int T = 0; T < 4; ++T) {
                        uint4 v4 = make_uint4(0u, 0u, 0u, 0u);
                        if (t0 + rT[T] < t_hi) v4 = chunk_at(1, rT[T], g >> 1);
                        w[T][0] = (g & 1) ? v4.z : v4.x;
                        w[T][1] = (g & 1) ? v4.w : v4.y;
                        zp[T] = 0x6400u | (__float_as_uint(vsc_s[rT[T]]) & 0xFu);  // 1024 + zero point
                    }
                    // (1024 + nibble) - (1024 + zp) = nibble - zp, exact in fp16; a register holds
                    // tokens (T0, T1) or (T2, T3)
                    const __half2 zq[2] = {u32_as_h2(zp[0] | (zp[1] << 16)), u32_as_h2(zp[2] | (zp[3] << 16))};
#pragma unroll
                    for (int i = 0; i < 2; ++i)
#pragma unroll
                        for (int kk = 0; kk < 4; kk += 2) {  // bytes (kk, kk+1) of word i -> m-tiles 4i+kk, 4i+kk+1
                            const uint32_t sel = kk ? 0x7362u : 0x5140u;
#pragma unroll
                            for (int pr = 0; pr < 2; ++pr) {
                                const uint32_t x = prmt(w[2 * pr][i], w[2 * pr + 1][i], sel);
                                const uint32_t lo = x & 0x0F0F0F0Fu, hi = (x >> 4) & 0x0F0F0F0Fu;
                                auto nz = [&](uint32_t u) { return h2_as_u32(__hsub2(u32_as_h2(u), zq[pr])); };
                                va[4 * i + kk][2 * pr] = nz(prmt(lo, 0x64646464u, 0x5140u));
                                va[4 * i + kk][2 * pr + 1] = nz(prmt(hi, 0x64646464u, 0x5140u));
                                va[4 * i + kk + 1][2 * pr] = nz(prmt(lo, 0x64646464u, 0x7362u));
                                va[4 * i + kk + 1][2 * pr + 1] = nz(prmt(hi, 0x64646464u, 0x7362u));
                            }
                        }
                }
            } else {
                // int4 tile with exact rows: each token's 16 values (d = 16g .. 16g+15) as 8 half2
                // (d, d+1), then paired across tokens
                uint32_t nat[4][8];
#pragma unroll
                for (int T = 0; T < 4; ++T) {
                    const int t = t0 + rT[T];
#pragma unroll
                    for (int p = 0; p < 8; ++p) nat[T][p] = 0u;
                    if (t >= t_hi) continue;
                    const int e = exact_of(t);
                    if (e >= 0) {
                        const uint4* ep = reinterpret_cast<const uint4*>(
                            a.exact_v + (((int64_t)rs * kExactRows + e) * a.num_kv_heads + kvh) * kHD + 16 * g);
                        const uint4 h0 = ep[0], h1 = ep[1];
                        nat[T][0] = h0.x; nat[T][1] = h0.y; nat[T][2] = h0.z; nat[T][3] = h0.w;
                        nat[T][4] = h1.x; nat[T][5] = h1.y; nat[T][6] = h1.z; nat[T][7] = h1.w;
                    } else {
                        const uint4 v4 = chunk_at(1, rT[T], g >> 1);
                        const uint32_t ww[2] = {(g & 1) ? v4.z : v4.x, (g & 1) ? v4.w : v4.y};
                        const uint32_t zp = 0x6400u | (__float_as_uint(vsc_s[rT[T]]) & 0xFu);
                        const __half2 z = u32_as_h2(zp | (zp << 16));
#pragma unroll
                        for (int p = 0; p < 8; ++p) {  // byte p: (d = 16g + 2p low nibble, 2p + 1 high)
                            const uint32_t b = (ww[p >> 2] >> (8 * (p & 3))) & 0xFFu;
                            const uint32_t v = (b & 0xFu) | ((b >> 4) << 16) | 0x64006400u;
                            nat[T][p] = h2_as_u32(__hsub2(u32_as_h2(v), z));
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int pr = 0; pr < 2; ++pr) {
                        va[j][2 * pr] = prmt(nat[2 * pr][j], nat[2 * pr + 1][j], 0x5410u);      // d = 16g + 2j
                        va[j][2 * pr + 1] = prmt(nat[2 * pr][j], nat[2 * pr + 1][j], 0x7632u);  // d + 1
                    }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    mma_f16(acc[nt][j], va[j][0], va[j][1], va[j][2], va[j][3], pb[nt][0], pb[nt][1]);
        }
        __syncwarp();  // the ring slot of this tile is refilled next iteration
    }
    cp_async_wait<0>();

    // lane shares of l -> row totals (the lanes of a row differ in g)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float l = l_i[nt][h];
#pragma unroll
            for (int d = 4; d <= 16; d <<= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, d);
            l_i[nt][h] = l;
        }

    if (NT == 1 && ts > 1) {  // the host shares a split among warps only when one n-tile holds all rows
        // merge the warps' (m, l, acc) of the same rows: each warp parks its values in its own ring
        // area (field-major, conflict-free), then warp 0 combines them with weights 2^(m_w - M)
        constexpr int kF = NT * 36;  // acc 32 + m 2 + l 2 per n-tile
        static_assert(NT > 1 || kF * 32 * 4 <= AttnSmem<KV>::kWarpBytes, "merge area");
        float* park = reinterpret_cast<float*>(wsm);
        __syncwarp();
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) park[(nt * 36 + 4 * j + e) * 32 + lane] = acc[nt][j][e];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                park[(nt * 36 + 32 + h) * 32 + lane] = m_i[nt][h];
                park[(nt * 36 + 34 + h) * 32 + lane] = l_i[nt][h];
            }
        }
        __syncthreads();
        if (warp != 0) return;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float M = -INFINITY;
                for (int w = 0; w < ts; ++w) {
                    const float* pw = reinterpret_cast<const float*>(smem_raw + w * SM::kWarpBytes);
                    M = fmaxf(M, pw[(nt * 36 + 32 + h) * 32 + lane]);
                }
                float l = 0.f, A[8][2];
#pragma unroll
                for (int j = 0; j < 8; ++j) A[j][0] = A[j][1] = 0.f;
                for (int w = 0; w < ts; ++w) {  // fixed warp order: deterministic
                    const float* pw = reinterpret_cast<const float*>(smem_raw + w * SM::kWarpBytes);
                    const float mw = pw[(nt * 36 + 32 + h) * 32 + lane];
                    const float f = (mw == -INFINITY) ? 0.f : ex2(mw - M);
                    l = fmaf(f, pw[(nt * 36 + 34 + h) * 32 + lane], l);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        A[j][0] = fmaf(f, pw[(nt * 36 + 4 * j + h) * 32 + lane], A[j][0]);
                        A[j][1] = fmaf(f, pw[(nt * 36 + 4 * j + 2 + h) * 32 + lane], A[j][1]);
                    }
                }
                m_i[nt][h] = M;
                l_i[nt][h] = l;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    acc[nt][j][h] = A[j][0];
                    acc[nt][j][2 + h] = A[j][1];
                }
            }
    }

    // ---- partial of this split: acc (d order restored), m, l ----
    // acc[nt][j][h] is (d = 16g + 2j, row 2q + h), acc[nt][j][2 + h] is (d = 16g + 2j + 1, row 2q + h)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = rbase + 8 * nt + 2 * q + h;
            if (r >= rows) continue;
            const int64_t tok = q0 + r / G;
            const int hq = kvh * G + r % G;
            float* dst = a.partial + ((tok * a.num_q_heads + hq) * a.num_splits + split) * kPartialStride;
            float4* d4 = reinterpret_cast<float4*>(dst + 16 * g);
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
                d4[k4] = make_float4(acc[nt][2 * k4][h], acc[nt][2 * k4][2 + h], acc[nt][2 * k4 + 1][h],
                                     acc[nt][2 * k4 + 1][2 + h]);
            if (g == 0) {
                // m is kept in the log2 domain; the reduce works in natural units
                dst[kHD] = m_i[nt][h] * 0.6931471805599453f;
                dst[kHD + 1] = l_i[nt][h];
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
    const float* out_bias;     // int4, optional: value mean [kv heads][128] added to the un-rotated output
    int group;                 // query heads per KV head
};

// One CTA per (query token, q head) of W = ceil(splits / 8) warps (at most 32).  The split maxima
// and row sums are read by one thread per split and reduced over the CTA; warp j then accumulates
// splits j, j + W, ... of the weighted outputs (at most 8 each, all loads in flight together) and
// warp 0 sums the W partial vectors in warp order (a fixed order: deterministic).  A programmatic
// dependent launch: it is scheduled while the attention runs and waits for its partials.
constexpr int kReduceWarps = 32;  // most warps a CTA takes
static_assert(kMaxSplits <= 8 * kReduceWarps, "at most 8 splits per warp");
static int reduce_warps(int splits) { return std::min(kReduceWarps, std::max(1, (splits + 7) / 8)); }

__global__ void __launch_bounds__(32 * kReduceWarps) kv_reduce_kernel(const KvReduceArgs a) {
    griddep_launch();  // the next kernel (an EXL3 linear) may start streaming its weights
    griddep_wait();    // the attention's partials
    const int64_t item = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int t = (int)(item / a.num_q_heads);
    const int s = seq_of_token(a.query_start_loc, a.num_seqs, t);
    const int L = a.seq_lens[s];
    const int per = ((L + a.num_splits - 1) / a.num_splits + 31) & ~31;
    const int nsp = (L + per - 1) / per;  // splits that held tokens
    const float* base = a.partial + item * a.num_splits * kPartialStride;
    __shared__ float w_s[kMaxSplits];
    __shared__ float red_m[kReduceWarps], red_l[kReduceWarps];
    __shared__ float4 acc_s[kReduceWarps][32];
    const int sp = threadIdx.x;
    float ms = -INFINITY, ls = 0.f;
    if (sp < nsp) {
        ms = base[sp * kPartialStride + kHD];
        ls = base[sp * kPartialStride + kHD + 1];
    }
    float M = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    if (lane == 0) red_m[warp] = M;
    __syncthreads();
    M = red_m[0];
    for (int i = 1; i < nw; ++i) M = fmaxf(M, red_m[i]);
    const float w = (ms == -INFINITY) ? 0.f : exp_f(ms - M);  // M is finite when any split is
    float l = w * ls;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    if (lane == 0) red_l[warp] = l;
    if (sp < kMaxSplits) w_s[sp] = w;
    __syncthreads();
    float lsum = 0.f;
    for (int i = 0; i < nw; ++i) lsum += red_l[i];
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 xs[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int j = warp + i * nw;
        xs[i] = (j < nsp && w_s[j] != 0.f) ? reinterpret_cast<const float4*>(base + j * kPartialStride)[lane]
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int j = warp + i * nw;
        const float wj = j < nsp ? w_s[j] : 0.f;
        v.x += wj * xs[i].x; v.y += wj * xs[i].y; v.z += wj * xs[i].z; v.w += wj * xs[i].w;
    }
    acc_s[warp][lane] = v;
    __syncthreads();
    if (warp != 0) return;
    float r[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < nw; ++i) {
        const float4 x = acc_s[i][lane];
        r[0] += x.x; r[1] += x.y; r[2] += x.z; r[3] += x.w;
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] *= inv;
    if (a.unrot_signs) {
        // the reference stores the rotated output as fp16 before un-rotating (kv_int4.py:539-563)
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = __half2float(__float2half_rn(r[i]));
        had128_warp(r);
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = r[i] * a.unrot_signs[4 * lane + i] * (1.f / kHD);
        if (a.out_bias) {  // the centering's value mean, added before the one fp16 rounding (kv_int4.py:563)
            const float* b = a.out_bias + (int64_t)((int)(item % a.num_q_heads) / a.group) * kHD + 4 * lane;
#pragma unroll
            for (int i = 0; i < 4; ++i) r[i] = __fadd_rn(r[i], b[i]);
        }
    }
    reinterpret_cast<uint2*>(a.out + item * kHD)[lane] =
        make_uint2(h2_as_u32(__floats2half2_rn(r[0], r[1])), h2_as_u32(__floats2half2_rn(r[2], r[3])));
}

// ---------------------------------------------------------------------------------------------
// prefill: gather + dequantise the blocks a batch uses into an fp16 buffer (reference
// vllm_plugin/exl3rocm/kv_dequant.py:42-152, kv_int4.py:566-621)
// ---------------------------------------------------------------------------------------------
struct KvGatherArgs {
    const uint8_t* cache;        // [blocks][bs][H][row bytes]
    const float* scale;          // [blocks][bs][H]
    const int32_t* block_ids;    // [n]: nb blocks per sequence, sequence s at s*nb .. s*nb+nb-1
    int64_t n;
    int bs, H, nb;
    __half* out;                 // [n][bs][H][128]
    float mul;                   // int4: 1/sqrt(128), the orthonormal rotated domain; int8: 1
    KvLayout lay;
    // int4 exact rows (optional): position p of sequence s is exact when its tag matches
    const __half* exact; const int32_t* exact_tag; const int32_t* seq_slots; const int32_t* seq_lens;
};

// One warp per output row (block entry j, slot, head); lane l writes elements 4l..4l+3.
template <int KV>
__global__ void kv_gather_kernel(const KvGatherArgs a) {
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= a.n * a.bs * a.H) return;
    const int lane = threadIdx.x & 31;
    const int64_t j = item / ((int64_t)a.bs * a.H);
    const int rem = (int)(item - j * a.bs * a.H);
    const int slot = rem / a.H, h = rem % a.H;
    const int64_t b = a.block_ids[j];
    const int64_t row = a.lay.row(b, slot, h), srow = a.lay.srow(b, slot, h);
    float v[4];
    bool done = false;
    if (KV == 4 && a.exact_tag) {
        const int sq = (int)(j / a.nb);
        const int pos = (int)(j % a.nb) * a.bs + slot;
        const int L = a.seq_lens[sq], rs = a.seq_slots[sq];
        if (rs >= 0 && pos < L && (pos < kSinks || pos >= L - kTail)) {
            const int e = exact_row(pos);
            if (a.exact_tag[(int64_t)rs * kExactRows + e] == pos) {
                const uint2 w = *reinterpret_cast<const uint2*>(a.exact + (((int64_t)rs * kExactRows + e) * a.H + h) * kHD + 4 * lane);
                const __half2 e01 = u32_as_h2(w.x), e23 = u32_as_h2(w.y);
                v[0] = __low2float(e01) * a.mul; v[1] = __high2float(e01) * a.mul;
                v[2] = __low2float(e23) * a.mul; v[3] = __high2float(e23) * a.mul;
                done = true;
            }
        }
    }
    if (!done) {
        if constexpr (KV == 8) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(a.cache + row + 4 * lane);
            const float sc = a.scale[srow];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = (float)(int8_t)((w >> (8 * i)) & 0xFFu) * sc;
        } else {
            const uint16_t w = *reinterpret_cast<const uint16_t*>(a.cache + row + 2 * lane);
            const uint32_t bits = __float_as_uint(a.scale[srow]);
            const float zp = (float)(bits & 0xFu);
            const float sc = __uint_as_float(bits & 0xFFFFFFF0u) * a.mul;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = ((float)((w >> (4 * i)) & 0xFu) - zp) * sc;
        }
    }
    *reinterpret_cast<uint2*>(a.out + item * kHD + 4 * lane) =
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

// Splits of the key range per (sequence, KV head).  Twelve single-warp CTAs per SM fit (registers
// and shared memory): fill them in one wave (rounded down: a few CTAs more than the slots would
// run as a second, almost empty wave).  A split must stream enough keys to pay for its start-up:
// 128 for up to 8 query rows per KV head (decode), 256 above (speculative verify).  rows = 1
// gives the most splits any call of the shape can take (the workspace bound).
// Splits per (sequence, KV head): enough one-warp CTAs to fill the SMs in one wave (the resident
// warps above), each split at least min_keys long per warp.  int4 decode splits keep >= 160 keys: at
// 4k x 8, 32 splits of 128 keys measured 553 GB/s against 683 for 27 of 152 (the per-split set-up and
// partial dominate such short splits).
static int kv_splits(int kv, int num_seqs, int num_kv_heads, int max_seq_len, int rows, int ts = 1) {
    const int want = ((kv == 4 ? kWarpsPerSm4 : kWarpsPerSm8) * kv_num_sms()) / (num_seqs * num_kv_heads * ts);
    const int min_keys = (rows <= 8 ? (kv == 4 ? 160 : 128) : 256) * ts;  // per warp: ts warps share a split
    const int by_len = (max_seq_len + min_keys - 1) / min_keys;
    return std::max(1, std::min(kMaxSplits, std::min(want, by_len)));
}

constexpr int kDecodeTsplit = 4;  // warps sharing a split's keys when one warp holds all query rows
constexpr int kMaxAttnWarps = 4;  // the widest launch (the kernel's launch bound is 32 * 4)
static_assert(kDecodeTsplit <= kMaxAttnWarps, "launch bound");

template <int KV, int NT>
static cudaError_t launch_attn(dim3 grid, int warps, const KvAttnArgs& a, cudaStream_t st) {
    const int smem = kMaxAttnWarps * AttnSmem<KV>::kWarpBytes;  // sized for the largest launch
    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [&] {
        attr_err[dev & 63] = cudaFuncSetAttribute(kv_attn_kernel<KV, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (attr_err[dev & 63] == cudaSuccess)  // all of the unified L1 as shared memory: most resident CTAs
            attr_err[dev & 63] =
                cudaFuncSetAttribute(kv_attn_kernel<KV, NT>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    });
    if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(32 * warps);
    cfg.dynamicSmemBytes = warps * AttnSmem<KV>::kWarpBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kv_attn_kernel<KV, NT>, a);
}

static bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }
static int ilog2(int v) { int l = 0; while ((1 << l) < v) ++l; return l; }

}  // namespace exl3b

using namespace exl3b;

// The device layout of a cache with rows of row_bytes bytes: the caller's strides, or dense.  Rows
// must sit on 4-byte boundaries; al16 reports whether every row also starts on a 16-byte one.
static int kv_layout(const exl3b_kv_layout* l, int block_size, int heads, int row_bytes, const void* kc,
                     const void* vc, KvLayout& out, int& al16) {
    if (!l) {
        out.head = row_bytes; out.slot = (int64_t)heads * row_bytes; out.blk = (int64_t)block_size * out.slot;
        out.shead = 1; out.sslot = heads; out.sblk = (int64_t)block_size * heads;
    } else {
        out.blk = l->cache_block; out.slot = l->cache_slot; out.head = l->cache_head;
        out.sblk = l->scale_block; out.sslot = l->scale_slot; out.shead = l->scale_head;
        if (out.blk <= 0 || out.slot <= 0 || out.head < row_bytes || out.sblk <= 0 || out.sslot <= 0 ||
            out.shead <= 0)
            return EXL3B_BAD_ARG;
        if (out.blk % 4 || out.slot % 4 || out.head % 4) return EXL3B_BAD_ARG;
    }
    if ((kc && !aligned(kc, 4)) || (vc && !aligned(vc, 4))) return EXL3B_BAD_ARG;
    al16 = out.blk % 16 == 0 && out.slot % 16 == 0 && out.head % 16 == 0 && (!kc || aligned(kc, 16)) &&
           (!vc || aligned(vc, 16));
    return EXL3B_OK;
}

static int kv_write_common(KvWriteArgs& a, const void* key, const void* value, int dtype, int64_t num_tokens,
                           int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                           int64_t v_stride_tok, int64_t v_stride_head, void* key_cache, void* value_cache,
                           float* k_scale, float* v_scale, const int64_t* slot_mapping, int block_size,
                           const exl3b_kv_layout* layout, int row_bytes) {
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
    int al16 = 0;
    return kv_layout(layout, block_size, num_kv_heads, row_bytes, key_cache, value_cache, a.lay, al16);
}

extern "C" int exl3b_kv_int8_write(const void* key, const void* value, int dtype, int64_t num_tokens,
                                   int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                                   int64_t v_stride_tok, int64_t v_stride_head, int8_t* key_cache,
                                   int8_t* value_cache, float* k_scale, float* v_scale, const int64_t* slot_mapping,
                                   int block_size, const exl3b_kv_layout* layout, void* stream) {
    KvWriteArgs a = {};
    int st = kv_write_common(a, key, value, dtype, num_tokens, num_kv_heads, head_size, k_stride_tok, k_stride_head,
                             v_stride_tok, v_stride_head, key_cache, value_cache, k_scale, v_scale, slot_mapping,
                             block_size, layout, kHD);
    if (st != EXL3B_OK || num_tokens == 0) return st;
    const int64_t items = num_tokens * num_kv_heads;
    kv_int8_write_kernel<<<(unsigned)((items + 7) / 8), 256, 0, (cudaStream_t)stream>>>(a);
    return cuda_status(cudaGetLastError());
}

extern "C" int exl3b_kv_int8_write_rope(const uint16_t* qkv, int64_t ld, uint16_t* q_out, int64_t ld_q,
                                        int64_t num_tokens, int num_q_heads, int num_kv_heads,
                                        const int64_t* positions, const float* cos_sin, int64_t max_position,
                                        int8_t* key_cache, int8_t* value_cache, float* k_scale, float* v_scale,
                                        const int64_t* slot_mapping, int block_size, const exl3b_kv_layout* layout,
                                        void* stream) {
    if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads <= 0 || max_position < 1) return EXL3B_BAD_ARG;
    if (num_tokens == 0) return EXL3B_OK;
    if (!qkv || !positions || !cos_sin || !key_cache || !value_cache || !k_scale || !v_scale || !slot_mapping ||
        (num_q_heads && !q_out))
        return EXL3B_BAD_ARG;
    if (ld < (int64_t)(num_q_heads + 2 * num_kv_heads) * kHD || ld % 4 || (num_q_heads && (ld_q < num_q_heads * kHD || ld_q % 4)))
        return EXL3B_BAD_ARG;
    if (!aligned(qkv, 8) || (q_out && !aligned(q_out, 8)) || !aligned(cos_sin, 4) || !aligned(key_cache, 4) ||
        !aligned(value_cache, 4))
        return EXL3B_BAD_ARG;
    if (block_size <= 0) return EXL3B_BAD_ARG;
    KvWriteArgs a = {};
    a.key_cache = key_cache; a.value_cache = value_cache; a.k_scale = k_scale; a.v_scale = v_scale;
    a.slot_mapping = slot_mapping; a.num_tokens = (int)num_tokens; a.num_heads = num_kv_heads;
    a.block_size = block_size;
    int al16 = 0;
    const int lst = kv_layout(layout, block_size, num_kv_heads, kHD, key_cache, value_cache, a.lay, al16);
    if (lst != EXL3B_OK) return lst;
    KvRopeArgs r = {};
    r.qkv = reinterpret_cast<const __half*>(qkv); r.ld = ld;
    r.q_out = reinterpret_cast<__half*>(q_out); r.ld_q = ld_q; r.nq = num_q_heads;
    r.positions = positions; r.cos_sin = cos_sin; r.max_pos = max_position;
    const int64_t items = num_tokens * (num_q_heads + num_kv_heads);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((items + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kv_int8_write_rope_kernel, a, r));
}

extern "C" int exl3b_kv_int4_write(const void* key, const void* value, int dtype, int64_t num_tokens,
                                   int num_kv_heads, int head_size, int64_t k_stride_tok, int64_t k_stride_head,
                                   int64_t v_stride_tok, int64_t v_stride_head, uint8_t* key_cache,
                                   uint8_t* value_cache, float* k_scale, float* v_scale, const int64_t* slot_mapping,
                                   int block_size, const float* rht_signs, const float* bias_k, const float* bias_v,
                                   const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* seq_slots,
                                   int num_seqs, uint16_t* exact_k, uint16_t* exact_v, int32_t* exact_tag,
                                   const exl3b_kv_layout* layout, void* stream) {
    KvWriteArgs a = {};
    int st = kv_write_common(a, key, value, dtype, num_tokens, num_kv_heads, head_size, k_stride_tok, k_stride_head,
                             v_stride_tok, v_stride_head, key_cache, value_cache, k_scale, v_scale, slot_mapping,
                             block_size, layout, kHD / 2);
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
    const int64_t per_block = 8 * kW4Rows;  // 8 warps of kW4Rows rows
    kv_int4_write_kernel<<<(unsigned)((items + per_block - 1) / per_block), 256, 0, (cudaStream_t)stream>>>(a, x);
    return cuda_status(cudaGetLastError());
}

extern "C" size_t exl3b_kv_attn_workspace_bytes(int num_tokens, int num_q_heads, int num_seqs, int num_kv_heads,
                                                int max_seq_len) {
    if (num_tokens <= 0 || num_q_heads <= 0 || num_seqs <= 0 || num_kv_heads <= 0) return 0;
    const int S = std::max(kv_splits(8, num_seqs, num_kv_heads, std::max(1, max_seq_len), 1),
                           kv_splits(4, num_seqs, num_kv_heads, std::max(1, max_seq_len), 1));
    const size_t qr = (size_t)num_tokens * num_q_heads * kHD * 2;
    return (qr + 255) / 256 * 256 + (size_t)num_tokens * num_q_heads * S * kPartialStride * 4;
}

static int kv_attn_common(int kv, const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                          int num_kv_heads, int head_size, const void* key_cache, const void* value_cache,
                          const float* k_scale, const float* v_scale, int block_size, const int32_t* block_table,
                          int64_t bt_stride, const int32_t* seq_lens, const int32_t* query_start_loc, int num_seqs,
                          int max_q_len, int max_seq_len, float softmax_scale, const float* rht_signs,
                          const uint16_t* exact_k, const uint16_t* exact_v, const int32_t* exact_tag,
                          const int32_t* seq_slots, const float* out_bias, void* workspace, size_t ws_bytes,
                          const exl3b_kv_layout* layout, void* stream) {
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
    // int4 decode over few (sequence, KV head) pairs (one warp holds all of a pair's query rows):
    // kDecodeTsplit warps share each split's keys, so a split is that many times longer and the
    // combine has as many times fewer partials (measured: int4 64k x 1 72.7 -> 58.2 us; int8 and
    // batched decode measured the same or slower, so they keep one warp per split)
    const int ts = (kv == 4 && max_q_len * G <= 8 && num_seqs * num_kv_heads <= 16) ? kDecodeTsplit : 1;
    const int S = kv_splits(kv, num_seqs, num_kv_heads, std::max(1, max_seq_len), max_q_len * G, ts);
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
    {
        const int lst = kv_layout(layout, block_size, num_kv_heads, kv == 8 ? kHD : kHD / 2, key_cache, value_cache,
                                  a.lay, a.al16);
        if (lst != EXL3B_OK) return lst;
    }
    const dim3 grid(num_seqs, num_kv_heads, S);
    // query rows per (sequence, KV head): up to 24 in one warp (8 per n-tile), 32 in two warps of 16
    const int rows = max_q_len * G;
    const int nt = rows <= 8 ? 1 : rows <= 16 ? 2 : rows <= 24 ? 3 : 2;
    const int warps = ts > 1 ? ts : rows <= 24 ? 1 : 2;
    a.tsplit = ts;
    cudaError_t e;
    if (kv == 8)
        e = nt == 1 ? launch_attn<8, 1>(grid, warps, a, st) : nt == 2 ? launch_attn<8, 2>(grid, warps, a, st)
                                                                     : launch_attn<8, 3>(grid, warps, a, st);
    else
        e = nt == 1 ? launch_attn<4, 1>(grid, warps, a, st) : nt == 2 ? launch_attn<4, 2>(grid, warps, a, st)
                                                                     : launch_attn<4, 3>(grid, warps, a, st);
    if (e != cudaSuccess) return cuda_status(e);
    KvReduceArgs r = {};
    r.partial = a.partial; r.out = reinterpret_cast<__half*>(out); r.seq_lens = seq_lens;
    r.query_start_loc = query_start_loc; r.num_seqs = num_seqs; r.num_tokens = num_tokens;
    r.num_q_heads = num_q_heads; r.num_splits = S; r.unrot_signs = kv == 4 ? rht_signs : nullptr;
    r.out_bias = kv == 4 ? out_bias : nullptr; r.group = G;
    const int64_t items = (int64_t)num_tokens * num_q_heads;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)items);
    cfg.blockDim = dim3(32 * reduce_warps(S));
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kv_reduce_kernel, r));
}

extern "C" int exl3b_kv_int8_attn(const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                                  int num_kv_heads, int head_size, const int8_t* key_cache,
                                  const int8_t* value_cache, const float* k_scale, const float* v_scale,
                                  int block_size, const int32_t* block_table, int64_t bt_stride,
                                  const int32_t* seq_lens, const int32_t* query_start_loc, int num_seqs,
                                  int max_q_len, int max_seq_len, float softmax_scale, void* workspace,
                                  size_t workspace_bytes, const exl3b_kv_layout* layout, void* stream) {
    return kv_attn_common(8, q, out, num_tokens, num_q_heads, num_kv_heads, head_size, key_cache, value_cache,
                          k_scale, v_scale, block_size, block_table, bt_stride, seq_lens, query_start_loc, num_seqs,
                          max_q_len, max_seq_len, softmax_scale, nullptr, nullptr, nullptr, nullptr, nullptr,
                          nullptr, workspace, workspace_bytes, layout, stream);
}

extern "C" int exl3b_kv_int4_attn(const uint16_t* q, uint16_t* out, int num_tokens, int num_q_heads,
                                  int num_kv_heads, int head_size, const uint8_t* key_cache,
                                  const uint8_t* value_cache, const float* k_scale, const float* v_scale,
                                  int block_size, const int32_t* block_table, int64_t bt_stride,
                                  const int32_t* seq_lens, const int32_t* query_start_loc, int num_seqs,
                                  int max_q_len, int max_seq_len, float softmax_scale, const float* rht_signs,
                                  const uint16_t* exact_k, const uint16_t* exact_v, const int32_t* exact_tag,
                                  const int32_t* seq_slots, const float* out_bias, void* workspace,
                                  size_t workspace_bytes, const exl3b_kv_layout* layout, void* stream) {
    return kv_attn_common(4, q, out, num_tokens, num_q_heads, num_kv_heads, head_size, key_cache, value_cache,
                          k_scale, v_scale, block_size, block_table, bt_stride, seq_lens, query_start_loc, num_seqs,
                          max_q_len, max_seq_len, softmax_scale, rht_signs, exact_k, exact_v, exact_tag, seq_slots,
                          out_bias, workspace, workspace_bytes, layout, stream);
}

static int kv_gather_common(int kv, const void* cache, const float* scale, int block_size, int num_kv_heads,
                            int head_size, const int32_t* block_ids, int64_t n, int blocks_per_seq, uint16_t* out,
                            const uint16_t* exact, const int32_t* exact_tag, const int32_t* seq_slots,
                            const int32_t* seq_lens, const exl3b_kv_layout* layout, void* stream) {
    if (head_size != kHD || block_size <= 0 || num_kv_heads <= 0 || blocks_per_seq <= 0) return EXL3B_DECLINED;
    if (n < 0) return EXL3B_BAD_ARG;
    if (n == 0) return EXL3B_OK;
    if (!cache || !scale || !block_ids || !out) return EXL3B_BAD_ARG;
    if (exact_tag && (!exact || !seq_slots || !seq_lens)) return EXL3B_BAD_ARG;
    KvGatherArgs a = {};
    a.cache = static_cast<const uint8_t*>(cache); a.scale = scale; a.block_ids = block_ids; a.n = n;
    a.bs = block_size; a.H = num_kv_heads; a.nb = blocks_per_seq; a.out = reinterpret_cast<__half*>(out);
    a.mul = kv == 4 ? 0.08838834764831845f : 1.f;
    a.exact = reinterpret_cast<const __half*>(exact); a.exact_tag = exact_tag; a.seq_slots = seq_slots;
    a.seq_lens = seq_lens;
    int al16 = 0;
    const int lst = kv_layout(layout, block_size, num_kv_heads, kv == 8 ? kHD : kHD / 2, cache, nullptr, a.lay, al16);
    if (lst != EXL3B_OK) return lst;
    const int64_t items = n * block_size * num_kv_heads;
    const unsigned grid = (unsigned)((items + 7) / 8);
    if (kv == 8) kv_gather_kernel<8><<<grid, 256, 0, (cudaStream_t)stream>>>(a);
    else kv_gather_kernel<4><<<grid, 256, 0, (cudaStream_t)stream>>>(a);
    return cuda_status(cudaGetLastError());
}

extern "C" int exl3b_kv_int8_gather(const int8_t* cache, const float* scale, int block_size, int num_kv_heads,
                                    int head_size, const int32_t* block_ids, int64_t n, uint16_t* out,
                                    const exl3b_kv_layout* layout, void* stream) {
    return kv_gather_common(8, cache, scale, block_size, num_kv_heads, head_size, block_ids, n, 1, out, nullptr,
                            nullptr, nullptr, nullptr, layout, stream);
}

extern "C" int exl3b_kv_int4_gather(const uint8_t* cache, const float* scale, int block_size, int num_kv_heads,
                                    int head_size, const int32_t* block_ids, int64_t n, int blocks_per_seq,
                                    uint16_t* out, const uint16_t* exact, const int32_t* exact_tag,
                                    const int32_t* seq_slots, const int32_t* seq_lens, const exl3b_kv_layout* layout,
                                    void* stream) {
    return kv_gather_common(4, cache, scale, block_size, num_kv_heads, head_size, block_ids, n, blocks_per_seq, out,
                            exact, exact_tag, seq_slots, seq_lens, layout, stream);
}
