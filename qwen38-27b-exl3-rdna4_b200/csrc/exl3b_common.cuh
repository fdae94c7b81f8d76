// Shared device helpers for the EXL3 B200 library (sm_100a only).
//
// Trellis format (reference vllm_plugin/exl3rocm/plugin.py:276, reference/exl3_oracle.py:13-16):
//   trellis int16 [k/16][n/16][16*K]; one 16x16 tile (rows = input features, cols = output features)
//   is a 256*K-bit ring, read as little-endian uint32 words whose bits are numbered from the MSB
//   of word 0.  Position t (0..255) holds the 16-bit state ending at bit (t+1)*K (mod 256*K).
//   t = 8L+i sits at row 2(L%4)+(i&1)+8((i>>1)&1), col 2(L>>3)+((L>>2)&1)+8(i>>2)
//   (reference/exl3_oracle.py:129-188).
//
// That placement is exactly the A operand of mma.m16n8k16 when A = W^T (16 output columns x 16
// input rows): lane L's eight positions t = 8L..8L+7 are its four A registers, pairs
// (i0,i1) (i4,i5) (i2,i3) (i6,i7).  So one lane decodes exactly what it feeds the tensor core.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/exl3b.h"

#define EXL3B_DEV __device__ __forceinline__

namespace exl3b {

// ---------------------------------------------------------------------------------------------
// codebooks (reference/exl3_oracle.py:40-47, 67-123)
// ---------------------------------------------------------------------------------------------
constexpr uint32_t kMul1Mult = 0x83DCD12Du;
constexpr uint32_t kMcgMult = 0xCBAC1FEDu;
constexpr uint32_t kCb0Mult = 89226354u;
constexpr uint32_t kCb0Add = 64248484u;
constexpr uint32_t kLopAnd = 0x8FFF8FFFu;
constexpr uint32_t kLopXor = 0x3B603B60u;
constexpr uint32_t kKInv2 = 0x1EEE1EEEu;   // half2(k_inv, k_inv)
constexpr uint32_t kKBias2 = 0xC931C931u;  // half2(k_bias, k_bias)
constexpr float kRScale = 0.088388347648f; // 1/sqrt(128) as every reference call site passes it

template <int CB>
EXL3B_DEV uint32_t cb_hash(uint32_t w) {
    if constexpr (CB == 2) return w * kMul1Mult;
    else if constexpr (CB == 1) return w * kMcgMult;
    else return w * kCb0Mult + kCb0Add;
}

EXL3B_DEV uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
EXL3B_DEV __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// silu(g) * u with the roundings of torch's fp16 F.silu(g) * u (vLLM SiluAndMul.forward_native):
// silu = g / (1 + exp(-g)) in fp32 rounded to fp16, then one fp16 multiply
EXL3B_DEV __half2 silu_mul2(__half2 g, __half2 u) {
    const float a = __low2float(g), b = __high2float(g);
    const __half2 s = __floats2half2_rn(a / (1.0f + expf(-a)), b / (1.0f + expf(-b)));
    return __hmul2(s, u);
}

// Two 16-bit states -> packed half2 (first state in the low half).
// cb2: fp16_fma(fp16(0x6400 + bytesum(w*M)), k_inv, k_bias), one rounding (fma.rn.f16x2).
// cb0/cb1: lop3 then fp16 add of the two halves of each hashed word, one rounding.
template <int CB>
EXL3B_DEV uint32_t decode_pair(uint32_t w0, uint32_t w1) {
    if constexpr (CB == 2) {
        uint32_t s0 = __dp4a(cb_hash<2>(w0), 0x01010101u, 0x6400u);
        uint32_t s1 = __dp4a(cb_hash<2>(w1), 0x01010101u, 0x6400u);
        uint32_t h = __byte_perm(s0, s1, 0x5410);
        return h2_as_u32(__hfma2(u32_as_h2(h), u32_as_h2(kKInv2), u32_as_h2(kKBias2)));
    } else {
        uint32_t x0 = (cb_hash<CB>(w0) & kLopAnd) ^ kLopXor;
        uint32_t x1 = (cb_hash<CB>(w1) & kLopAnd) ^ kLopXor;
        uint32_t lo = __byte_perm(x0, x1, 0x5410);
        uint32_t hi = __byte_perm(x0, x1, 0x7632);
        return h2_as_u32(__hadd2(u32_as_h2(lo), u32_as_h2(hi)));
    }
}

template <int CB>
EXL3B_DEV __half decode_one(uint32_t w) {
    uint32_t p = decode_pair<CB>(w, w);
    return __low2half(u32_as_h2(p));
}

// ---------------------------------------------------------------------------------------------
// window extraction for one lane of one tile
// ---------------------------------------------------------------------------------------------
// Lane L needs the bits [8LK + K - 16, 8LK + 8K) of the ring.  LaneGeom<K> holds the word
// offsets (mod 8K) of the NW words that cover that span and the bit phase phi of the span start
// inside the first word.  For K = 4 and 8 phi is the same for every lane (20 and 24) and the
// windows come straight from the raw words with constant shifts; for other K the lane first
// shifts its words left by phi so that every window sits at a constant position.
template <int K>
struct LaneGeom {
    static constexpr bool kConstPhi = (K == 4 || K == 8);
    static constexpr int kPhi = (K == 4) ? 20 : 24;          // used when kConstPhi
    static constexpr int kNY = (16 + 7 * K + 31) / 32;       // words after pre-alignment
    static constexpr int kNW = kConstPhi ? (kPhi + 16 + 7 * K + 31) / 32
                                         : (31 + 16 + 7 * K + 31) / 32;
    uint32_t off[kNW];  // byte offsets of the words inside the tile
    uint32_t phi;

    EXL3B_DEV void init(int lane) {
        const int b0 = 8 * lane * K + K - 16 + 256 * K;  // >= 0
        const int wf = b0 >> 5;
        phi = (uint32_t)(b0 & 31);
#pragma unroll
        for (int j = 0; j < kNW; ++j) off[j] = (uint32_t)(((wf + j) % (8 * K)) * 4);
    }
};

// bits [p-16, p) of the MSB-first word array V, p a compile-time constant
template <int P, int N>
EXL3B_DEV uint32_t window_at(const uint32_t (&V)[N]) {
    constexpr int j = (P - 1) / 32;
    constexpr int s = 32 * (j + 1) - P;
    static_assert(j < N, "window outside the lane's words");
    if constexpr (P - 16 >= 32 * j) {
        if constexpr (s == 16) return V[j] >> 16;
        else return (V[j] >> s) & 0xFFFFu;
    } else {
        return __funnelshift_r(V[j], V[j - 1], s) & 0xFFFFu;
    }
}

// 32 bits ending at bit p: low half = window ending at p, high half = window ending at p-16
template <int P, int N>
EXL3B_DEV uint32_t span32_at(const uint32_t (&V)[N]) {
    constexpr int j = (P - 1) / 32;
    constexpr int s = 32 * (j + 1) - P;
    if constexpr (s == 0) return V[j];
    else return __funnelshift_r(V[j], V[j - 1], s);
}

template <int K, int I, int N>
EXL3B_DEV void windows_generic(const uint32_t (&Y)[N], uint32_t (&w)[8]) {
    if constexpr (I < 8) {
        w[I] = window_at<16 + I * K>(Y);
        windows_generic<K, I + 1>(Y, w);
    }
}

// Extract the lane's eight states w[i] (position 8L+i) from its raw words W.
template <int K>
EXL3B_DEV void lane_windows(const uint32_t (&W)[LaneGeom<K>::kNW], uint32_t phi, uint32_t (&w)[8]) {
    using G = LaneGeom<K>;
    if constexpr (K == 4) {
        // p_i = 36 + 4i; the 32 bits ending at p_i hold windows i (low) and i-4 (high)
#pragma unroll
        for (int i = 4; i < 8; ++i) {
            const uint32_t r = (i == 7) ? W[1] : __funnelshift_r(W[1], W[0], 28 - 4 * i);
            w[i] = r & 0xFFFFu;
            w[i - 4] = r >> 16;
        }
    } else if constexpr (K == 8) {
        // p_i = 40 + 8i; spans ending at p_2, p_3, p_6, p_7 hold windows (2,0) (3,1) (6,4) (7,5)
        const uint32_t r2 = span32_at<56>(W), r3 = span32_at<64>(W);
        const uint32_t r6 = span32_at<88>(W), r7 = span32_at<96>(W);
        w[2] = r2 & 0xFFFFu; w[0] = r2 >> 16;
        w[3] = r3 & 0xFFFFu; w[1] = r3 >> 16;
        w[6] = r6 & 0xFFFFu; w[4] = r6 >> 16;
        w[7] = r7 & 0xFFFFu; w[5] = r7 >> 16;
    } else {
        uint32_t Y[G::kNY];
#pragma unroll
        for (int j = 0; j < G::kNY; ++j)
            Y[j] = (j + 1 < G::kNW) ? __funnelshift_l(W[j + 1], W[j], phi) : (W[j] << phi);
        windows_generic<K, 0>(Y, w);
    }
}

// Decode the lane's eight weights of one tile into its four mma A registers.
template <int K, int CB>
EXL3B_DEV void lane_decode_frag(const uint32_t (&W)[LaneGeom<K>::kNW], uint32_t phi, uint32_t (&a)[4]) {
    uint32_t w[8];
    lane_windows<K>(W, phi, w);
    a[0] = decode_pair<CB>(w[0], w[1]);
    a[1] = decode_pair<CB>(w[4], w[5]);
    a[2] = decode_pair<CB>(w[2], w[3]);
    a[3] = decode_pair<CB>(w[6], w[7]);
}

// ---------------------------------------------------------------------------------------------
// 128-point Hadamard over one warp: lane l holds elements 4l..4l+3 (natural-order Sylvester,
// H128 = H32 (lanes, xor butterflies) x H4 (slots); reference/exl3_oracle.py:236-258)
// ---------------------------------------------------------------------------------------------
EXL3B_DEV void had128_warp(float (&v)[4]) {
    const float s0 = v[0] + v[1], d0 = v[0] - v[1];
    const float s1 = v[2] + v[3], d1 = v[2] - v[3];
    v[0] = s0 + s1; v[1] = d0 + d1; v[2] = s0 - s1; v[3] = d0 - d1;
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const bool upper = (lane & d) != 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float o = __shfl_xor_sync(0xFFFFFFFFu, v[j], d);
            v[j] = upper ? (o - v[j]) : (v[j] + o);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// mma, mbarrier and bulk-copy wrappers
// ---------------------------------------------------------------------------------------------
EXL3B_DEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// the same without `volatile`, so that the compiler schedules it freely among the decode
EXL3B_DEV void mma_16816_nv(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

EXL3B_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

EXL3B_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" :: "r"(bar), "r"(count) : "memory");
}
EXL3B_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
EXL3B_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }\n" :: "r"(bar) : "memory");
}
EXL3B_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }\n"
                 :: "r"(bar), "r"(bytes) : "memory");
}
// add expected transaction bytes to the current phase without arriving
EXL3B_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n" :: "r"(bar), "r"(bytes) : "memory");
}
// try_wait with a suspend-time hint: a waiting warp sleeps in hardware (up to ~20 us per try)
// instead of spinning through issue slots that the decoding warps need
EXL3B_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }\n"
        : "=r"(ok) : "r"(bar), "r"(parity), "r"(20000u) : "memory");
    return ok != 0;
}

// Wait limit: about a second of SM clock.  Past it the kernel records an error and gives up;
// no wait in this library is unbounded.
constexpr long long kWaitCycles = 2000000000LL;

EXL3B_DEV bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            if (err) atomicExch(err, code);
            return false;
        }
    }
    return true;
}

// The same wait, but it also gives up (without recording an error) as soon as another warp of
// the CTA has raised *abort: a CTA whose wait failed stops within one try instead of one limit per
// remaining barrier.  The fast path is a single try_wait.
EXL3B_DEV bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, int* err, int code, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort != 0) return false;
        if (clock64() - t0 > kWaitCycles) {
            if (err) atomicExch(err, code);
            *abort = 1;
            return false;
        }
    }
    return true;
}

// Global -> shared bulk copy (no multicast), completion counted on an mbarrier.
EXL3B_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
        :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

EXL3B_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
EXL3B_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

EXL3B_DEV void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" :: "r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------------------------
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? EXL3B_OK : -(int)e; }

inline bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

}  // namespace exl3b
