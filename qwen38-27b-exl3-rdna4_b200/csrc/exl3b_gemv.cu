// The EXL3 linear for 1 <= m <= 16 rows (decode and speculative verify), fused end to end:
//
//   one launch:        stream-K over units of R trellis k-tile rows x one super-block of up to
//                      1024 output columns (64 n-tiles).  In the checkpoint layout
//                      [k/16][n/16][16K] a unit row is one contiguous run of up to 64 x 32K
//                      bytes (8 KB at K = 4), so a producer warp fetches a unit with R bulk
//                      copies (no multicast) into a shared-memory ring, and while they fly it
//                      writes the unit's input transform A_had = fp16(H128 fp16(x * suh) / sqrt(128))
//                      next to them, in mma B-fragment order.  Sixteen decode warps
//                      decode the trellis in registers straight into mma.m16n8k16 A fragments
//                      (W^T x A_had^T, fp32 accumulate); warp w owns n-tiles w, w+16, w+32, w+48 of
//                      the super-block.  When the CTA leaves a super-block the decode warps pool
//                      their accumulators in a shared-memory tile and warp b takes column block b:
//                      it reduces the block across the CTAs that shared it (partials in the
//                      workspace, fixed summation order, last arriver finishes) and applies
//                      had_out + svh.
//   The launch is a programmatic dependent launch: the first ring of trellis copies is issued
//   before griddepcontrol.wait, so weight streaming overlaps the end of the previous kernel; x,
//   the workspace and y are touched only after the wait.
//
// Reference semantics: reference/exl3_oracle.py:307-351 (gemv_mul1, all codebooks);
// kernels replaced: exl3_gemm / exl3_gemv_mr / exl3_mgemm / exl3_gemv_mr_grouped of the fork
// (vllm_plugin/exl3rocm/ops.py:80-85,134-170; 0002-gemv-multirow.patch:79-88 for the rule that
// every row equals the m = 1 result bit for bit: here the work partition depends only on
// (k, n, groups, K) and each mma column is one input row, so rows never interact).
#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kDecodeWarps = 16;
constexpr int kProducerWarp = kDecodeWarps;
constexpr int kThreads = (kDecodeWarps + 1) * 32;
constexpr int kFlushBar = 1;      // named barrier of the decode warps
constexpr int kNormBar = 2;       // named barrier of all warps after the fused RMSNorm's row sums
constexpr int kPairBar0 = 3;      // named barriers 3..10: the two warps that finish column block b
constexpr int kMaxBatch = 4;      // partials a finishing warp loads before summing them (8 spilled 1.2 KB)
constexpr int kSbTiles = 64;                 // n-tiles of a full super-block (1024 columns)
constexpr int kAccCols = kSbTiles * 16 + 4;  // accumulator-tile row, padded against bank conflicts

// trellis k-tile slots per unit (64 tiles each) at K <= 4; K > 4 takes 2.  Larger units measured
// faster: at K = 4, units of 4 slots made the layer step 10 % slower and units of 2 40 % slower
// than units of 8 (fewer hand-offs between producer and decode warps per byte).
#ifndef EXL3B_GEMV_R0_SMALLK
#define EXL3B_GEMV_R0_SMALLK 8
#endif
constexpr int kR0SmallK = EXL3B_GEMV_R0_SMALLK;
static_assert(kR0SmallK == 2 || kR0SmallK == 4 || kR0SmallK == 8, "rows per unit");
__host__ __device__ constexpr int rows_per_unit(int K) { return K <= 4 ? kR0SmallK : 2; }
constexpr int kMaxUnitRows = 16;  // k-rows of one unit at most (R0 * q), bounding the A_had area

struct GemvGroups {
    const uint16_t* trellis[EXL3B_MAX_GROUPS];
    const __half* svh[EXL3B_MAX_GROUPS];
    __half* y[EXL3B_MAX_GROUPS];
    int n_tiles[EXL3B_MAX_GROUPS];
    int blk_prefix[EXL3B_MAX_GROUPS + 1];  // first global 128-column block of each group
    int sb_prefix[EXL3B_MAX_GROUPS + 1];   // first global super-block of each group
    int sb_base[EXL3B_MAX_GROUPS];         // column blocks per super-block (the first sb_extra get one more)
    int sb_extra[EXL3B_MAX_GROUPS];
};

struct GemvParams {
    GemvGroups g;
    const void* x;        // [m][k] fp16, or bf16 when x_bf16
    int x_bf16;
    const __half* suh[EXL3B_MAX_GROUPS];
    float* partials;      // workspace: [ctas + super-blocks - 1][m][sb_cols], slot = cta + super-block
    int* counters;        // workspace: one per global column block
    int* err;             // workspace error word
    unsigned long long* ticket;  // workspace: the slot ticket counter (never reset)
    int groups, m, k, kt;  // kt = k / 16
    int ku;               // units per super-block = kt / (R0 * q)
    int q;                // k-rows per 64-tile stage slot (super-blocks of 64 / q n-tiles): 1, 2 or 4
    int units, ctas;
    int sb_cols;          // widest super-block of the call, in columns
    int64_t ldy;
    int y_add;            // y += result (the residual add of the caller's block)
    // fused RMSNorm of x (norm_w != null): the linear runs on fp16(fp16(x * s) * norm_w) with
    // s = rsqrt(mean(x^2) + norm_eps) per row
    const __half* norm_w;
    float norm_eps;
    // SwiGLU epilogue (act): groups 0 and 1 (gate, up) of equal width stage their fp16 outputs in
    // `stage` [m][2n]; the second finisher of column block b writes silu(gate) * up to y[0]
    int act;
    __half* stage;
    int act_ctr;          // first pair counter (after the per-block counters of the call)
    // fused tensor-parallel all-reduce (tp_size > 1): every rank's communication buffer
    int tp_size, tp_rank, tp_blocks, tp_rows;
    uint8_t* tp_buf[EXL3B_MAX_TP];
};


// Communication buffer of one rank: a 256-byte header (call counter, finished-CTA counter), then
// slots [2 parities][tp ranks][blocks][rows][128] of (fp32 value, call number) pairs, 8 bytes each.
// Rank s writes its partial of block b for call e into slot [e & 1][s][b] of every rank with 16-byte
// volatile stores of two such pairs; a reader polls its own slot until every pair carries e, so data
// and flag arrive together and no fence is needed (the low-latency protocol of NCCL's LL).
constexpr size_t kTpHeader = 256;
__host__ __device__ inline size_t tp_comm_bytes(int tp, int blocks, int rows) {
    return kTpHeader + (size_t)2 * tp * blocks * rows * 128 * 8;
}

EXL3B_DEV void st_pairs(uint32_t* p, float a, float b, int ep) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};\n"
                 :: "l"(p), "r"(__float_as_uint(a)), "r"(ep), "r"(__float_as_uint(b)), "r"(ep) : "memory");
}
EXL3B_DEV uint4 ld_pairs(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}

// ---------------------------------------------------------------------------------------------
// stream-K partition helpers (64-bit: U * P fits easily)
// ---------------------------------------------------------------------------------------------
// Slot c of P (U >= P units) takes units [unit_start(c), unit_start(c + 1)): the first U % P slots
// one unit more than the rest.  Slots are handed out in the order the CTAs start (see the kernel), so
// the CTAs that start last -- on the SMs the previous kernel's finishing CTAs leave last -- take the
// lighter shares.
EXL3B_DEV int unit_start(int c, int U, int P) { return c * (U / P) + min(c, U % P); }
EXL3B_DEV int cta_of_unit(int u, int U, int P) {
    const int b = U / P, e = U % P, heavy = e * (b + 1);
    return u < heavy ? u / (b + 1) : e + (u - heavy) / b;
}

struct SbInfo {
    int g;     // group
    int b0;    // first 128-column block of the super-block, inside the group
    int nblk;  // its column blocks
};

EXL3B_DEV SbInfo sb_info(const GemvGroups& gg, int groups, int sb) {
    int g = 0;
    while (g + 1 < groups && sb >= gg.sb_prefix[g + 1]) ++g;
    const int i = sb - gg.sb_prefix[g];
    const int base = gg.sb_base[g], extra = gg.sb_extra[g];
    return {g, i * base + min(i, extra), base + (i < extra ? 1 : 0)};
}

// ---------------------------------------------------------------------------------------------
// launch 2: the stream-K decode GEMV
// ---------------------------------------------------------------------------------------------
// Shared memory: a ring of `stages` stages (R trellis rows of up to 64 tiles at a fixed stride,
// then the unit's A_had rows), the fp32 accumulator tile [m rows][kAccCols] where the decode
// warps pool a finished super-block, and the mbarriers.  The ring depth is what the budget leaves
// beside a tile of 8 MT rows, whatever m: at m = 1 a third 64 KB stage (room for it exists) measured
// 3 % slower per layer step, its copies in flight competing with the next unit's.
template <int K, int MT, int R0_>
struct GemvSmem {
    static constexpr int R0 = R0_;                         // stage slots of 64 tiles
    static constexpr int kTile = 32 * K;                  // bytes of one 16x16 tile
    static constexpr int kRowBytes = kSbTiles * kTile;    // stride of the stage slots
    static constexpr int kTrellisStage = R0 * kRowBytes;
    static constexpr int kAhadStage = (R0 * 4 > kMaxUnitRows ? kMaxUnitRows : R0 * 4) * 8 * MT * 32;  // k-tiles x 8 MT rows x 16 halves
    static constexpr int kStageBytes = kTrellisStage + kAhadStage;
    static constexpr int kBudget = 220 * 1024;
    static constexpr int kMaxStages = 8;
    static constexpr int kTail = 2 * kMaxStages * 8 + 64 + 4 * EXL3B_GEMV_MAX_ROWS;  // barriers, flags, 1/rms
    static_assert((kBudget - 8 * MT * kAccCols * 4 - kTail) / kStageBytes >= 2, "shared-memory ring too small");
};

// Runtime part of the layout (depends on m): ring, accumulator tile, the m == 1 run sums, full[S], empty[S]
// barriers; flags: abort (int), the flush's abort snapshot (int), the finish decision of each column
// block shared by its two warps (8 ints), the CTA's stream-K slot (int); then the fused RMSNorm's 1/rms of each row.
struct GemvLayout {
    int stages, acc_off, hi_off, bar_off, flag_off, norm_off, total;
};
template <int K, int MT, int R0>
__host__ __device__ inline GemvLayout gemv_layout(int m) {
    using S = GemvSmem<K, MT, R0>;
    GemvLayout L;
    const int acc = (m * kAccCols * 4 + 127) / 128 * 128;
    L.stages = (S::kBudget - 8 * MT * kAccCols * 4 - S::kTail) / S::kStageBytes;
    if (L.stages > S::kMaxStages) L.stages = S::kMaxStages;
    L.acc_off = L.stages * S::kStageBytes;
    // m == 1: the second run sums of the flush, 128 floats per column block, inside the room the
    // budget keeps for 8 MT accumulator rows
    L.hi_off = L.acc_off + acc;
    L.bar_off = L.hi_off + (m == 1 ? 8 * 128 * 4 : 0);
    L.flag_off = L.bar_off + 2 * L.stages * 8;
    L.norm_off = L.flag_off + 64;
    L.total = L.norm_off + 4 * EXL3B_GEMV_MAX_ROWS;
    return L;
}

// Decode warps blk (half 0) and blk + 8 (half 1) finish column block `blk` of super-block `sb`
// (only when a CTA leaves a super-block); each takes half of the rows, half 0 the first ceil(m / 2).
// The partials of the CTAs that shared the block are summed as two runs, CTAs cf..mid-1 and mid..cl,
// each in CTA order, then added: with m == 1 half 1 sums the second run of row 0 (into hi_s) while
// half 0 sums the first, so two warps' loads are in flight; with m > 1 each warp sums both runs of its
// rows itself.  Every row takes the same operations either way, so it is bitwise the same for every m.
// The two warps meet at named barrier kPairBar0 + blk; `fin` is their shared decision word.
template <int MT>
__device__ __forceinline__ void flush_block(const GemvParams& p, const float* acc_s, float* hi_s,
                                         volatile int* abort_flag, int c, int sb, SbInfo si, int blk, int half,
                                         int u0, int u1, int lane, volatile int* fin) {
    const int ku = p.ku, U = p.units, P = p.ctas, m = p.m;
    const int mh = (m + 1) >> 1;
    const int r_lo = half * mh, r_hi = half ? m : mh;  // this warp's rows (none for half 1 when m == 1)
    auto pair_sync = [&]() { named_bar(kPairBar0 + blk, 64); };
    // If this CTA covered the super-block's whole k range, transform and store; otherwise
    // publish the partial and, if it is the last of the block's CTAs to arrive, gather all
    // partials in fixed CTA order and finish the block.
    const int seg_lo = max(u0, sb * ku), seg_hi = min(u1, (sb + 1) * ku);
    const bool whole = (seg_lo == sb * ku) && (seg_hi == (sb + 1) * ku);
    const int cf = cta_of_unit(sb * ku, U, P), cl = cta_of_unit((sb + 1) * ku - 1, U, P);
    const int Bg = p.g.blk_prefix[si.g] + si.b0 + blk;
    const int col = blk * 128 + 4 * lane;  // column inside the super-block
    bool finalize = whole;
    if (!whole) {
        // CTA ranges are contiguous and ordered, so cta + super-block is unique among the
        // (CTA, super-block) pairs that meet
        float* mine = p.partials + ((int64_t)(c + sb) * m) * p.sb_cols;
        for (int row = r_lo; row < r_hi; ++row)
            __stcg(reinterpret_cast<float4*>(mine + (int64_t)row * p.sb_cols + col),
                   *reinterpret_cast<const float4*>(acc_s + row * kAccCols + col));
        __syncwarp();
        pair_sync();  // both halves' partial stores come before the release below
        if (half == 0) {
            int v = 0;
            if (lane == 0) {
                // acq_rel at gpu scope: releases the pair's partial stores (ordered before this by
                // the barriers) and, for the last arriver, acquires the other CTAs' partials
                asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;\n" : "=r"(v) : "l"(p.counters + Bg) : "memory");
                *fin = v;
            }
            v = __shfl_sync(0xFFFFFFFFu, v, 0);
            __syncwarp();  // every lane's loads of the partials below come after lane 0's acquire
            finalize = (v == cl - cf);
        }
        pair_sync();  // half 1 reads the decision after the acquire
        if (half == 1) finalize = (*fin == cl - cf);
    }
    if (finalize) {
        const int b = si.b0 + blk;
        const uint2 sv = *reinterpret_cast<const uint2*>(p.g.svh[si.g] + b * 128 + 4 * lane);
        // the partials of CTAs lo..hi-1 (in CTA order) of `row`, one batch of loads in flight at a time
        auto run_sum = [&](int row, int lo, int hi, float (&v)[4]) {
            v[0] = v[1] = v[2] = v[3] = 0.f;
            for (int c0 = lo; c0 < hi; c0 += kMaxBatch) {
                float4 t[kMaxBatch];
#pragma unroll
                for (int q = 0; q < kMaxBatch; ++q) {
                    const int cc = c0 + q;
                    if (cc >= hi) break;
                    t[q] = (cc == c) ? *reinterpret_cast<const float4*>(acc_s + row * kAccCols + col)
                                     : __ldcg(reinterpret_cast<const float4*>(
                                           p.partials + ((int64_t)(cc + sb) * m + row) * p.sb_cols + col));
                }
#pragma unroll
                for (int q = 0; q < kMaxBatch; ++q) {
                    if (c0 + q >= hi) break;
                    v[0] += t[q].x; v[1] += t[q].y; v[2] += t[q].z; v[3] += t[q].w;
                }
            }
        };
        // c_rot is stored fp16 between the dot and the output transform (oracle :349-351)
        auto finish_row = [&](int row, const float (&v)[4]) {
            const __half2 c01 = __floats2half2_rn(v[0], v[1]), c23 = __floats2half2_rn(v[2], v[3]);
            float h[4] = {__low2float(c01), __high2float(c01), __low2float(c23), __high2float(c23)};
            had128_warp(h);
            __half2 y01 = __floats2half2_rn(h[0] * kRScale, h[1] * kRScale);
            __half2 y23 = __floats2half2_rn(h[2] * kRScale, h[3] * kRScale);
            y01 = __hmul2(y01, u32_as_h2(sv.x));
            y23 = __hmul2(y23, u32_as_h2(sv.y));
            if (p.act) {  // staged in L2 for the pair's second finisher
                __stcg(reinterpret_cast<uint2*>(p.stage + (int64_t)row * 2 * (p.g.n_tiles[0] * 16) +
                                                si.g * (p.g.n_tiles[0] * 16) + b * 128 + 4 * lane),
                       make_uint2(h2_as_u32(y01), h2_as_u32(y23)));
                return;
            }
            uint2* dst = reinterpret_cast<uint2*>(p.g.y[si.g] + row * p.ldy + b * 128 + 4 * lane);
            if (p.y_add) {  // one fp16 add (exact sum, one rounding), as torch's fp16 x + residual
                const uint2 o = *dst;
                y01 = __hadd2(y01, u32_as_h2(o.x));
                y23 = __hadd2(y23, u32_as_h2(o.y));
            }
            *dst = make_uint2(h2_as_u32(y01), h2_as_u32(y23));
        };
        // Exchange (tensor parallel): this rank's k-slice partial of block b goes to every rank as
        // (value, call) pairs in slot [par][rank][b] of each rank's buffer; then each rank polls its
        // own slots of every rank until all pairs carry this call's number, and sums in rank order.
        const int tp = p.tp_size, rk = p.tp_rank, nb = p.tp_blocks, rows = p.tp_rows;
        // the counter is written only by earlier kernels on this GPU (visible after griddepcontrol.wait)
        const int ep = tp > 1 ? *reinterpret_cast<volatile const int*>(p.tp_buf[rk]) + 1 : 0;
        const int par = ep & 1;
        auto slot = [&](int owner, int src, int row) {
            return reinterpret_cast<uint32_t*>(p.tp_buf[owner] + kTpHeader) +
                   ((((int64_t)par * tp + src) * nb + b) * rows + row) * 256 + 8 * lane;
        };
        // the block's k-range sum of a row, over the CTAs that shared it, then its output (or, under
        // tensor parallelism, its exchange)
        auto consume = [&](int row, const float (&v)[4]) {
            if (tp <= 1) {
                finish_row(row, v);
            } else {
                for (int r = 0; r < tp; ++r) {
                    uint32_t* d = slot(r, rk, row);
                    st_pairs(d, v[0], v[1], ep);
                    st_pairs(d + 4, v[2], v[3], ep);
                }
            }
        };
        // The sum runs: m == 1: half h sums run h of row 0 (half 1's through hi_s); m > 1: each warp
        // both runs of its rows.  One call site of run_sum for all of them.
        const int mid = cf + (cl - cf + 2) / 2;  // runs cf..mid-1 and mid..cl (the second empty when whole)
        float4* hi_mine = reinterpret_cast<float4*>(hi_s + blk * 128) + lane;
        const int jobs = m == 1 ? 1 : 2 * (r_hi - r_lo);
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        for (int it = 0; it < jobs; ++it) {
            const int row = m == 1 ? 0 : r_lo + (it >> 1);
            const int run = m == 1 ? half : (it & 1);
            float w[4];
            run_sum(row, run ? mid : cf, run ? cl + 1 : mid, w);
            if (run == 0) {
                v[0] = w[0]; v[1] = w[1]; v[2] = w[2]; v[3] = w[3];
            } else if (m == 1) {
                *hi_mine = make_float4(w[0], w[1], w[2], w[3]);
            } else {
                if (mid <= cl) { v[0] += w[0]; v[1] += w[1]; v[2] += w[2]; v[3] += w[3]; }
                consume(row, v);
            }
        }
        if (m == 1) {
            pair_sync();  // half 1's run sum before half 0 reads it
            if (half == 0) {
                if (mid <= cl) {
                    const float4 h = *hi_mine;
                    v[0] += h.x; v[1] += h.y; v[2] += h.z; v[3] += h.w;
                }
                consume(0, v);
            }
        }
        if (tp <= 1) {
            if (p.act) {
                // gate and up block b are finished by different warp pairs, in any order: the
                // second one (pair counter) reads both staged blocks and writes the activation
                __syncwarp();
                pair_sync();  // both halves' staged rows come before the release below
                int w = 0;
                if (half == 0) {
                    if (lane == 0) {
                        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;\n"
                                     : "=r"(w) : "l"(p.counters + p.act_ctr + b) : "memory");
                        *fin = w;
                    }
                    w = __shfl_sync(0xFFFFFFFFu, w, 0);
                    __syncwarp();
                }
                pair_sync();
                if (half == 1) w = *fin;
                if (w == 1) {
                    const int64_t nn = p.g.n_tiles[0] * 16;
                    for (int row = r_lo; row < r_hi; ++row) {
                        const __half* s = p.stage + (int64_t)row * 2 * nn + b * 128 + 4 * lane;
                        const uint2 g = __ldcg(reinterpret_cast<const uint2*>(s));
                        const uint2 u = __ldcg(reinterpret_cast<const uint2*>(s + nn));
                        const __half2 a01 = silu_mul2(u32_as_h2(g.x), u32_as_h2(u.x));
                        const __half2 a23 = silu_mul2(u32_as_h2(g.y), u32_as_h2(u.y));
                        *reinterpret_cast<uint2*>(p.g.y[0] + row * p.ldy + b * 128 + 4 * lane) =
                            make_uint2(h2_as_u32(a01), h2_as_u32(a23));
                    }
                    if (lane == 0 && half == 0) p.counters[p.act_ctr + b] = 0;
                }
            }
        } else {
            bool ok = true;
            for (int row = r_lo; row < r_hi; ++row) {
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                for (int r = 0; r < tp; ++r) {  // fixed rank order: identical sums on every rank
                    const uint32_t* q = slot(rk, r, row);
                    uint4 a0 = ld_pairs(q), a1 = ld_pairs(q + 4);
                    const long long t0 = clock64();
                    while (ok && (a0.y != (uint32_t)ep || a0.w != (uint32_t)ep || a1.y != (uint32_t)ep ||
                                  a1.w != (uint32_t)ep)) {
                        if (clock64() - t0 > kWaitCycles) ok = false;
                        a0 = ld_pairs(q);
                        a1 = ld_pairs(q + 4);
                    }
                    v[0] += __uint_as_float(a0.x); v[1] += __uint_as_float(a0.z);
                    v[2] += __uint_as_float(a1.x); v[3] += __uint_as_float(a1.z);
                }
                if (!__all_sync(0xFFFFFFFFu, ok)) {
                    if (lane == 0) { atomicExch(p.err, 6); *abort_flag = 1; }
                    break;
                }
                finish_row(row, v);
            }
        }
        if (!whole && lane == 0 && half == 0) p.counters[Bg] = 0;
    }
}

// Four inputs of row `row` starting at column col, as fp16 (bf16 x rounded to nearest even, as
// torch's .to(float16))
EXL3B_DEV uint2 load_x4(const GemvParams& p, int row, int col) {
    uint2 xr = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.x) + (int64_t)row * p.k + col);
    if (p.x_bf16) {
        const __nv_bfloat162 b01 = *reinterpret_cast<const __nv_bfloat162*>(&xr.x);
        const __nv_bfloat162 b23 = *reinterpret_cast<const __nv_bfloat162*>(&xr.y);
        xr.x = h2_as_u32(__floats2half2_rn(__low2float(b01), __high2float(b01)));
        xr.y = h2_as_u32(__floats2half2_rn(__low2float(b23), __high2float(b23)));
    }
    return xr;
}

// Fused RMSNorm, first half: every thread of the CTA sums the squares of the fp16 inputs of chunks
// threadIdx.x, threadIdx.x + kThreads, ... (4 inputs each) of each row; warp w's sums go to
// part[16 w + row].  The split of a row over threads is fixed, so its sum does not depend on m.
constexpr int kNormChunks = 8;  // 4-input chunks per thread and row: k <= 8 * 4 * kThreads = 17408
EXL3B_DEV void norm_partials(const GemvParams& p, float* part, int warp, int lane) {
    const int nch = p.k / 4;
    for (int row = 0; row < p.m; ++row) {
        uint2 xr[kNormChunks];  // all of the row's loads in flight together
#pragma unroll
        for (int j = 0; j < kNormChunks; ++j) {
            const int ch = threadIdx.x + j * kThreads;
            xr[j] = ch < nch ? load_x4(p, row, 4 * ch) : make_uint2(0u, 0u);
        }
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kNormChunks; ++j) {
            const float2 a = __half22float2(u32_as_h2(xr[j].x)), b = __half22float2(u32_as_h2(xr[j].y));
            ss = fmaf(a.x, a.x, ss);
            ss = fmaf(a.y, a.y, ss);
            ss = fmaf(b.x, b.x, ss);
            ss = fmaf(b.y, b.y, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
        if (lane == 0) part[16 * warp + row] = ss;
    }
}

template <int K, int CB, int MT, int R0_>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
    using S = GemvSmem<K, MT, R0_>;
    const GemvLayout lay = gemv_layout<K, MT, R0_>(p.m);
    const int kStages = lay.stages;
    constexpr int R0 = S::R0;
    const int q = p.q, R = R0 * p.q;  // k-rows per unit; row r sits in slot r / q at tile (r % q) * 64 / q
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full0 = sbase + lay.bar_off, empty0 = full0 + kStages * 8;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + lay.flag_off);
    volatile int* flush_snap = abort_flag + 1;  // the abort flag as every flushing warp sees it
    volatile int* fin_s = abort_flag + 2;       // [8] finish decisions of the column-block pairs
    float* inv_rms = reinterpret_cast<float*>(smem + lay.norm_off);
    // the fused RMSNorm's per-warp row sums borrow the accumulator tile: no flush can write it before
    // the producer has read them (the first flush follows the first published unit)
    float* norm_part = reinterpret_cast<float*>(smem + lay.acc_off);

    volatile int* slot_s = abort_flag + 10;  // this CTA's stream-K slot
    if (threadIdx.x == 0) {
        // Slots in start order: P consecutive tickets of the ever-growing 64-bit counter are P
        // distinct slots mod P.  Every CTA takes its ticket before griddepcontrol.launch_dependents,
        // so no later launch's tickets interleave with this one's.  The slot decides the work, never
        // the arithmetic: a slot's partial sums are the same whichever CTA runs it.
        const unsigned long long t = atomicAdd(p.ticket, 1ull);
        *slot_s = (int)(t % (unsigned long long)p.ctas);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kDecodeWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int c = *slot_s, P = p.ctas, U = p.units, ku = p.ku, m = p.m;
    const int u0 = unit_start(c, U, P), u1 = unit_start(c + 1, U, P);
    const int nunits = u1 - u0;

    griddep_launch();  // the next kernel in the stream may start its own prologue

    if (warp == kProducerWarp) {
        // ------------------------------ producer warp ------------------------------
        // issue(i): claim unit i's stage (after the decode warps released it), announce its bytes
        // and start its R trellis row copies.  transform(i): write its A_had rows, then arrive.
        int sb = -1;
        SbInfo si = {0, 0, 0};
        int issued = 0;
        auto locate = [&](int u) {
            if (u / ku != sb) {
                sb = u / ku;
                si = sb_info(p.g, p.groups, sb);
            }
        };
        auto issue = [&](int i) -> bool {
            const int s = i % kStages, n = i / kStages;
            if (n > 0) {
                const bool ok = mbar_wait_or_abort(empty0 + 8 * s, (n - 1) & 1, p.err, 1, abort_flag);
                if (!__all_sync(0xFFFFFFFFu, ok)) return false;
            }
            const int u = u0 + i;
            locate(u);
            const int kr0 = (u - sb * ku) * R;
            const uint32_t row_bytes = (uint32_t)si.nblk * 8 * S::kTile;
            if (lane == 0) mbar_expect_tx(full0 + 8 * s, R * row_bytes);
            __syncwarp();
            if (lane < R) {
                const uint16_t* src =
                    p.g.trellis[si.g] + ((int64_t)(kr0 + lane) * p.g.n_tiles[si.g] + si.b0 * 8) * (16 * K);
                const uint32_t dst = sbase + s * S::kStageBytes + (lane / q) * S::kRowBytes +
                                     (lane % q) * (kSbTiles / q) * S::kTile;
                bulk_g2s(dst, src, row_bytes, full0 + 8 * s);
            }
            issued = i + 1;
            return true;
        };
        // A_had of the unit's R k-tiles for rows 0..m-1, as fp16(H128 fp16(x * suh) / sqrt(128)), one
        // 128-input block at a time; lane l transforms inputs 4l..4l+3 of a block, which sit in
        // k-tile l/4 at fragment slots kk = 2q + b -> 4q + b, 8 + 2q + b -> 4q + 2 + b
        const int ktl = lane >> 2, kq = lane & 3;
        const int fslot = (kq < 2) ? 8 * kq : 8 * (kq - 2) + 2;
        auto transform = [&](int i) {
            const int u = u0 + i;
            locate(u);
            const int kr0 = (u - sb * ku) * R;
            for (int blk = kr0 >> 3; blk <= (kr0 + R - 1) >> 3; ++blk) {
                const int col = blk * 128 + 4 * lane;
                const int kt = blk * 8 + ktl;  // this lane's k-tile
                const bool mine = kt >= kr0 && kt < kr0 + R;
                const uint2 sr = *reinterpret_cast<const uint2*>(p.suh[si.g] + col);
                uint2 nw = make_uint2(0u, 0u);
                if (p.norm_w) nw = *reinterpret_cast<const uint2*>(p.norm_w + col);
                uint32_t* dst = reinterpret_cast<uint32_t*>(smem + (i % kStages) * S::kStageBytes + S::kTrellisStage +
                                                            (kt - kr0) * m * 32) + (fslot >> 1);
                auto one_row = [&](int row, uint2 xr) {
                    if (p.norm_w) {  // RMSNorm: fp16(fp16(x * s) * w), as exl3b_rmsnorm
                        const float sc = inv_rms[row];
                        const float2 a = __half22float2(u32_as_h2(xr.x)), b = __half22float2(u32_as_h2(xr.y));
                        xr.x = h2_as_u32(__hmul2(__floats2half2_rn(a.x * sc, a.y * sc), u32_as_h2(nw.x)));
                        xr.y = h2_as_u32(__hmul2(__floats2half2_rn(b.x * sc, b.y * sc), u32_as_h2(nw.y)));
                    }
                    const __half2 p01 = __hmul2(u32_as_h2(xr.x), u32_as_h2(sr.x));
                    const __half2 p23 = __hmul2(u32_as_h2(xr.y), u32_as_h2(sr.y));
                    float v[4] = {__low2float(p01), __high2float(p01), __low2float(p23), __high2float(p23)};
                    had128_warp(v);
                    if (mine) {
                        dst[row * 8] = h2_as_u32(__floats2half2_rn(v[0] * kRScale, v[1] * kRScale));
                        dst[row * 8 + 2] = h2_as_u32(__floats2half2_rn(v[2] * kRScale, v[3] * kRScale));
                    }
                };
                if (m == 1) {
                    one_row(0, load_x4(p, 0, col));
                } else {
                    for (int r0 = 0; r0 < m; r0 += 4) {
                        uint2 xg[4];  // four rows' loads in flight together
#pragma unroll
                        for (int i = 0; i < 4; ++i) xg[i] = r0 + i < m ? load_x4(p, r0 + i, col) : make_uint2(0u, 0u);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            if (r0 + i >= m) break;
                            one_row(r0 + i, xg[i]);
                        }
                    }
                }
            }
        };
        bool live = true;
        int published = 0;
        // Only the first two units go out before the wait: every CTA's first unit then arrives
        // ahead of the rest of the ring instead of queueing behind all CTAs' prefetch.
        const int early = min(nunits, 2);
        for (int i = 0; live && i < early; ++i) live = issue(i);
        griddep_wait();  // x may come from the previous kernel
        if (p.norm_w) {
            norm_partials(p, norm_part, warp, lane);
            named_bar(kNormBar, kThreads);
            if (lane < m) {  // warps summed in a fixed order
                float t = 0.f;
                for (int w = 0; w <= kDecodeWarps; ++w) t += norm_part[16 * w + lane];
                inv_rms[lane] = rsqrtf(t / (float)p.k + p.norm_eps);
            }
            __syncwarp();
        }
        for (int i = 0; live && i < nunits; ++i) {
            if (i >= early) live = issue(i);
            if (!live) break;
            transform(i);
            __syncwarp();
            if (lane == 0) mbar_arrive(full0 + 8 * (i % kStages));
            published = i + 1;
        }
        // No copy may still be landing in shared memory when the CTA exits: after an abort, arrive
        // on the stages whose copies were issued but never published (their phase then completes
        // with the copies), and wait (bounded) for the last fill of every stage.  Normally these
        // completed long ago.
        if (lane == 0) {
            if (!live) *abort_flag = 1;
            for (int i = published; i < issued; ++i) mbar_arrive(full0 + 8 * (i % kStages));
            for (int i = max(0, issued - kStages); i < issued; ++i)
                mbar_wait(full0 + 8 * (i % kStages), (i / kStages) & 1, p.err, 2);
        }
        return;
    }

    float* acc_s = reinterpret_cast<float*>(smem + lay.acc_off);
    float* hi_s = reinterpret_cast<float*>(smem + lay.hi_off);

    // ------------------------------ decode warps ------------------------------
    if (p.norm_w) {  // the fused RMSNorm's row sums, shared with the producer
        griddep_wait();
        norm_partials(p, norm_part, warp, lane);
        named_bar(kNormBar, kThreads);
    }
    LaneGeom<K> geom;
    geom.init(lane);
    const int gq = lane >> 2, tq = lane & 3;
    // this warp's first tile (n-tile `warp` of row 0) plus the lane's word offsets; the other
    // tiles of a unit sit at compile-time offsets from these
    uint32_t woff[LaneGeom<K>::kNW];
#pragma unroll
    for (int q = 0; q < LaneGeom<K>::kNW; ++q) woff[q] = (uint32_t)(warp * S::kTile) + geom.off[q];
    const uint32_t boff = (uint32_t)(S::kTrellisStage + gq * 32 + tq * 8);
    const uint32_t mstride = (uint32_t)m * 32;  // A_had bytes per k-tile in a stage

    float acc[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.f;
    // Stage position w + 16 j of a slot holds k-row (slot * q + j / wq) and n-tile (w + 16 (j % wq)) of
    // the super-block, wq = 4 / q: with q = 1 a warp covers four n-tiles of one k-row, with q = 4 one
    // n-tile of four k-rows (acc[j] then hold partial sums of the same columns, folded at the flush).
    const int wq = 4 / q;
    uint32_t jb[4];  // A_had offset of position j's k-row inside its slot
#pragma unroll
    for (int j = 0; j < 4; ++j) jb[j] = (uint32_t)(j / wq) * mstride;
    int sb = u0 / ku;
    SbInfo si = sb_info(p.g, p.groups, sb);
    auto valid_mask = [&](int nt) {
        int v = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (warp + 16 * (j % wq) < nt) v |= 1 << j;
        return v;
    };
    int vmask = valid_mask(si.nblk * 8);  // positions of this warp that hold a tile in this super-block

    // one unit: R0 slots x this warp's four positions (all of them when FULL, else those in vmask)
    auto unit = [&](const uint8_t* st, auto full_tag, auto q1_tag) {
        constexpr bool FULL = decltype(full_tag)::value;
        constexpr bool Q1 = decltype(q1_tag)::value;  // q == 1: one k-row per slot, one B fragment
#pragma unroll
        for (int r = 0; r < R0; ++r) {
            const uint8_t* bs = st + boff + (uint32_t)(r * q) * mstride;
            uint32_t b[MT][2];
            if (Q1) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint2 v = *reinterpret_cast<const uint2*>(bs + mt * 8 * 32);
                    b[mt][0] = v.x;
                    b[mt][1] = v.y;
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (FULL || ((vmask >> j) & 1)) {
                    if (!Q1) {
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            const uint2 v = *reinterpret_cast<const uint2*>(bs + jb[j] + mt * 8 * 32);
                            b[mt][0] = v.x;
                            b[mt][1] = v.y;
                        }
                    }
                    uint32_t Wd[LaneGeom<K>::kNW];
#pragma unroll
                    for (int qq = 0; qq < LaneGeom<K>::kNW; ++qq)
                        Wd[qq] = *reinterpret_cast<const uint32_t*>(st + woff[qq] + r * S::kRowBytes + j * 16 * S::kTile);
                    uint32_t a[4];
                    lane_decode_frag<K, CB>(Wd, geom.phi, a);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) mma_16816_nv(acc[mt][j], a, b[mt][0], b[mt][1]);
                }
            }
        }
    };

    for (int i = 0; i < nunits; ++i) {
        const int s = i % kStages, n = i / kStages;
        // On a wait that gives up, the warps keep walking the units without touching the ring,
        // so every barrier below still sees all of its arrivals.
        const bool ok = mbar_wait_or_abort(full0 + 8 * s, n & 1, p.err, 3, abort_flag);
        if (__all_sync(0xFFFFFFFFu, ok)) {
            const uint8_t* st = smem + s * S::kStageBytes;
            // the unguarded copy only where registers allow it (one m-tile)
            if (MT == 1 && vmask == 0xF) {
                if (q == 1) unit(st, std::true_type{}, std::true_type{});
                else unit(st, std::true_type{}, std::false_type{});
            } else if (vmask) {
                if (q == 1) unit(st, std::false_type{}, std::true_type{});
                else unit(st, std::false_type{}, std::false_type{});
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);

        const int u = u0 + i;
        const bool sb_end = (u + 1) % ku == 0 || i == nunits - 1;
        if (!sb_end) continue;

        // ---------------- pool the finished super-block, then one warp per column block ----------------
        griddep_wait();  // the workspace counters and y may still belong to the previous kernel
        named_bar(kFlushBar, kDecodeWarps * 32);  // the previous flush's readers are done with acc_s
        // positions j and j + wq hold the same columns when q > 1: fold them, in a fixed order
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (q >= 2) {
                    acc[mt][0][e] += acc[mt][2][e];
                    acc[mt][1][e] += acc[mt][3][e];
                }
                if (q == 4) acc[mt][0][e] += acc[mt][1][e];
            }
        // fragment -> acc_s[row][col]: lane (gq, tq) holds D[col gq (+8)][rows 2tq, 2tq+1] of n-tile
        // warp + 16 j, j < wq
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < wq && ((vmask >> j) & 1)) {
                    const int col = (warp + 16 * j) * 16 + gq;
                    const int r0 = 8 * mt + 2 * tq;
                    if (r0 < m) {
                        acc_s[r0 * kAccCols + col] = acc[mt][j][0];
                        acc_s[r0 * kAccCols + col + 8] = acc[mt][j][2];
                    }
                    if (r0 + 1 < m) {
                        acc_s[(r0 + 1) * kAccCols + col] = acc[mt][j][1];
                        acc_s[(r0 + 1) * kAccCols + col + 8] = acc[mt][j][3];
                    }
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.f;
            }
        if (threadIdx.x == 0) *flush_snap = *abort_flag;  // both warps of a pair must agree to enter
        named_bar(kFlushBar, kDecodeWarps * 32);
        {
            const int fb = warp & 7, half = warp >> 3;
            if (fb < si.nblk && *flush_snap == 0)
                flush_block<MT>(p, acc_s, hi_s, abort_flag, c, sb, si, fb, half, u0, u1, lane, fin_s + fb);
        }
        if (i + 1 < nunits) {
            ++sb;
            si = sb_info(p.g, p.groups, sb);
            vmask = valid_mask(si.nblk * 8);
        }
    }
    if (p.tp_size > 1) {
        // the last CTA of the grid to get here advances this rank's call counter: every CTA read
        // it (in its flushes) before arriving, and the next call reads it after griddepcontrol.wait
        named_bar(kFlushBar, kDecodeWarps * 32);
        if (threadIdx.x == 0) {
            int* hdr = reinterpret_cast<int*>(p.tp_buf[p.tp_rank]);
            __threadfence();
            if (atomicAdd(hdr + 1, 1) == P - 1) {
                hdr[1] = 0;
                __threadfence();
                atomicAdd(hdr, 1);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// decode ceiling: the GEMV's per-tile work (trellis words from shared memory, window extraction,
// codebook decode into mma A fragments, one m16n8k16 per tile) with no HBM traffic and no stage
// hand-offs, over one resident stage of 8 k-rows x 64 tiles, `iters` times.  It bounds the rate at
// which this decode can feed the tensor core, in tiles per second.
// ---------------------------------------------------------------------------------------------
#ifndef EXL3B_CEIL_ROWS
#define EXL3B_CEIL_ROWS 8
#endif
#ifndef EXL3B_CEIL_CTAS_PER_SM
#define EXL3B_CEIL_CTAS_PER_SM 1
#endif
constexpr int kCeilRows = EXL3B_CEIL_ROWS;  // k-rows of the resident stage (the GEMV's units: 8)
template <int K, int CB>
__global__ void __launch_bounds__(kDecodeWarps * 32, 1)
decode_ceiling_kernel(const uint16_t* trellis, int iters, int zero, float* out) {
    constexpr int kTile = 32 * K, kRowBytes = kSbTiles * kTile;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    {
        const uint4* src = reinterpret_cast<const uint4*>(trellis);
        uint4* dst = reinterpret_cast<uint4*>(smem);
        for (int i = threadIdx.x; i < kCeilRows * kRowBytes / 16; i += blockDim.x) dst[i] = src[i];
        // B fragments (A_had of one k-tile, 8 rows): fp16 1/8
        uint32_t* bf = reinterpret_cast<uint32_t*>(smem + kCeilRows * kRowBytes);
        for (int i = threadIdx.x; i < kCeilRows * 64; i += blockDim.x) bf[i] = 0x30003000u;
    }
    __syncthreads();
    LaneGeom<K> geom;
    geom.init(lane);
    uint32_t woff[LaneGeom<K>::kNW];
#pragma unroll
    for (int q = 0; q < LaneGeom<K>::kNW; ++q) woff[q] = (uint32_t)(warp * kTile) + geom.off[q];
    const uint32_t boff = (uint32_t)(kCeilRows * kRowBytes + (lane >> 2) * 32 + (lane & 3) * 8);
    float acc[4][4] = {};
#pragma unroll 1
    for (int it = 0; it < iters; ++it) {
        // `zero` is 0 at run time; an offset the compiler cannot see through keeps every load (and
        // the decode of what it loads) inside the loop, as in the GEMV, where each unit is new data
        const uint8_t* st = smem + (uint32_t)(it & zero) * 16u;
#pragma unroll
        for (int r = 0; r < kCeilRows; ++r) {
            const uint2 b = *reinterpret_cast<const uint2*>(st + boff + r * 256);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t Wd[LaneGeom<K>::kNW];
#pragma unroll
                for (int qq = 0; qq < LaneGeom<K>::kNW; ++qq)
                    Wd[qq] = *reinterpret_cast<const uint32_t*>(st + woff[qq] + r * kRowBytes + j * 16 * kTile);
                uint32_t a[4];
                lane_decode_frag<K, CB>(Wd, geom.phi, a);
                mma_16816_nv(acc[j], a, b.x, b.y);
            }
        }
    }
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) t += acc[j][0] + acc[j][1] + acc[j][2] + acc[j][3];
    out[(blockIdx.x * kDecodeWarps + warp) * 32 + lane] = t;
}

template <int K, int CB>
static cudaError_t launch_ceiling(const uint16_t* trellis, int iters, float* out, int ctas, cudaStream_t st) {
    const int bytes = kCeilRows * kSbTiles * 32 * K + kCeilRows * 256;
    auto kern = decode_ceiling_kernel<K, CB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    kern<<<ctas, kDecodeWarps * 32, bytes, st>>>(trellis, iters, 0, out);
    return cudaGetLastError();
}

template <int CB>
static cudaError_t launch_ceiling_k(int K, const uint16_t* trellis, int iters, float* out, int ctas, cudaStream_t st) {
    switch (K) {
        case 1: return launch_ceiling<1, CB>(trellis, iters, out, ctas, st);
        case 2: return launch_ceiling<2, CB>(trellis, iters, out, ctas, st);
        case 3: return launch_ceiling<3, CB>(trellis, iters, out, ctas, st);
        case 4: return launch_ceiling<4, CB>(trellis, iters, out, ctas, st);
        case 5: return launch_ceiling<5, CB>(trellis, iters, out, ctas, st);
        case 6: return launch_ceiling<6, CB>(trellis, iters, out, ctas, st);
        case 7: return launch_ceiling<7, CB>(trellis, iters, out, ctas, st);
        default: return launch_ceiling<8, CB>(trellis, iters, out, ctas, st);
    }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
constexpr size_t kHeaderBytes = 256;  // error word at 0, slot ticket counter at kTicketOffset
constexpr size_t kTicketOffset = 128;
// Counter region of fixed size (one int per global 128-column block, up to kMaxBlocks), so that
// calls of any shape find their counters at the same zeroed place.
constexpr int kMaxBlocks = 8192;
constexpr size_t kCounterBytes = 4 * (size_t)kMaxBlocks;

static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static int num_sms() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!sms[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = v > 0 ? v : 148;
    }
    return sms[dev];
}

// Stream-K width: one CTA per SM, independent of m and codebook, so the partition (and therefore
// every rounding) depends only on the layer shape and K.
static int gemv_ctas(int units) { return std::min(units, num_sms()); }

// Super-blocks of one group: its 128-column blocks split as evenly as possible into runs of at
// most `maxb` (8 / q: 1024, 512 or 256 columns).
static void split_super_blocks(int blocks, int maxb, int& count, int& base, int& extra) {
    count = (blocks + maxb - 1) / maxb;
    base = blocks / count;
    extra = blocks % count;
}

struct Partition {
    int r0, q, ku, units, ctas, sb_cols, super_blocks;
};

// The widest super-blocks (smallest q) that still give every column block at most about eight
// CTAs to reduce over: narrow layers (o, down, k/v) get 256- or 512-column super-blocks with more
// k-rows per unit, so that their cross-CTA sums stay short.  Depends on the shape and K only.
static Partition partition(int k, int K, int groups, const int* n, int r0) {
    const int kt = k / 16;
    Partition q = {};
    q.r0 = r0;
    for (int qq : {1, 2, 4}) {
        if (kt % (r0 * qq) || r0 * qq > kMaxUnitRows) break;  // rows per unit must divide k / 16
        Partition t = {};
        t.r0 = r0;
        t.q = qq;
        t.ku = kt / (r0 * qq);
        int widest = 0;
        for (int g = 0; g < groups; ++g) {
            int cnt, base, extra;
            split_super_blocks(n[g] / 128, 8 / qq, cnt, base, extra);
            t.super_blocks += cnt;
            widest = std::max(widest, base + (extra ? 1 : 0));
        }
        t.sb_cols = widest * 128;
        t.units = t.super_blocks * t.ku;
        t.ctas = gemv_ctas(std::max(t.units, 1));
        q = t;
        if (t.super_blocks * 8 >= num_sms()) break;
    }
    return q;
}

// Rows per unit slot: 8 (fewer unit hand-offs) at K <= 4 unless units of 2 balance the CTAs clearly
// better (small layers and tensor-parallel shards, whose few large units would leave SMs idle: an
// o shard at TP 8 has 25 units of 8 rows for 148 SMs).  Cost: the busiest CTA's units x (their
// k-rows + half a row of hand-off); units of 2 must cost under 0.8x, since a marginal gain measured
// as a loss inside a chain of launches (the full o at M = 1: 26.5 us alone with units of 2 against
// 27.5, but its layer step 122.2 against 119.6 us).  Depends on the shape and K only, never on m.
static Partition choose_partition(int k, int K, int groups, const int* n) {
    const Partition a = partition(k, K, groups, n, rows_per_unit(K));
    if (rows_per_unit(K) == 2) return a;
    const Partition b = partition(k, K, groups, n, 2);
    auto cost = [](const Partition& t) {
        return (double)((t.units + t.ctas - 1) / std::max(t.ctas, 1)) * (t.r0 + 0.5);
    };
    return cost(b) < 0.8 * cost(a) ? b : a;
}

struct WsLayout {
    size_t counters, partials, stage, total;
};

// stage_cols: columns of the SwiGLU staging area (both groups), 0 without the activation
static WsLayout ws_layout(int m, int k, int groups, const Partition& q, int64_t stage_cols) {
    WsLayout L;
    L.counters = kHeaderBytes;
    L.partials = round_up(L.counters + kCounterBytes, 256);
    L.stage = round_up(L.partials + (size_t)(q.ctas + q.super_blocks - 1) * m * q.sb_cols * 4, 256);
    L.total = round_up(L.stage + (size_t)m * stage_cols * 2, 256);
    return L;
}

// The workspace bytes a one-group call of this shape really uses (the partition its launch takes),
// for callers whose scratch has a fixed size.  k, n multiples of 128, 1 <= K <= 8.
size_t linear_workspace_exact(int m, int k, int n, int K) {
    const int nn[1] = {n};
    return ws_layout(m, k, 1, choose_partition(k, K, 1, nn), 0).total;
}

template <int K, int CB, int MT, int R0>
static cudaError_t launch_gemv(const GemvParams& p, cudaStream_t st) {
    using S = GemvSmem<K, MT, R0>;
    auto kern = gemv_kernel<K, CB, MT, R0>;
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    static cudaError_t attr_err[64];
    std::call_once(once[dev & 63], [&] {  // the budget covers every m
        attr_err[dev & 63] =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBudget);
    });
    if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = gemv_layout<K, MT, R0>(p.m).total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int CB, int MT>
static cudaError_t launch_gemv_k(int K, int r0, const GemvParams& p, cudaStream_t st) {
    const bool r2 = r0 == 2;  // K <= 4 has units of kR0SmallK or 2 rows per slot, K > 4 of 2
    constexpr int RS = kR0SmallK;
    switch (K) {
        case 1: return r2 ? launch_gemv<1, CB, MT, 2>(p, st) : launch_gemv<1, CB, MT, RS>(p, st);
        case 2: return r2 ? launch_gemv<2, CB, MT, 2>(p, st) : launch_gemv<2, CB, MT, RS>(p, st);
        case 3: return r2 ? launch_gemv<3, CB, MT, 2>(p, st) : launch_gemv<3, CB, MT, RS>(p, st);
        case 4: return r2 ? launch_gemv<4, CB, MT, 2>(p, st) : launch_gemv<4, CB, MT, RS>(p, st);
        case 5: return launch_gemv<5, CB, MT, 2>(p, st);
        case 6: return launch_gemv<6, CB, MT, 2>(p, st);
        case 7: return launch_gemv<7, CB, MT, 2>(p, st);
        default: return launch_gemv<8, CB, MT, 2>(p, st);
    }
}

int linear_impl(const uint16_t* x, int m, int k, int groups, const uint16_t* const* trellis, const int* n,
                int K, int codebook, const uint16_t* const* suh, const uint16_t* const* svh, uint16_t* const* y,
                int64_t ldy, void* workspace, size_t ws_bytes, void* stream, const exl3b_tp_comm* comm,
                const uint16_t* norm_w, float norm_eps) {
    const bool x_bf16 = (codebook & EXL3B_X_BF16) != 0;
    const bool act = (codebook & EXL3B_ACT_SILU_MUL) != 0;
    const bool y_add = (codebook & EXL3B_Y_ADD) != 0;
    codebook &= ~(EXL3B_X_BF16 | EXL3B_ACT_SILU_MUL | EXL3B_Y_ADD);
    if (K < 1 || K > 8 || codebook < 0 || codebook > 2) return EXL3B_DECLINED;
    if (act && (groups != 2 || !n || n[0] != n[1] || comm || y_add)) return EXL3B_DECLINED;
    if (m < 1 || m > EXL3B_GEMV_MAX_ROWS || groups < 1 || groups > EXL3B_MAX_GROUPS) return EXL3B_DECLINED;
    if (k <= 0 || k % 128) return EXL3B_DECLINED;
    if (!x || !trellis || !n || !suh || !svh || !y || !workspace) return EXL3B_BAD_ARG;
    if (!aligned(x, 8) || k % 4 || ldy % 4 || !aligned(workspace, 256)) return EXL3B_BAD_ARG;
    if (norm_w && (!aligned(norm_w, 8) || !(norm_eps >= 0.f))) return EXL3B_BAD_ARG;
    if (norm_w && k > kNormChunks * 4 * kThreads) return EXL3B_DECLINED;
    int64_t n_total = 0;
    for (int g = 0; g < groups; ++g) {
        if (n[g] <= 0 || n[g] % 128) return EXL3B_DECLINED;
        if (ldy < n[g]) return EXL3B_BAD_ARG;
        const uint16_t* yg = act ? y[0] : y[g];  // the activation has one output
        if (!trellis[g] || !suh[g] || !svh[g] || !yg) return EXL3B_BAD_ARG;
        if (!aligned(trellis[g], 16) || !aligned(suh[g], 8) || !aligned(svh[g], 8) || !aligned(yg, 8))
            return EXL3B_BAD_ARG;
        n_total += n[g];
    }
    // per-block counters, then (act) one pair counter per column block of a group
    if ((n_total + (act ? n[0] : 0)) / 128 > kMaxBlocks) return EXL3B_DECLINED;
    if (comm) {
        if (groups != 1 || comm->tp_size < 2 || comm->tp_size > EXL3B_MAX_TP || comm->tp_rank < 0 ||
            comm->tp_rank >= comm->tp_size || n[0] / 128 > comm->max_blocks || m > comm->max_rows)
            return EXL3B_BAD_ARG;
        for (int r = 0; r < comm->tp_size; ++r)
            if (!comm->buffers[r] || !aligned(comm->buffers[r], 256)) return EXL3B_BAD_ARG;
    }
    const Partition q = choose_partition(k, K, groups, n);
    const WsLayout L = ws_layout(m, k, groups, q, act ? n_total : 0);
    if (ws_bytes < L.total) return EXL3B_WORKSPACE;

    cudaStream_t st = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);

    GemvParams p = {};
    int blk = 0, sbs = 0;
    for (int g = 0; g < groups; ++g) {
        p.suh[g] = reinterpret_cast<const __half*>(suh[g]);
        p.g.trellis[g] = trellis[g];
        p.g.svh[g] = reinterpret_cast<const __half*>(svh[g]);
        p.g.y[g] = reinterpret_cast<__half*>(act ? y[0] : y[g]);
        p.g.n_tiles[g] = n[g] / 16;
        p.g.blk_prefix[g] = blk;
        p.g.sb_prefix[g] = sbs;
        int cnt, base, extra;
        split_super_blocks(n[g] / 128, 8 / q.q, cnt, base, extra);
        p.g.sb_base[g] = base;
        p.g.sb_extra[g] = extra;
        blk += n[g] / 128;
        sbs += cnt;
    }
    p.g.blk_prefix[groups] = blk;
    p.g.sb_prefix[groups] = sbs;
    p.x = x;
    p.x_bf16 = x_bf16 ? 1 : 0;
    p.partials = reinterpret_cast<float*>(ws + L.partials);
    p.counters = reinterpret_cast<int*>(ws + L.counters);
    p.err = reinterpret_cast<int*>(ws);
    p.ticket = reinterpret_cast<unsigned long long*>(ws + kTicketOffset);
    p.groups = groups;
    p.m = m;
    p.k = k;
    p.kt = k / 16;
    p.ku = q.ku;
    p.q = q.q;
    p.units = q.units;
    p.ctas = q.ctas;
    p.sb_cols = q.sb_cols;
    p.ldy = ldy;
    p.y_add = y_add ? 1 : 0;
    p.norm_w = reinterpret_cast<const __half*>(norm_w);
    p.norm_eps = norm_eps;
    p.act = act ? 1 : 0;
    p.stage = reinterpret_cast<__half*>(ws + L.stage);
    p.act_ctr = blk;
    p.tp_size = comm ? comm->tp_size : 1;
    if (comm) {
        p.tp_rank = comm->tp_rank;
        p.tp_blocks = comm->max_blocks;
        p.tp_rows = comm->max_rows;
        for (int r = 0; r < comm->tp_size; ++r) p.tp_buf[r] = static_cast<uint8_t*>(comm->buffers[r]);
    }

    cudaError_t e;
    const bool mt2 = m > 8;
    switch (codebook) {
        case 0: e = mt2 ? launch_gemv_k<0, 2>(K, q.r0, p, st) : launch_gemv_k<0, 1>(K, q.r0, p, st); break;
        case 1: e = mt2 ? launch_gemv_k<1, 2>(K, q.r0, p, st) : launch_gemv_k<1, 1>(K, q.r0, p, st); break;
        default: e = mt2 ? launch_gemv_k<2, 2>(K, q.r0, p, st) : launch_gemv_k<2, 1>(K, q.r0, p, st); break;
    }
    return cuda_status(e);
}

}  // namespace exl3b

using namespace exl3b;

extern "C" size_t exl3b_linear_workspace_bytes(int m, int k, int groups, int64_t n_total) {
    if (m < 1 || k < 128 || groups < 1 || n_total < 128) return 0;
    // an upper bound over every K and every split of n_total into `groups` widths
    const int64_t blocks = n_total / 128;
    Partition q = {};
    q.super_blocks = (int)std::min<int64_t>(blocks, (blocks + 1) / 2 + groups - 1);  // q = 4: 2 blocks each
    q.sb_cols = (int)std::min<int64_t>(blocks, 8) * 128;
    q.ctas = (int)std::min<int64_t>(num_sms(), (int64_t)q.super_blocks * ((k / 16) / rows_per_unit(8)));
    // two groups may carry the SwiGLU epilogue, which stages both outputs
    return ws_layout(m, k, groups, q, groups == 2 ? n_total : 0).total;
}

extern "C" int exl3b_linear_supported(int m, int k, int n, int K, int codebook) {
    // the shape rules of linear_impl for one group, without touching a device
    const int flags = EXL3B_X_BF16 | EXL3B_Y_ADD;  // the flags that do not change the shape rules
    codebook &= ~flags;
    return (m >= 1 && m <= EXL3B_GEMV_MAX_ROWS && k > 0 && k % 128 == 0 && n > 0 && n % 128 == 0 &&
            n / 128 <= kMaxBlocks && K >= 1 && K <= 8 && codebook >= 0 && codebook <= 2) ? 1 : 0;
}

extern "C" int exl3b_linear(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K, int codebook,
                            const uint16_t* suh, const uint16_t* svh, uint16_t* y, int64_t ldy, void* workspace,
                            size_t workspace_bytes, void* stream) {
    const uint16_t* tr[1] = {trellis};
    const uint16_t* su[1] = {suh};
    const uint16_t* sv[1] = {svh};
    uint16_t* yy[1] = {y};
    int nn[1] = {n};
    return linear_impl(x, m, k, 1, tr, nn, K, codebook, su, sv, yy, ldy, workspace, workspace_bytes, stream, nullptr,
                       nullptr, 0.f);
}

extern "C" int exl3b_linear_grouped(const uint16_t* x, int m, int k, int groups, const uint16_t* const* trellis,
                                    const int* n, int K, int codebook, const uint16_t* const* suh,
                                    const uint16_t* const* svh, uint16_t* const* y, int64_t ldy, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    return linear_impl(x, m, k, groups, trellis, n, K, codebook, suh, svh, y, ldy, workspace, workspace_bytes,
                       stream, nullptr, nullptr, 0.f);
}

extern "C" int exl3b_linear_grouped_rmsnorm(const uint16_t* x, int m, int k, int groups,
                                            const uint16_t* const* trellis, const int* n, int K, int codebook,
                                            const uint16_t* norm_weight, float eps, const uint16_t* const* suh,
                                            const uint16_t* const* svh, uint16_t* const* y, int64_t ldy,
                                            void* workspace, size_t workspace_bytes, void* stream) {
    if (!norm_weight) return EXL3B_BAD_ARG;
    return linear_impl(x, m, k, groups, trellis, n, K, codebook, suh, svh, y, ldy, workspace, workspace_bytes,
                       stream, nullptr, norm_weight, eps);
}

extern "C" size_t exl3b_tp_comm_bytes(int tp_size, int max_blocks, int max_rows) {
    if (tp_size < 2 || tp_size > EXL3B_MAX_TP || max_blocks < 1 || max_rows < 1 || max_rows > EXL3B_GEMV_MAX_ROWS)
        return 0;
    return tp_comm_bytes(tp_size, max_blocks, max_rows);
}

// Base of the allocation holding p, through the driver's cuMemGetAddressRange looked up at run
// time (the library does not link the driver, so that it loads on machines without one).
static bool allocation_base(const void* p, CUdeviceptr* base) {
    using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(f);
    });
    size_t size = 0;
    return fn && fn(base, &size, (CUdeviceptr)p) == CUDA_SUCCESS;
}

// The handle names the whole allocation; the offset of dev_ptr inside it travels alongside.
extern "C" int exl3b_ipc_get_handle(const void* dev_ptr, void* handle) {
    if (!dev_ptr || !handle) return EXL3B_BAD_ARG;
    CUdeviceptr base = 0;
    if (!allocation_base(dev_ptr, &base)) return EXL3B_BAD_ARG;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_status(e);
    const int64_t off = (int64_t)((CUdeviceptr)dev_ptr - base);
    static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(int64_t) == EXL3B_IPC_HANDLE_BYTES, "handle layout");
    memcpy(handle, &h, sizeof(h));
    memcpy(static_cast<uint8_t*>(handle) + sizeof(h), &off, sizeof(off));
    return EXL3B_OK;
}

extern "C" int exl3b_ipc_open_handle(const void* handle, void** dev_ptr) {
    if (!handle || !dev_ptr) return EXL3B_BAD_ARG;
    cudaIpcMemHandle_t h;
    int64_t off = 0;
    memcpy(&h, handle, sizeof(h));
    memcpy(&off, static_cast<const uint8_t*>(handle) + sizeof(h), sizeof(off));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_status(e);
    *dev_ptr = static_cast<uint8_t*>(base) + off;
    return EXL3B_OK;
}

extern "C" int exl3b_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return EXL3B_BAD_ARG;
    CUdeviceptr base = 0;
    if (!allocation_base(dev_ptr, &base)) return EXL3B_BAD_ARG;
    return cuda_status(cudaIpcCloseMemHandle(reinterpret_cast<void*>(base)));
}

extern "C" int exl3b_linear_tp(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K, int codebook,
                               const uint16_t* suh, const uint16_t* svh, uint16_t* y, int64_t ldy, void* workspace,
                               size_t workspace_bytes, const exl3b_tp_comm* comm, void* stream) {
    if (!comm) return EXL3B_BAD_ARG;
    const uint16_t* tr[1] = {trellis};
    const uint16_t* su[1] = {suh};
    const uint16_t* sv[1] = {svh};
    uint16_t* yy[1] = {y};
    int nn[1] = {n};
    return linear_impl(x, m, k, 1, tr, nn, K, codebook, su, sv, yy, ldy, workspace, workspace_bytes, stream, comm,
                       nullptr, 0.f);
}

extern "C" int exl3b_linear_workspace_error(const void* workspace, int* out, void* stream) {
    if (!workspace || !out) return EXL3B_BAD_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyAsync(out, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return cuda_status(e);
}

extern "C" int exl3b_decode_ceiling(int K, int codebook, const uint16_t* trellis, int iters, float* out,
                                    int* ctas, void* stream) {
    if (K < 1 || K > 8 || codebook < 0 || codebook > 2 || iters < 1) return EXL3B_DECLINED;
    if (!trellis || !out || !ctas || !aligned(trellis, 16) || !aligned(out, 4)) return EXL3B_BAD_ARG;
    *ctas = num_sms() * EXL3B_CEIL_CTAS_PER_SM;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    switch (codebook) {
        case 0: e = launch_ceiling_k<0>(K, trellis, iters, out, *ctas, st); break;
        case 1: e = launch_ceiling_k<1>(K, trellis, iters, out, *ctas, st); break;
        default: e = launch_ceiling_k<2>(K, trellis, iters, out, *ctas, st); break;
    }
    return cuda_status(e);
}
