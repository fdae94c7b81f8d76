// The EXL3 linear for 1 <= m <= 16 rows (decode and speculative verify), fused end to end:
//
//   launch 1  had_in:  A_had = fp16(H128 * fp16(x * suh) / sqrt(128))  -> workspace, stored in the
//                      mma B-fragment order, block-major [group][k/128][m][kAhadRow halves]
//   launch 2  gemv:    stream-K over units of (128 output columns x 128 inputs); a producer warp
//                      streams trellis rows and A_had blocks into a shared-memory ring of up to 8
//                      stages with bulk async copies (no multicast); eight consumer warps decode the
//                      trellis in registers straight into mma.m16n8k16 A fragments (W^T x A_had^T,
//                      fp32 accumulate) and hand each finished column block to an epilogue warp,
//                      which reduces it across the CTAs that shared it (partials in the workspace,
//                      fixed summation order, last arriver finishes) and applies had_out + svh.
//   Launch 2 is a programmatic dependent launch: its trellis copies start while launch 1 runs.
//
// Reference semantics: reference/exl3_oracle.py:307-351 (gemv_mul1, all codebooks);
// kernels replaced: exl3_gemm / exl3_gemv_mr / exl3_mgemm / exl3_gemv_mr_grouped of the fork
// (vllm_plugin/exl3rocm/ops.py:80-85,134-170; 0002-gemv-multirow.patch:79-88 for the rule that
// every row equals the m = 1 result bit for bit: here the work partition depends only on
// (k, n, groups) and each mma column is one input row, so rows never interact).
#include <algorithm>
#include <mutex>

#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kConsumerWarps = 8;  // warp w: n-tiles 2(w%4), 2(w%4)+1; k-tiles 4(w/4)..+3 of a unit
constexpr int kThreads = (kConsumerWarps + 2) * 32;  // + producer warp + epilogue warp
// One A_had row of a unit: 8 k-tiles x 16 fp16 in B-fragment order (256 B) + 32 B of padding, so
// that the eight rows a warp reads at once fall in distinct banks.
constexpr int kAhadRow = 144;  // halves

struct GemvGroups {
    const uint16_t* trellis[EXL3B_MAX_GROUPS];
    const __half* svh[EXL3B_MAX_GROUPS];
    __half* y[EXL3B_MAX_GROUPS];
    int n_tiles[EXL3B_MAX_GROUPS];
    int blk_prefix[EXL3B_MAX_GROUPS + 1];  // first global column block of each group
};

struct GemvParams {
    GemvGroups g;
    const __half* a_had;  // workspace
    float* partials;      // workspace: [2 * P][m][128]
    int* counters;        // workspace: one per global column block
    int* err;             // workspace error word
    int groups, m, nk;    // nk = k / 128
    int units, ctas;      // U = total column blocks * nk, P
    int64_t ldy;
};

struct HadInParams {
    const __half* suh[EXL3B_MAX_GROUPS];
};

// ---------------------------------------------------------------------------------------------
// launch 1: input transform, one warp per (row, k-block, group)
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) had_in_kernel(const __half* __restrict__ x, int m, int k,
                                                     const __grid_constant__ HadInParams p,
                                                     __half* __restrict__ a_had) {
    griddep_launch();
    const int row = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x, g = blockIdx.y, nk = k >> 7;
    if (row >= m) return;
    const int c = j * 128 + 4 * lane;
    const uint2 xr = *reinterpret_cast<const uint2*>(x + (int64_t)row * k + c);
    const uint2 sr = *reinterpret_cast<const uint2*>(p.suh[g] + c);
    const __half2 p01 = __hmul2(u32_as_h2(xr.x), u32_as_h2(sr.x));
    const __half2 p23 = __hmul2(u32_as_h2(xr.y), u32_as_h2(sr.y));
    float v[4] = {__low2float(p01), __high2float(p01), __low2float(p23), __high2float(p23)};
    had128_warp(v);
    const uint32_t h01 = h2_as_u32(__floats2half2_rn(v[0] * kRScale, v[1] * kRScale));
    const uint32_t h23 = h2_as_u32(__floats2half2_rn(v[2] * kRScale, v[3] * kRScale));
    // element e = 4*lane + s lives in k-tile e/16 at fragment slot of kk = e%16:
    // kk = 2q + b -> 4q + b (kk < 8);  kk = 8 + 2q + b -> 4q + 2 + b
    const int kt = lane >> 2, kq = lane & 3;
    const int base = (kq < 2) ? 8 * kq : 8 * (kq - 2) + 2;
    uint32_t* dst = reinterpret_cast<uint32_t*>(
        a_had + ((int64_t)(g * nk + j) * m + row) * kAhadRow + kt * 16);
    dst[base >> 1] = h01;
    dst[(base + 4) >> 1] = h23;
}

// ---------------------------------------------------------------------------------------------
// stream-K partition helpers (64-bit: U * P fits easily)
// ---------------------------------------------------------------------------------------------
EXL3B_DEV int unit_start(int c, int U, int P) { return (int)(((int64_t)c * U) / P); }
EXL3B_DEV int cta_of_unit(int u, int U, int P) { return (int)((((int64_t)u + 1) * P - 1) / U); }

// slot of CTA c's partial for global block B: 0 if B is the block its range starts in, else 1
EXL3B_DEV int partial_slot(int c, int B, int nk, int U, int P) {
    return 2 * c + ((unit_start(c, U, P) / nk) == B ? 0 : 1);
}

EXL3B_DEV int group_of_block(const GemvGroups& gg, int groups, int B) {
    int g = 0;
    while (g + 1 < groups && B >= gg.blk_prefix[g + 1]) ++g;
    return g;
}

// ---------------------------------------------------------------------------------------------
// launch 2: the stream-K decode GEMV
// ---------------------------------------------------------------------------------------------
// Shared memory per CTA: a ring of kStages stages (one unit each: 8 trellis rows + the unit's
// A_had rows, MT*8 rows of kAhadRow halves, rows >= m zero), a double-buffered fp32 accumulator
// tile [2 buffers][2 k-halves][MT*8 rows][128] handed from the consumers to the epilogue warp,
// and the mbarriers.  kStages is chosen so that two CTAs fit on an SM.
template <int K, int MT>
struct GemvSmem {
    static constexpr int kTrellisStage = 2048 * K;  // 8 k-tiles x 8 n-tiles x 32K bytes
    static constexpr int kRows = 8 * MT;
    static constexpr int kAhadBytes = kRows * kAhadRow * 2;
    static constexpr int kStageBytes = kTrellisStage + kAhadBytes;
    static constexpr int kAccBuf = 2 * kRows * 128 * 4;  // two k-halves
    static constexpr int kAccBytes = 2 * kAccBuf;
    static constexpr int kBudget = 110 * 1024;
    static constexpr int kStages0 = (kBudget - kAccBytes - 256) / kStageBytes;
    static constexpr int kStages = kStages0 > 8 ? 8 : (kStages0 < 2 ? 2 : kStages0);
    static constexpr int kAccOffset = kStages * kStageBytes;
    static constexpr int kBarOffset = kAccOffset + kAccBytes;  // full[S], empty[S], accf[2], acce[2]
    static constexpr int kFlagOffset = kBarOffset + (2 * kStages + 4) * 8;
    static constexpr int kTotal = kFlagOffset + 16;
};

constexpr int kProducerWarp = kConsumerWarps;
constexpr int kEpilogueWarp = kConsumerWarps + 1;

template <int K, int CB, int MT>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
    using S = GemvSmem<K, MT>;
    constexpr int kStages = S::kStages;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full0 = sbase + S::kBarOffset, empty0 = full0 + kStages * 8;
    const uint32_t accf0 = empty0 + kStages * 8, acce0 = accf0 + 16;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::kFlagOffset);

    const int c = blockIdx.x, P = p.ctas, U = p.units, nk = p.nk, m = p.m;
    const int u0 = unit_start(c, U, P), u1 = unit_start(c + 1, U, P);
    const int nunits = u1 - u0;

    // A_had rows m..kRows-1 are never written by the copies: zero them once so the consumers'
    // B fragments read zeros there without predicates
    {
        const int zero_words = (S::kRows - m) * kAhadRow / 2;
        for (int s = 0; s < kStages; ++s) {
            uint32_t* z = reinterpret_cast<uint32_t*>(smem + s * S::kStageBytes + S::kTrellisStage + m * kAhadRow * 2);
            for (int i = threadIdx.x; i < zero_words; i += kThreads) z[i] = 0u;
        }
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kConsumerWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accf0 + 8 * b, kConsumerWarps);
            mbar_init(acce0 + 8 * b, 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        // ------------------------------ producer warp ------------------------------
        const uint32_t ahad_bytes = (uint32_t)m * kAhadRow * 2;
        bool waited_dep = false;
        int issued = 0;
        int B = u0 / nk, j = u0 % nk;
        int g = group_of_block(p.g, p.groups, B);
        for (int i = 0; i < nunits; ++i) {
            const int s = i % kStages, n = i / kStages;
            bool ok = true;
            if (n > 0) ok = mbar_wait(empty0 + 8 * s, (n - 1) & 1, p.err, 1);
            if (!ok) *abort_flag = 1;
            if (__any_sync(0xFFFFFFFFu, *abort_flag != 0)) break;
            const int b = B - p.g.blk_prefix[g];
            const uint32_t st = sbase + s * S::kStageBytes;
            if (lane == 0) mbar_arrive_expect_tx(full0 + 8 * s, S::kTrellisStage + ahad_bytes);
            __syncwarp();
            if (lane < 8) {
                const uint16_t* src = p.g.trellis[g] + ((int64_t)(j * 8 + lane) * p.g.n_tiles[g] + b * 8) * (16 * K);
                bulk_g2s(st + lane * (256 * K), src, 256 * K, full0 + 8 * s);
            } else if (lane == 8) {
                if (!waited_dep) { griddep_wait(); waited_dep = true; }
                const __half* src = p.a_had + (int64_t)(g * nk + j) * m * kAhadRow;
                bulk_g2s(st + S::kTrellisStage, src, ahad_bytes, full0 + 8 * s);
            }
            issued = i + 1;
            if (++j == nk) {
                j = 0;
                ++B;
                if (g + 1 < p.groups && B >= p.g.blk_prefix[g + 1]) ++g;
            }
        }
        // No copy may still be landing in shared memory when the CTA exits: wait (bounded) for
        // the last fill of every stage.  Normally these completed long ago.
        if (lane == 0)
            for (int i = max(0, issued - kStages); i < issued; ++i)
                mbar_wait(full0 + 8 * (i % kStages), (i / kStages) & 1, p.err, 2);
        return;
    }

    float* acc_s = reinterpret_cast<float*>(smem + S::kAccOffset);

    if (warp == kEpilogueWarp) {
        // ------------------------------ epilogue warp ------------------------------
        // Walks the same column blocks the consumers flush, in the same order.  For each: sum the
        // two k-halves; if this CTA covered the whole block, transform and store; otherwise
        // publish the partial and, if it is the last of the block's CTAs to arrive, gather all
        // partials in fixed CTA order and finish the block.
        const int B_first = u0 / nk, B_last = (u1 - 1) / nk;
        const int col = 4 * lane;
        for (int Bc = B_first, f = 0; Bc <= B_last; ++Bc, ++f) {
            const int fb = f & 1;
            bool ok = (*abort_flag == 0) && mbar_wait(accf0 + 8 * fb, (f >> 1) & 1, p.err, 4);
            if (!ok) *abort_flag = 1;
            const bool live = !__any_sync(0xFFFFFFFFu, *abort_flag != 0);
            const float* ab = acc_s + fb * (S::kAccBuf / 4);
            const int seg_lo = max(u0, Bc * nk), seg_hi = min(u1, (Bc + 1) * nk);
            const bool whole = (seg_lo == Bc * nk) && (seg_hi == (Bc + 1) * nk);
            const int cf = cta_of_unit(Bc * nk, U, P), cl = cta_of_unit((Bc + 1) * nk - 1, U, P);
            bool finalize = whole;
            if (live && !whole) {
                float* mine = p.partials + (int64_t)partial_slot(c, Bc, nk, U, P) * m * 128;
                for (int row = 0; row < m; ++row) {
                    const float4 t0 = *reinterpret_cast<const float4*>(ab + row * 128 + col);
                    const float4 t1 = *reinterpret_cast<const float4*>(ab + (S::kRows + row) * 128 + col);
                    __stcg(reinterpret_cast<float4*>(mine + row * 128 + col),
                           make_float4(t0.x + t1.x, t0.y + t1.y, t0.z + t1.z, t0.w + t1.w));
                }
                __syncwarp();
                int v = 0;
                if (lane == 0) {
                    // cumulative fence over the warp's partial stores, then the counter; the
                    // second fence orders the reads of other CTAs' partials after it
                    __threadfence();
                    v = atomicAdd(p.counters + Bc, 1);
                    __threadfence();
                }
                v = __shfl_sync(0xFFFFFFFFu, v, 0);
                finalize = (v == cl - cf);
            }
            if (live && finalize) {
                const int g = group_of_block(p.g, p.groups, Bc);
                const int b = Bc - p.g.blk_prefix[g];
                const uint2 sv = *reinterpret_cast<const uint2*>(p.g.svh[g] + b * 128 + col);
                for (int row = 0; row < m; ++row) {
                    float v[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int cc = cf; cc <= cl; ++cc) {  // fixed order: deterministic sums
                        float4 t;
                        if (cc == c) {
                            const float4 t0 = *reinterpret_cast<const float4*>(ab + row * 128 + col);
                            const float4 t1 = *reinterpret_cast<const float4*>(ab + (S::kRows + row) * 128 + col);
                            t = make_float4(t0.x + t1.x, t0.y + t1.y, t0.z + t1.z, t0.w + t1.w);
                        } else {
                            t = __ldcg(reinterpret_cast<const float4*>(
                                p.partials + ((int64_t)partial_slot(cc, Bc, nk, U, P) * m + row) * 128 + col));
                        }
                        v[0] += t.x; v[1] += t.y; v[2] += t.z; v[3] += t.w;
                    }
                    // c_rot is stored fp16 between the dot and the output transform (oracle :349-351)
                    const __half2 c01 = __floats2half2_rn(v[0], v[1]), c23 = __floats2half2_rn(v[2], v[3]);
                    float h[4] = {__low2float(c01), __high2float(c01), __low2float(c23), __high2float(c23)};
                    had128_warp(h);
                    __half2 y01 = __floats2half2_rn(h[0] * kRScale, h[1] * kRScale);
                    __half2 y23 = __floats2half2_rn(h[2] * kRScale, h[3] * kRScale);
                    y01 = __hmul2(y01, u32_as_h2(sv.x));
                    y23 = __hmul2(y23, u32_as_h2(sv.y));
                    *reinterpret_cast<uint2*>(p.g.y[g] + row * p.ldy + b * 128 + col) =
                        make_uint2(h2_as_u32(y01), h2_as_u32(y23));
                }
                if (!whole && lane == 0) p.counters[Bc] = 0;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(acce0 + 8 * fb);
        }
        return;
    }

    // ------------------------------ consumer warps ------------------------------
    LaneGeom<K> geom;
    geom.init(lane);
    const int gq = lane >> 2, tq = lane & 3;
    const int tpair = warp & 3, kh = warp >> 2;
    // per-lane offsets inside a stage: this warp's first tile (k-tile 4kh, n-tile 2 tpair) plus the
    // lane's word offsets; the remaining tiles are compile-time offsets from these
    const uint32_t tile0 = (uint32_t)((kh * 4 * 8 + 2 * tpair) * 32 * K);
    uint32_t woff[LaneGeom<K>::kNW];
#pragma unroll
    for (int q = 0; q < LaneGeom<K>::kNW; ++q) woff[q] = tile0 + geom.off[q];
    const uint32_t boff = (uint32_t)(S::kTrellisStage + gq * kAhadRow * 2 + kh * 4 * 32 + tq * 8);

    float acc[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int jn = 0; jn < 2; ++jn)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][jn][e] = 0.f;
    int j = u0 % nk, nflush = 0;

    for (int i = 0; i < nunits; ++i) {
        const int s = i % kStages, n = i / kStages;
        // On a wait that gives up, the warps keep walking the units without touching the ring,
        // so every barrier below still sees all of its arrivals.
        bool ok = (*abort_flag == 0) && mbar_wait(full0 + 8 * s, n & 1, p.err, 3);
        if (!ok) *abort_flag = 1;
        const bool live = !__any_sync(0xFFFFFFFFu, *abort_flag != 0);
        if (live) {
            const uint8_t* st = smem + s * S::kStageBytes;
            const uint8_t* bp = st + boff;
#pragma unroll
            for (int kt = 0; kt < 4; ++kt) {
                uint32_t b[MT][2];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint2 v = *reinterpret_cast<const uint2*>(bp + mt * 8 * kAhadRow * 2 + kt * 32);
                    b[mt][0] = v.x;
                    b[mt][1] = v.y;
                }
#pragma unroll
                for (int jn = 0; jn < 2; ++jn) {
                    constexpr int kTile = 32 * K;
                    uint32_t Wd[LaneGeom<K>::kNW];
#pragma unroll
                    for (int q = 0; q < LaneGeom<K>::kNW; ++q)
                        Wd[q] = *reinterpret_cast<const uint32_t*>(st + woff[q] + (kt * 8 + jn) * kTile);
                    uint32_t a[4];
                    lane_decode_frag<K, CB>(Wd, geom.phi, a);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) mma_16816(acc[mt][jn], a, b[mt][0], b[mt][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);

        const bool block_end = (++j == nk);
        if (block_end) j = 0;
        if (!block_end && i != nunits - 1) continue;

        // ---------------- hand the finished block to the epilogue warp ----------------
        // acc buffer fb is free once the epilogue released its previous use (two flushes ago)
        const int fb = nflush & 1;
        if (nflush >= 2) {
            bool ok2 = (*abort_flag == 0) && mbar_wait(acce0 + 8 * fb, ((nflush >> 1) - 1) & 1, p.err, 5);
            if (!ok2) *abort_flag = 1;
        }
        // fragment -> acc_s[fb][kh][row][col]: lane (gq, tq) holds D[col gq (+8)][rows 2tq, 2tq+1]
        float* acc_h = acc_s + fb * (S::kAccBuf / 4) + kh * S::kRows * 128;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int jn = 0; jn < 2; ++jn) {
                const int col = (2 * tpair + jn) * 16 + gq;
                const int r0 = 8 * mt + 2 * tq;
                acc_h[r0 * 128 + col] = acc[mt][jn][0];
                acc_h[r0 * 128 + col + 8] = acc[mt][jn][2];
                acc_h[(r0 + 1) * 128 + col] = acc[mt][jn][1];
                acc_h[(r0 + 1) * 128 + col + 8] = acc[mt][jn][3];
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[mt][jn][e] = 0.f;
            }
        __syncwarp();
        if (lane == 0) mbar_arrive(accf0 + 8 * fb);
        ++nflush;
    }
}

// ---------------------------------------------------------------------------------------------

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
constexpr size_t kHeaderBytes = 256;
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

// Stream-K width: two CTAs per SM, independent of m, K and codebook, so the partition (and
// therefore every rounding) depends only on the layer shape.
static int gemv_ctas(int units) { return std::min(units, 2 * num_sms()); }

struct WsLayout {
    size_t counters, a_had, partials, total;
};

static WsLayout ws_layout(int m, int k, int groups, int64_t n_total) {
    WsLayout L;
    const int64_t blocks = n_total / 128;
    const int units = (int)(blocks * (k / 128));
    const int P = gemv_ctas(std::max(units, 1));
    L.counters = kHeaderBytes;
    L.a_had = round_up(L.counters + kCounterBytes, 256);
    L.partials = round_up(L.a_had + (size_t)groups * m * (k / 128) * kAhadRow * 2, 256);
    L.total = round_up(L.partials + (size_t)2 * P * m * 128 * 4, 256);
    return L;
}

template <int K, int CB, int MT>
static cudaError_t launch_gemv(const GemvParams& p, cudaStream_t st) {
    using S = GemvSmem<K, MT>;
    auto kern = gemv_kernel<K, CB, MT>;
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    static cudaError_t attr_err[64];
    std::call_once(once[dev & 63], [&] {
        attr_err[dev & 63] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    });
    if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = S::kTotal;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int CB, int MT>
static cudaError_t launch_gemv_k(int K, const GemvParams& p, cudaStream_t st) {
    switch (K) {
        case 1: return launch_gemv<1, CB, MT>(p, st);
        case 2: return launch_gemv<2, CB, MT>(p, st);
        case 3: return launch_gemv<3, CB, MT>(p, st);
        case 4: return launch_gemv<4, CB, MT>(p, st);
        case 5: return launch_gemv<5, CB, MT>(p, st);
        case 6: return launch_gemv<6, CB, MT>(p, st);
        case 7: return launch_gemv<7, CB, MT>(p, st);
        default: return launch_gemv<8, CB, MT>(p, st);
    }
}

int linear_impl(const uint16_t* x, int m, int k, int groups, const uint16_t* const* trellis, const int* n,
                       int K, int codebook, const uint16_t* const* suh, const uint16_t* const* svh,
                       uint16_t* const* y, int64_t ldy, void* workspace, size_t ws_bytes, void* stream) {
    if (K < 1 || K > 8 || codebook < 0 || codebook > 2) return EXL3B_DECLINED;
    if (m < 1 || m > EXL3B_GEMV_MAX_ROWS || groups < 1 || groups > EXL3B_MAX_GROUPS) return EXL3B_DECLINED;
    if (k <= 0 || k % 128) return EXL3B_DECLINED;
    if (!x || !trellis || !n || !suh || !svh || !y || !workspace) return EXL3B_BAD_ARG;
    if (!aligned(x, 8) || k % 4 || ldy % 4 || !aligned(workspace, 256)) return EXL3B_BAD_ARG;
    int64_t n_total = 0;
    for (int g = 0; g < groups; ++g) {
        if (n[g] <= 0 || n[g] % 128) return EXL3B_DECLINED;
        if (ldy < n[g]) return EXL3B_BAD_ARG;
        if (!trellis[g] || !suh[g] || !svh[g] || !y[g]) return EXL3B_BAD_ARG;
        if (!aligned(trellis[g], 16) || !aligned(suh[g], 8) || !aligned(svh[g], 8) || !aligned(y[g], 8))
            return EXL3B_BAD_ARG;
        n_total += n[g];
    }
    if (n_total / 128 > kMaxBlocks) return EXL3B_DECLINED;
    const WsLayout L = ws_layout(m, k, groups, n_total);
    if (ws_bytes < L.total) return EXL3B_WORKSPACE;

    cudaStream_t st = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    __half* a_had = reinterpret_cast<__half*>(ws + L.a_had);

    HadInParams hp = {};
    GemvParams p = {};
    int blk = 0;
    for (int g = 0; g < groups; ++g) {
        hp.suh[g] = reinterpret_cast<const __half*>(suh[g]);
        p.g.trellis[g] = trellis[g];
        p.g.svh[g] = reinterpret_cast<const __half*>(svh[g]);
        p.g.y[g] = reinterpret_cast<__half*>(y[g]);
        p.g.n_tiles[g] = n[g] / 16;
        p.g.blk_prefix[g] = blk;
        blk += n[g] / 128;
    }
    p.g.blk_prefix[groups] = blk;
    p.a_had = a_had;
    p.partials = reinterpret_cast<float*>(ws + L.partials);
    p.counters = reinterpret_cast<int*>(ws + L.counters);
    p.err = reinterpret_cast<int*>(ws);
    p.groups = groups;
    p.m = m;
    p.nk = k / 128;
    p.units = blk * p.nk;
    p.ctas = gemv_ctas(p.units);
    p.ldy = ldy;

    had_in_kernel<<<dim3(k / 128, groups), dim3(32 * m), 0, st>>>(reinterpret_cast<const __half*>(x), m, k, hp, a_had);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e);
    const bool mt2 = m > 8;
    switch (codebook) {
        case 0: e = mt2 ? launch_gemv_k<0, 2>(K, p, st) : launch_gemv_k<0, 1>(K, p, st); break;
        case 1: e = mt2 ? launch_gemv_k<1, 2>(K, p, st) : launch_gemv_k<1, 1>(K, p, st); break;
        default: e = mt2 ? launch_gemv_k<2, 2>(K, p, st) : launch_gemv_k<2, 1>(K, p, st); break;
    }
    return cuda_status(e);
}

}  // namespace exl3b

using namespace exl3b;

extern "C" size_t exl3b_linear_workspace_bytes(int m, int k, int groups, int64_t n_total) {
    if (m < 1 || k < 128 || groups < 1 || n_total < 128) return 0;
    return ws_layout(m, k, groups, n_total).total;
}

extern "C" int exl3b_linear(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K, int codebook,
                            const uint16_t* suh, const uint16_t* svh, uint16_t* y, int64_t ldy, void* workspace,
                            size_t workspace_bytes, void* stream) {
    const uint16_t* tr[1] = {trellis};
    const uint16_t* su[1] = {suh};
    const uint16_t* sv[1] = {svh};
    uint16_t* yy[1] = {y};
    int nn[1] = {n};
    return linear_impl(x, m, k, 1, tr, nn, K, codebook, su, sv, yy, ldy, workspace, workspace_bytes, stream);
}

extern "C" int exl3b_linear_grouped(const uint16_t* x, int m, int k, int groups, const uint16_t* const* trellis,
                                    const int* n, int K, int codebook, const uint16_t* const* suh,
                                    const uint16_t* const* svh, uint16_t* const* y, int64_t ldy, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    return linear_impl(x, m, k, groups, trellis, n, K, codebook, suh, svh, y, ldy, workspace, workspace_bytes,
                       stream);
}

extern "C" int exl3b_linear_workspace_error(const void* workspace, int* out, void* stream) {
    if (!workspace || !out) return EXL3B_BAD_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyAsync(out, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return cuda_status(e);
}
