// The EXL3 linear for many rows (prefill, M > 16) on the 5th-generation tensor cores (tcgen05).
//
//   y[M][n] = had_out( fp16( A_had @ W ), svh ),   A_had = had_in(x, suh) = fp16(H128 fp16(x * suh) / sqrt(128))
//
// The reference reconstructs W into a dense fp16 matrix in memory and runs an fp16-accumulate GEMM on it
// (vllm_plugin/exl3rocm/ops.py:86-97: had_r_128, reconstruct[_slice], hgemm_recon).  Here W never exists
// in global memory: the CTAs decode the trellis tiles of their output tile straight into the shared-
// memory B operand of tcgen05.mma, which accumulates in fp32 in tensor memory.
//
// CTA pairs (clusters of two, tcgen05 cta_group::2).  A pair owns output tiles of 512 rows x 256 columns
// (row tiles fastest, so the pairs working at the same time share each weight tile through L2) and
// issues M = 256, N = 256 MMAs: CTA r holds rows 128 r .. of each 256-row half in its A sub-tiles and
// columns 128 r .. of B, and its tensor memory receives its rows of both 256 x 256 accumulators (512
// columns).  Each CTA therefore decodes half of the weight tile, and reads half of B per MMA from its
// shared memory.  Per 64-input k-block, in each CTA:
//   * warp 8 (producer) streams the CTA's trellis bytes (four k-rows of eight 16x16 tiles, one bulk
//     copy per k-row) into a raw ring, and its two 128-row A_had sub-tiles by TMA (128-byte swizzle),
//     counted on the leader CTA's barrier;
//   * warps 0-7 decode the 32 trellis tiles (four each; the lane placement of mma.m16n8k16's A
//     operand, see exl3b_common.cuh) and store the fp16 weights K-major with the same swizzle, the
//     layout the MMA's shared-memory descriptors describe; they arrive on the leader's barrier;
//   * in the leader, warp 9 issues 2 x 4 tcgen05.mma (cta_group::2) and commits to the barriers of
//     both CTAs that free the stages.
// After the last k-block every CTA's warps 0-7 read their accumulator rows back (task t = w, w + 8:
// TMEM lanes 32 (t % 4) .., accumulator t / 8, 128-column block (t / 4) % 2), one output row per thread: fp16
// round (the reference's c_rot), the 128-point Hadamard of the block (H4 x H32 through tensor memory),
// 1/sqrt(128), fp16, times svh (fp16), stored.
//
// No load uses cluster multicast: every CTA loads only into its own shared memory.  All waits are
// bounded (about a second); a wait that gives up records an error word, raises the CTA's abort flag
// (its other waits then give up at once), and the CTA drains its copies and MMAs in flight before the
// pair frees its tensor memory and exits.
#include "exl3b_common.cuh"

namespace exl3b {

namespace gemm {

constexpr int kPairRows = 512;      // output rows per pair tile (two M = 256 accumulators)
constexpr int kBN = 256;            // output columns per tile (the MMA's N)
constexpr int kHalfN = kBN / 2;     // B columns held (and decoded) by one CTA
constexpr int kBK = 64;             // inputs per k-block (one 128-byte swizzle row of fp16)
constexpr int kSubRows = 128;       // rows of one A sub-tile / of one CTA's share of an accumulator
#ifndef EXL3B_GEMM_DECODE_WARPS
#define EXL3B_GEMM_DECODE_WARPS 8
#endif
// 8 decode warps of four tiles each per k-block measured faster than 16 of two (the per-k-block
// barrier traffic is the same per warp): 347 -> 326 us at M 2048, 5120 -> 17408
constexpr int kDecodeWarps = EXL3B_GEMM_DECODE_WARPS;   // 8 or 16
constexpr int kTilesPerWarp = 32 / kDecodeWarps;        // trellis tiles one decode warp takes per k-block
constexpr int kTasksPerWarp = 16 / kDecodeWarps;        // epilogue (lane quarter, accumulator, block) tasks
constexpr int kProducerWarp = kDecodeWarps;
constexpr int kMmaWarp = kDecodeWarps + 1;
constexpr int kThreads = 32 * (kDecodeWarps + 2);
static_assert(kDecodeWarps == 8 || kDecodeWarps == 16, "decode warps");
constexpr int kAStages = 4;
constexpr int kBStages = 3;
constexpr int kRawStages = 4;
constexpr int kASub = kSubRows * kBK * 2;  // 16 KB
constexpr int kAStage = 2 * kASub;         // 32 KB
constexpr int kBStage = kHalfN * kBK * 2;  // 16 KB
constexpr int kTmemCols = 512;

template <int K>
struct Smem {
    static constexpr int kTile = 32 * K;                         // bytes of one 16x16 trellis tile
    static constexpr int kRawRow = (kHalfN / 16) * kTile;        // one k-row of this CTA's trellis
    static constexpr int kRawStage = (kBK / 16) * kRawRow;       // four k-rows
    static constexpr int kA = 0;
    static constexpr int kB = kA + kAStages * kAStage;
    static constexpr int kRaw = kB + kBStages * kBStage;
    static constexpr int kBars = kRaw + kRawStages * kRawStage;
    // raw full/empty, a full/empty, b full/empty, acc full/empty, mma done
    static constexpr int kNumBars = 2 * kRawStages + 2 * kAStages + 2 * kBStages + 3;
    static constexpr int kTmemSlot = kBars + 8 * kNumBars;
    static constexpr int kAbort = kTmemSlot + 4;
    static constexpr int kTotal = kAbort + 4 + 1024;  // + alignment slack for the 1024-byte swizzle atoms
    static_assert(kTotal <= 232448, "shared memory");
};

struct Params {
    const uint16_t* trellis;  // [k/16][n/16][16K]
    const __half* svh;        // [n]
    __half* y;                // [m][ldy]
    int64_t ldy;
    int m, k, n;
    int m_pairs, n_tiles, tiles, kblocks;
    int* err;
};

// ---------------------------------------------------------------------------------------------
// cluster / tcgen05 / TMA wrappers
// ---------------------------------------------------------------------------------------------
EXL3B_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
EXL3B_DEV uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;\n" : "=r"(r));
    return r;
}
EXL3B_DEV uint32_t num_clusters() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;\n" : "=r"(r));
    return r;
}
// the shared::cluster address of the same shared-memory location in CTA `rank` of the cluster
EXL3B_DEV uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
EXL3B_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// arrive on an mbarrier of a CTA of the cluster (its shared::cluster address).  The default semantics
// (release at CTA scope) suffice: what the waiter consumes is shared memory read by the tensor core,
// made visible by fence.proxy.async before the arrive; a cluster-scope release here cost a third of
// the kernel's time (measured: 471 -> 347 us at M 2048, 5120 -> 17408).
EXL3B_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];\n" :: "r"(cluster_addr) : "memory");
}

EXL3B_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
EXL3B_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
EXL3B_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

EXL3B_DEV void tmem_alloc2(uint32_t slot_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" :: "r"(slot_smem), "r"(cols)
                 : "memory");
}
EXL3B_DEV void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
EXL3B_DEV void tmem_dealloc2(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" :: "r"(taddr), "r"(cols) : "memory");
}

// D (tmem of both CTAs) (+)= A (smem of both CTAs) x B (smem of both CTAs), kind::f16; leader only
EXL3B_DEV void umma2_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// arrive (once) on the mbarrier at this shared offset in both CTAs of the pair when every tcgen05
// operation this thread issued before has completed
EXL3B_DEV void umma2_commit_both(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n"
                 :: "r"(bar), "h"((uint16_t)0x3) : "memory");
}
// the same, arriving on this CTA's barrier only
EXL3B_DEV void umma2_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" :: "r"(bar) : "memory");
}

// 32 TMEM lanes (one per thread of the warp) x 32 consecutive 32-bit columns, load and store
EXL3B_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
EXL3B_DEV void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n"
        :: "r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
           "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]),
           "f"(v[16]), "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]),
           "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}
EXL3B_DEV void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
EXL3B_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
EXL3B_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// 2-D tiled TMA load (no multicast) into this CTA's shared memory, its bytes counted on an mbarrier
// that may sit in the peer CTA of the pair (cta_group::2); x = inner (k) coordinate, y = row
EXL3B_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];\n"
        :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster) : "memory");
}

// Shared-memory matrix descriptor of a K-major operand in the canonical 128-byte-swizzle layout:
// rows of 64 fp16 (128 B), 8-row groups 1024 B apart (SBO), 16-byte chunks XOR-ed with the row
// within the group; bits: start >> 4 [0,14), LBO >> 4 [16,30) (unused here), SBO >> 4 [32,46),
// version 1 [46,48), layout 2 = SWIZZLE_128B [61,64).
EXL3B_DEV uint64_t smem_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor, kind::f16: D fp32 [4,6) = 1, A and B fp16 (0), both K-major,
// N >> 3 at [17,23), M >> 4 at [24,29); M = 256 across the pair.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);

// A wait every lane of a warp makes; the warp proceeds only if all lanes saw the phase complete, so a
// wait that gives up in one lane cannot split the warp before a .sync.aligned instruction.
EXL3B_DEV bool warp_wait(uint32_t bar, uint32_t parity, int* err, int code, volatile int* abort) {
    const bool ok = mbar_wait_or_abort(bar, parity, err, code, abort);
    return __all_sync(0xFFFFFFFFu, ok);
}

// ---------------------------------------------------------------------------------------------
// The epilogue's 128-point Hadamard as H128 = H4 (x) H32 (natural-order Sylvester: element i = 32c + r
// gives H128[i][i'] = H4[c][c'] H32[r][r']): a 32-point transform of each 32-column chunk in
// registers, written back to tensor memory, then the 4-point transform across the chunks, 8 columns
// at a time.  One thread holds one output row; at most 32 values of it are live.
// ---------------------------------------------------------------------------------------------
template <int H, int N>
EXL3B_DEV void fwht_stage(float (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
        if ((i & H) == 0) {
            const float a = v[i], b = v[i + H];
            v[i] = a + b;
            v[i + H] = a - b;
        }
    }
}
EXL3B_DEV void fwht32(float (&v)[32]) {
    fwht_stage<1>(v); fwht_stage<2>(v); fwht_stage<4>(v); fwht_stage<8>(v); fwht_stage<16>(v);
}

// ---------------------------------------------------------------------------------------------
// the kernel (launched in clusters of two)
// ---------------------------------------------------------------------------------------------
template <int K, int CB>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const Params p) {
    using S = Smem<K>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment: the swizzle pattern is a function of the address bits [4, 10)
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = (int)cluster_id(), npairs = (int)num_clusters();
    const uint32_t bars = sbase + S::kBars;
    auto raw_full = [&](int s) { return bars + 8u * s; };
    auto raw_empty = [&](int s) { return bars + 8u * (kRawStages + s); };
    auto a_full = [&](int s) { return bars + 8u * (2 * kRawStages + s); };
    auto a_empty = [&](int s) { return bars + 8u * (2 * kRawStages + kAStages + s); };
    auto b_full = [&](int s) { return bars + 8u * (2 * kRawStages + 2 * kAStages + s); };
    auto b_empty = [&](int s) { return bars + 8u * (2 * kRawStages + 2 * kAStages + kBStages + s); };
    const uint32_t acc_full = bars + 8u * (2 * kRawStages + 2 * kAStages + 2 * kBStages);
    const uint32_t acc_empty = acc_full + 8u;
    const uint32_t mma_done = acc_full + 16u;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::kAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kTmemSlot);

    if (threadIdx.x == 0) {
        // a_full, b_full and acc_empty are used in the leader only and count both CTAs' arrivals;
        // the others are used in both CTAs
        for (int s = 0; s < kRawStages; ++s) { mbar_init(raw_full(s), 1); mbar_init(raw_empty(s), kDecodeWarps); }
        for (int s = 0; s < kAStages; ++s) { mbar_init(a_full(s), 1); mbar_init(a_empty(s), 1); }
        for (int s = 0; s < kBStages; ++s) { mbar_init(b_full(s), 2 * kDecodeWarps); mbar_init(b_empty(s), 1); }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * kDecodeWarps);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc2(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish2();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int kb_n = p.kblocks;

    if (warp == kProducerWarp) {
        // ---------------- producer: this CTA's trellis bytes + A_had sub-tiles ----------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];\n" :: "l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
            int it_raw = 0, it_a = 0;  // k-blocks whose raw / A copies were issued
            bool ok = true;
            const int nt16 = p.n / 16;
            for (int tile = pair; tile < p.tiles && ok; tile += npairs) {
                const int pm = tile % p.m_pairs, pn = tile / p.m_pairs;
                const int nt0 = pn * (kBN / 16) + (int)rank * (kHalfN / 16);
                const int nv = max(0, min(kHalfN / 16, nt16 - nt0));  // valid n-tiles of this CTA's half
                for (int kb = 0; kb < kb_n; ++kb) {
                    const int rs = it_raw % kRawStages, as = it_a % kAStages;
                    if (!mbar_wait_or_abort(raw_empty(rs), ((it_raw / kRawStages) & 1) ^ 1, p.err, 0x301,
                                            abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t row_bytes = (uint32_t)nv * S::kTile;
                    if (nv > 0) {
                        mbar_arrive_expect_tx(raw_full(rs), 4 * row_bytes);
                        for (int j = 0; j < 4; ++j) {
                            const int kt = kb * 4 + j;
                            bulk_g2s(sbase + S::kRaw + rs * S::kRawStage + j * S::kRawRow,
                                     p.trellis + ((int64_t)kt * nt16 + nt0) * 16 * K, row_bytes, raw_full(rs));
                        }
                    } else {
                        mbar_arrive(raw_full(rs));  // nothing of this half is in range: an empty stage
                    }
                    ++it_raw;
                    if (!mbar_wait_or_abort(a_empty(as), ((it_a / kAStages) & 1) ^ 1, p.err, 0x302, abort_flag)) {
                        ok = false;
                        break;
                    }
                    // both CTAs' A bytes complete on the leader's barrier; the leader expects them
                    const uint32_t full_leader = map_to_rank(a_full(as), 0);
                    if (leader) mbar_arrive_expect_tx(a_full(as), 2 * kAStage);
                    for (int sub = 0; sub < 2; ++sub)
                        tma_load_2d_pair(sbase + S::kA + as * kAStage + sub * kASub, &tmap_a, kb * kBK,
                                         pm * kPairRows + sub * 256 + (int)rank * kSubRows, full_leader);
                    ++it_a;
                }
            }
            // drain: every copy this CTA issued has landed before the CTA may exit (the follower's A
            // copies complete on the leader's barrier, which the leader drains)
            for (int j = max(0, it_raw - kRawStages); j < it_raw; ++j)
                mbar_wait(raw_full(j % kRawStages), (j / kRawStages) & 1, nullptr, 0);
            if (leader)
                for (int j = max(0, it_a - kAStages); j < it_a; ++j)
                    mbar_wait(a_full(j % kAStages), (j / kAStages) & 1, nullptr, 0);
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer (leader CTA) ----------------
        if (leader && lane == 0) {
            int it = 0, tcount = 0;
            bool ok = true, issued = false;
            for (int tile = pair; tile < p.tiles && ok; tile += npairs, ++tcount) {
                if (!mbar_wait_or_abort(acc_empty, (tcount & 1) ^ 1, p.err, 0x311, abort_flag)) break;
                tc_fence_after();
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int as = it % kAStages, bs = it % kBStages;
                    if (!mbar_wait_or_abort(a_full(as), (it / kAStages) & 1, p.err, 0x312, abort_flag) ||
                        !mbar_wait_or_abort(b_full(bs), (it / kBStages) & 1, p.err, 0x313, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = sbase + S::kA + as * kAStage, b0 = sbase + S::kB + bs * kBStage;
#pragma unroll
                    for (int sub = 0; sub < 2; ++sub)
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; ++kk)
                            umma2_f16(tmem + sub * kBN, smem_desc_sw128(a0 + sub * kASub + kk * 32),
                                      smem_desc_sw128(b0 + kk * 32), kIdesc, (kb | kk) != 0);
                    issued = true;
                    umma2_commit_both(a_empty(as));
                    umma2_commit_both(b_empty(bs));
                }
                if (ok) umma2_commit_both(acc_full);
            }
            // every MMA issued has completed before the tensor memory is freed
            if (issued) {
                umma2_commit(mma_done);
                mbar_wait(mma_done, 0, nullptr, 0);
            }
        }
    } else {
        // ---------------- decode warps, then the epilogue ----------------
        LaneGeom<K> geom;
        geom.init(lane);
        const int g = lane >> 2, c = lane & 3;
        const int nt16 = p.n / 16;
        // this warp's n-tile and the first of its kTilesPerWarp k-tiles
        const int ntl = warp & 7, kt0 = kTilesPerWarp * (warp >> 3);
        // byte offset inside a B stage of register r of this lane's fragment for k-tile kt: row
        // n = 16 ntl + g + 8 (r & 1), input k = 16 kt + 2c + 8 (r >> 1)
        auto b_off = [&](int kt, int r) -> uint32_t {
            return (uint32_t)((ntl * 2 + (r & 1)) * 1024 + g * 128 + ((((kt * 2 + (r >> 1)) ^ g)) << 4) + 4 * c);
        };
        const uint32_t b_full0 = map_to_rank(b_full(0), 0), acc_empty_leader = map_to_rank(acc_empty, 0);
        int it = 0, tcount = 0;
        bool ok = true;
        for (int tile = pair; tile < p.tiles && ok; tile += npairs, ++tcount) {
            const int pm = tile % p.m_pairs, pn = tile / p.m_pairs;
            const int nt0 = pn * (kBN / 16) + (int)rank * (kHalfN / 16);
            const int nv = max(0, min(kHalfN / 16, nt16 - nt0));
            for (int kb = 0; kb < kb_n; ++kb, ++it) {
                const int rs = it % kRawStages, bs = it % kBStages;
                if (!warp_wait(raw_full(rs), (it / kRawStages) & 1, p.err, 0x321, abort_flag) ||
                    !warp_wait(b_empty(bs), ((it / kBStages) & 1) ^ 1, p.err, 0x322, abort_flag)) {
                    ok = false;
                    break;
                }
                const uint8_t* raw = smem + S::kRaw + rs * S::kRawStage;
                uint8_t* bst = smem + S::kB + bs * kBStage;
                if (ntl < nv) {
#pragma unroll
                    for (int j = 0; j < kTilesPerWarp; ++j) {
                        const int kt = kt0 + j;
                        const uint8_t* tb = raw + kt * S::kRawRow + ntl * S::kTile;
                        uint32_t W[LaneGeom<K>::kNW];
#pragma unroll
                        for (int q = 0; q < LaneGeom<K>::kNW; ++q)
                            W[q] = *reinterpret_cast<const uint32_t*>(tb + geom.off[q]);
                        uint32_t a[4];
                        lane_decode_frag<K, CB>(W, geom.phi, a);
#pragma unroll
                        for (int r = 0; r < 4; ++r) *reinterpret_cast<uint32_t*>(bst + b_off(kt, r)) = a[r];
                    }
                }
                fence_proxy_async_smem();  // the weights are read by the tensor core (async proxy)
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_remote(b_full0 + 8u * bs);  // the leader's barrier counts both CTAs
                    mbar_arrive(raw_empty(rs));
                }
            }
            if (!ok) break;
            // ---- epilogue: warp w takes TMEM lanes 32 (w % 4) .. of accumulator (w / 8), columns
            //      128 ((w / 4) % 2) ..: one row and one 128-column block per thread ----
            if (!warp_wait(acc_full, tcount & 1, p.err, 0x323, abort_flag)) break;
            tc_fence_after();
#pragma unroll 1
            for (int tk = 0; tk < kTasksPerWarp; ++tk) {
                // task ids keep warp % 4: a warp may only access TMEM lanes 32 (warp % 4) ..
                const int tid = warp + tk * kDecodeWarps;
                const int lq = tid & 3, task = tid >> 2, sub = task >> 1, blk = task & 1;
                const int row = pm * kPairRows + sub * 256 + (int)rank * kSubRows + lq * 32 + lane;
                const int col0 = pn * kBN + blk * 128;
                const uint32_t tbase = tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(sub * kBN + blk * 128);
                // c_rot = fp16(acc), then the 32-point transform of each chunk, back into tensor memory
#pragma unroll 1
                for (int ch = 0; ch < 4; ++ch) {
                    float v[32];
                    tmem_ld32(tbase + 32 * ch, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __half2float(__float2half_rn(v[i]));
                    fwht32(v);
                    tmem_st32(tbase + 32 * ch, v);
                }
                tmem_st_wait();
                const bool live = row < p.m && col0 < p.n;
#pragma unroll 1
                for (int gi = 0; gi < 4; ++gi) {  // columns 8 gi .. 8 gi + 7 of every chunk
                    float z[4][8];
#pragma unroll
                    for (int ch = 0; ch < 4; ++ch) tmem_ld8(tbase + 32 * ch + 8 * gi, z[ch]);
                    tmem_ld_wait();
                    if (live) {
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) {
                            const int col = col0 + 32 * ch + 8 * gi;
                            const uint4 s4 = __ldg(reinterpret_cast<const uint4*>(p.svh + col));
                            const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
                            uint32_t o[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                float y2[2];
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const int i = 2 * e + h;
                                    // row ch of H4 over the chunks' values at this column
                                    const float z0 = z[0][i], z1 = z[1][i], z2 = z[2][i], z3 = z[3][i];
                                    const float t = ch == 0 ? (z0 + z1) + (z2 + z3)
                                                  : ch == 1 ? (z0 - z1) + (z2 - z3)
                                                  : ch == 2 ? (z0 + z1) - (z2 + z3)
                                                            : (z0 - z1) - (z2 - z3);
                                    y2[h] = t * kRScale;
                                }
                                o[e] = h2_as_u32(__hmul2(__floats2half2_rn(y2[0], y2[1]), u32_as_h2(sw[e])));
                            }
                            *reinterpret_cast<uint4*>(p.y + (int64_t)row * p.ldy + col) =
                                make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acc_empty_leader);  // the leader's MMA waits for both CTAs
        }
    }

    tc_fence_before();
    cluster_sync();  // neither CTA leaves while the pair's MMAs, copies or remote arrivals may touch it
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc2(tmem, kTmemCols);
    }
}

}  // namespace gemm

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
// cuTensorMapEncodeTiled, resolved through the runtime (no link-time dependency on the driver library,
// so the library loads on machines without a GPU driver)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

template <int K, int CB>
static cudaError_t launch_gemm(const CUtensorMap& map, const gemm::Params& p, cudaStream_t st) {
    using S = gemm::Smem<K>;
    auto kern = gemm::gemm_kernel<K, CB>;
    static cudaError_t attr_err[64];
    static int max_pairs[64];
    int dev = 0;
    cudaGetDevice(&dev);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(gemm::kThreads);
    cfg.dynamicSmemBytes = S::kTotal;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!max_pairs[dev & 63] && attr_err[dev & 63] == cudaSuccess) {
        attr_err[dev & 63] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
        if (attr_err[dev & 63] == cudaSuccess) {
            // pairs resident at once (one CTA per SM)
            cfg.gridDim = dim3(2);
            int clusters = 0;
            attr_err[dev & 63] = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
            if (attr_err[dev & 63] == cudaSuccess) max_pairs[dev & 63] = clusters > 0 ? clusters : 1;
        }
    }
    if (attr_err[dev & 63] != cudaSuccess) return attr_err[dev & 63];
    const int pairs = std::min(p.tiles, max_pairs[dev & 63]);
    cfg.gridDim = dim3(2 * pairs);
    return cudaLaunchKernelEx(&cfg, kern, map, p);
}

template <int CB>
static cudaError_t launch_gemm_k(int K, const CUtensorMap& map, const gemm::Params& p, cudaStream_t st) {
    switch (K) {
        case 1: return launch_gemm<1, CB>(map, p, st);
        case 2: return launch_gemm<2, CB>(map, p, st);
        case 3: return launch_gemm<3, CB>(map, p, st);
        case 4: return launch_gemm<4, CB>(map, p, st);
        case 5: return launch_gemm<5, CB>(map, p, st);
        case 6: return launch_gemm<6, CB>(map, p, st);
        case 7: return launch_gemm<7, CB>(map, p, st);
        default: return launch_gemm<8, CB>(map, p, st);
    }
}

}  // namespace exl3b

using namespace exl3b;

extern "C" size_t exl3b_gemm_workspace_bytes(int m, int k) {
    if (m < 1 || k < 128) return 0;
    return 256 + ((size_t)m * k * 2 + 255) / 256 * 256;
}

extern "C" int exl3b_gemm(const uint16_t* x, int m, int k, const uint16_t* trellis, int n, int K, int codebook,
                          const uint16_t* suh, const uint16_t* svh, uint16_t* y, int64_t ldy, void* workspace,
                          size_t workspace_bytes, void* stream) {
    if (m < 1 || k < 128 || n < 128 || k % 128 || n % 128 || K < 1 || K > 8) return EXL3B_DECLINED;
    const int cb = codebook & 0xFF;
    if (cb < 0 || cb > 2 || (codebook & ~0x1FF)) return EXL3B_DECLINED;
    const bool x_bf16 = (codebook & EXL3B_X_BF16) != 0;
    if (!x || !trellis || !suh || !svh || !y || !workspace) return EXL3B_BAD_ARG;
    if (!aligned(x, 16) || !aligned(trellis, 16) || !aligned(svh, 16) || !aligned(y, 16) || ldy < n || ldy % 8 ||
        !aligned(workspace, 256))
        return EXL3B_BAD_ARG;
    if (workspace_bytes < exl3b_gemm_workspace_bytes(m, k)) return EXL3B_WORKSPACE;
    if (x_bf16) return EXL3B_DECLINED;  // the host casts bf16 x to fp16 before this call
    const EncodeTiledFn encode = encode_tiled();
    if (!encode) return cuda_status(cudaErrorSymbolNotFound);
    cudaStream_t st = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint16_t* a_had = reinterpret_cast<uint16_t*>(ws + 256);

    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {gemm::kBK, gemm::kSubRows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a_had, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return EXL3B_BAD_ARG;

    // A_had = fp16(H128 fp16(x * suh) / sqrt(128)) (the reference's had_r_128(x, suh), ops.py:88)
    int status = exl3b_had128(x, k, a_had, k, m, k, suh, nullptr, 1.0f, stream);
    if (status != EXL3B_OK) return status;

    gemm::Params p = {};
    p.trellis = trellis;
    p.svh = reinterpret_cast<const __half*>(svh);
    p.y = reinterpret_cast<__half*>(y);
    p.ldy = ldy;
    p.m = m; p.k = k; p.n = n;
    p.m_pairs = (m + gemm::kPairRows - 1) / gemm::kPairRows;
    p.n_tiles = (n + gemm::kBN - 1) / gemm::kBN;
    p.tiles = p.m_pairs * p.n_tiles;
    p.kblocks = k / gemm::kBK;
    p.err = reinterpret_cast<int*>(ws);
    cudaError_t e;
    switch (cb) {
        case 0: e = launch_gemm_k<0>(K, map, p, st); break;
        case 1: e = launch_gemm_k<1>(K, map, p, st); break;
        default: e = launch_gemm_k<2>(K, map, p, st); break;
    }
    return cuda_status(e);
}
