// cm_gemm.cu -- MatmulKernel on B200 (reference: kernels/matmul/kernel/MatmulKernel.cpp)
// and the tcgen05 Q8.8 GEMM core it shares with ConvKernel.
//
// Exactness.  The reference accumulates exact Q8.8 x Q8.8 products in an
// ap_fixed<32,16> (int32, wraps mod 2^32) and narrows once (MatmulKernel.cpp:204,
// :217-218).  Write every int16 word as x = 256*h + l' + 128 with
// h = x >> 8 in [-128, 127] and l' = (x & 255) - 128 in [-128, 127], both int8.
// With x' = x - 128 = 256*h + l':
//   sum_k a*b = sum a'b' + 128*sum_k a' + 128*sum_k b' + 16384*K
//   sum a'b'  = 2^16*sum(ah*bh) + 2^8*(sum(ah*bl') + sum(al'*bh)) + sum(al'*bl')
// The four int8 dot products run on the tensor cores (tcgen05.mma kind::i8,
// s8 x s8 -> s32); the two rank-1 terms come from the split pre-pass.  All of it is reduced mod 2^32,
// which is exactly the reference's wrap, so the result is bit-identical.
// Each accumulator's magnitude stays below K * 2^15, so K <= 65535 never
// overflows an int32 on the way.
//
// Kernel (persistent, 1 CTA per SM or a CTA pair per 2 SMs, 576 threads):
//   warp 0   TMA producer: per K block of 128, the A planes' box (hi, lo') and the B
//            planes' box into a stage of a ring guarded by full/empty mbarriers.
//            No multicast.
//   warp 1   allocates all 512 TMEM columns; lane 0 issues the MMAs and commits.
//            128-column tiles: the B box lands as two N-major 128-column atoms
//            [Bh | Bl] = one 256-column operand, so each 32-deep K step is two M=128,
//            N=256 MMAs: Ah x [Bh|Bl] -> (HH | HL) and Al x [Bh|Bl] -> (LH | LL), four
//            128-column int32 accumulators (CTA pairs: M = 256, one B plane per CTA).
//            64-column tiles keep B packed ([64 hi | 64 lo] per K row, N = 128) with
//            double-buffered accumulators, or swap the operands (weights as A, N = 256:
//            see Cfg).
//   warps 2-17 epilogue: tcgen05.ld of the accumulators, recombine, narrow, fused
//            VectorOP epilogue, store int16 (or the next conv's plane image).
// Every mbarrier wait is bounded by %globaltimer; on expiry the kernel records
// CM_ETIMEOUT in the status word and winds down instead of hanging.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "cm_async.cuh"
#include "cm_gemm.cuh"

namespace cm {
namespace {

constexpr int BM = 128, BK = 128;
constexpr int PLANE_TILE = BM * BK;                 // 16 KB: one plane of a 128 x 128 operand tile
constexpr int OPERAND_TILE = 2 * PLANE_TILE;        // A hi + lo = 32 KB
// The per-CTA maximum of dynamic shared memory.  A GEMM CTA requests only what its
// configuration uses (Cfg::SMEM_LAUNCH, 190-205 KB: still one GEMM CTA per SM), which
// leaves room beside it for a small CTA of another kernel -- the split pre-pass of the
// next batch chunk of a large MatMul runs there while this chunk's GEMM computes.
constexpr int SMEM_BYTES = 232448;
constexpr uint32_t TMEM_COLS = 512;

// Column tile TBN = 128: B box = two N-major 128-column atoms [Bh | Bl] (32 KB),
// four 128-column accumulators fill TMEM (one buffer).  TBN = 64 (outputs with
// at most 64 columns): B is stored packed, each K row = [64 hi | 64 lo] bytes, so
// one 128-byte atom is the whole [Bh | Bl] operand (16 KB); the four 64-column
// accumulators take 256 TMEM columns and are double-buffered.
//
// WA ("weights as A", conv outputs of at most 64 channels): the roles swap so that the
// MMA is N = 256 wide.  A = the weight tile, 128 K-major rows (channel m's hi plane in
// row 2m, its lo' plane in row 2m + 1); B = the activation tile, K-major, its 128 hi
// rows followed by its 128 lo' rows (the two plane boxes are adjacent in shared
// memory).  One MMA per 32-deep step writes all four products of 64 channels x 128
// pixels into 256 accumulator columns (pixels of the hi plane, then of the lo' plane),
// double-buffered: half the MMA instructions of the packed form's two N = 128 MMAs per
// step (the tensor pipe runs N = 128 at the same rate per multiply-add).
template <int TBN, int CG = 1, bool WA = false>
struct Cfg {
    static_assert(CG == 1 || TBN == 128, "CTA pairs use 128-column tiles");
    static_assert(!WA || (TBN == 64 && CG == 1), "weights-as-A tiles hold 64 channels");
    // a CTA pair holds one B plane per CTA (Bh in the even CTA, Bl in the odd one)
    static constexpr int B_TILE = CG == 2 ? PLANE_TILE : (TBN == 128 ? 2 * PLANE_TILE : PLANE_TILE);
    static constexpr int STAGE = OPERAND_TILE + B_TILE;
    static constexpr int STAGES = CG == 2 ? 4 : (TBN == 128 ? 3 : 4);
    static constexpr int NBUF = TBN == 128 ? 1 : 2;
    static constexpr uint32_t ACC_COLS = 4 * TBN;      // HH | HL | LH | LL
    // epilogue warps: 4 TMEM lane quarters x 4 column groups (the epilogue must keep up
    // with short mainloops: conv tiles with few K blocks, fused residual reads)
    static constexpr int EPI_WARPS = 16;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr uint32_t MMA_N = WA ? 256u : 2 * TBN;   // [Bh | Bl], or WA: [hi pixels | lo' pixels]
    // Instruction descriptor: D s32, A s8 K-major, B s8 N-major (bit 16; K-major for WA),
    // M = 128 * CG, N = MMA_N.
    static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (WA ? 0u : (1u << 16)) | ((MMA_N >> 3) << 17) |
                                      ((uint32_t)((BM * CG) >> 4) << 24);
    // WA: a 16 x 16 int16 transpose buffer per epilogue warp, after the barriers
    static constexpr int XPOSE_BYTES = WA ? EPI_WARPS * 512 : 0;
    static constexpr int SMEM_USED = STAGES * STAGE + 1024 /*align*/ + 256 /*barriers*/ + XPOSE_BYTES;
    static constexpr int SMEM_LAUNCH = (SMEM_USED + 1023) / 1024 * 1024;
    static_assert(SMEM_LAUNCH <= SMEM_BYTES, "shared memory budget");
    static_assert(2 * SMEM_LAUNCH > SMEM_BYTES, "one GEMM CTA per SM");
    static_assert(NBUF * ACC_COLS <= TMEM_COLS, "TMEM budget");
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2,
                                            int c3, int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
        "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 bytes
// of K, 8-row groups 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// N-major, 128-byte swizzle: each K row holds 128 bytes of N; 8-row K groups are
// 1024 bytes apart (SBO); the two 128-column N atoms (hi plane, lo plane) are
// one plane tile apart (LBO = 16 KB).
__device__ __forceinline__ uint64_t sdesc_n(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)(16384 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}



__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA loads whose completion is signalled on the pair leader's mbarrier (bar is a
// shared::cluster address).  No multicast: each CTA loads into its own shared memory.
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2,
                                                 int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_load_5d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2,
                                                 int c3, int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
        "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on the mbarrier at this shared offset in every CTA of `mask` once the pair's
// MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint16_t mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
                 "h"(mask)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// ---------------------------------------------------------------------------
// Window-form MMA issue.  One thread issues all of a CTA's MMAs, and at M = 128,
// N = 128 (about 70 tensor cycles a step) its instruction stream, not the tensor
// pipe, set the pace: a loop with runtime bounds, a stage index taken modulo a
// runtime stage count and descriptors rebuilt per MMA issued one MMA every ~130
// cycles.  So descriptors advance by constant increments (the start-address field
// holds address / 16, and every operand lies below 2^18 bytes, so the additions
// never carry out of it), the stage ring advances without divisions, and the tile
// shapes of the shipped networks issue from fully unrolled code (ResNet-18: 3x3
// 64-channel convs, 3 rows x 2 K blocks, 2 steps in the last; the row-stacked
// space-to-depth stem, 2 rows x 1 block of 4 steps); other shapes take the loop.
// ---------------------------------------------------------------------------
struct WinIssue {
    uint64_t da0, db0;       // descriptors of stage 0's window and of the resident weights
    uint32_t stb16;          // one stage, in descriptor units
    uint32_t roff;           // kernel row offset inside a window, in descriptor units
    uint32_t wpl;            // lo' plane offset inside a window, in descriptor units
    uint32_t stages;
};

constexpr uint32_t kWinAStep = 32 >> 4;               // 32 K bytes of a K-major row
constexpr uint32_t kWinBStep = (32 * 128) >> 4;       // 32 K rows of 128 N bytes
constexpr uint32_t kWinBBlock = PLANE_TILE >> 4;      // one 128-deep weight block

// one 32-deep step: A's hi and lo' planes against [Bh | Bl]
template <uint32_t NOFF, uint32_t IDESC>
__device__ __forceinline__ void win_step(uint32_t d, uint64_t ah, uint64_t al, uint64_t bhl, uint32_t acc) {
    umma_i8(d, ah, bhl, IDESC, acc);           // -> HH | HL
    umma_i8(d + NOFF, al, bhl, IDESC, acc);    // -> LH | LL
}

// The K blocks of one tile.  Each block is one window stage holding all kernel rows;
// its MMAs free the stage once they have read it.  KH = 0: shape from the arguments.
template <uint32_t KH, uint32_t KBR, uint32_t LAST, uint32_t NOFF, uint32_t IDESC>
__device__ __forceinline__ bool win_tile(uint32_t d, const WinIssue& w, uint32_t kh, uint32_t kbr, uint32_t last,
                                         uint32_t& s, uint32_t& phase, uint64_t* full_b, uint64_t* empty_b,
                                         const WaitCtl& wc) {
    constexpr uint32_t BKS = BK / 32;
    if constexpr (KH != 0) {
#pragma unroll
        for (uint32_t kb = 0; kb < KBR; ++kb) {
            if (!mbar_wait(smem_u32(&full_b[s]), phase, wc)) return false;
            tc_fence_after();
            const uint64_t da = w.da0 + s * w.stb16;
#pragma unroll
            for (uint32_t r = 0; r < KH; ++r) {
                const uint64_t ar = da + r * w.roff, br = w.db0 + (r * KBR + kb) * kWinBBlock;
#pragma unroll
                for (uint32_t kk = 0; kk < (kb + 1 == KBR ? LAST : BKS); ++kk)
                    win_step<NOFF, IDESC>(d, ar + kk * kWinAStep, ar + w.wpl + kk * kWinAStep, br + kk * kWinBStep,
                                          (kb | r | kk) != 0u);
            }
            umma_commit(smem_u32(&empty_b[s]));
            if (++s == w.stages) { s = 0; phase ^= 1u; }
        }
    } else {
        for (uint32_t kb = 0; kb < kbr; ++kb) {
            if (!mbar_wait(smem_u32(&full_b[s]), phase, wc)) return false;
            tc_fence_after();
            const uint64_t da = w.da0 + s * w.stb16;
            const uint32_t steps = kb + 1u == kbr ? last : BKS;     // 32-deep steps holding any tap
            for (uint32_t r = 0; r < kh; ++r) {
                const uint64_t ar = da + r * w.roff, br = w.db0 + (r * kbr + kb) * kWinBBlock;
                const uint32_t first = (kb | r) != 0u;
#pragma unroll
                for (uint32_t kk = 0; kk < BKS; ++kk)
                    if (kk < steps)
                        win_step<NOFF, IDESC>(d, ar + kk * kWinAStep, ar + w.wpl + kk * kWinAStep, br + kk * kWinBStep,
                                              kk ? 1u : first);
            }
            umma_commit(smem_u32(&empty_b[s]));
            if (++s == w.stages) { s = 0; phase ^= 1u; }
        }
    }
    return true;
}

#define CM_R16(i) "=r"(r[i])
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : CM_R16(0), CM_R16(1), CM_R16(2), CM_R16(3), CM_R16(4), CM_R16(5), CM_R16(6), CM_R16(7), CM_R16(8),
          CM_R16(9), CM_R16(10), CM_R16(11), CM_R16(12), CM_R16(13), CM_R16(14), CM_R16(15)
        : "r"(taddr));
}
#undef CM_R16


__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Two raw accumulators narrowed as saturate_cast does (floor by 8 bits: arithmetic
// shift; clamp to int16) and packed, `lo` in the low half: one cvt.pack.sat per pair.
__device__ __forceinline__ uint32_t narrow_pack(uint32_t lo, uint32_t hi) {
    uint32_t d;
    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(d) : "r"((int32_t)hi >> 8), "r"((int32_t)lo >> 8));
    return d;
}

constexpr uint32_t GROUP_M = 8;

struct GemmArgs {
    uint32_t rows, cols, num_kb, a_batches, b_batches, tiles_m, tiles_n, batch;
    uint32_t tiles_mc;        // row tiles per CTA group: ceil(tiles_m / CG)
    const int32_t* rowterm;
    const int32_t* colterm;
    int16_t* out;
    uint64_t ldo, ldc, out_bs;
    int* status;
    uint64_t timeout_ns;
    // implicit conv (conv != 0): tile rows = bn images x bh rows x bw columns
    uint32_t conv, tiles_w, tiles_h, bw_log, bh_log, bn_log;
    uint32_t nimg, out_h, out_w, sw, sh, dh, kb_per_r;
    // rows_per_img != 0: row = n*rows_per_img + p -> out[n*out_bs + p + col*ldc]
    uint32_t rows_per_img;
    uint32_t ksteps;          // 32-deep MMA steps covering K (conv: covering one kernel row's KR bytes)
    // fused elementwise epilogue on the narrowed word v (bit 1: v = sat16(v + resid at the
    // output's index); bit 2: v = sat16(v + resid[col]), a bias row broadcast over the
    // rows; then bit 0: v = max(v, 0)) -- VectorOP ADD / RELU semantics
    uint32_t epi;
    const int16_t* resid;
    // conv mode: the residual (epi bit 1) read from a plane image of the output's shape
    // instead of `resid`
    const int8_t* rpl;
    uint64_t rpl_plane;
    uint32_t rpl_Hp, rpl_Wp, rpl_Cp, rpl_pt, rpl_pl;
    // conv mode: output also written as a channels-last plane image (see PlaneOut)
    int8_t* po;
    int32_t* po_S;
    uint64_t po_plane;
    uint32_t po_Hp, po_Wp, po_Cp, po_pt, po_pl;
    // divisors of the tile decode (set by launch_persistent): tiles per batch step, tiles
    // per row-tile group, conv tiles per image and per tile row
    FastDiv fd_z, fd_group, fd_hw, fd_w;
    // conv window form (win != 0): tile rows are (row, image, column); per K block one TMA
    // box brings the input window of all kh kernel rows (bh + (kh-1)*dh rows of bn images,
    // both planes: win_bytes, the lo' plane win_plane bytes after the hi plane) and kernel
    // row r reads it win_roff*r bytes in; the packed weights (w_bytes) stay resident
    uint32_t win, win_stages, win_bytes, win_plane, win_roff, w_bytes, kh;
    // profiling: CTA 0 adds its {SM cycles, ns} from start to exit here (prof_gemm_clock)
    unsigned long long* clk;
    // K-split (splits > 1; set by launch_persistent, 1 otherwise): work unit u is K blocks
    // [sp*num_kb/splits, (sp+1)*num_kb/splits) of tile u / splits, sp = u % splits.  Its
    // raw product sums go to slab (tile, CTA of the pair, sp) of ws, TBN columns of BM
    // int32 each; cnt counts the slabs landed per (tile, CTA, epilogue warp)
    uint32_t splits;
    FastDiv fd_split;
    int32_t* ws;
    uint32_t* cnt;
    uint32_t no_split;        // the launch may not allocate: never K-split
};

struct Tile {
    uint32_t m0, n0, z, ba, bb;
    uint32_t cw0, ch0, cn0;   // conv: first output column, row and image of the row tile
};

// Tile t of the flattened (batch, grouped row/column) order, for CTA `rank` of a
// group of CG CTAs that share it (CG = 2: a pair computes 2 x 128 rows; CTA r takes
// row tile CG*tmc + r).  Blocks of GROUP_M row tiles sweep the column tiles
// together, so the ~148 tiles in flight share a few A and B panels in L2.
template <int TBN, int CG>
__device__ __forceinline__ Tile decode_tile(const GemmArgs& g, uint64_t t, uint32_t rank) {
    Tile c;
    // t < batch * tiles_mc * tiles_n < 2^32 (checked at launch): 32-bit multiply-high divisions
    const uint32_t t32 = (uint32_t)t;
    c.z = g.fd_z.div(t32);
    const uint32_t local_t = t32 - c.z * g.fd_z.d;
    const uint32_t group = g.fd_group.div(local_t);
    const uint32_t first_m = group * GROUP_M;
    const uint32_t local = local_t - group * g.fd_group.d;
    uint32_t tmq, tnq;
    if (g.tiles_mc - first_m >= GROUP_M) {           // a full group: power-of-two size
        tmq = local % GROUP_M;
        tnq = local / GROUP_M;
    } else {                                         // the last, partial group
        const uint32_t gsize = g.tiles_mc - first_m;
        tnq = local / gsize;
        tmq = local - tnq * gsize;
    }
    const uint32_t tm = (first_m + tmq) * CG + rank;
    c.m0 = tm * BM;
    c.n0 = tnq * TBN;
    c.ba = g.a_batches == 1 ? 0u : c.z;
    c.bb = g.b_batches == 1 ? 0u : c.z;
    c.cw0 = c.ch0 = c.cn0 = 0;
    if (g.conv) {
        const uint32_t tn = g.fd_hw.div(tm), rem = tm - tn * g.fd_hw.d;
        const uint32_t th = g.fd_w.div(rem);
        c.cn0 = tn << g.bn_log;
        c.ch0 = th << g.bh_log;
        c.cw0 = (rem - th * g.fd_w.d) << g.bw_log;
    }
    return c;
}

// Work unit u: its tile and its share [kb0, kb1) of the tile's K blocks.
struct Unit {
    uint32_t t, sp, kb0, kb1;
};
template <bool KS>
__device__ __forceinline__ Unit decode_unit(const GemmArgs& g, uint64_t u) {
    if constexpr (!KS) return Unit{(uint32_t)u, 0u, 0u, g.num_kb};
    Unit r;
    const uint32_t u32 = (uint32_t)u;               // units < 2^32 (checked at launch)
    r.t = g.fd_split.div(u32);
    r.sp = u32 - r.t * g.fd_split.d;
    r.kb0 = g.fd_split.div(r.sp * g.num_kb);
    r.kb1 = g.fd_split.div((r.sp + 1u) * g.num_kb);
    return r;
}

// Column terms of output columns col0 .. col0+15 (0 past the last column): four 16-byte
// loads for a full, aligned chunk.
__device__ __forceinline__ void load_colterms(const int32_t* ct, uint32_t col0, uint32_t cols, uint32_t (&cv)[16]) {
    if (col0 + 16u <= cols && ((uintptr_t)(ct + col0) & 15u) == 0) {
        const int4* c4 = (const int4*)(ct + col0);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const int4 x = __ldg(c4 + v);
            cv[4 * v] = (uint32_t)x.x; cv[4 * v + 1] = (uint32_t)x.y;
            cv[4 * v + 2] = (uint32_t)x.z; cv[4 * v + 3] = (uint32_t)x.w;
        }
    } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) cv[k] = col0 + k < cols ? (uint32_t)__ldg(ct + col0 + k) : 0u;
    }
}

// Output pixel (n, oh, ow) of tile row i of a conv tile: rows are (image, row, column),
// or (row, image, column) in the window form.
__device__ __forceinline__ void conv_pixel(const GemmArgs& g, const Tile& tc, uint32_t i, uint32_t& n, uint32_t& oh,
                                           uint32_t& ow) {
    ow = tc.cw0 + (i & ((1u << g.bw_log) - 1u));
    if (g.win) {
        n = tc.cn0 + ((i >> g.bw_log) & ((1u << g.bn_log) - 1u));
        oh = tc.ch0 + (i >> (g.bw_log + g.bn_log));
    } else {
        oh = tc.ch0 + ((i >> g.bw_log) & ((1u << g.bh_log) - 1u));
        n = tc.cn0 + (i >> (g.bw_log + g.bh_log));
    }
}

// Persistent kernel: one CTA per SM (CG = 1), or one CTA pair per two SMs
// (CG = 2, a 2-CTA cluster), walking tiles cluster, +clusters, ...
//   warp 0      TMA producer (continuous stage ring across tiles)
//   warp 1      TMEM owner; lane 0 (of the pair's even CTA) issues the MMAs of each
//               tile into an accumulator buffer once the epilogue has drained it
//   warps 2-17  epilogue: warp w reads TMEM lanes 32*(w%4).. of column group (w-2)/4,
//               combines the four accumulators
//               into registers, releases the buffer,
//               then adds the rank-1 terms, narrows and stores while the next
//               tile's MMAs run.
// CTA pairs (tcgen05 cta_group::2, M = 256): each CTA loads its own 128 rows of A
// (both planes) and ONE plane of B (even CTA Bh, odd CTA Bl); one MMA per plane of A
// multiplies the pair's 256 rows by [Bh | Bl], each CTA's TMEM receiving its own rows'
// accumulators.  Per CTA and 32-deep K step that is 8 KB of A and 8 KB of B read for
// 256 tensor cycles, against 24 KB for a single CTA -- the shared-memory traffic the
// single-CTA kernel is bound by.  All TMA completions and epilogue releases go to the
// even CTA's barriers; its MMA commits arrive on both CTAs' barriers (multicast
// commit).  No TMA multicast is used.
template <int TBN, int CG, bool WA = false, bool WIN = false, bool KS = false>
__global__ void __launch_bounds__(Cfg<TBN, CG, WA>::THREADS, 1)
    gemm_q88_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs g) {
    griddep_wait();
    griddep_launch_dependents();   // all CTAs are resident: the next kernel may launch now
    uint64_t clk_c0 = 0, clk_t0 = 0;
    if (g.clk && blockIdx.x == 0 && threadIdx.x == 0) { clk_c0 = clock64(); clk_t0 = gtimer(); }
    using C = Cfg<TBN, CG, WA>;
    static_assert(!WIN || (TBN == 64 && CG == 1 && !WA), "the window form runs packed 64-column tiles");
    static_assert(!KS || (!WA && !WIN), "K-split units run the row-major epilogue");
    constexpr int NBUF = C::NBUF;
    constexpr uint32_t HALF = TBN / (C::EPI_WARPS / 4);  // columns per epilogue warp
    constexpr uint32_t CW = 16;                           // columns per TMEM load
    // the window form's stage count and size come with the launch; its resident weights
    // come first in shared memory
    const uint32_t STAGES = WIN ? g.win_stages : (uint32_t)C::STAGES;
    const uint32_t STAGE_B = WIN ? g.win_bytes : (uint32_t)C::STAGE;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* stg = WIN ? smem + g.w_bytes : smem;
    uint64_t* bars = (uint64_t*)(stg + STAGES * STAGE_B);
    // bars: [0,S) full, [S,2S) empty, [2S,2S+NBUF) acc_full, [2S+NBUF,2S+2NBUF) acc_empty, then
    // done, then (window form) the resident weights' barrier
    uint64_t* full_b = bars;
    uint64_t* empty_b = bars + STAGES;
    uint64_t* accf_b = bars + 2 * STAGES;
    uint64_t* acce_b = accf_b + NBUF;
    uint64_t* done_b = acce_b + NBUF;
    uint64_t* wbar = done_b + 1;
    volatile uint32_t* tmem_slot = (volatile uint32_t*)(wbar + 1);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
    const bool leader = rank == 0;
    const uint64_t cid = blockIdx.x / CG, ncl = gridDim.x / CG;
    // work units: tiles x K-split units per tile (1 but for K-split launches)
    const uint64_t total = (uint64_t)g.batch * g.tiles_mc * g.tiles_n * (KS ? g.splits : 1u);
    constexpr uint16_t kPairMask = 0x3;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full_b[s]), 1);
            mbar_init(smem_u32(&empty_b[s]), 1);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(smem_u32(&accf_b[b]), 1);
            mbar_init(smem_u32(&acce_b[b]), C::EPI_WARPS * CG);
        }
        mbar_init(smem_u32(done_b), 1);
        mbar_init(smem_u32(wbar), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        if (CG == 2)
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)),
                         "r"(TMEM_COLS)
                         : "memory");
        else
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)),
                         "r"(TMEM_COLS)
                         : "memory");
        if (CG == 2) asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        else asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    if (CG == 2) cluster_sync_all();      // both CTAs' barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const WaitCtl wc{abort_flag, g.status, g.timeout_ns};

    if (WIN && warp == 0) {
        if (lane == 0) {
            // the packed weights once, then per tile and K block one window box (both planes)
            mbar_expect_tx(smem_u32(wbar), g.w_bytes);
            for (uint32_t j = 0; j < g.w_bytes / (uint32_t)PLANE_TILE; ++j)
                tma_load_4d(smem_u32(smem + j * PLANE_TILE), &tmB, smem_u32(wbar), 0, (int)(j * BK), 0, 0);
            uint32_t it = 0;
            for (uint64_t t = cid; t < total && !*abort_flag; t += ncl) {
                const Tile tc = decode_tile<TBN, CG>(g, t, rank);
                for (uint32_t kb = 0; kb < g.kb_per_r; ++kb, ++it) {
                    const uint32_t s = it % STAGES, round = it / STAGES;
                    if (!mbar_wait(smem_u32(&empty_b[s]), (round & 1u) ^ 1u, wc)) break;
                    const uint32_t full = smem_u32(&full_b[s]);
                    mbar_expect_tx(full, STAGE_B);
                    tma_load_5d(smem_u32(stg + s * STAGE_B), &tmA, full, (int)(kb * BK), (int)(tc.cw0 * g.sw),
                                (int)tc.cn0, (int)(tc.ch0 * g.sh), 0);
                }
            }
            // let the copies still in flight land before the CTA exits
            volatile int never = 0;
            WaitCtl drain{&never, g.status, g.timeout_ns};
            mbar_wait(smem_u32(wbar), 0, drain);
            if (*abort_flag) {
                const uint32_t first = it > STAGES ? it - STAGES : 0u;
                for (uint32_t k = first; k < it; ++k) mbar_wait(smem_u32(&full_b[k % STAGES]), (k / STAGES) & 1u, drain);
            }
        }
    } else if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (uint64_t t = cid; t < total && !*abort_flag; t += ncl) {
                uint32_t tt = 0, kb_lo = 0, kb_hi = 0;    // K-split: this unit's tile and K blocks
                if constexpr (KS) {
                    const Unit un = decode_unit<true>(g, t);
                    tt = un.t; kb_lo = un.kb0; kb_hi = un.kb1;
                }
                const Tile tc = decode_tile<TBN, CG>(g, KS ? (uint64_t)tt : t, rank);
                for (uint32_t kb = KS ? kb_lo : 0u; kb < (KS ? kb_hi : g.num_kb); ++kb, ++it) {
                    const uint32_t s = it % STAGES, round = it / STAGES;
                    if (!mbar_wait(smem_u32(&empty_b[s]), (round & 1u) ^ 1u, wc)) break;
                    uint8_t* st = stg + s * STAGE_B;
                    if (CG == 2) {
                        const uint32_t full = map_to_rank(smem_u32(&full_b[s]), 0);   // the pair leader's barrier
                        if (leader) mbar_expect_tx(smem_u32(&full_b[s]), CG * C::STAGE);
                        if (g.conv) {
                            const uint32_t r = kb / g.kb_per_r, kk = (kb - r * g.kb_per_r) * BK;
                            const int c1 = (int)(tc.cw0 * g.sw), c2 = (int)(tc.ch0 * g.sh + r * g.dh);
                            tma_load_5d_pair(smem_u32(st), &tmA, full, (int)kk, c1, c2, (int)tc.cn0, 0);
                            tma_load_5d_pair(smem_u32(st + PLANE_TILE), &tmA, full, (int)kk, c1, c2, (int)tc.cn0, 1);
                        } else {
                            tma_load_4d_pair(smem_u32(st), &tmA, full, (int)(kb * BK), (int)tc.m0, 0, (int)tc.ba);
                        }
                        tma_load_4d_pair(smem_u32(st + OPERAND_TILE), &tmB, full, (int)tc.n0, (int)(kb * BK), (int)rank,
                                         (int)tc.bb);
                    } else {
                        const uint32_t full = smem_u32(&full_b[s]);
                        mbar_expect_tx(full, C::STAGE);
                        if (g.conv) {
                            const uint32_t r = kb / g.kb_per_r, kk = (kb - r * g.kb_per_r) * BK;
                            const int c1 = (int)(tc.cw0 * g.sw), c2 = (int)(tc.ch0 * g.sh + r * g.dh);
                            tma_load_5d(smem_u32(st), &tmA, full, (int)kk, c1, c2, (int)tc.cn0, 0);
                            tma_load_5d(smem_u32(st + PLANE_TILE), &tmA, full, (int)kk, c1, c2, (int)tc.cn0, 1);
                        } else {
                            tma_load_4d(smem_u32(st), &tmA, full, (int)(kb * BK), (int)tc.m0, 0, (int)tc.ba);
                        }
                        if (WA) tma_load_4d(smem_u32(st + OPERAND_TILE), &tmB, full, (int)(kb * BK), 0, 0, 0);   // weight rows
                        else tma_load_4d(smem_u32(st + OPERAND_TILE), &tmB, full, (int)tc.n0, (int)(kb * BK), 0, (int)tc.bb);
                    }
                }
            }
            if (*abort_flag && leader) {
                // let copies already in flight land before the CTA exits (a pair's copies
                // all complete on the leader's barriers)
                const uint32_t first = it > STAGES ? it - STAGES : 0u;
                volatile int never = 0;
                WaitCtl drain{&never, g.status, g.timeout_ns};
                for (uint32_t k = first; k < it; ++k) mbar_wait(smem_u32(&full_b[k % STAGES]), (k / STAGES) & 1u, drain);
            }
        }
    } else if (WIN && warp == 1) {
        if (lane == 0) {
            uint32_t j = 0, s = 0, phase = 0;
            const WaitCtl wcw = wc;
            bool ok = mbar_wait(smem_u32(wbar), 0, wcw);     // resident weights landed
            tc_fence_after();
            const WinIssue w{sdesc(smem_u32(stg)), sdesc_n(smem_u32(smem)), STAGE_B >> 4, g.win_roff >> 4,
                             g.win_plane >> 4, STAGES};
            const uint32_t kh = g.kh, kbr = g.kb_per_r;
            const uint32_t last = g.ksteps - (kbr - 1u) * (BK / 32u);   // 32-deep steps in a row's last block
            const uint32_t shape = kh == 3 && kbr == 2 && last == 2 ? 1u : kh == 2 && kbr == 1 && last == 4 ? 2u : 0u;
            constexpr uint32_t NOFF = 2 * TBN, ID = C::IDESC;
            for (uint64_t t = cid; ok && t < total; t += ncl, ++j) {
                const uint32_t buf = j % NBUF, use = j / NBUF;
                if (!mbar_wait(smem_u32(&acce_b[buf]), (use & 1u) ^ 1u, wc)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * C::ACC_COLS;
                if (shape == 1) ok = win_tile<3, 2, 2, NOFF, ID>(d, w, kh, kbr, last, s, phase, full_b, empty_b, wc);
                else if (shape == 2) ok = win_tile<2, 1, 4, NOFF, ID>(d, w, kh, kbr, last, s, phase, full_b, empty_b, wc);
                else ok = win_tile<0, 0, 0, NOFF, ID>(d, w, kh, kbr, last, s, phase, full_b, empty_b, wc);
                if (ok) umma_commit(smem_u32(&accf_b[buf]));
            }
            umma_commit(smem_u32(done_b));
            volatile int never = 0;
            WaitCtl drain{&never, g.status, g.timeout_ns};
            mbar_wait(smem_u32(done_b), 0, drain);
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            uint32_t it = 0, j = 0;
            bool ok = true;
            for (uint64_t t = cid; ok && t < total; t += ncl, ++j) {
                const uint32_t buf = j % NBUF, use = j / NBUF;
                if (!mbar_wait(smem_u32(&acce_b[buf]), (use & 1u) ^ 1u, wc)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * C::ACC_COLS;
                uint32_t kb_lo = 0, kb_hi = 0;            // K-split: this unit's K blocks
                if constexpr (KS) {
                    const Unit un = decode_unit<true>(g, t);
                    kb_lo = un.kb0; kb_hi = un.kb1;
                }
                for (uint32_t kb = KS ? kb_lo : 0u; kb < (KS ? kb_hi : g.num_kb); ++kb, ++it) {
                    const uint32_t s = it % STAGES, round = it / STAGES;
                    if (!mbar_wait(smem_u32(&full_b[s]), round & 1u, wc)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(stg + s * STAGE_B);
                    const uint32_t b0 = a0 + OPERAND_TILE;
                    // 32-deep steps of this block that hold any tap (the rest are zero in A and B)
                    const uint32_t steps = g.conv ? g.ksteps - (kb % g.kb_per_r) * (BK / 32) : g.ksteps - kb * (BK / 32);
#pragma unroll
                    for (uint32_t kk = 0; kk < BK / 32; ++kk) {
                        if (kk >= steps) break;
                        const uint64_t ah = sdesc(a0 + kk * 32), al = sdesc(a0 + PLANE_TILE + kk * 32);
                        const uint64_t bhl = sdesc_n(b0 + kk * 32 * 128);   // 32 K rows x [Bh | Bl]
                        const uint32_t acc = KS ? (uint32_t)(((kb - kb_lo) | kk) != 0u) : (uint32_t)((kb | kk) != 0u);
                        if (WA) {
                            // weights (A) x [hi pixels | lo' pixels] (B, 256 K-major rows)
                            umma_i8(d, sdesc(b0 + kk * 32), ah, C::IDESC, acc);
                        } else if (CG == 2) {
                            umma_i8_pair(d, ah, bhl, C::IDESC, acc);            // -> HH | HL (both CTAs)
                            umma_i8_pair(d + 2 * TBN, al, bhl, C::IDESC, acc);  // -> LH | LL
                        } else {
                            umma_i8(d, ah, bhl, C::IDESC, acc);                 // -> HH | HL
                            umma_i8(d + 2 * TBN, al, bhl, C::IDESC, acc);       // -> LH | LL
                        }
                    }
                    // frees the stage (in both CTAs of a pair) once these MMAs have read it
                    if (CG == 2) umma_commit_pair(smem_u32(&empty_b[s]), kPairMask);
                    else umma_commit(smem_u32(&empty_b[s]));
                }
                if (ok) {
                    if (CG == 2) umma_commit_pair(smem_u32(&accf_b[buf]), kPairMask);
                    else umma_commit(smem_u32(&accf_b[buf]));
                }
            }
            // every MMA issued by this thread has completed once `done` fires
            if (CG == 2) umma_commit_pair(smem_u32(done_b), 0x1);
            else umma_commit(smem_u32(done_b));
            volatile int never = 0;
            WaitCtl drain{&never, g.status, g.timeout_ns};
            mbar_wait(smem_u32(done_b), 0, drain);
        }
    } else if constexpr (WA) {
        // Outputs go to a plane image only (the host sends no NCHW output here).
        // TMEM lane = weight row: channel ch = 16*quarter + lane/2, hi plane in the even
        // lane, lo' plane in the odd one; columns = tile pixels (products with the pixels'
        // hi plane in columns 0..127, with their lo' plane in 128..255).  Per pixel
        // acc = 2^16*HH + 2^8*(HL + LH) + LL: the even lane holds HH and HL, the odd lane LH
        // and LL; of each 16-pixel chunk the even lane finishes pixels 0-7 and the odd lane
        // pixels 8-15, each taking its partner's partial sums by one shuffle per pixel.
        const uint32_t quarter = warp & 3u;
        const uint32_t cgrp = (warp - 2) >> 2;               // tile pixels 32*cgrp .. +31
        const uint32_t odd = lane & 1u;
        const uint32_t ch = 16u * quarter + (lane >> 1);
        const uint32_t m1 = odd ? 256u : 65536u, m2 = odd ? 1u : 256u;
        int16_t* xb = (int16_t*)(smem + STAGES * C::STAGE + 256) + (warp - 2) * 256;
        const uint32_t bwm = (1u << g.bw_log) - 1u, bhm = (1u << g.bh_log) - 1u, bsh = g.bw_log + g.bh_log;
        const bool cvalid = ch < g.cols;
        const uint32_t ct = cvalid ? (uint32_t)__ldg(g.colterm + ch) : 0u;
        const bool prl = (g.epi & 2u) && g.rpl;               // residual read from a plane image
        // channels 8*odd .. +7 of this quarter in the pixel-major phase
        const uint32_t cl0 = 16u * quarter + 8u * odd;
        const uint32_t live = g.cols > cl0 ? min(8u, g.cols - cl0) : 0u;
        const bool qlive = 16u * quarter < g.cols;
        uint32_t j = 0;
        for (uint64_t t = cid; t < total; t += ncl, ++j) {
            const uint32_t buf = j % NBUF, use = j / NBUF;
            const Tile tc = decode_tile<TBN, CG>(g, t, rank);
            // this thread's two runs of 8 pixels (tile pixels i0 .. i0+7, one image row: bw >= 8),
            // their row terms and residual words, fetched while the tile's MMAs run
            uint32_t nv[2];
            uint64_t ooff[2];
            uint32_t rt[2][8];
            uint4 rs[2];
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
                const uint32_t i0 = 32u * cgrp + 16u * h + 8u * odd;
                const uint32_t ow = tc.cw0 + (i0 & bwm);
                const uint32_t oh = tc.ch0 + ((i0 >> g.bw_log) & bhm);
                const uint32_t n = tc.cn0 + (i0 >> bsh);
                nv[h] = (oh < g.out_h && n < g.nimg && ow < g.out_w) ? min(8u, g.out_w - ow) : 0u;
                const uint64_t pix = (uint64_t)oh * g.out_w + ow;
                const uint64_t ri = (uint64_t)n * g.out_h * g.out_w + pix;
                ooff[h] = (uint64_t)n * g.out_bs + pix;
                if (nv[h] == 8u && (ri & 3u) == 0) {
                    const int4 a = __ldg((const int4*)(g.rowterm + ri)), b = __ldg((const int4*)(g.rowterm + ri + 4));
                    rt[h][0] = (uint32_t)a.x; rt[h][1] = (uint32_t)a.y; rt[h][2] = (uint32_t)a.z; rt[h][3] = (uint32_t)a.w;
                    rt[h][4] = (uint32_t)b.x; rt[h][5] = (uint32_t)b.y; rt[h][6] = (uint32_t)b.z; rt[h][7] = (uint32_t)b.w;
                } else {
#pragma unroll
                    for (uint32_t k = 0; k < 8; ++k) rt[h][k] = k < nv[h] ? (uint32_t)__ldg(g.rowterm + ri + k) : 0u;
                }
                rs[h] = make_uint4(0, 0, 0, 0);
                if ((g.epi & 2u) && !g.rpl && cvalid && nv[h]) {
                    const int16_t* src = g.resid + ooff[h] + (uint64_t)ch * g.ldc;
                    if (nv[h] == 8u && ((uintptr_t)src & 15u) == 0) {
                        rs[h] = __ldg((const uint4*)src);
                    } else {
                        uint32_t w4[4] = {0, 0, 0, 0};
#pragma unroll
                        for (uint32_t k = 0; k < 8; ++k)
                            if (k < nv[h]) w4[k / 2] |= (uint32_t)(uint16_t)__ldg(src + k) << (16 * (k & 1));
                        rs[h] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                }
            }
            // a residual plane image: this lane's pixel-major runs (8 channels of pixel lane/2
            // of each chunk), as hi and lo' bytes
            uint2 rh[2], rl[2];
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
                rh[h] = make_uint2(0, 0);
                rl[h] = make_uint2(0x80808080u, 0x80808080u);
                if (prl && live) {
                    const uint32_t i = 32u * cgrp + 16u * h + (lane >> 1);
                    const uint32_t ow = tc.cw0 + (i & bwm), oh = tc.ch0 + ((i >> g.bw_log) & bhm), n = tc.cn0 + (i >> bsh);
                    if (ow < g.out_w && oh < g.out_h && n < g.nimg) {
                        const int8_t* src =
                            g.rpl + (((uint64_t)n * g.rpl_Hp + oh + g.rpl_pt) * g.rpl_Wp + ow + g.rpl_pl) * g.rpl_Cp + cl0;
                        rh[h] = __ldg((const uint2*)src);
                        rl[h] = __ldg((const uint2*)(src + g.rpl_plane));
                    }
                }
            }
            uint32_t ok = 0;
            if (lane == 0) ok = (mbar_wait(smem_u32(&accf_b[buf]), use & 1u, wc) && !*abort_flag) ? 1u : 0u;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            __syncwarp();
            if (!ok) break;
            tc_fence_after();
            const uint32_t tl = tmem + buf * C::ACC_COLS + ((quarter * 32u) << 16) + 32u * cgrp;
            uint32_t v[2][4];
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
                uint32_t dh[16], dl[16];
                tmem_ld16(tl + 16u * h, dh);
                tmem_ld16(tl + 128u + 16u * h, dl);
                tmem_ld_wait();
                uint32_t acc[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint32_t p0 = dh[k] * m1 + dl[k] * m2, p1 = dh[k + 8] * m1 + dl[k + 8] * m2;
                    const uint32_t other = __shfl_xor_sync(0xFFFFFFFFu, odd ? p0 : p1, 1);
                    acc[k] = (odd ? p1 : p0) + other + rt[h][k] + ct;
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) v[h][q] = narrow_pack(acc[2 * q], acc[2 * q + 1]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acce_b[buf]));   // buffer free for the next tile
            if (!prl) {
                // channel-major: residual words (NCHW), ReLU
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    if (g.epi & 2u) {
                        v[h][0] = __vaddss2(v[h][0], rs[h].x); v[h][1] = __vaddss2(v[h][1], rs[h].y);
                        v[h][2] = __vaddss2(v[h][2], rs[h].z); v[h][3] = __vaddss2(v[h][3], rs[h].w);
                    }
                    if (g.epi & 1u) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) v[h][q] = __vmaxs2(v[h][q], 0u);
                    }
                }
            }
            {
                // pixel-major: each 16-pixel x 16-channel chunk through the warp's buffer;
                // lane -> pixel lane/2 of the chunk, channels cl0 .. cl0+7
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    __syncwarp();
#pragma unroll
                    for (uint32_t k = 0; k < 8; ++k)
                        xb[(8u * odd + k) * 16u + (lane >> 1)] = (int16_t)(uint16_t)(v[h][k / 2] >> (16 * (k & 1)));
                    __syncwarp();
                    const uint4 w = *(const uint4*)(xb + (lane >> 1) * 16u + 8u * odd);
                    uint32_t pw[4] = {w.x, w.y, w.z, w.w};
                    const uint32_t i = 32u * cgrp + 16u * h + (lane >> 1);
                    const uint32_t ow = tc.cw0 + (i & bwm), oh = tc.ch0 + ((i >> g.bw_log) & bhm), n = tc.cn0 + (i >> bsh);
                    const bool pv = ow < g.out_w && oh < g.out_h && n < g.nimg;
                    if (prl) {
                        const uint32_t h4[2] = {rh[h].x, rh[h].y}, l4[2] = {rl[h].x ^ 0x80808080u, rl[h].y ^ 0x80808080u};
#pragma unroll
                        for (uint32_t q = 0; q < 2; ++q) {
                            pw[2 * q] = __vaddss2(pw[2 * q], __byte_perm(l4[q], h4[q], 0x5140));
                            pw[2 * q + 1] = __vaddss2(pw[2 * q + 1], __byte_perm(l4[q], h4[q], 0x7362));
                        }
                        if (g.epi & 1u) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) pw[q] = __vmaxs2(pw[q], 0u);
                        }
                    }
                    {
                        const uint64_t pix = ((uint64_t)n * g.po_Hp + oh + g.po_pt) * g.po_Wp + ow + g.po_pl;
                        int32_t sum = 0;
                        if (pv && qlive) {
                            // channels past the output hold x = 0 (hi 0, lo' -128), not in the sum
#pragma unroll
                            for (uint32_t q = 0; q < 4; ++q) {
                                if (2 * q >= live) pw[q] &= 0xFFFF0000u;
                                if (2 * q + 1 >= live) pw[q] &= 0x0000FFFFu;
                            }
                            const uint32_t h0 = __byte_perm(pw[0], pw[1], 0x7531), h1 = __byte_perm(pw[2], pw[3], 0x7531);
                            const uint32_t l0 = __byte_perm(pw[0], pw[1], 0x6420) ^ 0x80808080u;
                            const uint32_t l1 = __byte_perm(pw[2], pw[3], 0x6420) ^ 0x80808080u;
                            const int sh = __dp4a((int)h1, 0x01010101, __dp4a((int)h0, 0x01010101, 0));
                            const int sl = __dp4a((int)l1, 0x01010101, __dp4a((int)l0, 0x01010101, 0));
                            sum = 256 * sh + sl + 128 * (int32_t)(8u - live);
                            int8_t* dst = g.po + pix * g.po_Cp + cl0;
                            *(uint2*)dst = make_uint2(h0, h1);
                            *(uint2*)(dst + g.po_plane) = make_uint2(l0, l1);
                        }
                        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
                        if (!odd && pv && qlive) atomicAdd(g.po_S + pix, sum);
                    }
                }
            }
        }
    } else {
        const uint32_t quarter = warp & 3u;
        const uint32_t half = (warp - 2) >> 2;
        const uint32_t i = quarter * 32 + lane;           // TMEM lane = A tile row
        const uint32_t cbase = half * HALF;
        uint32_t j = 0;
        for (uint64_t t = cid; t < total; t += ncl, ++j) {
            const uint32_t buf = j % NBUF, use = j / NBUF;
            // Everything that does not depend on the accumulator is fetched before the
            // wait, while the tile's MMAs run: the row's output offset, its row term and
            // the epilogue's addends (residual words or the bias row), packed in pairs.
            const Unit un = decode_unit<KS>(g, t);
            const Tile tc = decode_tile<TBN, CG>(g, KS ? (uint64_t)un.t : t, rank);
            bool valid;
            uint64_t rt_idx, o_off;
            if (g.conv) {
                uint32_t n, oh, ow;
                conv_pixel(g, tc, i, n, oh, ow);
                valid = ow < g.out_w && oh < g.out_h && n < g.nimg;
                const uint64_t pix = (uint64_t)oh * g.out_w + ow;
                rt_idx = (uint64_t)n * g.out_h * g.out_w + pix;
                o_off = (uint64_t)n * g.out_bs + pix * g.ldo;     // NCHW: ldo 1; channels-last: ldo = cols
            } else {
                const uint32_t row = tc.m0 + i;
                valid = row < g.rows;
                rt_idx = (uint64_t)tc.ba * g.rows + row;
                if (g.rows_per_img) {
                    const uint32_t n = row / g.rows_per_img;
                    o_off = (uint64_t)n * g.out_bs + (row - n * g.rows_per_img);
                } else {
                    o_off = (uint64_t)tc.z * g.out_bs + (uint64_t)row * g.ldo;
                }
            }
            const uint32_t rt = valid ? (uint32_t)__ldg(g.rowterm + rt_idx) : 0u;
            uint32_t addv[HALF / 2];                      // addend pairs (even column in the low half)
            if ((g.epi & 2u) && g.rpl) {
                // residual words rebuilt from its plane image: per 16 channels one 16-byte hi
                // run and one lo' run, x = 256*hi + lo' + 128, pairs assembled by byte permutes
                uint32_t n, oh, ow;
                conv_pixel(g, tc, i, n, oh, ow);
                const uint64_t pix = ((uint64_t)n * g.rpl_Hp + oh + g.rpl_pt) * g.rpl_Wp + ow + g.rpl_pl;
#pragma unroll
                for (uint32_t c0 = 0; c0 < HALF; c0 += 16) {
                    const uint32_t col0 = tc.n0 + cbase + c0;
                    uint4 hv = make_uint4(0, 0, 0, 0), lv = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
                    if (valid && col0 < g.cols) {
                        const int8_t* src = g.rpl + pix * g.rpl_Cp + col0;
                        hv = __ldg((const uint4*)src);
                        lv = __ldg((const uint4*)(src + g.rpl_plane));
                    }
                    const uint32_t h4[4] = {hv.x, hv.y, hv.z, hv.w};
                    const uint32_t l4[4] = {lv.x ^ 0x80808080u, lv.y ^ 0x80808080u, lv.z ^ 0x80808080u, lv.w ^ 0x80808080u};
#pragma unroll
                    for (uint32_t q = 0; q < 4; ++q) {
                        addv[c0 / 2 + 2 * q] = __byte_perm(l4[q], h4[q], 0x5140);
                        addv[c0 / 2 + 2 * q + 1] = __byte_perm(l4[q], h4[q], 0x7362);
                    }
                }
            } else if (g.epi & 6u) {
                const bool res = (g.epi & 2u) != 0u;
                const int16_t* src = res ? g.resid + o_off : g.resid;
                const uint64_t step = res ? g.ldc : 1u;
#pragma unroll
                for (uint32_t q = 0; q < HALF / 2; ++q) {
                    const uint32_t col = tc.n0 + cbase + 2 * q;
                    const uint32_t a0 = valid && col < g.cols ? (uint16_t)__ldg(src + (uint64_t)col * step) : 0u;
                    const uint32_t a1 = valid && col + 1 < g.cols ? (uint16_t)__ldg(src + (uint64_t)(col + 1) * step) : 0u;
                    addv[q] = a0 | (a1 << 16);
                }
            }
            // One lane waits; the verdict is broadcast so that the .sync.aligned
            // TMEM loads below are executed by the whole warp or not at all.
            uint32_t ok = 0;
            if (lane == 0) ok = (mbar_wait(smem_u32(&accf_b[buf]), use & 1u, wc) && !*abort_flag) ? 1u : 0u;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            __syncwarp();
            if (!ok) break;
            tc_fence_after();
            const int32_t* ct = g.colterm + (uint64_t)tc.bb * g.cols;
            // Drain: acc = 2^16*HH + 2^8*(HL + LH) + LL + rowterm + colterm, narrowed
            // and packed two int16 per word (even column in the low half).
            uint32_t pk[HALF / 2];
            const uint32_t tl = tmem + buf * C::ACC_COLS + ((quarter * 32u) << 16) + cbase;
            if constexpr (KS) {
                // the raw product sums 2^16*HH + 2^8*(HL + LH) + LL of this unit's K blocks into
                // its slab (column-major, so that a warp's stores are 128-byte runs of rows)
                int32_t* slab = g.ws + (((uint64_t)un.t * CG + rank) * g.splits + un.sp) * (uint64_t)(TBN * BM) + i;
#pragma unroll
                for (uint32_t c0 = 0; c0 < HALF; c0 += CW) {
                    if (tc.n0 + cbase + c0 < g.cols) {
                        uint32_t p[CW], q[CW];
                        tmem_ld16(tl + c0, p);
                        tmem_ld16(tl + TBN + c0, q);
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k) p[k] = (p[k] << 8) + q[k];
                        tmem_ld16(tl + 2 * TBN + c0, q);
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k) p[k] = (p[k] + q[k]) << 8;
                        tmem_ld16(tl + 3 * TBN + c0, q);
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k) __stcg(slab + (uint64_t)(cbase + c0 + k) * BM, (int)(p[k] + q[k]));
                    }
                }
            } else {
#pragma unroll
                for (uint32_t c0 = 0; c0 < HALF; c0 += CW) {
                    const uint32_t col0 = tc.n0 + cbase + c0;
                    if (col0 < g.cols) {
                        uint32_t p[CW], q[CW], cv[CW];
                        tmem_ld16(tl + c0, p);
                        tmem_ld16(tl + TBN + c0, q);
                        // column terms: four 16-byte loads for a full, aligned chunk
                        if (col0 + CW <= g.cols && ((uintptr_t)(ct + col0) & 15u) == 0) {
                            const int4* c4 = (const int4*)(ct + col0);
#pragma unroll
                            for (int v = 0; v < (int)CW / 4; ++v) {
                                const int4 x = __ldg(c4 + v);
                                cv[4 * v] = (uint32_t)x.x; cv[4 * v + 1] = (uint32_t)x.y;
                                cv[4 * v + 2] = (uint32_t)x.z; cv[4 * v + 3] = (uint32_t)x.w;
                            }
                        } else {
#pragma unroll
                            for (int k = 0; k < (int)CW; ++k) cv[k] = col0 + k < g.cols ? (uint32_t)__ldg(ct + col0 + k) : 0u;
                        }
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k) p[k] = (p[k] << 8) + q[k];
                        tmem_ld16(tl + 2 * TBN + c0, q);
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k) p[k] = (p[k] + q[k]) << 8;
                        tmem_ld16(tl + 3 * TBN + c0, q);
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < (int)CW; k += 2)
                            pk[(c0 + k) / 2] = narrow_pack(p[k] + q[k] + rt + cv[k], p[k + 1] + q[k + 1] + rt + cv[k + 1]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {                                      // buffer free for the next tile
                if (CG == 2) mbar_arrive_cluster(map_to_rank(smem_u32(&acce_b[buf]), 0));
                else mbar_arrive(smem_u32(&acce_b[buf]));
            }
            if constexpr (KS) {
                // The warp whose slab completes the tile's set adds the slabs up (int32 wrap:
                // exact in any order) and finishes the tile; the others are done with it.
                // Nothing waits: the slabs are published by a fence before the counter.
                __threadfence();
                __syncwarp();
                uint32_t last = 0;
                if (lane == 0) {
                    uint32_t* cnt = g.cnt + ((uint64_t)un.t * CG + rank) * C::EPI_WARPS + (warp - 2);
                    last = atomicAdd(cnt, 1u) == g.splits - 1u ? 1u : 0u;
                }
                last = __shfl_sync(0xFFFFFFFFu, last, 0);
                if (!last) continue;
                __threadfence();
#pragma unroll
                for (uint32_t c0 = 0; c0 < HALF; c0 += CW) {
                    const uint32_t col0 = tc.n0 + cbase + c0;
                    if (col0 < g.cols) {
                        uint32_t a[CW], cv[CW];
                        load_colterms(ct, col0, g.cols, cv);
                        const int32_t* sl =
                            g.ws + ((uint64_t)un.t * CG + rank) * g.splits * (uint64_t)(TBN * BM) + (uint64_t)(cbase + c0) * BM + i;
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k) a[k] = rt + cv[k];
                        for (uint32_t sp = 0; sp < g.splits; ++sp, sl += TBN * BM) {
#pragma unroll
                            for (int k = 0; k < (int)CW; ++k) a[k] += (uint32_t)__ldcg(sl + (uint64_t)k * BM);
                        }
#pragma unroll
                        for (int k = 0; k < (int)CW; k += 2) pk[(c0 + k) / 2] = narrow_pack(a[k], a[k + 1]);
                    }
                }
            }
            if (!valid) continue;
            // VectorOP ADD (saturating) and RELU on both halfwords of each pair
            if (g.epi & 6u) {
#pragma unroll
                for (uint32_t q = 0; q < HALF / 2; ++q) pk[q] = __vaddss2(pk[q], addv[q]);
            }
            if (g.epi & 1u) {
#pragma unroll
                for (uint32_t q = 0; q < HALF / 2; ++q) pk[q] = __vmaxs2(pk[q], 0u);
            }
            if (g.po) {
                // the output row as channels-last hi / lo' planes of the next conv's input,
                // 16 channels per 16-byte store, and its channel sum added into S
                uint32_t n, oh, ow;
                conv_pixel(g, tc, i, n, oh, ow);
                const uint64_t pix = ((uint64_t)n * g.po_Hp + oh + g.po_pt) * g.po_Wp + ow + g.po_pl;
                int32_t sum = 0;
#pragma unroll
                for (uint32_t c0 = 0; c0 < HALF; c0 += CW) {
                    const uint32_t col0 = tc.n0 + cbase + c0;
                    if (col0 >= g.cols) break;
                    const uint32_t live = min(CW, g.cols - col0);   // channels past the output hold x = 0
                    uint32_t hw[CW / 4], lw[CW / 4];
                    int32_t sh = 0, sl = 0;
#pragma unroll
                    for (uint32_t q = 0; q < CW / 4; ++q) {
                        uint32_t a = pk[(c0 + 4 * q) / 2], b = pk[(c0 + 4 * q) / 2 + 1];
                        if (4 * q + 4 > live) {
                            const uint32_t k0 = 4 * q;
                            if (k0 + 0 >= live) a &= 0xFFFF0000u;
                            if (k0 + 1 >= live) a &= 0x0000FFFFu;
                            if (k0 + 2 >= live) b &= 0xFFFF0000u;
                            if (k0 + 3 >= live) b &= 0x0000FFFFu;
                        }
                        hw[q] = __byte_perm(a, b, 0x7531);
                        lw[q] = __byte_perm(a, b, 0x6420) ^ 0x80808080u;
                        // x - 128 = 256*hi + lo': byte sums of both planes (signed)
                        sh = __dp4a((int)hw[q], 0x01010101, sh);
                        sl = __dp4a((int)lw[q], 0x01010101, sl);
                    }
                    // masked channels hold x = 0 (lo' = -128) and are not part of the sum
                    sum += 256 * sh + sl + 128 * (int32_t)(CW - live);
                    int8_t* dst = g.po + pix * g.po_Cp + col0;
#pragma unroll
                    for (uint32_t q = 0; q < CW / 16; ++q) {
                        *(uint4*)(dst + 16 * q) = make_uint4(hw[4 * q], hw[4 * q + 1], hw[4 * q + 2], hw[4 * q + 3]);
                        *(uint4*)(dst + g.po_plane + 16 * q) = make_uint4(lw[4 * q], lw[4 * q + 1], lw[4 * q + 2], lw[4 * q + 3]);
                    }
                }
                atomicAdd(g.po_S + pix, sum);
            }
            if (!g.out) continue;
            int16_t* orow = g.out + o_off;
#pragma unroll
            for (uint32_t c0 = 0; c0 < HALF; c0 += CW) {
                const uint32_t col0 = tc.n0 + cbase + c0;
                if (col0 >= g.cols) break;
                int16_t* dst = orow + col0;
                if (g.ldc != 1) {
                    // column-strided output (conv: y[m][p] with rows = pixels): each
                    // store is coalesced across the warp's consecutive rows
                    if (col0 + CW <= g.cols) {
                        int16_t* d = orow + (uint64_t)col0 * g.ldc;
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k, d += g.ldc)
                            *d = (int16_t)(uint16_t)(pk[(c0 + k) / 2] >> (16 * (k & 1)));
                    } else {
#pragma unroll
                        for (int k = 0; k < (int)CW; ++k)
                            if (col0 + k < g.cols)
                                orow[(uint64_t)(col0 + k) * g.ldc] = (int16_t)(uint16_t)(pk[(c0 + k) / 2] >> (16 * (k & 1)));
                    }
                } else if (col0 + CW <= g.cols && ((uintptr_t)dst & 15u) == 0) {
                    uint4* d4 = (uint4*)dst;
#pragma unroll
                    for (int q = 0; q < (int)CW / 8; ++q)
                        d4[q] = make_uint4(pk[c0 / 2 + 4 * q], pk[c0 / 2 + 4 * q + 1], pk[c0 / 2 + 4 * q + 2],
                                           pk[c0 / 2 + 4 * q + 3]);
                } else {
#pragma unroll
                    for (int k = 0; k < (int)CW; ++k)
                        if (col0 + k < g.cols) dst[k] = (int16_t)(uint16_t)(pk[(c0 + k) / 2] >> (16 * (k & 1)));
                }
            }
        }
    }
    __syncthreads();
    if (g.clk && blockIdx.x == 0 && threadIdx.x == 0) {
        atomicAdd(g.clk, (unsigned long long)(clock64() - clk_c0));
        atomicAdd(g.clk + 1, (unsigned long long)(gtimer() - clk_t0));
    }
    // a pair's CTAs read each other's shared memory and barriers until here
    if (CG == 2) cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        if (CG == 2)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------
// int8 tensor-pipe rate (a measurement; no reference counterpart)
// ---------------------------------------------------------------------------
// The GEMM's main loop with the operand traffic taken away: every CTA (CG = 1) or
// CTA pair (CG = 2) issues `iters` rounds of the same MMAs on one operand stage that
// stays in shared memory (hashed bytes, so the data are not trivially zero), into
// the same TMEM accumulators.  The rate reached is the int8 tensor pipe's own
// ceiling at the clocks of the moment: the denominator of the GEMM's roofline.
template <int CG>
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(uint32_t iters, int* status, uint64_t timeout_ns,
                                                          unsigned long long* clk) {
    griddep_wait();
    using C = Cfg<128, CG>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* done_b = (uint64_t*)(smem + C::STAGE);
    volatile uint32_t* tmem_slot = (volatile uint32_t*)(done_b + 1);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
    for (uint32_t i = threadIdx.x; i < (uint32_t)C::STAGE / 4; i += blockDim.x) {
        uint32_t x = (i + 1u) * 0x9E3779B1u ^ (blockIdx.x * 0x85EBCA77u);
        x ^= x >> 15;
        x *= 0x2C1B3C6Du;
        x ^= x >> 12;
        ((uint32_t*)smem)[i] = x;
    }
    // the operand bytes were written through the generic proxy; the MMAs read them
    // through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(done_b), 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        if (CG == 2) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)),
                         "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)),
                         "r"(TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
        tc_fence_before();
    }
    __syncthreads();
    if (CG == 2) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the SM clock over the stream: clock64 ticks against %globaltimer nanoseconds
    unsigned long long c0 = 0, t0 = 0;
    if (threadIdx.x == 0) {
        asm volatile("mov.u64 %0, %%clock64;" : "=l"(c0));
        t0 = gtimer();
    }
    if (warp == 0 && lane == 0 && rank == 0) {
        const uint32_t a0 = smem_u32(smem), b0 = a0 + OPERAND_TILE;
        for (uint32_t it = 0; it < iters; ++it) {
#pragma unroll
            for (uint32_t kk = 0; kk < BK / 32; ++kk) {
                const uint64_t ah = sdesc(a0 + kk * 32), al = sdesc(a0 + PLANE_TILE + kk * 32);
                const uint64_t bhl = sdesc_n(b0 + kk * 32 * 128);
                const uint32_t acc = (it | kk) != 0u;
                if (CG == 2) {
                    umma_i8_pair(tmem, ah, bhl, C::IDESC, acc);
                    umma_i8_pair(tmem + 256, al, bhl, C::IDESC, acc);
                } else {
                    umma_i8(tmem, ah, bhl, C::IDESC, acc);
                    umma_i8(tmem + 256, al, bhl, C::IDESC, acc);
                }
            }
        }
        // arrives on `done` in both CTAs of a pair once every MMA above has completed
        if (CG == 2) umma_commit_pair(smem_u32(done_b), 0x3);
        else umma_commit(smem_u32(done_b));
    }
    if (threadIdx.x == 0) {
        const WaitCtl wc{abort_flag, status, timeout_ns};
        mbar_wait(smem_u32(done_b), 0, wc);
        if (blockIdx.x == 0 && clk) {
            unsigned long long c1;
            asm volatile("mov.u64 %0, %%clock64;" : "=l"(c1));
            clk[0] = c1 - c0;
            clk[1] = gtimer() - t0;
        }
    }
    __syncthreads();
    if (CG == 2) cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        if (CG == 2)
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
        else
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------
// split pre-passes
// ---------------------------------------------------------------------------

__device__ __forceinline__ int32_t word_sum_minus128(uint32_t u) {
    return (int32_t)(int16_t)(u & 0xFFFFu) + (int32_t)(int16_t)(u >> 16) - 256;
}

// One warp per (bt, row).
__global__ void __launch_bounds__(256) split_rows_kernel(const int16_t* __restrict__ src, uint64_t src_bs, uint64_t ld,
                                                         uint32_t rows, uint32_t K, uint32_t K_pad, uint64_t nrows_total,
                                                         int8_t* __restrict__ planes, int32_t* __restrict__ rowterm,
                                                         const int16_t* __restrict__ bias) {
    griddep_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t t = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < nrows_total; t += warps) {
        const uint64_t bt = t / rows, r = t - bt * rows;
        const int16_t* s = src + bt * src_bs + r * ld;
        int8_t* dh = planes + ((bt * 2 + 0) * rows + r) * (uint64_t)K_pad;
        int8_t* dl = planes + ((bt * 2 + 1) * rows + r) * (uint64_t)K_pad;
        int32_t sum = 0;
        uint32_t k_done = 0;
        if (((uintptr_t)s & 15u) == 0) {
            const uint32_t nv = K / 8;
            const uint4* s4 = (const uint4*)s;
            auto one = [&](const uint4& v, uint32_t i) {
                uint2 h, l;
                h.x = __byte_perm(v.x, v.y, 0x7531);
                h.y = __byte_perm(v.z, v.w, 0x7531);
                l.x = __byte_perm(v.x, v.y, 0x6420) ^ 0x80808080u;
                l.y = __byte_perm(v.z, v.w, 0x6420) ^ 0x80808080u;
                *(uint2*)(dh + 8 * (uint64_t)i) = h;
                *(uint2*)(dl + 8 * (uint64_t)i) = l;
                sum += word_sum_minus128(v.x) + word_sum_minus128(v.y) + word_sum_minus128(v.z) + word_sum_minus128(v.w);
            };
            // four 16-byte loads in flight per lane before their first use (one memory round
            // trip per 128 pieces of the row instead of per 32)
            uint32_t i = lane;
            for (; i + 96 < nv; i += 128) {
                uint4 v[4];
#pragma unroll
                for (uint32_t u = 0; u < 4; ++u) v[u] = __ldcs(s4 + i + 32 * u);
#pragma unroll
                for (uint32_t u = 0; u < 4; ++u) one(v[u], i + 32 * u);
            }
            for (; i < nv; i += 32) one(__ldcs(s4 + i), i);
            k_done = nv * 8;
        }
        for (uint32_t k = k_done + lane; k < K; k += 32) {
            const int16_t x = s[k];
            dh[k] = (int8_t)(x >> 8);
            dl[k] = (int8_t)((x & 255) - 128);
            sum += (int32_t)x - 128;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
        if (lane == 0) {
            uint32_t term = (uint32_t)sum * 128u + (uint32_t)K * 16384u;
            if (bias) term += (uint32_t)((int32_t)bias[r] * 256);
            rowterm[t] = (int32_t)term;
        }
    }
}

// B rows -> N-major planes.  Thread = 8 consecutive columns over a chunk of K:
// 16-byte loads and 8-byte plane stores, both coalesced along N; the column
// terms are summed in registers and added once per chunk.
// Plane layout: element (bt, p, k, c) at planes[bt*batch_pitch + p*plane_off + k*C_pad + c]
// (C_pad = row pitch): [2][K][C_pad] per batch, or packed [K][64 hi | 64 lo].
__global__ void __launch_bounds__(256) split_kn_kernel(const int16_t* __restrict__ src, uint64_t src_bs, uint64_t ld,
                                                       uint32_t cols, uint32_t K, uint32_t C_pad, uint32_t k_chunk,
                                                       uint64_t plane_off, uint64_t batch_pitch,
                                                       int8_t* __restrict__ planes, int32_t* __restrict__ colterm) {
    griddep_wait();
    const uint32_t bt = blockIdx.z;
    const uint32_t c8 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (c8 >= cols) return;
    const uint32_t k0 = blockIdx.y * k_chunk, k1 = min(K, k0 + k_chunk);
    const int16_t* sp = src + (uint64_t)bt * src_bs + c8;
    int8_t* dh = planes + (uint64_t)bt * batch_pitch + c8;
    int8_t* dl = dh + plane_off;
    int32_t sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const bool vec = c8 + 8 <= cols && ((uintptr_t)sp & 15u) == 0 && (ld & 7u) == 0;
    if (vec) {
        uint32_t k = k0;
        for (; k + 4 <= k1; k += 4) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldcs((const uint4*)(sp + (uint64_t)(k + u) * ld));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint64_t o = (uint64_t)(k + u) * C_pad;
                *(uint2*)(dh + o) = make_uint2(__byte_perm(v[u].x, v[u].y, 0x7531), __byte_perm(v[u].z, v[u].w, 0x7531));
                *(uint2*)(dl + o) = make_uint2(__byte_perm(v[u].x, v[u].y, 0x6420) ^ 0x80808080u,
                                               __byte_perm(v[u].z, v[u].w, 0x6420) ^ 0x80808080u);
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    sum[2 * j] += (int32_t)(int16_t)(w[j] & 0xFFFFu) - 128;
                    sum[2 * j + 1] += (int32_t)(int16_t)(w[j] >> 16) - 128;
                }
            }
        }
        for (; k < k1; ++k) {
            const uint4 v = __ldcs((const uint4*)(sp + (uint64_t)k * ld));
            const uint64_t o = (uint64_t)k * C_pad;
            *(uint2*)(dh + o) = make_uint2(__byte_perm(v.x, v.y, 0x7531), __byte_perm(v.z, v.w, 0x7531));
            *(uint2*)(dl + o) = make_uint2(__byte_perm(v.x, v.y, 0x6420) ^ 0x80808080u,
                                           __byte_perm(v.z, v.w, 0x6420) ^ 0x80808080u);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sum[2 * j] += (int32_t)(int16_t)(w[j] & 0xFFFFu) - 128;
                sum[2 * j + 1] += (int32_t)(int16_t)(w[j] >> 16) - 128;
            }
        }
    } else {
        const uint32_t nc = min(8u, cols - c8);
        for (uint32_t k = k0; k < k1; ++k) {
            const uint64_t o = (uint64_t)k * C_pad;
            for (uint32_t j = 0; j < nc; ++j) {
                const int16_t x = sp[(uint64_t)k * ld + j];
                dh[o + j] = (int8_t)(x >> 8);
                dl[o + j] = (int8_t)((x & 255) - 128);
                sum[j] += (int32_t)x - 128;
            }
        }
    }
    const uint32_t nc = min(8u, cols - c8);
    for (uint32_t j = 0; j < nc; ++j)
        atomicAdd((unsigned int*)(colterm + (uint64_t)bt * cols + c8 + j), (uint32_t)sum[j] * 128u);
}

// Launch-bound sizes: G consecutive lanes per output word (G a power of two,
// <= 32) take the k products q = lane, lane + G, ...; their int32 wrap sums
// meet by shuffle (addition mod 2^32 is order-free, so the result is the exact
// reference sum) and one narrowing follows (MatmulKernel.cpp:204-218).
// epi: bit 1 adds bias[j] (saturating), bit 0 applies ReLU, after the narrowing.
__global__ void __launch_bounds__(256) matmul_direct_kernel(const int16_t* __restrict__ a, const int16_t* __restrict__ b,
                                                            int16_t* __restrict__ c, uint32_t n, uint32_t k, uint32_t m,
                                                            uint64_t a_bs, uint64_t b_bs, uint64_t c_bs, uint64_t total,
                                                            uint32_t G, uint32_t epi, const int16_t* __restrict__ bias) {
    griddep_wait();
    const uint64_t nm = (uint64_t)n * m;
    const uint32_t g = threadIdx.x & (G - 1);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x / G;
    // whole warps iterate together (the shuffles below need every lane)
    for (uint64_t t0 = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / G; t0 < (total + stride - 1) / stride * stride;
         t0 += stride) {
        const bool live = t0 < total;
        const uint64_t t = live ? t0 : 0;
        const uint64_t z = t / nm, r = t - z * nm;
        const uint32_t i = (uint32_t)(r / m), j = (uint32_t)(r - (uint64_t)i * m);
        const int16_t* ar = a + z * a_bs + (uint64_t)i * k;
        const int16_t* bc = b + z * b_bs + j;
        uint32_t acc = 0;
        if (live)
            for (uint32_t q = g; q < k; q += G) acc += (uint32_t)((int32_t)__ldg(ar + q) * (int32_t)__ldg(bc + (uint64_t)q * m));
        for (uint32_t o = G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (live && g == 0) {
            int32_t v = narrow_acc(acc);
            if (epi & 2u) v = sat16(v + (int32_t)__ldg(bias + j));
            if (epi & 1u) v = max(v, 0);
            c[z * c_bs + (uint64_t)i * m + j] = (int16_t)v;
        }
    }
}

// The same products for a few rows (n <= NR): a block owns 32 consecutive output columns
// of one batch step (grid (ceil(m / 32), batch)); lane = column, so each load of a B row
// reads 32 adjacent words, the block's kRowWarps warps take every kRowWarps-th k (32 warps:
// a batch-1 layer's few blocks finish their k in few memory round trips), the A words are
// broadcast loads, and each lane keeps one int32 wrap sum per row.  The partial sums meet in
// shared memory (wrap addition: order-free) and warp 0 narrows, adds the epilogue and stores.  Batch steps run in parallel: their output slices do not overlap
// (overlapping ones take the in-order loop before the direct path).
constexpr uint32_t kRowWarps = 32;

template <int NR>
__global__ void __launch_bounds__(32 * kRowWarps) matmul_rows_direct_kernel(const int16_t* __restrict__ a,
                                                                 const int16_t* __restrict__ b, int16_t* __restrict__ c,
                                                                 uint32_t n, uint32_t k, uint32_t m, uint64_t a_bs,
                                                                 uint64_t b_bs, uint64_t c_bs, uint32_t epi,
                                                                 const int16_t* __restrict__ bias) {
    griddep_wait();
    __shared__ uint32_t part[kRowWarps][NR][32];
    const uint32_t lane = threadIdx.x & 31u, w = threadIdx.x >> 5;
    const uint32_t j = blockIdx.x * 32u + lane;
    const uint64_t z = blockIdx.y;
    const int16_t* A = a + z * a_bs;
    const int16_t* B = b + z * b_bs + j;
    uint32_t acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0;
    if (j < m) {
#pragma unroll 4
        for (uint32_t q = w; q < k; q += kRowWarps) {
            const int32_t bv = __ldg(B + (uint64_t)q * m);
#pragma unroll
            for (int r = 0; r < NR; ++r)
                if ((uint32_t)r < n) acc[r] += (uint32_t)((int32_t)__ldg(A + (uint64_t)r * k + q) * bv);
        }
    }
#pragma unroll
    for (int r = 0; r < NR; ++r) part[w][r][lane] = acc[r];
    __syncthreads();
    if (w == 0 && j < m) {
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if ((uint32_t)r >= n) break;
            uint32_t s = part[0][r][lane];
#pragma unroll
            for (int x = 1; x < (int)kRowWarps; ++x) s += part[x][r][lane];
            int32_t v = narrow_acc(s);
            if (epi & 2u) v = sat16(v + (int32_t)__ldg(bias + j));
            if (epi & 1u) v = max(v, 0);
            c[z * c_bs + (uint64_t)r * m + j] = (int16_t)v;
        }
    }
}

__global__ void fill_zero_kernel(int16_t* out, uint32_t rows, uint32_t cols, uint64_t ldo, uint64_t out_bs, uint64_t total) {
    griddep_wait();
    const uint64_t rc = (uint64_t)rows * cols;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t z = t / rc, rem = t - z * rc;
        const uint64_t r = rem / cols, c = rem - r * cols;
        out[z * out_bs + r * ldo + c] = 0;
    }
}

// ---------------------------------------------------------------------------
// host: tensor maps
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// planes [batches][2][rows][K_pad] int8; box {128 k, 128 rows, 2 planes, 1 batch}.
int make_plane_map(CUtensorMap* m, const int8_t* base, uint32_t K, uint32_t K_pad, uint32_t rows, uint32_t batches) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)base & 15u) != 0 || (K_pad & 15u) != 0) return set_error(CM_EINVAL, "plane buffer misaligned");
    const cuuint64_t dims[4] = {K, rows, 2, batches};
    const cuuint64_t strides[3] = {(cuuint64_t)K_pad, (cuuint64_t)rows * K_pad, (cuuint64_t)2 * rows * K_pad};
    const cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)BM, 2, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void*)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CM_OK;
}

// planes [batches][2][K][C_pad] int8 (N-major); box {128 n, 128 k, 2 planes, 1 batch}.
// plane_box = 2: both planes per box (one CTA); 1: one plane per box (CTA pairs).
int make_nmajor_map(CUtensorMap* m, const int8_t* base, uint32_t cols, uint32_t C_pad, uint32_t K, uint32_t batches,
                    uint32_t plane_box = 2) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)base & 15u) != 0 || (C_pad & 15u) != 0) return set_error(CM_EINVAL, "plane buffer misaligned");
    const cuuint64_t dims[4] = {cols, K, 2, batches};
    const cuuint64_t strides[3] = {(cuuint64_t)C_pad, (cuuint64_t)K * C_pad, (cuuint64_t)2 * K * C_pad};
    const cuuint32_t box[4] = {128, (cuuint32_t)BK, plane_box, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void*)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CM_OK;
}

// Conv A planes [2][nimg][Hp][Wp][Cp] viewed as {KR k, Wp pixels, Hp rows, nimg, 2}:
// dim 0 (the taps (s, c) of one kernel row) overlaps dim 1 by design, the
// pixel stride being Cp bytes.  Box {128, bw*sw, bh*sh, bn, 1} with traversal
// strides {1, sw, sh, 1, 1} = 128 pixels x 128 bytes of K.  Every in-range
// (pixel, k) address stays inside the buffer plus (kw-1)*Cp bytes of slack.
// (No L2 promotion: the box rows are 128 bytes and overlap their neighbours; measured
// slightly faster than 256-byte promotion on the ResNet-18 layers.)
int make_conv_map(CUtensorMap* m, const ConvA& c) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)c.planes & 15u) != 0 || (c.Cp & 15u) != 0) return set_error(CM_EINVAL, "conv plane buffer misaligned");
    const uint32_t bw = 1u << c.bw_log, bh = 1u << c.bh_log, bn = 1u << c.bn_log;
    if (bw * bh * bn != (uint32_t)BM || bw * c.sw > 256 || bh * c.sh > 256 || c.sw > 8 || c.sh > 8)
        return set_error(CM_EINVAL, "conv tile shape");
    const uint64_t row = c.row_pitch ? c.row_pitch : (uint64_t)c.Wp * c.Cp;
    const uint64_t img = c.img_pitch ? c.img_pitch : row * c.Hp;
    const uint64_t plane = c.plane_pitch ? c.plane_pitch : img * c.nimg;
    if ((row | img | plane) & 15u) return set_error(CM_EINVAL, "conv plane pitches misaligned");
    const cuuint64_t dims[5] = {c.KR, c.Wp, c.Hp, c.nimg, 2};
    const cuuint64_t strides[4] = {(cuuint64_t)c.Cp, (cuuint64_t)row, (cuuint64_t)img, (cuuint64_t)plane};
    const cuuint32_t box[5] = {(cuuint32_t)BK, bw * c.sw, bh * c.sh, bn, 1};
    const cuuint32_t estr[5] = {1, c.sw, c.sh, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, (void*)c.planes, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled (conv) failed (%d)", (int)r);
    return CM_OK;
}

// The window form's operand: dims (K bytes of a kernel row, columns, images, rows, plane)
// so that one box {128 k, bw columns (stride sw), bn images, `rows` rows, 2 planes} lands
// as [plane][row][image][column][128 bytes] -- for every kernel row r, the 128 tile rows
// (row, image, column) start r*dh*bn*bw rows into each plane.
int make_conv_window_map(CUtensorMap* m, const ConvA& c, uint32_t rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)c.planes & 15u) != 0 || (c.Cp & 15u) != 0) return set_error(CM_EINVAL, "conv plane buffer misaligned");
    const uint32_t bw = 1u << c.bw_log, bn = 1u << c.bn_log;
    if (bw * (1u << c.bh_log) * bn != (uint32_t)BM || bw * c.sw > 256 || rows > 256 || c.sw > 8)
        return set_error(CM_EINVAL, "conv window shape");
    const uint64_t row = c.row_pitch ? c.row_pitch : (uint64_t)c.Wp * c.Cp;
    const uint64_t img = c.img_pitch ? c.img_pitch : row * c.Hp;
    const uint64_t plane = c.plane_pitch ? c.plane_pitch : img * c.nimg;
    if ((row | img | plane) & 15u) return set_error(CM_EINVAL, "conv plane pitches misaligned");
    const cuuint64_t dims[5] = {c.KR, c.Wp, c.nimg, c.Hp, 2};
    const cuuint64_t strides[4] = {(cuuint64_t)c.Cp, (cuuint64_t)img, (cuuint64_t)row, (cuuint64_t)plane};
    const cuuint32_t box[5] = {(cuuint32_t)BK, bw * c.sw, bn, rows, 2};
    const cuuint32_t estr[5] = {1, c.sw, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, (void*)c.planes, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled (conv window) failed (%d)", (int)r);
    return CM_OK;
}

// B planes packed for 64-column tiles: [batches][K][128] int8, each K row =
// [64 hi | 64 lo] bytes of one column tile; box {128, 128 k, 1, 1}.
int make_packed_map(CUtensorMap* m, const int8_t* base, uint32_t K, uint32_t batches) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)base & 15u) != 0) return set_error(CM_EINVAL, "plane buffer misaligned");
    const cuuint64_t dims[4] = {128, K, 1, batches};
    const cuuint64_t strides[3] = {128, (cuuint64_t)K * 128, (cuuint64_t)K * 128};
    const cuuint32_t box[4] = {128, (cuuint32_t)BK, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void*)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled (packed) failed (%d)", (int)r);
    return CM_OK;
}

// Weights-as-A operand: [128][Kt] int8, row 2m = channel m's hi plane, row 2m + 1 its
// lo' plane, K contiguous (Kt a multiple of 128).
int make_wa_map(CUtensorMap* m, const int8_t* base, uint32_t Kt) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled unavailable");
    if (((uintptr_t)base & 15u) != 0 || Kt % BK != 0) return set_error(CM_EINVAL, "weight rows misaligned");
    const cuuint64_t dims[4] = {Kt, 128, 1, 1};
    const cuuint64_t strides[3] = {Kt, (cuuint64_t)Kt * 128, (cuuint64_t)Kt * 128};
    const cuuint32_t box[4] = {(cuuint32_t)BK, 128, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void*)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(CM_ECUDA, "cuTensorMapEncodeTiled (weight rows) failed (%d)", (int)r);
    return CM_OK;
}

// Packed weight planes [Kt][64 hi | 64 lo] -> weight rows [128][Kt] (row 2m + p = byte
// p*64 + m of every K row).  Block = 128 K rows through shared memory.
__global__ void __launch_bounds__(256) packed_to_rows_kernel(const int8_t* __restrict__ packed, uint32_t Kt,
                                                             int8_t* __restrict__ rows) {
    griddep_wait();
    __shared__ uint32_t tile[128][33];            // [k][byte / 4] of the packed rows
    const uint32_t k0 = blockIdx.x * 128;
    for (uint32_t q = threadIdx.x; q < 128 * 8; q += 256) {
        const uint32_t k = q / 8, seg = q % 8;
        const uint4 v = __ldg((const uint4*)(packed + (uint64_t)(k0 + k) * 128 + seg * 16));
        tile[k][4 * seg] = v.x; tile[k][4 * seg + 1] = v.y; tile[k][4 * seg + 2] = v.z; tile[k][4 * seg + 3] = v.w;
    }
    __syncthreads();
    for (uint32_t q = threadIdx.x; q < 128 * 8; q += 256) {
        const uint32_t R = q / 8, seg = q % 8;    // output row, 16-byte run of K
        const uint32_t byte = (R & 1u) * 64 + (R >> 1);
        uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
        for (uint32_t b = 0; b < 16; ++b)
            w[b / 4] |= ((tile[seg * 16 + b][byte / 4] >> (8 * (byte % 4))) & 0xFFu) << (8 * (b % 4));
        *(uint4*)(rows + (uint64_t)R * Kt + k0 + seg * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Zeroes n words (a K-split launch's arrival counters, right before it).
__global__ void __launch_bounds__(256) clear_words_kernel(uint32_t* __restrict__ p, uint32_t n) {
    griddep_wait();
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = 0u;
}

// K-split units per tile for a launch of `tiles` tiles of num_kb K blocks on `slots`
// resident CTAs (pairs): as many units as keep the grid to one wave (at most 4, each of at
// least 4 K blocks), and none if that is fewer than 2.  Measured on ResNet-18's 3x3 convs
// (plane image in and out, back-to-back launches): 32 images' 7x7x512 conv, 32 pair tiles
// on 74 pairs, 29.7 -> 25.6 us with 2 units per tile; every split that made a second wave
// was slower (14x14x256 at 64 images, 98 pair tiles: 33.9 us unsplit, 39.4-62.2 us split 2-4
// ways) -- a unit's pipeline fill, accumulator drain and slab traffic cost more than the
// idle slots of a partly filled last wave.
uint32_t pick_splits(const Context* cx, uint64_t tiles, uint32_t num_kb, uint32_t slots, uint64_t counters_per_tile) {
    if (cx->gemm_split == 0 || cx->gemm_split == 1 || slots == 0 || tiles == 0) return 1;
    if (tiles * counters_per_tile > kSplitCounters) return 1;
    // forced splits: grids of at most four waves (the slabs grow with the grid)
    if (cx->gemm_split > 1)
        return tiles <= 4ull * slots ? std::max(1u, std::min<uint32_t>((uint32_t)cx->gemm_split, num_kb / 2)) : 1u;
    const uint64_t S = std::min<uint64_t>({4u, slots / tiles, num_kb / 4u});
    return S >= 2 ? (uint32_t)S : 1u;
}

template <int TBN, int CG, bool WA = false, bool WIN = false>
int launch_persistent(const Context* cx, const CUtensorMap& ta, const CUtensorMap& tb, GemmArgs& g, cudaStream_t s,
                      size_t win_smem = 0) {
    static int per_sm_clusters = -1;   // co-resident clusters of CG CTAs (one CTA per SM)
    // the window form's shared memory depends on the call (resident weights + windows)
    const size_t smem = WIN ? win_smem : (size_t)Cfg<TBN, CG, WA>::SMEM_LAUNCH;
    // the K-split variant (row-major epilogue forms only; otherwise the same kernel twice)
    constexpr bool CAN_KS = !WA && !WIN;
    const auto kern_one = gemm_q88_kernel<TBN, CG, WA, WIN, false>;
    const auto kern_ks = gemm_q88_kernel<TBN, CG, WA, WIN, CAN_KS>;
    if (per_sm_clusters < 0) {
        for (const auto kf : {kern_one, kern_ks}) {
            cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 WIN ? SMEM_BYTES : Cfg<TBN, CG, WA>::SMEM_LAUNCH);
            if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemm)");
            if (CG > 1) cudaFuncSetAttribute(kf, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
        }
        int n = cx->sm_count / CG;
        if (CG > 1) {
            cudaLaunchConfig_t q{};
            q.gridDim = dim3(CG * n);
            q.blockDim = dim3(Cfg<TBN, CG, WA>::THREADS);
            q.dynamicSmemBytes = Cfg<TBN, CG, WA>::SMEM_LAUNCH;
            cudaLaunchAttribute at{};
            at.id = cudaLaunchAttributeClusterDimension;
            at.val.clusterDim.x = CG; at.val.clusterDim.y = 1; at.val.clusterDim.z = 1;
            q.attrs = &at; q.numAttrs = 1;
            int m = 0;
            if (cudaOccupancyMaxActiveClusters(&m, kern_one, &q) == cudaSuccess && m > 0) n = m;
            cudaGetLastError();
        }
        per_sm_clusters = n;
    }
    g.tiles_n = (g.cols + TBN - 1) / TBN;
    g.tiles_mc = (g.tiles_m + CG - 1) / CG;
    const uint64_t total = (uint64_t)g.batch * g.tiles_mc * g.tiles_n;
    if (total == 0) return CM_OK;
    if ((uint64_t)g.tiles_m * g.tiles_n >= (1ull << 32) || total >= (1ull << 32))
        return set_error(CM_EUNSUPPORTED, "GEMM tile grid too large");
    g.fd_z = FastDiv(g.tiles_mc * g.tiles_n);
    g.fd_group = FastDiv(GROUP_M * g.tiles_n);
    g.fd_hw = FastDiv(g.conv ? g.tiles_w * g.tiles_h : 1u);
    g.fd_w = FastDiv(g.conv ? g.tiles_w : 1u);
    g.splits = 1; g.fd_split = FastDiv(1u); g.ws = nullptr; g.cnt = nullptr;
    if (CAN_KS && !g.no_split) {
        const uint32_t S = pick_splits(cx, total, g.num_kb, (uint32_t)per_sm_clusters,
                                       (uint64_t)CG * Cfg<TBN, CG, WA>::EPI_WARPS);
        if (S > 1 && total * S < (1ull << 32)) {
            // the launch's own slabs and arrival counters (stream-ordered scratch, so K-split
            // launches on different streams never share them); the counters start at zero
            const size_t slab_bytes = (size_t)total * CG * S * TBN * BM * sizeof(int32_t);
            const uint32_t ncnt = (uint32_t)(total * CG * Cfg<TBN, CG, WA>::EPI_WARPS);
            const int rc = scratch_alloc((void**)&g.ws, slab_bytes + (size_t)ncnt * sizeof(uint32_t), s);
            if (rc) return rc;
            g.splits = S; g.fd_split = FastDiv(S);
            g.cnt = (uint32_t*)((uint8_t*)g.ws + slab_bytes);
            launch_k(clear_words_kernel, std::min<uint32_t>((ncnt + 255) / 256, (uint32_t)cx->sm_count), 256, 0, s, g.cnt,
                     ncnt);
            count_launch();
        }
    }
    const uint64_t units = total * g.splits;
    const unsigned clusters = (unsigned)std::min<uint64_t>(units, (uint64_t)per_sm_clusters);
    const auto kern = g.splits > 1 ? kern_ks : kern_one;
    g.status = cx->status; g.timeout_ns = cx->timeout_ns;
    g.clk = prof_gemm_clock();
    cudaError_t e;
    {
        ProfScope ps_(PK_GEMM, s);
        if (CG == 1) {
            launch_k(kern, clusters, Cfg<TBN, CG, WA>::THREADS, smem, s, ta, tb, g);
            e = cudaGetLastError();
        } else {
            cudaLaunchConfig_t q{};
            q.gridDim = dim3(CG * clusters);
            q.blockDim = dim3(Cfg<TBN, CG, WA>::THREADS);
            q.dynamicSmemBytes = smem;
            q.stream = s;
            cudaLaunchAttribute at[2]{};
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = CG; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
            at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[1].val.programmaticStreamSerializationAllowed = g_pdl ? 1 : 0;
            q.attrs = at; q.numAttrs = 2;
            e = cudaLaunchKernelEx(&q, kern, ta, tb, g);
        }
    }
    if (g.ws) scratch_free(g.ws, s);
    count_launch();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "gemm launch");
}

// CTA pairs for 128-column tiles when there are at least two row tiles (off with
// CM_GEMM_PAIRS=0 in the environment at cm_init).
bool use_pairs(const Context* cx, uint32_t tiles_m) { return cx->gemm_pairs && tiles_m >= 2; }

}  // namespace

// Lanes per output for the direct kernels: enough threads to fill the GPU,
// at most 32 and at most the reduction length.
uint32_t direct_lanes(const Context* cx, uint64_t outputs, uint64_t red) {
    uint32_t G = 1;
    const uint64_t want = (uint64_t)cx->sm_count * 1024;
    while (G < 32 && outputs * G < want && 2ull * G <= red) G *= 2;
    return G;
}

// Direct MatMul launch: the row form for at most 8 rows, else the general one.
void launch_matmul_direct(const Context* cx, const int16_t* a, const int16_t* b, int16_t* c, uint32_t n, uint32_t k,
                          uint32_t m, uint32_t batch, uint64_t a_bs, uint64_t b_bs, uint64_t c_bs, uint32_t epi,
                          const int16_t* bias, cudaStream_t s) {
    if (n <= 8 && batch <= 65535u) {
        const dim3 grid((m + 31) / 32, batch);
        if (n == 1) launch_k(matmul_rows_direct_kernel<1>, grid, 32 * kRowWarps, 0, s, a, b, c, n, k, m, a_bs, b_bs, c_bs, epi, bias);
        else if (n == 2) launch_k(matmul_rows_direct_kernel<2>, grid, 32 * kRowWarps, 0, s, a, b, c, n, k, m, a_bs, b_bs, c_bs, epi, bias);
        else if (n <= 4) launch_k(matmul_rows_direct_kernel<4>, grid, 32 * kRowWarps, 0, s, a, b, c, n, k, m, a_bs, b_bs, c_bs, epi, bias);
        else launch_k(matmul_rows_direct_kernel<8>, grid, 32 * kRowWarps, 0, s, a, b, c, n, k, m, a_bs, b_bs, c_bs, epi, bias);
        return;
    }
    const uint64_t total = (uint64_t)batch * n * m;
    const uint32_t G = direct_lanes(cx, total, k);
    launch_k(matmul_direct_kernel, grid_for(cx, total * G, 256, 8), 256, 0, s, a, b, c, n, k, m, a_bs, b_bs, c_bs, total,
             G, epi, bias);
}


int gemm_launch(const Context* cx, const GemmPlan& p, cudaStream_t s) {
    if (p.conv) return gemm_launch_conv(cx, p, s);
    if (p.K == 0) return fill_zero(cx, p.out, p.batch, p.rows, p.cols, p.ldo, p.out_bs, s);
    if (p.K > kMaxGemmK) return set_error(CM_EUNSUPPORTED, "reduction length %u exceeds %u", p.K, kMaxGemmK);
    if (p.b_packed && p.cols > 64) return set_error(CM_EINVAL, "packed B needs at most 64 columns");
    CUtensorMap ta, tb;
    int rc = make_plane_map(&ta, p.a_planes, p.K, p.K_pad, p.rows, p.a_batches);
    if (rc) return rc;
    const uint32_t tiles_m = (p.rows + BM - 1) / BM;
    const bool pairs = !p.b_packed && use_pairs(cx, tiles_m);
    rc = p.b_packed ? make_packed_map(&tb, p.b_planes, p.K, p.b_batches)
                    : make_nmajor_map(&tb, p.b_planes, p.cols, p.C_pad, p.K, p.b_batches, pairs ? 1u : 2u);
    if (rc) return rc;
    GemmArgs g{};
    g.rows = p.rows; g.cols = p.cols; g.num_kb = (p.K + BK - 1) / BK;
    g.tiles_m = tiles_m;
    g.batch = p.batch;
    g.a_batches = p.a_batches; g.b_batches = p.b_batches;
    g.rowterm = p.rowterm; g.colterm = p.colterm;
    g.out = p.out; g.ldo = p.ldo; g.ldc = p.ldc ? p.ldc : 1; g.out_bs = p.out_bs;
    g.conv = 0;
    g.rows_per_img = p.rows_per_img;
    g.no_split = p.no_split;
    g.ksteps = (p.K + 31) / 32;
    g.epi = p.epi; g.resid = p.resid;
    if (p.b_packed) return launch_persistent<64, 1>(cx, ta, tb, g, s);
    return pairs ? launch_persistent<128, 2>(cx, ta, tb, g, s) : launch_persistent<128, 1>(cx, ta, tb, g, s);
}

int gemm_launch_conv(const Context* cx, const GemmPlan& p, cudaStream_t s) {
    const ConvA& c = *p.conv;
    if (p.K == 0 || p.K % BK != 0 || c.KR_pad % BK != 0 || p.K != c.kh * c.KR_pad)
        return set_error(CM_EINVAL, "conv GEMM reduction layout");
    if (p.b_packed && p.cols > 64) return set_error(CM_EINVAL, "packed B needs at most 64 columns");
    CUtensorMap ta, tb;
    int rc = make_conv_map(&ta, c);
    if (rc) return rc;
    const uint64_t tiles_img0 = (c.nimg + (1u << c.bn_log) - 1) >> c.bn_log;
    const uint64_t tiles_m0 = tiles_img0 * ((c.out_w + (1u << c.bw_log) - 1) >> c.bw_log) *
                              ((c.out_h + (1u << c.bh_log) - 1) >> c.bh_log);
    const bool pairs = !p.b_packed && use_pairs(cx, (uint32_t)std::min<uint64_t>(tiles_m0, 1u << 30));
    rc = p.b_packed ? make_packed_map(&tb, p.b_planes, p.K, 1)
                    : make_nmajor_map(&tb, p.b_planes, p.cols, p.C_pad, p.K, 1, pairs ? 1u : 2u);
    if (rc) return rc;
    GemmArgs g{};
    g.conv = 1;
    g.bw_log = c.bw_log; g.bh_log = c.bh_log; g.bn_log = c.bn_log;
    g.tiles_w = (c.out_w + (1u << c.bw_log) - 1) >> c.bw_log;
    g.tiles_h = (c.out_h + (1u << c.bh_log) - 1) >> c.bh_log;
    const uint64_t tiles_img = (c.nimg + (1u << c.bn_log) - 1) >> c.bn_log;
    const uint64_t tiles_m = tiles_img * g.tiles_w * g.tiles_h;
    if (tiles_m >= (1ull << 31)) return set_error(CM_EUNSUPPORTED, "GEMM tile grid too large");
    g.tiles_m = (uint32_t)tiles_m;
    g.cols = p.cols; g.num_kb = p.K / BK; g.kb_per_r = c.KR_pad / BK;
    g.ksteps = (c.KR + 31) / 32;
    g.batch = 1; g.rows = 0; g.a_batches = 1; g.b_batches = 1;
    g.nimg = c.nimg; g.out_h = c.out_h; g.out_w = c.out_w; g.sw = c.sw; g.sh = c.sh; g.dh = c.dh;
    g.rowterm = p.rowterm; g.colterm = p.colterm;
    g.out = p.out; g.ldo = p.ldo ? p.ldo : 1; g.ldc = p.ldc; g.out_bs = p.out_bs;   // ldo: output pixel stride
    g.epi = p.epi; g.resid = p.resid;
    g.po = p.po.planes; g.po_S = p.po.S; g.po_plane = p.po.plane_pitch;
    g.rpl = p.rp.planes; g.rpl_plane = p.rp.plane_pitch;
    g.rpl_Hp = p.rp.Hp; g.rpl_Wp = p.rp.Wp; g.rpl_Cp = p.rp.Cp; g.rpl_pt = p.rp.pt; g.rpl_pl = p.rp.pl;
    g.po_Hp = p.po.Hp; g.po_Wp = p.po.Wp; g.po_Cp = p.po.Cp; g.po_pt = p.po.pt; g.po_pl = p.po.pl;
    // Window form (packed weights, stride 1 down the rows, tiles at least 8 columns wide): one
    // TMA box per K block brings the input rows of all kh kernel rows, which read it at row
    // offsets, and the packed weights stay resident -- a quarter to a third of the TMA bytes
    // of one box per kernel row, which bounded these GEMMs (their K-block rounds, not the
    // tensor pipe, set the pace).
    if (p.b_packed && cx->conv_window && c.sh == 1 && c.bw_log >= 3 && !(p.epi & 4u)) {
        const uint32_t bw = 1u << c.bw_log, bn = 1u << c.bn_log;
        const uint32_t rows = (1u << c.bh_log) + (c.kh - 1) * c.dh;
        const uint64_t win_bytes = 2ull * BK * bw * bn * rows;
        const uint64_t w_bytes = (uint64_t)p.K * 128;
        const uint64_t avail = (uint64_t)SMEM_BYTES - 1024 - 256;
        if (rows <= 256 && w_bytes + 2 * win_bytes <= avail) {
            const uint32_t stages = (uint32_t)std::min<uint64_t>(4, (avail - w_bytes) / win_bytes);
            CUtensorMap tw;
            rc = make_conv_window_map(&tw, c, rows);
            if (rc) return rc;
            g.win = 1; g.win_stages = stages; g.win_bytes = (uint32_t)win_bytes; g.win_plane = (uint32_t)(win_bytes / 2);
            g.win_roff = c.dh * bn * bw * BK; g.w_bytes = (uint32_t)w_bytes; g.kh = c.kh;
            return launch_persistent<64, 1, false, true>(cx, tw, tb, g, s, (size_t)(w_bytes + stages * win_bytes + 1024 + 256));
        }
    }
    // Weights as A (one N = 256 MMA per step) for outputs written only as a plane image: its
    // channel-major epilogue goes through a shared-memory transpose for the image, but the
    // plain NCHW epilogue of the packed form is the cheaper one (ResNet-18 stem: 346 against
    // 383 us; layer-1 plane outputs: 181 against 189 us).
    if (p.b_packed && cx->gemm_wa && c.bw_log >= 3 && !(p.epi & 4u) && p.po.planes && !p.out) {
        // the packed planes regrouped as weight rows (prepared already, or here)
        void* wr = nullptr;
        if (!p.wa_rows) {
            rc = scratch_alloc(&wr, (size_t)p.K * 128, s);
            if (rc) return rc;
            rc = weights_to_rows(cx, p.b_planes, p.K, (int8_t*)wr, s);
        }
        if (!rc) rc = make_wa_map(&tb, p.wa_rows ? p.wa_rows : (const int8_t*)wr, p.K);
        if (!rc) rc = launch_persistent<64, 1, true>(cx, ta, tb, g, s);
        if (wr) scratch_free(wr, s);
        return rc;
    }
    if (p.b_packed) return launch_persistent<64, 1>(cx, ta, tb, g, s);
    return pairs ? launch_persistent<128, 2>(cx, ta, tb, g, s) : launch_persistent<128, 1>(cx, ta, tb, g, s);
}

int weights_to_rows(const Context* cx, const int8_t* packed, uint32_t Kt, int8_t* rows, cudaStream_t s) {
    (void)cx;
    if (Kt == 0 || Kt % 128 != 0) return set_error(CM_EINVAL, "weight rows: K = %u", Kt);
    {
        ProfScope ps_(PK_SPLIT, s);
        launch_k(packed_to_rows_kernel, Kt / 128, 256, 0, s, packed, Kt, rows);
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "weight rows");
}

int split_rows(const Context* cx, const int16_t* src, uint64_t src_bs, uint64_t ld, uint32_t rows, uint32_t K,
               uint32_t nbt, int8_t* planes, int32_t* rowterm, const int16_t* bias, cudaStream_t s) {
    const uint64_t total = (uint64_t)rows * nbt;
    if (total == 0) return CM_OK;
    // 128-thread blocks (48 registers a thread): one fits on an SM beside a GEMM CTA
    const unsigned grid = grid_for(cx, total * 32, 128, 16);
    {
        ProfScope ps_(PK_SPLIT, s);
        launch_k(split_rows_kernel, grid, 128, 0, s, src, src_bs, ld, rows, K, pad_k(K), total, planes, rowterm, bias);
    }
    count_launch();
    return CM_OK;
}

// K chunk so that the grid has a few waves of CTAs (each chunk adds one atomic per column).
static uint32_t pick_k_chunk(uint32_t K, uint64_t other_ctas, uint32_t sm_count) {
    const uint64_t target = 4ull * sm_count;
    uint64_t splits = other_ctas >= target ? 1 : (target + other_ctas - 1) / other_ctas;
    uint64_t chunk = (K + splits - 1) / splits;
    chunk = std::max<uint64_t>(chunk, 64);
    return (uint32_t)std::min<uint64_t>(chunk, K ? K : 1);
}

int split_kn(const Context* cx, const int16_t* src, uint64_t src_bs, uint64_t ld, uint32_t cols, uint32_t K,
             uint32_t nbt, int8_t* planes, int32_t* colterm, cudaStream_t s, bool packed) {
    if (packed && cols > 64) return set_error(CM_EINVAL, "packed B needs at most 64 columns");
    if ((uint64_t)cols * nbt == 0) return CM_OK;
    cudaError_t e = cudaMemsetAsync(colterm, 0, (size_t)cols * nbt * sizeof(int32_t), s);
    if (e != cudaSuccess) return cuda_error(e, "memset colterm");
    if (K == 0) return CM_OK;
    const uint32_t vec_threads = (cols + 7) / 8;
    // at most 128 threads (64 registers a thread): one block fits on an SM beside a GEMM CTA
    const uint32_t block = std::min<uint32_t>(128, (vec_threads + 31) / 32 * 32);
    const uint32_t gx = (vec_threads + block - 1) / block;
    const uint32_t k_chunk = pick_k_chunk(K, (uint64_t)gx * nbt, cx->sm_count);
    const uint32_t C_pad = packed ? 128u : pad_c(cols);
    const uint64_t plane_off = packed ? 64u : (uint64_t)K * C_pad;
    const uint64_t batch_pitch = packed ? (uint64_t)K * 128 : 2ull * K * C_pad;
    for (uint32_t b0 = 0; b0 < nbt; b0 += 65535u) {
        const uint32_t nb = std::min(65535u, nbt - b0);
        const dim3 grid(gx, (K + k_chunk - 1) / k_chunk, nb);
        {
            ProfScope ps_(PK_SPLIT, s);
            launch_k(split_kn_kernel, grid, block, 0, s, src + (uint64_t)b0 * src_bs, src_bs, ld, cols, K, C_pad, k_chunk,
                                                  plane_off, batch_pitch, planes + (uint64_t)b0 * batch_pitch,
                                                  colterm + (uint64_t)b0 * cols);
        }
        count_launch();
    }
    return CM_OK;
}

int fill_zero(const Context* cx, int16_t* out, uint32_t batch, uint32_t rows, uint32_t cols, uint64_t ldo,
              uint64_t out_bs, cudaStream_t s) {
    const uint64_t total = (uint64_t)batch * rows * cols;
    if (total == 0) return CM_OK;
    {
        ProfScope ps_(PK_CONV_AUX, s);
        launch_k(fill_zero_kernel, grid_for(cx, total, 256, 8), 256, 0, s, out, rows, cols, ldo, out_bs, total);
    }
    count_launch();
    return CM_OK;
}

}  // namespace cm

using namespace cm;

// ---------------------------------------------------------------------------
// MatmulKernel entry (MatmulKernel.h:68-79)
// ---------------------------------------------------------------------------
namespace {
// `rows` rows of A (row r at a + r*lda) times the shared B [k][m], row r of the result at
// c + r*ldc_row: one tensor-core GEMM over all rows (fused epilogue as in matmul_impl).
int matmul_rows_impl(const Context* cx, const int16_t* a, const int16_t* b, int16_t* c, uint32_t rows, uint32_t k,
                     uint32_t m, uint64_t lda, uint64_t ldc_row, unsigned epi, const int16_t* bias, cudaStream_t s) {
    const uint64_t K_pad = pad_k(k);
    const bool packed = m <= 64;
    const uint64_t a_bytes = (2ull * rows * K_pad + 255) & ~255ull;
    const uint64_t b_bytes = ((uint64_t)k * (packed ? 128 : 2 * pad_c(m)) + 255) & ~255ull;
    const uint64_t rt_bytes = ((uint64_t)rows * 4 + 255) & ~255ull;
    const uint64_t ct_bytes = ((uint64_t)m * 4 + 255) & ~255ull;
    void* scratch = nullptr;
    int rc = scratch_alloc(&scratch, a_bytes + b_bytes + rt_bytes + ct_bytes, s);
    if (rc) return rc;
    int8_t* ap = (int8_t*)scratch;
    int8_t* bp = ap + a_bytes;
    int32_t* rt = (int32_t*)(bp + b_bytes);
    int32_t* ct = (int32_t*)((uint8_t*)rt + rt_bytes);
    rc = split_rows(cx, a, 0, lda, rows, k, 1, ap, rt, nullptr, s);
    if (!rc) rc = split_kn(cx, b, 0, m, m, k, 1, bp, ct, s, packed);
    if (!rc) {
        GemmPlan p{ap, rows, 1, bp, m, 1, k, (uint32_t)K_pad, pad_c(m), rt, ct, c, ldc_row, 1, 0, 1};
        p.b_packed = packed ? 1u : 0u;
        p.epi = (epi & 1u) | ((epi & 2u) << 1);   // the kernel's bias-row bit is 4
        p.resid = (epi & 2u) ? bias : nullptr;
        rc = gemm_launch(cx, p, s);
    }
    scratch_free(scratch, s);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_matmul (row-strided)");
}

// A large batched MatMul as `chunks` batch chunks whose split pre-passes run on the
// context's side stream, chunk j + 1's while chunk j's GEMM runs on the caller's stream:
// the splits are HBM-bound, the GEMM tensor-bound, and the GEMM CTAs leave room on every
// SM for one split CTA (their shared-memory request and the splits' 128-thread blocks are
// sized for it).  Two plane buffers per advancing operand alternate between chunks; a
// broadcast operand (batch stride 0) is split once.  Events order every reuse; the
// caller's stream waits for the side stream before the scratch is released, so the call
// is stream-ordered on `s` like the one-shot path (and captures into a graph the same way).
int matmul_chunked(const Context* cx, const int16_t* a, const int16_t* b, int16_t* c, uint32_t n, uint32_t k,
                   uint32_t m, uint32_t batch, uint32_t a_bs, uint32_t b_bs, uint32_t c_bs, unsigned epi,
                   const int16_t* bias, cudaStream_t s, uint32_t chunks) {
    const uint32_t cb = (batch + chunks - 1) / chunks;
    chunks = (batch + cb - 1) / cb;
    const bool a_adv = a_bs != 0, b_adv = b_bs != 0;
    const uint64_t K_pad = pad_k(k);
    const bool packed = m <= 64;
    const uint64_t a_bytes = ((uint64_t)(a_adv ? cb : 1) * 2 * n * K_pad + 255) & ~255ull;
    const uint64_t b_bytes = ((uint64_t)(b_adv ? cb : 1) * k * (packed ? 128 : 2 * pad_c(m)) + 255) & ~255ull;
    const uint64_t rt_bytes = ((uint64_t)(a_adv ? cb : 1) * n * 4 + 255) & ~255ull;
    const uint64_t ct_bytes = ((uint64_t)(b_adv ? cb : 1) * m * 4 + 255) & ~255ull;
    const int na = a_adv ? 2 : 1, nbuf = b_adv ? 2 : 1;
    void* scratch = nullptr;
    int rc = scratch_alloc(&scratch, na * (a_bytes + rt_bytes) + nbuf * (b_bytes + ct_bytes), s);
    if (rc) return rc;
    uint8_t* q = (uint8_t*)scratch;
    int8_t* A[2] = {nullptr, nullptr};
    int8_t* B[2] = {nullptr, nullptr};
    int32_t* RT[2] = {nullptr, nullptr};
    int32_t* CT[2] = {nullptr, nullptr};
    for (int i = 0; i < na; ++i) { A[i] = (int8_t*)q; q += a_bytes; RT[i] = (int32_t*)q; q += rt_bytes; }
    for (int i = 0; i < nbuf; ++i) { B[i] = (int8_t*)q; q += b_bytes; CT[i] = (int32_t*)q; q += ct_bytes; }
    cudaStream_t aux = cx->aux_stream;
    std::vector<cudaEvent_t> ev(2 * chunks + 2, nullptr);
    for (auto& e : ev)
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) rc = set_error(CM_ECUDA, "event");
    cudaEvent_t ev_start = ev[2 * chunks], ev_join = ev[2 * chunks + 1];
    if (!rc) {
        cudaEventRecord(ev_start, s);
        cudaStreamWaitEvent(aux, ev_start, 0);      // the inputs are ready when the caller's stream is
        if (!a_adv) rc = split_rows(cx, a, 0, k, n, k, 1, A[0], RT[0], nullptr, aux);
        if (!rc && !b_adv) rc = split_kn(cx, b, 0, m, m, k, 1, B[0], CT[0], aux, packed);
    }
    for (uint32_t j = 0; j < chunks && !rc; ++j) {
        const uint32_t z0 = j * cb, nb = std::min(cb, batch - z0), buf = j & 1u;
        if (j >= 2) cudaStreamWaitEvent(aux, ev[2 * (j - 2) + 1], 0);   // chunk j-2's GEMM has read the buffers
        if (a_adv) rc = split_rows(cx, a + (uint64_t)z0 * a_bs, a_bs, k, n, k, nb, A[buf], RT[buf], nullptr, aux);
        if (!rc && b_adv) rc = split_kn(cx, b + (uint64_t)z0 * b_bs, b_bs, m, m, k, nb, B[buf], CT[buf], aux, packed);
        if (rc) break;
        cudaEventRecord(ev[2 * j], aux);
        cudaStreamWaitEvent(s, ev[2 * j], 0);
        const uint32_t ia = a_adv ? buf : 0u, ib = b_adv ? buf : 0u;
        GemmPlan p{A[ia], n, a_adv ? nb : 1u, B[ib], m, b_adv ? nb : 1u, k, (uint32_t)K_pad, pad_c(m), RT[ia], CT[ib],
                   c + (uint64_t)z0 * c_bs, m, 1, c_bs, nb};
        p.b_packed = packed ? 1u : 0u;
        p.epi = (epi & 1u) | ((epi & 2u) << 1);   // the kernel's bias-row bit is 4
        p.resid = (epi & 2u) ? bias : nullptr;
        rc = gemm_launch(cx, p, s);
        cudaEventRecord(ev[2 * j + 1], s);
    }
    // join the side stream before the scratch goes back to the pool (also on an error path)
    if (ev_join) {
        cudaEventRecord(ev_join, aux);
        cudaStreamWaitEvent(s, ev_join, 0);
    }
    for (auto& e : ev)
        if (e) cudaEventDestroy(e);
    scratch_free(scratch, s);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_matmul (chunked)");
}

// MatMul with an optional fused epilogue (epi bit 1: + bias[j] saturating, bit 0: ReLU).
int matmul_impl(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k, unsigned m, unsigned batch,
                unsigned a_batch_stride, unsigned b_batch_stride, unsigned c_batch_stride, unsigned epi,
                const int16_t* bias, cudaStream_t s) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (epi > 3u) return set_error(CM_EINVAL, "cm_matmul_fused: epilogue %u (0..3)", epi);
    if ((epi & 2u) && !bias) return set_error(CM_EINVAL, "cm_matmul_fused: null bias");
    if (n == 0 || m == 0 || batch == 0) return CM_OK;
    if (!c || (k > 0 && (!a || !b))) return set_error(CM_EINVAL, "cm_matmul: null buffer");
    if (batch > 1 && (uint64_t)c_batch_stride < (uint64_t)n * m) {
        // Output slices of different batch steps overlap; the reference's batch
        // loop runs in order (MatmulKernel.cpp:108-112), so later steps win.
        if (c_batch_stride == 0) {
            const uint64_t last = batch - 1;
            return matmul_impl(a ? a + last * a_batch_stride : a, b ? b + last * b_batch_stride : b, c, n, k, m, 1,
                               a_batch_stride, b_batch_stride, 0, epi, bias, s);
        }
        for (uint64_t bi = 0; bi < batch; ++bi) {
            rc = matmul_impl(a ? a + bi * a_batch_stride : a, b ? b + bi * b_batch_stride : b, c + bi * c_batch_stride,
                             n, k, m, 1, a_batch_stride, b_batch_stride, 0, epi, bias, s);
            if (rc) return rc;
        }
        return CM_OK;
    }
    if (k == 0) {
        // empty sums: every word is 0, then the epilogue's VectorOP calls in place
        rc = fill_zero(cx, c, batch, n, m, m, c_batch_stride, s);
        for (uint64_t bi = 0; !rc && epi && bi < batch; ++bi) {
            int16_t* cz = c + bi * c_batch_stride;
            if (epi & 2u) rc = cm_vectorop_async(cz, bias, cz, m, CM_OP_ADD, n, m, 0, s);
            if (!rc && (epi & 1u)) rc = cm_vectorop_async(cz, nullptr, cz, n * m, CM_OP_RELU, 1, 0, 0, s);
        }
        return rc;
    }
    const unsigned __int128 macs = (unsigned __int128)batch * n * m * k;
    if (macs <= cx->direct_max_macs) {
        {
            ProfScope ps_(PK_GEMM, s);
            launch_matmul_direct(cx, a, b, c, n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, epi, bias,
                                 s);
        }
        count_launch();
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_matmul direct");
    }
    if (k > kMaxGemmK) return set_error(CM_EUNSUPPORTED, "cm_matmul: k = %u exceeds %u", k, kMaxGemmK);
    if (n == 1 && batch > 1 && b_batch_stride == 0) {
        // Row-strided form (the reference scheduler's MatMul over gapped buffers,
        // inference-scheduler/src/nodes.py:785-801): `batch` one-row products with the
        // same B, A rows a_batch_stride apart and output rows c_batch_stride apart
        // (>= m here: overlapping rows took the ordered path above).  As batch steps
        // every 128-row tile would hold one row; folded, they are the rows of ONE GEMM
        // with those row pitches.
        return matmul_rows_impl(cx, a, b, c, batch, k, m, a_batch_stride, c_batch_stride, epi, bias, s);
    }
    if (cx->matmul_overlap && batch >= 2) {
        // large calls: batch chunks of >= 2^37 multiply-adds, at most 8 (smaller chunks lose
        // more to the extra launches than the overlap gains: a GEMM under the power cap runs
        // slower beside a concurrent split, so only the large ones gain)
        const uint64_t by_work = (uint64_t)(macs >> 37);
        const uint32_t chunks = (uint32_t)std::min<uint64_t>(std::min<uint64_t>(batch, 8), by_work);
        if (chunks >= 2)
            return matmul_chunked(cx, a, b, c, n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, epi,
                                  bias, s, chunks);
    }
    const uint32_t a_batches = a_batch_stride == 0 ? 1u : batch;
    const uint32_t b_batches = b_batch_stride == 0 ? 1u : batch;
    const uint64_t K_pad = pad_k(k);
    const uint64_t a_bytes = ((uint64_t)a_batches * 2 * n * K_pad + 255) & ~255ull;
    // outputs of at most 64 columns use 64-column tiles (packed B, double-buffered accumulators)
    const bool packed = m <= 64;
    const uint64_t b_bytes = ((uint64_t)b_batches * k * (packed ? 128 : 2 * pad_c(m)) + 255) & ~255ull;
    const uint64_t rt_bytes = ((uint64_t)a_batches * n * 4 + 255) & ~255ull;
    const uint64_t ct_bytes = ((uint64_t)b_batches * m * 4 + 255) & ~255ull;
    void* scratch = nullptr;
    rc = scratch_alloc(&scratch, a_bytes + b_bytes + rt_bytes + ct_bytes, s);
    if (rc) return rc;
    int8_t* ap = (int8_t*)scratch;
    int8_t* bp = ap + a_bytes;
    int32_t* rt = (int32_t*)(bp + b_bytes);
    int32_t* ct = (int32_t*)((uint8_t*)rt + rt_bytes);
    rc = split_rows(cx, a, a_batch_stride, k, n, k, a_batches, ap, rt, nullptr, s);
    if (!rc) rc = split_kn(cx, b, b_batch_stride, m, m, k, b_batches, bp, ct, s, packed);
    if (!rc) {
        GemmPlan p{ap, n, a_batches, bp, m, b_batches, k, (uint32_t)K_pad, pad_c(m), rt, ct, c, m, 1, c_batch_stride, batch};
        p.b_packed = packed ? 1u : 0u;
        p.epi = (epi & 1u) | ((epi & 2u) << 1);   // the kernel's bias-row bit is 4
        p.resid = (epi & 2u) ? bias : nullptr;
        rc = gemm_launch(cx, p, s);
    }
    scratch_free(scratch, s);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_matmul");
}
}  // namespace

// ---------------------------------------------------------------------------
// Prepared MatMul B (a network's Gemm weights): planes and column terms built once
// ---------------------------------------------------------------------------
struct cm_matmul_weights {
    const int16_t* b = nullptr;   // the live B, read by the calls that do not use the planes
    uint32_t k = 0, m = 0;
    int device = -1;
    uint32_t packed = 0;
    int8_t* planes = nullptr;     // null: every call takes cm_matmul's own path
    int32_t* colterm = nullptr;
    void* mem = nullptr;
};

extern "C" int cm_matmul_weights_create(const int16_t* b, unsigned k, unsigned m, cm_matmul_weights_t** out) {
    if (out) *out = nullptr;                // null on every failure
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!out) return set_error(CM_EINVAL, "cm_matmul_weights_create: null result pointer");
    if (k > 0 && m > 0 && !b) return set_error(CM_EINVAL, "cm_matmul_weights_create: null B");
    cm_matmul_weights* w = new (std::nothrow) cm_matmul_weights;
    if (!w) return set_error(CM_ENOMEM, "cm_matmul_weights_create: out of host memory");
    w->b = b; w->k = k; w->m = m; w->device = cx->device;
    if (k == 0 || m == 0 || k > kMaxGemmK) {   // nothing to prepare: calls take cm_matmul's path
        *out = w;
        return CM_OK;
    }
    w->packed = m <= 64 ? 1u : 0u;
    const uint64_t b_bytes = ((uint64_t)k * (w->packed ? 128 : 2 * pad_c(m)) + 255) & ~255ull;
    const uint64_t ct_bytes = ((uint64_t)m * 4 + 255) & ~255ull;
    cudaError_t e = cudaMalloc(&w->mem, b_bytes + ct_bytes);
    if (e != cudaSuccess) { delete w; return cuda_error(e, "cm_matmul_weights_create: cudaMalloc"); }
    w->planes = (int8_t*)w->mem;
    w->colterm = (int32_t*)((int8_t*)w->mem + b_bytes);
    cudaStream_t s = nullptr;
    rc = split_kn(cx, b, 0, m, m, k, 1, w->planes, w->colterm, s, w->packed != 0);
    if (!rc) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = cuda_error(e, "cm_matmul_weights_create");
    }
    if (rc) {
        cudaFree(w->mem);
        delete w;
        return rc;
    }
    *out = w;
    return CM_OK;
}

extern "C" void cm_matmul_weights_destroy(cm_matmul_weights_t* w) {
    if (!w) return;
    if (w->mem) {
        int cur = -1;
        cudaGetDevice(&cur);
        if (w->device >= 0 && cur != w->device) cudaSetDevice(w->device);
        cudaFree(w->mem);
        if (cur >= 0 && cur != w->device) cudaSetDevice(cur);
    }
    delete w;
}

extern "C" int cm_matmul_prepared_async(const cm_matmul_weights_t* w, const int16_t* a, int16_t* c, unsigned n,
                                        unsigned batch, unsigned a_batch_stride, unsigned c_batch_stride,
                                        unsigned epilogue, const int16_t* bias, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!w) return set_error(CM_EINVAL, "cm_matmul_prepared: null weights");
    if (w->device != cx->device) return set_error(CM_EINVAL, "cm_matmul_prepared: weights of device %d", w->device);
    const cudaStream_t s = (cudaStream_t)stream;
    const unsigned k = w->k, m = w->m;
    const unsigned __int128 macs = (unsigned __int128)batch * n * m * k;
    // cm_matmul_fused with B broadcast (b_batch_stride 0) and the prepared planes: the calls
    // that do not run the one-GEMM form (argument errors, empty and launch-bound sizes,
    // overlapping output steps, the row-strided form, batch chunks) take that path with the
    // live B
    const bool own = w->planes && epilogue <= 3u && !((epilogue & 2u) && !bias) && n > 0 && batch > 0 && a && c &&
                     macs > cx->direct_max_macs && !(batch > 1 && (uint64_t)c_batch_stride < (uint64_t)n * m) &&
                     !(n == 1 && batch > 1) &&
                     !(cx->matmul_overlap && batch >= 2 && std::min<uint64_t>(std::min<uint64_t>(batch, 8), (uint64_t)(macs >> 37)) >= 2);
    if (!own)
        return matmul_impl(a, w->b, c, n, k, m, batch, a_batch_stride, 0u, c_batch_stride, epilogue, bias, s);
    const uint32_t a_batches = a_batch_stride == 0 ? 1u : batch;
    const uint64_t K_pad = pad_k(k);
    const uint64_t a_bytes = ((uint64_t)a_batches * 2 * n * K_pad + 255) & ~255ull;
    const uint64_t rt_bytes = ((uint64_t)a_batches * n * 4 + 255) & ~255ull;
    void* scratch = nullptr;
    rc = scratch_alloc(&scratch, a_bytes + rt_bytes, s);
    if (rc) return rc;
    int8_t* ap = (int8_t*)scratch;
    int32_t* rt = (int32_t*)(ap + a_bytes);
    rc = split_rows(cx, a, a_batch_stride, k, n, k, a_batches, ap, rt, nullptr, s);
    if (!rc) {
        GemmPlan p{ap, n, a_batches, w->planes, m, 1, k, (uint32_t)K_pad, pad_c(m), rt, w->colterm, c, m, 1, c_batch_stride, batch};
        p.b_packed = w->packed;
        p.epi = (epilogue & 1u) | ((epilogue & 2u) << 1);   // the kernel's bias-row bit is 4
        p.resid = (epilogue & 2u) ? bias : nullptr;
        rc = gemm_launch(cx, p, s);
    }
    scratch_free(scratch, s);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_matmul_prepared");
}

extern "C" int cm_matmul_prepared(const cm_matmul_weights_t* w, const int16_t* a, int16_t* c, unsigned n, unsigned batch,
                                  unsigned a_batch_stride, unsigned c_batch_stride, unsigned epilogue, const int16_t* bias) {
    int rc = cm_matmul_prepared_async(w, a, c, n, batch, a_batch_stride, c_batch_stride, epilogue, bias, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_matmul_async(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k, unsigned m,
                               unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                               unsigned c_batch_stride, cm_stream_t stream) {
    return matmul_impl(a, b, c, n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, 0u, nullptr,
                       (cudaStream_t)stream);
}

extern "C" int cm_matmul_fused_async(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k,
                                     unsigned m, unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                                     unsigned c_batch_stride, unsigned epilogue, const int16_t* bias,
                                     cm_stream_t stream) {
    return matmul_impl(a, b, c, n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, epilogue, bias,
                       (cudaStream_t)stream);
}

extern "C" int cm_matmul_fused(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k, unsigned m,
                               unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                               unsigned c_batch_stride, unsigned epilogue, const int16_t* bias) {
    int rc = cm_matmul_fused_async(a, b, c, n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, epilogue,
                                   bias, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_matmul(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k, unsigned m,
                         unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride, unsigned c_batch_stride) {
    int rc = cm_matmul_async(a, b, c, n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

// ---------------------------------------------------------------------------
// cm_matmul_noalloc: the MatMul entry for callers that must not allocate.
//
// Some callers cannot call cudaMalloc at all once they are running: code whose
// device memory is owned by another allocator that has reserved the GPU, and
// run loops that by contract allocate nothing after initialisation (the
// reference's generated inference_run() is one: every buffer comes from the
// single pool that inference_init() sets up).  cm_matmul takes its scratch
// (the int8 operand planes and the row/column terms) from the stream-ordered
// pool; this variant uses the fixed array below instead, so it never calls
// cudaMalloc, cudaMallocAsync, cudaFree or any allocating routine.
//
// The array is a file-scope __device__ object, so every GPU that loads this
// library holds CM_MATMUL_NOALLOC_SCRATCH_BYTES of it until the process exits.
// Its host-side name is only a stand-in, never a device address: the device
// address comes from cudaGetSymbolAddress, taken once per device, with that
// device current, on the first call made on it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_matmul_noalloc_scratch[CM_MATMUL_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};

int noalloc_scratch(int device, void** out) {
    if (device < 0 || device >= 64) return set_error(CM_EUNSUPPORTED, "device ordinal %d", device);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_matmul_noalloc_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(noalloc scratch)");
        g_noalloc_addr[device] = p;
    }
    *out = g_noalloc_addr[device];
    return CM_OK;
}

// One batch-step range [bi0, bi0 + nb) of a matmul, all scratch in `base`.
int noalloc_run(const Context* cx, uint8_t* base, const int16_t* a, const int16_t* b, int16_t* c, uint32_t n,
                uint32_t k, uint32_t m, uint32_t nb, uint32_t a_bs, uint32_t b_bs, uint64_t c_bs, cudaStream_t s) {
    const unsigned __int128 macs = (unsigned __int128)nb * n * m * k;
    if (macs <= cx->direct_max_macs) {
        // launch-bound sizes: the one-kernel CUDA-core path, which needs no scratch at all
        {
            ProfScope ps_(PK_GEMM, s);
            launch_matmul_direct(cx, a, b, c, n, k, m, nb, a_bs, b_bs, c_bs, 0u, nullptr, s);
        }
        count_launch();
        return CM_OK;
    }
    const uint32_t a_batches = a_bs == 0 ? 1u : nb;
    const uint32_t b_batches = b_bs == 0 ? 1u : nb;
    const uint64_t K_pad = pad_k(k);
    const uint64_t a_bytes = ((uint64_t)a_batches * 2 * n * K_pad + 255) & ~255ull;
    const uint64_t b_bytes = ((uint64_t)b_batches * 2 * k * pad_c(m) + 255) & ~255ull;
    const uint64_t rt_bytes = ((uint64_t)a_batches * n * 4 + 255) & ~255ull;
    const uint64_t ct_bytes = ((uint64_t)b_batches * m * 4 + 255) & ~255ull;
    if (a_bytes + b_bytes + rt_bytes + ct_bytes > CM_MATMUL_NOALLOC_SCRATCH_BYTES)
        return set_error(CM_EINVAL,
                         "cm_matmul_noalloc: needs %llu bytes of scratch, the fixed array holds %llu "
                         "(use cm_matmul for larger calls)",
                         (unsigned long long)(a_bytes + b_bytes + rt_bytes + ct_bytes),
                         (unsigned long long)CM_MATMUL_NOALLOC_SCRATCH_BYTES);
    int8_t* ap = (int8_t*)base;
    int8_t* bp = ap + a_bytes;
    int32_t* rt = (int32_t*)(bp + b_bytes);
    int32_t* ct = (int32_t*)((uint8_t*)rt + rt_bytes);
    // Every word the GEMM reads is rewritten here: plane rows k < K and all row
    // terms by the splits; the column terms are cleared before they are summed.
    int rc = split_rows(cx, a, a_bs, k, n, k, a_batches, ap, rt, nullptr, s);
    if (!rc) rc = split_kn(cx, b, b_bs, m, m, k, b_batches, bp, ct, s);
    if (!rc) {
        GemmPlan p{ap, n, a_batches, bp, m, b_batches, k, (uint32_t)K_pad, pad_c(m), rt, ct, c, m, 1, c_bs, nb};
        p.no_split = 1;                 // a K-split launch would allocate its slabs
        rc = gemm_launch(cx, p, s);
    }
    return rc;
}
}  // namespace

extern "C" int cm_matmul_noalloc(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k, unsigned m,
                                 unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                                 unsigned c_batch_stride, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (n == 0 || m == 0 || batch == 0) return CM_OK;
    if (!c || (k > 0 && (!a || !b))) return set_error(CM_EINVAL, "cm_matmul_noalloc: null buffer");
    if (k > kMaxGemmK) return set_error(CM_EUNSUPPORTED, "cm_matmul_noalloc: k = %u exceeds %u", k, kMaxGemmK);
    cudaStream_t s = (cudaStream_t)stream;
    if (k == 0) return fill_zero(cx, c, batch, n, m, m, c_batch_stride, s);
    void* base = nullptr;
    rc = noalloc_scratch(cx->device, &base);
    if (rc) return rc;
    if (batch > 1 && (uint64_t)c_batch_stride < (uint64_t)n * m) {
        // Overlapping output slices: batch steps in order, later ones win; the
        // steps follow each other on `stream`, so they may reuse the scratch.
        const uint64_t first = c_batch_stride == 0 ? batch - 1 : 0;
        for (uint64_t bi = first; bi < batch && !rc; ++bi)
            rc = noalloc_run(cx, (uint8_t*)base, a + bi * a_batch_stride, b + bi * b_batch_stride,
                             c + bi * c_batch_stride, n, k, m, 1, a_batch_stride, b_batch_stride, 0, s);
    } else {
        rc = noalloc_run(cx, (uint8_t*)base, a, b, c, n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, s);
    }
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_matmul_noalloc");
}

extern "C" int cm_matmul_at(const int16_t* a, unsigned a_off, const int16_t* b, unsigned b_off, int16_t* c,
                            unsigned c_off, unsigned n, unsigned k, unsigned m, unsigned batch,
                            unsigned a_batch_stride, unsigned b_batch_stride, unsigned c_batch_stride) {
    return cm_matmul(a ? a + a_off : a, b ? b + b_off : b, c ? c + c_off : c, n, k, m, batch, a_batch_stride,
                     b_batch_stride, c_batch_stride);
}

// ---------------------------------------------------------------------------
// cm_int8_mma_rate: the int8 tensor pipe's ceiling, measured (no reference counterpart)
// ---------------------------------------------------------------------------
extern "C" int cm_int8_mma_rate(unsigned pairs, unsigned iters, double* tops, double* ms, double* sm_mhz) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!tops || !ms) return set_error(CM_EINVAL, "cm_int8_mma_rate: null output");
    if (iters == 0 || iters > (1u << 16)) return set_error(CM_EINVAL, "cm_int8_mma_rate: iters 1..65536");
    if (pairs > 1) return set_error(CM_EINVAL, "cm_int8_mma_rate: pairs is 0 or 1");
    const int CG = pairs ? 2 : 1;
    const void* fn = pairs ? (const void*)mma_rate_kernel<2> : (const void*)mma_rate_kernel<1>;
    // the whole per-CTA shared memory, so that one CTA runs per SM, as in the GEMM
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(mma rate)");
    int ctas = cx->sm_count;
    cudaLaunchConfig_t q{};
    q.blockDim = dim3(128);
    q.dynamicSmemBytes = SMEM_BYTES;
    cudaLaunchAttribute at{};
    at.id = cudaLaunchAttributeClusterDimension;
    at.val.clusterDim.x = CG; at.val.clusterDim.y = 1; at.val.clusterDim.z = 1;
    q.attrs = &at; q.numAttrs = 1;
    if (CG == 2) {
        q.gridDim = dim3(cx->sm_count);
        int m = 0;
        if (cudaOccupancyMaxActiveClusters(&m, (void*)fn, &q) == cudaSuccess && m > 0) ctas = 2 * m;
        else ctas = cx->sm_count & ~1;
        cudaGetLastError();
    }
    q.gridDim = dim3(ctas);
    cudaStream_t s = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if ((e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess) return cuda_error(e, "stream");
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    q.stream = s;
    unsigned long long* clk = nullptr;           // CTA 0's clock64 ticks and nanoseconds
    if ((e = cudaMalloc(&clk, 2 * sizeof(unsigned long long))) != cudaSuccess) rc = cuda_error(e, "cudaMalloc(mma rate)");
    // one untimed launch (module load, clocks up), then the timed one
    for (int pass = 0; pass < 2 && !rc; ++pass) {
        if (pass == 1) cudaEventRecord(e0, s);
        e = pairs ? cudaLaunchKernelEx(&q, mma_rate_kernel<2>, iters, cx->status, cx->timeout_ns, clk)
                  : cudaLaunchKernelEx(&q, mma_rate_kernel<1>, iters, cx->status, cx->timeout_ns, clk);
        count_launch();
        if (e != cudaSuccess) rc = cuda_error(e, "mma rate launch");
    }
    cudaEventRecord(e1, s);
    if (!rc) rc = finish_sync((cm_stream_t)s);
    float t = 0.f;
    if (!rc && (e = cudaEventElapsedTime(&t, e0, e1)) != cudaSuccess) rc = cuda_error(e, "mma rate events");
    unsigned long long hc[2] = {0, 0};
    if (!rc && (e = cudaMemcpy(hc, clk, sizeof(hc), cudaMemcpyDeviceToHost)) != cudaSuccess) rc = cuda_error(e, "mma rate clock");
    if (clk) cudaFree(clk);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(s);
    if (rc) return rc;
    if (sm_mhz) *sm_mhz = hc[1] ? 1e3 * (double)hc[0] / (double)hc[1] : 0.0;
    // per CTA and round: 4 K steps x 2 MMAs x 128 rows x 256 columns x 32 deep, 2 ops per MAC
    const double ops = (double)ctas * iters * 4.0 * 2.0 * 128.0 * 256.0 * 32.0 * 2.0;
    *ms = t;
    *tops = t > 0.f ? ops / (t * 1e-3) / 1e12 : 0.0;
    return CM_OK;
}
