// W4A16 group-128 GEMM for M > 16 on 5th-generation tensor cores (tcgen05 + TMEM).
//
// Reference semantics (src/ecpu/src/kernel/kernels.c:1089-1139):
//     C[m,n] = rne_bf16( sum_g s[n,g] * sum_{k in g} A[m,k] * q[n,k] )
// computed here with the same structure: every 128-wide quant group g is one exact
// group dot product on the tensor cores (int4 values are exact in bf16, products are
// exact in fp32), and the epilogue adds dot_g * s[n,g] into an fp32 accumulator with
// the product rounded before the add, as the reference does.
//
// CTA tile: 128 weight rows (the MMA M dimension, TMEM lanes) x up to 128 activation
// rows (the MMA N dimension), over a range of quant groups: the CTA's contiguous range of
// (tile, group) units under a stream-K or split schedule (below).  Warp roles
// (448 threads); a warp reaches TMEM lanes 32 * (warp % 4) .. + 31 only:
//   warp 0      TMA, one thread: per group the packed weight tile [128 rows x 64 B] (raw
//               ring) and the activation tile [Nm rows x 128 k] (two SWIZZLE_128B boxes,
//               X ring) on one barrier; every 16th group a [128 rows x 16 groups] fp32
//               tile of group scales
//   warp 1      TMEM owner + MMA issuer: 8 x tcgen05.mma (M=128, N=Nm, K=16) per group,
//               A from TMEM, B from shared memory, into one of two TMEM partials
//   warps 2-5   dequant: warp w owns TMEM lane quadrant w % 4 and dequantizes its 32 rows
//               of every group (64 packed bytes -> 128 bf16 per row) into one of four A
//               stages (tcgen05.st).  Four stages let it run up to four groups ahead of the
//               tensor pipe, so a stage is nearly always free when it gets there.
//   warps 6-13  fold: two per lane quadrant, each half of the activation columns (up to
//               64 fp32 accumulators a thread in 128 registers; four warps a quadrant, each
//               a quarter, spilled at their 80-register cap and ran 2-3% slower).
//               For every group in order: wait for its MMAs, tcgen05.ld the partial,
//               hand the partial buffer back to the issuer at once, then
//               acc = acc + rn(part * s[n,g]).
// The roles work on different groups at the same time: while the tensor pipe runs the
// MMAs of group i, the fold warps drain group i - 1 and the dequant warps fill group
// i + 1 .. i + 3.  Keeping A in TMEM (not shared memory) halves the shared-memory traffic
// per group.
// The MMA issuer pays for one barrier wait and one commit per group: the issuing thread
// is held while its MMAs execute, so every extra wait there leaves the tensor pipe idle.
// Measured with clock64 at Nm = 96: each 128 x 96 x 16 MMA holds the issuer about 70
// cycles (the tensor pipe's intake for this shape; a second issuer warp did not raise
// it), and the commit plus the next wait add about 400, so the issuer's ~1000 cycles per
// group, not the dequant or the fold, set the pace.
// Every mbarrier wait is bounded: on timeout the CTA records an error, drains, frees
// its TMEM and returns, and the host reports ECPU_ERR_KERNEL.
#include <cuda.h>
#include <cstring>
#include <mutex>

#include "common.cuh"

using namespace pilm;

namespace {

constexpr int kTileRows = 128;   // weight rows per CTA
constexpr int kMaxNm = 128;      // activation rows per CTA
constexpr int kRawStages = 8;
constexpr int kXStages = 4;
constexpr int kAStages = 4;                          // A buffers in TMEM (64 columns each)
constexpr int kRawBytes = kTileRows * 64;            // one group of packed weights
constexpr int kXSubBytes = kMaxNm * 128;             // Nm rows x 64 k bf16 (max)
constexpr int kXBytes = 2 * kXSubBytes;
constexpr int kDqWarps = 4;                          // warps 2-5
constexpr int kFoldWarps = 8;                        // warps 6-13
constexpr int kFoldSets = kFoldWarps / 4;            // fold warps per lane quadrant, each a column set
static_assert((kMaxNm / 16) / kFoldSets == 4, "a fold warp holds at most 4 chunks of 16 partial columns (CH)");
constexpr int kThreads = (2 + kDqWarps + kFoldWarps) * 32;
constexpr int kTBufs = 2;                            // TMEM partial buffers (kMaxNm columns each)
constexpr int kTmemCols = 512;
constexpr int kAColBase = 0;                         // TMEM columns [0, 256): A stages
constexpr int kAccColBase = kAStages * 64;           // TMEM columns [256, 512): partials
constexpr uint32_t kWaitLimit = 1u << 20;            // polls before a wait gives up (bounded wait)
constexpr uint32_t kSleepHintNs = 2000;              // longest sleep of one poll

// Every mbarrier operation costs a few hundred cycles inside this kernel, so each group
// has exactly three, all on rings indexed by slot i % kSlots:
//   in_full[q]   the TMA copies of group i (packed weights and activations) complete
//                here: the dequant warps' wait for their inputs
//   op_full[q]   the MMA issuer's one wait.  One arrival per dequant warp once its rows of
//                A(i) are in TMEM, and one per fold warp once it has loaded group i - 2's
//                partial (the buffer group i writes; groups 0 and 1 get theirs up front).
//                The producer also waits here before reusing raw slot i % 8.
//   mma_done[q]  the issuer's one commit: the fold warps wait for group i's partial, the
//                producer for X stage i % 4 (group i + 4); the dequant warps reuse A stage
//                i % 4 once in_full(i + 4) completes, which the producer issued only after
//                this commit
// A waiter's parity is (j / kSlots) & 1 for the group j it needs.  No waiter can fall
// kSlots or more completions behind: every later phase of its slot needs work that the
// waiter itself has not released yet, so parities never alias.
constexpr int kSlots = 8;
static_assert(kSlots == kRawStages && kXStages == 4 && kAStages == 4 && kTBufs == 2, "pipeline depths");
static_assert(kAccColBase + kTBufs * kMaxNm <= kTmemCols, "TMEM budget");

struct __align__(8) Barriers {
    uint64_t in_full[kSlots];
    uint64_t x_pre[kXStages];  // activations of the first kXStages groups (loaded after the wait)
    uint64_t op_full[kSlots], mma_done[kSlots];
    uint64_t s_full[2], s_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
};

constexpr size_t kSmemRaw = 0;
constexpr size_t kSmemX = kSmemRaw + (size_t)kRawStages * kRawBytes;   // 64 KB, 1024-aligned
constexpr int kScaleChunk = 16;                      // groups per scale tile [128 rows x 16 groups] fp32
constexpr int kScaleBytes = kTileRows * kScaleChunk * 4;
constexpr size_t kSmemScale = kSmemX + (size_t)kXStages * kXBytes;     // +128 KB
constexpr size_t kSmemBar = kSmemScale + 2 * (size_t)kScaleBytes;      // +16 KB (two scale tiles)
constexpr size_t kSmemTotal = kSmemBar + sizeof(Barriers) + 1024;      // + alignment slack
static_assert(kSmemTotal <= 227 * 1024, "shared memory budget");

// ---- PTX wrappers ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: a waiting warp sleeps until the phase completes (or
// the hint elapses) instead of re-issuing the poll, leaving issue slots to working warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(kSleepHintNs)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false (and raises the CTA abort flag) if the phase never completes.
// The MMA issuer polls (its waits are nearly always already satisfied); every other role
// sleeps between polls.  The abort flag is read every 16 polls.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag, uint32_t limit,
                                          bool sleep = true) {
    if (mbar_try_wait(b, parity)) return true;  // already complete: no suspend
    for (uint32_t i = 0; i < limit; ++i) {
        if (sleep ? mbar_try_wait_sleep(b, parity) : mbar_try_wait(b, parity)) return true;
        if ((i & 15) == 15 && *abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

// Bounded wait that ignores the abort flag: used to drain copies already issued, which
// always complete, before the CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t *b, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(b, parity)) return;
}

// Warp-collective bounded wait: every lane waits (each gets the acquire), then the warp
// reconverges before the .sync.aligned tcgen05 instructions that follow; a timeout in
// any lane makes the whole warp give up together.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *b, uint32_t parity, volatile int *abort_flag,
                                               uint32_t limit) {
    const bool ok = mbar_wait(b, parity, abort_flag, limit);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

// K-major SWIZZLE_128B shared-memory matrix descriptor (8-row x 128-byte atoms, 1024 B
// between 8-row groups), tcgen05 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// D[tmem] (+)= A[tmem] * B[smem desc]   (A: 128 lanes x K/2 columns, two bf16 per column)
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// int4 nibble pair at bits [0,4) and [16,20) -> bf16x2, exact (see linear.cu)
__device__ __forceinline__ uint32_t dq_pair(uint32_t w) {
    uint32_t t;
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(t) : "r"(w), "r"(0x000F000Fu), "r"(0x43084308u));
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&t);
    v = __hsub2(v, __floats2bfloat162_rn(136.0f, 136.0f));
    return *reinterpret_cast<uint32_t *>(&v);
}

// 8 packed int4 (one 32-bit word, k0..k7 at nibbles 0..7) -> 8 bf16 in k order (uint4)
__device__ __forceinline__ uint4 dq_word(uint32_t w) {
    const uint32_t p0 = dq_pair(w), p1 = dq_pair(w >> 4), p2 = dq_pair(w >> 8), p3 = dq_pair(w >> 12);
    // p0 = (k0,k4) p1 = (k1,k5) p2 = (k2,k6) p3 = (k3,k7)
    uint4 o;
    o.x = __byte_perm(p0, p1, 0x5410);  // k0,k1
    o.y = __byte_perm(p2, p3, 0x5410);  // k2,k3
    o.z = __byte_perm(p0, p1, 0x7632);  // k4,k5
    o.w = __byte_perm(p2, p3, 0x7632);  // k6,k7
    return o;
}

// The same 8 values from a word in the k-pair nibble order (nibble p holds k = 2p for
// p < 4 and 2(p - 4) + 1 above): each nibble pair (p, p + 4) is already (k_2j, k_2j+1),
// so no byte permute is needed.
__device__ __forceinline__ uint4 dq_word_kpairs(uint32_t w) {
    uint4 o;
    o.x = dq_pair(w);        // k0,k1
    o.y = dq_pair(w >> 4);   // k2,k3
    o.z = dq_pair(w >> 8);   // k4,k5
    o.w = dq_pair(w >> 12);  // k6,k7
    return o;
}

struct TcParams {
    const float *S;     // scales [N, G] (grouped) or [N] (per-row)
    __nv_bfloat16 *Y;   // [M, N]
    float *part;        // pieces of cut tiles: [P][2][kMaxNm columns][128 rows] fp32
    int *cnt;           // arrivals per (tile, fold warp): zero-initialised, self-resetting
    float *ws;          // split schedule: fp32 partials [splits, M, N] for splitk_combine
    int split_mode;     // 1: CTA c runs split c % splits of tile c / splits (gps groups)
    int splits, gps;
    int *err;           // device error word
    int M, N, K, G;
    int Nm;             // activation rows per tile (multiple of 16, <= 128)
    int tiles_n;        // 128-row weight tiles; tile t = tile_n + tiles_n * tile_m
    int U;              // work units: tiles x G (unit w = t * G + group); U * P < 2^31
    int P;              // CTAs, one per SM
    uint32_t idesc;
    int grouped;
    int scale_tma;      // group scales arrive by TMA (G % 4 == 0, group offsets 16-byte aligned)
    uint32_t wait_limit;  // polls before a pipeline wait gives up (drains keep kWaitLimit)
    unsigned long long *amax;  // AM: per output row, the max of argmax_key over the row's outputs
};

// Order-preserving key of output value f at column (vocab index) idx: the largest key is
// the largest value, ties going to the smallest index; NaN never wins and -0 equals +0,
// as in a first-max row argmax (row_top2).
__device__ __forceinline__ unsigned long long argmax_key(float f, int idx) {
    if (f != f) return 0ull;
    uint32_t b = f == 0.f ? 0u : __float_as_uint(f);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}



// Two schedules over the units w = t * G + group, each CTA running one contiguous range:
//  * stream-K (at least one tile per SM): CTA c takes [c U / P, (c+1) U / P), walking
//    through tiles and their groups in order, so every SM gets the same number of groups
//    and the rings stream straight across tile boundaries.  A tile cut by a range boundary
//    is reduced in the kernel (the last piece to arrive adds them up).
//  * split (fewer tiles than SMs): CTA c runs groups [s gps, (s+1) gps) of tile c / splits,
//    s = c % splits, and writes fp32 partials that splitk_combine sums in split order.  With
//    few tiles, stream-K would cut each into many pieces and put their reduction on the
//    critical path.
__device__ __forceinline__ int unit_begin(int c, const TcParams &p) { return (int)(((unsigned)c * (unsigned)p.U) / (unsigned)p.P); }
// the CTA whose range holds unit w
__device__ __forceinline__ int cta_of_unit(int w, const TcParams &p) {
    int c = (int)(((unsigned)w * (unsigned)p.P) / (unsigned)p.U);
    if (c >= p.P) c = p.P - 1;
    while (c + 1 < p.P && unit_begin(c + 1, p) <= w) ++c;
    while (c > 0 && unit_begin(c, p) > w) --c;
    return c;
}
// a CTA keeps a cut tile's piece in slot 0 for its first tile, slot 1 for its last
__device__ __forceinline__ float *piece_of(const TcParams &p, int c, int t) {
    const int slot = t == unit_begin(c, p) / p.G ? 0 : 1;
    return p.part + (size_t)(c * 2 + slot) * kMaxNm * kTileRows;
}

// AM: also fold each finished output row's argmax (over the tile's weight rows, the
// vocabulary of an LM head) into p.amax by atomicMax of argmax_key (stream-K schedule).
// CH: 16-column chunks of the partial per fold warp (3: Nm <= 96, 4: Nm <= 128).
template <bool KP, bool AM, int CH>
__global__ void __launch_bounds__(kThreads, 1) w4_gemm_tc(const __grid_constant__ CUtensorMap wmap,
                                                         const __grid_constant__ CUtensorMap xmap,
                                                         const __grid_constant__ CUtensorMap smap,
                                                         const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    // AM: each fold warp's running argmax key per output row over every tile it writes
    // (its own slots, so no atomics inside the loop); at the end the CTA takes the max over
    // its warps and makes one global atomicMax per row (one per tile and warp, on the same
    // few words, cost 0.2 ms per LM-head call)
    __shared__ unsigned long long s_amax[AM ? kFoldWarps * kMaxNm : 1];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    Barriers *bar = reinterpret_cast<Barriers *>(smem + kSmemBar);
    volatile int *abort_flag = &bar->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int G = p.G;
    int W0, ng, split = 0;  // this CTA's first unit and group count (>= 1)
    if (p.split_mode) {
        split = cta % p.splits;
        const int gs = split * p.gps;
        W0 = (cta / p.splits) * G + gs;
        ng = min(G, gs + p.gps) - gs;
    } else {
        W0 = unit_begin(cta, p);
        ng = unit_begin(cta + 1, p) - W0;
    }

    // programmatic dependent launch: the next kernel may launch now; this CTA's setup and
    // an L2 prefetch of its first weight tiles (never written by another kernel) overlap
    // the previous kernel, and nothing else touches global memory before it completes
    pdl_trigger();
    if (threadIdx.x == 32 * 2) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
        int t = W0 / G, g = W0 % G;
        int row0 = (t % p.tiles_n) * kTileRows;
        for (int i = 0; i < ng && i < kRawStages; ++i) {
            if (i >= kXStages)  // the first kXStages groups are copied to shared memory directly
                asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(&wmap),
                             "r"(g * 64), "r"(row0)
                             : "memory");
            if (++g == G) {
                g = 0;
                row0 = row0 + kTileRows >= p.tiles_n * kTileRows ? 0 : row0 + kTileRows;
            }
        }
    }
    if (threadIdx.x == 0) {
        // consumer-side barriers take one arrival per warp (lane 0 after __syncwarp)
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&bar->in_full[i], 1);  // the producer's arrive.expect_tx
            mbar_init(&bar->op_full[i], kDqWarps + kFoldWarps);
            mbar_init(&bar->mma_done[i], 1);
        }
        for (int i = 0; i < kXStages; ++i) mbar_init(&bar->x_pre[i], 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar->s_full[i], 1);
            mbar_init(&bar->s_empty[i], kFoldWarps);
        }
        mbar_init(&bar->drain, 1);
        bar->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(&bar->tmem_base, kTmemCols);
    if (AM)
        for (int i = threadIdx.x; i < kFoldWarps * kMaxNm; i += blockDim.x) s_amax[i] = 0ull;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bar->tmem_base;
    // No wait for the previous kernel here.  The first npre groups' weights (and their
    // scale tile) are copied and dequantized into TMEM while it runs: the dequant and MMA
    // warps touch only shared memory and TMEM.  The producer waits before it copies
    // activations (that kernel's output), the fold warps before they write.
    // (At most two scale tiles may be requested before the fold warps release one: with a
    // single group per tile (G = 1) every group starts a scale tile, so only two go early.)
    const int npre = min(ng, G >= 2 ? kXStages : 2);

    const int x_bytes = 2 * p.Nm * 128;

    if (warp == 0) {
        // ---- TMA: packed weights into the raw ring, activations into the X ring, and
        // group scales into a two-slot ring: a [128 rows x 16 groups] tile whenever a
        // group starts one (a slot is refilled once every fold warp has finished with it) ----
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
            if (p.scale_tma) asm volatile("prefetch.tensormap [%0];" ::"l"(&smap) : "memory");
            int issued = 0, s_issued = 0;
            int t = W0 / G, g = W0 % G - 1;
            int row0 = (t % p.tiles_n) * kTileRows, m0 = (t / p.tiles_n) * kMaxNm;
            int pre_g[kXStages], pre_m0[kXStages];
            for (int i = 0; i < ng; ++i) {
                if (++g == G) {  // next tile: next 128 weight rows, or the next activation tile
                    g = 0;
                    ++t;
                    row0 += kTileRows;
                    if (row0 >= p.tiles_n * kTileRows) {
                        row0 = 0;
                        m0 += kMaxNm;
                    }
                }
                if (p.scale_tma && (i == 0 || g % kScaleChunk == 0)) {
                    const int sq = s_issued, slot = sq & 1;
                    if (sq >= 2 && !mbar_wait(&bar->s_empty[slot], (uint32_t)((sq - 2) >> 1) & 1u, abort_flag, p.wait_limit)) break;
                    mbar_expect_tx(&bar->s_full[slot], kScaleBytes);
                    tma_load_2d(smem + kSmemScale + (size_t)slot * kScaleBytes, &smap, &bar->s_full[slot],
                                kScaleChunk * (g / kScaleChunk), row0);
                    ++s_issued;
                }
                // raw slot i % 8 held group i - 8, read by the dequant warps before they
                // arrived on that group's op_full; X stage i % 4 held group i - 4, read by
                // its MMAs
                if (i >= kRawStages && !mbar_wait(&bar->op_full[(i - kRawStages) % kSlots],
                                                  (uint32_t)((i - kRawStages) / kSlots) & 1u, abort_flag, p.wait_limit))
                    break;
                if (i >= kXStages && !mbar_wait(&bar->mma_done[(i - kXStages) % kSlots],
                                                (uint32_t)((i - kXStages) / kSlots) & 1u, abort_flag, p.wait_limit))
                    break;
                uint64_t *full = &bar->in_full[i % kSlots];
                if (i < npre) {
                    // weights only: in_full(i) completes without the activations, which
                    // land on x_pre(i) once the previous kernel has completed
                    mbar_expect_tx(full, (uint32_t)kRawBytes);
                    tma_load_2d(smem + kSmemRaw + (size_t)i * kRawBytes, &wmap, full, g * 64, row0);
                    pre_g[i] = g;
                    pre_m0[i] = m0;
                    ++issued;
                    if (i == npre - 1) {
                        pdl_wait();
                        for (int j = 0; j < npre; ++j) {
                            uint8_t *dst = smem + kSmemX + (size_t)j * kXBytes;
                            mbar_expect_tx(&bar->x_pre[j], (uint32_t)x_bytes);
                            tma_load_2d(dst, &xmap, &bar->x_pre[j], pre_g[j] * 128, pre_m0[j]);
                            tma_load_2d(dst + (size_t)p.Nm * 128, &xmap, &bar->x_pre[j], pre_g[j] * 128 + 64, pre_m0[j]);
                        }
                    }
                    continue;
                }
                mbar_expect_tx(full, (uint32_t)(kRawBytes + x_bytes));
                tma_load_2d(smem + kSmemRaw + (size_t)(i % kRawStages) * kRawBytes, &wmap, full, g * 64, row0);
                uint8_t *dst = smem + kSmemX + (size_t)(i % kXStages) * kXBytes;
                tma_load_2d(dst, &xmap, full, g * 128, m0);
                tma_load_2d(dst + (size_t)p.Nm * 128, &xmap, full, g * 128 + 64, m0);
                ++issued;
            }
            // drain: every issued copy has landed before the CTA may exit
            for (int i = issued > kSlots ? issued - kSlots : 0; i < issued; ++i)
                mbar_drain(&bar->in_full[i % kSlots], (uint32_t)(i / kSlots) & 1u);
            for (int c = s_issued > 2 ? s_issued - 2 : 0; c < s_issued; ++c)
                mbar_drain(&bar->s_full[c & 1], (uint32_t)(c >> 1) & 1u);
            if (issued >= npre)  // the activation copies of the first groups were issued
                for (int j = 0; j < npre; ++j) mbar_drain(&bar->x_pre[j], 0);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            for (int i = 0; i < ng; ++i) {
                const int q = i % kSlots, sa = i % kAStages, sx = i % kXStages, b = i % kTBufs;
                if (!mbar_wait(&bar->op_full[q], (uint32_t)(i / kSlots) & 1u, abort_flag, p.wait_limit)) break;
                if (i < npre && !mbar_wait(&bar->x_pre[i], 0, abort_flag, p.wait_limit)) break;
                tc_fence_after();
                const uint32_t a_col = tmem + (uint32_t)(kAColBase + sa * 64);
                const uint32_t x_base = smem_u32(smem + kSmemX + (size_t)sx * kXBytes);
                const uint32_t d = tmem + (uint32_t)(kAccColBase + b * kMaxNm);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint64_t bd = sw128_desc(x_base + h * p.Nm * 128);
#pragma unroll
                    for (int k = 0; k < 4; ++k)  // K=16 per MMA: 8 TMEM columns of A, 32 B of B
                        umma_bf16_ts(d, a_col + (uint32_t)(8 * (4 * h + k)), bd + 2 * k, p.idesc,
                                     (h | k) ? 1u : 0u);
                }
                umma_commit(&bar->mma_done[q]);
            }
            // drain: all issued MMAs have completed before TMEM is released
            umma_commit(&bar->drain);
            mbar_drain(&bar->drain, 0);
        }
        __syncwarp();
    } else if (warp < 2 + kDqWarps) {
        // ---- dequant: rows 32 * quad .. + 31 of every group into A stage i % 4 ----
        const int quad = warp & 3;
        const int rloc = 32 * quad + lane;  // this thread's weight row in the tile = TMEM lane
        const uint32_t lane_addr = (uint32_t)(32 * quad) << 16;
        const int sw = (rloc >> 1) & 3;
        for (int i = 0; i < ng; ++i) {
            const int sa = i % kAStages;
            // A stage sa held group i - 4.  Its MMAs have completed: the producer waited for
            // them (mma_done(i - 4)) before it loaded group i, whose copies completing is what
            // in_full(i) says, so this one wait covers both (one barrier wait fewer per group
            // and dequant warp: 3% faster)
            if (!mbar_wait_warp(&bar->in_full[i % kSlots], (uint32_t)(i / kSlots) & 1u, abort_flag, p.wait_limit)) break;
            tc_fence_after();
            // raw tile written with SWIZZLE_64B: 16-byte chunk c of row r sits at chunk
            // c ^ ((r >> 1) & 3), so 8 consecutive rows hit 8 distinct bank groups
            const uint8_t *rowp = smem + kSmemRaw + (size_t)(i % kRawStages) * kRawBytes + rloc * 64;
#pragma unroll 2
            for (int c = 0; c < 4; ++c) {  // 16 bytes = 32 k values -> 16 columns
                const uint4 v = *reinterpret_cast<const uint4 *>(rowp + ((c ^ sw) << 4));
                const uint32_t words[4] = {v.x, v.y, v.z, v.w};
                uint32_t cols[16];
#pragma unroll
                for (int q = 0; q < 4; ++q) {  // 8 k values per word -> 4 columns
                    const uint4 o = KP ? dq_word_kpairs(words[q]) : dq_word(words[q]);
                    cols[4 * q + 0] = o.x;
                    cols[4 * q + 1] = o.y;
                    cols[4 * q + 2] = o.z;
                    cols[4 * q + 3] = o.w;
                }
                tmem_st16(tmem + lane_addr + (uint32_t)(kAColBase + sa * 64 + 16 * c), cols);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->op_full[i % kSlots]);
        }
    } else {
        // ---- fold: activation-column set fq of lane quadrant quad, every group in order ----
        const int quad = warp & 3;
        const int fw = warp - 2 - kDqWarps;  // 0 .. kFoldWarps - 1
        const int fq = fw >> 2;              // column set 0 .. kFoldSets - 1
        const int rloc = 32 * quad + lane;
        const uint32_t lane_addr = (uint32_t)(32 * quad) << 16;
        const int nc = p.Nm / 16;            // 16-column chunks of the partial (<= 8)
        const int per = (nc + kFoldSets - 1) / kFoldSets;  // chunks per set (<= CH)
        const int c_lo = fq * per, c_hi = min(nc, c_lo + per);
        const float *sring = reinterpret_cast<const float *>(smem + kSmemScale);
        float2 acc[8 * CH];  // 16-column chunks as fp32 pairs: one packed multiply and add per pair

#pragma unroll
        for (int e = 0; e < 8 * CH; ++e) acc[e] = make_float2(0.f, 0.f);
        // partial buffers 0 and 1 start free
        __syncwarp();
        if (lane == 0)
            for (int i = 0; i < kTBufs && i < ng; ++i) mbar_arrive(&bar->op_full[i]);
        pdl_wait();  // before the first write (outputs, pieces, counters)
        int s_seen = 0;   // scale tiles started so far (the producer's sequence)
        int t = W0 / G, g = W0 % G;
        int row = (t % p.tiles_n) * kTileRows + rloc;
        // one pass per tile segment: the groups of tile t this CTA runs, then the write-out
        // (kept out of the per-group loop, whose registers the accumulators fill)
        for (int i = 0; i < ng;) {
            const int seg_g0 = g;
            const int seg_end = min(ng, i + (G - g));  // exclusive
            const bool row_ok = row < p.N;
            bool aborted = false;
            for (; i < seg_end; ++i, ++g) {
                // group g's scale first: the tile arrives long before the MMAs complete
                float sc = 1.0f;
                if (p.grouped) {
                    if (p.scale_tma) {
                        if (i == 0 || g % kScaleChunk == 0) {
                            const int sq = s_seen++;
                            if (!mbar_wait_warp(&bar->s_full[sq & 1], (uint32_t)(sq >> 1) & 1u, abort_flag, p.wait_limit)) {
                                aborted = true;
                                break;
                            }
                        }
                        const int slot = (s_seen - 1) & 1;
                        sc = sring[(size_t)slot * (kTileRows * kScaleChunk) + rloc * kScaleChunk + g % kScaleChunk];
                        if (i == ng - 1 || g == G - 1 || (g + 1) % kScaleChunk == 0) {
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&bar->s_empty[slot]);  // done with this scale tile
                        }
                    } else {
                        sc = row_ok ? __ldg(p.S + (size_t)row * G + g) : 0.f;
                    }
                }
                const float2 sc2 = make_float2(sc, sc);
                if (!mbar_wait_warp(&bar->mma_done[i % kSlots], (uint32_t)(i / kSlots) & 1u, abort_flag, p.wait_limit)) {
                    aborted = true;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem + lane_addr + (uint32_t)(kAccColBase + (i % kTBufs) * kMaxNm);
                if constexpr (CH <= 3) {
                    // all chunks into registers with one wait, the buffer straight back to the
                    // issuer for group i + 2, then the arithmetic (2-3% faster than holding
                    // the buffer through the chunks' arithmetic; four chunks do not fit)
                    uint32_t r[CH][16];
#pragma unroll
                    for (int u = 0; u < CH; ++u)
                        if (c_lo + u < c_hi) tmem_ld16(taddr + 16 * (c_lo + u), r[u]);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0 && i + kTBufs < ng) mbar_arrive(&bar->op_full[(i + kTBufs) % kSlots]);
#pragma unroll
                    for (int u = 0; u < CH; ++u) {
                        if (c_lo + u >= c_hi) continue;
#pragma unroll
                        for (int e = 0; e < 8; ++e) {  // acc += rn(p * s), per element as the reference
                            const float2 pv = make_float2(__uint_as_float(r[u][2 * e]), __uint_as_float(r[u][2 * e + 1]));
                            acc[u * 8 + e] = __fadd2_rn(acc[u * 8 + e], p.grouped ? __fmul2_rn(pv, sc2) : pv);
                        }
                    }
                } else {
                    // one 16-column chunk at a time (register budget); the buffer goes back to
                    // the issuer for group i + 2 as soon as the last chunk is in registers
#pragma unroll
                    for (int u = 0; u < CH; ++u) {
                        uint32_t r[16];
                        const bool have = c_lo + u < c_hi;
                        if (have) tmem_ld16(taddr + 16 * (c_lo + u), r);
                        tmem_ld_wait();
                        if (u == CH - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0 && i + kTBufs < ng) mbar_arrive(&bar->op_full[(i + kTBufs) % kSlots]);
                        }
                        if (!have) continue;
#pragma unroll
                        for (int e = 0; e < 8; ++e) {  // acc += rn(p * s), per element as the reference
                            const float2 pv = make_float2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
                            acc[u * 8 + e] = __fadd2_rn(acc[u * 8 + e], p.grouped ? __fmul2_rn(pv, sc2) : pv);
                        }
                    }
                }
            }
            if (aborted) break;
            // ---- end of this CTA's segment of tile t: write the tile, or its piece ----
            const int last_g = g - 1;
            const float sr = (p.grouped || !row_ok) ? 1.0f : __ldg(p.S + row);
            const int m0 = (t / p.tiles_n) * kMaxNm;
            const int mlim = min(p.Nm, p.M - m0);
            // the finished tile: bf16 outputs, and under AM each output row's argmax over the
            // warp's 32 weight rows folded into s_amax (ml < mlim is the same for the whole warp)
            auto write_tile = [&]() {
#pragma unroll
                for (int u = 0; u < CH; ++u) {
                    if (c_lo + u >= c_hi) continue;
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int ml = 16 * (c_lo + u) + k;  // activation row in the tile
                        if (ml >= mlim) continue;
                        const float a = (k & 1) ? acc[u * 8 + (k >> 1)].y : acc[u * 8 + (k >> 1)].x;
                        const __nv_bfloat16 v = f2bf(a * sr);
                        if (row_ok) p.Y[(size_t)(m0 + ml) * p.N + row] = v;
                        if (AM) {  // the warp's max key: max of the value words, then of the index words
                            const unsigned long long key = row_ok ? argmax_key(bf2f(v), row) : 0ull;
                            const uint32_t hi = (uint32_t)(key >> 32);
                            const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
                            const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (uint32_t)key : 0u);
                            const unsigned long long wk = ((unsigned long long)mhi << 32) | mlo;
                            unsigned long long *slot = &s_amax[fw * kMaxNm + ml];  // this warp's own: no atomics
                            if (lane == 0 && wk > *slot) *slot = wk;
                        }
                    }
                }
            };
            if (seg_g0 == 0 && last_g == G - 1) {
                write_tile();
            } else if (p.split_mode) {
                // split partial for splitk_combine
                if (row_ok) {
#pragma unroll
                    for (int u = 0; u < CH; ++u) {
                        if (c_lo + u >= c_hi) continue;
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            const int ml = 16 * (c_lo + u) + k;
                            const float a = (k & 1) ? acc[u * 8 + (k >> 1)].y : acc[u * 8 + (k >> 1)].x;
                            if (ml < mlim) p.ws[((size_t)split * p.M + m0 + ml) * p.N + row] = a;
                        }
                    }
                }
            } else {
                // cut tile: publish this piece; the last of the tile's CTAs to arrive (per fold
                // warp region) sums the pieces in CTA order and writes the tile
                float *pc = piece_of(p, cta, t) + rloc;
#pragma unroll
                for (int u = 0; u < CH; ++u) {
                    if (c_lo + u >= c_hi) continue;
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int ml = 16 * (c_lo + u) + 2 * e;
                        pc[(size_t)ml * kTileRows] = acc[u * 8 + e].x;
                        pc[(size_t)(ml + 1) * kTileRows] = acc[u * 8 + e].y;
                    }
                }
                __threadfence();
                __syncwarp();
                const int k0 = cta_of_unit(t * G, p), k1 = cta_of_unit(t * G + G - 1, p);
                int last = 0;
                if (lane == 0) last = atomicAdd(p.cnt + (size_t)t * kFoldWarps + fw, 1) == k1 - k0;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    // sum = 0 + piece(k0) + piece(k0 + 1) + ... in CTA order (deterministic)
#pragma unroll
                    for (int e = 0; e < 8 * CH; ++e) acc[e] = make_float2(0.f, 0.f);
                    for (int cc = k0; cc <= k1; ++cc) {
                        const float *pq = piece_of(p, cc, t) + rloc;
#pragma unroll
                        for (int u = 0; u < CH; ++u) {
                            if (c_lo + u >= c_hi) continue;
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const int ml = 16 * (c_lo + u) + 2 * e;
                                acc[u * 8 + e].x += __ldcg(pq + (size_t)ml * kTileRows);
                                acc[u * 8 + e].y += __ldcg(pq + (size_t)(ml + 1) * kTileRows);
                            }
                        }
                    }
                    write_tile();
                    if (lane == 0) p.cnt[(size_t)t * kFoldWarps + fw] = 0;  // self-reset for the next launch
                }
            }
#pragma unroll
            for (int e = 0; e < 8 * CH; ++e) acc[e] = make_float2(0.f, 0.f);
            // next tile: the next 128 weight rows, or the first of the next activation tile
            g = 0;
            ++t;
            row += kTileRows;
            if (row >= p.tiles_n * kTileRows) row = rloc;
        }
    }

    // ---- teardown ----
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        if (threadIdx.x == 0) atomicExch(p.err, 1);
    }
    if (AM)  // one activation tile (M <= 128): output row m is column m of every fold warp
        for (int i = threadIdx.x; i < p.Nm; i += blockDim.x) {
            unsigned long long k = 0ull;
#pragma unroll
            for (int w = 0; w < kFoldWarps; ++w) k = s_amax[w * kMaxNm + i] > k ? s_amax[w * kMaxNm + i] : k;
            if (k) atomicMax(p.amax + i, k);
        }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Split-K combine: Y[m, n] = rn_bf16((0 + P_0 + P_1 + ... + P_{s-1}) * sr[n]), the partials
// summed in split order (K order), as a separate fully parallel pass (8 outputs per thread).
// sr is the per-row scale of the ungrouped format (nullptr: grouped, already applied).
__global__ void __launch_bounds__(256) splitk_combine(const float *__restrict__ ws, int splits, int M, int N,
                                                      const float *__restrict__ sr, __nv_bfloat16 *__restrict__ Y) {
    pdl_entry();
    const size_t total8 = (size_t)M * N / 8;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total8) return;
    const size_t base = t * 8;  // N % 8 == 0: the 8 outputs share one row m
    const size_t plane = (size_t)M * N;
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = 0.f;
    for (int sp = 0; sp < splits; ++sp) {
        const float4 a = __ldcs(reinterpret_cast<const float4 *>(ws + sp * plane + base));
        const float4 b = __ldcs(reinterpret_cast<const float4 *>(ws + sp * plane + base + 4));
        v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
        v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    const int n0 = (int)(base % (size_t)N);
    uint32_t o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        float x0 = v[2 * u], x1 = v[2 * u + 1];
        if (sr) {
            x0 *= __ldg(sr + n0 + 2 * u);
            x1 *= __ldg(sr + n0 + 2 * u + 1);
        }
        const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
        o[u] = *reinterpret_cast<const uint32_t *>(&h);
    }
    *reinterpret_cast<uint4 *>(Y + base) = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- host side ---------------------------------------------------------------------------

// The schedule of one call: stream-K with one CTA per SM when there is at least one
// 128-row tile per SM, else `splits` CTAs per tile over gps groups each.
struct TcPlan {
    int G, tiles_m, tiles_n, tiles, Nm, P, splits, gps;
    bool stream_k;
};

TcPlan plan_tc(int M, int N, int K, bool can_split, int sms) {
    TcPlan t;
    t.G = K / 128;
    t.tiles_m = (M + kMaxNm - 1) / kMaxNm;
    // activation rows per CTA: all tiles use the same N (multiple of 16)
    t.Nm = t.tiles_m == 1 ? ((M + 15) / 16) * 16 : kMaxNm;
    t.tiles_n = (N + kTileRows - 1) / kTileRows;
    t.tiles = t.tiles_n * t.tiles_m;
    t.stream_k = t.tiles >= sms;
    t.P = sms;
    t.splits = 1;
    t.gps = t.G;
    if (!t.stream_k) {
        // Split K by a cost model in units of one group's pipeline time: every wave of CTAs
        // pays its groups per CTA plus a fixed prologue and pipeline fill (about 2 groups),
        // and a split adds one combine pass (about 3).  Splitting wants N % 8 == 0 and
        // 16-byte aligned output rows (the combine pass's vector loads and stores).
        double best = 1e30;
        const int max_splits = can_split ? (t.G < 16 ? t.G : 16) : 1;
        for (int s = 1; s <= max_splits; ++s) {
            const int g = (t.G + s - 1) / s;
            const int se = (t.G + g - 1) / g;
            if (se != s) continue;
            const int waves = (t.tiles * se + sms - 1) / sms;
            const double est = waves * (g + 2.0) + (se > 1 ? 3.0 : 0.0);
            if (est < best - 1e-9) {
                best = est;
                t.splits = se;
                t.gps = g;
            }
        }
        t.P = t.tiles * t.splits;
    }
    return t;
}
}  // namespace

namespace pilm {

size_t w4_tc_partials_bytes(int M, int N, int K) {
    if (M <= 16 || (K % 128) != 0 || N < 1) return 0;
    const TcPlan t = plan_tc(M, N, K, (N % 8) == 0, num_sms());
    return t.stream_k || t.splits <= 1 ? 0 : (size_t)t.splits * M * N * sizeof(float);
}

int linear_w4_tc(const __nv_bfloat16 *X, int M, int K, const uint8_t *W, const float *S, int N, __nv_bfloat16 *Y,
                 bool grouped, bool kpairs, const char *what, float *defer, size_t defer_cap, int *defer_splits,
                 unsigned long long *amax, int *amax_done) {
    if (defer_splits) *defer_splits = 0;
    if (amax_done) *amax_done = 0;
    static const bool disabled = getenv("PILM_DISABLE_TC") && getenv("PILM_DISABLE_TC")[0] == '1';
    if (disabled || M <= 16 || (K % 128) != 0 || N < 1) return ECPU_ERR_UNSUPPORTED;
    if ((((uintptr_t)X) & 15) || (((uintptr_t)W) & 15)) return ECPU_ERR_UNSUPPORTED;
    TensorMapEncodeTiledFn enc = tensor_map_encoder();
    int *err = device_error_word();
    if (!enc || !err) return ECPU_ERR_UNSUPPORTED;

    const int sms = num_sms();
    const TcPlan plan = plan_tc(M, N, K, (N % 8) == 0 && (((uintptr_t)Y) & 15) == 0, sms);
    const int G = plan.G, tiles_n = plan.tiles_n, tiles = plan.tiles, Nm = plan.Nm;
    const bool stream_k = plan.stream_k;
    const int P = plan.P, splits = plan.splits, gps = plan.gps;
    const long long U = (long long)tiles * G;
    if (stream_k && U * P >= (1ll << 31)) return ECPU_ERR_UNSUPPORTED;  // unit arithmetic is 32-bit

    CUtensorMap wmap, xmap;
    {
        cuuint64_t dims[2] = {(cuuint64_t)(K / 2), (cuuint64_t)N};
        cuuint64_t strides[1] = {(cuuint64_t)(K / 2)};
        cuuint32_t box[2] = {64, (cuuint32_t)kTileRows};
        cuuint32_t es[2] = {1, 1};
        if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)W, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return ECPU_ERR_UNSUPPORTED;
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)Nm};
        cuuint32_t es[2] = {1, 1};
        if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)X, dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return ECPU_ERR_UNSUPPORTED;
    }

    // Group scales by TMA: [128 rows x 16 groups] tiles at 16-group-aligned x (16-byte
    // aligned), which needs a 16-byte row pitch (G % 4 == 0) and base.
    const bool scale_tma = grouped && (G % 4) == 0 && ((uintptr_t)S & 15) == 0;

    CUtensorMap smap;
    memset(&smap, 0, sizeof(smap));
    bool smap_ok = false;
    if (scale_tma) {
        cuuint64_t dims[2] = {(cuuint64_t)G, (cuuint64_t)N};
        cuuint64_t strides[1] = {(cuuint64_t)G * 4};
        cuuint32_t box[2] = {(cuuint32_t)kScaleChunk, (cuuint32_t)kTileRows};
        cuuint32_t es[2] = {1, 1};
        smap_ok = enc(&smap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)S, dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }

    TcParams p;
    p.S = S;
    p.Y = Y;
    p.err = err;
    p.M = M;
    p.N = N;
    p.K = K;
    p.G = G;
    p.Nm = Nm;
    p.tiles_n = tiles_n;
    p.U = stream_k ? (int)U : 0;
    p.P = P;
    p.split_mode = stream_k ? 0 : 1;
    p.splits = splits;
    p.gps = gps;
    p.ws = nullptr;
    p.grouped = grouped ? 1 : 0;
    p.scale_tma = smap_ok ? 1 : 0;
    // kind::f16 instruction descriptor: D fp32, A/B bf16, K-major both, N = Nm, M = 128
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(Nm >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    p.part = nullptr;
    p.cnt = nullptr;
    p.wait_limit = wait_limit_override() >= 0 ? (uint32_t)wait_limit_override() : kWaitLimit;
    // the fused argmax needs every output written by this kernel: stream-K only (the split
    // schedule's outputs come from the combine pass), k-pair weights, one activation tile
    const bool am = amax && amax_done && stream_k && kpairs && plan.tiles_m == 1;
    p.amax = am ? amax : nullptr;
    if (stream_k) {
        p.part = (float *)workspace((size_t)P * 2 * kMaxNm * kTileRows * sizeof(float));
        p.cnt = counters((size_t)tiles * kFoldWarps);
        PILM_REQUIRE(p.part && p.cnt, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
    } else if (splits > 1) {
        // a caller that takes the partials itself (its own buffer, large enough) gets them
        // there and no combine pass runs
        const size_t need = (size_t)splits * M * N * sizeof(float);
        const bool deferred = defer && defer_splits && grouped && need <= defer_cap && (((uintptr_t)defer) & 15) == 0;
        p.ws = deferred ? defer : (float *)workspace(need);
        PILM_REQUIRE(p.ws, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
        if (deferred) *defer_splits = splits;
    }
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(w4_gemm_tc<false, false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        cudaFuncSetAttribute(w4_gemm_tc<true, false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        cudaFuncSetAttribute(w4_gemm_tc<true, true, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        cudaFuncSetAttribute(w4_gemm_tc<false, false, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        cudaFuncSetAttribute(w4_gemm_tc<true, false, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        cudaFuncSetAttribute(w4_gemm_tc<true, true, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        attr_set = true;
    }
    // fold chunks per warp: half of the Nm / 16 partial columns
    if (Nm <= 96) {
        if (am)
            launch_pdl(w4_gemm_tc<true, true, 3>, dim3(P), dim3(kThreads), kSmemTotal, wmap, xmap, smap, p);
        else if (kpairs)
            launch_pdl(w4_gemm_tc<true, false, 3>, dim3(P), dim3(kThreads), kSmemTotal, wmap, xmap, smap, p);
        else
            launch_pdl(w4_gemm_tc<false, false, 3>, dim3(P), dim3(kThreads), kSmemTotal, wmap, xmap, smap, p);
    } else {
        if (am)
            launch_pdl(w4_gemm_tc<true, true, 4>, dim3(P), dim3(kThreads), kSmemTotal, wmap, xmap, smap, p);
        else if (kpairs)
            launch_pdl(w4_gemm_tc<true, false, 4>, dim3(P), dim3(kThreads), kSmemTotal, wmap, xmap, smap, p);
        else
            launch_pdl(w4_gemm_tc<false, false, 4>, dim3(P), dim3(kThreads), kSmemTotal, wmap, xmap, smap, p);
    }
    int rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    if (am) *amax_done = 1;
    if (splits > 1 && !(defer_splits && *defer_splits)) {
        const size_t total8 = (size_t)M * N / 8;
        launch_pdl(splitk_combine, dim3((unsigned)((total8 + 255) / 256)), dim3(256), 0, p.ws, splits, M, N,
                                                                            grouped ? nullptr : S, Y);
        rc = check_launch(what);
        if (rc != ECPU_OK) return rc;
    }
    rc = check_error_word(what, "tensor-core GEMM pipeline timed out");
    if (rc != ECPU_OK && p.cnt) {
        // CTAs that gave up left some cut tiles' arrival counters short of their reset:
        // clear them so that the next call starts from zero
        cudaMemset(p.cnt, 0, (size_t)tiles * kFoldWarps * sizeof(int));
    }
    return rc;
}

}  // namespace pilm
