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
// rows (the MMA N dimension), over a range of quant groups (split-K).  Warp roles
// (640 threads):
//   warp 0      TMA: packed weight tile [128 rows x 64 B] per group -> raw ring
//   warp 1      TMA: activation tile [Nm rows x 128 k] (two SWIZZLE_128B boxes) -> X ring
//   warp 2      TMEM owner + MMA issuer: 8 x tcgen05.mma (M=128, N=Nm, K=16) per group,
//               A from TMEM, B from shared memory, into one of three TMEM partials
//   warp 3      TMA: group scales, [128 rows x 16 groups] fp32 tiles
//   warps 4-19  compute: warp w owns TMEM lane quadrant w%4 and quarter q = (w-4)/4 of the
//               work there.  Step i of a compute warp: wait for the MMAs of group i-2,
//               dequantize its quarter-row of group i (16 packed bytes -> 32 bf16, k in
//               [32q, 32q+32)) into the A stage those MMAs released (tcgen05.st), signal
//               the MMA issuer, then fold group i-2's partial into its accumulators
//               (tcgen05.ld, acc + rn(part * s[n,g]) for activation-row chunk q).  Four
//               compute warps share each SM sub-partition: the work of one step is a
//               short dependent chain, and the other warps' arithmetic hides its TMEM,
//               shared-memory and barrier latencies.  Keeping A in TMEM (not shared memory) halves
//               the shared-memory traffic per group.
// The MMA issuer pays for one barrier wait and one commit per group: the issuing thread
// is held while its MMAs execute, so every extra wait there leaves the tensor pipe idle.
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
constexpr int kAStages = 2;                          // A buffers in TMEM (64 columns each)
constexpr int kRawBytes = kTileRows * 64;            // one group of packed weights
constexpr int kXSubBytes = kMaxNm * 128;             // Nm rows x 64 k bf16 (max)
constexpr int kXBytes = 2 * kXSubBytes;
constexpr int kThreads = 640;
constexpr int kComputeWarps = 16;
constexpr int kTBufs = 3;                            // TMEM partial buffers (MMA runs 2 groups ahead)
constexpr int kTmemCols = 512;
constexpr int kAColBase = 0;                         // TMEM columns [0, 128): A stages
constexpr int kAccColBase = 128;                     // TMEM columns [128, 512): partials
constexpr uint32_t kWaitLimit = 1u << 20;            // polls before a wait gives up (bounded wait)
constexpr uint32_t kSleepHintNs = 2000;              // longest sleep of one poll

// Every mbarrier operation costs a few hundred cycles inside this kernel, so each group
// has exactly three, all on rings indexed by slot i % kSlots:
//   in_full[q]   both TMA copies of group i (packed weights and activations) complete
//                here: the compute warps' one wait for their inputs
//   op_full[q]   the MMA issuer's one wait: one arrival per compute warp once its part of
//                A is in TMEM.  Partial buffer i % kTBufs is free by then (the same warps
//                folded group i - 3 out of it one step earlier).  The weight producer
//                also waits here before reusing raw slot i % kRawStages (group i - 8).
//   mma_done[q]  the issuer's one commit: the compute warps wait for group i - 2 (partial
//                ready, A stage i % 2 free), the activation producer for group i - 4
// A waiter's parity is (j / kSlots) & 1 for the group j it needs.  No waiter can fall
// kSlots or more completions behind: every later phase of its slot needs work that the
// waiter itself has not released yet, so parities never alias.
constexpr int kSlots = 8;
static_assert(kSlots == kRawStages && kXStages == 4 && kAStages == 2 && kTBufs == 3, "pipeline depths");

struct __align__(8) Barriers {
    uint64_t in_full[kSlots];
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
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag,
                                          bool sleep = true) {
    if (mbar_try_wait(b, parity)) return true;  // already complete: no suspend
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
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
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *b, uint32_t parity, volatile int *abort_flag) {
    const bool ok = mbar_wait(b, parity, abort_flag);
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

struct TcParams {
    const float *S;     // scales [N, G]
    __nv_bfloat16 *Y;   // [M, N]
    float *ws;          // split-K partials [splits, M, N]
    int *err;           // device error word
    int M, N, K, G;
    int Nm;             // activation rows per CTA (multiple of 16, <= 128)
    int splits, gps;    // number of K splits, groups per split
    uint32_t idesc;
    int grouped;
    int scale_tma;      // group scales arrive by TMA (G % 4 == 0, group offsets 16-byte aligned)
};

__global__ void __launch_bounds__(kThreads, 1) w4_gemm_tc(const __grid_constant__ CUtensorMap wmap,
                                                         const __grid_constant__ CUtensorMap xmap,
                                                         const __grid_constant__ CUtensorMap smap,
                                                         const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    Barriers *bar = reinterpret_cast<Barriers *>(smem + kSmemBar);
    volatile int *abort_flag = &bar->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_n = blockIdx.x, tile_m = blockIdx.y, split = blockIdx.z;
    const int row0 = tile_n * kTileRows, m0 = tile_m * kMaxNm;
    const int g0 = split * p.gps, g1 = min(p.G, g0 + p.gps);
    const int ng = g1 - g0;
    const int nchunks = p.scale_tma ? (ng + kScaleChunk - 1) / kScaleChunk : 0;

    if (threadIdx.x == 0) {
        // consumer-side barriers take one arrival per warp (lane 0 after __syncwarp)
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&bar->in_full[i], 2);  // the two producers' arrive.expect_tx
            mbar_init(&bar->op_full[i], kComputeWarps);
            mbar_init(&bar->mma_done[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar->s_full[i], 1);
            mbar_init(&bar->s_empty[i], kComputeWarps);
        }
        mbar_init(&bar->drain, 1);
        bar->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) tmem_alloc(&bar->tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bar->tmem_base;

    float2 acc[16];  // one 32-column chunk as fp32 pairs: one packed multiply and add per pair
    const int x_bytes = 2 * p.Nm * 128;

    if (warp == 0) {
        // ---- packed weights: TMA into the raw ring ----
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
            int issued = 0;
            for (int i = 0; i < ng; ++i) {
                const int s = i % kRawStages;
                // raw slot s held group i - kRawStages, read by every compute warp before it
                // arrived on that group's op_full
                if (i >= kRawStages && !mbar_wait(&bar->op_full[(i - kRawStages) % kSlots],
                                                  (uint32_t)((i - kRawStages) / kSlots) & 1u, abort_flag))
                    break;
                mbar_expect_tx(&bar->in_full[i % kSlots], kRawBytes);
                tma_load_2d(smem + kSmemRaw + (size_t)s * kRawBytes, &wmap, &bar->in_full[i % kSlots], (g0 + i) * 64,
                            row0);
                ++issued;
            }
            // drain: every issued copy has landed before the CTA may exit (after an abort a
            // phase may lack the other producer's arrival: the bounded drain then just waits
            // out its limit, far longer than any copy takes)
            for (int i = issued > kSlots ? issued - kSlots : 0; i < issued; ++i)
                mbar_drain(&bar->in_full[i % kSlots], (uint32_t)(i / kSlots) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- activations: TMA (SWIZZLE_128B) into the X ring ----
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
            int issued = 0;
            for (int i = 0; i < ng; ++i) {
                const int s = i % kXStages;
                // X stage s is free once the MMAs of group i - kXStages have completed
                if (i >= kXStages && !mbar_wait(&bar->mma_done[(i - kXStages) % kSlots],
                                                (uint32_t)((i - kXStages) / kSlots) & 1u, abort_flag))
                    break;
                uint64_t *full = &bar->in_full[i % kSlots];
                mbar_expect_tx(full, (uint32_t)x_bytes);
                uint8_t *dst = smem + kSmemX + (size_t)s * kXBytes;
                tma_load_2d(dst, &xmap, full, (g0 + i) * 128, m0);
                tma_load_2d(dst + (size_t)p.Nm * 128, &xmap, full, (g0 + i) * 128 + 64, m0);
                ++issued;
            }
            for (int i = issued > kXStages ? issued - kXStages : 0; i < issued; ++i)
                mbar_drain(&bar->in_full[i % kSlots], (uint32_t)(i / kSlots) & 1u);
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---- MMA issuer ----
        if (lane == 0) {
            for (int i = 0; i < ng; ++i) {
                const int q = i % kSlots, sa = i % kAStages, sx = i % kXStages, b = i % kTBufs;
                if (!mbar_wait(&bar->op_full[q], (uint32_t)(i / kSlots) & 1u, abort_flag, false)) break;
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
    } else if (warp == 3) {
        // ---- group scales: TMA, [128 rows x 16 groups] tiles into a two-slot ring.  A slot
        // is refilled once every compute warp has finished the tile's last group. ----
        if (lane == 0 && nchunks > 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&smap) : "memory");
            int issued = 0;
            for (int c = 0; c < nchunks; ++c) {
                const int slot = c & 1;
                if (c >= 2 && !mbar_wait(&bar->s_empty[slot], (uint32_t)((c - 2) >> 1) & 1u, abort_flag)) break;
                mbar_expect_tx(&bar->s_full[slot], kScaleBytes);
                tma_load_2d(smem + kSmemScale + (size_t)slot * kScaleBytes, &smap, &bar->s_full[slot],
                            g0 + kScaleChunk * c, row0);
                ++issued;
            }
            for (int c = issued > 2 ? issued - 2 : 0; c < issued; ++c)
                mbar_drain(&bar->s_full[c & 1], (uint32_t)(c >> 1) & 1u);
        }
        __syncwarp();
    } else {
        // ---- compute warps ----
        const int quad = warp & 3;
        const int part = (warp - 4) >> 2;  // k quarter of the dequant, activation-row chunk of the fold
        const int rloc = 32 * quad + lane;  // this thread's weight row in the tile = TMEM lane
        const int row = row0 + rloc;
        const bool row_ok = row < p.N;
        const uint32_t lane_addr = (uint32_t)(32 * quad) << 16;
        const float *srow = p.S + (size_t)(row_ok ? row : 0) * p.G + g0;
        const float *sring = reinterpret_cast<const float *>(smem + kSmemScale);
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = make_float2(0.f, 0.f);
        // per-row scales (no group scales) or the fallback path: one group ahead by __ldg
        float sc_next = (p.grouped && !p.scale_tma) ? __ldg(srow) : 1.0f;
        float4 sc4 = make_float4(1.f, 1.f, 1.f, 1.f);  // four groups' scales of this row

        for (int i = 0; i < ng + 2; ++i) {
            const int j = i - 2;  // the group folded in this step
            const int c = j / kScaleChunk, ci = j % kScaleChunk;
            // the MMAs of group j have completed: their partial is ready and A stage i % 2 is free
            if (i >= 2 && !mbar_wait_warp(&bar->mma_done[j % kSlots], (uint32_t)(j / kSlots) & 1u, abort_flag)) break;
            tc_fence_after();
            // -- dequantize this warp's quarter of group i into A stage i % 2, then release the
            // group to the MMA issuer before folding: the fold is off the MMA's critical path --
            if (i < ng) {
                const int s = i % kRawStages, sa = i % kAStages;
                if (!mbar_wait_warp(&bar->in_full[i % kSlots], (uint32_t)(i / kSlots) & 1u, abort_flag)) break;
                // raw tile written with SWIZZLE_64B: 16-byte chunk c of row r sits at chunk
                // c ^ ((r >> 1) & 3), so 8 consecutive rows hit 8 distinct bank groups
                const uint8_t *rowp = smem + kSmemRaw + (size_t)s * kRawBytes + rloc * 64;
                const int sw = (rloc >> 1) & 3;
                const uint4 v0 = *reinterpret_cast<const uint4 *>(rowp + ((part ^ sw) << 4));
                uint32_t cols[16];
                const uint32_t words[4] = {v0.x, v0.y, v0.z, v0.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {  // 8 k values per word -> 4 columns
                    const uint4 o = dq_word(words[q]);
                    cols[4 * q + 0] = o.x;
                    cols[4 * q + 1] = o.y;
                    cols[4 * q + 2] = o.z;
                    cols[4 * q + 3] = o.w;
                }
                tmem_st16(tmem + lane_addr + (uint32_t)(kAColBase + sa * 64 + 16 * part), cols);
                tmem_st_wait();
                // partial buffer i % 3 is free: group i - 3 was folded last step
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar->op_full[i % kSlots]);
            }
            // -- fold group j into the accumulators --
            if (i >= 2) {
                float sc = sc_next;
                if (p.scale_tma) {
                    if (ci == 0 && !mbar_wait_warp(&bar->s_full[c & 1], (uint32_t)(c >> 1) & 1u, abort_flag)) break;
                    if ((ci & 3) == 0)
                        sc4 = *reinterpret_cast<const float4 *>(
                            &sring[(size_t)(c & 1) * (kTileRows * kScaleChunk) + rloc * kScaleChunk + ci]);
                    const int k4 = ci & 3;
                    sc = k4 == 0 ? sc4.x : k4 == 1 ? sc4.y : k4 == 2 ? sc4.z : sc4.w;
                } else if (p.grouped && j + 1 < ng) {
                    sc_next = __ldg(srow + j + 1);
                }
                const uint32_t taddr = tmem + lane_addr + (uint32_t)(kAccColBase + (j % kTBufs) * kMaxNm);
                const float2 sc2 = make_float2(sc, sc);
                if (part * 32 < p.Nm) {
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        uint32_t r[16];
                        tmem_ld16(taddr + part * 32 + u * 16, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 8; ++e) {  // acc += rn(p * s), per element as the reference
                            const float2 pv = make_float2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
                            acc[u * 8 + e] = __fadd2_rn(acc[u * 8 + e], p.grouped ? __fmul2_rn(pv, sc2) : pv);
                        }
                    }
                }
                tc_fence_before();  // the loads are complete before the buffer is handed back
                if (p.scale_tma && (ci == kScaleChunk - 1 || j == ng - 1)) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar->s_empty[c & 1]);  // done with scale tile c
                }
            }
        }
        // ---- write out: direct (no split) or fp32 partial for the split-K reduction ----
        if (!*abort_flag && row_ok) {
            const float sr = p.grouped ? 1.0f : __ldg(p.S + row);
            const int mlim = min(p.Nm, p.M - m0);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int ml = part * 32 + j;  // activation row in the tile
                const float a = (j & 1) ? acc[j >> 1].y : acc[j >> 1].x;
                if (ml < mlim) {
                    const int m = m0 + ml;
                    if (p.splits == 1)
                        p.Y[(size_t)m * p.N + row] = f2bf(a * sr);
                    else
                        p.ws[((size_t)split * p.M + m) * p.N + row] = a;
                }
            }
        }
    }

    // ---- teardown ----
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        if (threadIdx.x == 0) atomicExch(p.err, 1);
    }
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Split-K combine: Y[m, n] = rn_bf16((0 + P_0 + P_1 + ... + P_{s-1}) * sr[n]), the partials
// summed in split order (K order), as a separate fully parallel pass (8 outputs per thread).
// sr is the per-row scale of the ungrouped format (nullptr: grouped, already applied).
__global__ void __launch_bounds__(256) splitk_combine(const float *__restrict__ ws, int splits, int M, int N,
                                                      const float *__restrict__ sr, __nv_bfloat16 *__restrict__ Y) {
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
}  // namespace

namespace pilm {

int linear_w4_tc(const __nv_bfloat16 *X, int M, int K, const uint8_t *W, const float *S, int N, __nv_bfloat16 *Y,
                 bool grouped, const char *what) {
    static const bool disabled = getenv("PILM_DISABLE_TC") && getenv("PILM_DISABLE_TC")[0] == '1';
    if (disabled || M <= 16 || (K % 128) != 0 || N < 1) return ECPU_ERR_UNSUPPORTED;
    if ((((uintptr_t)X) & 15) || (((uintptr_t)W) & 15)) return ECPU_ERR_UNSUPPORTED;
    TensorMapEncodeTiledFn enc = tensor_map_encoder();
    int *err = device_error_word();
    if (!enc || !err) return ECPU_ERR_UNSUPPORTED;

    const int G = K / 128;
    const int tiles_m = (M + kMaxNm - 1) / kMaxNm;
    const int rows_last = M - (tiles_m - 1) * kMaxNm;
    // activation rows per CTA: all tiles use the same N (multiple of 16)
    int Nm = tiles_m == 1 ? ((M + 15) / 16) * 16 : kMaxNm;
    (void)rows_last;
    const int tiles_n = (N + kTileRows - 1) / kTileRows;

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

    // Split K by a cost model in units of one group's pipeline time: every wave of CTAs pays
    // its groups per CTA plus a fixed prologue and pipeline fill (about 2 groups), and a
    // split adds one combine pass (about 3).  Group scales by TMA need every split's first
    // group (the scale tile's x coordinate) at a multiple of 4; the combine pass wants
    // N % 8 == 0 and 16-byte aligned output rows.
    const bool scale_tma = grouped && (G % 4) == 0 && ((uintptr_t)S & 15) == 0;
    const int base = tiles_n * tiles_m;
    const int sms = num_sms();
    int splits = 1, gps = G;
    {
        double best = 1e30;
        const bool can_split = (N % 8) == 0 && (((uintptr_t)Y) & 15) == 0;
        const int max_splits = can_split ? (G < 16 ? G : 16) : 1;
        for (int s = 1; s <= max_splits; ++s) {
            int g = (G + s - 1) / s;
            if (scale_tma) g = (g + 3) & ~3;
            const int se = (G + g - 1) / g;
            if (se != s) continue;
            const int waves = (base * se + sms - 1) / sms;
            const double est = waves * (g + 2.0) + (se > 1 ? 3.0 : 0.0);
            if (est < best - 1e-9) {
                best = est;
                splits = se;
                gps = g;
            }
        }
    }

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
    p.ws = nullptr;
    p.err = err;
    p.M = M;
    p.N = N;
    p.K = K;
    p.G = G;
    p.Nm = Nm;
    p.splits = splits;
    p.gps = gps;
    p.grouped = grouped ? 1 : 0;
    p.scale_tma = smap_ok ? 1 : 0;
    // kind::f16 instruction descriptor: D fp32, A/B bf16, K-major both, N = Nm, M = 128
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(Nm >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    if (splits > 1) {
        p.ws = (float *)workspace((size_t)splits * M * N * sizeof(float));
        PILM_REQUIRE(p.ws, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
    }
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(w4_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        attr_set = true;
    }
    dim3 grid(tiles_n, tiles_m, splits);
    w4_gemm_tc<<<grid, kThreads, kSmemTotal, stream()>>>(wmap, xmap, smap, p);
    int rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    if (splits > 1) {
        const size_t total8 = (size_t)M * N / 8;
        splitk_combine<<<(unsigned)((total8 + 255) / 256), 256, 0, stream()>>>(p.ws, splits, M, N,
                                                                            grouped ? nullptr : S, Y);
        rc = check_launch(what);
        if (rc != ECPU_OK) return rc;
    }
    return check_error_word(what, "tensor-core GEMM pipeline timed out");
}

}  // namespace pilm
