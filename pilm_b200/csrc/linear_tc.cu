// W4A16 group-128 GEMM for M >= 64 on 5th-generation tensor cores (tcgen05 + TMEM).
//
// Reference semantics (src/ecpu/src/kernel/kernels.c:1089-1139):
//     C[m,n] = rne_bf16( sum_g s[n,g] * sum_{k in g} A[m,k] * q[n,k] )
// computed here with the same structure: every 128-wide quant group g is one exact
// group dot product on the tensor cores (int4 values are exact in bf16, products are
// exact in fp32), and the epilogue adds dot_g * s[n,g] into an fp32 accumulator with
// the product rounded before the add, as the reference does.
//
// CTA tile: 128 weight rows (the MMA M dimension, TMEM lanes) x up to 128 activation
// rows (the MMA N dimension, TMEM columns), over a range of quant groups (split-K).
// Warp roles (352 threads):
//   warp 0      TMA: packed weight tile [128 rows x 64 B] per group -> raw ring (4 deep)
//   warp 1      TMA: activation tile [Nm rows x 128 k] (two SWIZZLE_128B boxes) -> X ring
//               (4 deep: every CTA reads the same activation lines from L2, so this
//               load has the longest latency of the pipeline)
//   warp 2      TMEM owner + MMA issuer: 8 x tcgen05.mma (M=128, N=Nm, K=16) per group
//               into one of two TMEM partial buffers, then tcgen05.commit to the
//               barriers that free the A/X stages and publish the partial
//   warps 3-6   dequant: raw int4 -> bf16 A tile in the K-major SWIZZLE_128B layout
//   warps 7-10  epilogue: tcgen05.ld of the partial, acc = acc + part * s[n,g]
// Every mbarrier wait is bounded: on timeout the CTA records an error, drains, frees
// its TMEM and returns, and the host reports ECPU_ERR_KERNEL.
#include <cuda.h>
#include <mutex>

#include "common.cuh"

using namespace pilm;

namespace {

constexpr int kTileRows = 128;   // weight rows per CTA
constexpr int kMaxNm = 128;      // activation rows per CTA
constexpr int kRawStages = 4;
constexpr int kXStages = 4;
constexpr int kAStages = 2;
constexpr int kRawBytes = kTileRows * 64;            // one group of packed weights
constexpr int kASubBytes = kTileRows * 128;          // 128 rows x 64 k bf16
constexpr int kABytes = 2 * kASubBytes;              // one group (128 k)
constexpr int kXSubBytes = kMaxNm * 128;             // Nm rows x 64 k bf16 (max)
constexpr int kXBytes = 2 * kXSubBytes;
constexpr int kThreads = 352;
constexpr int kTBufs = 4;                            // TMEM partial buffers (MMA runs 3 groups ahead)
constexpr int kTmemCols = 512;                       // kTBufs x 128 columns
constexpr uint32_t kWaitLimit = 1u << 22;            // bounded wait (try_wait re-checks on completion)

struct __align__(8) Barriers {
    uint64_t raw_full[kRawStages], raw_empty[kRawStages];
    uint64_t x_full[kXStages], x_empty[kXStages];
    uint64_t a_full[kAStages], a_empty[kAStages];
    uint64_t t_full[kTBufs], t_empty[kTBufs];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
};

constexpr size_t kSmemRaw = 0;
constexpr size_t kSmemX = kSmemRaw + (size_t)kRawStages * kRawBytes;   // 32 KB, 1024-aligned
constexpr size_t kSmemA = kSmemX + (size_t)kXStages * kXBytes;         // +128 KB
constexpr size_t kSmemBar = kSmemA + (size_t)kAStages * kABytes;       // +64 KB
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
// Bounded wait: returns false (and raises the CTA abort flag) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag) {
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(b, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
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

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
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
    int *ctr;           // arrival counters per (tile_n, tile_m)
    int *err;           // device error word
    int M, N, K, G;
    int Nm;             // activation rows per CTA (multiple of 16, <= 128)
    int splits, gps;    // number of K splits, groups per split
    uint32_t idesc;
    int grouped;
};

__global__ void __launch_bounds__(kThreads, 1) w4_gemm_tc(const __grid_constant__ CUtensorMap wmap,
                                                         const __grid_constant__ CUtensorMap xmap,
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

    if (threadIdx.x == 0) {
        // consumer-side barriers take one arrival per warp (lane 0 after __syncwarp)
        for (int i = 0; i < kRawStages; ++i) {
            mbar_init(&bar->raw_full[i], 1);
            mbar_init(&bar->raw_empty[i], 4);
        }
        for (int i = 0; i < kXStages; ++i) {
            mbar_init(&bar->x_full[i], 1);
            mbar_init(&bar->x_empty[i], 1);
        }
        for (int i = 0; i < kAStages; ++i) {
            mbar_init(&bar->a_full[i], 4);
            mbar_init(&bar->a_empty[i], 1);
        }
        for (int i = 0; i < kTBufs; ++i) {
            mbar_init(&bar->t_full[i], 1);
            mbar_init(&bar->t_empty[i], 4);
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

    float acc[kMaxNm];
    const int x_bytes = 2 * p.Nm * 128;

    if (warp == 0) {
        // ---- packed weights: TMA into the raw ring ----
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
            int issued = 0;
            for (int i = 0; i < ng; ++i) {
                const int s = i % kRawStages;
                const uint32_t ph = (uint32_t)(i / kRawStages) & 1u;
                if (i >= kRawStages && !mbar_wait(&bar->raw_empty[s], ph ^ 1u, abort_flag)) break;
                mbar_expect_tx(&bar->raw_full[s], kRawBytes);
                tma_load_2d(smem + kSmemRaw + (size_t)s * kRawBytes, &wmap, &bar->raw_full[s], (g0 + i) * 64, row0);
                ++issued;
            }
            // drain: every issued copy has landed before the CTA may exit
            for (int i = issued > kRawStages ? issued - kRawStages : 0; i < issued; ++i)
                mbar_wait(&bar->raw_full[i % kRawStages], (uint32_t)(i / kRawStages) & 1u, abort_flag);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- activations: TMA (SWIZZLE_128B) into the X ring ----
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
            int issued = 0;
            for (int i = 0; i < ng; ++i) {
                const int s = i % kXStages;
                const uint32_t ph = (uint32_t)(i / kXStages) & 1u;
                if (i >= kXStages && !mbar_wait(&bar->x_empty[s], ph ^ 1u, abort_flag)) break;
                mbar_expect_tx(&bar->x_full[s], (uint32_t)x_bytes);
                uint8_t *dst = smem + kSmemX + (size_t)s * kXBytes;
                tma_load_2d(dst, &xmap, &bar->x_full[s], (g0 + i) * 128, m0);
                tma_load_2d(dst + (size_t)p.Nm * 128, &xmap, &bar->x_full[s], (g0 + i) * 128 + 64, m0);
                ++issued;
            }
            for (int i = issued > kXStages ? issued - kXStages : 0; i < issued; ++i)
                mbar_wait(&bar->x_full[i % kXStages], (uint32_t)(i / kXStages) & 1u, abort_flag);
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---- MMA issuer ----
        if (lane == 0) {
            for (int i = 0; i < ng; ++i) {
                const int sa = i % kAStages, sx = i % kXStages, b = i % kTBufs;
                if (!mbar_wait(&bar->a_full[sa], (uint32_t)(i / kAStages) & 1u, abort_flag)) break;
                if (!mbar_wait(&bar->x_full[sx], (uint32_t)(i / kXStages) & 1u, abort_flag)) break;
                if (i >= kTBufs && !mbar_wait(&bar->t_empty[b], ((uint32_t)(i / kTBufs) & 1u) ^ 1u, abort_flag))
                    break;
                tc_fence_after();
                const uint32_t a_base = smem_u32(smem + kSmemA + (size_t)sa * kABytes);
                const uint32_t x_base = smem_u32(smem + kSmemX + (size_t)sx * kXBytes);
                const uint32_t d = tmem + (uint32_t)(b * kMaxNm);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint64_t ad = sw128_desc(a_base + h * kASubBytes);
                    const uint64_t bd = sw128_desc(x_base + h * p.Nm * 128);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_bf16(d, ad + 2 * k, bd + 2 * k, p.idesc, (h | k) ? 1u : 0u);
                }
                umma_commit(&bar->a_empty[sa]);
                umma_commit(&bar->x_empty[sx]);
                umma_commit(&bar->t_full[b]);
            }
            // drain: all issued MMAs have completed before TMEM is released
            umma_commit(&bar->drain);
            mbar_wait(&bar->drain, 0, abort_flag);
        }
        __syncwarp();
    } else if (warp >= 3 && warp <= 6) {
        // ---- dequant: raw [128 rows x 64 B] -> A [2 x (128 rows x 128 B)] SWIZZLE_128B ----
        const int wq = warp - 3;           // rows 32*wq .. 32*wq+31
        const int c = lane & 3;            // 16-byte chunk of the 64-byte row (k = 32c..32c+31)
        const int rsub = lane >> 2;        // row within an 8-row slab
        for (int i = 0; i < ng; ++i) {
            const int s = i % kRawStages, sa = i % kAStages;
            if (!mbar_wait(&bar->raw_full[s], (uint32_t)(i / kRawStages) & 1u, abort_flag)) break;
            if (i >= kAStages && !mbar_wait(&bar->a_empty[sa], ((uint32_t)(i / kAStages) & 1u) ^ 1u, abort_flag))
                break;
            const uint8_t *raw = smem + kSmemRaw + (size_t)s * kRawBytes;
            uint8_t *a = smem + kSmemA + (size_t)sa * kABytes + (c >> 1) * kASubBytes;
            uint4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = 32 * wq + 8 * j + rsub;
                v[j] = *reinterpret_cast<const uint4 *>(raw + r * 64 + c * 16);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->raw_empty[s]);  // raw slot consumed (values in registers)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = 32 * wq + 8 * j + rsub;
                uint8_t *rowp = a + r * 128;
                const uint32_t words[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int chunk = ((c & 1) * 4 + q) ^ (r & 7);  // 8 bf16 (k = 32c + 8q ..) per chunk
                    *reinterpret_cast<uint4 *>(rowp + chunk * 16) = dq_word(words[q]);
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->a_full[sa]);
        }
    } else {
        // ---- epilogue: warps 7..10 own TMEM lanes 32*(warp%4) .. +31 ----
        const int quad = warp & 3;
        const int row = row0 + 32 * quad + lane;
        const bool row_ok = row < p.N;
#pragma unroll
        for (int j = 0; j < kMaxNm; ++j) acc[j] = 0.f;
        // group scales are prefetched one group ahead (they are the only DRAM reads here)
        const float *srow = p.S + (size_t)(row_ok ? row : 0) * p.G + g0;
        float sc_next = (row_ok && p.grouped) ? __ldg(srow) : 1.0f;
        for (int i = 0; i < ng; ++i) {
            const int b = i % kTBufs;
            const float sc = sc_next;
            if (p.grouped && row_ok && i + 1 < ng) sc_next = __ldg(srow + i + 1);
            if (!mbar_wait(&bar->t_full[b], (uint32_t)(i / kTBufs) & 1u, abort_flag)) break;
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)(b * kMaxNm);
#pragma unroll
            for (int cb = 0; cb < kMaxNm / 32; ++cb) {
                if (cb * 32 < p.Nm) {
                    uint32_t r[32];
                    tmem_ld32(taddr + cb * 32, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const float part = __uint_as_float(r[e]);
                        acc[cb * 32 + e] = p.grouped ? __fadd_rn(acc[cb * 32 + e], __fmul_rn(part, sc))
                                                     : __fadd_rn(acc[cb * 32 + e], part);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->t_empty[b]);
        }
        // ---- write out: direct (no split) or fp32 partial for the split-K reduction ----
        if (!*abort_flag && row_ok) {
            const float sr = p.grouped ? 1.0f : __ldg(p.S + row);
            const int mlim = min(p.Nm, p.M - m0);
#pragma unroll
            for (int j = 0; j < kMaxNm; ++j) {
                if (j < mlim) {
                    const int m = m0 + j;
                    if (p.splits == 1)
                        p.Y[(size_t)m * p.N + row] = f2bf(acc[j] * sr);
                    else
                        p.ws[((size_t)split * p.M + m) * p.N + row] = acc[j];
                }
            }
        }
    }

    // ---- teardown ----
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        if (threadIdx.x == 0) atomicExch(p.err, 1);
    } else if (p.splits > 1) {
        // split-K: every CTA has written its fp32 partial; the last CTA to arrive for this
        // tile sums the partials of its cells in split order (deterministic) and rounds.
        __shared__ int s_last;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int prev = atomicAdd(p.ctr + blockIdx.y * gridDim.x + blockIdx.x, 1);
            s_last = (prev == p.splits - 1);
        }
        __syncthreads();
        if (s_last) {
            // all threads: 8 cells per thread per pass, every partial load issued up front
            __threadfence();
            const int mlim = min(p.Nm, p.M - m0);
            const int cells = kTileRows * mlim;
            for (int base = threadIdx.x; base < cells; base += 8 * kThreads) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = 0.f;
                for (int sp = 0; sp < p.splits; ++sp) {
                    float t[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int e = base + u * kThreads;
                        const int r = row0 + (e % kTileRows), m = m0 + e / kTileRows;
                        t[u] = (e < cells && r < p.N) ? __ldcg(p.ws + ((size_t)sp * p.M + m) * p.N + r) : 0.f;
                    }
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] += t[u];
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int e = base + u * kThreads;
                    const int r = row0 + (e % kTileRows), m = m0 + e / kTileRows;
                    if (e < cells && r < p.N) p.Y[(size_t)m * p.N + r] = f2bf(p.grouped ? v[u] : v[u] * __ldg(p.S + r));
                }
            }
        }
        if (s_last && threadIdx.x == 0) p.ctr[blockIdx.y * gridDim.x + blockIdx.x] = 0;
    }
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---- host side ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

int *device_error_word() {
    static int *err = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        if (cudaMalloc(&err, sizeof(int)) == cudaSuccess) cudaMemset(err, 0, sizeof(int));
    });
    return err;
}

}  // namespace

namespace pilm {

int linear_w4_tc(const __nv_bfloat16 *X, int M, int K, const uint8_t *W, const float *S, int N, __nv_bfloat16 *Y,
                 bool grouped, const char *what) {
    static const bool disabled = getenv("PILM_DISABLE_TC") && getenv("PILM_DISABLE_TC")[0] == '1';
    if (disabled || M < 64 || (K % 128) != 0 || N < 1) return ECPU_ERR_UNSUPPORTED;
    if ((((uintptr_t)X) & 15) || (((uintptr_t)W) & 15)) return ECPU_ERR_UNSUPPORTED;
    EncodeTiledFn enc = encode_fn();
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
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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

    // split K so that the grid covers the SMs once (one CTA per SM: shared memory)
    const int base = tiles_n * tiles_m;
    const int sms = num_sms();
    int splits = 1;
    if (base < sms) {
        splits = sms / base;
        if (splits > G) splits = G;
        if (splits < 1) splits = 1;
    }
    const int gps = (G + splits - 1) / splits;
    splits = (G + gps - 1) / gps;

    TcParams p;
    p.S = S;
    p.Y = Y;
    p.ws = nullptr;
    p.ctr = nullptr;
    p.err = err;
    p.M = M;
    p.N = N;
    p.K = K;
    p.G = G;
    p.Nm = Nm;
    p.splits = splits;
    p.gps = gps;
    p.grouped = grouped ? 1 : 0;
    // kind::f16 instruction descriptor: D fp32, A/B bf16, K-major both, N = Nm, M = 128
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(Nm >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    if (splits > 1) {
        p.ws = (float *)workspace((size_t)splits * M * N * sizeof(float));
        p.ctr = counters((size_t)tiles_n * tiles_m);
        PILM_REQUIRE(p.ws && p.ctr, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
    }
    static bool attr_set = false;
    if (!attr_set) {
        cudaFuncSetAttribute(w4_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemTotal);
        attr_set = true;
    }
    dim3 grid(tiles_n, tiles_m, splits);
    w4_gemm_tc<<<grid, kThreads, kSmemTotal, stream()>>>(wmap, xmap, p);
    int rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    if (sync_mode()) {
        int h = 0;
        cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
        if (h) {
            cudaMemset(err, 0, sizeof(int));
            set_error("%s: tensor-core GEMM pipeline timed out", what);
            return ECPU_ERR_KERNEL;
        }
    }
    return ECPU_OK;
}

}  // namespace pilm
