// Quantized linears: W4A16 (group-128, group-32, per-row), W8A16, W8A32, F32 GEMM.
//
// Reference semantics (src/ecpu/src/kernel/kernels.c):
//   W4 g128 / g32 (linear_w4a16g_bf16_impl, :1089-1139):
//       C[m,n] = rne_bf16( sum_g s[n,g] * sum_{k in g} bf16(A[m,k]) * q[n,k] )
//   W4 per-row (:1002-1087), W8A16 (:469-656):  C = rne_bf16( s[n] * sum_k A q )
//   W8A32 (:437-467):                            C = s[n] * sum_k A q     (fp32)
// q is the signed int4 nibble (even k in the low nibble, :43-46) or int8.
//
// Small M (M <= 16; larger M goes to the tensor-core GEMM) is HBM-bound: the packed
// weights are streamed once with 128-bit loads and dequantised in registers straight
// into tensor-core A fragments (mma.sync m16n8k16, bf16 x bf16 -> fp32); the
// activations form the B fragments.  The k order inside each 128-wide group is
// permuted so that every thread's 16-byte weight load holds exactly the values its
// fragments need (see w4_gemv_mma); the activations are permuted identically, so
// each group's fp32 partial is the exact group dot of the reference, which is then
// scaled by s[n,g] in fp32 like the reference.  Split-K partials are reduced in a
// fixed order by the last-arriving CTA (deterministic, no spin-waits).
#include "common.cuh"

using namespace pilm;

namespace {

constexpr int kGemvWarps = 8;

// (nibble ^ 8) | 0x4300 in both 16-bit halves: the bf16 value 136 + q, exact.
__device__ __forceinline__ uint32_t nib_magic(uint32_t w) {
    uint32_t t;
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(t) : "r"(w), "r"(0x000F000Fu), "r"(0x43084308u));
    return t;
}

// Two int4 nibbles at bits [0,4) and [16,20) -> bf16x2 (q_lo, q_hi), exact.
__device__ __forceinline__ uint32_t dq_pair(uint32_t w) {
    uint32_t t = nib_magic(w);
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&t);
    const __nv_bfloat162 bias = __floats2bfloat162_rn(136.0f, 136.0f);
    v = __hsub2(v, bias);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// One group of one 16-row tile against one 8-row activation tile (w4_gemv_mma with RT = NT
// = 1): the weight words w0 (rows r) and w1 (rows r + 8) and the four activation words of
// the thread, into the fp32 group partial d, exactly as the general loop in w4_gemv_mma.
template <bool KP>
__device__ __forceinline__ void gemv_group_dot(uint4 w0, uint4 w1, uint4 x0, uint4 x1, uint4 x2, uint4 x3,
                                               float (&d)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 xw = i == 0 ? x0 : (i == 1 ? x1 : (i == 2 ? x2 : x3));
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            uint32_t b0, b1;
            if (KP) {  // nibble pairs (2hh, 2hh+4) and (2hh+1, 2hh+5) are k (4hh, 4hh+1), (4hh+2, 4hh+3)
                b0 = hh ? xw.z : xw.x;
                b1 = hh ? xw.w : xw.y;
            } else {
                const uint32_t lo = hh ? xw.y : xw.x;
                const uint32_t hi = hh ? xw.w : xw.z;
                b0 = __byte_perm(lo, hi, 0x5410);
                b1 = __byte_perm(lo, hi, 0x7632);
            }
            const uint32_t wr = word_of(w0, i), wr8 = word_of(w1, i);
            mma16816(d, dq_pair(wr >> (8 * hh)), dq_pair(wr8 >> (8 * hh)), dq_pair(wr >> (8 * hh + 4)),
                     dq_pair(wr8 >> (8 * hh + 4)), b0, b1);
        }
    }
}

// Register-dequant W4 GEMV on tensor cores.
//
// Tile: a warp owns RT row tiles of 16 output rows and NT batch tiles of 8 rows of A.
// Lane t = 4r + c.  For a 128-wide group g, thread c loads bytes [16c, 16c+16) of the
// group (k in [32c, 32c+32)) for its weight rows r and r+8 of every row tile: four
// 32-bit words, word i holding k = 32c + 8i + j at nibble j.  MMA step (i, h) uses
// nibble pairs (2h, 2h+4) as A slots {2c, 2c+1} and (2h+1, 2h+5) as slots {2c+8, 2c+9};
// the B fragment of the same thread carries A[m, k] for exactly those k (gathered
// with byte permutes from one 16-byte load), so every MMA slot pairs W[n,k] with
// A[m,k] for the same k and the 8 steps of a group sum the whole group.
template <int RT, int NT, bool GROUPED, bool KP, bool PF>
__global__ void __launch_bounds__(kGemvWarps * 32) w4_gemv_mma(
    const __nv_bfloat16 *__restrict__ X, int M, int K, const uint8_t *__restrict__ W,
    const float *__restrict__ S, int N, __nv_bfloat16 *__restrict__ Y, float *__restrict__ ws,
    int *__restrict__ ctr, int splits, int groups_per_split) {
    // PF: weights are never written by another kernel, so this CTA's weight slab is
    // prefetched into L2 before the wait for the previous kernel, and the fetch overlaps
    // that kernel's tail.  In the model's layer chain (a norm, SwiGLU or attention kernel
    // before each linear) that took 3% off a config 2 step (M = 4).  It is used for grids
    // of one wave at M <= 8 only: CTAs of later waves start after the previous kernel has
    // ended, and at M = 16 or for back-to-back launches of large shapes the variant
    // measured up to 24% slower alone.
    if (PF) pdl_trigger();
    else pdl_entry();
    constexpr int ROWS = 16 * RT;
    constexpr int NACC = RT * NT * 4;
    __shared__ float red[kGemvWarps][NACC][32];
    __shared__ int s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, c = lane & 3;
    const int row_base = blockIdx.x * ROWS;
    const int G = K >> 7;
    const int g0 = blockIdx.y * groups_per_split;
    const int g1 = min(G, g0 + groups_per_split);
    const size_t ldw = (size_t)K >> 1;

    const uint8_t *wp[RT][2];
    bool rv[RT][2];
    int rows[RT][2];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int row = row_base + rt * 16 + h * 8 + r;
            rows[rt][h] = row;
            rv[rt][h] = row < N;
            wp[rt][h] = W + (size_t)(row < N ? row : 0) * ldw + c * 16;
        }
    const __nv_bfloat16 *xp[NT];
    bool xv[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        int m = nt * 8 + r;
        xv[nt] = m < M;
        xp[nt] = X + (size_t)(m < M ? m : 0) * K + c * 32;
    }

    float acc[RT][NT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[rt][nt][j] = 0.f;

    // the slab: rows [row_base, row_base + ROWS), bytes [64 g0, 64 g1) of each (one row per
    // lane of the last warp; every address and size is a multiple of 64 bytes).  Loading
    // each warp's next group a loop iteration ahead as well was slower (more registers).
    if (PF && warp == kGemvWarps - 1 && lane < ROWS && row_base + lane < N)
        prefetch_l2_bulk(W + (size_t)(row_base + lane) * ldw + (size_t)g0 * 64, (uint32_t)(g1 - g0) * 64u);
    if (PF) pdl_wait();

    if constexpr (RT == 1 && NT == 1) {
        // One 16-row tile and one activation tile (the small projections at M <= 8): the
        // next group's weights, scales and activations are loaded before this group's math,
        // so a warp's groups wait on memory once, not once each.
        uint4 w0 = make_uint4(0, 0, 0, 0), w1 = w0, x0 = w0, x1 = w0, x2 = w0, x3 = w0;
        float s0 = 0.f, s1 = 0.f;
        int g = g0 + warp;
        if (g < g1) {
            if (rv[0][0]) w0 = ldg_nc_v4(wp[0][0] + (size_t)g * 64);
            if (rv[0][1]) w1 = ldg_nc_v4(wp[0][1] + (size_t)g * 64);
            if (GROUPED && rv[0][0]) s0 = __ldg(S + (size_t)rows[0][0] * G + g);
            if (GROUPED && rv[0][1]) s1 = __ldg(S + (size_t)rows[0][1] * G + g);
            if (xv[0]) {
                x0 = ldg_v4(xp[0] + (size_t)g * 128);
                x1 = ldg_v4(xp[0] + (size_t)g * 128 + 8);
                x2 = ldg_v4(xp[0] + (size_t)g * 128 + 16);
                x3 = ldg_v4(xp[0] + (size_t)g * 128 + 24);
            }
        }
        for (; g < g1; g += kGemvWarps) {
            const int gn = g + kGemvWarps;
            uint4 nw0 = make_uint4(0, 0, 0, 0), nw1 = nw0, nx0 = nw0, nx1 = nw0, nx2 = nw0, nx3 = nw0;
            float ns0 = 0.f, ns1 = 0.f;
            if (gn < g1) {
                if (rv[0][0]) nw0 = ldg_nc_v4(wp[0][0] + (size_t)gn * 64);
                if (rv[0][1]) nw1 = ldg_nc_v4(wp[0][1] + (size_t)gn * 64);
                if (GROUPED && rv[0][0]) ns0 = __ldg(S + (size_t)rows[0][0] * G + gn);
                if (GROUPED && rv[0][1]) ns1 = __ldg(S + (size_t)rows[0][1] * G + gn);
                if (xv[0]) {
                    nx0 = ldg_v4(xp[0] + (size_t)gn * 128);
                    nx1 = ldg_v4(xp[0] + (size_t)gn * 128 + 8);
                    nx2 = ldg_v4(xp[0] + (size_t)gn * 128 + 16);
                    nx3 = ldg_v4(xp[0] + (size_t)gn * 128 + 24);
                }
            }
            float part[4] = {0.f, 0.f, 0.f, 0.f};
            gemv_group_dot<KP>(w0, w1, x0, x1, x2, x3, part);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (GROUPED)  // reference: acc = acc + dot_g * s[n,g], product rounded first
                    acc[0][0][j] = __fadd_rn(acc[0][0][j], __fmul_rn(part[j], (j >> 1) ? s1 : s0));
                else
                    acc[0][0][j] = __fadd_rn(acc[0][0][j], part[j]);
            }
            w0 = nw0, w1 = nw1, x0 = nx0, x1 = nx1, x2 = nx2, x3 = nx3, s0 = ns0, s1 = ns1;
        }
    } else {
    for (int g = g0 + warp; g < g1; g += kGemvWarps) {
        uint4 wq[RT][2];
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                wq[rt][h] = rv[rt][h] ? ldg_nc_v4(wp[rt][h] + (size_t)g * 64) : make_uint4(0, 0, 0, 0);
        float sc[RT][2];
        if (GROUPED) {
#pragma unroll
            for (int rt = 0; rt < RT; ++rt)
#pragma unroll
                for (int h = 0; h < 2; ++h) sc[rt][h] = rv[rt][h] ? __ldg(S + (size_t)rows[rt][h] * G + g) : 0.f;
        }
        float part[RT][NT][4];
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) part[rt][nt][j] = 0.f;

#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint4 xw[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                xw[nt] = xv[nt] ? ldg_v4(xp[nt] + (size_t)g * 128 + i * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t b0[NT], b1[NT];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if (KP) {  // nibble pairs (2hh, 2hh+4) and (2hh+1, 2hh+5) are k (4hh, 4hh+1), (4hh+2, 4hh+3)
                        b0[nt] = hh ? xw[nt].z : xw[nt].x;
                        b1[nt] = hh ? xw[nt].w : xw[nt].y;
                    } else {
                        uint32_t lo = hh ? xw[nt].y : xw[nt].x;
                        uint32_t hi = hh ? xw[nt].w : xw[nt].z;
                        b0[nt] = __byte_perm(lo, hi, 0x5410);
                        b1[nt] = __byte_perm(lo, hi, 0x7632);
                    }
                }
#pragma unroll
                for (int rt = 0; rt < RT; ++rt) {
                    uint32_t wr = word_of(wq[rt][0], i), wr8 = word_of(wq[rt][1], i);
                    uint32_t a0 = dq_pair(wr >> (8 * hh));
                    uint32_t a1 = dq_pair(wr8 >> (8 * hh));
                    uint32_t a2 = dq_pair(wr >> (8 * hh + 4));
                    uint32_t a3 = dq_pair(wr8 >> (8 * hh + 4));
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) mma16816(part[rt][nt], a0, a1, a2, a3, b0[nt], b1[nt]);
                }
            }
        }
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (GROUPED)  // reference: acc = acc + dot_g * s[n,g], product rounded first
                        acc[rt][nt][j] = __fadd_rn(acc[rt][nt][j], __fmul_rn(part[rt][nt][j], sc[rt][j >> 1]));
                    else
                        acc[rt][nt][j] = __fadd_rn(acc[rt][nt][j], part[rt][nt][j]);
                }
    }
    }

#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) red[warp][(rt * NT + nt) * 4 + j][lane] = acc[rt][nt][j];
    __syncthreads();

    // Fixed-order reduction over warps; entry e -> (tile slot, lane) -> (row, m).
    for (int e = threadIdx.x; e < NACC * 32; e += blockDim.x) {
        const int idx = e >> 5, ln = e & 31;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) v += red[w][idx][ln];
        const int rt = idx / (NT * 4), nt = (idx / 4) % NT, j = idx & 3;
        const int row = row_base + rt * 16 + (ln >> 2) + ((j & 2) ? 8 : 0);
        const int m = nt * 8 + 2 * (ln & 3) + (j & 1);
        if (row < N && m < M) {
            if (splits == 1) {
                if (!GROUPED) v = v * __ldg(S + row);
                Y[(size_t)m * N + row] = f2bf(v);
            } else {
                ws[((size_t)blockIdx.y * M + m) * N + row] = v;
            }
        }
    }
    if (splits == 1) return;

    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int prev = atomicAdd(ctr + blockIdx.x, 1);
        s_last = (prev == splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int e = threadIdx.x; e < ROWS * M; e += blockDim.x) {
        const int m = e / ROWS, row = row_base + e % ROWS;
        if (row >= N) continue;
        float v = 0.f;
        for (int s = 0; s < splits; ++s) v += __ldcg(ws + ((size_t)s * M + m) * N + row);
        if (!GROUPED) v = v * __ldg(S + row);
        Y[(size_t)m * N + row] = f2bf(v);
    }
    if (threadIdx.x == 0) ctr[blockIdx.x] = 0;  // self-reset for the next launch / graph replay
}

// bf16-weight GEMV on tensor cores: C[m, n] = rne_bf16(sum_k A[m, k] * W[n, k]), fp32
// accumulation (F.linear on bf16 tensors: the reference's default BackendLinear,
// src/models/base/linear.py:170-183, which the MTP draft module uses unless
// PILM_MTP_QUANTIZE=w4a16).
//
// Tile: a warp owns RT row tiles of 16 weight rows and NT tiles of 8 activation rows; the
// CTA's 8 warps split K into 32-wide blocks.  In block b, lane 4r + c loads the 16 bytes
// W[row][32b + 8c .. + 7] (rows r and r + 8 of each row tile) and A[m][32b + 8c .. + 7]:
// words x, y feed MMA step 0 (k slots {2c, 2c+1} and {2c+8, 2c+9}), words z, w step 1, for
// A and B alike, so the loaded words are the fragments with no permutes.  Split-K partials
// are reduced in a fixed order by the last CTA of each row tile, as in w4_gemv_mma.
template <int RT, int NT>
__global__ void __launch_bounds__(kGemvWarps * 32) bf16w_gemv_mma(
    const __nv_bfloat16 *__restrict__ X, int M, int K, const __nv_bfloat16 *__restrict__ W, int N,
    __nv_bfloat16 *__restrict__ Y, float *__restrict__ ws, int *__restrict__ ctr, int splits, int blocks_per_split) {
    pdl_entry();
    constexpr int ROWS = 16 * RT;
    constexpr int NACC = RT * NT * 4;
    __shared__ float red[kGemvWarps][NACC][32];
    __shared__ int s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, c = lane & 3;
    const int row_base = blockIdx.x * ROWS;
    const int nb = (K + 31) >> 5;
    const int b0 = blockIdx.y * blocks_per_split;
    const int b1 = min(nb, b0 + blocks_per_split);

    const __nv_bfloat16 *wp[RT][2];
    bool rv[RT][2];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = row_base + rt * 16 + h * 8 + r;
            rv[rt][h] = row < N;
            wp[rt][h] = W + (size_t)(row < N ? row : 0) * K + c * 8;
        }
    const __nv_bfloat16 *xp[NT];
    bool xv[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + r;
        xv[nt] = m < M;
        xp[nt] = X + (size_t)(m < M ? m : 0) * K + c * 8;
    }

    float acc[RT][NT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[rt][nt][j] = 0.f;

    for (int b = b0 + warp; b < b1; b += kGemvWarps) {
        const int k = b * 32 + c * 8;  // this lane's 8 k values (K % 8 == 0: all or none)
        const bool kin = k < K;
        uint4 wq[RT][2];
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                wq[rt][h] = (rv[rt][h] && kin) ? ldg_nc_v4(wp[rt][h] + (size_t)b * 32) : make_uint4(0, 0, 0, 0);
        uint4 xw[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            xw[nt] = (xv[nt] && kin) ? ldg_v4(xp[nt] + (size_t)b * 32) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int st = 0; st < 2; ++st)
#pragma unroll
            for (int rt = 0; rt < RT; ++rt)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    mma16816(acc[rt][nt], st ? wq[rt][0].z : wq[rt][0].x, st ? wq[rt][1].z : wq[rt][1].x,
                             st ? wq[rt][0].w : wq[rt][0].y, st ? wq[rt][1].w : wq[rt][1].y,
                             st ? xw[nt].z : xw[nt].x, st ? xw[nt].w : xw[nt].y);
    }

#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) red[warp][(rt * NT + nt) * 4 + j][lane] = acc[rt][nt][j];
    __syncthreads();
    for (int e = threadIdx.x; e < NACC * 32; e += blockDim.x) {
        const int idx = e >> 5, ln = e & 31;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) v += red[w][idx][ln];
        const int rt = idx / (NT * 4), nt = (idx / 4) % NT, j = idx & 3;
        const int row = row_base + rt * 16 + (ln >> 2) + ((j & 2) ? 8 : 0);
        const int m = nt * 8 + 2 * (ln & 3) + (j & 1);
        if (row < N && m < M) {
            if (splits == 1)
                Y[(size_t)m * N + row] = f2bf(v);
            else
                ws[((size_t)blockIdx.y * M + m) * N + row] = v;
        }
    }
    if (splits == 1) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(ctr + blockIdx.x, 1);
        s_last = (prev == splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int e = threadIdx.x; e < ROWS * M; e += blockDim.x) {
        const int m = e / ROWS, row = row_base + e % ROWS;
        if (row >= N) continue;
        float v = 0.f;
        for (int sp = 0; sp < splits; ++sp) v += __ldcg(ws + ((size_t)sp * M + m) * N + row);
        Y[(size_t)m * N + row] = f2bf(v);
    }
    if (threadIdx.x == 0) ctr[blockIdx.x] = 0;  // self-reset for the next launch / graph replay
}

template <int RT, int NT>
int launch_bf16w(const __nv_bfloat16 *X, int M, int K, const __nv_bfloat16 *W, int N, __nv_bfloat16 *Y,
                 const char *what) {
    const int tiles = (N + 16 * RT - 1) / (16 * RT);
    const int nb = (K + 31) / 32;
    const int target = 2 * pilm::num_sms();
    int splits = 1;
    if (tiles < target) {
        splits = (target + tiles - 1) / tiles;
        int max_splits = nb / kGemvWarps;  // keep every warp busy
        if (max_splits < 1) max_splits = 1;
        if (splits > max_splits) splits = max_splits;
    }
    const int bps = (nb + splits - 1) / splits;
    splits = (nb + bps - 1) / bps;
    float *ws = nullptr;
    int *ctr = nullptr;
    if (splits > 1) {
        ws = (float *)pilm::workspace((size_t)splits * M * N * sizeof(float));
        ctr = pilm::counters((size_t)tiles);
        PILM_REQUIRE(ws && ctr, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
    }
    launch_pdl(bf16w_gemv_mma<RT, NT>, dim3(dim3(tiles, splits)), dim3(kGemvWarps * 32), 0, X, M, K, W, N, Y, ws, ctr,
                                                                                          splits, bps);
    return pilm::check_launch(what);
}

// Generic fallback (any K, any alignment): one warp per output row; lanes stride
// over k; per scale group the lanes' partial dots are summed, then
// acc = acc + dot_g * s[n,g] (QF 0), or the row dot is scaled once (QF 1: W4 per-row,
// QF 2: W8 per-row).  Activations bf16; output bf16.
template <int QF>
__global__ void __launch_bounds__(256) linear_generic(const __nv_bfloat16 *__restrict__ X, int M, int K,
                                                      const void *__restrict__ Wv, const float *__restrict__ S,
                                                      int N, int gs, __nv_bfloat16 *__restrict__ Y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + warp;
    if (n >= N) return;
    const int G = QF == 0 ? (K + gs - 1) / gs : 1;
    const int glen = QF == 0 ? gs : K;
    const uint8_t *W4 = reinterpret_cast<const uint8_t *>(Wv) + (size_t)n * ((K + 1) / 2);
    const int8_t *W8 = reinterpret_cast<const int8_t *>(Wv) + (size_t)n * K;
    for (int m = 0; m < M; ++m) {
        const __nv_bfloat16 *x = X + (size_t)m * K;
        float acc = 0.f;
        for (int g = 0; g < G; ++g) {
            const int k0 = g * glen, k1 = min(K, k0 + glen);
            float part = 0.f;
            for (int k = k0 + lane; k < k1; k += 32) {
                float q;
                if (QF == 2) {
                    q = (float)W8[k];
                } else {
                    int v = (W4[k >> 1] >> ((k & 1) * 4)) & 0xF;
                    q = (float)(v >= 8 ? v - 16 : v);
                }
                part = fmaf(bf2f(x[k]), q, part);
            }
            part = warp_sum(part);
            if (QF == 0)
                acc = __fadd_rn(acc, __fmul_rn(part, __ldg(S + (size_t)n * G + g)));
            else
                acc += part;
        }
        if (QF != 0) acc = acc * __ldg(S + n);
        if (lane == 0) Y[(size_t)m * N + n] = f2bf(acc);
    }
}

// W8A32: fp32 activations, int8 weights, per-row scale, fp32 out.  A warp owns kW8Rows
// weight rows and streams them once per chunk of MC activation rows: each lane keeps
// kW8Rows x kW8Unroll 16-byte weight loads in flight, and every activation value it
// loads serves all of the warp's rows.  Each lane sums its k positions in increasing
// order (16 per 512-wide step), then the warp sums its lanes.  Ragged K or unaligned
// pointers take the scalar loop.
constexpr int kW8Rows = 4, kW8Unroll = 2;

// Signed byte e of w as an exact fp32: with the sign bit flipped, the byte u = q + 128 is
// placed in the low mantissa bits of 2^23 (exponent byte 0x4B), giving 2^23 + u exactly,
// and subtracting 2^23 + 128 leaves q.  One byte permute and one add instead of an
// integer-to-float conversion.
__device__ __forceinline__ float i8_to_f32(uint32_t w, int e) {
    const uint32_t t = __byte_perm(w ^ 0x80808080u, 0x4B000000u, (uint32_t)e | 0x7440u);
    return __uint_as_float(t) - 8388736.0f;
}

// The row scales are never written by another kernel: they are read before the wait for
// the previous kernel.  (An L2 prefetch of the warp's weight rows there as well made the
// GEMV faster but its neighbours in the config 1 step slower by as much: not kept.)
template <int MC>
__global__ void __launch_bounds__(256) w8a32_gemv(const float *__restrict__ X, int M, int K,
                                                  const int8_t *__restrict__ W, const float *__restrict__ S, int N,
                                                  float *__restrict__ Y) {
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = (blockIdx.x * 8 + warp) * kW8Rows;
    if (n0 >= N) return;
    const bool vec = ((K & 15) == 0) && ((((uintptr_t)W) & 15) == 0) && ((((uintptr_t)X) & 15) == 0);
    const int8_t *w[kW8Rows];
    bool rv[kW8Rows];
    float sc[kW8Rows];
#pragma unroll
    for (int r = 0; r < kW8Rows; ++r) {
        rv[r] = n0 + r < N;
        w[r] = W + (size_t)(rv[r] ? n0 + r : n0) * K;
        sc[r] = rv[r] ? __ldg(S + n0 + r) : 0.f;
    }
    pdl_wait();
    for (int m0 = 0; m0 < M; m0 += MC) {
        const int mc = min(MC, M - m0);
        float acc[MC][kW8Rows];
#pragma unroll
        for (int mm = 0; mm < MC; ++mm)
#pragma unroll
            for (int r = 0; r < kW8Rows; ++r) acc[mm][r] = 0.f;
        if (vec) {
            for (int kb = lane * 16; kb < K; kb += 512 * kW8Unroll) {
                uint4 q[kW8Unroll][kW8Rows];
#pragma unroll
                for (int u = 0; u < kW8Unroll; ++u) {
                    const int k = kb + u * 512;
#pragma unroll
                    for (int r = 0; r < kW8Rows; ++r) q[u][r] = k < K ? ldg_nc_v4(w[r] + k) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < kW8Unroll; ++u) {
                    const int k = kb + u * 512;
                    if (k >= K) continue;
                    float4 xv[MC][4];  // activation rows x 16 k
#pragma unroll
                    for (int mm = 0; mm < MC; ++mm) {
                        const float4 *xr = reinterpret_cast<const float4 *>(X + (size_t)(m0 + (mm < mc ? mm : 0)) * K + k);
#pragma unroll
                        for (int v = 0; v < 4; ++v) xv[mm][v] = mm < mc ? __ldg(xr + v) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int r = 0; r < kW8Rows; ++r) {
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            const uint32_t w4 = word_of(q[u][r], v);
                            float f[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) f[e] = i8_to_f32(w4, e);
#pragma unroll
                            for (int mm = 0; mm < MC; ++mm) {
                                if (mm >= mc) continue;
                                acc[mm][r] = fmaf(xv[mm][v].x, f[0], acc[mm][r]);
                                acc[mm][r] = fmaf(xv[mm][v].y, f[1], acc[mm][r]);
                                acc[mm][r] = fmaf(xv[mm][v].z, f[2], acc[mm][r]);
                                acc[mm][r] = fmaf(xv[mm][v].w, f[3], acc[mm][r]);
                            }
                        }
                    }
                }
            }
        } else {
            for (int k = lane; k < K; k += 32) {
                float qf[kW8Rows];
#pragma unroll
                for (int r = 0; r < kW8Rows; ++r) qf[r] = (float)w[r][k];
#pragma unroll
                for (int mm = 0; mm < MC; ++mm) {
                    if (mm >= mc) continue;
                    const float xk = X[(size_t)(m0 + mm) * K + k];
#pragma unroll
                    for (int r = 0; r < kW8Rows; ++r) acc[mm][r] = fmaf(xk, qf[r], acc[mm][r]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kW8Rows; ++r) {
#pragma unroll
            for (int mm = 0; mm < MC; ++mm) {
                const float v = warp_sum(acc[mm][r]);
                if (lane == 0 && mm < mc && rv[r]) Y[(size_t)(m0 + mm) * N + n0 + r] = v * sc[r];
            }
        }
    }
}

__global__ void gemm_f32_naive(const float *A, const float *B, float *C, int M, int N, int K, int ta, int tb) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
    if (n >= N || m >= M) return;
    const int lda = ta ? M : K, ldb = tb ? K : N;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) {
        float a = ta ? A[(size_t)k * lda + m] : A[(size_t)m * lda + k];
        float b = tb ? B[(size_t)n * ldb + k] : B[(size_t)k * ldb + n];
        acc = fmaf(a, b, acc);
    }
    C[(size_t)m * N + n] = acc;
}

__global__ void argmax_bf16_row(const __nv_bfloat16 *__restrict__ v, int n, int *out_idx, float *out_val) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float x = bf2f(v[i]);
        if (x > best || (x == best && i < bi)) { best = x; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ob = __shfl_xor_sync(0xffffffffu, best, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ob = __shfl_xor_sync(0xffffffffu, best, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (lane == 0) { *out_idx = bi; *out_val = best; }
    }
}

// split_k: spread short grids over more CTAs by splitting K (partials reduced by the last
// CTA of each row tile); false keeps one CTA per row tile, which saves that reduction's
// round trip where the grid is already wide enough.
template <int RT, int NT, bool GROUPED, bool KP>
int launch_mma(const __nv_bfloat16 *X, int M, int K, const uint8_t *W, const float *S, int N, __nv_bfloat16 *Y,
               const char *what, bool split_k = true) {
    const int tiles = (N + 16 * RT - 1) / (16 * RT);
    const int G = K >> 7;
    const int target = 2 * pilm::num_sms();
    int splits = 1;
    if (split_k && tiles < target) {
        splits = (target + tiles - 1) / tiles;
        int max_splits = G / kGemvWarps;  // keep every warp busy
        if (max_splits < 1) max_splits = 1;
        if (splits > max_splits) splits = max_splits;
    }
    const int gps = (G + splits - 1) / splits;
    splits = (G + gps - 1) / gps;
    float *ws = nullptr;
    int *ctr = nullptr;
    if (splits > 1) {
        ws = (float *)pilm::workspace((size_t)splits * M * N * sizeof(float));
        ctr = pilm::counters((size_t)tiles);
        PILM_REQUIRE(ws && ctr, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
    }
    dim3 grid(tiles, splits);
    static int per_sm = 0;  // resident CTAs per SM of the prefetching instantiation
    if (NT == 1 && per_sm == 0 &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, w4_gemv_mma<RT, NT, GROUPED, KP, true>,
                                                      kGemvWarps * 32, 0) != cudaSuccess)
        per_sm = 1;
    if (NT == 1 && tiles * splits <= per_sm * pilm::num_sms())  // M <= 8, the grid is one wave
        launch_pdl(w4_gemv_mma<RT, NT, GROUPED, KP, true>, dim3(grid), dim3(kGemvWarps * 32), 0, X, M, K, W, S, N,
                   Y, ws, ctr, splits, gps);
    else
        launch_pdl(w4_gemv_mma<RT, NT, GROUPED, KP, false>, dim3(grid), dim3(kGemvWarps * 32), 0, X, M, K, W, S, N,
                   Y, ws, ctr, splits, gps);
    return pilm::check_launch(what);
}

template <bool GROUPED, bool KP>
int dispatch_mma(const __nv_bfloat16 *X, int M, int K, const uint8_t *W, const float *S, int N, __nv_bfloat16 *Y,
                 const char *what) {
    // M <= 8.  Projections narrow enough for fewer than two 32-row tiles per SM and with at
    // most 32 groups (each warp then walks at most 4 of them): 16-row tiles, no split-K, and
    // the next group's loads in flight during the current group's math.  Measured at M = 4:
    // 2048 x 4096 6.0 -> 4.2 us, 2048 x 2048 5.8 -> 4.1 us, 4096 x 6144 8.2 -> 7.4 us; wider
    // or deeper shapes keep the 32-row tiles and split-K (16-row tiles there were 5-40% slower).
    if (M <= 8 && (N + 31) / 32 < 2 * pilm::num_sms() && (K >> 7) <= 4 * kGemvWarps)
        return launch_mma<1, 1, GROUPED, KP>(X, M, K, W, S, N, Y, what, false);
    if (M <= 8) return launch_mma<2, 1, GROUPED, KP>(X, M, K, W, S, N, Y, what);
    if (M <= 16) return launch_mma<2, 2, GROUPED, KP>(X, M, K, W, S, N, Y, what);
    if (M <= 32) return launch_mma<1, 4, GROUPED, KP>(X, M, K, W, S, N, Y, what);
    return launch_mma<1, 8, GROUPED, KP>(X, M, K, W, S, N, Y, what);
}

// k-pair nibble order: within every 32-bit word (k = 8i .. 8i + 7 of a row, k at nibble
// k - 8i in the reference packing), nibble p holds k = 8i + 2p for p < 4 and
// 8i + 2(p - 4) + 1 for p >= 4.  One thread per word; in place is allowed.
__global__ void repack_w4_kpairs(const uint32_t *__restrict__ in, uint32_t *out, size_t words) {
    for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < words; t += (size_t)gridDim.x * blockDim.x) {
        const uint32_t w = in[t];
        uint32_t r = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int pos = (j & 1) ? 4 + (j >> 1) : (j >> 1);
            r |= ((w >> (4 * j)) & 15u) << (4 * pos);
        }
        out[t] = r;
    }
}

bool aligned16(const void *p) { return (((uintptr_t)p) & 15) == 0; }

}  // namespace

namespace pilm {

// Shared entry used by the ABI wrappers and by the fused SwiGLU path.
// qf: 0 = W4 grouped (gs = 32 or 128), 1 = W4 per-row, 2 = W8 per-row.
int linear_bf16(int qf, int gs, const void *A, int M, int K, const void *W, const float *S, int N, void *C,
                const char *what, bool kpairs, float *defer, size_t defer_cap, int *defer_splits,
                unsigned long long *amax, int *amax_done) {
    if (defer_splits) *defer_splits = 0;
    if (amax_done) *amax_done = 0;
    const __nv_bfloat16 *X = (const __nv_bfloat16 *)A;
    __nv_bfloat16 *Y = (__nv_bfloat16 *)C;
    if (M == 0 || N == 0) return ECPU_OK;
    const bool mma_ok = (qf == 1 || (qf == 0 && gs == 128)) && (K % 128 == 0) && aligned16(A) && aligned16(W);
    PILM_REQUIRE(!kpairs || mma_ok, ECPU_ERR_UNSUPPORTED,
                 "%s: k-pair weights need K %% 128 == 0 and 16-byte aligned activations and weights", what);
    if (mma_ok) {
        // above 16 rows the register-dequant GEMV re-reads each activation tile per 16
        // weight rows; the tensor-core GEMM stages it once per 128 (N = 32, 48, ... rows)
        if (M > 16) {
            int rc = linear_w4_tc(X, M, K, (const uint8_t *)W, S, N, Y, qf == 0, kpairs, what, defer, defer_cap,
                                  defer_splits, amax, amax_done);
            if (rc != ECPU_ERR_UNSUPPORTED) return rc;
        }
        // register-dequant GEMV, in slabs of at most 64 activation rows
        for (int m0 = 0; m0 < M; m0 += 64) {
            const int mm = M - m0 < 64 ? M - m0 : 64;
            const __nv_bfloat16 *Xs = X + (size_t)m0 * K;
            __nv_bfloat16 *Ys = Y + (size_t)m0 * N;
            const uint8_t *Wq = (const uint8_t *)W;
            int rc = qf == 0 ? (kpairs ? dispatch_mma<true, true>(Xs, mm, K, Wq, S, N, Ys, what)
                                       : dispatch_mma<true, false>(Xs, mm, K, Wq, S, N, Ys, what))
                             : (kpairs ? dispatch_mma<false, true>(Xs, mm, K, Wq, S, N, Ys, what)
                                       : dispatch_mma<false, false>(Xs, mm, K, Wq, S, N, Ys, what));
            if (rc != ECPU_OK) return rc;
        }
        return ECPU_OK;
    }
    dim3 grid((N + 7) / 8);
    switch (qf) {
        case 0: linear_generic<0><<<grid, 256, 0, stream()>>>(X, M, K, W, S, N, gs, Y); break;
        case 1: linear_generic<1><<<grid, 256, 0, stream()>>>(X, M, K, W, S, N, gs, Y); break;
        default: linear_generic<2><<<grid, 256, 0, stream()>>>(X, M, K, W, S, N, gs, Y); break;
    }
    return check_launch(what);
}

}  // namespace pilm

#define LINEAR_ARGS_OK(fn)                                                                   \
    PILM_REQUIRE(desc &&A &&W &&scales &&C, ECPU_ERR_PARAM, fn ": null argument");            \
    PILM_REQUIRE(desc->M <= 0x7fffffff && desc->N <= 0x7fffffff && desc->K <= 0x7fffffff, ECPU_ERR_PARAM, \
                 fn ": dimension too large")

extern "C" {

int ekernel_gemm(const ekernel_gemm_desc_t *desc, const void *A, const void *B, void *C, ekernel_isa_t isa) {
    (void)isa;
    PILM_REQUIRE(desc && A && B && C, ECPU_ERR_PARAM, "ekernel_gemm: null argument");
    PILM_REQUIRE(desc->a_prec == ECPU_PRECISION_F32 && desc->b_prec == ECPU_PRECISION_F32 &&
                     desc->out_prec == ECPU_PRECISION_F32,
                 ECPU_ERR_UNSUPPORTED, "ekernel_gemm: only F32 is supported");
    if (desc->M == 0 || desc->N == 0) return ECPU_OK;
    dim3 grid((unsigned)((desc->N + 127) / 128), (unsigned)desc->M);
    gemm_f32_naive<<<grid, 128, 0, pilm::stream()>>>((const float *)A, (const float *)B, (float *)C, (int)desc->M,
                                                     (int)desc->N, (int)desc->K, desc->transpose_a, desc->transpose_b);
    return pilm::check_launch("ekernel_gemm");
}

int ekernel_linear_w8a32(const ekernel_linear_w8a32_desc_t *desc, const float *A, const int8_t *W,
                         const float *scales, float *C, ekernel_isa_t isa) {
    (void)isa;
    LINEAR_ARGS_OK("ekernel_linear_w8a32");
    if (desc->M == 0 || desc->N == 0) return ECPU_OK;
    const unsigned grid = (unsigned)((desc->N + 8 * kW8Rows - 1) / (8 * kW8Rows));
    const int M = (int)desc->M, K = (int)desc->K, N = (int)desc->N;
    if (M == 1)
        launch_pdl(w8a32_gemv<1>, dim3(grid), dim3(256), 0, A, M, K, W, scales, N, C);
    else if (M == 2)
        launch_pdl(w8a32_gemv<2>, dim3(grid), dim3(256), 0, A, M, K, W, scales, N, C);
    else
        launch_pdl(w8a32_gemv<4>, dim3(grid), dim3(256), 0, A, M, K, W, scales, N, C);
    return pilm::check_launch("ekernel_linear_w8a32");
}

int ekernel_linear_w8a16_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const int8_t *W,
                              const float *scales, uint16_t *C, ekernel_isa_t isa) {
    (void)isa;
    LINEAR_ARGS_OK("ekernel_linear_w8a16_bf16");
    return pilm::linear_bf16(2, 0, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                             "ekernel_linear_w8a16_bf16");
}

int ekernel_linear_w8a16_bf16_argmax(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                     const int8_t *W, const float *scales, size_t *out_index, float *out_value,
                                     ekernel_isa_t isa) {
    (void)isa;
    PILM_REQUIRE(desc && A && W && scales && out_index && out_value, ECPU_ERR_PARAM,
                 "ekernel_linear_w8a16_bf16_argmax: null argument");
    PILM_REQUIRE(desc->M == 1 && desc->N > 0 && desc->K > 0 && desc->N <= 0x7fffffff, ECPU_ERR_UNSUPPORTED,
                 "ekernel_linear_w8a16_bf16_argmax: M must be 1");
    const size_t n = desc->N;
    char *ws = (char *)pilm::workspace(n * 2 + 64);
    PILM_REQUIRE(ws, ECPU_ERR_MEM, "ekernel_linear_w8a16_bf16_argmax: workspace allocation failed");
    int rc = pilm::linear_bf16(2, 0, A, 1, (int)desc->K, W, scales, (int)n, ws + 64,
                               "ekernel_linear_w8a16_bf16_argmax");
    if (rc != ECPU_OK) return rc;
    argmax_bf16_row<<<1, 1024, 0, pilm::stream()>>>((const __nv_bfloat16 *)(ws + 64), (int)n, (int *)ws,
                                                   (float *)(ws + 4));
    rc = pilm::check_launch("ekernel_linear_w8a16_bf16_argmax");
    if (rc != ECPU_OK) return rc;
    int idx = 0;
    float val = 0.f;
    cudaMemcpyAsync(&idx, ws, 4, cudaMemcpyDeviceToHost, pilm::stream());
    cudaMemcpyAsync(&val, ws + 4, 4, cudaMemcpyDeviceToHost, pilm::stream());
    if (cudaStreamSynchronize(pilm::stream()) != cudaSuccess) {
        pilm::set_error("ekernel_linear_w8a16_bf16_argmax: %s", cudaGetErrorString(cudaGetLastError()));
        return ECPU_ERR_KERNEL;
    }
    *out_index = (size_t)idx;
    *out_value = val;
    return ECPU_OK;
}

int ekernel_linear_w4a16_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                              const float *scales, uint16_t *C, ekernel_isa_t isa) {
    (void)isa;
    LINEAR_ARGS_OK("ekernel_linear_w4a16_bf16");
    return pilm::linear_bf16(1, 0, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                             "ekernel_linear_w4a16_bf16");
}

int ekernel_linear_w4a16g32_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                                 const float *scales, uint16_t *C, ekernel_isa_t isa) {
    (void)isa;
    LINEAR_ARGS_OK("ekernel_linear_w4a16g32_bf16");
    return pilm::linear_bf16(0, 32, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                             "ekernel_linear_w4a16g32_bf16");
}

int ekernel_linear_w4a16g128_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                                  const float *scales, uint16_t *C, ekernel_isa_t isa) {
    (void)isa;
    LINEAR_ARGS_OK("ekernel_linear_w4a16g128_bf16");
    return pilm::linear_bf16(0, 128, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                             "ekernel_linear_w4a16g128_bf16");
}

int ekernel_linear_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint16_t *W, uint16_t *C) {
    PILM_REQUIRE(desc && A && W && C, ECPU_ERR_PARAM, "ekernel_linear_bf16: null argument");
    PILM_REQUIRE(desc->M <= 0x7fffffff && desc->N <= 0x7fffffff && desc->K <= 0x7fffffff, ECPU_ERR_PARAM,
                 "ekernel_linear_bf16: dimension too large");
    const int M = (int)desc->M, N = (int)desc->N, K = (int)desc->K;
    if (M == 0 || N == 0) return ECPU_OK;
    PILM_REQUIRE(K % 8 == 0 && aligned16(A) && aligned16(W), ECPU_ERR_UNSUPPORTED,
                 "ekernel_linear_bf16: needs K %% 8 == 0 and 16-byte aligned A and W");
    const __nv_bfloat16 *X = (const __nv_bfloat16 *)A, *Wb = (const __nv_bfloat16 *)W;
    __nv_bfloat16 *Y = (__nv_bfloat16 *)C;
    for (int m0 = 0; m0 < M; m0 += 64) {  // slabs of at most 64 activation rows
        const int mm = M - m0 < 64 ? M - m0 : 64;
        const __nv_bfloat16 *Xs = X + (size_t)m0 * K;
        __nv_bfloat16 *Ys = Y + (size_t)m0 * N;
        int rc;
        if (mm <= 8)
            rc = launch_bf16w<2, 1>(Xs, mm, K, Wb, N, Ys, "ekernel_linear_bf16");
        else if (mm <= 16)
            rc = launch_bf16w<2, 2>(Xs, mm, K, Wb, N, Ys, "ekernel_linear_bf16");
        else if (mm <= 32)
            rc = launch_bf16w<2, 4>(Xs, mm, K, Wb, N, Ys, "ekernel_linear_bf16");
        else
            rc = launch_bf16w<1, 8>(Xs, mm, K, Wb, N, Ys, "ekernel_linear_bf16");
        if (rc != ECPU_OK) return rc;
    }
    return ECPU_OK;
}

int ekernel_repack_w4_kpairs(const uint8_t *qweight, size_t N, size_t K, uint8_t *out) {
    PILM_REQUIRE(qweight && out, ECPU_ERR_PARAM, "ekernel_repack_w4_kpairs: null argument");
    PILM_REQUIRE(K % 8 == 0, ECPU_ERR_PARAM, "ekernel_repack_w4_kpairs: K must be a multiple of 8");
    PILM_REQUIRE((((uintptr_t)qweight) & 3) == 0 && (((uintptr_t)out) & 3) == 0, ECPU_ERR_PARAM,
                 "ekernel_repack_w4_kpairs: buffers must be 4-byte aligned");
    const size_t words = N * (K / 8);
    if (words == 0) return ECPU_OK;
    const size_t blocks = (words + 255) / 256;
    repack_w4_kpairs<<<(unsigned)(blocks < 8192 ? blocks : 8192), 256, 0, pilm::stream()>>>(
        (const uint32_t *)qweight, (uint32_t *)out, words);
    return pilm::check_launch("ekernel_repack_w4_kpairs");
}

int ekernel_linear_w4a16g128_bf16_kpairs(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                         const uint8_t *W, const float *scales, uint16_t *C, ekernel_isa_t isa) {
    (void)isa;
    LINEAR_ARGS_OK("ekernel_linear_w4a16g128_bf16_kpairs");
    return pilm::linear_bf16(0, 128, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                             "ekernel_linear_w4a16g128_bf16_kpairs", true);
}

int ekernel_linear_w4a16g128_bf16_kpairs_deferred(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                                  const uint8_t *W, const float *scales, uint16_t *C,
                                                  float *partials, size_t partials_bytes, int32_t *splits) {
    LINEAR_ARGS_OK("ekernel_linear_w4a16g128_bf16_kpairs_deferred");
    PILM_REQUIRE(splits, ECPU_ERR_PARAM, "ekernel_linear_w4a16g128_bf16_kpairs_deferred: null splits");
    int s = 0;
    const int rc = pilm::linear_bf16(0, 128, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                                     "ekernel_linear_w4a16g128_bf16_kpairs_deferred", true, partials,
                                     partials ? partials_bytes : 0, &s);
    *splits = rc == ECPU_OK ? s : 0;
    return rc;
}

int ekernel_linear_w4a16g128_bf16_kpairs_argmax(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                                const uint8_t *W, const float *scales, uint16_t *C,
                                                uint64_t *row_keys, int32_t *fused) {
    LINEAR_ARGS_OK("ekernel_linear_w4a16g128_bf16_kpairs_argmax");
    PILM_REQUIRE(row_keys && fused, ECPU_ERR_PARAM, "ekernel_linear_w4a16g128_bf16_kpairs_argmax: null argument");
    int done = 0;
    const int rc = pilm::linear_bf16(0, 128, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                                     "ekernel_linear_w4a16g128_bf16_kpairs_argmax", true, nullptr, 0, nullptr,
                                     (unsigned long long *)row_keys, &done);
    *fused = rc == ECPU_OK ? done : 0;
    return rc;
}

size_t ekernel_linear_w4a16g128_partials_bytes(size_t M, size_t N, size_t K) {
    if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return 0;
    return pilm::w4_tc_partials_bytes((int)M, (int)N, (int)K);
}

int ekernel_linear_w4a16_bf16_kpairs(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                                     const float *scales, uint16_t *C, ekernel_isa_t isa) {
    (void)isa;
    LINEAR_ARGS_OK("ekernel_linear_w4a16_bf16_kpairs");
    return pilm::linear_bf16(1, 0, A, (int)desc->M, (int)desc->K, W, scales, (int)desc->N, C,
                             "ekernel_linear_w4a16_bf16_kpairs", true);
}

}  // extern "C"
