// Paged-KV attention for the MTP verify rows (GQA, QK-RMSNorm, RoPE, KV append).
//
// Reference: FullAttention.forward (src/models/qwen3/attention.py:68-141) with
// apply_rope (src/models/base/layers.py:122-176) and the paged cache layout of
// src/runtime/kvcache/physical_kv.py:30-33: per layer K and V tensors
// [num_blocks, block_size, n_kv, head_dim] bf16.
//
// Kernels:
//   qk_prologue   one warp per (row, head): RMSNorm (module rounding) + RoPE for q/k,
//                 K/V written into their page slots, q/gate written for attention.
//   attn_verify   split-KV decode attention.  A CTA owns (sequence, kv head, split,
//                 row chunk); its query rows are all q_len x (n_heads / n_kv) rows that
//                 share the kv head, so every K/V byte of the split is read from HBM
//                 once per CTA.  Each of the 4 warps streams every 4th page of the split
//                 through a private TMA ring (3 pages deep): one page of one KV head is
//                 four cp.async.bulk.tensor loads (K and V, two 128-byte SWIZZLE_128B
//                 halves each) completing on the stage's mbarrier.  The warp computes
//                 S = Q K^T and O += P V with mma.sync m16n8k16 (bf16 in, fp32
//                 accumulate) and keeps an fp32 online softmax; warps then merge.
//   attn_merge    combines split partials (m, l, O) and applies the output gate.
#include <cstring>
#include <mutex>

#include "common.cuh"

using namespace pilm;

// Fixed device scratch for ekernel_paged_attention_verify_noalloc (see below).  Every
// GPU that loads this library holds these bytes until the process exits.
constexpr size_t kNoAllocAttnScratchBytes = (size_t)8 << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_noalloc_attn_scratch[kNoAllocAttnScratchBytes];
// The allocation-free entry point's own error word (a page wait that gave up), so that
// it never needs the library's allocated one.
static __device__ int g_noalloc_err_word;

namespace {

constexpr int kHD = 128;         // head_dim supported by the tensor-core path
constexpr int kWarps = 4;        // warps per attention CTA
constexpr int kMinPagesPerCta = 8;  // whole-page kernel: pages per CTA at least (short batches)
constexpr int kStages = 3;       // pages in flight per warp
constexpr int kPageBytes = 16 * kHD * 2;  // one K (or V) tile of a 16-token page
constexpr uint32_t kAttnWaitLimit = 1u << 22;  // polls before a page wait gives up

// ---------------------------------------------------------------------------------
// Prologue: q/k RMSNorm + RoPE, KV append
// ---------------------------------------------------------------------------------
// The projection row comes as bf16 (qkv) or as split-K partial sums of the W4 linear
// (part: [splits][total_q][qkv_stride] fp32), summed in split order and rounded to bf16
// exactly as the GEMM's combine pass would have written them.
struct QkvSrc {
    const __nv_bfloat16 *qkv;
    const float *part;
    int splits;
    size_t plane;
};

__global__ void qk_prologue(const QkvSrc src_in, int total_q, int nh, int nkv, int qkv_stride,
                            int gated, const __nv_bfloat16 *__restrict__ qnw, const __nv_bfloat16 *__restrict__ knw,
                            float eps, int add_one, const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                            int rope_rows, int rot_dim, const int32_t *__restrict__ positions,
                            const int32_t *__restrict__ slots, long long num_slots, __nv_bfloat16 *__restrict__ kc,
                            __nv_bfloat16 *__restrict__ vc, __nv_bfloat16 *__restrict__ q_out,
                            __nv_bfloat16 *__restrict__ gate_out) {
    pdl_trigger();
    __shared__ float buf[8][kHD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * 8 + warp;
    const int heads = nh + nkv;
    if (item >= total_q * heads) return;
    const int row = item / heads, h = item % heads;
    const bool is_q = h < nh;
    size_t src;  // element offset of this head's 128 values
    const int qsec = nh * kHD * (gated ? 2 : 1);
    if (is_q)
        src = (size_t)row * qkv_stride + (size_t)h * kHD * (gated ? 2 : 1);
    else
        src = (size_t)row * qkv_stride + qsec + (size_t)(h - nh) * kHD;
    const __nv_bfloat16 *nw = is_q ? qnw : knw;
    // The norm weights, RoPE tables, positions and slots are constant or written by the
    // host before the step, so they are read before the wait for the previous kernel; the
    // projection (its output) after it.
    const int pos = positions[row];
    const int nf = rot_dim >> 1;
    const bool pos_ok = pos >= 0 && pos < rope_rows;
    const long long slot = is_q ? -1 : slots[row];
    float wv[4], cv[4], sv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        float wf = bf2f(nw[d]);
        if (add_one) wf = bf16_round(__fadd_rn(wf, 1.0f));
        wv[j] = wf;
        const int f = d < nf ? d : d - nf;
        const bool rot = d < rot_dim && pos_ok;
        cv[j] = rot ? cos_t[(size_t)pos * nf + f] : 1.f;
        sv[j] = rot ? sin_t[(size_t)pos * nf + f] : 0.f;
    }
    // The values only copied through, loaded with the head's own: a K head's V values (to
    // the cache), a gated Q head's gate values (to gate_out).
    const bool has_aux = !is_q || (gated && gate_out);
    const size_t asrc = is_q ? src + kHD : (size_t)row * qkv_stride + qsec + (size_t)nkv * kHD + (size_t)(h - nh) * kHD;
    pdl_wait();
    float x[4];
    __nv_bfloat16 vv[4];
    if (src_in.part) {
        // every split of the lane's 4 values (and 4 aux values) is loaded before the adds,
        // which run per element in split order from 0 as the combine pass adds: one wait
        // on memory for up to 4 splits, not one per element
        float xs[4] = {0.f, 0.f, 0.f, 0.f}, as[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s0 = 0; s0 < src_in.splits; s0 += 4) {
            float tx[4][4], ta[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const bool ok = s0 + u < src_in.splits;
                const float *pl = src_in.part + (size_t)(s0 + u) * src_in.plane;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    tx[u][j] = ok ? __ldcs(pl + src + lane + 32 * j) : 0.f;
                    ta[u][j] = ok && has_aux ? __ldcs(pl + asrc + lane + 32 * j) : 0.f;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (s0 + u < src_in.splits)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        xs[j] += tx[u][j];
                        as[j] += ta[u][j];
                    }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[j] = bf16_round(xs[j]);
            vv[j] = f2bf(as[j]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[j] = bf2f(src_in.qkv[src + lane + 32 * j]);
            vv[j] = has_aux ? src_in.qkv[asrc + lane + 32 * j] : __float2bfloat16_rn(0.f);
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) ss = fmaf(x[j], x[j], ss);
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHD), eps)));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        float xn = bf16_round(__fmul_rn(x[j], inv));
        buf[warp][d] = bf16_round(__fmul_rn(xn, wv[j]));
    }
    __syncwarp();
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        float v = buf[warp][d];
        if (d < rot_dim && pos_ok) {
            // out_first = a*cos - b*sin ; out_second = a*sin + b*cos  (layers.py:161-164)
            const float cs = cv[j], sn = sv[j];
            if (d < nf) {
                const float b = buf[warp][d + nf];
                v = __fsub_rn(__fmul_rn(v, cs), __fmul_rn(b, sn));
            } else {
                const float a = buf[warp][d - nf];
                v = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(v, cs));
            }
        }
        y[j] = v;
    }
    if (is_q) {
        __nv_bfloat16 *qo = q_out + ((size_t)row * nh + h) * kHD;
#pragma unroll
        for (int j = 0; j < 4; ++j) qo[lane + 32 * j] = f2bf(y[j]);
        if (has_aux) {
            __nv_bfloat16 *go = gate_out + (size_t)row * nh * kHD + (size_t)h * kHD;
#pragma unroll
            for (int j = 0; j < 4; ++j) go[lane + 32 * j] = vv[j];
        }
    } else {
        if (slot < 0 || slot >= num_slots) return;  // rejected / padded rows are not written
        const int kvh = h - nh;
        __nv_bfloat16 *kd = kc + ((size_t)slot * nkv + kvh) * kHD;
        __nv_bfloat16 *vd = vc + ((size_t)slot * nkv + kvh) * kHD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            kd[lane + 32 * j] = f2bf(y[j]);
            vd[lane + 32 * j] = vv[j];
        }
    }
}

// ---------------------------------------------------------------------------------
// Tensor-core helpers
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// Byte offset of 16-byte chunk `ch` (0..15, dims 8ch..8ch+7) of key row `row` (0..15) in a
// 4 KB K or V tile as TMA writes it: two halves of 16 rows x 128 B (dims 0-63, 64-127), each
// SWIZZLE_128B (chunk c of row r at c ^ (r & 7); the tile is 1024-byte aligned).
__device__ __forceinline__ uint32_t swz(int row, int ch) {
    return (uint32_t)(((ch >> 3) << 11) + row * 128 + (((ch & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"((uint32_t)__cvta_generic_to_shared(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"((uint32_t)__cvta_generic_to_shared(b)) : "memory");
}
// bounded wait; false if the phase did not complete within the poll limit
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *b, uint32_t parity) {
    for (uint32_t i = 0; i < kAttnWaitLimit; ++i)
        if (mbar_try_wait(b, parity)) return true;
    return false;
}
// 3-D tile copy global -> shared (no multicast), completing on an mbarrier
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            dst),
        "l"(map), "r"((uint32_t)__cvta_generic_to_shared(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

struct AttnParams {
    const __nv_bfloat16 *q;      // [total_q, nh, 128]
    const __nv_bfloat16 *kc;     // [num_blocks, 16, nkv, 128]
    const __nv_bfloat16 *vc;
    const int32_t *block_table;  // [B, max_blocks]
    const int32_t *cu_q;         // [B+1]
    const int32_t *ctx;          // [B]
    const __nv_bfloat16 *gate;   // [total_q, nh*128] or null
    __nv_bfloat16 *out;          // [total_q, nh*128]
    float *part_o;               // [splits, total_q, nh, 128]
    float *part_ml;              // [splits, total_q, nh, 2]
    int *err;                    // device error word: set when a page wait gave up
    int nh, nkv, gsz, max_blocks, num_blocks, total_q;
    int splits, pages_per_split, row_chunk;  // rows per CTA = 16 * MT; pages_per_split: host sizing only
    float scale;                 // rne_bf16-compatible fp32 value of 1/sqrt(head_dim)
};

// grid: (splits, nkv * row_chunks, B); block: 128 threads.  kmap / vmap: the K and V
// caches as 3-D tensors (dim, kv head, slot) with 64 x 1 x 16 SWIZZLE_128B boxes.
template <int MT>
__global__ void __launch_bounds__(kWarps * 32, 2) attn_verify(const __grid_constant__ CUtensorMap kmap,
                                                             const __grid_constant__ CUtensorMap vmap,
                                                             const AttnParams p) {
    pdl_entry();
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kWarps][kStages];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, c = lane & 3;
    const int split = blockIdx.x;
    const int b = blockIdx.z;
    const int chunks = (int)gridDim.y / p.nkv;
    const int kvh = blockIdx.y / chunks, rc = blockIdx.y % chunks;

    const int q0 = p.cu_q[b], q_len = p.cu_q[b + 1] - q0;
    const int ctx = p.ctx[b];
    const int R = q_len * p.gsz;
    const int row_base = rc * 16 * MT;
    if (row_base >= R || q_len <= 0 || ctx <= 0) return;
    const int p0 = ctx - q_len;  // position of the first verify row
    // every sequence divides its own pages evenly over the splits, so the split count
    // (chosen on the host from a context bound) never leaves a long sequence's work on
    // one CTA or a short one spread thin
    const int P = (ctx + 15) >> 4;
    const int pps = (P + p.splits - 1) / p.splits;
    const int pg0 = split * pps;
    const int pg1 = min(P, pg0 + pps);
    // the last row of this CTA sees keys up to p0 + jmax
    const int jmax = min(q_len - 1, (row_base + 16 * MT - 1) / p.gsz);
    const int pg_vis = min(pg1, ((p0 + jmax) >> 4) + 1);

    // ---- Q fragments (A operand), rows row_base + mt*16 + {r, r+8} ----
    uint32_t qf[MT][8][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int rho = row_base + mt * 16 + r + hh * 8;
            const bool ok = rho < R;
            const int j = ok ? rho / p.gsz : 0, g = ok ? rho % p.gsz : 0;
            const __nv_bfloat16 *qrow = p.q + ((size_t)(q0 + j) * p.nh + (size_t)kvh * p.gsz + g) * kHD;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                uint32_t lo = ok ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 2 * c) : 0u;
                uint32_t hi = ok ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 8 + 2 * c) : 0u;
                qf[mt][ks][hh] = lo;      // a0 (row r) / a1 (row r+8)
                qf[mt][ks][2 + hh] = hi;  // a2 / a3
            }
        }
    // query position of each of the thread's rows (for the causal mask)
    int qpos[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int rho = row_base + mt * 16 + r + hh * 8;
            qpos[mt][hh] = rho < R ? p0 + rho / p.gsz : -1;
        }

    float o[MT][16][4];
    float mrow[MT][2], lrow[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) o[mt][nt][j] = 0.f;
        mrow[mt][0] = mrow[mt][1] = -INFINITY;
        lrow[mt][0] = lrow[mt][1] = 0.f;
    }

    if (threadIdx.x == 0) {
        for (int w = 0; w < kWarps; ++w)
            for (int st = 0; st < kStages; ++st) mbar_init(&full_bar[w][st], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    uint8_t *ring = smem + (size_t)warp * kStages * 2 * kPageBytes;
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    const int32_t *bt = p.block_table + (size_t)b * p.max_blocks;

    // pages handled by this warp: pg0 + warp, pg0 + warp + 4, ... (< pg_vis)
    const int n_it = pg_vis > pg0 + warp ? (pg_vis - (pg0 + warp) + kWarps - 1) / kWarps : 0;
    int issued = 0;  // lane 0's count of pages put in flight
    // lane 0 loads page `it` of this warp into `stage`: K and V of this KV head, 8 KB.
    // The stage's previous contents were read (ldmatrix) or written (zeroing) through
    // the generic proxy, which the proxy fence orders before the TMA's writes.
    auto issue = [&](int it, int stage) {
        if (lane != 0 || it >= n_it) return;
        const int pg = pg0 + warp + it * kWarps;
        int blk = bt[pg];
        if (blk < 0 || blk >= p.num_blocks) blk = 0;  // zeroed after it lands
        const uint32_t dst = ring_s + stage * 2 * kPageBytes;
        uint64_t *bar = &full_bar[warp][stage];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(bar, 2 * kPageBytes);
        tma_load_3d(dst, &kmap, bar, 0, kvh, blk * 16);
        tma_load_3d(dst + kPageBytes / 2, &kmap, bar, 64, kvh, blk * 16);
        tma_load_3d(dst + kPageBytes, &vmap, bar, 0, kvh, blk * 16);
        tma_load_3d(dst + kPageBytes + kPageBytes / 2, &vmap, bar, 64, kvh, blk * 16);
        ++issued;
    };

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) issue(s, s);

    int consumed = 0;
    for (int it = 0; it < n_it; ++it) {
        issue(it + kStages - 1, (it + kStages - 1) % kStages);
        const int stage = it % kStages;
        const bool landed = mbar_wait_bounded(&full_bar[warp][stage], (uint32_t)(it / kStages) & 1u);
        if (!__all_sync(0xffffffffu, landed)) {
            if (lane == 0) atomicExch(p.err, 1);
            break;
        }
        consumed = it + 1;
        const uint32_t ks_base = ring_s + stage * 2 * kPageBytes, vs_base = ks_base + kPageBytes;
        const int pg = pg0 + warp + it * kWarps;
        {
            // keys past the context get P = 0, so their V rows must be finite: zero them
            // (and the whole page for an invalid block id, whose K then scores 0)
            const int blk = bt[pg];
            const bool blk_ok = blk >= 0 && blk < p.num_blocks;
            const int valid = min(16, ctx - pg * 16);
            if (!blk_ok || valid < 16) {
                const int r0 = blk_ok ? valid : 0;
                uint8_t *kp = ring + (size_t)stage * 2 * kPageBytes, *vp = kp + kPageBytes;
                for (int idx = lane; idx < (16 - r0) * 16; idx += 32) {
                    const int row = r0 + (idx >> 4), ch = idx & 15;
                    const size_t off = (size_t)((ch >> 3) << 11) + row * 128 + ((ch & 7) << 4);
                    *reinterpret_cast<uint4 *>(vp + off) = make_uint4(0u, 0u, 0u, 0u);
                    if (!blk_ok) *reinterpret_cast<uint4 *>(kp + off) = make_uint4(0u, 0u, 0u, 0u);
                }
                __syncwarp();
            }
        }

        // ---- S = Q K^T over the 16 keys of the page ----
        float sacc[MT][2][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) sacc[mt][nt][j] = 0.f;
        {
            const int qm = lane >> 3, i8 = lane & 7;
            const int key = (qm >= 2 ? 8 : 0) + i8;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                uint32_t b00, b01, b10, b11;
                ldsm_x4(ks_base + swz(key, 2 * ks + (qm & 1)), b00, b01, b10, b11);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma16816(sacc[mt][0], qf[mt][ks], b00, b01);
                    mma16816(sacc[mt][1], qf[mt][ks], b10, b11);
                }
            }
        }
        // ---- reference rounding, causal mask, online softmax ----
        uint32_t pa[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float mx = -INFINITY;
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int kp = pg * 16 + nt * 8 + 2 * c + e;
                        float s = sacc[mt][nt][hh * 2 + e];
                        // scores = bmm(q, k^T) in bf16, then * scale in bf16 (attention.py:128-129)
                        s = bf16_round(__fmul_rn(bf16_round(s), p.scale));
                        if (kp > qpos[mt][hh] || kp >= ctx) s = -INFINITY;
                        sacc[mt][nt][hh * 2 + e] = s;
                        mx = fmaxf(mx, s);
                    }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float mnew = fmaxf(mrow[mt][hh], mx);
                const float alpha = (mnew == -INFINITY) ? 1.f : expf(mrow[mt][hh] - mnew);
                mrow[mt][hh] = mnew;
                float ls = 0.f;
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        float s = sacc[mt][nt][hh * 2 + e];
                        float pv = (s == -INFINITY) ? 0.f : expf(s - mnew);
                        sacc[mt][nt][hh * 2 + e] = pv;
                        ls += pv;
                    }
                lrow[mt][hh] = lrow[mt][hh] * alpha + ls;
                // once the running maxima settle, alpha is exactly 1 for every row: skip the
                // multiplies (a product by 1 is exact, so results are unchanged)
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                    for (int nt = 0; nt < 16; ++nt) {
                        o[mt][nt][hh * 2 + 0] *= alpha;
                        o[mt][nt][hh * 2 + 1] *= alpha;
                    }
                }
            }
            pa[mt][0] = pack_bf16(sacc[mt][0][0], sacc[mt][0][1]);
            pa[mt][1] = pack_bf16(sacc[mt][0][2], sacc[mt][0][3]);
            pa[mt][2] = pack_bf16(sacc[mt][1][0], sacc[mt][1][1]);
            pa[mt][3] = pack_bf16(sacc[mt][1][2], sacc[mt][1][3]);
        }
        // ---- O += P V ----
        {
            const int qm = lane >> 3, i8 = lane & 7;
            const int key = ((qm & 1) ? 8 : 0) + i8;
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {
                uint32_t b0a, b1a, b0b, b1b;
                ldsm_x4_t(vs_base + swz(key, 2 * dp + (qm >> 1)), b0a, b1a, b0b, b1b);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma16816(o[mt][2 * dp], pa[mt], b0a, b1a);
                    mma16816(o[mt][2 * dp + 1], pa[mt], b0b, b1b);
                }
            }
        }
        __syncwarp();
    }
    if (lane == 0) {  // after a failed wait: the copies still in flight land before the CTA exits
        for (int j = consumed; j < issued; ++j) mbar_wait_bounded(&full_bar[warp][j % kStages], (uint32_t)(j / kStages) & 1u);
    }
    __syncwarp();
    __syncthreads();

    // ---- merge the 4 warps: smem holds per-warp m, l and O (fp32) ----
    float *sm_o = reinterpret_cast<float *>(smem);                 // [kWarps][16*MT][128]
    float *sm_ml = sm_o + (size_t)kWarps * 16 * MT * kHD;          // [kWarps][16*MT][2]
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float l = lrow[mt][hh];
            l += __shfl_xor_sync(0xffffffffu, l, 1);
            l += __shfl_xor_sync(0xffffffffu, l, 2);
            const int rl = mt * 16 + r + hh * 8;
            if (c == 0) {
                sm_ml[((size_t)warp * 16 * MT + rl) * 2 + 0] = mrow[mt][hh];
                sm_ml[((size_t)warp * 16 * MT + rl) * 2 + 1] = l;
            }
#pragma unroll
            for (int nt = 0; nt < 16; ++nt) {
                float *dst = sm_o + ((size_t)warp * 16 * MT + rl) * kHD + nt * 8 + 2 * c;
                dst[0] = o[mt][nt][hh * 2 + 0];
                dst[1] = o[mt][nt][hh * 2 + 1];
            }
        }
    __syncthreads();
    const int rows_here = min(16 * MT, R - row_base);
    for (int e = threadIdx.x; e < rows_here * kHD; e += blockDim.x) {
        const int rl = e / kHD, d = e % kHD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_ml[((size_t)w * 16 * MT + rl) * 2]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float mw = sm_ml[((size_t)w * 16 * MT + rl) * 2];
            if (mw == -INFINITY) continue;
            const float f = expf(mw - M);
            L += sm_ml[((size_t)w * 16 * MT + rl) * 2 + 1] * f;
            O += sm_o[((size_t)w * 16 * MT + rl) * kHD + d] * f;
        }
        const int rho = row_base + rl;
        const int j = rho / p.gsz, g = rho % p.gsz;
        const int qrow = q0 + j, head = kvh * p.gsz + g;
        if (p.splits == 1) {
            float v = L > 0.f ? bf16_round(__fdiv_rn(O, L)) : 0.f;
            if (p.gate) {
                const float gt = bf2f(p.gate[(size_t)qrow * p.nh * kHD + (size_t)head * kHD + d]);
                const float sg = bf16_round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gt))));
                v = __fmul_rn(v, sg);
            }
            p.out[(size_t)qrow * p.nh * kHD + (size_t)head * kHD + d] = f2bf(v);
        } else {
            const size_t pidx = ((size_t)split * p.total_q + qrow) * p.nh + head;
            p.part_o[pidx * kHD + d] = O;
            if (d == 0) {
                p.part_ml[pidx * 2 + 0] = M;
                p.part_ml[pidx * 2 + 1] = L;
            }
        }
    }
}

// grid: (total_q * nh); block: 128 (one thread per dim)
__global__ void attn_merge(const AttnParams p) {
    pdl_entry();
    const int item = blockIdx.x;
    const int d = threadIdx.x;
    if (item >= p.total_q * p.nh) return;
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) {
        const size_t pidx = (size_t)s * p.total_q * p.nh + item;
        if (p.part_ml[pidx * 2 + 1] > 0.f) M = fmaxf(M, p.part_ml[pidx * 2]);
    }
    float L = 0.f, O = 0.f;
    for (int s = 0; s < p.splits; ++s) {
        const size_t pidx = (size_t)s * p.total_q * p.nh + item;
        const float l = p.part_ml[pidx * 2 + 1];
        if (!(l > 0.f)) continue;
        const float f = expf(p.part_ml[pidx * 2] - M);
        L += l * f;
        O += p.part_o[pidx * kHD + d] * f;
    }
    float v = L > 0.f ? bf16_round(__fdiv_rn(O, L)) : 0.f;
    if (p.gate) {
        const float gt = bf2f(p.gate[(size_t)item * kHD + d]);
        const float sg = bf16_round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gt))));
        v = __fmul_rn(v, sg);
    }
    p.out[(size_t)item * kHD + d] = f2bf(v);
}

// ---------------------------------------------------------------------------------
// Whole-page persistent attention.
//
// Reading one KV head at a time touches 256 of every 2048 bytes of a slot row (the other
// heads' bytes go to other CTAs), which holds a read-only stream near 5.9 TB/s on B200;
// reading whole pages (16 slots x all KV heads, 32 KB of K and 32 KB of V contiguous)
// reaches about 6.8 TB/s.  So here one CTA per SM takes a contiguous range of the batch's
// page list (every sequence's pages, in sequence order): a producer warp streams whole
// pages through a TMA ring, and consumer warp h computes KV head h's query rows against
// them with the same per-page math as attn_verify.  A sequence lying entirely inside one
// CTA's range is finished there; a sequence cut by range boundaries leaves one partial
// (m, l, O) per CTA (slot 0 if it is the CTA's first sequence, else slot 1), which
// attn_merge_pages combines in CTA order.  The ranges come from the context lengths on
// the device, so a captured launch stays valid as contexts grow.
// ---------------------------------------------------------------------------------
constexpr int kPMaxKv = 8;       // KV heads per CTA (one consumer warp each)
constexpr int kPStages = 3;      // pages in flight
constexpr int kPMaxSeqs = 1024;  // sequences per call (page prefix kept in shared memory)
constexpr int kPRec = kHD + 4;   // one cut-sequence record: O[128], m, l and two pad floats (16-byte rows)
constexpr int kMergeHeads = 4;   // heads per merge CTA (one warp each)

struct PageAttnParams {
    const __nv_bfloat16 *q;      // [total_q, nh, 128]
    const int32_t *block_table;  // [B, max_blocks]
    const int32_t *cu_q;         // [B+1]
    const int32_t *ctx;          // [B]
    const __nv_bfloat16 *gate;   // [total_q, nh*128] or null
    __nv_bfloat16 *out;          // [total_q, nh*128]
    float *part;                 // [G][2][max_q][nh][kPRec]: O, m, l
    int *err;                    // device error word
    int nh, nkv, gsz, max_blocks, num_blocks, B, max_q, G, total_q;
    float scale;
};

// CTA whose page range [c*T/G, (c+1)*T/G) holds page x
__device__ __forceinline__ int cta_of_page(long long x, long long T, int G) {
    int c = (int)((x * G) / T);
    if (c >= G) c = G - 1;
    while (c + 1 < G && ((long long)(c + 1) * T) / G <= x) ++c;
    while (c > 0 && ((long long)c * T) / G > x) --c;
    return c;
}

// byte offset of 16-byte chunk ch of key row `row` in one head's tile of a page stage:
// the tile's two 128-byte halves are hs bytes apart (SWIZZLE_128B, 1024-byte aligned)
__device__ __forceinline__ uint32_t pswz(int row, int ch, uint32_t hs) {
    return (uint32_t)((ch >> 3) * hs + row * 128 + (((ch & 7) ^ (row & 7)) << 4));
}

// grid: G (one CTA per SM); block: (nkv + 1) warps, warp nkv is the producer.  kmap / vmap:
// the caches as (dim, slot, head) tensors with 64 x 16 x nkv SWIZZLE_128B boxes.
template <int MT>
__global__ void __launch_bounds__((kPMaxKv + 1) * 32, 1) attn_pages(const __grid_constant__ CUtensorMap kmap,
                                                                    const __grid_constant__ CUtensorMap vmap,
                                                                    const PageAttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_prefix[kPMaxSeqs + 1];
    __shared__ __align__(8) uint64_t full_bar[kPStages], empty_bar[kPStages];
    __shared__ int s_blk_ok[kPStages];  // the stage's block id was valid (else zero its tiles)
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // the merge kernel may be scheduled now (programmatic dependent launch).  The page
    // prefix comes from the context lengths, which the host writes before the step, so it
    // is worked out before the wait for the previous kernel (which appends this step's
    // K/V and writes the queries).
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkv = p.nkv;
    const int cta = blockIdx.x;
    const uint32_t hs = (uint32_t)nkv * 2048;       // bytes of one 128-byte half for all heads
    const uint32_t stage_bytes = 4 * hs;             // K (2 halves) + V (2 halves)

    if (warp == 0) {  // page prefix over the sequences, 32 per pass
        int carry = 0;
        if (lane == 0) s_prefix[0] = 0;
        for (int b0 = 0; b0 < p.B; b0 += 32) {
            const int b = b0 + lane;
            int pages = 0;
            if (b < p.B) {
                const int cx = p.ctx[b];
                pages = cx > 0 ? (cx + 15) >> 4 : 0;
            }
            int incl = pages;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            if (b < p.B) s_prefix[b + 1] = carry + incl;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    if (threadIdx.x == 0) {
        for (int st = 0; st < kPStages; ++st) {
            mbar_init(&full_bar[st], 1);
            mbar_init(&empty_bar[st], (uint32_t)nkv);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const long long T = s_prefix[p.B];
    const long long s_c = ((long long)cta * T) / p.G, e_c = ((long long)(cta + 1) * T) / p.G;
    if (s_c >= e_c) return;
    pdl_wait();
    // largest b with prefix[b] <= x (sequences without pages are skipped)
    auto seq_of = [&](long long x) {
        int lo = 0, hi = p.B - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_prefix[mid] <= x) lo = mid; else hi = mid - 1;
        }
        return lo;
    };
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(smem);

    if (warp == nkv) {
        // ---- producer: whole pages (K and V of every KV head) into the ring.  The warp
        // fetches the block ids of 32 pages at once (one per lane); lane 0 issues. ----
        int b = seq_of(s_c);
        int issued = 0;
        bool stop = false;
        for (long long xb = s_c; xb < e_c && !stop; xb += 32) {
            const long long x = xb + lane;
            int blk = -1, bb = b;
            if (x < e_c) {
                while (x >= s_prefix[bb + 1]) ++bb;
                blk = p.block_table[(size_t)bb * p.max_blocks + (int)(x - s_prefix[bb])];
            }
            b = __shfl_sync(0xffffffffu, bb, 31);  // sequence of the chunk's last lane (>= any page issued)
            const int n = (int)min((long long)32, e_c - xb);
            for (int k = 0; k < n; ++k) {
                const int blk_k = __shfl_sync(0xffffffffu, blk, k);
                int ok = 1;
                if (lane == 0) {
                    const int st = issued % kPStages;
                    // stage st held page issued - kPStages: every consumer warp has released it
                    if (issued >= kPStages &&
                        !mbar_wait_bounded(&empty_bar[st], (uint32_t)((issued / kPStages) - 1) & 1u)) {
                        atomicExch(p.err, 1);
                        ok = 0;
                    } else {
                        const bool valid = blk_k >= 0 && blk_k < p.num_blocks;
                        const int blk_use = valid ? blk_k : 0;  // zeroed by the consumers
                        s_blk_ok[st] = valid ? 1 : 0;           // published by the arrive below
                        const uint32_t base = ring_s + (uint32_t)st * stage_bytes;
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        mbar_expect_tx(&full_bar[st], stage_bytes);
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {  // one box: half hf of the page, all heads
                            tma_load_3d(base + hf * hs, &kmap, &full_bar[st], 64 * hf, blk_use * 16, 0);
                            tma_load_3d(base + (2 + hf) * hs, &vmap, &full_bar[st], 64 * hf, blk_use * 16, 0);
                        }
                        ++issued;
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) {
                    stop = true;
                    break;
                }
            }
        }
        if (lane == 0)  // every copy issued has landed before the CTA may exit
            for (int j = issued > kPStages ? issued - kPStages : 0; j < issued; ++j)
                mbar_wait_bounded(&full_bar[j % kPStages], (uint32_t)(j / kPStages) & 1u);
        __syncwarp();
        return;
    }

    // ---- consumer warp h: query rows of KV head h against every page of the range ----
    const int h = warp;
    const int r = lane >> 2, c = lane & 3;
    int b = seq_of(s_c);
    long long x = s_c;
    int i = 0;  // pages consumed by this warp
    while (x < e_c) {
        while (x >= s_prefix[b + 1]) ++b;
        const long long seg0 = x, seg1 = min(e_c, (long long)s_prefix[b + 1]);
        const bool whole = seg0 == s_prefix[b] && seg1 == s_prefix[b + 1];
        const int slot = seg0 == s_c ? 0 : 1;
        const int q0 = p.cu_q[b], q_len = p.cu_q[b + 1] - q0, ctx = p.ctx[b];
        const int R = q_len * p.gsz;
        const bool active = q_len > 0 && R <= 16 * MT;
        const int p0 = ctx - q_len;

        uint32_t qf[MT][8][4];
        int qpos[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int rho = mt * 16 + r + hh * 8;
                const bool ok = active && rho < R;
                const int j = ok ? rho / p.gsz : 0, g = ok ? rho % p.gsz : 0;
                qpos[mt][hh] = ok ? p0 + j : -1;
                const __nv_bfloat16 *qrow = p.q + ((size_t)(q0 + j) * p.nh + (size_t)h * p.gsz + g) * kHD;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    qf[mt][ks][hh] = ok ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 2 * c) : 0u;
                    qf[mt][ks][2 + hh] = ok ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 8 + 2 * c) : 0u;
                }
            }
        float o[MT][16][4];
        float mrow[MT][2], lrow[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) o[mt][nt][j] = 0.f;
            mrow[mt][0] = mrow[mt][1] = -INFINITY;
            lrow[mt][0] = lrow[mt][1] = 0.f;
        }

        bool failed = false;
        for (; x < seg1; ++x, ++i) {
            const int st = i % kPStages;
            const bool landed = mbar_wait_bounded(&full_bar[st], (uint32_t)(i / kPStages) & 1u);
            if (!__all_sync(0xffffffffu, landed)) {
                if (lane == 0) atomicExch(p.err, 1);
                failed = true;
                break;
            }
            const int pg = (int)(x - s_prefix[b]);
            uint8_t *kp = smem + (size_t)st * stage_bytes + h * 2048;
            uint8_t *vp = kp + 2 * hs;
            {
                // keys past the context get P = 0, so their V rows must be finite: zero them
                // (and this head's whole page for an invalid block id, whose K then scores 0)
                const bool blk_ok = s_blk_ok[st] != 0;
                const int valid = min(16, ctx - pg * 16);
                if (!blk_ok || valid < 16) {
                    const int r0 = blk_ok ? valid : 0;
                    for (int idx = lane; idx < (16 - r0) * 16; idx += 32) {
                        const int row = r0 + (idx >> 4), ch = idx & 15;
                        const size_t off = (size_t)(ch >> 3) * hs + row * 128 + ((ch & 7) << 4);
                        *reinterpret_cast<uint4 *>(vp + off) = make_uint4(0u, 0u, 0u, 0u);
                        if (!blk_ok) *reinterpret_cast<uint4 *>(kp + off) = make_uint4(0u, 0u, 0u, 0u);
                    }
                    __syncwarp();
                }
            }
            if (active) {
                const uint32_t ks_base = (uint32_t)__cvta_generic_to_shared(kp);
                const uint32_t vs_base = (uint32_t)__cvta_generic_to_shared(vp);
                float sacc[MT][2][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int j = 0; j < 4; ++j) sacc[mt][nt][j] = 0.f;
                {
                    const int qm = lane >> 3, i8 = lane & 7;
                    const int key = (qm >= 2 ? 8 : 0) + i8;
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        uint32_t b00, b01, b10, b11;
                        ldsm_x4(ks_base + pswz(key, 2 * ks + (qm & 1), hs), b00, b01, b10, b11);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            mma16816(sacc[mt][0], qf[mt][ks], b00, b01);
                            mma16816(sacc[mt][1], qf[mt][ks], b10, b11);
                        }
                    }
                }
                uint32_t pa[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        float mx = -INFINITY;
#pragma unroll
                        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int kpos = pg * 16 + nt * 8 + 2 * c + e;
                                float sv = sacc[mt][nt][hh * 2 + e];
                                // scores = bmm(q, k^T) in bf16, then * scale in bf16 (attention.py:128-129)
                                sv = bf16_round(__fmul_rn(bf16_round(sv), p.scale));
                                if (kpos > qpos[mt][hh] || kpos >= ctx) sv = -INFINITY;
                                sacc[mt][nt][hh * 2 + e] = sv;
                                mx = fmaxf(mx, sv);
                            }
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                        const float mnew = fmaxf(mrow[mt][hh], mx);
                        const float alpha = (mnew == -INFINITY) ? 1.f : expf(mrow[mt][hh] - mnew);
                        mrow[mt][hh] = mnew;
                        float ls = 0.f;
#pragma unroll
                        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const float sv = sacc[mt][nt][hh * 2 + e];
                                const float pv = (sv == -INFINITY) ? 0.f : expf(sv - mnew);
                                sacc[mt][nt][hh * 2 + e] = pv;
                                ls += pv;
                            }
                        lrow[mt][hh] = lrow[mt][hh] * alpha + ls;
                        // once the running maxima settle, alpha is exactly 1 for every row:
                        // skip the multiplies (a product by 1 is exact)
                        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                            for (int nt = 0; nt < 16; ++nt) {
                                o[mt][nt][hh * 2 + 0] *= alpha;
                                o[mt][nt][hh * 2 + 1] *= alpha;
                            }
                        }
                    }
                    pa[mt][0] = pack_bf16(sacc[mt][0][0], sacc[mt][0][1]);
                    pa[mt][1] = pack_bf16(sacc[mt][0][2], sacc[mt][0][3]);
                    pa[mt][2] = pack_bf16(sacc[mt][1][0], sacc[mt][1][1]);
                    pa[mt][3] = pack_bf16(sacc[mt][1][2], sacc[mt][1][3]);
                }
                {
                    const int qm = lane >> 3, i8 = lane & 7;
                    const int key = ((qm & 1) ? 8 : 0) + i8;
#pragma unroll
                    for (int dp = 0; dp < 8; ++dp) {
                        uint32_t b0a, b1a, b0b, b1b;
                        ldsm_x4_t(vs_base + pswz(key, 2 * dp + (qm >> 1), hs), b0a, b1a, b0b, b1b);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            mma16816(o[mt][2 * dp], pa[mt], b0a, b1a);
                            mma16816(o[mt][2 * dp + 1], pa[mt], b0b, b1b);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[st]);  // this warp is done with the stage
        }
        if (failed) break;
        if (!active) continue;

        // ---- finish the segment: the final output, or this CTA's partial ----
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float l = lrow[mt][hh];
                l += __shfl_xor_sync(0xffffffffu, l, 1);
                l += __shfl_xor_sync(0xffffffffu, l, 2);
                const int rho = mt * 16 + r + hh * 8;
                if (rho >= R) continue;
                const int j = rho / p.gsz, g = rho % p.gsz;
                const int qrow = q0 + j, head = h * p.gsz + g;
                if (whole) {
                    const size_t ob = (size_t)qrow * p.nh * kHD + (size_t)head * kHD;
#pragma unroll
                    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int d = nt * 8 + 2 * c + e;
                            float v = l > 0.f ? bf16_round(__fdiv_rn(o[mt][nt][hh * 2 + e], l)) : 0.f;
                            if (p.gate) {
                                const float gt = bf2f(p.gate[ob + d]);
                                const float sg = bf16_round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gt))));
                                v = __fmul_rn(v, sg);
                            }
                            p.out[ob + d] = f2bf(v);
                        }
                } else {
                    float *rec = p.part + ((((size_t)cta * 2 + slot) * p.max_q + j) * p.nh + head) * kPRec;
#pragma unroll
                    for (int nt = 0; nt < 16; ++nt) {
                        rec[nt * 8 + 2 * c] = o[mt][nt][hh * 2 + 0];
                        rec[nt * 8 + 2 * c + 1] = o[mt][nt][hh * 2 + 1];
                    }
                    if (c == 0) {
                        rec[kHD] = mrow[mt][hh];
                        rec[kHD + 1] = l;
                    }
                }
            }
    }
}

// grid: (ceil(nh / 4), max_q, B); block: 128.  Warp w combines, in CTA order, the pieces
// that CTA range boundaries cut from head 4 * blockIdx.x + w of row j of sequence b; lane l
// takes dims 4l .. 4l + 3.  A sequence one CTA holds whole was written by that CTA.  The
// page ranges come from the context lengths, which the page kernel does not write, so they
// are worked out before the programmatic-dependent wait: once attn_pages completes, one
// round of independent loads remains (every piece's m, l and four O values).
__global__ void __launch_bounds__(kMergeHeads * 32) attn_merge_pages(const PageAttnParams p) {
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x * kMergeHeads + warp, j = blockIdx.y, b = blockIdx.z;
    const int q0 = p.cu_q[b], q1 = p.cu_q[b + 1];
    // pages before sequence b (P0), of sequence b and in total (T): the page kernel's prefix
    long long P0 = 0, T = 0;
    for (int i0 = 0; i0 < p.B; i0 += 32) {
        const int i = i0 + lane;
        int pg = 0;
        if (i < p.B) {
            const int cx = p.ctx[i];
            pg = cx > 0 ? (cx + 15) >> 4 : 0;
        }
        T += __reduce_add_sync(0xffffffffu, (unsigned)pg);
        P0 += __reduce_add_sync(0xffffffffu, (unsigned)(i < b ? pg : 0));
    }
    const int cxb = p.ctx[b];
    const long long P1 = P0 + (cxb > 0 ? (cxb + 15) >> 4 : 0);
    if (head >= p.nh || j >= q1 - q0 || P1 <= P0 || T <= 0) return;
    // The range bounds c T / G are 64-bit divisions: lanes work them out in parallel and
    // share them, instead of every lane repeating all of them (they dominated the kernel's
    // instructions).  Lane 0 finds the first CTA, lane 1 the last.
    const int cl = cta_of_page(lane == 0 ? P0 : P1 - 1, T, p.G);
    const int c0 = __shfl_sync(0xffffffffu, cl, 0), c1 = __shfl_sync(0xffffffffu, cl, 1);
    if (c0 == c1) return;  // finished by its CTA
    const size_t ob = (size_t)(q0 + j) * p.nh * kHD + (size_t)head * kHD + 4 * lane;
    pdl_wait();
    // CTA c's record for this sequence: slot 0 if the sequence starts inside c's range,
    // slot 1 if it runs on from before; CTAs with an empty range (more CTAs than pages)
    // wrote nothing and are skipped
    constexpr int U = 8;
    float M = -INFINITY, L = 0.f, O[4] = {0.f, 0.f, 0.f, 0.f};
    for (int cb = c0; cb <= c1; cb += U) {
        // lane u < U: the page range [lo, hi) of CTA cb + u
        long long lo_l = 0, hi_l = 0;
        if (lane < U) {
            lo_l = ((long long)(cb + lane) * T) / p.G;
            hi_l = ((long long)(cb + lane + 1) * T) / p.G;
        }
        float m[U], l[U];
        float4 o[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            m[u] = -INFINITY;
            l[u] = 0.f;
            o[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            const int c = cb + u;
            const long long lo = __shfl_sync(0xffffffffu, lo_l, u), hi = __shfl_sync(0xffffffffu, hi_l, u);
            if (c <= c1 && lo < hi) {
                const float *rec =
                    p.part + ((((size_t)c * 2 + (lo >= P0 ? 0 : 1)) * p.max_q + j) * p.nh + head) * kPRec;
                m[u] = __ldcg(rec + kHD);
                l[u] = __ldcg(rec + kHD + 1);
                o[u] = __ldcg(reinterpret_cast<const float4 *>(rec + 4 * lane));
            }
        }
        float mc = M;
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (l[u] > 0.f) mc = fmaxf(mc, m[u]);
        if (mc == -INFINITY) continue;
        if (mc > M && L > 0.f) {  // only when the pieces exceed one chunk of U
            const float f = expf(M - mc);
            L *= f;
#pragma unroll
            for (int e = 0; e < 4; ++e) O[e] *= f;
        }
        M = mc;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (!(l[u] > 0.f)) continue;
            const float f = expf(m[u] - M);
            L += l[u] * f;
            O[0] += o[u].x * f;
            O[1] += o[u].y * f;
            O[2] += o[u].z * f;
            O[3] += o[u].w * f;
        }
    }
    __align__(8) __nv_bfloat16 outv[4];
    uint2 gbits = make_uint2(0u, 0u);
    if (p.gate) gbits = *reinterpret_cast<const uint2 *>(p.gate + ob);
    const __nv_bfloat16 *gv = reinterpret_cast<const __nv_bfloat16 *>(&gbits);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float v = L > 0.f ? bf16_round(__fdiv_rn(O[e], L)) : 0.f;
        if (p.gate) {
            const float sg = bf16_round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-bf2f(gv[e])))));
            v = __fmul_rn(v, sg);
        }
        outv[e] = f2bf(v);
    }
    *reinterpret_cast<uint2 *>(p.out + ob) = *reinterpret_cast<const uint2 *>(outv);
}

// Clear the split partials of every (row, head) so that CTAs which exit early (no
// rows or no visible pages in their split) leave an empty record (l = 0).
__global__ void attn_clear_ml(float *ml, size_t n) {
    pdl_entry();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        ml[i] = (i & 1) ? 0.f : -INFINITY;
}

// K/V cache [num_blocks * 16 slots, n_kv, 128] bf16 as a 3-D tensor (dim, head, slot);
// one box is 64 dims x 1 head x 16 slots (a 128-byte SWIZZLE_128B half of one head's page)
int encode_kv_maps(const __nv_bfloat16 *kc, const __nv_bfloat16 *vc, int nkv, int num_blocks, CUtensorMap (&maps)[2],
                   const char *what) {
    TensorMapEncodeTiledFn enc = tensor_map_encoder();
    PILM_REQUIRE(enc, ECPU_ERR_UNSUPPORTED, "%s: cuTensorMapEncodeTiled is unavailable", what);
    PILM_REQUIRE((((uintptr_t)kc) & 15) == 0 && (((uintptr_t)vc) & 15) == 0, ECPU_ERR_PARAM,
                 "%s: the K and V caches must be 16-byte aligned", what);
    const __nv_bfloat16 *src[2] = {kc, vc};
    for (int i = 0; i < 2; ++i) {
        cuuint64_t dims[3] = {(cuuint64_t)kHD, (cuuint64_t)nkv, (cuuint64_t)num_blocks * 16};
        cuuint64_t strides[2] = {(cuuint64_t)kHD * 2, (cuuint64_t)nkv * kHD * 2};
        cuuint32_t box[3] = {64, 1, 16};
        cuuint32_t es[3] = {1, 1, 1};
        const CUresult r = enc(&maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void *)src[i], dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        PILM_REQUIRE(r == CUDA_SUCCESS, ECPU_ERR_PARAM, "%s: the K/V cache tensor map was rejected (error %d)", what,
                     (int)r);
    }
    return ECPU_OK;
}

// K/V cache as a 3-D tensor (dim, slot, head): one box of 64 dims x 16 slots x all heads
// is a 128-byte half of a whole page, landing as [head][slot][128 B] (each head's 16 rows
// a 2 KB, 1024-byte aligned SWIZZLE_128B block).  Four boxes load a page's K and V.
int encode_kv_page_maps(const __nv_bfloat16 *kc, const __nv_bfloat16 *vc, int nkv, int num_blocks,
                        CUtensorMap (&maps)[2], const char *what) {
    TensorMapEncodeTiledFn enc = tensor_map_encoder();
    PILM_REQUIRE(enc, ECPU_ERR_UNSUPPORTED, "%s: cuTensorMapEncodeTiled is unavailable", what);
    PILM_REQUIRE((((uintptr_t)kc) & 15) == 0 && (((uintptr_t)vc) & 15) == 0, ECPU_ERR_PARAM,
                 "%s: the K and V caches must be 16-byte aligned", what);
    const __nv_bfloat16 *src[2] = {kc, vc};
    for (int i = 0; i < 2; ++i) {
        cuuint64_t dims[3] = {(cuuint64_t)kHD, (cuuint64_t)num_blocks * 16, (cuuint64_t)nkv};
        cuuint64_t strides[2] = {(cuuint64_t)nkv * kHD * 2, (cuuint64_t)kHD * 2};
        cuuint32_t box[3] = {64, 16, (cuuint32_t)nkv};
        cuuint32_t es[3] = {1, 1, 1};
        const CUresult r = enc(&maps[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void *)src[i], dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        PILM_REQUIRE(r == CUDA_SUCCESS, ECPU_ERR_PARAM, "%s: the K/V page tensor map was rejected (error %d)", what,
                     (int)r);
    }
    return ECPU_OK;
}

// ---------------------------------------------------------------------------------
// Prefill-sized passes on 5th-generation tensor cores (tcgen05 + TMEM): flash attention
// over the paged cache for 128 query rows per CTA.
//
// A CTA owns one KV head and 128 / gsz consecutive query positions of one sequence, so its
// 128 rows are (position, query head of the group) pairs, row r = position * gsz + head.
// TMA loads the Q tile once (two 64-dim SWIZZLE_128B halves), and the K and V blocks of 128
// keys (8 pages, 16 boxes each) into two two-stage rings: a K stage is free again once the
// scores that read it are done, a V stage once the P V product is, so K runs ahead of V.
// Per KV block j:
//   S(j) = Q K(j)^T      8 x tcgen05.mma M=128 N=128 K=16, both operands K-major in shared
//                        memory, into one of two TMEM score buffers
//   softmax (8 warps)    two threads per row, each 64 keys: the scores rounded as the
//                        reference's bf16 bmm and scale are, the causal / context mask, the
//                        running max (shared by the pair) and sum; P = exp(S - max) as bf16
//                        into one of two TMEM P buffers, and O rescaled in TMEM when a
//                        row's max moved
//   O += P(j) V(j)       8 x tcgen05.mma M=128 N=128 K=16, A = P from TMEM, B = V as it lies
//                        in the cache (keys x dims, an MN-major SWIZZLE_128B operand)
// S(j + 1) is issued before PV(j), so the tensor pipe works on the next block while the
// softmax warps work on this one.  The causal and context masks are those of the other
// attention kernels (a key is seen by a row iff key <= the row's position and key <
// context), so the results agree with them up to fp32 summation order.
// Warps: 0 TMA producer of Q and K, 2 of V, 1 TMEM owner and MMA issuer (its lanes also zero
// the V rows past the context, and K and V of pages with an invalid block id), 4-11 softmax
// and epilogue,
// two per TMEM lane quadrant (one half of the keys of each block, one half of O's dims).
// Every mbarrier wait is bounded; a wait that gives up sets the device error word.
// ---------------------------------------------------------------------------------
constexpr int kPfRows = 128;                   // query rows per CTA (MMA M)
constexpr int kPfKeys = 128;                   // keys per KV block
constexpr int kPfHalf = kPfKeys * 128;         // one 64-dim half of a K or V block: 16 KB
constexpr int kPfKV = 2 * kPfHalf;             // K (or V) block: 32 KB
constexpr int kPfQ = kPfRows * kHD * 2;        // Q tile: 32 KB
constexpr int kPfThreads = 12 * 32;  // Q/K producer, issuer, V producer, one idle, 8 softmax
constexpr int kPfTmemCols = 512;               // S0 [0,128) S1 [128,256) O [256,384) P0 [384,448) P1 [448,512)
constexpr int kPfStages = 2;                 // K blocks in flight, and V blocks
constexpr size_t kPfSmemK = kPfQ;                                  // K ring
constexpr size_t kPfSmemV = kPfSmemK + kPfStages * (size_t)kPfKV;  // V ring
constexpr size_t kPfSmemBar = kPfSmemV + kPfStages * (size_t)kPfKV;
struct __align__(8) PfBars {
    uint64_t q_full, k_full[kPfStages], k_empty[kPfStages], v_full[kPfStages], v_empty[kPfStages];
    uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], drain;
    uint64_t pair_max[4][2], pair_sum[4];  // the two softmax warps of a lane quadrant: row maxima, row sums
    uint32_t tmem_base;
    int abort_flag;
};
constexpr size_t kPfSmemTotal = kPfSmemBar + sizeof(PfBars) + 1024;
static_assert(kPfSmemTotal <= 227 * 1024, "shared memory budget");

struct PfParams {
    const int32_t *block_table;  // [B, max_blocks]
    const int32_t *cu_q;         // [B+1]
    const int32_t *ctx;          // [B]
    const __nv_bfloat16 *gate;   // [total_q, nh*128] or null
    __nv_bfloat16 *out;          // [total_q, nh*128]
    int *err;
    int nh, gsz, ppt, tiles, max_blocks, num_blocks;
    float scale;
};

__device__ __forceinline__ uint32_t pf_s32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
// two floats rounded to bf16 (nearest even) by one conversion, returned as floats
__device__ __forceinline__ float2 bf16x2_round(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return __bfloat1622float2(h);
}

__device__ __forceinline__ void pf_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void pf_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void pf_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(pf_s32(bar))
                 : "memory");
}
// K-major SWIZZLE_128B operand: 8-row x 128-byte atoms, 1024 bytes between 8-row groups
__device__ __forceinline__ uint64_t pf_kdesc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major SWIZZLE_128B operand (V: key rows of 64 contiguous dims): 1024 bytes between
// 8-key groups (stride byte offset), kPfHalf bytes between the two 64-dim halves (leading
// byte offset)
__device__ __forceinline__ uint64_t pf_mndesc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)(kPfHalf >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void pf_mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void pf_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void pf_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void pf_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void pf_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void pf_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// bounded wait shared by a warp: every lane waits, the warp reconverges, a timeout in any
// lane (or an abort raised elsewhere) ends it for all
__device__ __forceinline__ bool pf_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag) {
    bool ok = false;
    for (uint32_t i = 0; i < kAttnWaitLimit; ++i) {
        if (mbar_try_wait(b, parity)) {
            ok = true;
            break;
        }
        if ((i & 255) == 255 && *abort_flag) break;
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) *abort_flag = 1;
    return ok;
}

// grid: (sequences x tiles, n_kv); block: 256.  qmap: q as (dim, head, row) with 64 x gsz x
// ppt boxes; kmap / vmap: the caches as (dim, head, slot) with 64 x 1 x 16 boxes.
__global__ void __launch_bounds__(kPfThreads, 1) attn_prefill_tc(const __grid_constant__ CUtensorMap qmap,
                                                                 const __grid_constant__ CUtensorMap kmap,
                                                                 const __grid_constant__ CUtensorMap vmap,
                                                                 const PfParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t s_inv[2][kPfStages];  // [K, V][stage]: pages inside the context with an invalid block id
    __shared__ float s_pmax[2][2][kPfRows];  // [block parity][key half][row]: partial row maxima
    __shared__ float s_psum[2][kPfRows];     // [key half][row]: partial row sums
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    PfBars *bar = reinterpret_cast<PfBars *>(smem + kPfSmemBar);
    volatile int *abort_flag = &bar->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    // the tile: heaviest (last positions, most keys) first.  cu_q and the context lengths
    // are host-written before the step, so they are read before the wait.
    const int b = blockIdx.x / p.tiles, t = p.tiles - 1 - blockIdx.x % p.tiles;
    const int kvh = blockIdx.y;
    const int q0 = p.cu_q[b], q_len = p.cu_q[b + 1] - q0, ctx = p.ctx[b];
    const int pos0 = t * p.ppt;
    if (pos0 >= q_len) return;
    const int p0 = ctx - q_len;                          // position of the sequence's first query row
    const int kmax = min(ctx, p0 + pos0 + p.ppt);        // keys that any row of the tile sees
    const int nb = (kmax + kPfKeys - 1) / kPfKeys;
    const int ctx_pages = (ctx + 15) >> 4;
    const int32_t *bt = p.block_table + (size_t)b * p.max_blocks;
    if (threadIdx.x == 0) {
        mbar_init(&bar->q_full, 1);
        for (int i = 0; i < kPfStages; ++i) {
            mbar_init(&bar->k_full[i], 1);
            mbar_init(&bar->k_empty[i], 1);
            mbar_init(&bar->v_full[i], 1);
            mbar_init(&bar->v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar->s_full[i], 1);
            mbar_init(&bar->s_free[i], 8);
            mbar_init(&bar->p_full[i], 8);
            mbar_init(&bar->pv_done[i], 1);
        }
        mbar_init(&bar->drain, 1);
        for (int q = 0; q < 4; ++q) {
            mbar_init(&bar->pair_max[q][0], 64);
            mbar_init(&bar->pair_max[q][1], 64);
            mbar_init(&bar->pair_sum[q], 64);
        }
        bar->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(pf_s32(&bar->tmem_base)),
                     "r"(kPfTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pf_fence_before();
    __syncthreads();
    pf_fence_after();
    const uint32_t tmem = bar->tmem_base;
    pdl_wait();

    if (warp == 0 || warp == 2) {
        // ---- producers: warp 0 Q once and the K blocks, warp 2 the V blocks, each block's 8
        // pages into a two-stage ring ----
        const bool is_k = warp == 0;
        const CUtensorMap *map = is_k ? &kmap : &vmap;
        uint64_t *full = is_k ? bar->k_full : bar->v_full;
        uint64_t *empty = is_k ? bar->k_empty : bar->v_empty;
        int issued = 0;
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
            if (is_k) {
                asm volatile("prefetch.tensormap [%0];" ::"l"(&qmap) : "memory");
                mbar_expect_tx(&bar->q_full, kPfQ);
                for (int h = 0; h < 2; ++h)
                    tma_load_3d(pf_s32(smem) + h * (kPfQ / 2), &qmap, &bar->q_full, 64 * h, kvh * p.gsz, q0 + pos0);
            }
        }
        for (int j = 0; j < nb; ++j) {
            const int st = j % kPfStages;
            // block ids of the block's 8 pages, one per lane (invalid ones load page 0,
            // which the issuer warp zeroes)
            int blk = 0;
            bool inv = false;  // a page inside the context whose block id is out of range
            if (lane < 8) {
                const int pg = 8 * j + lane;
                if (pg < ctx_pages) {
                    blk = pg < p.max_blocks ? bt[pg] : -1;
                    inv = blk < 0 || blk >= p.num_blocks;
                }
                if (inv) blk = 0;
            }
            const uint32_t inv_mask = __ballot_sync(0xffffffffu, inv);
            if (j >= kPfStages && !pf_wait(&empty[st], (uint32_t)((j - kPfStages) / kPfStages) & 1u, abort_flag)) break;
            const uint32_t base = pf_s32(smem + (is_k ? kPfSmemK : kPfSmemV)) + (uint32_t)st * kPfKV;
            int blks[8];
#pragma unroll
            for (int pg = 0; pg < 8; ++pg) blks[pg] = __shfl_sync(0xffffffffu, blk, pg);
            if (lane == 0) {
                s_inv[is_k ? 0 : 1][st] = inv_mask;  // published by the arrive below
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect_tx(&full[st], kPfKV);
#pragma unroll
                for (int pg = 0; pg < 8; ++pg)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        tma_load_3d(base + (uint32_t)(h * kPfHalf + pg * 2048), map, &full[st], 64 * h, kvh, blks[pg] * 16);
            }
            ++issued;
        }
        // drain: every copy issued has landed before the CTA may exit
        if (lane == 0) {
            if (is_k) mbar_wait_bounded(&bar->q_full, 0);
            for (int j = issued > kPfStages ? issued - kPfStages : 0; j < issued; ++j)
                mbar_wait_bounded(&full[j % kPfStages], (uint32_t)(j / kPfStages) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer (lane 0); the warp zeroes what must not reach the MMAs ----
        const uint32_t idesc_s = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPfKeys >> 3) << 17) |
                                 ((uint32_t)(kPfRows >> 4) << 24);
        const uint32_t idesc_pv = idesc_s | (1u << 16);  // B (V) MN-major; N = 128 dims
        const uint32_t q_s = pf_s32(smem);
        // the rows of a stage that must not reach the MMAs: rows of keys past the context
        // (V only: their P is 0, but 0 x NaN is NaN) and whole pages with an invalid block id
        auto zero_rows = [&](uint8_t *stage, int j, uint32_t inv_mask, bool is_v) {
            const int key0 = j * kPfKeys;
            if (!(is_v && key0 + kPfKeys > ctx) && !inv_mask) return;
            for (int pg = 0; pg < 8; ++pg) {
                const int k16 = key0 + pg * 16;
                const bool invalid = (inv_mask >> pg) & 1u;
                const int r0 = invalid ? 0 : (is_v ? max(0, min(16, ctx - k16)) : 16);
                if (r0 >= 16) continue;
                for (int idx = lane; idx < (16 - r0) * 16; idx += 32) {  // 16-byte chunks, both halves
                    const int row = pg * 16 + r0 + (idx >> 4), ch = idx & 15;
                    const size_t off = (size_t)(ch >> 3) * kPfHalf + (size_t)row * 128 + ((ch & 7) << 4);
                    *reinterpret_cast<uint4 *>(stage + off) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        };
        auto issue_s = [&](int j) -> bool {
            const int st = j % kPfStages, sb = j & 1;  // K stage, S buffer
            if (j == 0 && !pf_wait(&bar->q_full, 0, abort_flag)) return false;
            if (!pf_wait(&bar->k_full[st], (uint32_t)(j / kPfStages) & 1u, abort_flag)) return false;
            if (j >= 2 && !pf_wait(&bar->s_free[sb], (uint32_t)((j - 2) >> 1) & 1u, abort_flag)) return false;
            uint8_t *kst = smem + kPfSmemK + (size_t)st * kPfKV;
            zero_rows(kst, j, s_inv[0][st], false);
            pf_fence_after();
            if (lane == 0) {
                const uint32_t k_s = pf_s32(kst);
                const uint32_t d = tmem + (uint32_t)(sb * 128);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {  // K = 16 dims per MMA: 32 bytes of each 128-byte row
                    const uint32_t off = (uint32_t)((ks >> 2) * (kPfQ / 2));
                    pf_mma_ss(d, pf_kdesc(q_s + off) + 2 * (ks & 3), pf_kdesc(k_s + (uint32_t)((ks >> 2) * kPfHalf)) + 2 * (ks & 3),
                              idesc_s, ks > 0 ? 1u : 0u);
                }
                pf_commit(&bar->s_full[sb]);
                pf_commit(&bar->k_empty[st]);
            }
            __syncwarp();
            return true;
        };
        bool ok = issue_s(0);
        for (int j = 0; ok && j < nb; ++j) {
            const int st = j % kPfStages, sb = j & 1;  // V stage, P buffer
            if (j + 1 < nb && !issue_s(j + 1)) break;
            if (!pf_wait(&bar->v_full[st], (uint32_t)(j / kPfStages) & 1u, abort_flag)) break;
            uint8_t *vst = smem + kPfSmemV + (size_t)st * kPfKV;
            zero_rows(vst, j, s_inv[1][st], true);
            if (!pf_wait(&bar->p_full[sb], (uint32_t)(j >> 1) & 1u, abort_flag)) break;
            pf_fence_after();
            if (lane == 0) {
                const uint32_t v_s = pf_s32(vst);
                const uint32_t pa = tmem + (uint32_t)(384 + sb * 64);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)  // K = 16 keys per MMA: 8 TMEM columns of P, 16 key rows of V
                    pf_mma_ts(tmem + 256u, pa + (uint32_t)(8 * ks), pf_mndesc(v_s + (uint32_t)(ks * 2048)), idesc_pv,
                              (j > 0 || ks > 0) ? 1u : 0u);
                pf_commit(&bar->pv_done[sb]);
                pf_commit(&bar->v_empty[st]);
            }
            __syncwarp();
        }
        if (lane == 0) {
            pf_commit(&bar->drain);
            mbar_wait_bounded(&bar->drain, 0);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---- softmax and epilogue: two warps per row quadrant, each one half of the keys of
        // a block (64 columns of S, 32 of P) and one half of the dims of O; the row maxima
        // and, at the end, the row sums are exchanged through shared memory ----
        const int q4 = warp & 3, half = (warp - 4) >> 2;
        const int r = 32 * q4 + lane;
        const uint32_t lane_addr = (uint32_t)(32 * q4) << 16;
        const int pos = r / p.gsz, g = r % p.gsz;
        const int qp = p0 + pos0 + pos;                  // this row's position (its last key)
        const int qp_min = p0 + pos0;                    // the tile's first position
        const bool row_ok = pos0 + pos < q_len;
        // a quadrant whose 32 rows are all past the sequence's queries (short passes: 20 rows
        // of a 128-row tile at q_len 5 with 4 query heads per KV head) skips the softmax; it
        // still takes each block's s_full before its arrivals, so the barriers keep phase
        const bool skip = __all_sync(0xffffffffu, !row_ok);
        float m = -INFINITY, l = 0.f;
        bool failed = false;
        for (int j = 0; j < nb; ++j) {
            const int st = j & 1;
            if (!pf_wait(&bar->s_full[st], (uint32_t)(j >> 1) & 1u, abort_flag)) {
                failed = true;
                break;
            }
            if (skip) {
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&bar->s_free[st]);
                    mbar_arrive(&bar->p_full[st]);
                }
                continue;
            }
            pf_fence_after();
            float s[64];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t u[32];
                pf_ld32(tmem + lane_addr + (uint32_t)(st * 128 + 64 * half + 32 * c), u);
                pf_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e) s[32 * c + e] = __uint_as_float(u[e]);
            }
            pf_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->s_free[st]);
            // scores = bmm(q, k^T) in bf16, then * scale in bf16 (attention.py:128-129); a
            // block whose keys every row of the tile sees needs no mask
            const int k0 = j * kPfKeys + 64 * half;
            const bool masked = (j + 1) * kPfKeys - 1 > qp_min || (j + 1) * kPfKeys > ctx;
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < 64; c += 2) {
                // two scores per bf16x2 conversion (each rounded to nearest even, as alone)
                float2 v = bf16x2_round(s[c], s[c + 1]);
                v = bf16x2_round(__fmul_rn(v.x, p.scale), __fmul_rn(v.y, p.scale));
                if (masked) {
                    if (k0 + c > qp || k0 + c >= ctx) v.x = -INFINITY;
                    if (k0 + c + 1 > qp || k0 + c + 1 >= ctx) v.y = -INFINITY;
                }
                s[c] = v.x;
                s[c + 1] = v.y;
                mx4[c & 3] = fmaxf(mx4[c & 3], v.x);
                mx4[(c + 1) & 3] = fmaxf(mx4[(c + 1) & 3], v.y);
            }
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            s_pmax[st][half][r] = mx;
            mbar_arrive(&bar->pair_max[q4][st]);  // every lane: each publishes its own row's value
            if (!pf_wait(&bar->pair_max[q4][st], (uint32_t)(j >> 1) & 1u, abort_flag)) {
                failed = true;
                break;
            }
            const float mnew = fmaxf(m, fmaxf(mx, s_pmax[st][half ^ 1][r]));
            const float alpha = (m == -INFINITY || mnew == -INFINITY) ? 1.f : __expf(m - mnew);
            // PV(j - 1) has completed: O holds blocks < j, and P buffer st (PV(j - 2)) is free
            if (j >= 1 && !pf_wait(&bar->pv_done[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, abort_flag)) {
                failed = true;
                break;
            }
            pf_fence_after();
            if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t u[32];
                    pf_ld32(tmem + lane_addr + (uint32_t)(256 + 64 * half + 32 * c), u);
                    pf_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
                    pf_st32(tmem + lane_addr + (uint32_t)(256 + 64 * half + 32 * c), u);
                }
            }
            float ls4[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t u[32];
            if (masked) {
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float a0 = s[2 * e], a1 = s[2 * e + 1];
                    const float p0v = (a0 == -INFINITY) ? 0.f : __expf(a0 - mnew);
                    const float p1v = (a1 == -INFINITY) ? 0.f : __expf(a1 - mnew);
                    ls4[e & 3] += p0v + p1v;
                    u[e] = pack_bf16(p0v, p1v);
                }
            } else {  // every score finite: no -inf tests
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float p0v = __expf(s[2 * e] - mnew), p1v = __expf(s[2 * e + 1] - mnew);
                    ls4[e & 3] += p0v + p1v;
                    u[e] = pack_bf16(p0v, p1v);
                }
            }
            pf_st32(tmem + lane_addr + (uint32_t)(384 + st * 64 + 32 * half), u);
            l = l * alpha + ((ls4[0] + ls4[1]) + (ls4[2] + ls4[3]));
            m = mnew;
            pf_st_wait();
            pf_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->p_full[st]);
        }
        // the row sum over both halves of every block
        s_psum[half][r] = l;
        if (!skip) mbar_arrive(&bar->pair_sum[q4]);
        if (!failed && !skip && pf_wait(&bar->pair_sum[q4], 0u, abort_flag) &&
            pf_wait(&bar->pv_done[(nb - 1) & 1], (uint32_t)((nb - 1) >> 1) & 1u, abort_flag)) {
            const float lt = l + s_psum[half ^ 1][r];
            pf_fence_after();
            const int qrow = q0 + pos0 + pos, head = kvh * p.gsz + g;
            const size_t ob = ((size_t)qrow * p.nh + head) * kHD + 64 * half;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t u[32];
                pf_ld32(tmem + lane_addr + (uint32_t)(256 + 64 * half + 32 * c), u);
                pf_ld_wait();
                if (row_ok) {
#pragma unroll
                    for (int e8 = 0; e8 < 4; ++e8) {
                        uint32_t w[4];
#pragma unroll
                        for (int e2 = 0; e2 < 4; ++e2) {
                            float v2[2];
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int e = 8 * e8 + 2 * e2 + h;
                                const int d = 32 * c + e;
                                float v = lt > 0.f ? bf16_round(__fdiv_rn(__uint_as_float(u[e]), lt)) : 0.f;
                                if (p.gate) {
                                    const float gt = bf2f(p.gate[ob + d]);
                                    const float sg = bf16_round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gt))));
                                    v = __fmul_rn(v, sg);
                                }
                                v2[h] = v;
                            }
                            w[e2] = pack_bf16(v2[0], v2[1]);
                        }
                        *reinterpret_cast<uint4 *>(p.out + ob + 32 * c + 8 * e8) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
    }

    // ---- teardown ----
    pf_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 0) atomicExch(p.err, 1);
    if (warp == 1) {
        pf_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols) : "memory");
    }
}

// Prefill-sized passes (at least 64 query rows per KV head, at least one CTA per SM) on
// the tcgen05 kernel; ECPU_ERR_UNSUPPORTED (nothing launched) for other shapes: fewer rows
// or CTAs, a query group that does not divide 128 rows, or q not 16-byte aligned.  PILM_ATTN_TC=0 leaves every pass to
// the other kernels.
int launch_attention_prefill_tc(const ekernel_paged_attn_desc_t *desc, const AttnParams &a, const char *what) {
    static const bool off = getenv("PILM_ATTN_TC") && getenv("PILM_ATTN_TC")[0] == '0';
    const int max_q = (int)(desc->max_q_len ? desc->max_q_len : 1);
    // at least 64 rows per KV head: below that the softmax chain per 128-key block (which
    // does not shrink with fewer valid rows) makes it no faster than the per-head kernel
    if (off || a.gsz < 1 || a.gsz > 16 || (kPfRows % a.gsz) != 0 || max_q * a.gsz < 64 ||
        (((uintptr_t)a.q) & 15) != 0)
        return ECPU_ERR_UNSUPPORTED;
    // a CTA streams its whole key range (no split over keys), so fewer CTAs than SMs leave
    // SMs idle: such passes (a few long sequences with short chunks) stay on the per-head
    // kernel, which splits the keys
    const int tiles = (max_q + kPfRows / a.gsz - 1) / (kPfRows / a.gsz);
    if ((long long)desc->num_seqs * tiles * a.nkv < num_sms()) return ECPU_ERR_UNSUPPORTED;
    TensorMapEncodeTiledFn enc = tensor_map_encoder();
    PILM_REQUIRE(enc, ECPU_ERR_UNSUPPORTED, "%s: cuTensorMapEncodeTiled is unavailable", what);
    PfParams p;
    p.block_table = a.block_table;
    p.cu_q = a.cu_q;
    p.ctx = a.ctx;
    p.gate = a.gate;
    p.out = a.out;
    p.err = device_error_word();
    PILM_REQUIRE(p.err, ECPU_ERR_MEM, "%s: error word allocation failed", what);
    p.nh = a.nh;
    p.gsz = a.gsz;
    p.ppt = kPfRows / a.gsz;
    p.tiles = (max_q + p.ppt - 1) / p.ppt;
    p.max_blocks = a.max_blocks;
    p.num_blocks = a.num_blocks;
    p.scale = a.scale;
    CUtensorMap qmap;
    {
        // q [total_q, nh, 128] as (dim, head, row): a box of 64 dims x gsz heads x ppt rows
        // lands as [row][head][64 dims], the Q tile's row r = position * gsz + head
        cuuint64_t dims[3] = {(cuuint64_t)kHD, (cuuint64_t)a.nh, (cuuint64_t)a.total_q};
        cuuint64_t strides[2] = {(cuuint64_t)kHD * 2, (cuuint64_t)a.nh * kHD * 2};
        cuuint32_t box[3] = {64, (cuuint32_t)a.gsz, (cuuint32_t)p.ppt};
        cuuint32_t es[3] = {1, 1, 1};
        const CUresult r = enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, (void *)a.q, dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        PILM_REQUIRE(r == CUDA_SUCCESS, ECPU_ERR_PARAM, "%s: the query tensor map was rejected (error %d)", what, (int)r);
    }
    CUtensorMap maps[2];
    int rc = encode_kv_maps(a.kc, a.vc, a.nkv, a.num_blocks, maps, what);
    if (rc != ECPU_OK) return rc;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmemTotal);
        attr = true;
    }
    launch_pdl(attn_prefill_tc, dim3((unsigned)(desc->num_seqs * p.tiles), (unsigned)a.nkv), dim3(kPfThreads),
               kPfSmemTotal, qmap, maps[0], maps[1], p);
    rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    return check_error_word(what, "a prefill attention wait did not complete");
}

// The whole-page persistent kernel and its merge; ECPU_ERR_UNSUPPORTED (nothing launched)
// for shapes it does not take: more than 8 KV heads, more than 1024 sequences, or more
// than 16 query rows per KV head (q_len x n_heads / n_kv; more would spill registers).
int launch_attention_pages(const ekernel_paged_attn_desc_t *desc, const AttnParams &a, const char *what) {
    const int max_q = (int)(desc->max_q_len ? desc->max_q_len : 1);
    const int R = max_q * a.gsz;
    if (a.nkv > kPMaxKv || desc->num_seqs > (size_t)kPMaxSeqs || R > 16) return ECPU_ERR_UNSUPPORTED;
    PageAttnParams p;
    p.q = a.q;
    p.block_table = a.block_table;
    p.cu_q = a.cu_q;
    p.ctx = a.ctx;
    p.gate = a.gate;
    p.out = a.out;
    p.nh = a.nh;
    p.nkv = a.nkv;
    p.gsz = a.gsz;
    p.max_blocks = a.max_blocks;
    p.num_blocks = a.num_blocks;
    p.B = (int)desc->num_seqs;
    p.max_q = max_q;
    // one CTA per SM, but at least kMinPagesPerCta pages each by the host's bound on the
    // batch's pages (sequences x pages of max_context, a capacity that captured graphs keep):
    // a short batch split over every SM leaves most CTAs one page or none, and its merge
    // then walks as many pieces
    {
        const long long t_upper = (long long)desc->num_seqs * (long long)((desc->max_context + 15) / 16);
        const long long g = (t_upper + kMinPagesPerCta - 1) / kMinPagesPerCta;
        p.G = (int)(g < 1 ? 1 : (g < num_sms() ? g : num_sms()));
    }
    p.total_q = a.total_q;
    p.scale = a.scale;
    p.err = device_error_word();
    PILM_REQUIRE(p.err, ECPU_ERR_MEM, "%s: error word allocation failed", what);
    const size_t part_bytes = (size_t)p.G * 2 * max_q * p.nh * kPRec * sizeof(float);
    char *ws = (char *)scratch(kScratchAttn, part_bytes + 256);
    PILM_REQUIRE(ws, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
    p.part = (float *)ws;
    CUtensorMap maps[2];
    int rc = encode_kv_page_maps(a.kc, a.vc, a.nkv, a.num_blocks, maps, what);
    if (rc != ECPU_OK) return rc;
    const size_t smem = (size_t)kPStages * 4 * p.nkv * 2048 + 1024;  // + alignment slack
    const unsigned threads = (unsigned)(p.nkv + 1) * 32;
    cudaFuncSetAttribute(attn_pages<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(attn_pages<1>, dim3(p.G), dim3(threads), smem, maps[0], maps[1], p);
    rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    rc = check_error_word(what, "a K/V page load did not complete");
    if (rc != ECPU_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.nh + kMergeHeads - 1) / kMergeHeads), (unsigned)p.max_q, (unsigned)p.B);
    cfg.blockDim = dim3(kMergeHeads * 32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_merge_pages, p);
    PILM_REQUIRE(e == cudaSuccess, ECPU_ERR_KERNEL, "%s: merge launch failed: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

// Encodes the K/V tensor maps, launches attn_verify (and attn_merge when split), and in
// synchronous mode reports a page wait that gave up.
int launch_attention(AttnParams &p, const ekernel_paged_attn_desc_t *desc, int MT, int row_chunks, int splits,
                     int *err, const char *what) {
    p.err = err;
    PILM_REQUIRE(p.err, ECPU_ERR_MEM, "%s: no device error word", what);
    CUtensorMap maps[2];
    int rc0 = encode_kv_maps(p.kc, p.vc, p.nkv, p.num_blocks, maps, what);
    if (rc0 != ECPU_OK) return rc0;
    const size_t ring = (size_t)kWarps * kStages * 2 * kPageBytes;
    const size_t mergebuf = (size_t)kWarps * 16 * MT * (kHD + 2) * sizeof(float);
    const size_t smem = (ring > mergebuf ? ring : mergebuf) + 1024;  // + alignment slack
    dim3 grid(splits, p.nkv * row_chunks, (unsigned)desc->num_seqs);
    if (MT == 1) {
        cudaFuncSetAttribute(attn_verify<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        launch_pdl(attn_verify<1>, dim3(grid), dim3(kWarps * 32), smem, maps[0], maps[1], p);
    } else {
        cudaFuncSetAttribute(attn_verify<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        launch_pdl(attn_verify<2>, dim3(grid), dim3(kWarps * 32), smem, maps[0], maps[1], p);
    }
    int rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    rc = check_error_word_at(p.err, what, "a K/V page load did not complete");
    if (rc != ECPU_OK || splits == 1) return rc;
    launch_pdl(attn_merge, dim3((unsigned)(desc->total_q * desc->n_heads)), dim3(kHD), 0, p);
    return check_launch(what);
}

// Split-KV plan of the per-head kernel: query-row tiles per KV head, KV splits and the
// (O, m, l) records the splits leave behind.  Both attention entry points plan through
// here, so the allocation-free variant's size check always matches what the kernel indexes.
struct SplitPlan {
    int MT, row_chunks, splits, pages_per_split;
    size_t n_rec;  // split records (0 when the call is not split)
};

SplitPlan plan_splits(const ekernel_paged_attn_desc_t *desc, int gsz, int nkv) {
    SplitPlan s;
    const int rows = (int)(desc->max_q_len ? desc->max_q_len : 1) * gsz;
    s.MT = rows > 16 ? 2 : 1;
    s.row_chunks = (rows + 16 * s.MT - 1) / (16 * s.MT);
    const int max_pages = (int)((desc->max_context + 15) / 16);
    const int base = (int)desc->num_seqs * nkv * s.row_chunks;
    const int target = 2 * num_sms() * 2;  // 2 resident CTAs per SM, two waves
    int splits = (target + base - 1) / base;
    int max_splits = max_pages / (2 * kWarps);  // at least 2 pages per warp
    if (max_splits < 1) max_splits = 1;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    s.pages_per_split = (max_pages + splits - 1) / splits;
    if (s.pages_per_split < 1) s.pages_per_split = 1;
    splits = (max_pages + s.pages_per_split - 1) / s.pages_per_split;
    if (splits < 1) splits = 1;
    s.splits = splits;
    s.n_rec = splits > 1 ? (size_t)splits * desc->total_q * desc->n_heads : 0;
    return s;
}

int check_desc(const ekernel_paged_attn_desc_t *d, const char *what) {
    PILM_REQUIRE(d, ECPU_ERR_PARAM, "%s: null descriptor", what);
    PILM_REQUIRE(d->head_dim == kHD, ECPU_ERR_UNSUPPORTED, "%s: head_dim must be 128", what);
    PILM_REQUIRE(d->block_size == 16, ECPU_ERR_UNSUPPORTED, "%s: block_size must be 16", what);
    PILM_REQUIRE(d->n_kv_heads > 0 && d->n_heads % d->n_kv_heads == 0, ECPU_ERR_PARAM,
                 "%s: n_heads must be a multiple of n_kv_heads", what);
    PILM_REQUIRE(d->total_q <= 0x7fffff && d->num_seqs <= 0xffff && d->n_heads <= 1024, ECPU_ERR_PARAM,
                 "%s: sizes out of range", what);
    PILM_REQUIRE(d->rot_dim <= kHD && (d->rot_dim & 1) == 0, ECPU_ERR_PARAM, "%s: bad rot_dim", what);
    return ECPU_OK;
}

}  // namespace

extern "C" {

int ekernel_qk_norm_rope_kv_append(const ekernel_paged_attn_desc_t *desc, const uint16_t *qkv,
                                   const uint16_t *q_norm_w, const uint16_t *k_norm_w, const float *rope_cos,
                                   const float *rope_sin, const int32_t *positions, const int32_t *slot_mapping,
                                   uint16_t *k_cache, uint16_t *v_cache, uint16_t *q_out, uint16_t *gate_out) {
    const char *what = "ekernel_qk_norm_rope_kv_append";
    int rc = check_desc(desc, what);
    if (rc != ECPU_OK) return rc;
    PILM_REQUIRE(qkv && q_norm_w && k_norm_w && rope_cos && rope_sin && positions && slot_mapping && k_cache &&
                     v_cache && q_out,
                 ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(!desc->output_gate || gate_out, ECPU_ERR_PARAM, "%s: gate_out required when output_gate", what);
    if (desc->total_q == 0) return ECPU_OK;
    const int items = (int)(desc->total_q * (desc->n_heads + desc->n_kv_heads));
    const QkvSrc src{(const __nv_bfloat16 *)qkv, nullptr, 0, 0};
    launch_pdl(qk_prologue, dim3((items + 7) / 8), dim3(256), 0, 
        src, (int)desc->total_q, (int)desc->n_heads, (int)desc->n_kv_heads,
        (int)desc->qkv_stride, desc->output_gate, (const __nv_bfloat16 *)q_norm_w, (const __nv_bfloat16 *)k_norm_w,
        desc->eps, desc->add_one, rope_cos, rope_sin, (int)desc->rope_rows, (int)desc->rot_dim, positions,
        slot_mapping, (long long)desc->num_blocks * (long long)desc->block_size, (__nv_bfloat16 *)k_cache,
        (__nv_bfloat16 *)v_cache, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)gate_out);
    return check_launch(what);
}

int ekernel_qk_norm_rope_kv_append_splitk(const ekernel_paged_attn_desc_t *desc, const float *partials,
                                          int32_t splits, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                          const float *rope_cos, const float *rope_sin, const int32_t *positions,
                                          const int32_t *slot_mapping, uint16_t *k_cache, uint16_t *v_cache,
                                          uint16_t *q_out, uint16_t *gate_out) {
    const char *what = "ekernel_qk_norm_rope_kv_append_splitk";
    int rc = check_desc(desc, what);
    if (rc != ECPU_OK) return rc;
    PILM_REQUIRE(partials && splits > 0 && q_norm_w && k_norm_w && rope_cos && rope_sin && positions &&
                     slot_mapping && k_cache && v_cache && q_out,
                 ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(!desc->output_gate || gate_out, ECPU_ERR_PARAM, "%s: gate_out required when output_gate", what);
    if (desc->total_q == 0) return ECPU_OK;
    const int items = (int)(desc->total_q * (desc->n_heads + desc->n_kv_heads));
    const QkvSrc src{nullptr, partials, (int)splits, (size_t)desc->total_q * desc->qkv_stride};
    launch_pdl(qk_prologue, dim3((items + 7) / 8), dim3(256), 0, 
        src, (int)desc->total_q, (int)desc->n_heads, (int)desc->n_kv_heads,
        (int)desc->qkv_stride, desc->output_gate, (const __nv_bfloat16 *)q_norm_w, (const __nv_bfloat16 *)k_norm_w,
        desc->eps, desc->add_one, rope_cos, rope_sin, (int)desc->rope_rows, (int)desc->rot_dim, positions,
        slot_mapping, (long long)desc->num_blocks * (long long)desc->block_size, (__nv_bfloat16 *)k_cache,
        (__nv_bfloat16 *)v_cache, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)gate_out);
    return check_launch(what);
}

int ekernel_paged_attention_verify(const ekernel_paged_attn_desc_t *desc, const uint16_t *q,
                                   const uint16_t *k_cache, const uint16_t *v_cache, const int32_t *block_table,
                                   const int32_t *cu_q, const int32_t *context_lens, const uint16_t *gate,
                                   uint16_t *out) {
    const char *what = "ekernel_paged_attention_verify";
    int rc = check_desc(desc, what);
    if (rc != ECPU_OK) return rc;
    PILM_REQUIRE(q && k_cache && v_cache && block_table && cu_q && context_lens && out, ECPU_ERR_PARAM,
                 "%s: null argument", what);
    PILM_REQUIRE(!desc->output_gate || gate, ECPU_ERR_PARAM, "%s: gate required when output_gate", what);
    if (desc->total_q == 0 || desc->num_seqs == 0) return ECPU_OK;

    AttnParams p;
    p.q = (const __nv_bfloat16 *)q;
    p.kc = (const __nv_bfloat16 *)k_cache;
    p.vc = (const __nv_bfloat16 *)v_cache;
    p.block_table = block_table;
    p.cu_q = cu_q;
    p.ctx = context_lens;
    p.gate = desc->output_gate ? (const __nv_bfloat16 *)gate : nullptr;
    p.out = (__nv_bfloat16 *)out;
    p.nh = (int)desc->n_heads;
    p.nkv = (int)desc->n_kv_heads;
    p.gsz = p.nh / p.nkv;
    p.max_blocks = (int)desc->max_blocks_per_seq;
    p.num_blocks = (int)desc->num_blocks;
    p.total_q = (int)desc->total_q;
    // scale = 1/sqrt(head_dim) as the Python float the reference multiplies by,
    // narrowed to fp32 (the bf16 kernel's opmath type)
    p.scale = (float)(1.0 / sqrt((double)kHD));

    // prefill-sized passes on tensor cores; whole pages per CTA where the shape allows it;
    // else the per-head split kernel
    rc = launch_attention_prefill_tc(desc, p, what);
    if (rc != ECPU_ERR_UNSUPPORTED) return rc;
    rc = launch_attention_pages(desc, p, what);
    if (rc != ECPU_ERR_UNSUPPORTED) return rc;

    const SplitPlan sp = plan_splits(desc, p.gsz, p.nkv);
    p.pages_per_split = sp.pages_per_split;
    p.splits = sp.splits;
    p.row_chunk = 16 * sp.MT;
    p.part_o = nullptr;
    p.part_ml = nullptr;
    if (sp.splits > 1) {
        char *ws = (char *)scratch(kScratchAttn, sp.n_rec * (kHD + 2) * sizeof(float) + 256);
        PILM_REQUIRE(ws, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
        p.part_o = (float *)ws;
        p.part_ml = p.part_o + sp.n_rec * kHD;
        launch_pdl(attn_clear_ml, dim3((int)((sp.n_rec * 2 + 255) / 256 < 4096 ? (sp.n_rec * 2 + 255) / 256 : 4096)),
                   dim3(256), 0, p.part_ml, sp.n_rec * 2);
        rc = check_launch(what);
        if (rc != ECPU_OK) return rc;
    }
    return launch_attention(p, desc, sp.MT, sp.row_chunks, sp.splits, device_error_word(), what);
}

}  // extern "C"

// ---------------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot let a kernel library allocate GPU memory: an engine whose
// allocator owns the whole device and forbids side allocations, a caller that must
// never hit cudaMalloc's implicit device-wide synchronisation on its serving path,
// or a host written in another language that only hands over buffers it already
// owns.  For them ekernel_paged_attention_verify_noalloc takes the same inputs and
// outputs as ekernel_paged_attention_verify but keeps its split-KV partials in
// g_noalloc_attn_scratch, a fixed 8 MiB array compiled into the library, records a
// page wait that gave up in g_noalloc_err_word, and calls no allocator at all.  The host
// cannot pass either symbol itself to a kernel (in host code those names are only
// host-side stand-ins), so their device addresses are looked up once per device with
// cudaGetSymbolAddress and cached here.
// ---------------------------------------------------------------------------------
namespace {

constexpr int kNoAllocMaxDevices = 64;
struct NoAllocAddrs {
    void *scratch = nullptr;  // g_noalloc_attn_scratch on this device
    int *err = nullptr;       // g_noalloc_err_word on this device
};
NoAllocAddrs g_noalloc_addr[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Device addresses of g_noalloc_attn_scratch and g_noalloc_err_word on the current device
// (looked up on the first call for that device, with that device current).
int noalloc_addresses(NoAllocAddrs *out, const char *what) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    PILM_REQUIRE(e == cudaSuccess && dev >= 0 && dev < kNoAllocMaxDevices, ECPU_ERR_DEVICE,
                 "%s: no usable current device (%s)", what, cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocAddrs &a = g_noalloc_addr[dev];
    if (!a.scratch || !a.err) {
        void *ptr = nullptr, *eptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_attn_scratch);
        PILM_REQUIRE(e == cudaSuccess && ptr, ECPU_ERR_DEVICE, "%s: cudaGetSymbolAddress failed: %s", what,
                     cudaGetErrorString(e));
        e = cudaGetSymbolAddress(&eptr, g_noalloc_err_word);
        PILM_REQUIRE(e == cudaSuccess && eptr, ECPU_ERR_DEVICE, "%s: cudaGetSymbolAddress failed: %s", what,
                     cudaGetErrorString(e));
        a.scratch = ptr;
        a.err = (int *)eptr;
    }
    *out = a;
    return ECPU_OK;
}

}  // namespace

extern "C" int ekernel_paged_attention_verify_noalloc(const ekernel_paged_attn_desc_t *desc, const uint16_t *q,
                                                      const uint16_t *k_cache, const uint16_t *v_cache,
                                                      const int32_t *block_table, const int32_t *cu_q,
                                                      const int32_t *context_lens, const uint16_t *gate,
                                                      uint16_t *out) {
    const char *what = "ekernel_paged_attention_verify_noalloc";
    int rc = check_desc(desc, what);
    if (rc != ECPU_OK) return rc;
    PILM_REQUIRE(q && k_cache && v_cache && block_table && cu_q && context_lens && out, ECPU_ERR_PARAM,
                 "%s: null argument", what);
    PILM_REQUIRE(!desc->output_gate || gate, ECPU_ERR_PARAM, "%s: gate required when output_gate", what);
    if (desc->total_q == 0 || desc->num_seqs == 0) return ECPU_OK;

    AttnParams p;
    p.q = (const __nv_bfloat16 *)q;
    p.kc = (const __nv_bfloat16 *)k_cache;
    p.vc = (const __nv_bfloat16 *)v_cache;
    p.block_table = block_table;
    p.cu_q = cu_q;
    p.ctx = context_lens;
    p.gate = desc->output_gate ? (const __nv_bfloat16 *)gate : nullptr;
    p.out = (__nv_bfloat16 *)out;
    p.nh = (int)desc->n_heads;
    p.nkv = (int)desc->n_kv_heads;
    p.gsz = p.nh / p.nkv;
    p.max_blocks = (int)desc->max_blocks_per_seq;
    p.num_blocks = (int)desc->num_blocks;
    p.total_q = (int)desc->total_q;
    p.scale = (float)(1.0 / sqrt((double)kHD));

    // the per-head split kernel (its partials are bounded by the split count, so they fit the
    // fixed array); results agree with ekernel_paged_attention_verify within fp32 rounding
    const SplitPlan sp = plan_splits(desc, p.gsz, p.nkv);
    p.pages_per_split = sp.pages_per_split;
    p.splits = sp.splits;
    p.row_chunk = 16 * sp.MT;
    p.part_o = nullptr;
    p.part_ml = nullptr;
    const size_t need = sp.n_rec * (kHD + 2) * sizeof(float);
    PILM_REQUIRE(need <= kNoAllocAttnScratchBytes, ECPU_ERR_PARAM,
                 "%s: this call needs %zu bytes of split-KV scratch (%d splits x %zu rows x %zu heads) but the "
                 "allocation-free variant holds at most %zu bytes; use ekernel_paged_attention_verify",
                 what, need, sp.splits, desc->total_q, desc->n_heads, kNoAllocAttnScratchBytes);
    NoAllocAddrs a;
    rc = noalloc_addresses(&a, what);
    if (rc != ECPU_OK) return rc;
    if (sp.splits > 1) {
        p.part_o = (float *)a.scratch;
        p.part_ml = p.part_o + sp.n_rec * kHD;
        // the array keeps the previous call's contents: reset every (m, l) record
        launch_pdl(attn_clear_ml, dim3((int)((sp.n_rec * 2 + 255) / 256 < 4096 ? (sp.n_rec * 2 + 255) / 256 : 4096)),
                   dim3(256), 0, p.part_ml, sp.n_rec * 2);
        rc = check_launch(what);
        if (rc != ECPU_OK) return rc;
    }
    return launch_attention(p, desc, sp.MT, sp.row_chunks, sp.splits, a.err, what);
}
