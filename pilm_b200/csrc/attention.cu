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
//                 through a private cp.async ring (3 pages deep, XOR-swizzled smem),
//                 computes S = Q K^T and O += P V with mma.sync m16n8k16 (bf16 in,
//                 fp32 accumulate) and keeps an fp32 online softmax; warps then merge.
//   attn_merge    combines split partials (m, l, O) and applies the output gate.
#include <mutex>

#include "common.cuh"

using namespace pilm;

// Fixed device scratch for ekernel_paged_attention_verify_noalloc (see below).  Every
// GPU that loads this library holds these bytes until the process exits.
constexpr size_t kNoAllocAttnScratchBytes = (size_t)8 << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_noalloc_attn_scratch[kNoAllocAttnScratchBytes];

namespace {

constexpr int kHD = 128;         // head_dim supported by the tensor-core path
constexpr int kWarps = 4;        // warps per attention CTA
constexpr int kStages = 3;       // pages in flight per warp
constexpr int kPageBytes = 16 * kHD * 2;  // one K (or V) tile of a 16-token page

// ---------------------------------------------------------------------------------
// Prologue: q/k RMSNorm + RoPE, KV append
// ---------------------------------------------------------------------------------
__global__ void qk_prologue(const __nv_bfloat16 *__restrict__ qkv, int total_q, int nh, int nkv, int qkv_stride,
                            int gated, const __nv_bfloat16 *__restrict__ qnw, const __nv_bfloat16 *__restrict__ knw,
                            float eps, int add_one, const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                            int rope_rows, int rot_dim, const int32_t *__restrict__ positions,
                            const int32_t *__restrict__ slots, long long num_slots, __nv_bfloat16 *__restrict__ kc,
                            __nv_bfloat16 *__restrict__ vc, __nv_bfloat16 *__restrict__ q_out,
                            __nv_bfloat16 *__restrict__ gate_out) {
    __shared__ float buf[8][kHD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * 8 + warp;
    const int heads = nh + nkv;
    if (item >= total_q * heads) return;
    const int row = item / heads, h = item % heads;
    const bool is_q = h < nh;
    const __nv_bfloat16 *src;
    const int qsec = nh * kHD * (gated ? 2 : 1);
    if (is_q)
        src = qkv + (size_t)row * qkv_stride + (size_t)h * kHD * (gated ? 2 : 1);
    else
        src = qkv + (size_t)row * qkv_stride + qsec + (size_t)(h - nh) * kHD;
    const __nv_bfloat16 *nw = is_q ? qnw : knw;
    float x[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x[j] = bf2f(src[lane + 32 * j]);
        ss = fmaf(x[j], x[j], ss);
    }
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHD), eps)));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        float xn = bf16_round(__fmul_rn(x[j], inv));
        float wf = bf2f(nw[d]);
        if (add_one) wf = bf16_round(__fadd_rn(wf, 1.0f));
        buf[warp][d] = bf16_round(__fmul_rn(xn, wf));
    }
    __syncwarp();
    const int pos = positions[row];
    const int nf = rot_dim >> 1;
    const bool pos_ok = pos >= 0 && pos < rope_rows;
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        float v = buf[warp][d];
        if (d < rot_dim && pos_ok) {
            // out_first = a*cos - b*sin ; out_second = a*sin + b*cos  (layers.py:161-164)
            const int f = d < nf ? d : d - nf;
            const float cs = cos_t[(size_t)pos * nf + f], sn = sin_t[(size_t)pos * nf + f];
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
        if (gated && gate_out) {
            const __nv_bfloat16 *gsrc = src + kHD;
            __nv_bfloat16 *go = gate_out + (size_t)row * nh * kHD + (size_t)h * kHD;
#pragma unroll
            for (int j = 0; j < 4; ++j) go[lane + 32 * j] = gsrc[lane + 32 * j];
        }
    } else {
        const long long slot = slots[row];
        if (slot < 0 || slot >= num_slots) return;  // rejected / padded rows are not written
        const int kvh = h - nh;
        __nv_bfloat16 *kd = kc + ((size_t)slot * nkv + kvh) * kHD;
        __nv_bfloat16 *vd = vc + ((size_t)slot * nkv + kvh) * kHD;
        const __nv_bfloat16 *vsrc = qkv + (size_t)row * qkv_stride + qsec + (size_t)nkv * kHD + (size_t)kvh * kHD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            kd[lane + 32 * j] = f2bf(y[j]);
            vd[lane + 32 * j] = vsrc[lane + 32 * j];
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// byte offset of 16-byte chunk `ch` (0..15) of row `row` (0..15) inside a 4 KB tile
__device__ __forceinline__ uint32_t swz(int row, int ch) { return (uint32_t)(row * 256 + ((ch ^ (row & 7)) << 4)); }

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
    int nh, nkv, gsz, max_blocks, num_blocks, total_q;
    int splits, pages_per_split, row_chunk;  // rows per CTA = 16 * MT; pages_per_split: host sizing only
    float scale;                 // rne_bf16-compatible fp32 value of 1/sqrt(head_dim)
};

// grid: (splits, nkv * row_chunks, B); block: 128 threads
template <int MT>
__global__ void __launch_bounds__(kWarps * 32, 2) attn_verify(const AttnParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
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

    uint8_t *ring = smem + (size_t)warp * kStages * 2 * kPageBytes;
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    const int32_t *bt = p.block_table + (size_t)b * p.max_blocks;
    const size_t kv_row_stride = (size_t)p.nkv * kHD;  // elements between consecutive slots

    // pages handled by this warp: pg0 + warp, pg0 + warp + 4, ... (< pg_vis)
    auto issue = [&](int it, int stage) {
        const int pg = pg0 + warp + it * kWarps;
        const uint32_t kdst = ring_s + stage * 2 * kPageBytes, vdst = kdst + kPageBytes;
        if (pg < pg_vis) {
            int blk = bt[pg];
            const bool blk_ok = blk >= 0 && blk < p.num_blocks;
            if (!blk_ok) blk = 0;
            const int valid = min(16, ctx - pg * 16);  // tokens of this page inside the context
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int idx = lane + 32 * e;  // 256 chunks: row = idx / 16, ch = idx % 16
                const int row = idx >> 4, ch = idx & 15;
                const int bytes = (blk_ok && row < valid) ? 16 : 0;
                const size_t off = ((size_t)blk * 16 + row) * kv_row_stride + (size_t)kvh * kHD + ch * 8;
                cp_async16(kdst + swz(row, ch), p.kc + off, bytes);
                cp_async16(vdst + swz(row, ch), p.vc + off, bytes);
            }
        }
        cp_async_commit();
    };

    const int n_it = pg_vis > pg0 + warp ? (pg_vis - (pg0 + warp) + kWarps - 1) / kWarps : 0;
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) issue(s, s);

    for (int it = 0; it < n_it; ++it) {
        issue(it + kStages - 1, (it + kStages - 1) % kStages);
        cp_async_wait<kStages - 1>();
        __syncwarp();
        const int stage = it % kStages;
        const uint32_t ks_base = ring_s + stage * 2 * kPageBytes, vs_base = ks_base + kPageBytes;
        const int pg = pg0 + warp + it * kWarps;

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
#pragma unroll
                for (int nt = 0; nt < 16; ++nt) {
                    o[mt][nt][hh * 2 + 0] *= alpha;
                    o[mt][nt][hh * 2 + 1] *= alpha;
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
    cp_async_wait<0>();
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

// Clear the split partials of every (row, head) so that CTAs which exit early (no
// rows or no visible pages in their split) leave an empty record (l = 0).
__global__ void attn_clear_ml(float *ml, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        ml[i] = (i & 1) ? 0.f : -INFINITY;
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
    qk_prologue<<<(items + 7) / 8, 256, 0, stream()>>>(
        (const __nv_bfloat16 *)qkv, (int)desc->total_q, (int)desc->n_heads, (int)desc->n_kv_heads,
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

    const int rows = (int)(desc->max_q_len ? desc->max_q_len : 1) * p.gsz;
    const int MT = rows > 16 ? 2 : 1;
    const int row_chunks = (rows + 16 * MT - 1) / (16 * MT);
    const int max_pages = (int)((desc->max_context + 15) / 16);
    const int base = (int)desc->num_seqs * p.nkv * row_chunks;
    const int target = 2 * num_sms() * 2;  // 2 resident CTAs per SM, two waves
    int splits = (target + base - 1) / base;
    int max_splits = max_pages / (2 * kWarps);  // at least 2 pages per warp
    if (max_splits < 1) max_splits = 1;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    p.pages_per_split = (max_pages + splits - 1) / splits;
    if (p.pages_per_split < 1) p.pages_per_split = 1;
    splits = (max_pages + p.pages_per_split - 1) / p.pages_per_split;
    if (splits < 1) splits = 1;
    p.splits = splits;
    p.row_chunk = 16 * MT;
    p.part_o = nullptr;
    p.part_ml = nullptr;
    if (splits > 1) {
        const size_t n_rec = (size_t)splits * desc->total_q * desc->n_heads;
        char *ws = (char *)scratch(kScratchAttn, n_rec * (kHD + 2) * sizeof(float) + 256);
        PILM_REQUIRE(ws, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
        p.part_o = (float *)ws;
        p.part_ml = p.part_o + n_rec * kHD;
        attn_clear_ml<<<(int)((n_rec * 2 + 255) / 256 < 4096 ? (n_rec * 2 + 255) / 256 : 4096), 256, 0,
                        stream()>>>(p.part_ml, n_rec * 2);
        rc = check_launch(what);
        if (rc != ECPU_OK) return rc;
    }
    const size_t ring = (size_t)kWarps * kStages * 2 * kPageBytes;
    const size_t mergebuf = (size_t)kWarps * 16 * MT * (kHD + 2) * sizeof(float);
    const size_t smem = ring > mergebuf ? ring : mergebuf;
    dim3 grid(splits, p.nkv * row_chunks, (unsigned)desc->num_seqs);
    if (MT == 1) {
        cudaFuncSetAttribute(attn_verify<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attn_verify<1><<<grid, kWarps * 32, smem, stream()>>>(p);
    } else {
        cudaFuncSetAttribute(attn_verify<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attn_verify<2><<<grid, kWarps * 32, smem, stream()>>>(p);
    }
    rc = check_launch(what);
    if (rc != ECPU_OK || splits == 1) return rc;
    attn_merge<<<(unsigned)(desc->total_q * desc->n_heads), kHD, 0, stream()>>>(p);
    return check_launch(what);
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
// g_noalloc_attn_scratch, a fixed 8 MiB array compiled into the library, and calls
// no allocator at all.  The host cannot pass g_noalloc_attn_scratch itself to a
// kernel (in host code that name is only a host-side stand-in), so the device address
// is looked up once per device with cudaGetSymbolAddress and cached here.
// ---------------------------------------------------------------------------------
namespace {

constexpr int kNoAllocMaxDevices = 64;
void *g_noalloc_addr[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

// Device address of g_noalloc_attn_scratch on the current device (looked up on the
// first call for that device, with that device current).
int noalloc_scratch_address(void **out, const char *what) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    PILM_REQUIRE(e == cudaSuccess && dev >= 0 && dev < kNoAllocMaxDevices, ECPU_ERR_DEVICE,
                 "%s: no usable current device (%s)", what, cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_attn_scratch);
        PILM_REQUIRE(e == cudaSuccess && ptr, ECPU_ERR_DEVICE, "%s: cudaGetSymbolAddress failed: %s", what,
                     cudaGetErrorString(e));
        g_noalloc_addr[dev] = ptr;
    }
    *out = g_noalloc_addr[dev];
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

    // the same split choice as ekernel_paged_attention_verify, so both give the same result
    const int rows = (int)(desc->max_q_len ? desc->max_q_len : 1) * p.gsz;
    const int MT = rows > 16 ? 2 : 1;
    const int row_chunks = (rows + 16 * MT - 1) / (16 * MT);
    const int max_pages = (int)((desc->max_context + 15) / 16);
    const int base = (int)desc->num_seqs * p.nkv * row_chunks;
    const int target = 2 * num_sms() * 2;
    int splits = (target + base - 1) / base;
    int max_splits = max_pages / (2 * kWarps);
    if (max_splits < 1) max_splits = 1;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    p.pages_per_split = (max_pages + splits - 1) / splits;
    if (p.pages_per_split < 1) p.pages_per_split = 1;
    splits = (max_pages + p.pages_per_split - 1) / p.pages_per_split;
    if (splits < 1) splits = 1;
    p.splits = splits;
    p.row_chunk = 16 * MT;
    p.part_o = nullptr;
    p.part_ml = nullptr;
    if (splits > 1) {
        const size_t n_rec = (size_t)splits * desc->total_q * desc->n_heads;
        const size_t need = n_rec * (kHD + 2) * sizeof(float);
        PILM_REQUIRE(need <= kNoAllocAttnScratchBytes, ECPU_ERR_PARAM,
                     "%s: this call needs %zu bytes of split-KV scratch (%d splits x %zu rows x %zu heads) but the "
                     "allocation-free variant holds at most %zu bytes; use ekernel_paged_attention_verify",
                     what, need, splits, desc->total_q, desc->n_heads, kNoAllocAttnScratchBytes);
        void *base_ptr = nullptr;
        rc = noalloc_scratch_address(&base_ptr, what);
        if (rc != ECPU_OK) return rc;
        p.part_o = (float *)base_ptr;
        p.part_ml = p.part_o + n_rec * kHD;
        // the array keeps the previous call's contents: reset every (m, l) record
        attn_clear_ml<<<(int)((n_rec * 2 + 255) / 256 < 4096 ? (n_rec * 2 + 255) / 256 : 4096), 256, 0,
                        stream()>>>(p.part_ml, n_rec * 2);
        rc = check_launch(what);
        if (rc != ECPU_OK) return rc;
    }
    const size_t ring = (size_t)kWarps * kStages * 2 * kPageBytes;
    const size_t mergebuf = (size_t)kWarps * 16 * MT * (kHD + 2) * sizeof(float);
    const size_t smem = ring > mergebuf ? ring : mergebuf;
    dim3 grid(splits, p.nkv * row_chunks, (unsigned)desc->num_seqs);
    if (MT == 1) {
        cudaFuncSetAttribute(attn_verify<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attn_verify<1><<<grid, kWarps * 32, smem, stream()>>>(p);
    } else {
        cudaFuncSetAttribute(attn_verify<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attn_verify<2><<<grid, kWarps * 32, smem, stream()>>>(p);
    }
    rc = check_launch(what);
    if (rc != ECPU_OK || splits == 1) return rc;
    attn_merge<<<(unsigned)(desc->total_q * desc->n_heads), kHD, 0, stream()>>>(p);
    return check_launch(what);
}
