// fp32-activation verify path: the Qwen3Model forward when the model dtype is float32
// (the W8A32 configuration: QuantizedW8A32Linear, linear.py:188-233, fp32 KV cache).
//
// The same operations as the bf16 path with every intermediate kept in fp32, as torch
// computes them for float32 tensors:
//   add_rmsnorm_f32   RMSNorm / GemmaRMSNorm (layers.py:94-98, 115-119):
//                     y = w' * (x * rsqrt(mean(x^2) + eps)), w' = w or 1 + w, after an
//                     optional residual add (model.py:66-72)
//   qk_prologue_f32   q/k head RMSNorm, half-split RoPE on the first rot_dim dims
//                     (layers.py:122-176), K/V written to their page slots
//   attn_f32          paged decode attention (attention.py:95-139): scores = q.k * scale,
//                     causal mask, softmax, P.V, times sigmoid(gate) when gated.  One warp
//                     per (query row, head); keys 32 at a time (one per lane) with an
//                     online softmax; the output dims are spread over the lanes.
//   silu_mul_f32      SwiGLU activation silu(g) * u (layers.py:193)
//   embedding_f32     token rows of the fp32 embedding table (model.py:110)
// These serve the small W8A32 configuration (M = 2 verify rows); they are plain CUDA-core
// kernels, not tuned for long contexts.
#include "common.cuh"

using namespace pilm;

namespace {

constexpr int kHD = 128;

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__global__ void embedding_f32_kernel(const int32_t *__restrict__ ids, int rows, const float *__restrict__ table,
                                     int vocab, int hidden, float *__restrict__ out, int *__restrict__ err) {
    pdl_entry();
    const int r = blockIdx.x;
    if (r >= rows) return;
    int id = ids[r];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) atomicExch(err, 1);
        id = 0;
    }
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) out[(size_t)r * hidden + i] = table[(size_t)id * hidden + i];
}

// one CTA (256 threads) per row, any n (the rows above 8192 values)
__global__ void __launch_bounds__(256) add_rmsnorm_f32_loop(float *__restrict__ res, const float *__restrict__ delta,
                                                            const float *__restrict__ w, int n, float eps,
                                                            int add_one, float *__restrict__ out) {
    pdl_entry();
    __shared__ float red[8];
    const int row = blockIdx.x;
    float *r = res + (size_t)row * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) {
        float x = r[i];
        if (delta) {
            x = __fadd_rn(x, delta[(size_t)row * n + i]);
            r[i] = x;
        }
        ss = fmaf(x, x, ss);
    }
    ss = warp_sum32(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += 256) {
        float wf = w[i];
        if (add_one) wf = __fadd_rn(wf, 1.0f);
        out[(size_t)row * n + i] = __fmul_rn(wf, __fmul_rn(r[i], inv));
    }
}

// The same with the row in registers (VPT values a thread, n <= 256 VPT): the norm
// weights are read before the wait for the previous kernel, the residual and delta in one
// batch after it.  Each thread's squares are added in index order, as the strided loop adds
// them.
template <int VPT>
__global__ void __launch_bounds__(256) add_rmsnorm_f32_kernel(float *__restrict__ res, const float *__restrict__ delta,
                                                              const float *__restrict__ w, int n, float eps,
                                                              int add_one, float *__restrict__ out) {
    pdl_trigger();
    __shared__ float red[8];
    const int row = blockIdx.x;
    float *r = res + (size_t)row * n;
    float wv[VPT], x[VPT], d[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = threadIdx.x + 256 * v;
        wv[v] = i < n ? w[i] : 0.f;
    }
    pdl_wait();
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = threadIdx.x + 256 * v;
        x[v] = i < n ? r[i] : 0.f;
        d[v] = i < n && delta ? delta[(size_t)row * n + i] : 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = threadIdx.x + 256 * v;
        if (i >= n) continue;
        if (delta) {
            x[v] = __fadd_rn(x[v], d[v]);
            r[i] = x[v];
        }
        ss = fmaf(x[v], x[v], ss);
    }
    ss = warp_sum32(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = threadIdx.x + 256 * v;
        if (i >= n) continue;
        float wf = wv[v];
        if (add_one) wf = __fadd_rn(wf, 1.0f);
        out[(size_t)row * n + i] = __fmul_rn(wf, __fmul_rn(x[v], inv));
    }
}

// one warp per (row, head) over the q heads then the kv heads; 8 warps per CTA
__global__ void qk_prologue_f32_kernel(const float *__restrict__ qkv, int total_q, int nh, int nkv, int qkv_stride,
                                       int gated, const float *__restrict__ qnw, const float *__restrict__ knw,
                                       float eps, int add_one, const float *__restrict__ cos_t,
                                       const float *__restrict__ sin_t, int rope_rows, int rot_dim,
                                       const int32_t *__restrict__ positions, const int32_t *__restrict__ slots,
                                       long long num_slots, float *__restrict__ kc, float *__restrict__ vc,
                                       float *__restrict__ q_out, float *__restrict__ gate_out) {
    pdl_trigger();
    __shared__ float buf[8][kHD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * 8 + warp;
    const int heads = nh + nkv;
    if (item >= total_q * heads) return;
    const int row = item / heads, h = item % heads;
    const bool is_q = h < nh;
    const int qsec = nh * kHD * (gated ? 2 : 1);
    const float *src = is_q ? qkv + (size_t)row * qkv_stride + (size_t)h * kHD * (gated ? 2 : 1)
                            : qkv + (size_t)row * qkv_stride + qsec + (size_t)(h - nh) * kHD;
    const float *nw = is_q ? qnw : knw;
    // norm weights, RoPE tables, positions and slots (constant or host-written) before the
    // wait for the previous kernel, the projection after it
    const int pos = positions[row];
    const int nf = rot_dim >> 1;
    const bool pos_ok = pos >= 0 && pos < rope_rows;
    const long long slot = is_q ? -1 : slots[row];
    float wv[4], cv[4], sv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        float wf = nw[d];
        if (add_one) wf = __fadd_rn(wf, 1.0f);
        wv[j] = wf;
        const int f = d < nf ? d : d - nf;
        const bool rot = d < rot_dim && pos_ok;
        cv[j] = rot ? cos_t[(size_t)pos * nf + f] : 1.f;
        sv[j] = rot ? sin_t[(size_t)pos * nf + f] : 0.f;
    }
    pdl_wait();
    float x[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x[j] = src[lane + 32 * j];
        ss = fmaf(x[j], x[j], ss);
    }
    ss = warp_sum32(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHD), eps)));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        buf[warp][d] = __fmul_rn(wv[j], __fmul_rn(x[j], inv));
    }
    __syncwarp();
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        float v = buf[warp][d];
        if (d < rot_dim && pos_ok) {
            const float cs = cv[j], sn = sv[j];
            if (d < nf)
                v = __fsub_rn(__fmul_rn(v, cs), __fmul_rn(buf[warp][d + nf], sn));
            else
                v = __fadd_rn(__fmul_rn(buf[warp][d - nf], sn), __fmul_rn(v, cs));
        }
        y[j] = v;
    }
    if (is_q) {
        float *qo = q_out + ((size_t)row * nh + h) * kHD;
#pragma unroll
        for (int j = 0; j < 4; ++j) qo[lane + 32 * j] = y[j];
        if (gated && gate_out) {
            float *go = gate_out + (size_t)row * nh * kHD + (size_t)h * kHD;
#pragma unroll
            for (int j = 0; j < 4; ++j) go[lane + 32 * j] = src[kHD + lane + 32 * j];
        }
    } else {
        if (slot < 0 || slot >= num_slots) return;  // rejected / padded rows are not written
        const int kvh = h - nh;
        float *kd = kc + ((size_t)slot * nkv + kvh) * kHD;
        float *vd = vc + ((size_t)slot * nkv + kvh) * kHD;
        const float *vsrc = qkv + (size_t)row * qkv_stride + qsec + (size_t)nkv * kHD + (size_t)kvh * kHD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            kd[lane + 32 * j] = y[j];
            vd[lane + 32 * j] = vsrc[lane + 32 * j];
        }
    }
}

// One CTA per (query row, head); its kFA warps take every kFA-th chunk of 32 keys, each
// with its own online softmax (m, l, o), and the CTA merges the warps' states at the end.
// In a chunk each lane holds 4 of the 128 dims: every key row is one coalesced 512-byte
// load, a lane forms its 4-dim part of all 32 dot products, and a transposing butterfly
// (31 shuffles) leaves key k0 + j's score in lane j.  The warp then accumulates P V over
// the chunk's keys the same way, lane by dims.  The chunk's 32 key rows are loaded at
// once, and its 32 value rows are in flight during the score reduction and the softmax.
constexpr int kFA = 8;
__global__ void __launch_bounds__(kFA * 32, 1) attn_f32_kernel(const float *__restrict__ q, const float *__restrict__ kc,
                                                            const float *__restrict__ vc,
                                                            const int32_t *__restrict__ block_table,
                                                            const int32_t *__restrict__ cu_q,
                                                            const int32_t *__restrict__ ctx_lens,
                                                            const float *__restrict__ gate, float *__restrict__ out,
                                                            int B, int total_q, int nh, int nkv, int max_blocks,
                                                            int num_blocks, float scale) {
    pdl_trigger();
    __shared__ float sm[kFA], sl[kFA];
    __shared__ float4 so[kFA][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x;
    if (item >= total_q * nh) return;
    // The row's sequence, query length and context come from host-written metadata, so
    // they are worked out before the wait for the previous kernel (which appends this
    // step's K/V and writes the queries).
    const int row = item / nh, h = item % nh;
    int lo = 0, hi = B - 1;  // sequence of this row: largest b with cu_q[b] <= row
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu_q[mid] <= row) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int q_len = cu_q[b + 1] - cu_q[b];
    const int ctx = ctx_lens[b];
    const int qpos = ctx - q_len + (row - cu_q[b]);
    const int kvh = h / (nh / nkv);
    const float *qrow = q + ((size_t)row * nh + h) * kHD;
    pdl_wait();
    const float4 q4 = reinterpret_cast<const float4 *>(qrow)[lane];  // dims 4 lane .. 4 lane + 3
    const int32_t *bt = block_table + (size_t)b * max_blocks;
    const int last = min(qpos, ctx - 1);  // the last key this row sees
    float m = -INFINITY, l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k0 = 32 * warp; k0 <= last; k0 += 32 * kFA) {
        const int key = k0 + lane;
        const int n = min(32, last - k0 + 1);  // keys of this chunk the row sees
        size_t off = 0;                        // element offset of key k0 + lane's row
        if (key <= last) {
            int blk = bt[key >> 4];
            if (blk < 0 || blk >= num_blocks) blk = 0;
            off = (((size_t)blk * 16 + (key & 15)) * nkv + kvh) * kHD;
        }
        // The row loads are unconditional, so that all are in flight at once: a key past
        // `last` reads row 0 of the cache (offset 0, always allocated); its score is
        // replaced by -inf and its P V term skipped.
        float4 kv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const size_t oj = (size_t)__shfl_sync(0xffffffffu, (unsigned long long)off, j);
            kv[j] = reinterpret_cast<const float4 *>(kc + oj)[lane];
        }
        // p[j]: this lane's 4-dim part of key k0 + j's dot product
        float p[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
            p[j] = fmaf(q4.w, kv[j].w, fmaf(q4.z, kv[j].z, fmaf(q4.y, kv[j].y, __fmul_rn(q4.x, kv[j].x))));
        float4 vv[32];
#pragma unroll
        for (int kk = 0; kk < 32; ++kk) {
            const size_t ok = (size_t)__shfl_sync(0xffffffffu, (unsigned long long)off, kk);
            vv[kk] = reinterpret_cast<const float4 *>(vc + ok)[lane];
        }
        // butterfly: at offset sh a lane keeps the half of its sums whose key index has bit
        // sh equal to its own lane bit and adds its partner's copy of that half; after five
        // rounds p[0] is the full dot product of key k0 + lane
#pragma unroll
        for (int sh = 16; sh >= 1; sh >>= 1) {
            const bool upper = (lane & sh) != 0;
#pragma unroll
            for (int j = 0; j < sh; ++j) {
                const float keep = upper ? p[j + sh] : p[j];
                const float send = upper ? p[j] : p[j + sh];
                p[j] = keep + __shfl_xor_sync(0xffffffffu, send, sh);
            }
        }
        const float s = key <= last ? __fmul_rn(p[0], scale) : -INFINITY;
        const float mnew = fmaxf(m, warp_max32(s));
        const float alpha = (m == -INFINITY) ? 0.f : expf(m - mnew);
        const float pl = (s == -INFINITY) ? 0.f : expf(s - mnew);
        l = l * alpha + warp_sum32(pl);
        o.x *= alpha;
        o.y *= alpha;
        o.z *= alpha;
        o.w *= alpha;
        m = mnew;
#pragma unroll
        for (int kk = 0; kk < 32; ++kk) {  // in key order over the keys the row sees
            const float pk = __shfl_sync(0xffffffffu, pl, kk);
            if (kk < n) {
                o.x = fmaf(pk, vv[kk].x, o.x);
                o.y = fmaf(pk, vv[kk].y, o.y);
                o.z = fmaf(pk, vv[kk].z, o.z);
                o.w = fmaf(pk, vv[kk].w, o.w);
            }
        }
    }
    if (lane == 0) {
        sm[warp] = m;
        sl[warp] = l;
    }
    so[warp][lane] = o;
    __syncthreads();
    if (warp != 0) return;
    // merge the warps' states in warp order
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kFA; ++w)
        if (sl[w] > 0.f) M = fmaxf(M, sm[w]);
    float L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kFA; ++w) {
        if (!(sl[w] > 0.f)) continue;
        const float f = expf(sm[w] - M);
        const float4 ow = so[w][lane];
        L += sl[w] * f;
        O.x = fmaf(ow.x, f, O.x);
        O.y = fmaf(ow.y, f, O.y);
        O.z = fmaf(ow.z, f, O.z);
        O.w = fmaf(ow.w, f, O.w);
    }
    const float invl = L > 0.f ? __fdiv_rn(1.0f, L) : 0.f;
    float r4[4] = {O.x * invl, O.y * invl, O.z * invl, O.w * invl};
    const size_t ob = (size_t)row * nh * kHD + (size_t)h * kHD + 4 * lane;
    if (gate) {
#pragma unroll
        for (int e = 0; e < 4; ++e) r4[e] = __fmul_rn(r4[e], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gate[ob + e]))));
    }
    *reinterpret_cast<float4 *>(out + ob) = make_float4(r4[0], r4[1], r4[2], r4[3]);
}

__global__ void silu_mul_f32_kernel(const float *__restrict__ gu, size_t rows, int inter, float *__restrict__ out) {
    pdl_entry();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * (size_t)inter) return;
    const size_t r = i / inter;
    const int c = (int)(i % inter);
    const float g = gu[r * 2 * inter + c], u = gu[r * 2 * inter + inter + c];
    out[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

int check_desc_f32(const ekernel_paged_attn_desc_t *d, const char *what) {
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

int ekernel_embedding_f32(const int32_t *ids, size_t rows, const float *table, size_t vocab, size_t hidden,
                          float *out) {
    const char *what = "ekernel_embedding_f32";
    PILM_REQUIRE(ids && table && out, ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(vocab > 0 && vocab <= 0x7fffffff && hidden > 0 && hidden <= (1u << 24) && rows <= 0x7fffffff,
                 ECPU_ERR_PARAM, "%s: sizes out of range", what);
    if (rows == 0) return ECPU_OK;
    int *err = device_error_word();
    PILM_REQUIRE(err, ECPU_ERR_MEM, "%s: error word allocation failed", what);
    launch_pdl(embedding_f32_kernel, dim3((unsigned)rows), dim3(256), 0, ids, (int)rows, table, (int)vocab, (int)hidden, out,
                                                                err);
    const int rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    return check_error_word(what, "a token id was outside the vocabulary");
}

int ekernel_add_rmsnorm_f32(float *residual, const float *delta, const float *weight, size_t rows, size_t n, float eps,
                            int add_one, float *out) {
    const char *what = "ekernel_add_rmsnorm_f32";
    PILM_REQUIRE(residual && weight && out, ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(n > 0 && n <= (1u << 24) && rows <= 0x7fffffff, ECPU_ERR_PARAM, "%s: sizes out of range", what);
    if (rows == 0) return ECPU_OK;
    const dim3 grid((unsigned)rows), block(256);
    if (n <= 1024)
        launch_pdl(add_rmsnorm_f32_kernel<4>, grid, block, 0, residual, delta, weight, (int)n, eps, add_one, out);
    else if (n <= 2048)
        launch_pdl(add_rmsnorm_f32_kernel<8>, grid, block, 0, residual, delta, weight, (int)n, eps, add_one, out);
    else if (n <= 4096)
        launch_pdl(add_rmsnorm_f32_kernel<16>, grid, block, 0, residual, delta, weight, (int)n, eps, add_one, out);
    else if (n <= 8192)
        launch_pdl(add_rmsnorm_f32_kernel<32>, grid, block, 0, residual, delta, weight, (int)n, eps, add_one, out);
    else
        launch_pdl(add_rmsnorm_f32_loop, grid, block, 0, residual, delta, weight, (int)n, eps, add_one, out);
    return check_launch(what);
}

int ekernel_qk_norm_rope_kv_append_f32(const ekernel_paged_attn_desc_t *desc, const float *qkv, const float *q_norm_w,
                                       const float *k_norm_w, const float *rope_cos, const float *rope_sin,
                                       const int32_t *positions, const int32_t *slot_mapping, float *k_cache,
                                       float *v_cache, float *q_out, float *gate_out) {
    const char *what = "ekernel_qk_norm_rope_kv_append_f32";
    int rc = check_desc_f32(desc, what);
    if (rc != ECPU_OK) return rc;
    PILM_REQUIRE(qkv && q_norm_w && k_norm_w && rope_cos && rope_sin && positions && slot_mapping && k_cache &&
                     v_cache && q_out,
                 ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(!desc->output_gate || gate_out, ECPU_ERR_PARAM, "%s: gate_out required when output_gate", what);
    if (desc->total_q == 0) return ECPU_OK;
    const int items = (int)(desc->total_q * (desc->n_heads + desc->n_kv_heads));
    launch_pdl(qk_prologue_f32_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0, 
        qkv, (int)desc->total_q, (int)desc->n_heads, (int)desc->n_kv_heads, (int)desc->qkv_stride, desc->output_gate,
        q_norm_w, k_norm_w, desc->eps, desc->add_one, rope_cos, rope_sin, (int)desc->rope_rows, (int)desc->rot_dim,
        positions, slot_mapping, (long long)desc->num_blocks * (long long)desc->block_size, k_cache, v_cache, q_out,
        gate_out);
    return check_launch(what);
}

int ekernel_paged_attention_verify_f32(const ekernel_paged_attn_desc_t *desc, const float *q, const float *k_cache,
                                       const float *v_cache, const int32_t *block_table, const int32_t *cu_q,
                                       const int32_t *context_lens, const float *gate, float *out) {
    const char *what = "ekernel_paged_attention_verify_f32";
    int rc = check_desc_f32(desc, what);
    if (rc != ECPU_OK) return rc;
    PILM_REQUIRE(q && k_cache && v_cache && block_table && cu_q && context_lens && out, ECPU_ERR_PARAM,
                 "%s: null argument", what);
    PILM_REQUIRE(!desc->output_gate || gate, ECPU_ERR_PARAM, "%s: gate required when output_gate", what);
    if (desc->total_q == 0 || desc->num_seqs == 0) return ECPU_OK;
    const int items = (int)(desc->total_q * desc->n_heads);
    launch_pdl(attn_f32_kernel, dim3((unsigned)items), dim3(kFA * 32), 0, 
        q, k_cache, v_cache, block_table, cu_q, context_lens, desc->output_gate ? gate : nullptr, out,
        (int)desc->num_seqs, (int)desc->total_q, (int)desc->n_heads, (int)desc->n_kv_heads,
        (int)desc->max_blocks_per_seq, (int)desc->num_blocks, (float)(1.0 / sqrt((double)kHD)));
    return check_launch(what);
}

int ekernel_silu_mul_f32(const float *gate_up, size_t rows, size_t inter, float *out) {
    const char *what = "ekernel_silu_mul_f32";
    PILM_REQUIRE(gate_up && out, ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(inter > 0 && inter <= (1u << 24), ECPU_ERR_PARAM, "%s: sizes out of range", what);
    const size_t total = rows * inter;
    if (total == 0) return ECPU_OK;
    launch_pdl(silu_mul_f32_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, gate_up, rows, (int)inter, out);
    return check_launch(what);
}

}  // extern "C"
