// MTP acceptance: row top-2 of the LM-head logits, greedy accept + rollback, and
// rejection sampling with caller-supplied uniforms.
//
// Reference: src/engine.py:479-503 (greedy accept loop over the verify rows),
// :551-557 (bonus token), :505-510 (rollback of num_computed_tokens).  torch.argmax
// returns the first maximal index; the same tie rule is used here.
#include "common.cuh"

using namespace pilm;

namespace {

struct Top2 {
    float v1;
    int i1;
    float v2;
};

__device__ __forceinline__ void top2_push(Top2 &t, float v, int i) {
    if (v > t.v1 || (v == t.v1 && i < t.i1)) {
        t.v2 = fmaxf(t.v2, t.v1);
        t.v1 = v;
        t.i1 = i;
    } else {
        t.v2 = fmaxf(t.v2, v);
    }
}

__device__ __forceinline__ Top2 top2_merge(Top2 a, Top2 b) {
    Top2 r;
    if (b.v1 > a.v1 || (b.v1 == a.v1 && b.i1 < a.i1)) {
        r.v1 = b.v1;
        r.i1 = b.i1;
        r.v2 = fmaxf(fmaxf(a.v1, a.v2), b.v2);
    } else {
        r.v1 = a.v1;
        r.i1 = a.i1;
        r.v2 = fmaxf(fmaxf(b.v1, b.v2), a.v2);
    }
    return r;
}

template <typename T>
__device__ __forceinline__ float ld_logit(const T *p, size_t i);
template <>
__device__ __forceinline__ float ld_logit<float>(const float *p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_logit<__nv_bfloat16>(const __nv_bfloat16 *p, size_t i) { return bf2f(p[i]); }

// the e-th logit held in a 16-byte vector
template <typename T>
__device__ __forceinline__ float vec_logit(const uint4 &r, int e);
template <>
__device__ __forceinline__ float vec_logit<float>(const uint4 &r, int e) {
    const uint32_t w = e == 0 ? r.x : (e == 1 ? r.y : (e == 2 ? r.z : r.w));
    return __uint_as_float(w);
}
template <>
__device__ __forceinline__ float vec_logit<__nv_bfloat16>(const uint4 &r, int e) {
    const int k = e >> 1;
    const uint32_t w = k == 0 ? r.x : (k == 1 ? r.y : (k == 2 ? r.z : r.w));
    return __uint_as_float((e & 1) ? (w & 0xffff0000u) : (w << 16));
}

constexpr int kTop2Threads = 1024;
constexpr int kTop2Unroll = 4;

// One CTA per row.  The row's 16-byte-aligned middle is read with 16-byte loads, four in
// flight per thread (64 KB per CTA), so a single CTA streams its row near an SM's share
// of HBM bandwidth; the unaligned head and tail are read element by element.  The result
// does not depend on the visiting order: ties keep the smallest index, like torch.argmax.
template <typename T>
__global__ void __launch_bounds__(kTop2Threads) row_top2(const T *__restrict__ logits, int rows, int V,
                                                         int32_t *__restrict__ top1, float *__restrict__ top1_val,
                                                         float *__restrict__ margin) {
    pdl_entry();
    __shared__ Top2 sh[kTop2Threads / 32];
    const int row = blockIdx.x;
    if (row >= rows) return;
    const T *x = logits + (size_t)row * V;
    constexpr int E = 16 / sizeof(T);
    const int head = min(V, (int)(((16 - ((uintptr_t)x & 15)) & 15) / sizeof(T)));
    const int nvec = (V - head) / E;
    const int tail0 = head + nvec * E;
    Top2 t{-INFINITY, 0x7fffffff, -INFINITY};
    for (int i = threadIdx.x; i < head; i += blockDim.x) top2_push(t, ld_logit<T>(x, i), i);
    const uint4 *xv = reinterpret_cast<const uint4 *>(x + head);
    for (int v0 = threadIdx.x; v0 < nvec; v0 += kTop2Unroll * blockDim.x) {
        uint4 r[kTop2Unroll];
#pragma unroll
        for (int u = 0; u < kTop2Unroll; ++u) {
            const int v = v0 + u * blockDim.x;
            r[u] = v < nvec ? ldg_nc_v4(xv + v) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kTop2Unroll; ++u) {
            const int v = v0 + u * blockDim.x;
            if (v < nvec) {
#pragma unroll
                for (int e = 0; e < E; ++e) top2_push(t, vec_logit<T>(r[u], e), head + v * E + e);
            }
        }
    }
    for (int i = tail0 + threadIdx.x; i < V; i += blockDim.x) top2_push(t, ld_logit<T>(x, i), i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Top2 u;
        u.v1 = __shfl_xor_sync(0xffffffffu, t.v1, o);
        u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
        u.v2 = __shfl_xor_sync(0xffffffffu, t.v2, o);
        t = top2_merge(t, u);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sh[warp] = t;
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        t = lane < nw ? sh[lane] : Top2{-INFINITY, 0x7fffffff, -INFINITY};
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            Top2 u;
            u.v1 = __shfl_xor_sync(0xffffffffu, t.v1, o);
            u.i1 = __shfl_xor_sync(0xffffffffu, t.i1, o);
            u.v2 = __shfl_xor_sync(0xffffffffu, t.v2, o);
            t = top2_merge(t, u);
        }
        if (lane == 0) {
            if (top1) top1[row] = t.i1;
            if (top1_val) top1_val[row] = t.v1;
            if (margin) margin[row] = t.v1 - t.v2;
        }
    }
}

// one thread per sequence
__global__ void greedy_accept(int B, const int32_t *__restrict__ ids, const int32_t *__restrict__ top1,
                              const int32_t *__restrict__ cu_q, int32_t *__restrict__ acc_out,
                              int32_t *__restrict__ next_out, int32_t *__restrict__ ctx, int32_t *__restrict__ slots) {
    pdl_entry();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int q0 = cu_q[b], q_len = cu_q[b + 1] - q0;
    if (q_len <= 0) {
        acc_out[b] = 0;
        next_out[b] = -1;
        return;
    }
    int acc = 0;
    while (acc < q_len - 1 && top1[q0 + acc] == ids[q0 + 1 + acc]) ++acc;
    acc_out[b] = acc;
    next_out[b] = top1[q0 + acc];
    ctx[b] = ctx[b] - q_len + 1 + acc;
    if (slots)
        for (int j = 1 + acc; j < q_len; ++j) slots[q0 + j] = -1;
}

// ---------------------------------------------------------------------------------
// Rejection sampling
// ---------------------------------------------------------------------------------
constexpr int kRsThreads = 1024;

__device__ __forceinline__ float block_sum(float v, float *sh) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = (lane < (int)(blockDim.x >> 5)) ? sh[lane] : 0.f;
    t = warp_sum(t);
    return t;
}

__device__ __forceinline__ float block_max(float v, float *sh) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float t = (lane < (int)(blockDim.x >> 5)) ? sh[lane] : -INFINITY;
    return warp_max(t);
}

// order-preserving map of a float to an unsigned key
__device__ __forceinline__ uint32_t fkey(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct Nucleus {
    float mx;      // max logit
    uint32_t cut;  // tokens with fkey(logit) >= cut are in the nucleus
    float z;       // sum of e_j over the nucleus, e_j = exp((l_j - mx) / T)
};

// Nucleus of softmax(l / T): {j : mass of strictly more probable tokens < top_p}.
// Bisection over the ordered float keys finds the smallest cut whose strictly-above
// mass is < top_p * Z; every token at or above it is kept (ties kept together).
__device__ Nucleus find_nucleus(const float *x, int V, float T, float top_p, float *sh) {
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, x[i]);
    mx = block_max(mx, sh);
    float z = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) z += expf(__fdiv_rn(x[i] - mx, T));
    z = block_sum(z, sh);
    const float target = top_p * z;
    // smallest key k such that mass(l > key^-1(k-1)...) : search cut in [lo, hi]
    uint32_t lo = 0u, hi = fkey(mx);  // cut = hi keeps only the maxima (always valid)
    while (lo < hi) {
        const uint32_t mid = lo + ((hi - lo) >> 1);
        // mass strictly above the candidate cut value `mid` must be < target for the
        // token(s) at `mid` to be kept; keep searching lower cuts while that holds
        float above = 0.f;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            const float l = x[i];
            if (fkey(l) > mid) above += expf(__fdiv_rn(l - mx, T));
        }
        above = block_sum(above, sh);
        if (above < target)
            hi = mid;
        else
            lo = mid + 1;
    }
    // `hi` is the smallest key whose strictly-above mass is < target; the nucleus is
    // every token with key >= the smallest existing key >= hi
    float zn = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float l = x[i];
        if (fkey(l) >= hi) zn += expf(__fdiv_rn(l - mx, T));
    }
    zn = block_sum(zn, sh);
    return Nucleus{mx, hi, zn};
}

// Inverse-CDF sample in index order over the nucleus with token `skip` removed:
// smallest j with cumsum(e_j) > u * (sum e_j).  Falls back to the last nonzero index.
__device__ int sample_index(const float *x, int V, float T, const Nucleus &nu, int skip, float u, float *sh,
                            float *scan) {
    const int chunk = (V + blockDim.x - 1) / blockDim.x;
    const int i0 = threadIdx.x * chunk, i1 = min(V, i0 + chunk);
    float s = 0.f;
    int last = -1;
    for (int i = i0; i < i1; ++i) {
        const float l = x[i];
        if (i != skip && fkey(l) >= nu.cut) {
            s += expf(__fdiv_rn(l - nu.mx, T));
            last = i;
        }
    }
    // exclusive scan of the chunk sums (sequential over threads for determinism)
    __syncthreads();
    scan[threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float run = 0.f;
        for (int t = 0; t < (int)blockDim.x; ++t) {
            const float v = scan[t];
            scan[t] = run;
            run += v;
        }
        scan[blockDim.x] = run;
    }
    __syncthreads();
    const float total = scan[blockDim.x];
    const float target = u * total;
    __shared__ int s_pick;
    __shared__ int s_last;
    if (threadIdx.x == 0) {
        s_pick = 0x7fffffff;
        s_last = -1;
    }
    __syncthreads();
    if (last >= 0) atomicMax(&s_last, last);
    const float before = scan[threadIdx.x];
    if (before <= target && before + s > target) {
        float run = before;
        for (int i = i0; i < i1; ++i) {
            const float l = x[i];
            if (i != skip && fkey(l) >= nu.cut) {
                run += expf(__fdiv_rn(l - nu.mx, T));
                if (run > target) {
                    atomicMin(&s_pick, i);
                    break;
                }
            }
        }
    }
    __syncthreads();
    int pick = s_pick;
    if (pick == 0x7fffffff) pick = s_last;
    __syncthreads();
    return pick;
}

// one CTA per sequence
__global__ void __launch_bounds__(kRsThreads) rejection_accept(const float *__restrict__ logits, int V,
                                                                const int32_t *__restrict__ ids,
                                                                const int32_t *__restrict__ cu_q,
                                                                const float *__restrict__ uni, float T, float top_p,
                                                                int32_t *__restrict__ acc_out,
                                                                int32_t *__restrict__ next_out,
                                                                int32_t *__restrict__ ctx, int32_t *__restrict__ slots) {
    __shared__ float sh[32];
    __shared__ float scan[kRsThreads + 1];
    const int b = blockIdx.x;
    const int q0 = cu_q[b], q_len = cu_q[b + 1] - q0;
    if (q_len <= 0) {
        if (threadIdx.x == 0) {
            acc_out[b] = 0;
            next_out[b] = -1;
        }
        return;
    }
    int acc = 0, next = -1;
    for (int i = 0; i < q_len; ++i) {
        const float *x = logits + (size_t)(q0 + i) * V;
        const Nucleus nu = find_nucleus(x, V, T, top_p, sh);
        if (i == q_len - 1) {  // bonus row: every draft accepted
            next = sample_index(x, V, T, nu, -1, uni[(size_t)(q0 + i) * 2 + 1], sh, scan);
            break;
        }
        const int d = ids[q0 + 1 + i];
        float pd = 0.f;
        if (d >= 0 && d < V && fkey(x[d]) >= nu.cut) pd = __fdiv_rn(expf(__fdiv_rn(x[d] - nu.mx, T)), nu.z);
        if (uni[(size_t)(q0 + i) * 2 + 0] < pd) {
            ++acc;
            continue;
        }
        next = sample_index(x, V, T, nu, d, uni[(size_t)(q0 + i) * 2 + 1], sh, scan);
        if (next < 0) next = sample_index(x, V, T, nu, -1, uni[(size_t)(q0 + i) * 2 + 1], sh, scan);
        break;
    }
    if (threadIdx.x == 0) {
        acc_out[b] = acc;
        next_out[b] = next;
        ctx[b] = ctx[b] - q_len + 1 + acc;
        if (slots)
            for (int j = 1 + acc; j < q_len; ++j) slots[q0 + j] = -1;
    }
}

}  // namespace

extern "C" {

int ekernel_argmax_top2_f32(const ekernel_accept_desc_t *desc, const float *logits, int32_t *top1, float *top1_val,
                            float *margin) {
    PILM_REQUIRE(desc && logits, ECPU_ERR_PARAM, "ekernel_argmax_top2_f32: null argument");
    PILM_REQUIRE(desc->vocab > 0 && desc->vocab <= 0x7fffffff, ECPU_ERR_PARAM, "ekernel_argmax_top2_f32: bad vocab");
    if (desc->total_q == 0) return ECPU_OK;
    launch_pdl(row_top2<float>, dim3((unsigned)desc->total_q), dim3(kTop2Threads), 0, logits, (int)desc->total_q, (int)desc->vocab, top1,
                                                                   top1_val, margin);
    return check_launch("ekernel_argmax_top2_f32");
}

int ekernel_argmax_top2_bf16(const ekernel_accept_desc_t *desc, const uint16_t *logits, int32_t *top1,
                             float *top1_val, float *margin) {
    PILM_REQUIRE(desc && logits, ECPU_ERR_PARAM, "ekernel_argmax_top2_bf16: null argument");
    PILM_REQUIRE(desc->vocab > 0 && desc->vocab <= 0x7fffffff, ECPU_ERR_PARAM, "ekernel_argmax_top2_bf16: bad vocab");
    if (desc->total_q == 0) return ECPU_OK;
    launch_pdl(row_top2<__nv_bfloat16>, dim3((unsigned)desc->total_q), dim3(kTop2Threads), 0, 
        (const __nv_bfloat16 *)logits, (int)desc->total_q, (int)desc->vocab, top1, top1_val, margin);
    return check_launch("ekernel_argmax_top2_bf16");
}

int ekernel_verify_accept_greedy(const ekernel_accept_desc_t *desc, const int32_t *verify_ids, const int32_t *top1,
                                 const int32_t *cu_q, int32_t *accept_counts, int32_t *next_tokens,
                                 int32_t *context_lens, int32_t *slot_mapping) {
    PILM_REQUIRE(desc && verify_ids && top1 && cu_q && accept_counts && next_tokens && context_lens, ECPU_ERR_PARAM,
                 "ekernel_verify_accept_greedy: null argument");
    if (desc->num_seqs == 0) return ECPU_OK;
    launch_pdl(greedy_accept, dim3((unsigned)((desc->num_seqs + 127) / 128)), dim3(128), 0, 
        (int)desc->num_seqs, verify_ids, top1, cu_q, accept_counts, next_tokens, context_lens, slot_mapping);
    return check_launch("ekernel_verify_accept_greedy");
}

int ekernel_verify_accept_rejection(const ekernel_accept_desc_t *desc, const float *logits,
                                    const int32_t *verify_ids, const int32_t *cu_q, const float *uniforms,
                                    float temperature, float top_p, int32_t *accept_counts, int32_t *next_tokens,
                                    int32_t *context_lens, int32_t *slot_mapping) {
    PILM_REQUIRE(desc && logits && verify_ids && cu_q && uniforms && accept_counts && next_tokens && context_lens,
                 ECPU_ERR_PARAM, "ekernel_verify_accept_rejection: null argument");
    PILM_REQUIRE(temperature > 0.f && top_p > 0.f && top_p <= 1.f, ECPU_ERR_PARAM,
                 "ekernel_verify_accept_rejection: temperature must be > 0 and top_p in (0, 1]");
    PILM_REQUIRE(desc->vocab > 0 && desc->vocab <= 0x7fffffff, ECPU_ERR_PARAM,
                 "ekernel_verify_accept_rejection: bad vocab");
    if (desc->num_seqs == 0) return ECPU_OK;
    rejection_accept<<<(unsigned)desc->num_seqs, kRsThreads, 0, stream()>>>(
        logits, (int)desc->vocab, verify_ids, cu_q, uniforms, temperature, top_p, accept_counts, next_tokens,
        context_lens, slot_mapping);
    return check_launch("ekernel_verify_accept_rejection");
}

}  // extern "C"
