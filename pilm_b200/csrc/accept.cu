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

// The same acceptance from row argmax keys that the LM-head GEMM folded in
// (ekernel_linear_w4a16g128_bf16_kpairs_argmax: value bits << 32 | (0xFFFFFFFF - index)
// per row): each row's key is decoded into top1 and reset to 0 for the next step.
__global__ void greedy_accept_keys(int B, const int32_t *__restrict__ ids, unsigned long long *__restrict__ keys,
                                   const int32_t *__restrict__ cu_q, int32_t *__restrict__ acc_out,
                                   int32_t *__restrict__ next_out, int32_t *__restrict__ ctx,
                                   int32_t *__restrict__ slots, int32_t *__restrict__ top1) {
    pdl_entry();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int q0 = cu_q[b], q_len = cu_q[b + 1] - q0;
    if (q_len <= 0) {
        acc_out[b] = 0;
        next_out[b] = -1;
        return;
    }
    int acc = 0, next = -1;
    bool matching = true;
    for (int j = 0; j < q_len; ++j) {
        const unsigned long long k = keys[q0 + j];
        const int t = k ? (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
        keys[q0 + j] = 0ull;
        if (top1) top1[q0 + j] = t;
        if (matching) {
            if (j < q_len - 1 && t == ids[q0 + 1 + j]) {
                ++acc;
            } else {
                matching = false;
                next = t;
            }
        }
    }
    acc_out[b] = acc;
    next_out[b] = next;
    ctx[b] = ctx[b] - q_len + 1 + acc;
    if (slots)
        for (int j = 1 + acc; j < q_len; ++j) slots[q0 + j] = -1;
}

// ---------------------------------------------------------------------------------
// Rejection sampling (standard speculative sampling with a one-hot greedy draft; the
// reference has none).  Two kernels:
//   rs_row_stats     one CTA per verify row, all rows in parallel: the row's target
//                    distribution p = softmax(l / T) restricted to the nucleus {j : mass of
//                    strictly more probable tokens < top_p}, as its max logit, the nucleus
//                    cut (the smallest order-preserving key kept) and nucleus mass, and the
//                    mass of the draft that the row verifies
//   rs_decide_sample one CTA per sequence: the accept tests u < p(d) row by row from those
//                    statistics, then the next token by inverse CDF in token-index order
//                    from the first rejected row with its draft removed, or from the bonus
//                    row, and the rollback
// Masses e_j = exp((l_j - mx) / T) <= 1 are summed in unsigned 64-bit fixed point with 40
// fractional bits.  Integer sums do not depend on the order of summation, so every pass,
// thread count and launch agrees exactly; V < 2^23 keeps them below 2^63.  The nucleus cut
// takes three reads of the row: its max; a histogram of masses over 2048 linear bins of
// (mx - l) / T (one shared-memory atomic per token of nonzero mass), which locates the bin
// holding the cut; and a gather of that bin's
// tokens (at most 2048), among which the cut is found by exact pairwise comparison.  A cut
// bin with more tokens falls back to a radix select over the 32-bit keys of the whole row
// (11 + 11 + 10 bits, three more reads).
// ---------------------------------------------------------------------------------
constexpr int kRsThreads = 1024;
constexpr int kRsBins = 2048;
constexpr double kFix = 1099511627776.0;  // 2^40

struct RsRow {
    float mx;               // max logit
    uint32_t cut;           // keys >= cut are in the nucleus
    unsigned long long zn;  // nucleus mass (fixed point)
    unsigned long long ed;  // mass of the draft this row verifies if in the nucleus, else 0
};

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

template <typename T>
__device__ __forceinline__ float logit_at(const T *x, int i) {
    if constexpr (sizeof(T) == 2) return __bfloat162float(x[i]);
    else return x[i];
}

// f(i, logit) for every token of a row, spread over the block; bf16 rows on 16-byte
// boundaries are read 8 logits per load
template <typename T, typename F>
__device__ __forceinline__ void row_for_each(const T *x, int V, F &&f) {
    if constexpr (sizeof(T) == 2) {
        if ((((uintptr_t)x) & 15) == 0) {
            const int nv = V >> 3;
            const uint4 *xv = reinterpret_cast<const uint4 *>(x);
            for (int v = threadIdx.x; v < nv; v += blockDim.x) {
                const uint4 w = __ldg(xv + v);
                const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    f(8 * v + 2 * e, __uint_as_float(wd[e] << 16));
                    f(8 * v + 2 * e + 1, __uint_as_float(wd[e] & 0xffff0000u));
                }
            }
            for (int i = 8 * nv + threadIdx.x; i < V; i += blockDim.x) f(i, logit_at(x, i));
            return;
        }
    }
    for (int i = threadIdx.x; i < V; i += blockDim.x) f(i, logit_at(x, i));
}

// the mass of a token: exp((l - mx) / T) in fixed point; every pass and both kernels use
// this one function, so their sums agree exactly
__device__ __forceinline__ unsigned long long rs_mass(float l, float mx, float inv_t) {
    const float e = expf(-((mx - l) * inv_t));  // in [0, 1]
    return __double2ull_rn((double)e * kFix);
}

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// block-wide sum (every thread gets it); wsum holds 32 slots
__device__ unsigned long long block_sum_u64(unsigned long long v, unsigned long long *wsum) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_u64(v);
    __syncthreads();
    if (lane == 0) wsum[warp] = v;
    __syncthreads();
    unsigned long long t = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0ull;
    return warp_sum_u64(t);
}

// Inclusive suffix sums of kRsBins values held two per thread: sfx[d] = sum of bins[d..]
// (kRsThreads threads).
__device__ void suffix_sums(const unsigned long long *bins, unsigned long long *sfx, unsigned long long *wsum) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    // reverse order: thread t handles bins kRsBins-1-2t and kRsBins-2-2t, so a prefix scan
    // over threads is a suffix scan over bins
    const int hi = kRsBins - 1 - 2 * t, lo = hi - 1;
    const unsigned long long a = bins[hi], b = bins[lo];
    unsigned long long v = a + b, x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        unsigned long long w = wsum[lane], z = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(0xffffffffu, z, o);
            if (lane >= o) z += y;
        }
        wsum[lane] = z - w;  // exclusive over warps
    }
    __syncthreads();
    const unsigned long long before = wsum[warp] + x - v;  // sum of bins above `hi`
    sfx[hi] = before + a;
    sfx[lo] = before + a + b;
    __syncthreads();
}

// Level 0 bins tokens linearly by u = (mx - l) / T: bin floor(u * kRsBins / kRsSpan), the
// last bin collecting u >= kRsSpan (masses below 2^-57).  A bin index never decreases as
// the logit decreases, so bins order the tokens by logit, ties kept together.
constexpr float kRsSpan = 40.f;
constexpr int kRsGather = 2048;  // tokens of the cut's bin resolved by pairwise comparison

__device__ __forceinline__ int rs_bin(float l, float mx, float inv_t) {
    const float u = (mx - l) * inv_t;
    return u < kRsSpan ? min(kRsBins - 1, (int)(u * (kRsBins / kRsSpan))) : kRsBins - 1;
}

// Level 0 adds each token's mass to one of kRsSub copies of the histogram (warp w to copy
// w % kRsSub): lanes of a warp still collide on bins near the mode, but warps no longer
// collide with most other warps.  Integer sums, so the copies' sum is the same whatever
// the split.  After the copies are summed, sub[0] is the histogram (hist) and sub[1] its
// suffix sums (sfx); sub[2] and sub[3] hold the gather of the cut's bin.
constexpr int kRsSub = 4;
static_assert(kRsGather <= kRsBins, "the gather fits in one histogram copy");

struct RsSmem {
    unsigned long long sub[kRsSub][kRsBins];
    unsigned long long wsum[32];
    float shf[32];
    int s_bin, s_n;
    uint32_t s_cut;
    __device__ unsigned long long *hist() { return sub[0]; }  // level-0 masses; later the fallback's histograms
    __device__ unsigned long long *sfx() { return sub[1]; }
    __device__ unsigned long long *gmass() { return sub[2]; }
    __device__ uint32_t *gkey() { return reinterpret_cast<uint32_t *>(sub[3]); }
};

// Fallback for a cut bin with more than kRsGather tokens: radix select over the 32-bit keys
// (11 + 11 + 10 bits) of the whole row for the lowest present key whose strictly-above mass
// is < target; returns the cut and the nucleus mass.
template <typename T>
__device__ void rs_radix_cut(const T *x, int V, float mx, float inv_t, double target, RsSmem &sm, uint32_t &cut,
                             unsigned long long &zn) {
    constexpr int kBits[3] = {11, 11, 10};
    uint32_t prefix = 0;
    int consumed = 0;
    unsigned long long above = 0, at_cut = 0;
    for (int lv = 0; lv < 3; ++lv) {
        const int bits = kBits[lv];
        const int shift = 32 - consumed - bits;
        for (int d = threadIdx.x; d < kRsBins; d += blockDim.x) sm.hist()[d] = 0;
        __syncthreads();
        row_for_each(x, V, [&](int, float l) {
            const uint32_t k = fkey(l);
            if (consumed == 0 || (k >> (32 - consumed)) == prefix)
                atomicAdd(&sm.hist()[(k >> shift) & ((1u << bits) - 1)], rs_mass(l, mx, inv_t));
        });
        __syncthreads();
        suffix_sums(sm.hist(), sm.sfx(), sm.wsum);
        if (threadIdx.x == 0) sm.s_bin = kRsBins;
        __syncthreads();
        for (int d = threadIdx.x; d < (1 << bits); d += blockDim.x) {
            const unsigned long long higher = above + sm.sfx()[d] - sm.hist()[d];
            if (sm.hist()[d] && (double)higher < target) atomicMin(&sm.s_bin, d);
        }
        __syncthreads();
        int dg = sm.s_bin;
        if (dg == kRsBins) dg = 0;
        above += sm.sfx()[dg] - sm.hist()[dg];
        at_cut = sm.hist()[dg];
        prefix = (prefix << bits) | (uint32_t)dg;
        consumed += bits;
        __syncthreads();
    }
    cut = prefix;
    zn = above + at_cut;
}

template <typename T>
__global__ void __launch_bounds__(kRsThreads) rs_row_stats(const T *__restrict__ logits, int rows, int V,
                                                            const int32_t *__restrict__ ids, float temp, float top_p,
                                                            RsRow *__restrict__ out) {
    pdl_entry();
    extern __shared__ __align__(16) uint8_t rs_smem_raw[];
    RsSmem &sm = *reinterpret_cast<RsSmem *>(rs_smem_raw);
    const int r = blockIdx.x;
    const T *x = logits + (size_t)r * V;
    const float inv_t = __fdiv_rn(1.0f, temp);
    float mx = -INFINITY;
    row_for_each(x, V, [&](int, float l) { mx = fmaxf(mx, l); });
    mx = block_max(mx, sm.shf);

    // level 0: masses per bin.  Only tokens of nonzero fixed-point mass are added: a
    // token of zero mass has the whole total strictly above it, so it is never in the
    // nucleus (top_p <= 1); and since masses never grow with distance from the max, a bin
    // holding only such tokens is followed by such bins only, so "the last bin of nonzero
    // mass whose higher bins hold less than the target" is the bin of the cut.  The
    // catch-all bin (u >= kRsSpan) holds masses below 2^-57, zero in fixed point.
    for (int d = threadIdx.x; d < kRsSub * kRsBins; d += blockDim.x) (&sm.sub[0][0])[d] = 0;
    __syncthreads();
    unsigned long long *mine = sm.sub[(threadIdx.x >> 5) % kRsSub];
    row_for_each(x, V, [&](int, float l) {
        const int bn = rs_bin(l, mx, inv_t);
        if (bn == kRsBins - 1) return;
        const unsigned long long m = rs_mass(l, mx, inv_t);
        if (m) atomicAdd(&mine[bn], m);
    });
    __syncthreads();
    for (int d = threadIdx.x; d < kRsBins; d += blockDim.x) {
        unsigned long long v = sm.sub[0][d];
#pragma unroll
        for (int c = 1; c < kRsSub; ++c) v += sm.sub[c][d];
        sm.sub[0][d] = v;
    }
    __syncthreads();
    suffix_sums(sm.hist(), sm.sfx(), sm.wsum);
    const unsigned long long total = sm.sfx()[0];
    const double target = (double)top_p * (double)total;  // the nucleus keeps above-mass < top_p Z
    if (threadIdx.x == 0) sm.s_bin = -1;
    __syncthreads();
    for (int d = threadIdx.x; d < kRsBins; d += blockDim.x) {
        const unsigned long long higher = total - sm.sfx()[d];  // mass of bins before d
        if (sm.hist()[d] && (double)higher < target) atomicMax(&sm.s_bin, d);
    }
    if (threadIdx.x == 0) {
        sm.s_n = 0;
        sm.s_cut = 0xffffffffu;
    }
    __syncthreads();
    const int bstar = sm.s_bin;
    const unsigned long long base = total - sm.sfx()[bstar];  // mass strictly above the cut's bin
    uint32_t cut;
    unsigned long long zn;
    // gather the bin's tokens (slots past kRsGather are counted, not stored); a token's
    // above-mass is base + the masses of the bin's tokens with a greater key, and the cut
    // is the smallest key whose above-mass < target
    row_for_each(x, V, [&](int, float l) {
        if (rs_bin(l, mx, inv_t) == bstar) {
            const int slot = atomicAdd(&sm.s_n, 1);
            if (slot < kRsGather) {
                sm.gkey()[slot] = fkey(l);
                sm.gmass()[slot] = rs_mass(l, mx, inv_t);
            }
        }
    });
    __syncthreads();
    if (sm.s_n <= kRsGather) {
        const int n = sm.s_n;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t ki = sm.gkey()[i];
            unsigned long long above = base;
            for (int j = 0; j < n; ++j)
                if (sm.gkey()[j] > ki) above += sm.gmass()[j];
            if ((double)above < target) atomicMin(&sm.s_cut, ki);
        }
        __syncthreads();
        cut = sm.s_cut;
        unsigned long long in_bin = 0;
        for (int i = threadIdx.x; i < n; i += blockDim.x)
            if (sm.gkey()[i] >= cut) in_bin += sm.gmass()[i];
        zn = base + block_sum_u64(in_bin, sm.wsum);
    } else {
        rs_radix_cut(x, V, mx, inv_t, target, sm, cut, zn);
    }
    if (threadIdx.x == 0) {
        RsRow o;
        o.mx = mx;
        o.cut = cut;
        o.zn = zn;
        o.ed = 0;
        if (r + 1 < rows) {
            const int d = ids[r + 1];
            if (d >= 0 && d < V) {
                const float l = logit_at(x, d);
                if (fkey(l) >= cut) o.ed = rs_mass(l, mx, inv_t);
            }
        }
        out[r] = o;
    }
}

template <typename T>
__global__ void __launch_bounds__(kRsThreads) rs_decide_sample(const T *__restrict__ logits, int V,
                                                                const int32_t *__restrict__ ids,
                                                                const int32_t *__restrict__ cu_q,
                                                                const float *__restrict__ uni, float temp,
                                                                const RsRow *__restrict__ stats,
                                                                int32_t *__restrict__ acc_out,
                                                                int32_t *__restrict__ next_out,
                                                                int32_t *__restrict__ ctx, int32_t *__restrict__ slots) {
    pdl_entry();
    __shared__ unsigned long long wsum[32];
    __shared__ int s_row, s_skip, s_acc, s_pick, s_last;
    const int b = blockIdx.x;
    const int q0 = cu_q[b], q_len = cu_q[b + 1] - q0;
    if (q_len <= 0) {
        if (threadIdx.x == 0) {
            acc_out[b] = 0;
            next_out[b] = -1;
        }
        return;
    }
    if (threadIdx.x == 0) {
        int acc = 0, row = q0 + q_len - 1, skip = -1;
        for (int i = 0; i + 1 < q_len; ++i) {
            const RsRow st = stats[q0 + i];
            const double pd = st.zn ? (double)st.ed / (double)st.zn : 0.0;
            if ((double)uni[(size_t)(q0 + i) * 2] < pd) {
                ++acc;
                continue;
            }
            row = q0 + i;
            skip = ids[q0 + 1 + i];
            break;
        }
        s_row = row;
        s_skip = skip;
        s_acc = acc;
        s_pick = 0x7fffffff;
        s_last = -1;
    }
    __syncthreads();
    const int row = s_row;
    const RsRow st = stats[row];
    int skip = s_skip;
    unsigned long long total = st.zn;
    if (skip >= 0) {
        if (st.ed == st.zn) skip = -1;  // the draft was the whole nucleus: sample from p itself
        else total -= st.ed;
    }
    const T *x = logits + (size_t)row * V;
    const float inv_t = __fdiv_rn(1.0f, temp);
    // chunk sums over contiguous index ranges (a multiple of 8 logits each, so bf16 rows on
    // 16-byte boundaries are read 8 logits per load), then the chunk that crosses u x total
    const int chunk = ((V + blockDim.x * 8 - 1) / (blockDim.x * 8)) * 8;
    const int i0 = min(V, (int)threadIdx.x * chunk), i1 = min(V, i0 + chunk);
    const bool vec8 = sizeof(T) == 2 && (((uintptr_t)x) & 15) == 0;
    unsigned long long s = 0;
    int last = -1;
    auto visit = [&](int i, float l) {
        if (i != skip && fkey(l) >= st.cut) {
            s += rs_mass(l, st.mx, inv_t);
            last = i;
        }
    };
    if (vec8) {
        int i = i0;
        for (; i + 8 <= i1; i += 8) {
            const uint4 w = __ldg(reinterpret_cast<const uint4 *>(x + i));
            const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                visit(i + 2 * e, __uint_as_float(wd[e] << 16));
                visit(i + 2 * e + 1, __uint_as_float(wd[e] & 0xffff0000u));
            }
        }
        for (; i < i1; ++i) visit(i, logit_at(x, i));
    } else {
        for (int i = i0; i < i1; ++i) visit(i, logit_at(x, i));
    }
    if (last >= 0) atomicMax(&s_last, last);
    // exclusive prefix over threads
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        unsigned long long w = wsum[lane], z = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(0xffffffffu, z, o);
            if (lane >= o) z += y;
        }
        wsum[lane] = z - w;
    }
    __syncthreads();
    const unsigned long long before = wsum[warp] + incl - s;
    const double target = (double)uni[(size_t)row * 2 + 1] * (double)total;
    if ((double)before <= target && (double)(before + s) > target) {
        unsigned long long run = before;
        for (int i = i0; i < i1; ++i) {
            const float l = logit_at(x, i);
            if (i != skip && fkey(l) >= st.cut) {
                run += rs_mass(l, st.mx, inv_t);
                if ((double)run > target) {
                    atomicMin(&s_pick, i);
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int acc = s_acc;
        const int next = s_pick != 0x7fffffff ? s_pick : s_last;
        acc_out[b] = acc;
        next_out[b] = next;
        ctx[b] = ctx[b] - q_len + 1 + acc;
        if (slots)
            for (int j = 1 + acc; j < q_len; ++j) slots[q0 + j] = -1;
    }
}

template <typename T>
int launch_rejection(const ekernel_accept_desc_t *desc, const T *logits, const int32_t *verify_ids,
                     const int32_t *cu_q, const float *uniforms, float temperature, float top_p,
                     int32_t *accept_counts, int32_t *next_tokens, int32_t *context_lens, int32_t *slot_mapping,
                     const char *what) {
    PILM_REQUIRE(desc && logits && verify_ids && cu_q && uniforms && accept_counts && next_tokens && context_lens,
                 ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(temperature > 0.f && top_p > 0.f && top_p <= 1.f, ECPU_ERR_PARAM,
                 "%s: temperature must be > 0 and top_p in (0, 1]", what);
    PILM_REQUIRE(desc->vocab > 0 && desc->vocab < (1u << 23), ECPU_ERR_PARAM, "%s: vocab must be in [1, 2^23)", what);
    PILM_REQUIRE(desc->total_q <= 0x7fffffff, ECPU_ERR_PARAM, "%s: too many rows", what);
    if (desc->num_seqs == 0) return ECPU_OK;
    RsRow *stats = nullptr;
    if (desc->total_q > 0) {
        stats = (RsRow *)scratch(kScratchAccept, desc->total_q * sizeof(RsRow));
        PILM_REQUIRE(stats, ECPU_ERR_MEM, "%s: workspace allocation failed", what);
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(rs_row_stats<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(RsSmem));
            attr = true;
        }
        launch_pdl(rs_row_stats<T>, dim3((unsigned)desc->total_q), dim3(kRsThreads), sizeof(RsSmem), logits,
                   (int)desc->total_q, (int)desc->vocab, verify_ids, temperature, top_p, stats);
        const int rc = check_launch(what);
        if (rc != ECPU_OK) return rc;
    }
    launch_pdl(rs_decide_sample<T>, dim3((unsigned)desc->num_seqs), dim3(kRsThreads), 0, logits, (int)desc->vocab,
               verify_ids, cu_q, uniforms, temperature, (const RsRow *)stats, accept_counts, next_tokens,
               context_lens, slot_mapping);
    return check_launch(what);
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

int ekernel_verify_accept_greedy_keys(const ekernel_accept_desc_t *desc, const int32_t *verify_ids,
                                      uint64_t *row_keys, const int32_t *cu_q, int32_t *accept_counts,
                                      int32_t *next_tokens, int32_t *context_lens, int32_t *slot_mapping,
                                      int32_t *top1) {
    PILM_REQUIRE(desc && verify_ids && row_keys && cu_q && accept_counts && next_tokens && context_lens,
                 ECPU_ERR_PARAM, "ekernel_verify_accept_greedy_keys: null argument");
    if (desc->num_seqs == 0) return ECPU_OK;
    launch_pdl(greedy_accept_keys, dim3((unsigned)((desc->num_seqs + 127) / 128)), dim3(128), 0, (int)desc->num_seqs,
               verify_ids, (unsigned long long *)row_keys, cu_q, accept_counts, next_tokens, context_lens,
               slot_mapping, top1);
    return check_launch("ekernel_verify_accept_greedy_keys");
}

int ekernel_verify_accept_rejection(const ekernel_accept_desc_t *desc, const float *logits,
                                    const int32_t *verify_ids, const int32_t *cu_q, const float *uniforms,
                                    float temperature, float top_p, int32_t *accept_counts, int32_t *next_tokens,
                                    int32_t *context_lens, int32_t *slot_mapping) {
    return launch_rejection(desc, logits, verify_ids, cu_q, uniforms, temperature, top_p, accept_counts, next_tokens,
                            context_lens, slot_mapping, "ekernel_verify_accept_rejection");
}

int ekernel_verify_accept_rejection_bf16(const ekernel_accept_desc_t *desc, const uint16_t *logits,
                                         const int32_t *verify_ids, const int32_t *cu_q, const float *uniforms,
                                         float temperature, float top_p, int32_t *accept_counts,
                                         int32_t *next_tokens, int32_t *context_lens, int32_t *slot_mapping) {
    return launch_rejection(desc, (const __nv_bfloat16 *)logits, verify_ids, cu_q, uniforms, temperature, top_p,
                            accept_counts, next_tokens, context_lens, slot_mapping,
                            "ekernel_verify_accept_rejection_bf16");
}

}  // extern "C"
