/*
 * TEST INFRASTRUCTURE -- the parity oracle, not the product.
 *
 * A plain-C restatement of the piLM CPU kernels that the MTP verify path calls
 * (reference: src/ecpu/src/kernel/kernels.c).  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg load this library, and only to check or time
 * the CUDA path.  Nothing in pilm_b200/ links against it.
 *
 * Arithmetic contract: the reference's AVX2 kernels accumulate in eight fp32
 * lanes with fused multiply-adds and reduce the lanes in a fixed tree
 * (hsum256_ps, kernels.c:56-63).  This file reproduces that lane assignment,
 * FMA placement and reduction order with scalar code, so its outputs are
 * bit-identical to the reference library built with the same toolchain.  The
 * reference is built -std=gnu11, where gcc contracts `a += b * c` into an FMA;
 * those statements are written here as explicit fmaf() and the file is compiled
 * with -ffp-contract=off so nothing else gets contracted.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_ERR_PARAM (-1)
#define ORC_ERR_MEM (-2)
#define ORC_ERR_UNSUPPORTED (-5)

/* bf16 <-> fp32, kernels.c:12-25: truncating widen; RNE narrow without NaN handling. */
static inline float bf16_to_f32(uint16_t x) {
    uint32_t bits = ((uint32_t)x) << 16;
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

static inline uint16_t f32_to_bf16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, sizeof(bits));
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

/* int4 nibble decode, kernels.c:43-46: even k in the low nibble, two's complement. */
static inline int nib(uint8_t packed, int high) {
    int v = high ? (packed >> 4) : (packed & 0x0F);
    return v >= 8 ? v - 16 : v;
}

/* Eight-lane horizontal sum in the order of hsum256_ps (kernels.c:56-63):
 * (l0+l4, l1+l5, l2+l6, l3+l7) -> pairwise hadd -> ((s0+s1)+(s2+s3)). */
static inline float hsum8(const float l[8]) {
    float s0 = l[0] + l[4], s1 = l[1] + l[5], s2 = l[2] + l[6], s3 = l[3] + l[7];
    float a = s0 + s1, b = s2 + s3;
    return a + b;
}

/* dot_bf16_i4_packed_avx2 (kernels.c:111-154) and the per-row body of
 * dot_bf16_i4_8_packed_avx2 (kernels.c:168-225): blocks of 16 k; k..k+7 go to
 * accumulator 0 and k+8..k+15 to accumulator 1, one lane per k mod 8; the two
 * accumulators are added lane-wise before the horizontal sum; the remainder is
 * added pairwise with contracted FMAs. */
static float dot_bf16_i4(const uint16_t *a, const uint8_t *w, size_t K) {
    float acc0[8] = {0}, acc1[8] = {0};
    size_t k = 0;
    for (; k + 16 <= K; k += 16) {
        for (int l = 0; l < 8; l++) {
            int kk = (int)k + l;
            acc0[l] = fmaf(bf16_to_f32(a[kk]), (float)nib(w[kk / 2], kk & 1), acc0[l]);
        }
        for (int l = 0; l < 8; l++) {
            int kk = (int)k + 8 + l;
            acc1[l] = fmaf(bf16_to_f32(a[kk]), (float)nib(w[kk / 2], kk & 1), acc1[l]);
        }
    }
    float lanes[8];
    for (int l = 0; l < 8; l++) lanes[l] = acc0[l] + acc1[l];
    float out = hsum8(lanes);
    for (; k + 1 < K; k += 2) {
        uint8_t p = w[k / 2];
        out = fmaf(bf16_to_f32(a[k + 0]), (float)nib(p, 0), out);
        out = fmaf(bf16_to_f32(a[k + 1]), (float)nib(p, 1), out);
    }
    if (k < K) out = fmaf(bf16_to_f32(a[k]), (float)nib(w[k / 2], 0), out);
    return out;
}

/* dot_f32_i8_avx2 (kernels.c:77-91): one 8-lane accumulator.  The scalar remainder
 * is NOT contracted in the reference build (pinned against oracle/_ref/libecpu.so). */
static float dot_f32_i8(const float *a, const int8_t *w, size_t K) {
    float acc[8] = {0};
    size_t k = 0;
    for (; k + 8 <= K; k += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(a[k + l], (float)w[k + l], acc[l]);
    float out = hsum8(acc);
    for (; k < K; k++) out += a[k] * (float)w[k];
    return out;
}

/* dot_bf16_i8_avx2 / dot_bf16_i8_{4,8}_avx2 (kernels.c:93-109, 227-356): identical
 * per-row structure to dot_f32_i8 with bf16 activations. */
static float dot_bf16_i8(const uint16_t *a, const int8_t *w, size_t K) {
    float acc[8] = {0};
    size_t k = 0;
    for (; k + 8 <= K; k += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(bf16_to_f32(a[k + l]), (float)w[k + l], acc[l]);
    float out = hsum8(acc);
    for (; k < K; k++) out = fmaf(bf16_to_f32(a[k]), (float)w[k], out);
    return out;
}

/* dot_f32_f32_avx2 (kernels.c:64-75). */
static float dot_f32_f32(const float *a, const float *b, size_t K) {
    float acc[8] = {0};
    size_t k = 0;
    for (; k + 8 <= K; k += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(a[k + l], b[k + l], acc[l]);
    float out = hsum8(acc);
    for (; k < K; k++) out = fmaf(a[k], b[k], out);
    return out;
}

/* ekernel_gemm (kernels.c:396-435), F32 only; the AVX2 dot is used when B is
 * transposed and A is not, otherwise a contracted scalar loop. */
int orc_gemm_f32(size_t M, size_t N, size_t K, const float *A, const float *B, float *C,
                 int transpose_a, int transpose_b) {
    if (!A || !B || !C) return ORC_ERR_PARAM;
    const size_t lda = transpose_a ? M : K;
    const size_t ldb = transpose_b ? K : N;
#pragma omp parallel for collapse(2) if (M * N >= 256)
    for (long long mi = 0; mi < (long long)M; mi++) {
        for (long long ni = 0; ni < (long long)N; ni++) {
            size_t m = (size_t)mi, n = (size_t)ni;
            float acc;
            if (!transpose_a && transpose_b) {
                acc = dot_f32_f32(A + m * lda, B + n * ldb, K);
            } else {
                acc = 0.0f;
                for (size_t k = 0; k < K; k++) {
                    float av = transpose_a ? A[k * lda + m] : A[m * lda + k];
                    float bv = transpose_b ? B[n * ldb + k] : B[k * ldb + n];
                    acc = fmaf(av, bv, acc);
                }
            }
            C[m * N + n] = acc;
        }
    }
    return ORC_OK;
}

/* ekernel_linear_w8a32 (kernels.c:437-467): C = dot(A_m, W_n) * s_n in fp32. */
int orc_linear_w8a32(size_t M, size_t N, size_t K, const float *A, const int8_t *W,
                     const float *scales, float *C) {
    if (!A || !W || !scales || !C) return ORC_ERR_PARAM;
#pragma omp parallel for collapse(2) if (M * N >= 256)
    for (long long mi = 0; mi < (long long)M; mi++)
        for (long long ni = 0; ni < (long long)N; ni++)
            C[mi * N + ni] = dot_f32_i8(A + mi * K, W + ni * K, K) * scales[ni];
    return ORC_OK;
}

/* ekernel_linear_w8a16_bf16 default path (kernels.c:469-612): bf16(dot * s_n). */
int orc_linear_w8a16_bf16(size_t M, size_t N, size_t K, const uint16_t *A, const int8_t *W,
                          const float *scales, uint16_t *C) {
    if (!A || !W || !scales || !C) return ORC_ERR_PARAM;
#pragma omp parallel for collapse(2) if (M * N >= 256)
    for (long long mi = 0; mi < (long long)M; mi++)
        for (long long ni = 0; ni < (long long)N; ni++)
            C[mi * N + ni] = f32_to_bf16(dot_bf16_i8(A + mi * K, W + ni * K, K) * scales[ni]);
    return ORC_OK;
}

/* ekernel_linear_w8a16_bf16_argmax (kernels.c:658-737): M=1; the value compared is
 * the bf16-rounded logit; ties resolve to the lowest index. */
int orc_linear_w8a16_bf16_argmax(size_t M, size_t N, size_t K, const uint16_t *A,
                                 const int8_t *W, const float *scales, size_t *out_index,
                                 float *out_value) {
    if (!A || !W || !scales || !out_index || !out_value) return ORC_ERR_PARAM;
    if (M != 1 || N == 0 || K == 0) return ORC_ERR_UNSUPPORTED;
    size_t best = 0;
    float bestv = -INFINITY;
    for (size_t n = 0; n < N; n++) {
        float v = bf16_to_f32(f32_to_bf16(dot_bf16_i8(A, W + n * K, K) * scales[n]));
        if (v > bestv) { bestv = v; best = n; }
    }
    *out_index = best;
    *out_value = bestv;
    return ORC_OK;
}

/* ekernel_linear_w4a16_bf16 (kernels.c:1002-1087): per-output-row fp32 scale. */
int orc_linear_w4a16_bf16(size_t M, size_t N, size_t K, const uint16_t *A, const uint8_t *W,
                          const float *scales, uint16_t *C) {
    if (!A || !W || !scales || !C) return ORC_ERR_PARAM;
    const size_t pk = (K + 1) / 2;
#pragma omp parallel for collapse(2) if (M * N >= 256)
    for (long long mi = 0; mi < (long long)M; mi++)
        for (long long ni = 0; ni < (long long)N; ni++)
            C[mi * N + ni] = f32_to_bf16(dot_bf16_i4(A + mi * K, W + ni * pk, K) * scales[ni]);
    return ORC_OK;
}

/* linear_w4a16g_bf16_impl (kernels.c:1089-1139): per group g of `group` k values,
 * acc = acc + dot_g * s[n,g] with the product rounded before the add (the reference
 * build does not contract this statement; pinned against oracle/_ref/libecpu.so),
 * then one bf16 rounding. */
int orc_linear_w4a16g_bf16(size_t M, size_t N, size_t K, const uint16_t *A, const uint8_t *W,
                           const float *scales, uint16_t *C, size_t group) {
    if (!A || !W || !scales || !C || group == 0) return ORC_ERR_PARAM;
    const size_t G = (K + group - 1) / group;
    const size_t pk = (K + 1) / 2;
#pragma omp parallel for collapse(2) if (M * N >= 256)
    for (long long mi = 0; mi < (long long)M; mi++) {
        for (long long ni = 0; ni < (long long)N; ni++) {
            const uint16_t *a = A + mi * K;
            const uint8_t *w = W + ni * pk;
            const float *s = scales + ni * G;
            float acc = 0.0f;
            for (size_t g = 0; g < G; g++) {
                size_t k0 = g * group;
                size_t gk = K - k0 < group ? K - k0 : group;
                float block = dot_bf16_i4(a + k0, w + k0 / 2, gk);
                acc = acc + block * s[g];
            }
            C[mi * N + ni] = f32_to_bf16(acc);
        }
    }
    return ORC_OK;
}

/* ekernel_rmsnorm_bf16 (kernels.c:1485-1526): 8-lane sum of squares, contracted
 * tail, inv = 1/sqrtf(ss/n + eps), y = bf16((x * inv) * (w [+1])). */
int orc_rmsnorm_bf16(const uint16_t *x, uint16_t *out, const uint16_t *weight, size_t rows,
                     size_t n, float eps, int add_one) {
    if (!x || !out || !weight || rows == 0 || n == 0) return ORC_ERR_PARAM;
#pragma omp parallel for if (rows >= 8)
    for (long long ri = 0; ri < (long long)rows; ri++) {
        const uint16_t *xr = x + ri * n;
        uint16_t *o = out + ri * n;
        float acc[8] = {0};
        size_t i = 0;
        for (; i + 8 <= n; i += 8)
            for (int l = 0; l < 8; l++) {
                float v = bf16_to_f32(xr[i + l]);
                acc[l] = fmaf(v, v, acc[l]);
            }
        float ss = hsum8(acc);
        for (; i < n; i++) {
            float v = bf16_to_f32(xr[i]);
            ss = fmaf(v, v, ss);
        }
        float inv = 1.0f / sqrtf(ss / (float)n + eps);
        for (i = 0; i < n; i++) {
            float w = bf16_to_f32(weight[i]);
            if (add_one) w += 1.0f;
            float v = bf16_to_f32(xr[i]) * inv * w;
            o[i] = f32_to_bf16(v);
        }
    }
    return ORC_OK;
}

/* ekernel_swiglu_bf16 (kernels.c:1580-1596): bf16(g / (1 + expf(-g)) * u). */
int orc_swiglu_bf16(const uint16_t *gate, const uint16_t *up, uint16_t *out, size_t n) {
    if (!gate || !up || !out) return ORC_ERR_PARAM;
    for (size_t i = 0; i < n; i++) {
        float g = bf16_to_f32(gate[i]);
        float u = bf16_to_f32(up[i]);
        float silu = g / (1.0f + expf(-g));
        out[i] = f32_to_bf16(silu * u);
    }
    return ORC_OK;
}

/* ekernel_swiglu_w4a16_bf16 (kernels.c:1598-1735): M=1 only, per-row W4 scales.
 * gate/up rows are [0,I) and [I,2I) of gate_up_W; each projection is rounded to
 * bf16 before the activation; the hidden vector is bf16; then the down linear. */
int orc_swiglu_w4a16_bf16(size_t M, size_t H, size_t I, size_t K, size_t down_in,
                          const uint16_t *A, const uint8_t *gate_up_W, const float *gate_up_s,
                          const uint8_t *down_W, const float *down_s, uint16_t *C) {
    if (!A || !gate_up_W || !gate_up_s || !down_W || !down_s || !C) return ORC_ERR_PARAM;
    if (M != 1 || H == 0 || I == 0 || K == 0 || down_in != I) return ORC_ERR_UNSUPPORTED;
    const size_t gpk = (K + 1) / 2, dpk = (I + 1) / 2;
    uint16_t *hidden = (uint16_t *)malloc(I * sizeof(uint16_t));
    if (!hidden) return ORC_ERR_MEM;
#pragma omp parallel for if (I >= 256)
    for (long long ii = 0; ii < (long long)I; ii++) {
        float g = bf16_to_f32(f32_to_bf16(dot_bf16_i4(A, gate_up_W + ii * gpk, K) * gate_up_s[ii]));
        float u = bf16_to_f32(f32_to_bf16(dot_bf16_i4(A, gate_up_W + (I + ii) * gpk, K) * gate_up_s[I + ii]));
        float silu = g / (1.0f + expf(-g));
        hidden[ii] = f32_to_bf16(silu * u);
    }
#pragma omp parallel for if (H >= 256)
    for (long long h = 0; h < (long long)H; h++)
        C[h] = f32_to_bf16(dot_bf16_i4(hidden, down_W + h * dpk, I) * down_s[h]);
    free(hidden);
    return ORC_OK;
}
