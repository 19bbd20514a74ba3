// RMSNorm (C-kernel and torch-module rounding), residual add, SwiGLU activations,
// embedding gather, and the W4 SwiGLU MLP entry point.
#include "common.cuh"

using namespace pilm;

namespace {


// Sum of squares of a bf16 row, fp32, fixed lane order then a butterfly.
__device__ __forceinline__ float row_sumsq(const __nv_bfloat16 *x, int n, int lane) {
    float ss = 0.f;
    if ((n & 7) == 0 && ((((uintptr_t)x) & 15) == 0)) {
        for (int i = lane * 8; i < n; i += 256) {
            uint4 v = *reinterpret_cast<const uint4 *>(x + i);
            const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(&v);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float f = bf2f(e[j]);
                ss = fmaf(f, f, ss);
            }
        }
    } else {
        for (int i = lane; i < n; i += 32) {
            float f = bf2f(x[i]);
            ss = fmaf(f, f, ss);
        }
    }
    return warp_sum(ss);
}

// ekernel_rmsnorm_bf16 semantics (kernels.c:1485-1526): inv = 1/sqrtf(ss/n + eps),
// y = rne((x * inv) * w'), w' = w (+1 when add_one) in fp32.
__global__ void rmsnorm_c_kernel(const __nv_bfloat16 *__restrict__ x, __nv_bfloat16 *__restrict__ out,
                                 const __nv_bfloat16 *__restrict__ w, int rows, int n, float eps, int add_one) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= rows) return;
    const __nv_bfloat16 *xr = x + (size_t)row * n;
    const float ss = row_sumsq(xr, n, lane);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    __nv_bfloat16 *o = out + (size_t)row * n;
    for (int i = lane; i < n; i += 32) {
        float wf = bf2f(w[i]);
        if (add_one) wf = __fadd_rn(wf, 1.0f);
        o[i] = f2bf(__fmul_rn(__fmul_rn(bf2f(xr[i]), inv), wf));
    }
}

// RMSNorm / GemmaRMSNorm torch-module semantics (layers.py:94-98, 115-119), with an
// optional residual add first (model.py:66-72): r = rne(r + d); var = mean(r^2);
// xn = rne(r * (1/sqrt(var+eps))); y = rne(xn * w'), w' = w or rne(w + 1).
__global__ void add_rmsnorm_kernel(__nv_bfloat16 *__restrict__ res, const __nv_bfloat16 *__restrict__ delta,
                                   const __nv_bfloat16 *__restrict__ w, int rows, int n, float eps, int add_one,
                                   __nv_bfloat16 *__restrict__ out) {
    pdl_entry();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= rows) return;
    __nv_bfloat16 *r = res + (size_t)row * n;
    if (delta) {
        const __nv_bfloat16 *d = delta + (size_t)row * n;
        for (int i = lane; i < n; i += 32) r[i] = f2bf(__fadd_rn(bf2f(r[i]), bf2f(d[i])));
        __syncwarp();
    }
    const float ss = row_sumsq(r, n, lane);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    __nv_bfloat16 *o = out + (size_t)row * n;
    for (int i = lane; i < n; i += 32) {
        float xn = bf16_round(__fmul_rn(bf2f(r[i]), inv));
        float wf = bf2f(w[i]);
        if (add_one) wf = bf16_round(__fadd_rn(wf, 1.0f));
        o[i] = f2bf(__fmul_rn(xn, wf));
    }
}

// Same semantics as add_rmsnorm_kernel, one CTA (256 threads) per row with the row
// held in registers: 16-byte loads/stores, one read of the residual and delta, one
// block reduction.  n % 8 == 0 and n <= 256 * 8 * VPT.
template <int VPT>
// The delta comes as bf16 (delta) or as split-K partial sums of a W4 linear (part:
// [splits][rows][n] fp32), which are summed in split order and rounded to bf16 exactly as
// the GEMM's combine pass would have written them.
__global__ void __launch_bounds__(256) add_rmsnorm_row_kernel(__nv_bfloat16 *__restrict__ res,
                                                              const __nv_bfloat16 *__restrict__ delta,
                                                              const __nv_bfloat16 *__restrict__ w, int n, float eps,
                                                              int add_one, __nv_bfloat16 *__restrict__ out,
                                                              const float *__restrict__ part, int splits,
                                                              size_t plane) {
    pdl_trigger();
    __shared__ float red[8];
    const int row = blockIdx.x;
    __nv_bfloat16 *r = res + (size_t)row * n;
    const __nv_bfloat16 *d = delta ? delta + (size_t)row * n : nullptr;
    const float *pr = part ? part + (size_t)row * n : nullptr;
    // The norm weights are constant: read before the wait for the previous kernel.  The
    // residual is read with the partial sums, so that the row waits on memory once.
    uint4 wv[VPT], rv[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = (v * 256 + threadIdx.x) * 8;
        if (i < n) wv[v] = *reinterpret_cast<const uint4 *>(w + i);
    }
    pdl_wait();
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = (v * 256 + threadIdx.x) * 8;
        if (i < n) rv[v] = *reinterpret_cast<const uint4 *>(r + i);
    }
    // partial sums: every element's splits added in split order, the loads of a batch of
    // splits for all of this thread's elements issued before the adds (16 in flight)
    float ps[VPT][8];
    if (pr) {
        constexpr int SB = VPT <= 2 ? 4 : 2;
#pragma unroll
        for (int v = 0; v < VPT; ++v)
#pragma unroll
            for (int j = 0; j < 8; ++j) ps[v][j] = 0.f;
        for (int s0 = 0; s0 < splits; s0 += SB) {
            float4 t[SB][VPT][2];
#pragma unroll
            for (int u = 0; u < SB; ++u)
#pragma unroll
                for (int v = 0; v < VPT; ++v) {
                    const int i = (v * 256 + threadIdx.x) * 8;
                    if (s0 + u < splits && i < n) {
                        const float *q = pr + (size_t)(s0 + u) * plane + i;
                        t[u][v][0] = __ldcs(reinterpret_cast<const float4 *>(q));
                        t[u][v][1] = __ldcs(reinterpret_cast<const float4 *>(q + 4));
                    }
                }
#pragma unroll
            for (int u = 0; u < SB; ++u)
#pragma unroll
                for (int v = 0; v < VPT; ++v) {
                    const int i = (v * 256 + threadIdx.x) * 8;
                    if (s0 + u < splits && i < n) {
                        ps[v][0] += t[u][v][0].x; ps[v][1] += t[u][v][0].y;
                        ps[v][2] += t[u][v][0].z; ps[v][3] += t[u][v][0].w;
                        ps[v][4] += t[u][v][1].x; ps[v][5] += t[u][v][1].y;
                        ps[v][6] += t[u][v][1].z; ps[v][7] += t[u][v][1].w;
                    }
                }
        }
    }
    float x[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = (v * 256 + threadIdx.x) * 8;
        if (i < n) {
            const __nv_bfloat16 *re = reinterpret_cast<const __nv_bfloat16 *>(&rv[v]);
            if (d || pr) {
                float dl[8];
                if (pr) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) dl[j] = bf16_round(ps[v][j]);
                } else {
                    uint4 dv = *reinterpret_cast<const uint4 *>(d + i);
                    const __nv_bfloat16 *de = reinterpret_cast<const __nv_bfloat16 *>(&dv);
#pragma unroll
                    for (int j = 0; j < 8; ++j) dl[j] = bf2f(de[j]);
                }
                uint4 o;
                __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&o);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    oe[j] = f2bf(__fadd_rn(bf2f(re[j]), dl[j]));
                    x[v][j] = bf2f(oe[j]);
                }
                *reinterpret_cast<uint4 *>(r + i) = o;
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) x[v][j] = bf2f(re[j]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) ss = fmaf(x[v][j], x[v][j], ss);
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    __nv_bfloat16 *o = out + (size_t)row * n;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
        const int i = (v * 256 + threadIdx.x) * 8;
        if (i < n) {
            const __nv_bfloat16 *we = reinterpret_cast<const __nv_bfloat16 *>(&wv[v]);
            uint4 ov;
            __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&ov);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float xn = bf16_round(__fmul_rn(x[v][j], inv));
                float wf = bf2f(we[j]);
                if (add_one) wf = bf16_round(__fadd_rn(wf, 1.0f));
                oe[j] = f2bf(__fmul_rn(xn, wf));
            }
            *reinterpret_cast<uint4 *>(o + i) = ov;
        }
    }
}

__device__ __forceinline__ float silu_f(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// ekernel_swiglu_bf16 (kernels.c:1580-1596): rne(silu(g) * u), fp32 math.
__global__ void swiglu_c_kernel(const __nv_bfloat16 *__restrict__ g, const __nv_bfloat16 *__restrict__ u,
                                __nv_bfloat16 *__restrict__ out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = f2bf(__fmul_rn(silu_f(bf2f(g[i])), bf2f(u[i])));
}

// Same activation over a [rows, 2*inter] gate|up buffer (C-kernel rounding), used by
// the fused W4 SwiGLU MLP (kernels.c:1640-1646: gate/up already rounded to bf16).
__global__ void swiglu_c_rows_kernel(const __nv_bfloat16 *__restrict__ gu, int rows, int inter,
                                     __nv_bfloat16 *__restrict__ out) {
    const size_t n = (size_t)rows * inter;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / inter, c = i % inter;
        const __nv_bfloat16 *row = gu + r * 2 * inter;
        out[i] = f2bf(__fmul_rn(silu_f(bf2f(row[c])), bf2f(row[inter + c])));
    }
}

// torch semantics (layers.py:193): h = rne(rne(silu(g)) * u).
__global__ void silu_mul_module_kernel(const __nv_bfloat16 *__restrict__ gu, int rows, int inter,
                                       __nv_bfloat16 *__restrict__ out) {
    pdl_entry();
    const size_t n = (size_t)rows * inter;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / inter, c = i % inter;
        const __nv_bfloat16 *row = gu + r * 2 * inter;
        const float s = bf16_round(silu_f(bf2f(row[c])));
        out[i] = f2bf(__fmul_rn(s, bf2f(row[inter + c])));
    }
}

// The same with 8 consecutive outputs per thread (inter % 8 == 0, 16-byte aligned rows):
// one 16-byte load each of gate and up, one 16-byte store; grid (chunks of 2048, rows).
__global__ void __launch_bounds__(256) silu_mul_module_v8_kernel(const __nv_bfloat16 *__restrict__ gu, int inter,
                                                                 __nv_bfloat16 *__restrict__ out) {
    pdl_entry();
    const int r = blockIdx.y;
    const int c = (blockIdx.x * 256 + threadIdx.x) * 8;
    if (c >= inter) return;
    const __nv_bfloat16 *row = gu + (size_t)r * 2 * inter;
    const uint4 gv = *reinterpret_cast<const uint4 *>(row + c);
    const uint4 uv = *reinterpret_cast<const uint4 *>(row + inter + c);
    const __nv_bfloat16 *ge = reinterpret_cast<const __nv_bfloat16 *>(&gv);
    const __nv_bfloat16 *ue = reinterpret_cast<const __nv_bfloat16 *>(&uv);
    uint4 o;
    __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float s = bf16_round(silu_f(bf2f(ge[j])));
        oe[j] = f2bf(__fmul_rn(s, bf2f(ue[j])));
    }
    *reinterpret_cast<uint4 *>(out + (size_t)r * inter + c) = o;
}

__global__ void embedding_kernel(const int32_t *__restrict__ ids, int rows, const __nv_bfloat16 *__restrict__ table,
                                 int vocab, int hidden, __nv_bfloat16 *__restrict__ out) {
    pdl_entry();
    const int row = blockIdx.x;
    if (row >= rows) return;
    const int id = ids[row];
    __nv_bfloat16 *o = out + (size_t)row * hidden;
    if (id < 0 || id >= vocab) {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = f2bf(0.f);
        return;
    }
    const __nv_bfloat16 *t = table + (size_t)id * hidden;
    if ((hidden & 7) == 0 && ((((uintptr_t)t) & 15) == 0) && ((((uintptr_t)o) & 15) == 0)) {
        for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8)
            *reinterpret_cast<uint4 *>(o + i) = *reinterpret_cast<const uint4 *>(t + i);
    } else {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = t[i];
    }
}

int grid_for(size_t n, int block) {
    size_t g = (n + block - 1) / block;
    size_t cap = (size_t)num_sms() * 16;
    return (int)(g < cap ? (g ? g : 1) : cap);
}

}  // namespace

extern "C" {

int ekernel_rmsnorm_bf16(const uint16_t *x, uint16_t *out, const uint16_t *weight, size_t rows, size_t n, float eps,
                         int add_one) {
    PILM_REQUIRE(x && out && weight && rows > 0 && n > 0, ECPU_ERR_PARAM, "ekernel_rmsnorm_bf16: bad argument");
    PILM_REQUIRE(rows <= 0x7fffffff && n <= 0x7fffffff, ECPU_ERR_PARAM, "ekernel_rmsnorm_bf16: too large");
    rmsnorm_c_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream()>>>(
        (const __nv_bfloat16 *)x, (__nv_bfloat16 *)out, (const __nv_bfloat16 *)weight, (int)rows, (int)n, eps,
        add_one);
    return check_launch("ekernel_rmsnorm_bf16");
}

int ekernel_add_rmsnorm_bf16(uint16_t *residual, const uint16_t *delta, const uint16_t *weight, size_t rows,
                             size_t n, float eps, int add_one, uint16_t *out) {
    PILM_REQUIRE(residual && weight && out && rows > 0 && n > 0, ECPU_ERR_PARAM,
                 "ekernel_add_rmsnorm_bf16: bad argument");
    const bool vec = (n % 8) == 0 && n <= 256 * 8 * 4 && ((((uintptr_t)residual) | ((uintptr_t)out) |
                                                          ((uintptr_t)weight) | ((uintptr_t)delta)) & 15) == 0;
    if (vec) {
        const __nv_bfloat16 *dl = (const __nv_bfloat16 *)delta;
        if (n <= 256 * 8 * 2)
            launch_pdl(add_rmsnorm_row_kernel<2>, dim3((unsigned)rows), dim3(256), 0, (__nv_bfloat16 *)residual, dl,
                       (const __nv_bfloat16 *)weight, (int)n, eps, add_one, (__nv_bfloat16 *)out,
                       (const float *)nullptr, 0, (size_t)0);
        else
            launch_pdl(add_rmsnorm_row_kernel<4>, dim3((unsigned)rows), dim3(256), 0, (__nv_bfloat16 *)residual, dl,
                       (const __nv_bfloat16 *)weight, (int)n, eps, add_one, (__nv_bfloat16 *)out,
                       (const float *)nullptr, 0, (size_t)0);
        return check_launch("ekernel_add_rmsnorm_bf16");
    }
    launch_pdl(add_rmsnorm_kernel, dim3((unsigned)((rows + 3) / 4)), dim3(128), 0, 
        (__nv_bfloat16 *)residual, (const __nv_bfloat16 *)delta, (const __nv_bfloat16 *)weight, (int)rows, (int)n,
        eps, add_one, (__nv_bfloat16 *)out);
    return check_launch("ekernel_add_rmsnorm_bf16");
}

int ekernel_add_rmsnorm_bf16_splitk(uint16_t *residual, const float *partials, int32_t splits, const uint16_t *weight,
                                    size_t rows, size_t n, float eps, int add_one, uint16_t *out) {
    const char *what = "ekernel_add_rmsnorm_bf16_splitk";
    PILM_REQUIRE(residual && partials && weight && out && rows > 0 && n > 0 && splits > 0, ECPU_ERR_PARAM,
                 "%s: bad argument", what);
    PILM_REQUIRE((n % 8) == 0 && n <= 256 * 8 * 4 &&
                     ((((uintptr_t)residual) | ((uintptr_t)out) | ((uintptr_t)weight) | ((uintptr_t)partials)) & 15) == 0,
                 ECPU_ERR_UNSUPPORTED, "%s: needs n %% 8 == 0, n <= 8192 and 16-byte aligned buffers", what);
    const size_t plane = rows * n;
    if (n <= 256 * 8 * 2)
        launch_pdl(add_rmsnorm_row_kernel<2>, dim3((unsigned)rows), dim3(256), 0, (__nv_bfloat16 *)residual,
                   (const __nv_bfloat16 *)nullptr, (const __nv_bfloat16 *)weight, (int)n, eps, add_one,
                   (__nv_bfloat16 *)out, partials, (int)splits, plane);
    else
        launch_pdl(add_rmsnorm_row_kernel<4>, dim3((unsigned)rows), dim3(256), 0, (__nv_bfloat16 *)residual,
                   (const __nv_bfloat16 *)nullptr, (const __nv_bfloat16 *)weight, (int)n, eps, add_one,
                   (__nv_bfloat16 *)out, partials, (int)splits, plane);
    return check_launch(what);
}

int ekernel_swiglu_bf16(const uint16_t *gate, const uint16_t *up, uint16_t *out, size_t n) {
    PILM_REQUIRE(gate && up && out, ECPU_ERR_PARAM, "ekernel_swiglu_bf16: null argument");
    if (n == 0) return ECPU_OK;
    swiglu_c_kernel<<<grid_for(n, 256), 256, 0, stream()>>>((const __nv_bfloat16 *)gate, (const __nv_bfloat16 *)up,
                                                             (__nv_bfloat16 *)out, n);
    return check_launch("ekernel_swiglu_bf16");
}

int ekernel_silu_mul_bf16(const uint16_t *gate_up, size_t rows, size_t inter, uint16_t *out) {
    PILM_REQUIRE(gate_up && out, ECPU_ERR_PARAM, "ekernel_silu_mul_bf16: null argument");
    if (rows == 0 || inter == 0) return ECPU_OK;
    if (inter % 8 == 0 && (((uintptr_t)gate_up) & 15) == 0 && (((uintptr_t)out) & 15) == 0 && rows <= 65535)
        launch_pdl(silu_mul_module_v8_kernel, dim3((unsigned)((inter / 8 + 255) / 256), (unsigned)rows), dim3(256), 0,
                   (const __nv_bfloat16 *)gate_up, (int)inter, (__nv_bfloat16 *)out);
    else
        launch_pdl(silu_mul_module_kernel, dim3(grid_for(rows * inter, 256)), dim3(256), 0,
                   (const __nv_bfloat16 *)gate_up, (int)rows, (int)inter, (__nv_bfloat16 *)out);
    return check_launch("ekernel_silu_mul_bf16");
}

int ekernel_embedding_bf16(const int32_t *ids, size_t rows, const uint16_t *table, size_t vocab, size_t hidden,
                           uint16_t *out) {
    PILM_REQUIRE(ids && table && out, ECPU_ERR_PARAM, "ekernel_embedding_bf16: null argument");
    if (rows == 0) return ECPU_OK;
    launch_pdl(embedding_kernel, dim3((unsigned)rows), dim3(128), 0, ids, (int)rows, (const __nv_bfloat16 *)table, (int)vocab,
                                                           (int)hidden, (__nv_bfloat16 *)out);
    return check_launch("ekernel_embedding_bf16");
}

int ekernel_swiglu_w4a16_bf16(const ekernel_w4a16_swiglu_desc_t *desc, const uint16_t *A,
                              const uint8_t *gate_up_W, const float *gate_up_scales, const uint8_t *down_W,
                              const float *down_scales, uint16_t *C, ekernel_isa_t isa) {
    (void)isa;
    PILM_REQUIRE(desc && A && gate_up_W && gate_up_scales && down_W && down_scales && C, ECPU_ERR_PARAM,
                 "ekernel_swiglu_w4a16_bf16: null argument");
    PILM_REQUIRE(desc->M > 0 && desc->hidden_size > 0 && desc->intermediate_size > 0 &&
                     desc->gate_up_in_features > 0 && desc->down_in_features == desc->intermediate_size,
                 ECPU_ERR_UNSUPPORTED, "ekernel_swiglu_w4a16_bf16: unsupported shape");
    const int M = (int)desc->M, H = (int)desc->hidden_size, I = (int)desc->intermediate_size;
    const int K = (int)desc->gate_up_in_features;
    char *aux = (char *)scratch(kScratchAux, (size_t)M * 3 * I * 2 + 256);
    PILM_REQUIRE(aux, ECPU_ERR_MEM, "ekernel_swiglu_w4a16_bf16: workspace allocation failed");
    uint16_t *gu = (uint16_t *)aux;
    uint16_t *h = (uint16_t *)(aux + (((size_t)M * 2 * I * 2 + 255) / 256) * 256);
    int rc = linear_bf16(1, 0, A, M, K, gate_up_W, gate_up_scales, 2 * I, gu, "ekernel_swiglu_w4a16_bf16");
    if (rc != ECPU_OK) return rc;
    swiglu_c_rows_kernel<<<grid_for((size_t)M * I, 256), 256, 0, stream()>>>((const __nv_bfloat16 *)gu, M, I,
                                                                              (__nv_bfloat16 *)h);
    rc = check_launch("ekernel_swiglu_w4a16_bf16");
    if (rc != ECPU_OK) return rc;
    return linear_bf16(1, 0, h, M, I, down_W, down_scales, H, C, "ekernel_swiglu_w4a16_bf16");
}

}  // extern "C"
