// Kernels of the MTP draft module (src/models/qwen3/mtp.py:15-82) that the verify path's
// kernels do not already cover.
//
//   mtp_fc_input      the draft step's fc input torch.cat([e, h], -1) (mtp.py:35-39): e is
//                     the RMSNorm / GemmaRMSNorm of the draft token's embedding row, h that
//                     of the state hidden row, each with torch-module rounding.  The hidden
//                     row is gathered by index, so the first draft step can read the verify
//                     row that produced the next token straight from the verify output
//                     (row cu_q[b] + accepted[b]).
//   self_attention    the draft block's attention.  The block runs without a KV cache, so a
//                     token attends to itself alone (attention.py:113-116): the softmax over
//                     one key is exactly 1 and the output is the token's V expanded over the
//                     GQA group (attention.py:118-121, 134-136), times sigmoid(gate) when the
//                     q projection is gated (attention.py:139).  Q, K, their norms and RoPE
//                     cannot change the result and are not computed.
#include "common.cuh"

using namespace pilm;

namespace {

__device__ __forceinline__ float block_sum_256(float v, float *red) {
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k];
    return t;
}

// grid (B, 2): y = 0 normalises the embedding row of tokens[b] into out[b, 0:H], y = 1 the
// hidden row into out[b, H:2H].  Torch-module rounding (layers.py:94-98, 115-119):
// xn = rne(x * (1/sqrt(mean(x^2) + eps))), y = rne(xn * w'), w' = w or rne(w + 1).
__global__ void __launch_bounds__(256) mtp_fc_input_kernel(const __nv_bfloat16 *__restrict__ hidden,
                                                           const int32_t *__restrict__ row_base,
                                                           const int32_t *__restrict__ row_offset,
                                                           const __nv_bfloat16 *__restrict__ embed,
                                                           const int32_t *__restrict__ tokens, int vocab,
                                                           const __nv_bfloat16 *__restrict__ w_embed,
                                                           const __nv_bfloat16 *__restrict__ w_hidden, int H,
                                                           float eps, int add_one, __nv_bfloat16 *__restrict__ out,
                                                           int *__restrict__ err) {
    pdl_entry();
    __shared__ float red[8];
    const int b = blockIdx.x;
    const bool is_hidden = blockIdx.y == 1;
    const __nv_bfloat16 *x;
    if (is_hidden) {
        const int row = row_base ? row_base[b] + (row_offset ? row_offset[b] : 0) : b;
        x = hidden + (size_t)row * H;
    } else {
        int tok = tokens[b];
        if (tok < 0 || tok >= vocab) {  // a bad token id is reported, the row reads token 0
            if (threadIdx.x == 0) atomicExch(err, 1);
            tok = 0;
        }
        x = embed + (size_t)tok * H;
    }
    const __nv_bfloat16 *w = is_hidden ? w_hidden : w_embed;
    __nv_bfloat16 *o = out + (size_t)b * 2 * H + (is_hidden ? H : 0);
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += 256) {
        const float v = bf2f(x[i]);
        ss = fmaf(v, v, ss);
    }
    const float tot = block_sum_256(ss, red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
    for (int i = threadIdx.x; i < H; i += 256) {
        const float xn = bf16_round(__fmul_rn(bf2f(x[i]), inv));
        float wf = bf2f(w[i]);
        if (add_one) wf = bf16_round(__fadd_rn(wf, 1.0f));
        o[i] = f2bf(__fmul_rn(xn, wf));
    }
}

// out[r, h*hd + d] = v[r, (h / gsz)*hd + d], times rne(sigmoid(gate[r, h*hd + d])) when
// gate is given (the attention kernels' gate rounding); one thread per output element.
__global__ void self_attention_kernel(const __nv_bfloat16 *__restrict__ v, const __nv_bfloat16 *__restrict__ gate,
                                      size_t total, int nh, int nkv, int hd, __nv_bfloat16 *__restrict__ out) {
    pdl_entry();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int width = nh * hd;
    const size_t r = i / width;
    const int c = (int)(i % width);
    const int h = c / hd, d = c % hd;
    const int kvh = h / (nh / nkv);
    float y = bf2f(v[r * (size_t)(nkv * hd) + (size_t)kvh * hd + d]);
    if (gate) {
        const float gt = bf2f(gate[i]);
        const float sg = bf16_round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gt))));
        y = __fmul_rn(y, sg);
    }
    out[i] = f2bf(y);
}

}  // namespace

extern "C" {

int ekernel_mtp_fc_input_bf16(const uint16_t *hidden, const int32_t *row_base, const int32_t *row_offset,
                              const uint16_t *embed, const int32_t *tokens, size_t vocab, const uint16_t *w_embed_norm,
                              const uint16_t *w_hidden_norm, size_t num_seqs, size_t hidden_size, float eps,
                              int add_one, uint16_t *out) {
    const char *what = "ekernel_mtp_fc_input_bf16";
    PILM_REQUIRE(hidden && embed && tokens && w_embed_norm && w_hidden_norm && out, ECPU_ERR_PARAM,
                 "%s: null argument", what);
    PILM_REQUIRE(hidden_size > 0 && hidden_size <= (1u << 20) && vocab > 0 && vocab <= 0x7fffffff &&
                     num_seqs <= 0x7fffffff,
                 ECPU_ERR_PARAM, "%s: sizes out of range", what);
    if (num_seqs == 0) return ECPU_OK;
    int *err = device_error_word();
    PILM_REQUIRE(err, ECPU_ERR_MEM, "%s: error word allocation failed", what);
    launch_pdl(mtp_fc_input_kernel, dim3(dim3((unsigned)num_seqs, 2)), dim3(256), 0, 
        (const __nv_bfloat16 *)hidden, row_base, row_offset, (const __nv_bfloat16 *)embed, tokens, (int)vocab,
        (const __nv_bfloat16 *)w_embed_norm, (const __nv_bfloat16 *)w_hidden_norm, (int)hidden_size, eps, add_one,
        (__nv_bfloat16 *)out, err);
    const int rc = check_launch(what);
    if (rc != ECPU_OK) return rc;
    return check_error_word(what, "a draft token id was outside the vocabulary");
}

int ekernel_self_attention_bf16(const uint16_t *v, const uint16_t *gate, size_t rows, size_t n_heads,
                                size_t n_kv_heads, size_t head_dim, uint16_t *out) {
    const char *what = "ekernel_self_attention_bf16";
    PILM_REQUIRE(v && out, ECPU_ERR_PARAM, "%s: null argument", what);
    PILM_REQUIRE(n_kv_heads > 0 && n_heads % n_kv_heads == 0 && head_dim > 0 && n_heads * head_dim <= (1u << 24),
                 ECPU_ERR_PARAM, "%s: n_heads must be a multiple of n_kv_heads", what);
    const size_t total = rows * n_heads * head_dim;
    if (total == 0) return ECPU_OK;
    launch_pdl(self_attention_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, 
        (const __nv_bfloat16 *)v, (const __nv_bfloat16 *)gate, total, (int)n_heads, (int)n_kv_heads, (int)head_dim,
        (__nv_bfloat16 *)out);
    return check_launch(what);
}

}  // extern "C"
