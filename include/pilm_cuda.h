/*
 * libpilm_cuda -- B200 (sm_100a) implementation of piLM's MTP speculative-verify path.
 *
 * C ABI, drop-in for the piLM CPU library (libecpu) on the calls the verify path
 * makes: the same symbol names, descriptor structs and return codes as the
 * reference headers src/ecpu/include/{ecpu_base.h, ecpu.h, device/api.h,
 * kernel/api.h}, as bound by src/abi/bindings.py:59-233.  Differences:
 *   - every data pointer is a DEVICE pointer (cudaMalloc / torch CUDA tensors);
 *   - calls are enqueued on the library stream (ekernel_set_stream) and return
 *     without waiting, unless PILM_CUDA_SYNC=1 is set, in which case each call
 *     synchronises and reports execution errors like the synchronous reference;
 *   - the `isa` argument is ignored, exactly as in the reference ((void)isa).
 * Entry points after the "verify-path extensions" banner have no counterpart in
 * the reference; each comment names the reference code whose work it takes over.
 *
 * Return codes (ecpu_base.h:11-16): 0 ok, -1 bad parameter, -2 out of memory,
 * -3 device error, -4 kernel launch/execution error, -5 unsupported.
 * ecpu_last_error() returns the message of the last failure (or NULL).
 */
#ifndef PILM_CUDA_H
#define PILM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- ecpu_base.h:11-26 -------------------------------------------------------- */
#define ECPU_OK 0
#define ECPU_ERR_PARAM (-1)
#define ECPU_ERR_MEM (-2)
#define ECPU_ERR_DEVICE (-3)
#define ECPU_ERR_KERNEL (-4)
#define ECPU_ERR_UNSUPPORTED (-5)

typedef enum {
    ECPU_PRECISION_F32 = 0,
    ECPU_PRECISION_F16 = 1,
    ECPU_PRECISION_BF16 = 2,
    ECPU_PRECISION_F8_E4M3 = 3,
    ECPU_PRECISION_F8_E5M2 = 4,
    ECPU_PRECISION_I8 = 5,
    ECPU_PRECISION_I4 = 6,
} ecpu_precision_t;

/* ---- device/api.h:10-53 -------------------------------------------------------- */
typedef enum { EDEV_ECPU = 0, EDEV_CUDA = 1, EDEV_COUNT } edevice_t;

typedef enum {
    EDEV_CAP_NONE = 0,
    EDEV_CAP_F16 = 1 << 0,
    EDEV_CAP_BF16 = 1 << 1,
    EDEV_CAP_FP8 = 1 << 2,
    EDEV_CAP_INT8_AMX = 1 << 3,
    EDEV_CAP_AVX512 = 1 << 4,
    EDEV_CAP_AVX2 = 1 << 5,
    EDEV_CAP_NEON = 1 << 6,
    EDEV_CAP_SVE = 1 << 7,
    EDEV_CAP_NUMA = 1 << 8,
    EDEV_CAP_UNIFIED_MEM = 1 << 9,
} edevice_caps_t;

typedef struct edevice_vtable {
    const char *name;
    edevice_t id;
    uint64_t caps;
    void *(*alloc)(size_t bytes, size_t alignment);
    void (*free)(void *ptr);
    void (*memcpy_h2d)(void *dst, const void *src, size_t n);
    void (*memcpy_d2h)(void *dst, const void *src, size_t n);
    void (*memcpy_d2d)(void *dst, const void *src, size_t n);
    int (*synchronize)(void);
    size_t (*mem_total)(void);
    size_t (*mem_free)(void);
    int (*init)(void);
    int (*shutdown)(void);
} edevice_vtable_t;

/* device/api.h:48-53.  Slot EDEV_CUDA holds the B200 device (cudaMalloc & co.);
 * slot EDEV_ECPU holds a host-memory device so callers that enumerate both work. */
const edevice_vtable_t *edevice_get(edevice_t dev);
int edevice_register(edevice_t dev, const edevice_vtable_t *vtable);
int edevice_set_active(edevice_t dev);
const edevice_vtable_t *edevice_active(void);
int edevice_init_all(void);
void edevice_shutdown_all(void);

/* ---- ecpu.h:15-39 -------------------------------------------------------------- */
typedef struct {
    int n_threads;
    int numa_policy;
    int disable_amx;
    int disable_avx512;
    size_t eram_budget_bytes;
    size_t kv_cache_budget_bytes;
    edevice_t device_type;
} ecpu_config_t;

ecpu_config_t ecpu_config_default(void); /* device_type = EDEV_CUDA here */
int ecpu_init(const ecpu_config_t *config);
void ecpu_shutdown(void);
int ecpu_is_initialized(void);
const char *ecpu_version(void);
const char *ecpu_last_error(void);

/* ---- kernel/api.h:14-24 -------------------------------------------------------- */
typedef enum {
    EKERNEL_ISA_SCALAR = 0,
    EKERNEL_ISA_AVX2 = 1,
    EKERNEL_ISA_AVX512 = 2,
    EKERNEL_ISA_AMX = 3,
    EKERNEL_ISA_NEON = 4,
    EKERNEL_ISA_SVE = 5,
    EKERNEL_ISA_SM100A = 16, /* not in the reference enum: this library's target */
} ekernel_isa_t;

ekernel_isa_t ekernel_detect_isa(void);          /* always EKERNEL_ISA_SM100A */
const char *ekernel_isa_name(ekernel_isa_t isa); /* "sm_100a" for 16 */

/* ---- kernel/api.h:26-50 -------------------------------------------------------- */
typedef struct {
    size_t M, N, K;
    ecpu_precision_t a_prec;
    ecpu_precision_t b_prec;
    ecpu_precision_t out_prec;
    int transpose_a;
    int transpose_b;
} ekernel_gemm_desc_t;

typedef struct {
    size_t M, N, K;
} ekernel_linear_w8a32_desc_t;

typedef struct {
    size_t M;
    size_t hidden_size;
    size_t intermediate_size;
    size_t gate_up_in_features;
    size_t down_in_features;
} ekernel_w4a16_swiglu_desc_t;

/* kernel/api.h:35-38 (kernels.c:396-435): F32 GEMM, C[M,N] = op(A) op(B). */
int ekernel_gemm(const ekernel_gemm_desc_t *desc, const void *A, const void *B, void *C, ekernel_isa_t isa);

/* kernel/api.h:52-57 (kernels.c:437-467): fp32 A[M,K], int8 W[N,K], fp32 scales[N],
 * fp32 C[M,N] = (A . W_n) * s_n. */
int ekernel_linear_w8a32(const ekernel_linear_w8a32_desc_t *desc, const float *A, const int8_t *W,
                         const float *scales, float *C, ekernel_isa_t isa);

/* kernel/api.h:59-64 (kernels.c:469-656): bf16 A, int8 W, bf16 C = rne(dot * s_n). */
int ekernel_linear_w8a16_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const int8_t *W,
                              const float *scales, uint16_t *C, ekernel_isa_t isa);

/* kernel/api.h:66-72 (kernels.c:658-737): M=1 argmax over bf16-rounded logits, first
 * index on ties.  out_index / out_value are HOST pointers, as in the reference. */
int ekernel_linear_w8a16_bf16_argmax(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                     const int8_t *W, const float *scales, size_t *out_index,
                                     float *out_value, ekernel_isa_t isa);

/* kernel/api.h:107-112 (kernels.c:1002-1087): packed int4 W[N, ceil(K/2)] (even k in the
 * low nibble), fp32 scales[N]; bf16 C = rne(dot * s_n). */
int ekernel_linear_w4a16_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                              const float *scales, uint16_t *C, ekernel_isa_t isa);

/* kernel/api.h:114-119 (kernels.c:1141-1148): group-32 scales[N, ceil(K/32)]. */
int ekernel_linear_w4a16g32_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                                 const float *scales, uint16_t *C, ekernel_isa_t isa);

/* kernel/api.h:121-126 (kernels.c:1150-1157): group-128 scales[N, ceil(K/128)];
 * C = rne(sum_g s[n,g] * dot_g).  M <= 16 runs the register-dequant tensor-core GEMV;
 * larger M runs the tcgen05 GEMM. */
int ekernel_linear_w4a16g128_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                                  const float *scales, uint16_t *C, ekernel_isa_t isa);

/* C[M, N] = rne_bf16(A[M, K] . W[N, K]^T), fp32 accumulation: F.linear on bf16 tensors,
 * the reference's default BackendLinear (models/base/linear.py:170-183) as the MTP draft
 * module uses it (mtp.py:21, 137).  K % 8 == 0; A and W 16-byte aligned. */
int ekernel_linear_bf16(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint16_t *W, uint16_t *C);

/* Load-time repack of reference-packed int4 weights (uint8 [N, K/2], even k in the low
 * nibble; ckernel.py:70-161) into the k-pair nibble order: within every 32-bit word
 * (k = 8i .. 8i+7 of a row) nibble p holds k = 8i + 2p for p < 4 and 8i + 2(p-4) + 1 for
 * p >= 4.  The kernels then dequantize a word into consecutive-k bf16 pairs without byte
 * permutes.  K % 8 == 0; buffers 4-byte aligned; out may equal qweight. */
int ekernel_repack_w4_kpairs(const uint8_t *qweight, size_t N, size_t K, uint8_t *out);

/* ekernel_linear_w4a16g128_bf16 and ekernel_linear_w4a16_bf16 on k-pair repacked weights
 * (same scales, same results); K % 128 == 0 and 16-byte aligned A and W. */
int ekernel_linear_w4a16g128_bf16_kpairs(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                         const uint8_t *W, const float *scales, uint16_t *C, ekernel_isa_t isa);
int ekernel_linear_w4a16_bf16_kpairs(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A, const uint8_t *W,
                                     const float *scales, uint16_t *C, ekernel_isa_t isa);

/* ekernel_linear_w4a16g128_bf16_kpairs that may leave its result as split-K partial sums
 * instead of bf16 (no reference counterpart).  When the tensor-core GEMM runs its split
 * schedule (fewer 128-row weight tiles than SMs) with s splits and s * M * N fp32 values
 * fit in partials_bytes at partials (16-byte aligned), it writes them there as
 * [s][M][N] (split order = K order), does not write C, skips its combine pass and sets
 * *splits = s.  Otherwise it writes C like the plain call and sets *splits = 0.  The
 * partials are meant for a consumer that sums them itself
 * (ekernel_add_rmsnorm_bf16_splitk, ekernel_qk_norm_rope_kv_append_splitk). */
int ekernel_linear_w4a16g128_bf16_kpairs_deferred(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                                  const uint8_t *W, const float *scales, uint16_t *C,
                                                  float *partials, size_t partials_bytes, int32_t *splits);

/* Bytes of partials a deferred call of this shape leaves on this GPU (0: it writes C). */
size_t ekernel_linear_w4a16g128_partials_bytes(size_t M, size_t N, size_t K);

/* ekernel_linear_w4a16g128_bf16_kpairs that, on its stream-K schedule (at least one 128-row
 * weight tile per SM and M > 16: an LM head), also folds each output row's argmax into
 * row_keys[m] (uint64, zero before the call): atomicMax of (order-preserving bits of the
 * bf16 output << 32) | (0xFFFFFFFF - n), so the largest value wins with ties going to the
 * smallest n, NaN never wins and -0 equals +0, as in a first-max argmax over the bf16
 * logits.  *fused = 1 when it did; 0 when it only wrote C (then run
 * ekernel_argmax_top2_bf16 as usual).  The fused LM head -> acceptance of the verify
 * step (engine.py:479-503); no reference counterpart. */
int ekernel_linear_w4a16g128_bf16_kpairs_argmax(const ekernel_linear_w8a32_desc_t *desc, const uint16_t *A,
                                                const uint8_t *W, const float *scales, uint16_t *C,
                                                uint64_t *row_keys, int32_t *fused);

/* kernel/api.h:180-186 (kernels.c:1485-1526): rne(x * rsqrt(mean(x^2)+eps) * (w [+1])). */
int ekernel_rmsnorm_bf16(const uint16_t *x, uint16_t *out, const uint16_t *weight, size_t rows, size_t n,
                         float eps, int add_one);

/* kernel/api.h:196-199 (kernels.c:1580-1596): out = rne(silu(g) * u), fp32 math. */
int ekernel_swiglu_bf16(const uint16_t *gate, const uint16_t *up, uint16_t *out, size_t n);

/* kernel/api.h:205-212 (kernels.c:1598-1735): gate/up rows [0,I) and [I,2I) of one packed
 * per-row-scaled W4 tensor, bf16 activation, then the down projection.  The reference
 * supports M=1 only; this library accepts any M. */
int ekernel_swiglu_w4a16_bf16(const ekernel_w4a16_swiglu_desc_t *desc, const uint16_t *A,
                              const uint8_t *gate_up_W, const float *gate_up_scales, const uint8_t *down_W,
                              const float *down_scales, uint16_t *C, ekernel_isa_t isa);

/* ============================ verify-path extensions ============================ */

/* Stream control.  `stream` is a cudaStream_t (NULL = legacy default stream).  The
 * reference has no streams: its calls are synchronous (bindings.py:59-233). */
int ekernel_set_stream(void *stream);
void *ekernel_get_stream(void);
int ekernel_synchronize(void);

/* Number of kernels this library has launched since it was loaded (host-side count,
 * one per launch; used to report how many of the library's kernels ran in a region). */
unsigned long long ekernel_launch_count(void);

/* Number of device allocations the library has made for its own use since it was loaded
 * (scratch buffers, stream-K counters, per-device error words; memory handed out by the
 * device vtable's alloc is not counted).  A diagnostic: a caller can check that a region
 * of its program made the library allocate nothing. */
unsigned long long ekernel_alloc_count(void);

/* Test hook for the bounded waits of the tensor-core GEMM's pipeline (it has no
 * counterpart in the reference): later launches give up a wait after `polls` polls
 * (0: at the first wait not already met), raise the kernel's error word, drain their copies
 * and MMAs, free their tensor memory and exit, so the call reports ECPU_ERR_KERNEL in
 * synchronous mode (PILM_CUDA_SYNC=1).  polls < 0 restores the kernel's own limit. */
int ekernel_set_wait_limit(long long polls);

/* Token embedding gather: out[r,:] = table[ids[r],:] (bf16).  Takes over
 * nn.Embedding in Qwen3Model.forward (model.py:110). */
int ekernel_embedding_bf16(const int32_t *ids, size_t rows, const uint16_t *table, size_t vocab, size_t hidden,
                           uint16_t *out);

/* Residual add + RMSNorm with the torch-module rounding of RMSNorm / GemmaRMSNorm
 * (layers.py:94-98, 115-119): if delta != NULL, residual = rne(residual + delta) in
 * place (TransformerBlock.forward, model.py:66-72); then
 * out = rne( rne(residual * rsqrt(mean(residual^2)+eps)) * w' ), w' = w or rne(w+1). */
int ekernel_add_rmsnorm_bf16(uint16_t *residual, const uint16_t *delta, const uint16_t *weight, size_t rows,
                             size_t n, float eps, int add_one, uint16_t *out);

/* The same with the delta given as the split-K partial sums of a deferred W4 linear
 * ([splits][rows][n] fp32, summed in split order and rounded to bf16: the linear's own
 * output).  n % 8 == 0, n <= 8192, 16-byte aligned buffers (else ECPU_ERR_UNSUPPORTED). */
int ekernel_add_rmsnorm_bf16_splitk(uint16_t *residual, const float *partials, int32_t splits,
                                    const uint16_t *weight, size_t rows, size_t n, float eps, int add_one,
                                    uint16_t *out);

/* SwiGLU activation with torch bf16 semantics (layers.py:193): h = rne(rne(silu(g)) * u)
 * where gate_up is [rows, 2*inter] with gate in columns [0,inter) and up in
 * [inter, 2*inter); out is [rows, inter]. */
int ekernel_silu_mul_bf16(const uint16_t *gate_up, size_t rows, size_t inter, uint16_t *out);

/* MTP draft step input (Qwen3MTPDraft.hidden, mtp.py:35-39): for sequence b,
 * out[b, 0:H]  = norm(embed[tokens[b], :], w_embed_norm)        (pre_fc_norm_embedding)
 * out[b, H:2H] = norm(hidden[src(b), :], w_hidden_norm)        (pre_fc_norm_hidden)
 * i.e. torch.cat([e, h], -1), with the torch-module rounding of ekernel_add_rmsnorm_bf16
 * (add_one: GemmaRMSNorm).  src(b) = row_base[b] + row_offset[b] (row_offset NULL: 0), or b
 * when row_base is NULL; after a verify step row_base = cu_q and row_offset = the accept
 * counts select the row that produced the next token.  Token ids outside [0, vocab) read
 * row 0 and make the call return ECPU_ERR_KERNEL in synchronous mode. */
int ekernel_mtp_fc_input_bf16(const uint16_t *hidden, const int32_t *row_base, const int32_t *row_offset,
                              const uint16_t *embed, const int32_t *tokens, size_t vocab, const uint16_t *w_embed_norm,
                              const uint16_t *w_hidden_norm, size_t num_seqs, size_t hidden_size, float eps,
                              int add_one, uint16_t *out);

/* Attention of each row over itself alone: FullAttention.forward without a KV cache
 * (attention.py:113-139), as in the MTP draft block (mtp.py:40).  The softmax over one key
 * is 1, so out[r, h*hd + d] = v[r, (h / (n_heads / n_kv_heads))*hd + d], multiplied by
 * rne(sigmoid(gate[r, h*hd + d])) when gate != NULL (Qwen3.5 gated attention). */
int ekernel_self_attention_bf16(const uint16_t *v, const uint16_t *gate, size_t rows, size_t n_heads,
                                size_t n_kv_heads, size_t head_dim, uint16_t *out);

typedef struct {
    size_t num_seqs;           /* B */
    size_t total_q;            /* rows = sum of per-sequence query lengths */
    size_t max_q_len;          /* upper bound of per-sequence query length */
    size_t n_heads;            /* query heads */
    size_t n_kv_heads;         /* KV heads (GQA); n_heads % n_kv_heads == 0 */
    size_t head_dim;           /* 128 */
    size_t block_size;         /* tokens per KV page (16) */
    size_t num_blocks;         /* pages in the pool (bounds check) */
    size_t max_blocks_per_seq; /* row stride of block_table */
    size_t max_context;        /* upper bound of context_lens (sizes the KV split) */
    size_t qkv_stride;         /* elements per row of the fused projection output */
    size_t rope_rows;          /* rows of the cos/sin tables (positions) */
    size_t rot_dim;            /* rotary dims, even, <= head_dim */
    float eps;                 /* RMSNorm eps for q_norm / k_norm */
    int add_one;               /* Gemma norms: weight + 1 */
    int output_gate;           /* Qwen3.5 gated attention: q_proj is [q_h | gate_h] per head */
} ekernel_paged_attn_desc_t;

/* QK-RMSNorm + RoPE + paged KV append for the verify rows.  qkv: [total_q, qkv_stride]
 * bf16 rows laid out [q section | k (n_kv*hd) | v (n_kv*hd)], the q section being
 * n_heads*hd, or n_heads*2*hd with [q_h | gate_h] per head when output_gate.
 * positions[total_q], slot_mapping[total_q] (= page*block_size + offset).  Writes the
 * normed, rotated queries to q_out [total_q, n_heads, hd] and the gate half (if any)
 * to gate_out [total_q, n_heads*hd]; writes K (normed, rotated) and V into the
 * caches [num_blocks, block_size, n_kv, hd] (physical_kv.py:30-33 layout).
 * Takes over attention.py:79-97 and layers.py:122-176. */
int ekernel_qk_norm_rope_kv_append(const ekernel_paged_attn_desc_t *desc, const uint16_t *qkv,
                                   const uint16_t *q_norm_w, const uint16_t *k_norm_w, const float *rope_cos,
                                   const float *rope_sin, const int32_t *positions, const int32_t *slot_mapping,
                                   uint16_t *k_cache, uint16_t *v_cache, uint16_t *q_out, uint16_t *gate_out);

/* ekernel_qk_norm_rope_kv_append taking the fused projection as the split-K partial sums
 * that ekernel_linear_w4a16g128_bf16_kpairs_deferred left ([splits][total_q][qkv_stride]
 * fp32): each element is their sum in split order rounded to bf16, the value the
 * projection would have had, so the results are identical.  No reference counterpart:
 * it saves the GEMM's separate combine pass. */
int ekernel_qk_norm_rope_kv_append_splitk(const ekernel_paged_attn_desc_t *desc, const float *partials,
                                          int32_t splits, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                                          const float *rope_cos, const float *rope_sin, const int32_t *positions,
                                          const int32_t *slot_mapping, uint16_t *k_cache, uint16_t *v_cache,
                                          uint16_t *q_out, uint16_t *gate_out);

/* Paged attention over the verify rows.  q: [total_q, n_heads, hd] (from the call
 * above), block_table [num_seqs, max_blocks_per_seq], cu_q [num_seqs+1] row offsets,
 * context_lens [num_seqs] (keys per sequence, including the appended rows).  Row j of
 * sequence b sits at position context_lens[b] - q_len_b + j and sees keys <= that
 * position (the causal triu mask of attention.py:131-134).  Scores are rounded like
 * the reference's bf16 bmm (rne(rne(q.k) * rne_scale)), softmax in fp32, split-KV
 * partials merged in fp32; out [total_q, n_heads*hd] bf16, multiplied by
 * rne(sigmoid(gate)) when output_gate (attention.py:135-139). */
int ekernel_paged_attention_verify(const ekernel_paged_attn_desc_t *desc, const uint16_t *q,
                                   const uint16_t *k_cache, const uint16_t *v_cache, const int32_t *block_table,
                                   const int32_t *cu_q, const int32_t *context_lens, const uint16_t *gate,
                                   uint16_t *out);

/* Allocation-free variant of ekernel_paged_attention_verify.  It has no counterpart in
 * the reference.  It is for callers that cannot let a kernel library allocate GPU
 * memory: an engine whose allocator owns the device and forbids side allocations, a
 * serving loop that must never hit cudaMalloc's implicit synchronisation, or a host
 * language that only passes in buffers it already owns.  Same arguments and result as
 * ekernel_paged_attention_verify; the split-KV partials live in a fixed 8 MiB device
 * array inside the library (held on every GPU that loads the library until exit)
 * instead of library-allocated scratch, and no allocator is called.
 *  - A call whose partials would exceed 8 MiB (splits x total_q x n_heads x 520 bytes)
 *    is rejected with ECPU_ERR_PARAM and a message naming the needed size.
 *  - A page wait that gives up is recorded in a fixed device word inside the library
 *    too (not the library's allocated error word), so no call of this entry point
 *    allocates, including the first one in a process.
 *  - The first call on each device looks up the device addresses of the array and of
 *    that word with that device current; make that first call before any stream
 *    capture.
 *  - All calls share the one array and it keeps the previous call's contents (each
 *    call resets the records it reads): calls that overlap on the GPU race, so issue
 *    them on one stream or otherwise ordered. */
int ekernel_paged_attention_verify_noalloc(const ekernel_paged_attn_desc_t *desc, const uint16_t *q,
                                           const uint16_t *k_cache, const uint16_t *v_cache,
                                           const int32_t *block_table, const int32_t *cu_q,
                                           const int32_t *context_lens, const uint16_t *gate, uint16_t *out);

typedef struct {
    size_t num_seqs; /* B */
    size_t total_q;  /* logit rows */
    size_t vocab;    /* V */
} ekernel_accept_desc_t;

/* Row-wise top-2 of fp32 logits [total_q, vocab]: top1 index (first maximum, like
 * torch.argmax), top1 value and the top1-top2 gap.  Any output may be NULL. */
int ekernel_argmax_top2_f32(const ekernel_accept_desc_t *desc, const float *logits, int32_t *top1,
                            float *top1_val, float *margin);

/* Same over bf16 logits [total_q, vocab] (the LM-head linear's output dtype; the
 * reference casts these bf16 values to fp32 before argmax, engine.py:480). */
int ekernel_argmax_top2_bf16(const ekernel_accept_desc_t *desc, const uint16_t *logits, int32_t *top1,
                             float *top1_val, float *margin);

/* Greedy MTP acceptance (engine.py:479-503, 551-557) + rollback of the verify slots.
 * verify_ids [total_q] are the rows fed to the verify forward ([last, d1..dn] per
 * sequence), top1 [total_q] their argmax.  Per sequence: accepted = number of leading
 * drafts d_i == top1[row i-1]; next_token = top1 of the first mismatching row (or of
 * the bonus row); context_lens[b] (in: keys incl. all verify rows) is rolled back to
 * start + 1 + accepted, the reference's num_computed_tokens (engine.py:505-510);
 * rejected verify slots in slot_mapping (may be NULL) are set to -1. */
int ekernel_verify_accept_greedy(const ekernel_accept_desc_t *desc, const int32_t *verify_ids,
                                 const int32_t *top1, const int32_t *cu_q, int32_t *accept_counts,
                                 int32_t *next_tokens, int32_t *context_lens, int32_t *slot_mapping);

/* ekernel_verify_accept_greedy taking the row argmax keys of
 * ekernel_linear_w4a16g128_bf16_kpairs_argmax: decodes each row's key into top1 (optional
 * output) and resets the key to 0 for the next step, then accepts and rolls back as the
 * greedy call does. */
int ekernel_verify_accept_greedy_keys(const ekernel_accept_desc_t *desc, const int32_t *verify_ids,
                                      uint64_t *row_keys, const int32_t *cu_q, int32_t *accept_counts,
                                      int32_t *next_tokens, int32_t *context_lens, int32_t *slot_mapping,
                                      int32_t *top1);

/* Rejection-sampling acceptance (no reference implementation: the reference verifies
 * greedily only, engine.py:373-379; this is standard speculative sampling with a one-hot
 * greedy draft).  p_i = softmax(logits_i / temperature) restricted to the nucleus
 * {j : mass of strictly more probable tokens < top_p}, renormalised.  Draft d_i is
 * accepted iff uniforms[row,0] < p_i(d_i); at the first rejection the next token is
 * sampled (inverse CDF in index order with uniforms[row,1]) from p_i with d_i removed,
 * else the bonus row's p_n.  Outputs and rollback as in ekernel_verify_accept_greedy.
 * Masses are summed in 64-bit fixed point (2^-40), so results do not depend on the
 * order of summation.  vocab < 2^23. */
int ekernel_verify_accept_rejection(const ekernel_accept_desc_t *desc, const float *logits,
                                    const int32_t *verify_ids, const int32_t *cu_q, const float *uniforms,
                                    float temperature, float top_p, int32_t *accept_counts,
                                    int32_t *next_tokens, int32_t *context_lens, int32_t *slot_mapping);

/* The same over bf16 logits (the LM head's output, read as fp32 like the reference's
 * lm_head(h).float(), engine.py:480). */
int ekernel_verify_accept_rejection_bf16(const ekernel_accept_desc_t *desc, const uint16_t *logits,
                                         const int32_t *verify_ids, const int32_t *cu_q, const float *uniforms,
                                         float temperature, float top_p, int32_t *accept_counts,
                                         int32_t *next_tokens, int32_t *context_lens, int32_t *slot_mapping);

/* ---- fp32-activation verify path (model dtype float32: the W8A32 configuration,
 * QuantizedW8A32Linear, linear.py:188-233).  The bf16 operations above with every
 * intermediate in fp32, as torch computes them for float32 tensors. ---- */

/* out[r,:] = table[ids[r],:] (fp32 embedding, model.py:110); ids outside [0, vocab) read
 * row 0 and make the call return ECPU_ERR_KERNEL in synchronous mode. */
int ekernel_embedding_f32(const int32_t *ids, size_t rows, const float *table, size_t vocab, size_t hidden,
                          float *out);

/* residual += delta (if delta != NULL), then out = w' * (residual * rsqrt(mean(residual^2) + eps)),
 * w' = w or 1 + w (RMSNorm / GemmaRMSNorm on fp32 tensors, layers.py:94-98, 115-119). */
int ekernel_add_rmsnorm_f32(float *residual, const float *delta, const float *weight, size_t rows, size_t n, float eps,
                            int add_one, float *out);

/* ekernel_qk_norm_rope_kv_append with fp32 projections, norm weights, caches and outputs. */
int ekernel_qk_norm_rope_kv_append_f32(const ekernel_paged_attn_desc_t *desc, const float *qkv, const float *q_norm_w,
                                       const float *k_norm_w, const float *rope_cos, const float *rope_sin,
                                       const int32_t *positions, const int32_t *slot_mapping, float *k_cache,
                                       float *v_cache, float *q_out, float *gate_out);

/* ekernel_paged_attention_verify with fp32 queries, caches, gate and output: scores
 * q.k * (1/sqrt(128)), causal mask, softmax and P.V in fp32 (attention.py:95-139). */
int ekernel_paged_attention_verify_f32(const ekernel_paged_attn_desc_t *desc, const float *q, const float *k_cache,
                                       const float *v_cache, const int32_t *block_table, const int32_t *cu_q,
                                       const int32_t *context_lens, const float *gate, float *out);

/* out = silu(gate) * up in fp32 (layers.py:193); gate_up is [rows, 2*inter]. */
int ekernel_silu_mul_f32(const float *gate_up, size_t rows, size_t inter, float *out);

#ifdef __cplusplus
}
#endif

#endif /* PILM_CUDA_H */
