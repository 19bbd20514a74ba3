// Shared device/host helpers for libpilm_cuda (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/pilm_cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libpilm_cuda targets sm_100a (B200) only"
#endif

namespace pilm {

// ---------------------------------------------------------------------------------
// Library state (defined in runtime.cu)
// ---------------------------------------------------------------------------------
cudaStream_t stream();
int sync_mode();
int num_sms();
void set_error(const char *fmt, ...);
// Device scratch owned by the library, one independent buffer per slot so nested
// calls never alias (grown on demand, never inside stream capture).
enum ScratchSlot { kScratchSplitK = 0, kScratchAux = 1, kScratchAttn = 2, kScratchAccept = 3, kScratchSlots = 4 };
void *scratch(int slot, size_t bytes);
inline void *workspace(size_t bytes) { return scratch(kScratchSplitK, bytes); }
int *counters(size_t n);  // zero-initialised, self-resetting arrival counters

// W4 GEMM for M > 16 (tcgen05 path, linear_tc.cu); returns ECPU_ERR_UNSUPPORTED
// when the shape is not handled there, in which case the caller uses the GEMV.
// kpairs: the packed weights are in the k-pair nibble order (ekernel_repack_w4_kpairs).
// defer (optional): when the call runs the split schedule with grouped scales and its
// [splits][M][N] fp32 partials fit in defer_cap bytes at defer (16-byte aligned), they are
// left there, Y is not written, no combine pass runs and *defer_splits = splits; otherwise
// *defer_splits = 0 and Y holds the result.
// amax (optional, k-pair weights): when the call runs the stream-K schedule it also folds
// every output row m's argmax over n into amax[m] (atomicMax of an order-preserving key:
// value bits << 32 | (0xFFFFFFFF - n)) and sets *amax_done = 1; else *amax_done = 0.
int linear_w4_tc(const __nv_bfloat16 *X, int M, int K, const uint8_t *W, const float *S, int N,
                 __nv_bfloat16 *Y, bool grouped, bool kpairs, const char *what, float *defer = nullptr,
                 size_t defer_cap = 0, int *defer_splits = nullptr, unsigned long long *amax = nullptr,
                 int *amax_done = nullptr);
// Bytes of split-K partials a deferred call of this shape would leave (0: it would not).
size_t w4_tc_partials_bytes(int M, int N, int K);
// Quantized bf16 linear (linear.cu).  qf: 0 = W4 grouped (gs 32/128), 1 = W4 per-row,
// 2 = W8 per-row.  kpairs (W4 only): weights in the k-pair nibble order.
int linear_bf16(int qf, int gs, const void *A, int M, int K, const void *W, const float *S, int N, void *C,
                const char *what, bool kpairs = false, float *defer = nullptr, size_t defer_cap = 0,
                int *defer_splits = nullptr, unsigned long long *amax = nullptr, int *amax_done = nullptr);

// cuTensorMapEncodeTiled, reached through the runtime's driver entry point (no link
// against libcuda); null if the driver does not provide it.
typedef CUresult (*TensorMapEncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                           const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                           const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                           CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
TensorMapEncodeTiledFn tensor_map_encoder();
// Device word that pipelined kernels set when a bounded wait gave up, one per device,
// allocated on first use there (null if it could not be allocated).  In synchronous mode check_error_word reads and clears it and turns a set
// word into ECPU_ERR_KERNEL with the message "<what>: <msg>".
int *device_error_word();
bool capturing();  // the library stream is being captured into a CUDA graph
int check_error_word(const char *what, const char *msg);
// The same check on a given error word (the allocation-free entry point's own word).
int check_error_word_at(int *err, const char *what, const char *msg);

// The poll limit set by ekernel_set_wait_limit for pipeline waits (-1: each kernel's own).
long long wait_limit_override();

// Post-launch check: ECPU_ERR_KERNEL on a launch error; in synchronous mode
// (PILM_CUDA_SYNC=1) also waits for the stream and reports execution errors.
int check_launch(const char *what);

// ---------------------------------------------------------------------------------
// Programmatic dependent launch.  The verify path's kernels are launched with
// launch_pdl and start with pdl_entry(): the next kernel in the stream may then launch
// while this one runs (its CTAs become resident and wait in their own pdl_entry), and
// this one touches no global memory before the previous kernel has completed.  Only the
// launch and CTA setup of consecutive kernels overlap.  The next kernel can launch only
// once every CTA of this one has run the trigger, so all of them are already resident.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_entry() {
    pdl_trigger();
    pdl_wait();
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------------
// bf16 helpers.  The reference rounds fp32 -> bf16 to nearest-even
// (kernels.c:19-25); __float2bfloat16_rn is the same rounding for finite values.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float bits2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ldg_v4(const void *p) {
    return *reinterpret_cast<const uint4 *>(p);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace pilm

#define PILM_REQUIRE(cond, code, ...)      \
    do {                                   \
        if (!(cond)) {                     \
            pilm::set_error(__VA_ARGS__);  \
            return (code);                 \
        }                                  \
    } while (0)
