// W4A16 GEMM for M >= 64 on 5th-generation tensor cores (tcgen05 + TMEM).
#include "common.cuh"

namespace pilm {

int linear_w4_tc(const __nv_bfloat16 *X, int M, int K, const uint8_t *W, const float *S, int N,
                 __nv_bfloat16 *Y, bool grouped, const char *what) {
    (void)X; (void)M; (void)K; (void)W; (void)S; (void)N; (void)Y; (void)grouped; (void)what;
    return ECPU_ERR_UNSUPPORTED;
}

}  // namespace pilm
