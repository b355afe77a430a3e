// MATMUL_T tensor-core instantiations: A [n,h,c] by 3-D tiled TMA as for MATMUL, B [d,w,c]
// K-major (128-byte K blocks, 128-byte swizzle, the layout of the convolution weights), its
// batch coordinate 0 when d == 1 is broadcast.
#include "gemm_launch.cuh"

namespace tb {

tb_status launch_i8_matmul_t(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                             const GemmParams& p, cudaStream_t st) {
    if (bn == 256) return launch_int_ek<GemmCfg<0, 256, 128, false, false, gemm_stages(256, 128)>, false>(ctx, ek, a, b, p, st);
    if (bn == 128) return launch_int_ek<GemmCfg<0, 128, 128, false, false, gemm_stages(128, 128)>, false>(ctx, ek, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "int8 MATMUL_T: no tile configuration for BN=%d", bn);
}

tb_status launch_f16_matmul_t(tb_context* ctx, int bn, const CUtensorMap& a, const CUtensorMap& b,
                              const GemmParams& p, cudaStream_t st) {
    if (bn == 256) return launch_gemm<GemmCfg<1, 256, 128, false, false, gemm_stages(256, 128)>, EK_F32>(ctx, a, b, p, st);
    if (bn == 128) return launch_gemm<GemmCfg<1, 128, 128, false, false, gemm_stages(128, 128)>, EK_F32>(ctx, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "float MATMUL_T: no tile configuration for BN=%d", bn);
}

}  // namespace tb
