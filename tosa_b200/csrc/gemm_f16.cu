// bf16 / f16 (fp32 accumulation) tensor-core instantiations: MATMUL and CONV2D.
#include "gemm_launch.cuh"

namespace tb {

tb_status launch_f16_matmul(tb_context* ctx, int bn, const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                            cudaStream_t st) {
    if (bn == 256) return launch_gemm<GemmCfg<1, 256, 128, true, false, gemm_stages(256, 128)>, EK_F32>(ctx, a, b, p, st);
    if (bn == 128) return launch_gemm<GemmCfg<1, 128, 128, true, false, gemm_stages(128, 128)>, EK_F32>(ctx, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "float MATMUL: no tile configuration for BN=%d", bn);
}

tb_status launch_f16_conv(tb_context* ctx, int bn, const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                          cudaStream_t st) {
    if (bn == 256) return launch_gemm<GemmCfg<1, 256, 128, false, true, gemm_stages(256, 128)>, EK_FCONV>(ctx, a, b, p, st);
    if (bn == 128) return launch_gemm<GemmCfg<1, 128, 128, false, true, gemm_stages(128, 128)>, EK_FCONV>(ctx, a, b, p, st);
    if (bn == 64) return launch_gemm<GemmCfg<1, 64, 128, false, true, gemm_stages(64, 128)>, EK_FCONV>(ctx, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "float CONV2D: no tile configuration for BN=%d", bn);
}

}  // namespace tb
