// int8 implicit-GEMM CONV2D tensor-core instantiations with 128-byte K blocks (more than 64
// input channels); split from gemm_i8_conv.cu so the two compile in parallel.
#include "gemm_launch.cuh"

namespace tb {

tb_status launch_i8_conv_k128(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                              const GemmParams& p, cudaStream_t st) {
    if (bn == 256) return launch_int_ek<GemmCfg<0, 256, 128, false, true, gemm_stages(256, 128)>, true>(ctx, ek, a, b, p, st);
    if (bn == 128) return launch_int_ek<GemmCfg<0, 128, 128, false, true, gemm_stages(128, 128)>, true>(ctx, ek, a, b, p, st);
    if (bn == 64) return launch_int_ek<GemmCfg<0, 64, 128, false, true, gemm_stages(64, 128)>, true>(ctx, ek, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "int8 CONV2D: no tile configuration for BN=%d BK=128", bn);
}

}  // namespace tb
