// int8 implicit-GEMM CONV2D tensor-core instantiations with two filter taps per stage
// (exactly 64 input channels, more than one tap; see GemmCfg's TAP2).
#include "gemm_launch.cuh"

namespace tb {

tb_status launch_i8_conv_tap2(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                              const GemmParams& p, cudaStream_t st) {
    if (bn == 128) return launch_int_ek<GemmCfg<0, 128, 64, false, true, gemm_stages_tap2(128), true>, true>(ctx, ek, a, b, p, st);
    if (bn == 64) return launch_int_ek<GemmCfg<0, 64, 64, false, true, gemm_stages_tap2(64), true>, true>(ctx, ek, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "int8 CONV2D: no two-tap tile configuration for BN=%d", bn);
}

}  // namespace tb
