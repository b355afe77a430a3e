// int8 implicit-GEMM CONV2D tensor-core instantiations with 32-byte K blocks (at most 32
// input channels: a 64-byte box would be half outside the channel extent, and the TMA fills
// such boxes far more slowly than whole ones).
#include "gemm_launch.cuh"

namespace tb {

tb_status launch_i8_conv_k32(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                             const GemmParams& p, cudaStream_t st) {
    if (bn == 256) return launch_int_ek<GemmCfg<0, 256, 32, false, true, gemm_stages(256, 32)>, true>(ctx, ek, a, b, p, st);
    if (bn == 128) return launch_int_ek<GemmCfg<0, 128, 32, false, true, gemm_stages(128, 32)>, true>(ctx, ek, a, b, p, st);
    if (bn == 64) return launch_int_ek<GemmCfg<0, 64, 32, false, true, gemm_stages(64, 32)>, true>(ctx, ek, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "int8 CONV2D: no tile configuration for BN=%d BK=32", bn);
}

}  // namespace tb
