// int8 implicit-GEMM CONV2D (im2col TMA, K-major weights) tensor-core instantiations with
// 64-byte K blocks; 128-byte K blocks are in gemm_i8_conv_k128.cu.
#include "gemm_launch.cuh"

namespace tb {

tb_status launch_i8_conv(tb_context* ctx, int bn, int bk, int ek, const CUtensorMap& a, const CUtensorMap& b,
                         const GemmParams& p, cudaStream_t st) {
#define TB_CONV_CASE(BN_, BK_)                                                                       \
    if (bn == BN_ && bk == BK_)                                                                      \
        return launch_int_ek<GemmCfg<0, BN_, BK_, false, true, gemm_stages(BN_, BK_)>, true>(ctx, ek, a, b, p, st);
    if (bk == 128) return launch_i8_conv_k128(ctx, bn, ek, a, b, p, st);
    if (bk == 32) return launch_i8_conv_k32(ctx, bn, ek, a, b, p, st);
    TB_CONV_CASE(256, 64)
    TB_CONV_CASE(128, 64)
    TB_CONV_CASE(64, 64)
#undef TB_CONV_CASE
    return fail(TB_ERR_NOT_ACCELERATED, "int8 CONV2D: no tile configuration for BN=%d BK=%d", bn, bk);
}

}  // namespace tb
