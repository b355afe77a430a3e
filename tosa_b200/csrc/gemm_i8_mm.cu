// int8 batched MATMUL (B MN-major, [n,c,w]) tensor-core instantiations.
#include "gemm_launch.cuh"

namespace tb {

tb_status launch_i8_matmul(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                           const GemmParams& p, cudaStream_t st) {
    if (bn == 256) return launch_int_ek<GemmCfg<0, 256, 128, true, false, gemm_stages(256, 128)>, false>(ctx, ek, a, b, p, st);
    if (bn == 128) return launch_int_ek<GemmCfg<0, 128, 128, true, false, gemm_stages(128, 128)>, false>(ctx, ek, a, b, p, st);
    return fail(TB_ERR_NOT_ACCELERATED, "int8 MATMUL: no tile configuration for BN=%d", bn);
}

}  // namespace tb
