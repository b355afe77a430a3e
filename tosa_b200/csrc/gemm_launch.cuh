// Launch helpers of the tensor-core GEMM: one template instantiation per tile
// configuration and epilogue kind. The instantiations are spread over gemm_i8_mm.cu,
// gemm_i8_conv.cu, gemm_i8_conv_k128.cu, gemm_i8_conv_tap2.cu and gemm_f16.cu, which expose the plain
// functions declared at the bottom.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "internal.hpp"
#include "tc_gemm.cuh"

namespace tb {

#define TB_GEMM_LAUNCHED(ctx)                                                                          \
    do {                                                                                               \
        cudaError_t e_ = cudaGetLastError();                                                           \
        if (e_ != cudaSuccess) return ::tb::fail(TB_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e_)); \
        (ctx)->launches++;                                                                             \
    } while (0)

// Host side of FastDiv (tc_gemm.cuh): s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1.
inline FastDiv make_fastdiv(int d) {
    FastDiv f{};
    f.d = static_cast<uint32_t>(d < 1 ? 1 : d);
    int s = 0;
    while ((1ull << s) < f.d) ++s;
    f.s = s;
    f.m = static_cast<uint32_t>(((1ull << 32) * ((1ull << s) - f.d)) / f.d + 1);
    return f;
}

template <class Cfg, int EK, int EF = 0>
tb_status launch_gemm(tb_context* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB, GemmParams p,
                      cudaStream_t stream) {
    static bool attr_set = false;  // the attribute is per function and process-wide
    if (!attr_set) {
        // The kernel's warpgroups re-split the registers it was launched with (setmaxnreg); that
        // needs the full launch allocation, or the epilogue warps would wait for registers forever.
        cudaFuncAttributes fa;
        TB_CUDA(cudaFuncGetAttributes(&fa, tc_gemm_kernel<Cfg, EK, EF>));
        if (fa.numRegs < kLaunchRegs)
            return fail(TB_ERR_CUDA, "tensor-core GEMM built with %d registers a thread; its register split needs %d",
                        fa.numRegs, kLaunchRegs);
        TB_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<Cfg, EK, EF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cfg::SMEM_BYTES));
        attr_set = true;
    }
    p.m_tiles = (p.M + Cfg::BM - 1) / Cfg::BM;
    p.n_tiles = (p.N + Cfg::kBN - 1) / Cfg::kBN;
    p.total_tiles = p.batch * p.m_tiles * p.n_tiles;
    // big MATMULs (many row and column tiles): bands of 16 row tiles in the tile order. Not for
    // convolutions: their weights (B) are small, and walking column tiles within a band would
    // make each CTA reload B and restage its column constants on every tile.
    p.group_m = (!Cfg::kIm2col && p.m_tiles >= 32 && p.n_tiles >= 4) ? 16 : 0;
    p.fd_mtiles = make_fastdiv(p.m_tiles);
    p.fd_ntiles = make_fastdiv(p.n_tiles);
    p.fd_ow = make_fastdiv(p.conv_OW);
    p.fd_ohow = make_fastdiv(p.conv_OHOW);
    // the ring: a multiple of the k blocks per tile when that costs at most one stage
    {
        const int S = Cfg::kStages, kb = p.k_blocks < 1 ? 1 : p.k_blocks;
        const int mult = kb <= S ? (S / kb) * kb : S;
        p.s_eff = S - mult <= 1 ? mult : S;
    }
    p.err = ctx->dev_err;
    p.timeout_cycles = ctx->timeout_cycles;
    p.trace = ctx->trace;
    const int grid = std::min(p.total_tiles, ctx->num_sms);
    // the three epilogue groups take whole tiles in turn (three TMEM buffers: BN <= 128) when
    // every CTA has several tiles; otherwise they share each tile by column thirds
    if (Cfg::kWholeTiles)
        p.epi_groups = ctx->epi_groups >= 0 ? ctx->epi_groups : (p.total_tiles >= 4 * grid ? 1 : 0);
    else
        p.epi_groups = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = stream;
    // Programmatic dependent launch: the GEMM may be placed on the SMs as the preceding kernel's
    // blocks leave (its barrier setup, TMEM allocation and descriptor prefetch overlap that
    // kernel's tail); its producer waits for the preceding kernel before the first copy.
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    cfg.attrs = attr;
    cfg.numAttrs = na;
    // the output map (fast int8 epilogue with TMA stores), or an unused placeholder
    CUtensorMap tmO;
    if (p.tma_out && p.tmo_host != nullptr) tmO = *p.tmo_host;
    else {
        std::memset(&tmO, 0, sizeof tmO);
        p.tma_out = 0;
    }
    TB_CUDA(cudaLaunchKernelEx(&cfg, tc_gemm_kernel<Cfg, EK, EF>, tmA, tmB, tmO, p));
    TB_GEMM_LAUNCHED(ctx);
    return TB_OK;
}

constexpr int gemm_stages(int bn, int bk) { return (kStageBudget / ((128 + bn) * bk)) < 8 ? (kStageBudget / ((128 + bn) * bk)) : 8; }
// Stages with two taps per stage (A: two 64-byte boxes, B: one 128-byte box).
constexpr int gemm_stages_tap2(int bn) { return (kStageBudget / ((128 + bn) * 128)) < 8 ? (kStageBudget / ((128 + bn) * 128)) : 8; }

// Epilogue kind for a prepared epilogue.
inline int epilogue_kind(const GemmEpilogue& e) {
    if (e.mode == EPI_I32) return EK_I32;
    if (e.mode == EPI_F32) return EK_F32;
    if (e.mode == EPI_FCONV) return EK_FCONV;
    if (!e.rs_fast || e.out_dtype != DT_INT8) return EK_SLOW;
    const bool dbl = e.rs.rounding == ROUND_DOUBLE;
    if (e.rs.per_channel) return dbl ? EK_FAST_PC_D : EK_FAST_PC_S;
    return dbl ? EK_FAST_T_D : EK_FAST_T_S;
}

// The fast int8 epilogue kind EK with its flags: row terms when B has a zero point, border
// deltas when the convolution has border classes (CONV: only convolutions have them).
template <class Cfg, int EK, bool CONV>
tb_status launch_fast_ek(tb_context* ctx, const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                         cudaStream_t st) {
    const bool row = p.epi.row_zp_neg != 0;
    if constexpr (CONV) {
        if (p.epi.rowclass != nullptr) {
            return row ? launch_gemm<Cfg, EK, kEfRow | kEfDelta>(ctx, a, b, p, st)
                       : launch_gemm<Cfg, EK, kEfDelta>(ctx, a, b, p, st);
        }
    }
    return row ? launch_gemm<Cfg, EK, kEfRow>(ctx, a, b, p, st) : launch_gemm<Cfg, EK, 0>(ctx, a, b, p, st);
}

// Switch over the integer epilogue kinds for one tile configuration.
template <class Cfg, bool CONV>
tb_status launch_int_ek(tb_context* ctx, int ek, const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                        cudaStream_t st) {
    switch (ek) {
    case EK_I32: return launch_gemm<Cfg, EK_I32>(ctx, a, b, p, st);
    case EK_SLOW: return launch_gemm<Cfg, EK_SLOW>(ctx, a, b, p, st);
    case EK_FAST_T_S: return launch_fast_ek<Cfg, EK_FAST_T_S, CONV>(ctx, a, b, p, st);
    case EK_FAST_T_D: return launch_fast_ek<Cfg, EK_FAST_T_D, CONV>(ctx, a, b, p, st);
    case EK_FAST_PC_S: return launch_fast_ek<Cfg, EK_FAST_PC_S, CONV>(ctx, a, b, p, st);
    case EK_FAST_PC_D: return launch_fast_ek<Cfg, EK_FAST_PC_D, CONV>(ctx, a, b, p, st);
    default: return fail(TB_ERR_NOT_ACCELERATED, "no integer epilogue kind %d", ek);
    }
}

// Implemented in gemm_i8_mm.cu / gemm_i8_conv*.cu / gemm_f16.cu.
tb_status launch_i8_matmul(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                           const GemmParams& p, cudaStream_t st);
tb_status launch_i8_conv(tb_context* ctx, int bn, int bk, int ek, const CUtensorMap& a, const CUtensorMap& b,
                         const GemmParams& p, cudaStream_t st);
tb_status launch_i8_conv_k128(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                              const GemmParams& p, cudaStream_t st);
tb_status launch_i8_conv_k32(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                              const GemmParams& p, cudaStream_t st);
tb_status launch_i8_conv_tap2(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                              const GemmParams& p, cudaStream_t st);
tb_status launch_f16_matmul(tb_context* ctx, int bn, const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                            cudaStream_t st);
// MATMUL_T (B K-major, [d,w,c]); in gemm_mm_t.cu.
tb_status launch_i8_matmul_t(tb_context* ctx, int bn, int ek, const CUtensorMap& a, const CUtensorMap& b,
                             const GemmParams& p, cudaStream_t st);
tb_status launch_f16_matmul_t(tb_context* ctx, int bn, const CUtensorMap& a, const CUtensorMap& b,
                              const GemmParams& p, cudaStream_t st);
tb_status launch_f16_conv(tb_context* ctx, int bn, const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p,
                          cudaStream_t st);

}  // namespace tb
