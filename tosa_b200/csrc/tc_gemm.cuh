// Persistent warp-specialised tcgen05 GEMM / implicit-GEMM convolution for
// sm_100a with a fused TOSA epilogue.
//
// One CTA per SM (512 threads, 16 warps):
//   warp 0      TMA producer: A tiles (plain 3-D tiles, or im2col windows of
//               an NHWC activation for CONV2D) and B tiles into a STAGES-deep
//               shared-memory ring; no multicast.
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma (kind::i8 -> s32, or
//               kind::f16 -> f32) into one of the 128 x BN accumulators.
//   warps 2-3   zero-point row sums: when the B-side zero point is non-zero,
//               sum every A row of each stage from shared memory (dp4a, bank-
//               conflict-free chunk order) so the epilogue can apply
//               -zp_b * rowsum(A). 64 rows per warp.
//   warps 4-15  epilogue, three warps per SM sub-partition in three groups of
//               four (one warp per TMEM lane quadrant: warp w reads lanes
//               32*(w%4)..+31, one output row per thread); with several tiles
//               per CTA and BN <= 128 group (w-4)/4 takes every third tile and
//               all its columns, otherwise the groups share every tile by
//               column thirds; the next columns are loaded from TMEM while the
//               current ones are processed.
// Warpgroup 0 needs few registers: it hands most of them to the epilogue
// warpgroups (setmaxnreg), whose arithmetic needs them.
//
// The accumulator has four (whole tiles per group) or two buffers in TMEM, so
// the epilogue of a tile overlaps the main loop of the next one and the
// epilogues of the tiles before it. All waits are bounded: a wait that
// gives up sets DEV_ERR_TIMEOUT in the device error word and the CTA unwinds.
//
// Arithmetic contract (integer): the tensor core forms sum(a*b) over raw
// int8 operands exactly; with the zero points the reference's
//   sum_valid (x - zx)(w - zw)
//     = sum x*w - zw*sum_valid x - zx*sum_valid w + n_valid*zx*zw  (mod 2^32)
// is rebuilt in the epilogue. Padded convolution taps are zero-filled by TMA
// and so drop out of sum x*w and of the row sums; the per-output-channel
// terms depend only on which taps are valid, so they are precomputed per
// border class by the convolution plan (a base table plus per-class deltas).
// All sums wrap mod 2^32 like AccI32 (src/ops/accum.rs:28-41), so the result
// is bit-exact in any order.
//
// RESCALE fast path (every shift in [32, 62], multiplier >= 0; checked on the
// host): the reference's apply_scale_32 (src/ops/quant.rs:17-32) computes
// (v*m + round) >> s with round = 2^(s-1) [+2^30 for v >= 0, -2^30 for v < 0
// under double rounding], then adds the output zero point. In this range every
// int32 v is admissible and nothing overflows, so the kernel evaluates the
// high word of the 64-bit sum v*m + R with two instructions (mad.lo.cc +
// madc.hi) and shifts it right by s-32. The host packs per channel
// {m, s-32, R_lo, R_hi} for v >= 0 and {R_lo, R_hi} for v < 0, where R already
// contains the output zero point as zp * 2^s when s <= 55 (exact: the sum stays
// below 2^63 and zp * 2^s only adds zp to the shifted result).
#pragma once

#include <cstdint>
#include <cuda.h>

#include "ptx.cuh"
#include "quant.cuh"

namespace tb {

enum : int { EPI_I32 = 0, EPI_RESCALE = 1, EPI_F32 = 2, EPI_FCONV = 3 };

// Compile-time epilogue kind: each kernel instantiation carries only the code
// of one epilogue, which keeps its hot loop small and well scheduled.
enum : int {
    EK_I32 = 0,        // int32 store of acc + zero-point terms
    EK_SLOW = 1,       // general RESCALE (range checks, inexact, scale16), any integer output type
    EK_FAST_T_S = 2,   // fast RESCALE, per-tensor, single rounding, int8 out
    EK_FAST_T_D = 3,   // fast RESCALE, per-tensor, double rounding, int8 out
    EK_FAST_PC_S = 4,  // fast RESCALE, per-channel, single rounding, int8 out
    EK_FAST_PC_D = 5,  // fast RESCALE, per-channel, double rounding, int8 out
    EK_F32 = 6,        // float accumulator stored as fp32
    EK_FCONV = 7,      // float convolution: round(round(acc) + bias) to the output type
};

// 16 warps: warpgroup 0 = TMA producer, MMA issuer and two row-sum warps; warpgroups 1-3 =
// 12 epilogue warps in three groups of four (one warp per TMEM lane quadrant). Launched with
// 128 registers a thread (65,536 for the CTA); warpgroup 0 gives back down to kRoleRegs and
// the epilogue warpgroups take up to kEpiRegs: 128 * kRoleRegs + 384 * kEpiRegs <= 65,536.
constexpr int kGemmThreads = 512;
constexpr int kEpiWarps = 12;
constexpr int kEpiGroups = 3;
constexpr int kLaunchRegs = 128;
constexpr int kRoleRegs = 88;
constexpr int kEpiRegs = 136;
static_assert(128 * kRoleRegs + 384 * kEpiRegs <= kGemmThreads * kLaunchRegs, "register split above the launch total");
// Shared memory per CTA: the stage ring, then 1 KB of alignment slack, the barriers and row
// sums, and the epilogue scratch (a convolution's border-class tables and the staged column
// constants, 12 KB, then two 2 KB output staging buffers per epilogue warp).
constexpr int kSmemLimit = 232448;
constexpr int kBarrierBytes = 3072;
constexpr int kScratchBytes = 12288 + 4096 * kEpiWarps;
constexpr int kStageBudget = kSmemLimit - 1024 - kBarrierBytes - kScratchBytes;
// Bound (clock cycles) on a CTA's final waits for its own TMA loads and MMAs.
constexpr long long kDrainCycles = 2000000000ll;

struct GemmEpilogue {
    int mode;                  // EPI_*
    // Integer terms: v = acc + colterm[b][n] (+ ct_delta[class][n] on border rows) + row_zp_neg * rowsum(A row)
    const int32_t* colterm;    // [batch or 1][>= N padded to the tile] or nullptr (then 0)
    long long colterm_bstride; // per batch index (MATMUL: per-batch column sums), 0 otherwise
    const int32_t* ct_delta;   // [n_classes][ct_ld] or nullptr (CONV2D border classes)
    long long ct_ld;
    int base_class;            // class whose terms are in colterm
    int32_t row_zp_neg;        // -zp of the B side (0 disables the row sums)
    int pdl_wait;              // colterm is produced by the preceding kernel (programmatic dependent launch)
    // Convolution border classes: class = rowclass[oy] * n_col_classes + colclass[ox]
    const uint8_t* rowclass;   // [OH] or nullptr (single class)
    const uint8_t* colclass;   // [OW]
    int n_col_classes;
    // RESCALE
    RescaleArgs rs;
    // Fast RESCALE to int8 (every shift s in [33, 62], multipliers >= 0), small-range form: the
    // column terms, deltas and row_zp_neg arrive multiplied by sr_mul = 2^k and the host bounds
    // |v| < 2^(31-k), so v' = v * 2^k is exact; with d = 32 - k
    //   r = (mulhi(v', m) + sr_c [- sr_k2 when v' < 0, double rounding]) >> sr_sh [+ out_zp],
    // the exact apply_scale_32 (floor((v m + 2^(s-1) [+-2^30]) / 2^s); the added terms are
    // whole multiples of 2^d, so the inner floor division by 2^d is exact).
    int rs_fast;
    int rs_zp_folded;          // out_zp rides in sr_c
    int32_t sr_mul, sr_k2;
    // [channels padded to 256]: multiplier, s - d (at most 31), 2^(s-1-d) [+ 2^(30-d)] [+ zp 2^(s-d)]
    const int32_t* fq_m;
    const int32_t* sr_sh;
    const int32_t* sr_c;
    int out_dtype;             // DT_INT8 / DT_INT16 / DT_INT32 / DT_FP32 / DT_BF16 / DT_FP16
    // Float convolution: out = round(round(acc) + fbias[n])
    const float* fbias;        // [N] or [1]
    int fbias_len;
};

// Division by a runtime constant d as a multiply-high (Granlund-Montgomery): with
// s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1, n / d = (mulhi(n, m) + n) >> s
// for 0 <= n < 2^31. The host fills it (make_fastdiv).
struct FastDiv {
    uint32_t d, m;
    int s;
};

__device__ __forceinline__ int fdiv(int n, const FastDiv& f) {
    return static_cast<int>((__umulhi(static_cast<uint32_t>(n), f.m) + static_cast<uint32_t>(n)) >> f.s);
}

struct GemmParams {
    int M, N, K;               // per batch
    int batch;
    int in_bf16;               // kind::f16 operands: 1 = bf16, 0 = f16
    int m_tiles, n_tiles, k_blocks;
    int total_tiles;
    // im2col geometry (CONV2D)
    int conv_OW, conv_OHOW;
    FastDiv fd_mtiles, fd_ntiles, fd_ow, fd_ohow;  // the divisions of the per-tile index arithmetic
    int stride_h, stride_w, pad_t, pad_l;
    int KW, dil_h, dil_w;
    int c_blocks;              // k blocks per filter tap
    int IC;                    // channels per tap (B column offset per tap)
    int taps;                  // filter taps (KH * KW) of a convolution
    // output
    void* out;
    long long out_batch_stride;  // elements
    long long ldo;               // elements per output row
    GemmEpilogue epi;
    uint32_t* err;
    long long timeout_cycles;
    // Optional timeline of CTA 0 (clock64 stamps), nullptr in normal runs:
    // [0,128) producer per stage issue, [128,256) MMA per stage start,
    // [256,384) row-sum per stage done, [384,400) epilogue tile start/end.
    long long* trace;
    // epilogue warps in two groups taking alternate tiles (set by the launcher when every CTA
    // has many tiles; otherwise both groups share each tile by column halves)
    int epi_groups;
    // K-major B without im2col (MATMUL_T): 1 when B has one batch shared by every batch of A
    int b_bcast;
    // stages of the ring in use (at most STAGES): a multiple of k_blocks when that costs at most
    // one stage, so that stage s always holds the same k block and a B tile that the previous
    // load into the stage already brought need not be loaded again
    int s_eff;
    // fast int8 epilogue: each warp writes its staged 32-row block with a TMA store through the
    // output tensor map (the kernel's third parameter) instead of per-thread stores
    int tma_out;
    const CUtensorMap* tmo_host;  // host side only: the map the launcher passes, when tma_out
    int group_m;                  // row tiles per band of the tile order (0: row tiles fastest throughout)
};

// TAP2 (int8 im2col convolutions with exactly 64 input channels): two filter taps per stage,
// each tap's A box in its own 64-byte-swizzled sub-tile, the two taps' weights as one
// 128-byte-swizzled B box (they are adjacent in K), four MMAs per stage. Halves the number of
// stages of a 3x3 convolution over 64 channels, whose time is set by the per-stage latency of
// the producer and MMA issue chains rather than by either unit's throughput.
template <int KIND, int BN, int BK_BYTES, bool B_MN_MAJOR, bool IM2COL, int STAGES, bool TAP2 = false>
struct GemmCfg {
    static constexpr int kKind = KIND;            // 0: int8, 1: f16/bf16
    static constexpr int BM = 128;
    static constexpr int kBN = BN;
    static constexpr int kBKBytes = BK_BYTES;     // 32 (SW32), 64 (SW64) or 128 (SW128)
    static constexpr int kElem = KIND == 0 ? 1 : 2;
    static constexpr int BK = BK_BYTES / kElem;   // elements of K per stage
    static constexpr int kMmaK = 32 / kElem;      // K per tcgen05.mma (32 bytes)
    static constexpr int kStages = STAGES;
    static constexpr bool kBMN = B_MN_MAJOR;
    static constexpr bool kIm2col = IM2COL;
    static constexpr bool kTap2 = TAP2;
    static constexpr int A_SUB = BM * BK_BYTES;                     // one tap's A box
    static constexpr int A_BYTES = TAP2 ? 2 * A_SUB : A_SUB;
    static constexpr int kBKBytesB = TAP2 ? 2 * BK_BYTES : BK_BYTES;  // K bytes of B per stage
    static constexpr int B_BYTES = BN * kBKBytesB;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int SW_CODE = BK_BYTES == 128 ? 2 : (BK_BYTES == 64 ? 4 : 6);  // UMMA layout type
    static constexpr int ATOM_SBO = 8 * BK_BYTES;                   // 8 rows of one swizzle atom
    static constexpr int SW_CODE_B = kBKBytesB == 128 ? 2 : (kBKBytesB == 64 ? 4 : 6);
    static constexpr int ATOM_SBO_B = 8 * kBKBytesB;
    // MN-major B: 128-byte rows of N, one box per 128 bytes of N.
    static constexpr int B_MN_CHUNK = 128 / kElem;                  // N elements per box
    static constexpr int B_MN_BOX_BYTES = BK * 128;                 // BK k-rows x 128 bytes
    // accumulator buffers in TMEM (512 columns): four when the epilogue groups take whole tiles
    // in turn (BN <= 128 only), otherwise two
    static constexpr bool kWholeTiles = BN <= 128;
    static constexpr int kTmemNeed = kWholeTiles ? 4 * BN : 2 * BN;
    static constexpr int TMEM_COLS = kTmemNeed <= 32 ? 32 : (kTmemNeed <= 64 ? 64 : (kTmemNeed <= 128 ? 128 : (kTmemNeed <= 256 ? 256 : 512)));
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + kBarrierBytes + kScratchBytes;
    static_assert(SMEM_BYTES <= kSmemLimit, "shared memory above 227 KB");
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "UMMA N for M=128; each epilogue warp walks pairs of 16-column chunks");
    static_assert(BK_BYTES == 32 || BK_BYTES == 64 || BK_BYTES == 128, "K blocks of 32, 64 or 128 bytes");
    static_assert(!B_MN_MAJOR || BK_BYTES == 128, "MN-major B uses 128-byte K blocks");
    static_assert(!TAP2 || (KIND == 0 && IM2COL && BK_BYTES == 64), "two taps per stage: int8 im2col, 64 channels");
};

// ---------------------------------------------------------------------------

__device__ __forceinline__ void tile_coords(const GemmParams& p, int tile, int& b, int& mt, int& nt) {
    if (p.group_m == 0) {
        // m fastest so CTAs running concurrently share the B tile in L2.
        const int rest = fdiv(tile, p.fd_mtiles);
        mt = tile - rest * p.m_tiles;
        b = fdiv(rest, p.fd_ntiles);
        nt = rest - b * p.n_tiles;
        return;
    }
    // Large A and B: bands of group_m row tiles, each walked row tile fastest across all column
    // tiles, so the tiles that run at once share a band of A and a few B tiles in L2 instead of
    // streaming all of A once per column tile.
    const int per_batch = p.m_tiles * p.n_tiles;
    b = tile / per_batch;
    int t = tile - b * per_batch;
    const int span = p.group_m * p.n_tiles;
    const int g = t / span;
    t -= g * span;
    const int gm = min(p.group_m, p.m_tiles - g * p.group_m);
    nt = t / gm;
    mt = g * p.group_m + (t - nt * gm);
}

// Makes the 16 registers of a finished tcgen05.ld visible only after the
// wait: the asm redefines them, so no use can be scheduled above it.
__device__ __forceinline__ void tmem_wait_regs(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]));
}

__device__ __forceinline__ void tmem_wait_regs(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

constexpr int kChunk = 16;   // output columns per thread per TMEM load (general epilogue)
constexpr int kChunkF = 16;  // the same for the fast int8 RESCALE epilogue

__device__ __forceinline__ uint32_t pack4_i8(int32_t a, int32_t b, int32_t c, int32_t d) {
    const uint32_t lo = __byte_perm(static_cast<uint32_t>(a), static_cast<uint32_t>(b), 0x0040);
    const uint32_t hi = __byte_perm(static_cast<uint32_t>(c), static_cast<uint32_t>(d), 0x0040);
    return __byte_perm(lo, hi, 0x5410);
}

// Epilogue for kChunk consecutive output columns n0.. of one row (one thread).
// v = acc + column terms (+ border-class delta) + row term, the zero-point and bias
// terms of the integer contraction. colterm / delta are padded by the host to
// whole tiles, so n0 + j needs no clamp.
template <int W = kChunk>
__device__ __forceinline__ void int_terms(const uint32_t (&acc)[W], int n0, int32_t rowterm,
                                          const int32_t* colterm, const int32_t* delta, int32_t (&v)[W]) {
    if (colterm != nullptr) {
        // 16-byte loads of the column terms (tables are 16-byte aligned and padded to whole tiles)
        // column terms staged in shared memory for the tile (16-byte loads)
        const int4* ct4 = reinterpret_cast<const int4*>(colterm + n0);
#pragma unroll
        for (int j = 0; j < W; j += 4) {
            const int4 c = ct4[j / 4];
            v[j + 0] = static_cast<int32_t>(acc[j + 0] + static_cast<uint32_t>(c.x) + static_cast<uint32_t>(rowterm));
            v[j + 1] = static_cast<int32_t>(acc[j + 1] + static_cast<uint32_t>(c.y) + static_cast<uint32_t>(rowterm));
            v[j + 2] = static_cast<int32_t>(acc[j + 2] + static_cast<uint32_t>(c.z) + static_cast<uint32_t>(rowterm));
            v[j + 3] = static_cast<int32_t>(acc[j + 3] + static_cast<uint32_t>(c.w) + static_cast<uint32_t>(rowterm));
        }
        if (delta != nullptr) {
            const int4* d4 = reinterpret_cast<const int4*>(delta + n0);
#pragma unroll
            for (int j = 0; j < W; j += 4) {
                const int4 c = __ldg(d4 + j / 4);
                v[j + 0] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 0]) + static_cast<uint32_t>(c.x));
                v[j + 1] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 1]) + static_cast<uint32_t>(c.y));
                v[j + 2] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 2]) + static_cast<uint32_t>(c.z));
                v[j + 3] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 3]) + static_cast<uint32_t>(c.w));
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] = static_cast<int32_t>(acc[j] + static_cast<uint32_t>(rowterm));
    }
}

// Per-tensor fast RESCALE constants (channel 0) and the clamp decision, loaded once.
struct FastConst {
    int32_t m, sh, c, add_zp;
    bool clamp;     // the range is narrower than int8's (a fused CLAMP): saturation alone does not do it
    bool clamp_lo;  // lower bound above -128
    bool clamp_hi;  // upper bound below 127
};

template <int EK>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, const uint32_t (&acc)[kChunk], int n0,
                                               long long orow, int32_t rowterm, const int32_t* colterm,
                                               const int32_t* delta, const int32_t* fm, const int32_t* fsh,
                                               const int32_t* fhz, const FastConst& fk, uint32_t& err) {
    const GemmEpilogue& e = p.epi;
    uint8_t* outp = reinterpret_cast<uint8_t*>(p.out);
    const int ncols = min(kChunk, p.N - n0);
    if constexpr (EK == EK_F32 || EK == EK_FCONV) {
        float v[kChunk];
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
            float a = __uint_as_float(acc[j]);
            if constexpr (EK == EK_FCONV) {
                const int n = min(n0 + j, p.N - 1);
                const float bias = __ldg(e.fbias + (e.fbias_len == 1 ? 0 : n));
                a = round_to_dtype(__fadd_rn(round_to_dtype(a, e.out_dtype), bias), e.out_dtype);
            }
            v[j] = a;
        }
        if (e.out_dtype == DT_FP32) {
            float* o = reinterpret_cast<float*>(outp) + orow + n0;
            if (ncols == kChunk && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
                for (int j = 0; j < kChunk; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < kChunk; ++j) if (j < ncols) o[j] = v[j];
            }
        } else if (e.out_dtype == DT_BF16) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(outp) + orow + n0;
#pragma unroll
            for (int j = 0; j < kChunk; ++j) if (j < ncols) o[j] = __float2bfloat16_rn(v[j]);
        } else {
            __half* o = reinterpret_cast<__half*>(outp) + orow + n0;
#pragma unroll
            for (int j = 0; j < kChunk; ++j) if (j < ncols) o[j] = __float2half_rn(v[j]);
        }
        return;
    } else {
    int32_t v[kChunk];
    int_terms(acc, n0, rowterm, colterm, delta, v);
    if constexpr (EK == EK_I32) {
        int32_t* o = reinterpret_cast<int32_t*>(outp) + orow + n0;
        if (ncols == kChunk && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < kChunk; j += 4) *reinterpret_cast<int4*>(o + j) = make_int4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < kChunk; ++j) if (j < ncols) o[j] = v[j];
        }
        return;
    }
    // RESCALE (+ fused CLAMP through r.lo / r.hi)
    const RescaleArgs& r = e.rs;
    int32_t res[kChunk];
    {
        // General apply_scale semantics with range checks (shifts below 32, inexact rounding, scale16).
        uint32_t dummy = 0;
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
            const int ch = r.per_channel ? min(n0 + j, p.N - 1) : 0;
            res[j] = static_cast<int32_t>(rescale_value(v[j], __ldg(r.multiplier + ch), __ldg(r.shift + ch),
                                                        r.rounding, r.scale32, r.out_zp, r.lo, r.hi,
                                                        j < ncols ? &err : &dummy));
        }
    }
    if (e.out_dtype == DT_INT8) {
        int8_t* o = reinterpret_cast<int8_t*>(outp) + orow + n0;
        if (ncols == kChunk && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
            *reinterpret_cast<uint4*>(o) = make_uint4(pack4_i8(res[0], res[1], res[2], res[3]),
                                                      pack4_i8(res[4], res[5], res[6], res[7]),
                                                      pack4_i8(res[8], res[9], res[10], res[11]),
                                                      pack4_i8(res[12], res[13], res[14], res[15]));
        } else {
#pragma unroll
            for (int j = 0; j < kChunk; ++j) if (j < ncols) o[j] = static_cast<int8_t>(res[j]);
        }
    } else if (e.out_dtype == DT_INT16) {
        int16_t* o = reinterpret_cast<int16_t*>(outp) + orow + n0;
#pragma unroll
        for (int j = 0; j < kChunk; ++j) if (j < ncols) o[j] = static_cast<int16_t>(res[j]);
    } else {
        int32_t* o = reinterpret_cast<int32_t*>(outp) + orow + n0;
#pragma unroll
        for (int j = 0; j < kChunk; ++j) if (j < ncols) o[j] = res[j];
    }
    }
}

// Fast int8 RESCALE of W consecutive columns, W/16 x 16 packed bytes into out16[]
// (small-range form, see GemmEpilogue): v' = acc * 2^k + column term [+ row term]
// [+ border-class delta], all terms pre-multiplied by 2^k (int32 wrap-around; the
// host's bound makes the sum exact), then r = (mulhi(v', m) + c [- k2 if v' < 0]) >> sh,
// then max(r + zp, lo) [min(., hi)] and saturating packs. ROW (a B zero point) and DELTA
// (a convolution with border classes) are kernel template flags, so kernels without them
// carry no code for them; the remaining conditions are uniform across the warp.
constexpr int kEfRow = 1;
constexpr int kEfDelta = 2;

template <int EK, int W, bool ROW, bool DELTA>
__device__ __forceinline__ void fast_chunk_i8(const GemmParams& p, const uint32_t (&acc)[W], int n0, int32_t rowterm,
                                              const int32_t* colterm, const int32_t* delta, const int4 (&dl)[W / 4],
                                              const int32_t* fm, const int32_t* fsh, const int32_t* fc,
                                              const FastConst& fk, uint4 (&out16)[W / 16]) {
    constexpr bool PC = EK == EK_FAST_PC_S || EK == EK_FAST_PC_D;
    constexpr bool DBL = EK == EK_FAST_T_D || EK == EK_FAST_PC_D;
    const uint32_t mul = static_cast<uint32_t>(p.epi.sr_mul);
    int32_t v[W];
#pragma unroll
    for (int j = 0; j < W; j += 4) {
        const int4 c = *reinterpret_cast<const int4*>(colterm + n0 + j);
        v[j + 0] = static_cast<int32_t>(acc[j + 0] * mul + static_cast<uint32_t>(c.x));
        v[j + 1] = static_cast<int32_t>(acc[j + 1] * mul + static_cast<uint32_t>(c.y));
        v[j + 2] = static_cast<int32_t>(acc[j + 2] * mul + static_cast<uint32_t>(c.z));
        v[j + 3] = static_cast<int32_t>(acc[j + 3] * mul + static_cast<uint32_t>(c.w));
    }
    if constexpr (ROW) {
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] = static_cast<int32_t>(static_cast<uint32_t>(v[j]) + static_cast<uint32_t>(rowterm));
    }
    if (DELTA && delta != nullptr) {  // warp-uniform: null for a warp without border rows
        // (the deltas of the chunk's columns, loaded by the caller one chunk ahead)
#pragma unroll
        for (int j = 0; j < W; j += 4) {
            const int4 c = dl[j / 4];
            v[j + 0] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 0]) + static_cast<uint32_t>(c.x));
            v[j + 1] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 1]) + static_cast<uint32_t>(c.y));
            v[j + 2] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 2]) + static_cast<uint32_t>(c.z));
            v[j + 3] = static_cast<int32_t>(static_cast<uint32_t>(v[j + 3]) + static_cast<uint32_t>(c.w));
        }
    }
    const int32_t k2 = p.epi.sr_k2;
    auto one = [&](int32_t x, int32_t m, int32_t sh, int32_t c) -> int32_t {
        int32_t add = c;
        if (DBL) add += (x >> 31) * k2;  // -2^(31-d) for a negative value
        int32_t h;
        asm("mad.hi.s32 %0, %1, %2, %3;" : "=r"(h) : "r"(x), "r"(m), "r"(add));
        return h >> sh;
    };
    if constexpr (PC) {
#pragma unroll
        for (int j = 0; j < W; j += 4) {
            const int4 m4 = *reinterpret_cast<const int4*>(fm + n0 + j);
            const int4 s4 = *reinterpret_cast<const int4*>(fsh + n0 + j);
            const int4 c4 = *reinterpret_cast<const int4*>(fc + n0 + j);
            v[j + 0] = one(v[j + 0], m4.x, s4.x, c4.x);
            v[j + 1] = one(v[j + 1], m4.y, s4.y, c4.y);
            v[j + 2] = one(v[j + 2], m4.z, s4.z, c4.z);
            v[j + 3] = one(v[j + 3], m4.w, s4.w, c4.w);
        }
    } else {
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] = one(v[j], fk.m, fk.sh, fk.c);
    }
    // output zero point (when not folded into c) and the lower clamp in one add-max; the
    // saturating packs complete the clamp to the int8 range
    const int32_t zp = fk.add_zp, lo = p.epi.rs.lo;
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = max(v[j] + zp, lo);
    if (fk.clamp_hi) {  // an upper bound below 127 (uniform; rare)
        const int32_t hi = p.epi.rs.hi;
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] = min(v[j], hi);
    }
#pragma unroll
    for (int q = 0; q < W / 16; ++q)
        out16[q] = make_uint4(pack4_sat_i8(v[16 * q + 0], v[16 * q + 1], v[16 * q + 2], v[16 * q + 3]),
                              pack4_sat_i8(v[16 * q + 4], v[16 * q + 5], v[16 * q + 6], v[16 * q + 7]),
                              pack4_sat_i8(v[16 * q + 8], v[16 * q + 9], v[16 * q + 10], v[16 * q + 11]),
                              pack4_sat_i8(v[16 * q + 12], v[16 * q + 13], v[16 * q + 14], v[16 * q + 15]));
}

// One epilogue warp's pass over its part of a tile (32 rows x h.cols columns) in the fast
// int8 form: TMEM loads of 32 columns (the next one in flight while this one is rescaled),
// packing into the warp's shared staging buffer, and row-contiguous stores of 64-byte groups.
struct FastTile {
    const CUtensorMap* tmo; // output tensor map (p.tma_out)
    int oz;                 // batch coordinate of the tile
    uint32_t taddr;         // TMEM address of the warp's first column (lane quadrant in the high half)
    int cols;               // columns of the tile this warp covers (BN, or its share of a tile)
    int n_end;              // of them, the ones that exist (at most cols, and N - first column)
    int nb;                 // absolute output column of the warp's first column
    int32_t rowterm;
    const int32_t* cst_n;   // staged column terms, indexed by absolute column
    const int32_t* delta;   // border-class delta row, or null when no row of the warp is on a border
    const int32_t* fm;
    const int32_t* fsh;
    const int32_t* fc;
    uint4* wst;             // the warp's two staging buffers, 2 KB apart: [32 rows][GW bytes] each
    int lane, mrow0;
    int8_t* obase;
    bool vec_ok;
    long long* ftr;         // trace slots (CTA 0, first tiles) or null
};

template <int EK, int GW, bool ROW, bool DELTA>
__device__ __forceinline__ void fast_tile_pass(const GemmParams& p, const FastConst& fk, const FastTile& h,
                                               uint32_t& npass) {
    constexpr int FW = kChunkF;                // columns per TMEM load
    constexpr int FPK = FW / 16;               // 16-byte packs per chunk
    constexpr int NCH = GW / FW;               // chunks per staging group (an even number)
    static_assert(NCH % 2 == 0, "staging groups alternate the two TMEM register sets");
    // GW: columns per staging group (32 or 64). Each of the warp's two staging buffers (used by
    // alternate groups, `npass` counts the warp's groups) holds 32 rows of GW bytes, the 16-byte
    // slots of a row permuted as the TMA's 32- / 64-byte swizzle lays them out (slot j of row r
    // at j ^ (r >> 2 & 1) or j ^ (r >> 1 & 3)): conflict-free row writes, and the layout a TMA
    // store of a [32 rows][GW] box reads. With two buffers a group waits only for the store of
    // the group before last, not for the one just issued.
    constexpr int RS = GW / 16;                // 16-byte slots per staging row
    const int COLS = h.cols;
    const int lane = h.lane;
    const int swz = GW == 64 ? (lane >> 1) & 3 : (lane >> 2) & 1;
    // Two register sets of FW columns: chunk c of a group uses set c % 2, and the next chunk's
    // TMEM load is in flight while chunk c is rescaled (tcgen05.wait::ld waits for all of this
    // thread's loads, so exactly one is outstanding at each wait).
    uint32_t fA[FW], fB[FW];
    // border-class deltas of a chunk (a warp with a border row), loaded with the chunk's TMEM
    // load one chunk ahead, so their latency overlaps the previous chunk's arithmetic
    int4 dA[FW / 4], dB[FW / 4];
    auto dload = [&](int col, int4(&d)[FW / 4]) {
        if constexpr (DELTA) {
            if (h.delta != nullptr) {
                const int4* d4 = reinterpret_cast<const int4*>(h.delta + h.nb + col);
#pragma unroll
                for (int i = 0; i < FW / 4; ++i) d[i] = __ldg(d4 + i);
            }
        }
    };
    __syncwarp();
    if (h.n_end > 0) {
        tmem_ld_32x32b(h.taddr, fA);
        dload(0, dA);
        tmem_wait_regs(fA);
    }
#pragma unroll 1
    for (int g0 = 0; g0 < COLS && g0 < h.n_end; g0 += GW) {
        if (h.ftr && g0 / GW < 8) h.ftr[3 * (g0 / GW)] = clock64();
        // a TMA store writes all GW columns of the box: only when they are this warp's (or lie
        // past N, where the store writes nothing); a block wholly below M is not stored at all
        const bool tma = p.tma_out && (g0 + GW <= COLS || h.nb + COLS >= p.N) && h.mrow0 < p.M;
        uint4* wst = h.wst + (npass & 1) * 128;  // 2 KB apart
        ++npass;
        if (p.tma_out) {  // the store that read this buffer (the group before last) is done reading
            if (lane == 0) bulk_wait_read1();
            __syncwarp();
        }
        // chunk c of the group: its accumulators in register set c % 2, the next chunk's TMEM load
        // in flight into the other set. Pairs of chunks per iteration (not the whole group
        // unrolled) keep the loop's code small.
        auto chunk = [&](int c, uint32_t(&cur)[FW], uint32_t(&nxt)[FW], int4(&dcur)[FW / 4],
                         int4(&dnxt)[FW / 4]) -> bool {
            const int col = g0 + c * FW;
            if (col >= h.n_end) return false;  // warp-uniform
            const bool next = col + FW < COLS && col + FW < h.n_end;
            __syncwarp();
            if (next) {
                tmem_ld_32x32b(h.taddr + col + FW, nxt);
                dload(col + FW, dnxt);
            }
            uint4 pk[FPK];
            fast_chunk_i8<EK, FW, ROW, DELTA>(p, cur, h.nb + col, h.rowterm, h.cst_n, h.delta, dcur, h.fm, h.fsh,
                                                   h.fc, fk, pk);
#pragma unroll
            for (int j = 0; j < FPK; ++j) wst[lane * RS + ((c * FPK + j) ^ swz)] = pk[j];
            __syncwarp();
            if (next) tmem_wait_regs(nxt);
            return true;
        };
#pragma unroll 1
        for (int c = 0; c < NCH; c += 2) {
            if (!chunk(c, fA, fB, dA, dB)) break;
            if (!chunk(c + 1, fB, fA, dB, dA)) break;
        }
        if (h.ftr && g0 / GW < 8) h.ftr[3 * (g0 / GW) + 1] = clock64();
        if (tma) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_3d(h.tmo, wst, h.nb + g0, h.mrow0, h.oz);
                bulk_commit();
            }
        } else {
            // every pass commits one bulk group (an empty one here), so that the wait before a
            // buffer's reuse always refers to the pass that last used it
            if (p.tma_out && lane == 0) bulk_commit();
            __syncwarp();
#pragma unroll
            for (int it = 0; it < RS; ++it) {
                const int idx = it * 32 + lane;
                const int r = idx / RS, k = idx % RS;
                const int rs = GW == 64 ? (r >> 1) & 3 : (r >> 2) & 1;
                const uint4 pv = wst[r * RS + (k ^ rs)];
                const int mr = h.mrow0 + r;
                const int n = h.nb + g0 + k * kChunk;
                // only this pass's columns: a group's share of a tile can end before N (column thirds)
                if (mr < p.M && g0 + k * kChunk < h.n_end) {
                    int8_t* o = h.obase + static_cast<long long>(mr) * p.ldo + n;
                    if (h.vec_ok && n + kChunk <= p.N) {
                        *reinterpret_cast<uint4*>(o) = pv;
                    } else {
                        const uint32_t w4[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
                        for (int j = 0; j < kChunk; ++j)
                            if (n + j < p.N) o[j] = static_cast<int8_t>(w4[j >> 2] >> (8 * (j & 3)));
                    }
                }
            }
        }
        if (h.ftr && g0 / GW < 8) h.ftr[3 * (g0 / GW) + 2] = clock64();
        __syncwarp();
    }
}

// EF: flags of the fast int8 epilogue (kEfRow: B zero point row terms; kEfDelta: convolution
// border classes); 0 for the other epilogue kinds.
template <class Cfg, int EK, int EF>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const __grid_constant__ GemmParams p) {
    constexpr int BM = Cfg::BM, BN = Cfg::kBN, S = Cfg::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment by an offset into the shared array: pointer arithmetic on smem_raw keeps the
    // shared address space visible to the compiler (shared loads/stores rather than generic ones).
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* stage_base = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * Cfg::STAGE_BYTES);
    uint64_t* full = bars;               // [S]
    uint64_t* empty = bars + S;          // [S]
    // TMEM accumulator buffers: with whole tiles per group (p.epi_groups) tile t takes buffer
    // t % 4 and is processed by group t % 3, so the next tile can fill while all three groups
    // work; otherwise every tile is shared by the groups (column thirds) and two buffers
    // alternate. No waiter is ever more than one phase ahead: a group's first tile takes a
    // fresh buffer, and the previous use of the buffer of its later tile t (tile t - 4) was
    // filled before the group's previous tile t - 3, which it has already waited for.
    const int NB = p.epi_groups ? 4 : 2;
    const int NB_LOG = p.epi_groups ? 2 : 1;  // buffer of tile count t: t & (NB - 1), its use: t >> NB_LOG
    uint64_t* tfull = bars + 2 * S;      // [4]
    uint64_t* tempty = tfull + 4;        // [4]
    uint64_t* rsfull = tempty + 4;       // [4]
    uint64_t* rsempty = rsfull + 4;      // [4]
    uint64_t* mdrain = rsempty + 4;      // [1]
    uint64_t* ebar = mdrain + 1;         // [1] barrier of the 12 epilogue warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int32_t* rowsum_buf = reinterpret_cast<int32_t*>(tmem_slot + 4);  // [4][128]
    int32_t* scratch = reinterpret_cast<int32_t*>(smem + S * Cfg::STAGE_BYTES + kBarrierBytes);  // kScratchBytes

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const bool need_rowsum = Cfg::kKind == 0 && p.epi.row_zp_neg != 0;

    // epilogue warps that release each accumulator buffer: the 4 of the group that took the
    // tile, or those of the groups that have a share of its columns (32-column chunks split in
    // thirds: with BN 64 group 0 has none)
    const int n_chunks = BN / 32;
    const uint32_t epi_arrivals = p.epi_groups ? 4 : 4 * (n_chunks < kEpiGroups ? n_chunks : kEpiGroups);
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], need_rowsum ? 3 : 1);  // MMA commit + two row-sum warps
        }
        for (int b = 0; b < NB; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], epi_arrivals);
            mbar_init(&rsfull[b], 2);
            mbar_init(&rsempty[b], epi_arrivals);
        }
        mbar_init(&mdrain[0], 1);
        mbar_init(&ebar[0], kEpiWarps);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const long long limit = p.timeout_cycles;
    // waits for this CTA's own copies and MMAs before it exits get a fixed, generous bound (about
    // a second), whatever the configured timeout: they end once work already issued completes
    const long long drain_limit = limit > kDrainCycles ? limit : kDrainCycles;
    const int SE = p.s_eff;  // stages of the ring in use
    if (kGemmTrace && p.trace && blockIdx.x == 0 && threadIdx.x == 0) p.trace[400] = clock64();
    // The next kernel on the stream, when launched as a programmatic dependent, may be placed on
    // the SMs this grid leaves; it waits for this grid's completion before touching its data.
    if (threadIdx.x == 0) grid_launch_dependents();
    if (kGemmTrace && p.trace && threadIdx.x == 0) {
        if (blockIdx.x == 0) p.trace[403] = static_cast<long long>(globaltimer_ns());
        atomicMax(reinterpret_cast<unsigned long long*>(p.trace + 405), globaltimer_ns());
    }

    if (warp < 4) {
        // warpgroup 0: producer, MMA issuer, row sums -- few registers, the rest to the epilogue
        setmaxnreg_dec<kRoleRegs>();
        if (warp == 0) {
            // ------------------------------------------------------------ producer
            if (lane == 0) {
                uint32_t it = 0;
                bool ok = true;
                // the B tile each stage holds: (B batch, N tile, k block), -1 before its first load.
                // B tiles are the same for every M tile of a (batch, N tile) pair; for short K
                // (few k blocks, a ring that is a multiple of them) the stages keep their B tiles
                // across tiles and only A is loaded.
                long long bkey[S];
#pragma unroll
                for (int i = 0; i < S; ++i) bkey[i] = -1;
                int rs_s = 0;       // ring position of `it`: stage it % SE and its phase parity, stepped
                uint32_t rs_ph = 0; // (no division by the runtime stage count)
                // launched as a programmatic dependent: the preceding kernel's outputs (A, and B
                // of a MATMUL) are complete and visible only after this wait; nothing of this
                // kernel reads or writes global data before the first copy (the epilogue's stores
                // follow the MMAs of these copies)
                grid_dependency_wait();
                for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
                    int b, mt, nt;
                    tile_coords(p, tile, b, mt, nt);
                    const int m0 = mt * BM, n0 = nt * BN;
                    const int bb = Cfg::kIm2col || p.b_bcast ? 0 : b;  // batch of the B tile
                    const long long key0 = (static_cast<long long>(bb) * p.n_tiles + nt) * p.k_blocks;
                    int img = 0, wb = 0, hb = 0;
                    if constexpr (Cfg::kIm2col) {
                        img = fdiv(m0, p.fd_ohow);
                        const int rem = m0 - img * p.conv_OHOW;
                        const int oy = fdiv(rem, p.fd_ow), ox = rem - oy * p.conv_OW;
                        wb = ox * p.stride_w - p.pad_l;
                        hb = oy * p.stride_h - p.pad_t;
                    }
                    int cb = 0, kx = 0, ky = 0, tap = 0;  // k block kb = (ky * KW + kx) * c_blocks + cb, stepped
                    for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
                        const int s = rs_s;
                        const uint32_t ph = rs_ph;
                        if (++rs_s == SE) { rs_s = 0; rs_ph ^= 1; }  // the ring position of it + 1
                        if (!mbar_wait_bounded(&empty[s], ph ^ 1, abort_flag, limit)) { ok = false; break; }
                        uint8_t* sa = stage_base + s * Cfg::STAGE_BYTES;
                        uint8_t* sb = sa + Cfg::A_BYTES;
                        if (kGemmTrace && p.trace && blockIdx.x == 0 && it < 128) p.trace[it] = clock64();
                        const bool load_b = bkey[s] != key0 + kb;
                        bkey[s] = key0 + kb;
                        const uint32_t b_tx = load_b ? Cfg::B_BYTES : 0u;
                        if constexpr (Cfg::kTap2) {
                            // taps tap and tap + 1 (the last stage of an odd tap count has one; the B box's
                            // second half then lies past K and is filled with zeros)
                            const bool two = tap + 1 < p.taps;
                            mbar_arrive_expect_tx(&full[s], Cfg::A_SUB * (two ? 2 : 1) + b_tx);
                            tma_load_im2col_4d(sa, &tmA, &full[s], 0, wb, hb, img, static_cast<uint16_t>(kx * p.dil_w),
                                               static_cast<uint16_t>(ky * p.dil_h));
                            if (load_b) tma_load_3d(sb, &tmB, &full[s], tap * p.IC, n0, 0);
                            ++tap;
                            if (++kx == p.KW) {
                                kx = 0;
                                ++ky;
                            }
                            if (two) {
                                tma_load_im2col_4d(sa + Cfg::A_SUB, &tmA, &full[s], 0, wb, hb, img,
                                                   static_cast<uint16_t>(kx * p.dil_w), static_cast<uint16_t>(ky * p.dil_h));
                                ++tap;
                                if (++kx == p.KW) {
                                    kx = 0;
                                    ++ky;
                                }
                            }
                            continue;
                        }
                        mbar_arrive_expect_tx(&full[s], Cfg::A_BYTES + b_tx);
                        if constexpr (Cfg::kIm2col) {
                            tma_load_im2col_4d(sa, &tmA, &full[s], cb * Cfg::BK, wb, hb, img,
                                               static_cast<uint16_t>(kx * p.dil_w), static_cast<uint16_t>(ky * p.dil_h));
                            if (load_b) tma_load_3d(sb, &tmB, &full[s], tap * p.IC + cb * Cfg::BK, n0, 0);
                            if (++cb == p.c_blocks) {
                                cb = 0;
                                ++tap;
                                if (++kx == p.KW) {
                                    kx = 0;
                                    ++ky;
                                }
                            }
                        } else {
                            tma_load_3d(sa, &tmA, &full[s], kb * Cfg::BK, m0, b);
                            if (!load_b) {
                            } else if constexpr (Cfg::kBMN) {
    #pragma unroll
                                for (int j = 0; j < BN / Cfg::B_MN_CHUNK; ++j)
                                    tma_load_3d(sb + j * Cfg::B_MN_BOX_BYTES, &tmB, &full[s], n0 + j * Cfg::B_MN_CHUNK,
                                                kb * Cfg::BK, b);
                            } else {
                                tma_load_3d(sb, &tmB, &full[s], kb * Cfg::BK, n0, p.b_bcast ? 0 : b);
                            }
                        }
                    }
                }
                if (!ok) { atomicOr(p.err, DEV_ERR_TIMEOUT); *abort_flag = 1; }
                // Drain: every issued load must land before the CTA may exit.
                const uint32_t first = it > static_cast<uint32_t>(SE) ? it - SE : 0;
                for (uint32_t i = first; i < it; ++i)
                    mbar_wait_bounded(&full[i % SE], (i / SE) & 1, nullptr, drain_limit);
            }
        } else if (warp == 1) {
            // ------------------------------------------------------------ MMA issuer
            if (lane == 0) {
                const uint32_t idesc = Cfg::kKind == 0 ? idesc_i8(BM, BN, Cfg::kBMN)
                                                       : idesc_f16(BM, BN, p.in_bf16 != 0, Cfg::kBMN);
                uint32_t it = 0, tcount = 0;
                int rs_s = 0;        // ring position of `it`, stepped
                uint32_t rs_ph = 0;
                bool ok = true;
                for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++tcount) {
                    const int buf = tcount & (NB - 1);
                    const uint32_t tph = (tcount >> NB_LOG) & 1;
                    if (!mbar_wait_bounded(&tempty[buf], tph ^ 1, abort_flag, limit)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
                    for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
                        const int s = rs_s;
                        const uint32_t ph = rs_ph;
                        if (++rs_s == SE) { rs_s = 0; rs_ph ^= 1; }
                        if (!mbar_wait_bounded(&full[s], ph, abort_flag, limit)) { ok = false; break; }
                        tc_fence_after();
                        if (kGemmTrace && p.trace && blockIdx.x == 0 && it < 128) p.trace[128 + it] = clock64();
                        const uint32_t sa = smem_u32(stage_base + s * Cfg::STAGE_BYTES);
                        const uint32_t sb = sa + Cfg::A_BYTES;
    #pragma unroll
                        for (int k = 0; k < Cfg::kBKBytesB / 32; ++k) {
                            // two taps per stage: k-steps 0-1 read A sub-tile 0, 2-3 sub-tile 1 (its stale
                            // contents meet zero weights in a one-tap stage)
                            const uint32_t a_k = Cfg::kTap2 ? sa + (k >> 1) * Cfg::A_SUB + (k & 1) * 32 : sa + k * 32;
                            const uint64_t ad = smem_desc(a_k, 16, Cfg::ATOM_SBO, Cfg::SW_CODE);
                            uint64_t bd;
                            if constexpr (Cfg::kBMN) {
                                // k-rows of 128 bytes; 8-row groups 1024 B apart; 128-byte N chunks one box apart.
                                bd = smem_desc(sb + k * Cfg::kMmaK * 128, Cfg::B_MN_BOX_BYTES, 1024, 2);
                            } else {
                                bd = smem_desc(sb + k * 32, 16, Cfg::ATOM_SBO_B, Cfg::SW_CODE_B);
                            }
                            tc_mma<Cfg::kKind>(d_tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                        }
                        tc_commit(&empty[s]);  // frees the stage once these MMAs have read it
                    }
                    if (!ok) break;
                    tc_commit(&tfull[buf]);    // accumulator ready for the epilogue
                }
                if (!ok) {
                    atomicOr(p.err, DEV_ERR_TIMEOUT);
                    *abort_flag = 1;
                }
                // Every issued MMA finishes before TMEM is released (also when the epilogue gave up
                // on tiles whose MMAs are still running).
                tc_commit(&mdrain[0]);
                mbar_wait_bounded(&mdrain[0], 0, nullptr, drain_limit);
            }
        } else {
            // ------------------------------------------------------------ A row sums (int8, zp_b != 0)
            if (need_rowsum) {
                const int row0 = (warp - 2) * 64;
                uint32_t it = 0, tcount = 0;
                int rs_s = 0;        // ring position of `it`, stepped
                uint32_t rs_ph = 0;
                bool ok = true;
                for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++tcount) {
                    int sum0 = 0, sum1 = 0;
                    for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
                        const int s = rs_s;
                        const uint32_t ph = rs_ph;
                        if (++rs_s == SE) { rs_s = 0; rs_ph ^= 1; }
                        if (!mbar_wait_bounded(&full[s], ph, abort_flag, limit)) { ok = false; break; }
                        const uint8_t* sa0 = stage_base + s * Cfg::STAGE_BYTES;
                        // two taps per stage: the second sub-tile holds data only when the stage has two taps
                        const int subs = Cfg::kTap2 && 2 * kb + 1 < p.taps ? 2 : 1;
                        for (int sub = 0; sub < subs; ++sub) {
                        const uint8_t* sa = sa0 + sub * Cfg::A_SUB;
                        const int4* r0 = reinterpret_cast<const int4*>(sa + (row0 + lane) * Cfg::kBKBytes);
                        const int4* r1 = reinterpret_cast<const int4*>(sa + (row0 + 32 + lane) * Cfg::kBKBytes);
                        // Chunk order rotated per lane: the 8 lanes of a shared-memory phase hit 8 different
                        // 16-byte bank groups (rows are 128, 64 or 32 bytes long).
                        const int rot = Cfg::kBKBytes == 128 ? (lane & 7)
                                                             : (Cfg::kBKBytes == 64 ? ((lane >> 1) & 3) : ((lane >> 2) & 1));
    #pragma unroll
                        for (int c = 0; c < Cfg::kBKBytes / 16; ++c) {
                            const int cc = c ^ rot;
                            const int4 v0 = r0[cc];
                            const int4 v1 = r1[cc];
                            sum0 = __dp4a(v0.x, 0x01010101, sum0);
                            sum0 = __dp4a(v0.y, 0x01010101, sum0);
                            sum0 = __dp4a(v0.z, 0x01010101, sum0);
                            sum0 = __dp4a(v0.w, 0x01010101, sum0);
                            sum1 = __dp4a(v1.x, 0x01010101, sum1);
                            sum1 = __dp4a(v1.y, 0x01010101, sum1);
                            sum1 = __dp4a(v1.z, 0x01010101, sum1);
                            sum1 = __dp4a(v1.w, 0x01010101, sum1);
                        }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[s]);
                        if (kGemmTrace && p.trace && blockIdx.x == 0 && it < 128 && warp == 2 && lane == 0) p.trace[256 + it] = clock64();
                    }
                    if (!ok) break;
                    const int buf = tcount & (NB - 1);
                    const uint32_t tph = (tcount >> NB_LOG) & 1;
                    if (!mbar_wait_bounded(&rsempty[buf], tph ^ 1, abort_flag, limit)) { ok = false; break; }
                    rowsum_buf[buf * 128 + row0 + lane] = sum0;
                    rowsum_buf[buf * 128 + row0 + 32 + lane] = sum1;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&rsfull[buf]);
                }
                if (!ok && lane == 0) { atomicOr(p.err, DEV_ERR_TIMEOUT); *abort_flag = 1; }
            }
        }
    } else {
        setmaxnreg_inc<kEpiRegs>();
        // ------------------------------------------------------------ epilogue (warps 4..15)
        // Three groups of 4 warps (one per TMEM lane quadrant). With p.epi_groups (several tiles
        // per CTA, BN <= 128) group g takes the tiles with tcount % 3 == g (accumulator buffer
        // tcount % 4) and every column of them, so each group's per-tile waits overlap the other
        // groups' work; otherwise the groups share every tile, group g taking chunks
        // [g * n / 3, (g + 1) * n / 3) of its n 32-column chunks.
        const int q = warp & 3;                 // TMEM lane quadrant
        const int grp = (warp - 4) >> 2;
        const int c_lo = 32 * ((grp * n_chunks) / kEpiGroups);
        const int c_hi = 32 * (((grp + 1) * n_chunks) / kEpiGroups);
        const int cols = p.epi_groups ? BN : c_hi - c_lo;  // columns per warp and tile
        const int cbase = p.epi_groups ? 0 : c_lo;
        const int row = q * 32 + lane;          // row within the tile
        const GemmEpilogue& e = p.epi;
        if (e.pdl_wait) grid_dependency_wait();
        const int et = threadIdx.x - 128;       // 0..383 within the epilogue warps
        // Bounded barrier of the 8 epilogue warps (an mbarrier phase per use).
        uint32_t ephase = 0;
        auto epi_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(&ebar[0]);
            const bool done = mbar_wait_bounded(&ebar[0], ephase, abort_flag, limit);
            ephase ^= 1;
            return done;
        };
        // [2 buffers][column terms, multiplier, shift - 32, hz][256] of the current tile
        int32_t* ct_stage = scratch + 1024;
        constexpr bool kPC = EK == EK_FAST_PC_S || EK == EK_FAST_PC_D;
        bool ok = true;
        uint32_t tcount = 0;
        uint32_t err = 0;
        uint32_t npass = 0;  // staging groups this warp has written (fast int8 epilogue)
        constexpr bool kFast = EK >= EK_FAST_T_S && EK <= EK_FAST_PC_D;
        // Tile-invariant RESCALE constants (per-tensor values are channel 0's).
        FastConst fk{0, 0, 0, 0, false, false, false};
        if constexpr (kFast) {
            fk.m = __ldg(e.fq_m);
            fk.sh = __ldg(e.sr_sh);
            fk.c = __ldg(e.sr_c);
            fk.add_zp = e.rs_zp_folded ? 0 : e.rs.out_zp;
            fk.clamp_lo = e.rs.lo > -128;
            fk.clamp_hi = e.rs.hi < 127;
            fk.clamp = fk.clamp_lo || fk.clamp_hi;
        }
        // Border-class tables of a convolution, copied to shared memory once.
        const uint8_t* rcls = e.rowclass;
        const uint8_t* ccls = e.colclass;
        if (e.rowclass != nullptr) {
            const int oh = p.conv_OHOW / p.conv_OW, ow = p.conv_OW;
            uint8_t* cl = reinterpret_cast<uint8_t*>(scratch);
            if (oh + ow <= 4096) {
                for (int i = et; i < oh; i += kEpiWarps * 32) cl[i] = e.rowclass[i];
                for (int i = et; i < ow; i += kEpiWarps * 32) cl[oh + i] = e.colclass[i];
                if (!epi_sync()) ok = false;
                rcls = cl;
                ccls = cl + oh;
            }
        }
        // Column constants (column terms and per-channel multiplier, shift - 32, hz) of the
        // current (batch, N tile) in shared memory; restaged only when the tile's batch or N
        // block changes (tiles walk M fastest). Two buffers: a warp that runs ahead writes
        // the other one; it cannot lap, as each staging ends in a barrier of all 12 warps.
        // The fast path always stages (zero column terms when there are none), so its
        // pointers are plain shared-memory pointers.
        const bool stage_cols = kFast || kPC || e.colterm != nullptr;
        int staged_key = -1;
        int sbuf = 0;
        // Whole tiles with at most four (batch, column tile) keys: every key's constants are
        // staged once, [key][column terms, multiplier, shift, c][128], and each group walks only
        // its own tiles (no per-tile key checks, no staging barriers inside the loop).
        const bool static_keys = p.epi_groups != 0 && stage_cols && BN <= 128 && p.batch * p.n_tiles <= 4;
        int cstride = 256;  // elements between the staged arrays of one key
        if (static_keys) {
            cstride = 128;
            for (int k = 0; k < p.batch * p.n_tiles; ++k) {
                const int bk = k / p.n_tiles, nk = k - bk * p.n_tiles;
                int32_t* cst = ct_stage + k * 512;
                for (int i = et; i < BN; i += kEpiWarps * 32) {
                    const int n = nk * BN + i;
                    cst[i] = e.colterm != nullptr ? e.colterm[bk * e.colterm_bstride + n] : 0;
                    if constexpr (kPC) {
                        cst[128 + i] = __ldg(e.fq_m + n);
                        cst[256 + i] = __ldg(e.sr_sh + n);
                        cst[384 + i] = __ldg(e.sr_c + n);
                    }
                }
            }
            if (!epi_sync()) ok = false;
            tcount = static_cast<uint32_t>(grp);
        }
        const int tstep = static_keys ? kEpiGroups : 1;
        for (int tile = blockIdx.x + (static_keys ? grp * static_cast<int>(gridDim.x) : 0); tile < p.total_tiles && ok;
             tile += tstep * gridDim.x, tcount += tstep) {
            int b, mt, nt;
            tile_coords(p, tile, b, mt, nt);
            const int buf = tcount & (NB - 1);
            const uint32_t tph = (tcount >> NB_LOG) & 1;
            const int key = b * p.n_tiles + nt;
            if (static_keys) {
                sbuf = key;  // (ct_stage + key * 512 below)
            } else if (stage_cols && key != staged_key) {
                sbuf ^= 1;
                int32_t* cst = ct_stage + sbuf * 1024;
                // (the tables are padded to whole 256-column tiles)
                if (et < BN) {
                    const int n = nt * BN + et;
                    cst[et] = e.colterm != nullptr ? e.colterm[b * e.colterm_bstride + n] : 0;
                    if constexpr (kPC) {
                        cst[256 + et] = __ldg(e.fq_m + n);
                        cst[512 + et] = __ldg(e.sr_sh + n);
                        cst[768 + et] = __ldg(e.sr_c + n);
                    }
                }
                if (!epi_sync()) { ok = false; break; }
                staged_key = key;
            }
            // (the column-constant staging above is shared by both groups: every warp passes
            // every tile's key check, so the staging barriers pair up)
            if (!static_keys && (p.epi_groups ? static_cast<int>(tcount % kEpiGroups) != grp : cols == 0)) continue;
            // Pointers indexed by the absolute output column.
            const int32_t* cst_n = ct_stage + sbuf * (static_keys ? 512 : 1024) - nt * BN;
            // Border class of this thread's row (before the accumulator wait: the lookups overlap it).
            const int m = mt * BM + row;
            const bool row_ok = m < p.M;
            const int32_t* delta = nullptr;       // general epilogue: null for the interior class
            const int32_t* delta_fast = nullptr;  // fast epilogue: the interior class's row is all zeros
            if (rcls != nullptr) {
                int cls = e.base_class;
                if (row_ok) {
                    const int rem = m - fdiv(m, p.fd_ohow) * p.conv_OHOW;
                    const int oy = fdiv(rem, p.fd_ow), ox = rem - oy * p.conv_OW;
                    cls = rcls[oy] * e.n_col_classes + ccls[ox];
                }
                delta_fast = e.ct_delta + static_cast<long long>(cls) * e.ct_ld;
                if (cls != e.base_class) delta = delta_fast;
            }
            // whether any row of this warp lies on a border (warp-uniform choice of the fast path)
            bool warp_delta = false;
            if constexpr ((EF & kEfDelta) != 0) warp_delta = __any_sync(0xffffffffu, delta != nullptr);
            if (!mbar_wait_bounded(&tfull[buf], tph, abort_flag, limit)) { ok = false; break; }
            tc_fence_after();
            if (kGemmTrace && p.trace && blockIdx.x == 0 && tcount < 8 && threadIdx.x == 128) p.trace[384 + 2 * tcount] = clock64();
            int32_t rowterm = 0;
            if (need_rowsum) {
                if (!mbar_wait_bounded(&rsfull[buf], tph, abort_flag, limit)) { ok = false; break; }
                rowterm = static_cast<int32_t>(static_cast<uint32_t>(e.row_zp_neg) *
                                               static_cast<uint32_t>(rowsum_buf[buf * 128 + row]));
                __syncwarp();
                if (lane == 0) mbar_arrive(&rsempty[buf]);
            }
            const int32_t* colterm = e.colterm != nullptr ? cst_n : nullptr;
            const int32_t* fm = cst_n + cstride;
            const int32_t* fsh = cst_n + 2 * cstride;
            const int32_t* fhz = cst_n + 3 * cstride;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(buf * BN + cbase);
            const long long orow = static_cast<long long>(b) * p.out_batch_stride + static_cast<long long>(m) * p.ldo;
            const int nb = nt * BN + cbase;
            if constexpr (EK >= EK_FAST_T_S && EK <= EK_FAST_PC_D) {
                // int8 results pass through a per-warp shared buffer [32 rows][GW bytes] (16-byte slots
                // swizzled by row): one TMA store of the block when the output allows it (p.tma_out),
                // else row-contiguous stores (a warp writes 8 rows x 64 B per store instead of 32
                // scattered 16 B pieces).
                uint4* wst = reinterpret_cast<uint4*>(scratch + 3072) + (warp - 4) * 256;
                int8_t* obase = reinterpret_cast<int8_t*>(p.out) + static_cast<long long>(b) * p.out_batch_stride;
                const bool vec_ok = (p.ldo & 15) == 0 && (p.out_batch_stride & 15) == 0 &&
                                    (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
                const int mrow0 = mt * BM + q * 32;
                // chunks that start at or beyond N (a partial last N tile) are skipped (the
                // conditions are warp-uniform, so the TMEM loads stay warp-collective)
                const int n_end = min(cols, p.N - nb);  // columns of this warp's part that exist
                // trace slots 416..479: per staging group, start / chunks done / stores done (CTA 0, tiles 0-1)
                long long* ftr = (kGemmTrace && p.trace && blockIdx.x == 0 && tcount < 2 && threadIdx.x == 128)
                                     ? p.trace + 416 + 32 * tcount : nullptr;
                // a warp with a border row adds every row's delta (zeros for interior rows)
                const FastTile h{&tmO, b, taddr, cols, n_end, nb, rowterm, cst_n, warp_delta ? delta_fast : nullptr,
                                 fm, fsh, fhz, wst, lane, mrow0, obase, vec_ok, ftr};
                fast_tile_pass<EK, (BN / 2 < 64 ? BN / 2 : 64), (EF & kEfRow) != 0, (EF & kEfDelta) != 0>(p, fk, h,
                                                                                                          npass);
            } else {
            // Two register sets: the next chunk's TMEM load overlaps this chunk's epilogue.
            uint32_t accA[kChunk], accB[kChunk];
            __syncwarp();
            tmem_ld_32x32b_x16(taddr, accA);
            tmem_wait_regs(accA);
#pragma unroll 1
            for (int c0 = 0; c0 < cols; c0 += 2 * kChunk) {
                const bool tr = kGemmTrace && p.trace && blockIdx.x == 0 && tcount == 0 && threadIdx.x == 128;
                if (tr) p.trace[408 + (c0 / kChunk) * 2] = clock64();
                __syncwarp();
                tmem_ld_32x32b_x16(taddr + c0 + kChunk, accB);
                if (row_ok && nb + c0 < p.N)
                    epilogue_chunk<EK>(p, accA, nb + c0, orow, rowterm, colterm, delta, fm, fsh, fhz, fk, err);
                if (tr) p.trace[409 + (c0 / kChunk) * 2] = clock64();
                __syncwarp();
                tmem_wait_regs(accB);
                if (c0 + 2 * kChunk < cols) tmem_ld_32x32b_x16(taddr + c0 + 2 * kChunk, accA);
                if (row_ok && nb + c0 + kChunk < p.N)
                    epilogue_chunk<EK>(p, accB, nb + c0 + kChunk, orow, rowterm, colterm, delta, fm, fsh, fhz, fk,
                                       err);
                __syncwarp();
                if (c0 + 2 * kChunk < cols) tmem_wait_regs(accA);
            }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            if (kGemmTrace && p.trace && blockIdx.x == 0 && tcount < 8 && threadIdx.x == 128) p.trace[385 + 2 * tcount] = clock64();
        }
        if (!ok && lane == 0) { atomicOr(p.err, DEV_ERR_TIMEOUT); *abort_flag = 1; }
        if (err) atomicOr(p.err, err);
        if (p.tma_out && lane == 0) bulk_wait0();  // the warp's TMA stores are done before the CTA exits
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
    // trace slots 403..405 (global timer, ns): CTA 0's start, the last CTA exit, the last CTA start
    if (kGemmTrace && p.trace && threadIdx.x == 0)
        atomicMax(reinterpret_cast<unsigned long long*>(p.trace + 404), globaltimer_ns());
}

}  // namespace tb
