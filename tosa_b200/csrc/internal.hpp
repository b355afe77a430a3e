// Internal host-side definitions shared by the backend's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/tosa_b200.h"

// GEMM timeline stamps (clock64 of CTA 0 into tb_context::trace): compiled into the
// tensor-core kernels only when the library is built with -DTB_GEMM_TRACE=1.
#ifndef TB_GEMM_TRACE
#define TB_GEMM_TRACE 0
#endif
constexpr bool kGemmTrace = TB_GEMM_TRACE != 0;

struct tb_context {
    int device = 0;
    int num_sms = 148;
    uint32_t* dev_err = nullptr;     // device error word (DEV_ERR_* bits)
    long long timeout_cycles = 0;    // bound on every in-kernel wait
    uint64_t launches = 0;
    long long* trace = nullptr;      // optional GEMM timeline buffer (TB_TRACE=1, TB_GEMM_TRACE builds)
    int epi_groups = -1;             // TB_GEMM_EPI_GROUPS: 0 / 1 force the GEMM epilogue form, -1 by tile count
};

namespace tb {

// Records the calling thread's last error message and returns `st`.
tb_status fail(tb_status st, const char* fmt, ...);

#define TB_CUDA(call)                                                                          \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return ::tb::fail(TB_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));    \
    } while (0)

// After a kernel launch: report a launch error, else count the launch.
#define TB_LAUNCHED(ctx)                                                                               \
    do {                                                                                               \
        cudaError_t e_ = cudaGetLastError();                                                           \
        if (e_ != cudaSuccess) return ::tb::fail(TB_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e_)); \
        (ctx)->launches++;                                                                             \
    } while (0)

#define TB_TRY(expr)                         \
    do {                                     \
        tb_status s_ = (expr);               \
        if (s_ != TB_OK) return s_;          \
    } while (0)

// Driver entry points fetched through the runtime (no libcuda link).
tb_status encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                       const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);
tb_status encode_im2col(CUtensorMap* map, CUtensorMapDataType dt, const void* base, const uint64_t* dims /*C,W,H,N*/,
                        const uint64_t* strides_bytes /*3*/, const int* lower /*w,h*/, const int* upper /*w,h*/,
                        uint32_t channels, uint32_t pixels, const uint32_t* elem_strides /*4*/,
                        CUtensorMapSwizzle swz);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int elem_bytes(int dt) {
    switch (dt) {
    case TB_DT_BOOL: case TB_DT_INT4: case TB_DT_INT8: case TB_DT_FP8E4M3: case TB_DT_FP8E5M2: return 1;
    case TB_DT_INT16: case TB_DT_FP16: case TB_DT_BF16: return 2;
    case TB_DT_INT32: case TB_DT_FP32: return 4;
    default: return 8;
    }
}

// Resolved RESCALE epilogue (device copies of multiplier/shift).
struct RescalePlan {
    bool enabled = false;
    int scale32 = 1, rounding = 1, per_channel = 0, channels = 1;
    int32_t out_zp = 0, lo = 0, hi = 0;
    int out_dtype = TB_DT_INT32;
    bool fast = false;             // every shift in [33, 62], multiplier >= 0 (scale32 single/double)
    bool zp_folded = false;        // the output zero point rides in fq_hz
    int32_t* d_mult = nullptr;     // [channels]
    int32_t* d_shift = nullptr;    // [channels]
    // Fast path, three arrays of `padded` (channels rounded up to 256) words:
    //   fq_m  multiplier, fq_sh  shift - 32, fq_hz  2^(shift-33) (+ out_zp * 2^(shift-32) when folded)
    // r = ((high word of v*m [+-2^30 by the sign of v under double rounding]) + hz) >> sh [+ out_zp]
    int32_t* fq_m = nullptr;
    int32_t* fq_sh = nullptr;
    int32_t* fq_hz = nullptr;
    int32_t* d_blob = nullptr;     // owned allocation holding the fast arrays, multiplier and shift
};

// Small-range constants of a GEMM's fused int8 RESCALE (tc_gemm.cuh GemmEpilogue): with a
// host bound |v| <= bound on the int32 value, k = the largest shift with bound * 2^k < 2^31,
// d = 32 - k, per channel sh = s - d and c = 2^(s-1-d) [+ 2^(30-d)] [+ zp * 2^(s-d)].
struct SmallRange {
    bool ok = false;
    int k = 0;
    int32_t mul = 1, k2 = 0;
    bool zp_folded = false;
    int32_t* d_blob = nullptr;  // owned (make_small_range): sh then c, each padded to 256 channels
    int32_t* d_sh = nullptr;
    int32_t* d_c = nullptr;
};
// Host half: fills sr (ok = false when the form does not apply) and the blob words.
void prepare_small_range(const tb_rescale_attr& a, const RescalePlan& rs, long long bound, SmallRange* sr,
                         std::vector<int32_t>* blob);
void place_small_range(SmallRange* sr, int32_t* dev_blob, int channels);
tb_status make_small_range(const tb_rescale_attr& a, const RescalePlan& rs, long long bound, SmallRange* sr);
void free_small_range(SmallRange* sr);

// Validate a fused/standalone RESCALE (src/ops/type_conv.rs:128-171) for
// input type in_dtype with `shape_last` as the last dimension.
tb_status check_rescale(const tb_rescale_attr* a, int in_dtype, int64_t shape_last, int64_t* in_zp_ext,
                        int64_t* out_zp_ext, int32_t* lo, int32_t* hi);
tb_status make_rescale_plan(tb_context* ctx, const tb_rescale_attr* a, int in_dtype, int64_t shape_last,
                            RescalePlan* out);
void free_rescale_plan(RescalePlan* r);
// Host half of make_rescale_plan: validates and builds the device blob
// (packed fast-path constants, multipliers, shifts) without allocating.
tb_status prepare_rescale(const tb_rescale_attr* a, int in_t, int64_t shape_last, RescalePlan* r,
                          std::vector<int32_t>* blob);
// Points the plan's device arrays into a blob already copied to the device.
void place_rescale(RescalePlan* r, int32_t* dev_blob);

int grid_for(const tb_context* ctx, long long work, int block = 256);

struct RescaleArgs;
RescaleArgs rescale_args(const RescalePlan& r);

// Index map of an N-d elementwise pass (rank <= 6): output dims, and the
// element strides of operands a/b along each output dimension (0 = broadcast).
struct NdMap {
    long long dims[6];
    long long a_stride[6];
    long long b_stride[6];
};

// AVG_POOL2D / MAX_POOL2D geometry checks (src/ops/pool.rs:31-70).
tb_status pool_check(const char* op, const tb_pool2d_desc* d, int* oh, int* ow);

// Graph glue launchers (glue.cu).
tb_status launch_transpose(tb_context* ctx, const void* in, void* out, int elem, long long total, int rank,
                           const NdMap& map, cudaStream_t st);
tb_status launch_add_broadcast(tb_context* ctx, int dtype, const void* a, const void* b, long long total, int rank,
                               const NdMap& map, void* out, cudaStream_t st);
tb_status launch_rescale(tb_context* ctx, const RescalePlan& r, int in_dtype, int in_uns, int32_t izp, const void* in,
                         long long count, int channels, void* out, cudaStream_t st);
// Per-tensor constants of the residual chain's two input RESCALEs when neither can
// raise an error (int8 inputs, scale32 single/double rounding, every |x - zp| below
// 2^(shift-1) and every result inside int32): r = (x * m + R) >> shift, R chosen by
// the sign of x. `ok` false: the general kernel runs.
struct ResidualFast {
    bool ok = false;
    int32_t ma = 0, za = 0, sa = 0, mb = 0, zb = 0, sb = 0;
    long long ra_pos = 0, ra_neg = 0, rb_pos = 0, rb_neg = 0;
    // Small-range output RESCALE (per-tensor, shift in [33, 62]): every table value is
    // pre-shifted by k (|a| + |b| < 2^(31-k)), so sum' = sum * 2^k, and with d = 32 - k
    // r = (mulhi(sum', om) + oc [- ok2 when sum' < 0, double rounding]) >> osh [+ ozp_add],
    // oc = 2^(s-1-d) [+ 2^(30-d)] [+ zp * 2^(s-d)], ok2 = 2^(31-d), osh = s - d.
    bool small = false;
    int k = 0;
    int32_t om = 0, osh = 0, oc = 0, ok2 = 0, ozp_add = 0;
    // With a per-tensor output RESCALE the whole chain is a function of the two input bytes:
    // d_table holds its int8 result for every byte pair, at a * 256 + (b ^ ((a & 31) << 2))
    // (bank swizzle; glue.cu) (owned; null when not built).
    uint8_t* d_table = nullptr;
};
// Fills `f` from host copies of the two input RESCALE attributes (int8 inputs, int32
// outputs) and of the output RESCALE (int32 -> int8).
void residual_fast_constants(const tb_rescale_attr& a, int a_dt, const tb_rescale_attr& b, int b_dt,
                             const tb_rescale_attr& o, ResidualFast* f);
// Builds f->d_table (see ResidualFast) when f->ok, the output RESCALE `o` is per-tensor
// int32 -> int8 with a 32-bit multiplier and no entry of the table raises a RESCALE error;
// `ro` supplies the combined clamp. Leaves d_table null otherwise.
tb_status make_residual_table(const tb_rescale_attr& o, const RescalePlan& ro, ResidualFast* f);
void free_residual_table(ResidualFast* f);
tb_status launch_residual(tb_context* ctx, const void* a, int a_dt, int a_uns, int32_t za, const RescalePlan& ra,
                          const void* b, int b_dt, int b_uns, int32_t zb, const RescalePlan& rb,
                          const RescalePlan& ro, const ResidualFast& fast, long long count, int channels, void* out,
                          cudaStream_t st);

// MATMUL static checks (src/ops/matmul.rs:112-153) and path choice:
// path 0 tensor-core int8, 1 tensor-core f16/bf16, 2 direct int8, 3 direct float.
// t_batch: 0 for MATMUL; for MATMUL_T the batch of B [t_batch, w, c] (n or 1)
tb_status matmul_validate(const tb_matmul_desc* d, bool has_rescale, int* path, int* bn, int t_batch = 0);

}  // namespace tb

// A prepared MATMUL (see tb_matmul_plan_create).
struct tb_matmul_plan {
    tb_context* ctx = nullptr;
    tb_matmul_desc d{};
    int path = 0;  // 0 TC int8, 1 TC f16/bf16, 2 direct int, 3 direct float, 4 direct int16, 5 TC int8, padded B
    int t_batch = 0;  // MATMUL_T: batch of B [t_batch, w, c] (n, or 1 broadcast); 0 for MATMUL
    tb::RescalePlan rs;
    tb::SmallRange sr;
    int bn = 256;
    int32_t* d_colterm = nullptr;  // [n][w] (+ one tile of padding) when a_zp != 0
    int wp = 0;                // path 5: padded B row length
    int8_t* d_bpad = nullptr;  // path 5: [n][c][wp] copy of B
    const void* a_cached = nullptr;
    const void* b_cached = nullptr;
    const void* b_const = nullptr;  // B declared constant: d_colterm / d_bpad hold its column terms / padded rows
    const void* o_cached = nullptr; // output the TMA-store map tmO was made for
    CUtensorMap tmA, tmB, tmO;
};
