// Host side of libtosa_b200: contexts, tensor maps, the static ERROR_IF
// checks of each operator (as the reference performs them before computing),
// plans that precompute zero-point terms, and kernel launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.hpp"
#include "simt_kernels.cuh"
#include "simt_ops.cuh"
#include "gemm_launch.cuh"

namespace tb {

static thread_local std::string g_last_error;

tb_status fail(tb_status st, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

// ---------------------------------------------------------------------------
// Tensor maps (driver entry points resolved through the runtime)
// ---------------------------------------------------------------------------

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
typedef CUresult (*PFN_encodeIm2col)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                     const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                     CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled g_encode_tiled = nullptr;
static PFN_encodeIm2col g_encode_im2col = nullptr;
static std::once_flag g_encode_once;

static tb_status load_encoders() {
    std::call_once(g_encode_once, [] {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode_tiled = reinterpret_cast<PFN_encodeTiled>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode_im2col = reinterpret_cast<PFN_encodeIm2col>(fn);
    });
    if (!g_encode_tiled || !g_encode_im2col) return fail(TB_ERR_CUDA, "cuTensorMapEncode* entry points unavailable");
    return TB_OK;
}

tb_status encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                       const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
    TB_TRY(load_encoders());
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    CUresult r = g_encode_tiled(map, dt, rank, const_cast<void*>(base), dims, strides_bytes, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return TB_OK;
}

tb_status encode_im2col(CUtensorMap* map, CUtensorMapDataType dt, const void* base, const uint64_t* dims,
                        const uint64_t* strides_bytes, const int* lower, const int* upper, uint32_t channels,
                        uint32_t pixels, const uint32_t* elem_strides, CUtensorMapSwizzle swz) {
    TB_TRY(load_encoders());
    CUresult r = g_encode_im2col(map, dt, 4, const_cast<void*>(base), dims, strides_bytes, lower, upper, channels,
                                 pixels, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TB_ERR_CUDA, "cuTensorMapEncodeIm2col failed (%d)", static_cast<int>(r));
    return TB_OK;
}

static CUtensorMapDataType tmap_dtype(int dt) {
    if (dt == TB_DT_BF16) return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (dt == TB_DT_FP16) return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return CU_TENSOR_MAP_DATA_TYPE_UINT8;
}

int grid_for(const tb_context* ctx, long long work, int block) {
    long long g = (work + block - 1) / block;
    long long cap = static_cast<long long>(ctx->num_sms) * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}


// ---------------------------------------------------------------------------
// RESCALE validation (src/ops/type_conv.rs:128-171) and device plan
// ---------------------------------------------------------------------------

static int bit_width(int dt) { return dt == TB_DT_INT8 ? 8 : dt == TB_DT_INT16 ? 16 : dt == TB_DT_INT32 ? 32 : 48; }
static void int_range(int dt, int64_t* lo, int64_t* hi) {
    switch (dt) {
    case TB_DT_INT8: *lo = -128; *hi = 127; break;
    case TB_DT_INT16: *lo = -32768; *hi = 32767; break;
    case TB_DT_INT32: *lo = INT32_MIN; *hi = INT32_MAX; break;
    default: *lo = -(1ll << 47); *hi = (1ll << 47) - 1;
    }
}

tb_status check_rescale(const tb_rescale_attr* a, int in_t, int64_t shape_last, int64_t* in_zp_ext, int64_t* out_zp_ext,
                        int32_t* lo, int32_t* hi) {
    const int out_t = a->out_dtype;
    if (!(in_t == TB_DT_INT8 || in_t == TB_DT_INT16 || in_t == TB_DT_INT32 || in_t == TB_DT_INT48) ||
        !(out_t == TB_DT_INT8 || out_t == TB_DT_INT16 || out_t == TB_DT_INT32))
        return fail(TB_ERR_DTYPE_MISMATCH, "RESCALE: unsupported types %d -> %d", in_t, out_t);
    if (a->rounding_mode < 1 || a->rounding_mode > 3) return fail(TB_ERR_GRAPH, "RESCALE: unsupported rounding mode");
    if (a->scale32 && in_t == TB_DT_INT48) return fail(TB_ERR_GRAPH, "RESCALE: scale32 is not allowed for INT48 input");
    if (!a->scale32 && a->rounding_mode == TB_ROUND_DOUBLE)
        return fail(TB_ERR_GRAPH, "RESCALE: double rounding requires scale32");
    const bool has32 = in_t == TB_DT_INT32 || in_t == TB_DT_INT48 || out_t == TB_DT_INT32;
    if ((a->input_unsigned && a->output_unsigned) || ((a->input_unsigned || a->output_unsigned) && has32))
        return fail(TB_ERR_GRAPH, "RESCALE: invalid combination of input_unsigned/output_unsigned and types");
    const int64_t channels = a->per_channel ? shape_last : 1;
    if (a->channels != channels)
        return fail(TB_ERR_GRAPH, "RESCALE: multiplier and shift must have %lld elements", (long long)channels);
    if (!a->multiplier || !a->shift) return fail(TB_ERR_INVALID_ARGUMENT, "RESCALE: null multiplier/shift");
    auto extend = [](int dt, int64_t v, bool uns) { return uns ? (v & ((1ll << bit_width(dt)) - 1)) : v; };
    const int64_t izp = extend(in_t, a->input_zp, a->input_unsigned);
    const int64_t ozp = extend(out_t, a->output_zp, a->output_unsigned);
    auto zp_ok = [](int dt, int64_t zp, bool uns) {
        return dt == TB_DT_INT8 || zp == 0 || (dt == TB_DT_INT16 && uns && zp == 32768);
    };
    if (!zp_ok(in_t, izp, a->input_unsigned) || !zp_ok(out_t, ozp, a->output_unsigned))
        return fail(TB_ERR_GRAPH, "RESCALE: zero point not allowed for this type");
    int64_t l, h;
    if (a->output_unsigned) { l = 0; h = (1ll << bit_width(out_t)) - 1; }
    else int_range(out_t, &l, &h);
    if (a->clamp_enabled) {
        if (a->clamp_max < a->clamp_min) return fail(TB_ERR_GRAPH, "CLAMP: max_val must not be smaller than min_val");
        if (a->output_unsigned) return fail(TB_ERR_NOT_ACCELERATED, "CLAMP fusion after an unsigned RESCALE");
        // clamp(clamp(v, l, h), cmin, cmax) as one clamp (constant when disjoint).
        int64_t nl = std::max<int64_t>(l, a->clamp_min), nh = std::min<int64_t>(h, a->clamp_max);
        if (nl > nh) {
            const int64_t c = a->clamp_min > h ? a->clamp_min : a->clamp_max;
            nl = nh = c;
        }
        l = nl;
        h = nh;
    }
    *in_zp_ext = izp;
    *out_zp_ext = ozp;
    *lo = static_cast<int32_t>(l);
    *hi = static_cast<int32_t>(h);
    return TB_OK;
}

tb_status prepare_rescale(const tb_rescale_attr* a, int in_t, int64_t shape_last, RescalePlan* r,
                          std::vector<int32_t>* blob) {
    int64_t izp, ozp;
    int32_t lo, hi;
    TB_TRY(check_rescale(a, in_t, shape_last, &izp, &ozp, &lo, &hi));
    r->enabled = true;
    r->scale32 = a->scale32;
    r->rounding = a->rounding_mode;
    r->per_channel = a->per_channel;
    r->channels = a->channels;
    r->out_zp = static_cast<int32_t>(ozp);
    r->lo = lo;
    r->hi = hi;
    r->out_dtype = a->out_dtype;
    std::vector<int32_t> m(a->channels), s(a->channels);
    bool fast = a->scale32 && a->rounding_mode != TB_ROUND_INEXACT && izp == 0;
    for (int i = 0; i < a->channels; ++i) {
        m[i] = a->multiplier[i];
        s[i] = a->shift[i];
        if (m[i] < 0 || s[i] < 33 || s[i] > 62) fast = false;
    }
    r->fast = fast;
    // Blob layout (int32 words): [fast path: m, sh, hz, each padded to whole 256-channel tiles with
    // channel 0] [multiplier] [shift].
    //   With s >= 33 every int32 v is in apply_scale_32's range and
    //   (v*m + 2^(s-1) +- 2^30) >> s == (hi32(v*m +- 2^30) + 2^(s-33)) >> (s-32)
    // (adding a multiple of 2^32 to the 64-bit sum adds it to the high word; the nested floor is
    // exact). The output zero point joins hz as zp * 2^(s-32) when that stays inside int32.
    const size_t padded = (static_cast<size_t>(a->channels) + 255) / 256 * 256;
    const size_t fq_words = fast ? 3 * padded : 0;
    blob->assign(fq_words + 2 * static_cast<size_t>(a->channels), 0);
    if (fast) {
        bool fold = true;
        for (int i = 0; i < a->channels; ++i) {
            const long long hz = (1ll << (s[i] - 33)) + static_cast<long long>(ozp) * (1ll << (s[i] - 32));
            if (hz < INT32_MIN || hz > INT32_MAX) fold = false;
        }
        r->zp_folded = fold;
        for (size_t pi = 0; pi < padded; ++pi) {
            const int i = pi < static_cast<size_t>(a->channels) ? static_cast<int>(pi) : 0;
            const long long hz = (1ll << (s[i] - 33)) + (fold ? static_cast<long long>(ozp) * (1ll << (s[i] - 32)) : 0);
            (*blob)[pi] = m[i];
            (*blob)[padded + pi] = s[i] - 32;
            (*blob)[2 * padded + pi] = static_cast<int32_t>(hz);
        }
    }
    std::copy(m.begin(), m.end(), blob->begin() + fq_words);
    std::copy(s.begin(), s.end(), blob->begin() + fq_words + a->channels);
    return TB_OK;
}

void place_rescale(RescalePlan* r, int32_t* dev_blob) {
    const size_t padded = (static_cast<size_t>(r->channels) + 255) / 256 * 256;
    const size_t fq_words = r->fast ? 3 * padded : 0;
    r->fq_m = r->fast ? dev_blob : nullptr;
    r->fq_sh = r->fast ? dev_blob + padded : nullptr;
    r->fq_hz = r->fast ? dev_blob + 2 * padded : nullptr;
    r->d_mult = dev_blob + fq_words;
    r->d_shift = dev_blob + fq_words + r->channels;
}

tb_status make_rescale_plan(tb_context* ctx, const tb_rescale_attr* a, int in_t, int64_t shape_last, RescalePlan* r) {
    (void)ctx;
    std::vector<int32_t> blob;
    TB_TRY(prepare_rescale(a, in_t, shape_last, r, &blob));
    TB_CUDA(cudaMalloc(&r->d_blob, sizeof(int32_t) * blob.size()));
    TB_CUDA(cudaMemcpy(r->d_blob, blob.data(), sizeof(int32_t) * blob.size(), cudaMemcpyHostToDevice));
    place_rescale(r, r->d_blob);
    return TB_OK;
}

void prepare_small_range(const tb_rescale_attr& a, const RescalePlan& rs, long long bound, SmallRange* sr,
                         std::vector<int32_t>* blob) {
    *sr = SmallRange{};
    blob->clear();
    if (!rs.enabled || !rs.fast || rs.out_dtype != TB_DT_INT8 || bound < 0) return;
    int k = 0;
    while (k < 30 && (std::max(bound, 1ll) << (k + 1)) <= 2147483647ll) ++k;
    if ((std::max(bound, 1ll) << k) > 2147483647ll) return;
    const bool dbl = rs.rounding == TB_ROUND_DOUBLE;
    if (dbl && k < 2) return;
    const int d = 32 - k;
    const long long k2 = dbl ? (1ll << (31 - d)) : 0;
    const int ch = a.channels;
    auto cterm = [&](int i, bool fold) {
        const int s = a.shift[i];
        return (1ll << (s - 1 - d)) + (dbl ? (1ll << (30 - d)) : 0) +
               (fold ? static_cast<long long>(rs.out_zp) * (1ll << (s - d)) : 0);
    };
    bool fold = true, plain = true;
    for (int i = 0; i < ch; ++i) {
        if (a.shift[i] - 1 < d) return;
        if (std::llabs(cterm(i, true)) + k2 >= (1ll << 30)) fold = false;
        if (std::llabs(cterm(i, false)) + k2 >= (1ll << 30)) plain = false;
    }
    if (!fold && !plain) return;
    const size_t padded = (static_cast<size_t>(ch) + 255) / 256 * 256;
    blob->assign(2 * padded, 0);
    for (size_t pi = 0; pi < padded; ++pi) {
        const int i = pi < static_cast<size_t>(ch) ? static_cast<int>(pi) : 0;
        (*blob)[pi] = std::min(a.shift[i] - d, 31);
        (*blob)[padded + pi] = static_cast<int32_t>(cterm(i, fold));
    }
    sr->ok = true;
    sr->k = k;
    sr->mul = static_cast<int32_t>(1u << k);
    sr->k2 = static_cast<int32_t>(k2);
    sr->zp_folded = fold;
}

void place_small_range(SmallRange* sr, int32_t* dev_blob, int channels) {
    const size_t padded = (static_cast<size_t>(channels) + 255) / 256 * 256;
    sr->d_sh = dev_blob;
    sr->d_c = dev_blob + padded;
}

tb_status make_small_range(const tb_rescale_attr& a, const RescalePlan& rs, long long bound, SmallRange* sr) {
    std::vector<int32_t> blob;
    prepare_small_range(a, rs, bound, sr, &blob);
    if (!sr->ok) return TB_OK;
    TB_CUDA(cudaMalloc(&sr->d_blob, sizeof(int32_t) * blob.size()));
    TB_CUDA(cudaMemcpy(sr->d_blob, blob.data(), sizeof(int32_t) * blob.size(), cudaMemcpyHostToDevice));
    place_small_range(sr, sr->d_blob, a.channels);
    return TB_OK;
}

void free_small_range(SmallRange* sr) {
    if (sr->d_blob) cudaFree(sr->d_blob);
    *sr = SmallRange{};
}

void free_rescale_plan(RescalePlan* r) {
    if (r->d_blob) cudaFree(r->d_blob);
    r->d_blob = nullptr;
    r->d_mult = r->d_shift = r->fq_m = r->fq_sh = r->fq_hz = nullptr;
}

// The GEMM's fast int8 RESCALE (small-range form) when both the plan's RESCALE and its
// bound allow it; otherwise the general epilogue (rs_fast = 0) with unscaled terms.
static void set_fast_epilogue(GemmEpilogue* ep, const RescalePlan& rs, const SmallRange& sr) {
    ep->rs_fast = rs.fast && sr.ok;
    ep->rs_zp_folded = sr.zp_folded;
    ep->sr_mul = sr.ok ? sr.mul : 1;
    ep->sr_k2 = sr.k2;
    ep->fq_m = rs.fq_m;
    ep->sr_sh = sr.d_sh;
    ep->sr_c = sr.d_c;
}

// The fast int8 epilogue stores each warp's staged [32 rows][GW] block with one TMA store when
// the output rows are 16-byte multiples and the output is 16-byte aligned: a 3-D map
// (N, M, batch) over the output, box [GW = min(BN / 2, 64), 32, 1], swizzled as the staging
// buffer is laid out. The map is made once per output pointer (`cached`). Otherwise (or if the
// map cannot be made) the epilogue keeps its per-thread stores.
static void prepare_tma_out(GemmParams* gp, int bn, CUtensorMap* map, const void** cached) {
    gp->tma_out = 0;
    const int ek = epilogue_kind(gp->epi);
    if (ek < EK_FAST_T_S || ek > EK_FAST_PC_D) return;
    const long long bstride = gp->batch > 1 ? gp->out_batch_stride : gp->ldo * gp->M;
    if (gp->ldo % 16 != 0 || bstride % 16 != 0 || !aligned16(gp->out)) return;
    if (gp->out != *cached) {
        const uint32_t gw = bn / 2 < 64 ? static_cast<uint32_t>(bn / 2) : 64u;
        const uint64_t dims[3] = {static_cast<uint64_t>(gp->N), static_cast<uint64_t>(gp->M),
                                  static_cast<uint64_t>(gp->batch)};
        const uint64_t str[2] = {static_cast<uint64_t>(gp->ldo), static_cast<uint64_t>(bstride)};
        const uint32_t box[3] = {gw, 32, 1};
        if (encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, gp->out, dims, str, box,
                         gw == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B) != TB_OK)
            return;
        *cached = gp->out;
    }
    gp->tma_out = 1;
    gp->tmo_host = map;
}

RescaleArgs rescale_args(const RescalePlan& r) {
    RescaleArgs a;
    a.multiplier = r.d_mult;
    a.shift = r.d_shift;
    a.per_channel = r.per_channel;
    a.scale32 = r.scale32;
    a.rounding = r.rounding;
    a.out_zp = r.out_zp;
    a.lo = r.lo;
    a.hi = r.hi;
    return a;
}

IntEpiDev int_epi(const RescalePlan& r) {
    IntEpiDev e;
    e.rescale = r.enabled ? 1 : 0;
    e.rs = rescale_args(r);
    e.out_dtype = r.enabled ? r.out_dtype : TB_DT_INT32;
    return e;
}

// ---------------------------------------------------------------------------
// Tensor-core GEMM launch (one instantiation per tile configuration)
// ---------------------------------------------------------------------------

// Tensor-core GEMM launches live in gemm_i8_mm.cu, gemm_i8_conv.cu and gemm_f16.cu
// (one translation unit per family so they compile in parallel).

}  // namespace tb

using namespace tb;

// ===========================================================================
// C ABI: context
// ===========================================================================

extern "C" {

TB_API const char* tb_last_error(void) { return g_last_error.c_str(); }

TB_API tb_status tb_context_create(int device, tb_context** out) {
    if (!out) return fail(TB_ERR_INVALID_ARGUMENT, "null output pointer");
    *out = nullptr;
    int count = 0;
    TB_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count) return fail(TB_ERR_INVALID_ARGUMENT, "no CUDA device %d", device);
    TB_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    TB_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(TB_ERR_NOT_ACCELERATED, "device %d is sm_%d%d; this library is built for sm_100a", device,
                    prop.major, prop.minor);
    tb_context* ctx = new tb_context;
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    double ms = 2000.0;
    if (const char* env = getenv("TB_WAIT_TIMEOUT_MS")) ms = atof(env);
    ctx->timeout_cycles = static_cast<long long>(ms * 1e-3 * prop.clockRate * 1e3);
    cudaError_t e = cudaMalloc(&ctx->dev_err, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(ctx->dev_err, 0, sizeof(uint32_t));
    if (e != cudaSuccess) {
        delete ctx;
        return fail(TB_ERR_CUDA, "error-word allocation failed: %s", cudaGetErrorString(e));
    }
    if (const char* env = getenv("TB_TRACE")) {
        if (kGemmTrace && atoi(env) && cudaMalloc(&ctx->trace, 512 * sizeof(long long)) == cudaSuccess)
            cudaMemset(ctx->trace, 0, 512 * sizeof(long long));
    }
    // TB_GEMM_EPI_GROUPS=0 / 1: every tensor-core GEMM splits each tile's epilogue by column
    // thirds (0) or, for tiles of at most 128 columns, gives whole tiles to the three epilogue
    // groups in turn (1), whatever the tile count (tests run both forms on small shapes)
    if (const char* env = getenv("TB_GEMM_EPI_GROUPS")) {
        const int v = atoi(env);
        if (v == 0 || v == 1) ctx->epi_groups = v;
    }
    *out = ctx;
    return TB_OK;
}

TB_API tb_status tb_context_set_wait_timeout_ms(tb_context* ctx, double ms) {
    if (!ctx) return fail(TB_ERR_INVALID_ARGUMENT, "null context");
    if (!(ms >= 0.0) || ms > 3.6e6) return fail(TB_ERR_INVALID_ARGUMENT, "wait timeout %g ms out of range", ms);
    int khz = 0;
    TB_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, ctx->device));
    ctx->timeout_cycles = static_cast<long long>(ms * 1e-3 * khz * 1e3);
    return TB_OK;
}

TB_API tb_status tb_debug_trace(tb_context* ctx, long long* host512) {
    if (!ctx || !host512) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    if (!ctx->trace)
        return fail(TB_ERR_INVALID_ARGUMENT, "no trace buffer: a library built with -DTB_GEMM_TRACE=1 and TB_TRACE=1 "
                                             "at context creation are both needed");
    TB_CUDA(cudaMemcpy(host512, ctx->trace, 512 * sizeof(long long), cudaMemcpyDeviceToHost));
    return TB_OK;
}

TB_API void tb_context_destroy(tb_context* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->trace) cudaFree(ctx->trace);
    delete ctx;
}

TB_API tb_status tb_synchronize(tb_context* ctx, void* stream) {
    if (!ctx) return fail(TB_ERR_INVALID_ARGUMENT, "null context");
    TB_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    uint32_t word = 0;
    TB_CUDA(cudaMemcpy(&word, ctx->dev_err, sizeof word, cudaMemcpyDeviceToHost));
    if (word) {
        TB_CUDA(cudaMemset(ctx->dev_err, 0, sizeof(uint32_t)));
        if (word & DEV_ERR_TIMEOUT) return fail(TB_ERR_TIMEOUT, "a device wait timed out (error word 0x%x)", word);
        if (word & DEV_ERR_SCALE)
            return fail(TB_ERR_GRAPH, "apply_scale: value out of range for the shift, or result exceeds int32");
        return fail(TB_ERR_GRAPH, "device error word 0x%x", word);
    }
    return TB_OK;
}

TB_API tb_status tb_malloc(tb_context* ctx, size_t bytes, void** dptr) {
    if (!ctx || !dptr) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    TB_CUDA(cudaMalloc(dptr, bytes ? bytes : 1));
    return TB_OK;
}

TB_API tb_status tb_free(tb_context* ctx, void* dptr) {
    if (!ctx) return fail(TB_ERR_INVALID_ARGUMENT, "null context");
    if (dptr) TB_CUDA(cudaFree(dptr));
    return TB_OK;
}

TB_API tb_status tb_memcpy_h2d(tb_context* ctx, void* dst, const void* src, size_t bytes, void* stream) {
    if (!ctx) return fail(TB_ERR_INVALID_ARGUMENT, "null context");
    TB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
    return TB_OK;
}

TB_API tb_status tb_memcpy_d2h(tb_context* ctx, void* dst, const void* src, size_t bytes, void* stream) {
    if (!ctx) return fail(TB_ERR_INVALID_ARGUMENT, "null context");
    TB_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
    return TB_OK;
}

TB_API uint64_t tb_launch_count(tb_context* ctx) { return ctx ? ctx->launches : 0; }

}  // extern "C"

// ===========================================================================
// MATMUL
// ===========================================================================


namespace tb {

tb_status matmul_validate(const tb_matmul_desc* d, bool has_rescale, int* path, int* bn, int t_batch) {
    const bool tr = t_batch != 0;
    const char* name = tr ? "MATMUL_T" : "MATMUL";
    if (d->n < 0 || d->h < 0 || d->c < 0 || d->w < 0) return fail(TB_ERR_SHAPE_MISMATCH, "%s: negative dimension", name);
    if (tr && t_batch != d->n && t_batch != 1)
        return fail(TB_ERR_SHAPE_MISMATCH, "MATMUL_T: b batch %d is neither n=%d nor 1", t_batch, d->n);
    const int at = d->a_dtype, bt = d->b_dtype, ot = d->out_dtype;
    const bool int8 = at == TB_DT_INT8 && bt == TB_DT_INT8 && ot == TB_DT_INT32;
    const bool int16 = at == TB_DT_INT16 && bt == TB_DT_INT16 && ot == TB_DT_INT48;
    const bool fp8a = at == TB_DT_FP8E4M3 || at == TB_DT_FP8E5M2, fp8b = bt == TB_DT_FP8E4M3 || bt == TB_DT_FP8E5M2;
    bool fl;
    if (!tr) {
        // matmul_types (src/ops/matmul.rs:30-38):
        // (F16, F16, F16|F32), (BF16, BF16, F32), (F32, F32, F32), (FP8, FP8, F16|F32)
        fl = (at == TB_DT_FP16 && bt == TB_DT_FP16 && (ot == TB_DT_FP16 || ot == TB_DT_FP32)) ||
             (at == TB_DT_BF16 && bt == TB_DT_BF16 && ot == TB_DT_FP32) ||
             (at == TB_DT_FP32 && bt == TB_DT_FP32 && ot == TB_DT_FP32) ||
             (fp8a && fp8b && (ot == TB_DT_FP16 || ot == TB_DT_FP32));
    } else {
        // matmul_t_types (src/ops/matmul.rs:42-51): (F16, F16, F16); any FP8/F16/BF16/F32 pair
        // into F32; into BF16 without F32 operands and not (F16, F16)
        auto isf = [](int t) {
            return t == TB_DT_FP8E4M3 || t == TB_DT_FP8E5M2 || t == TB_DT_FP16 || t == TB_DT_BF16 || t == TB_DT_FP32;
        };
        fl = (at == TB_DT_FP16 && bt == TB_DT_FP16 && ot == TB_DT_FP16) || (ot == TB_DT_FP32 && isf(at) && isf(bt)) ||
             (ot == TB_DT_BF16 && isf(at) && isf(bt) && at != TB_DT_FP32 && bt != TB_DT_FP32 &&
              !(at == TB_DT_FP16 && bt == TB_DT_FP16));
    }
    if (!int8 && !int16 && !fl)
        return fail(TB_ERR_DTYPE_MISMATCH, "%s: unsupported types a=%d b=%d output=%d", name, at, bt, ot);
    if (int8 || int16) {
        if ((d->a_zp != 0 && at != TB_DT_INT8) || (d->b_zp != 0 && bt != TB_DT_INT8))
            return fail(TB_ERR_GRAPH, "%s: zero points must be zero for non-int8 inputs", name);
    } else if (d->a_zp != 0 || d->b_zp != 0) {
        return fail(TB_ERR_GRAPH, "%s: zero points must be zero for floating-point inputs", name);
    }
    if (has_rescale && !int8) return fail(TB_ERR_DTYPE_MISMATCH, "%s: RESCALE needs an int32 result", name);
    const int e = int8 ? 1 : 2;
    // TMA row strides: A's and B's rows are c elements long for MATMUL_T; B's are w long for MATMUL
    const bool tma_ok = (static_cast<long long>(d->c) * e) % 16 == 0 &&
                        (tr || (static_cast<long long>(d->w) * e) % 16 == 0) && d->c > 0 && d->w > 0 && d->h > 0 &&
                        d->n > 0;
    // tensor cores: int8 -> int32, and BF16/F16 pairs with an FP32 result; everything else runs
    // the direct kernels in the reference's accumulation order (path 2 int8, 3 float, 4 int16)
    const bool tc_float = at == bt && (at == TB_DT_BF16 || at == TB_DT_FP16) && ot == TB_DT_FP32;
    // int8 with A rows TMA-addressable but B rows not (e.g. 1000 classes): B is copied
    // into column-padded rows each run and the tensor cores take it (path 5)
    // (w % 4 == 0: the in-kernel column sums of B read 4-byte words of its rows)
    const bool pad_b = !tr && int8 && !tma_ok && d->c % 16 == 0 && d->c > 0 && d->h > 0 && d->n > 0 && d->w >= 16 &&
                       d->w % 4 == 0 && static_cast<long long>(d->h) * d->n >= 64;
    if (int16) *path = 4;
    else if (int8) *path = tma_ok ? 0 : (pad_b ? 5 : 2);
    else *path = tma_ok && tc_float ? 1 : 3;
    *bn = d->w <= 128 ? 128 : 256;
    return TB_OK;
}

}  // namespace tb

namespace {

tb_status matmul_plan_create(tb_context* ctx, const tb_matmul_desc* d, int t_batch, const tb_rescale_attr* rescale,
                             tb_matmul_plan** out) {
    if (!ctx || !d || !out) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    TB_CUDA(cudaSetDevice(ctx->device));
    int path = 0, bn = 256;
    TB_TRY(matmul_validate(d, rescale != nullptr, &path, &bn, t_batch));
    // Few tiles (a classifier over one batch of images): 128-wide tiles when even those fit one
    // wave of the SMs, so twice as many SMs stream the contraction
    if (bn == 256 && (path == 0 || path == 1 || path == 5) &&
        static_cast<long long>(d->n) * ((d->h + 127) / 128) * ((d->w + 127) / 128) <= ctx->num_sms)
        bn = 128;
    tb_matmul_plan* p = new tb_matmul_plan;
    p->ctx = ctx;
    p->d = *d;
    p->path = path;
    p->bn = bn;
    p->t_batch = t_batch;
    if (rescale) {
        tb_status s = make_rescale_plan(ctx, rescale, TB_DT_INT32, d->w, &p->rs);
        if (s != TB_OK) { delete p; return s; }
        if (d->a_dtype == TB_DT_INT8 && d->b_dtype == TB_DT_INT8) {
            // |sum (a - za)(b - zb)| <= c * (128 + |za|) * (128 + |zb|)
            const long long bound = static_cast<long long>(d->c) * (128 + std::abs(d->a_zp)) * (128 + std::abs(d->b_zp));
            s = make_small_range(*rescale, p->rs, bound, &p->sr);
            if (s != TB_OK) { free_rescale_plan(&p->rs); delete p; return s; }
        }
    }
    if (p->path == 5) {
        p->wp = (d->w + 15) / 16 * 16;
        cudaError_t ce = cudaMalloc(&p->d_bpad, static_cast<size_t>(d->n) * d->c * p->wp);
        if (ce != cudaSuccess) { free_rescale_plan(&p->rs); delete p; return fail(TB_ERR_CUDA, "B padding alloc failed"); }
    }
    if ((p->path == 0 || p->path == 5) && d->a_zp != 0) {
        // padded by one tile: the epilogue reads whole 16-column chunks without clamping
        const size_t cbatch = t_batch ? static_cast<size_t>(t_batch) : static_cast<size_t>(d->n);
        cudaError_t ce = cudaMalloc(&p->d_colterm, sizeof(int32_t) * (cbatch * d->w + 256));
        if (ce != cudaSuccess) { free_rescale_plan(&p->rs); delete p; return fail(TB_ERR_CUDA, "colterm alloc failed"); }
    }
    *out = p;
    return TB_OK;
}

}  // namespace

extern "C" TB_API tb_status tb_matmul_plan_create(tb_context* ctx, const tb_matmul_desc* d,
                                                  const tb_rescale_attr* rescale, tb_matmul_plan** out) {
    return matmul_plan_create(ctx, d, 0, rescale, out);
}

extern "C" TB_API tb_status tb_matmul_t_plan_create(tb_context* ctx, const tb_matmul_desc* d, int32_t b_batch,
                                                    const tb_rescale_attr* rescale, tb_matmul_plan** out) {
    if (b_batch <= 0) {
        if (out) *out = nullptr;
        return fail(TB_ERR_SHAPE_MISMATCH, "MATMUL_T: b batch %d is neither n nor 1", b_batch);
    }
    return matmul_plan_create(ctx, d, b_batch, rescale, out);
}

extern "C" TB_API tb_status tb_matmul_plan_run(tb_matmul_plan* p, const void* a, const void* b, void* out,
                                               void* stream_) {
    if (!p || !a || !b || !out) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    tb_context* ctx = p->ctx;
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    const tb_matmul_desc& d = p->d;
    const long long total = static_cast<long long>(d.n) * d.h * d.w;
    if (total == 0) return TB_OK;
    const void* b_tma = b;
    const bool b_prepared = p->b_const != nullptr && b == p->b_const;  // column terms / padded rows kept
    // another B overwrites the kept buffers below: the constant one must be prepared again
    if (!b_prepared) p->b_const = nullptr;
    if (p->path == 5 && aligned16(a)) {
        if (!b_prepared) {
            pad_weight_rows_i8<<<grid_for(ctx, static_cast<long long>(d.n) * d.c * p->wp), 256, 0, st>>>(
                d.n * d.c, d.w, p->wp, static_cast<const int8_t*>(b), p->d_bpad);
            TB_LAUNCHED(ctx);
        }
        b_tma = p->d_bpad;
    } else if (p->path >= 2 || !aligned16(a) || !aligned16(b)) {
        const int bt = p->t_batch != 0, bb = p->t_batch == 1;
        if (d.a_dtype == TB_DT_INT8) {
            matmul_direct_int<<<grid_for(ctx, total), 256, 0, st>>>(d.n, d.h, d.c, d.w, static_cast<const int8_t*>(a),
                                                                    static_cast<const int8_t*>(b), bt, bb, d.a_zp,
                                                                    d.b_zp, int_epi(p->rs), out, ctx->dev_err);
        } else if (d.a_dtype == TB_DT_INT16) {
            matmul_direct_i48<<<grid_for(ctx, total), 256, 0, st>>>(d.n, d.h, d.c, d.w, static_cast<const int16_t*>(a),
                                                                    static_cast<const int16_t*>(b), bt, bb,
                                                                    static_cast<int64_t*>(out));
        } else {
            matmul_direct_float<<<grid_for(ctx, total), 256, 0, st>>>(d.n, d.h, d.c, d.w, a, b, bt, bb, d.a_dtype,
                                                                      d.b_dtype, d.out_dtype, out);
        }
        TB_LAUNCHED(ctx);
        return TB_OK;
    }
    const int e = p->path == 1 ? 2 : 1;
    const int wt = p->path == 5 ? p->wp : d.w;  // B row length of the tensor map
    if (a != p->a_cached) {
        const uint64_t dims[3] = {static_cast<uint64_t>(d.c), static_cast<uint64_t>(d.h), static_cast<uint64_t>(d.n)};
        const uint64_t str[2] = {static_cast<uint64_t>(d.c) * e, static_cast<uint64_t>(d.c) * d.h * e};
        const uint32_t box[3] = {static_cast<uint32_t>(128 / e), 128, 1};
        TB_TRY(encode_tiled(&p->tmA, tmap_dtype(d.a_dtype), 3, a, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
        p->a_cached = a;
    }
    if (b_tma != p->b_cached && p->t_batch) {
        // MATMUL_T: B [t_batch][w][c], K-major rows of c elements
        const uint64_t dims[3] = {static_cast<uint64_t>(d.c), static_cast<uint64_t>(d.w),
                                  static_cast<uint64_t>(p->t_batch)};
        const uint64_t str[2] = {static_cast<uint64_t>(d.c) * e, static_cast<uint64_t>(d.c) * d.w * e};
        const uint32_t box[3] = {static_cast<uint32_t>(128 / e), static_cast<uint32_t>(p->bn), 1};
        TB_TRY(encode_tiled(&p->tmB, tmap_dtype(d.b_dtype), 3, b_tma, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
        p->b_cached = b_tma;
    } else if (b_tma != p->b_cached) {
        const uint64_t dims[3] = {static_cast<uint64_t>(wt), static_cast<uint64_t>(d.c), static_cast<uint64_t>(d.n)};
        const uint64_t str[2] = {static_cast<uint64_t>(wt) * e, static_cast<uint64_t>(wt) * d.c * e};
        const uint32_t box[3] = {static_cast<uint32_t>(128 / e), static_cast<uint32_t>(128 / e), 1};
        TB_TRY(encode_tiled(&p->tmB, tmap_dtype(d.b_dtype), 3, b_tma, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
        p->b_cached = b_tma;
    }
    GemmParams gp{};
    gp.M = d.h;
    gp.N = d.w;
    gp.K = d.c;
    gp.batch = d.n;
    gp.in_bf16 = d.a_dtype == TB_DT_BF16;
    gp.k_blocks = (d.c + (128 / e) - 1) / (128 / e);
    gp.out = out;
    gp.out_batch_stride = static_cast<long long>(d.h) * d.w;
    gp.ldo = d.w;
    gp.b_bcast = p->t_batch == 1;
    GemmEpilogue& ep = gp.epi;
    // the small-range epilogue takes its integer terms pre-multiplied by 2^k
    const uint32_t tmul = p->sr.ok ? static_cast<uint32_t>(p->sr.mul) : 1u;
    if (p->path == 0 && p->t_batch) {
        if (d.a_zp != 0) {
            // colterm = -a_zp * rowsum(B) + c * a_zp * b_zp per B row (x 2^k for the small-range
            // epilogue); computed by the kernel before the GEMM, which waits for it in its epilogue
            if (!b_prepared) {
                const long long rows = static_cast<long long>(p->t_batch) * d.w;
                const int32_t add = static_cast<int32_t>(static_cast<uint32_t>(d.c) * static_cast<uint32_t>(d.a_zp) *
                                                         static_cast<uint32_t>(d.b_zp) * tmul);
                colterm_rows_i8<<<static_cast<unsigned>(std::min<long long>((rows + 7) / 8, 4LL * ctx->num_sms)), 256, 0,
                                  st>>>(rows, d.c, static_cast<const int8_t*>(b),
                                        static_cast<int32_t>(static_cast<uint32_t>(-d.a_zp) * tmul), add, p->d_colterm);
                TB_LAUNCHED(ctx);
                ep.pdl_wait = 1;
            }
            ep.colterm = p->d_colterm;
            ep.colterm_bstride = p->t_batch == 1 ? 0 : d.w;
        }
        ep.row_zp_neg = static_cast<int32_t>(static_cast<uint32_t>(-d.b_zp) * tmul);
        if (p->rs.enabled) {
            ep.mode = EPI_RESCALE;
            ep.rs = rescale_args(p->rs);
            set_fast_epilogue(&ep, p->rs, p->sr);
            ep.out_dtype = p->rs.out_dtype;
        } else {
            ep.mode = EPI_I32;
            ep.out_dtype = TB_DT_INT32;
        }
        prepare_tma_out(&gp, p->bn, &p->tmO, &p->o_cached);
        return launch_i8_matmul_t(ctx, p->bn, epilogue_kind(ep), p->tmA, p->tmB, gp, st);
    }
    if (p->path == 0 || p->path == 5) {
        if (d.a_zp != 0 && b_prepared) {
            ep.colterm = p->d_colterm;
            ep.colterm_bstride = d.w;
        } else if (d.a_zp != 0) {
            // colterm = -a_zp * colsum(B) + c * a_zp * b_zp (x 2^k for the small-range epilogue), by a
            // kernel before the GEMM; the GEMM is a programmatic dependent launch and waits for the
            // column terms only in its epilogue, so its main loop overlaps the column sums
            const int32_t scale = static_cast<int32_t>(static_cast<uint32_t>(-d.a_zp) * tmul);
            const int32_t add = static_cast<int32_t>(static_cast<uint32_t>(d.c) * static_cast<uint32_t>(d.a_zp) *
                                                     static_cast<uint32_t>(d.b_zp) * tmul);
            if (p->path == 0)  // 16-byte B rows
                colterm_cols_i8<<<dim3((d.w + 63) / 64, d.n), kColtermThreads, 0, st>>>(
                    d.c, d.w, static_cast<const int8_t*>(b), scale, add, p->d_colterm);
            else
                colterm_const_i8<<<dim3((d.w + 31) / 32, d.n), dim3(32, 8), 0, st>>>(
                    d.c, d.w, static_cast<const int8_t*>(b), scale, add, p->d_colterm);
            TB_LAUNCHED(ctx);
            ep.pdl_wait = 1;
            ep.colterm = p->d_colterm;
            ep.colterm_bstride = d.w;
        }
        ep.row_zp_neg = static_cast<int32_t>(static_cast<uint32_t>(-d.b_zp) * tmul);
        if (p->rs.enabled) {
            ep.mode = EPI_RESCALE;
            ep.rs = rescale_args(p->rs);
            set_fast_epilogue(&ep, p->rs, p->sr);
            ep.out_dtype = p->rs.out_dtype;
        } else {
            ep.mode = EPI_I32;
            ep.out_dtype = TB_DT_INT32;
        }
        prepare_tma_out(&gp, p->bn, &p->tmO, &p->o_cached);
        return launch_i8_matmul(ctx, p->bn, epilogue_kind(ep), p->tmA, p->tmB, gp, st);
    }
    ep.mode = EPI_F32;
    ep.out_dtype = TB_DT_FP32;
    if (p->t_batch) return launch_f16_matmul_t(ctx, p->bn, p->tmA, p->tmB, gp, st);
    return launch_f16_matmul(ctx, p->bn, p->tmA, p->tmB, gp, st);
}

extern "C" TB_API tb_status tb_matmul_plan_set_constant_b(tb_matmul_plan* p, const void* b, void* stream_) {
    if (!p || !b) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    tb_context* ctx = p->ctx;
    const tb_matmul_desc& d = p->d;
    p->b_const = nullptr;
    if (!(p->path == 0 || p->path == 5) || (p->path == 0 && d.a_zp == 0)) return TB_OK;
    TB_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    if (static_cast<long long>(d.n) * d.c * d.w == 0) return TB_OK;
    if (p->path == 5 && !p->t_batch) {
        pad_weight_rows_i8<<<grid_for(ctx, static_cast<long long>(d.n) * d.c * p->wp), 256, 0, st>>>(
            d.n * d.c, d.w, p->wp, static_cast<const int8_t*>(b), p->d_bpad);
        TB_LAUNCHED(ctx);
    }
    if (d.a_zp != 0 && p->t_batch) {
        // runs with an unaligned B take the direct kernel, which keeps nothing per B
        if (!aligned16(b)) return TB_OK;
        const uint32_t tmul = p->sr.ok ? static_cast<uint32_t>(p->sr.mul) : 1u;
        const long long rows = static_cast<long long>(p->t_batch) * d.w;
        const int32_t add = static_cast<int32_t>(static_cast<uint32_t>(d.c) * static_cast<uint32_t>(d.a_zp) *
                                                 static_cast<uint32_t>(d.b_zp) * tmul);
        colterm_rows_i8<<<static_cast<unsigned>(std::min<long long>((rows + 7) / 8, 4LL * ctx->num_sms)), 256, 0, st>>>(
            rows, d.c, static_cast<const int8_t*>(b), static_cast<int32_t>(static_cast<uint32_t>(-d.a_zp) * tmul), add,
            p->d_colterm);
        TB_LAUNCHED(ctx);
    } else if (d.a_zp != 0) {
        // colterm = -a_zp * colsum(B) + c * a_zp * b_zp (the in-GEMM column-sum job's values)
        const uint32_t tmul = p->sr.ok ? static_cast<uint32_t>(p->sr.mul) : 1u;  // small-range epilogue: x 2^k
        const int32_t add = static_cast<int32_t>(static_cast<uint32_t>(d.c) * static_cast<uint32_t>(d.a_zp) *
                                                 static_cast<uint32_t>(d.b_zp) * tmul);
        colterm_const_i8<<<dim3((d.w + 31) / 32, d.n), dim3(32, 8), 0, st>>>(
            d.c, d.w, static_cast<const int8_t*>(b), static_cast<int32_t>(static_cast<uint32_t>(-d.a_zp) * tmul), add,
            p->d_colterm);
        TB_LAUNCHED(ctx);
    }
    TB_CUDA(cudaStreamSynchronize(st));
    p->b_const = b;
    return TB_OK;
}

extern "C" TB_API void tb_matmul_plan_destroy(tb_matmul_plan* p) {
    if (!p) return;
    free_rescale_plan(&p->rs);
    free_small_range(&p->sr);
    if (p->d_colterm) cudaFree(p->d_colterm);
    if (p->d_bpad) cudaFree(p->d_bpad);
    delete p;
}

extern "C" TB_API tb_status tb_matmul_t(tb_context* ctx, const tb_matmul_desc* d, int32_t b_batch,
                                        const tb_rescale_attr* rescale, const void* a, const void* b, void* out,
                                        void* stream) {
    tb_matmul_plan* p = nullptr;
    TB_TRY(tb_matmul_t_plan_create(ctx, d, b_batch, rescale, &p));
    tb_status s = tb_matmul_plan_run(p, a, b, out, stream);
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    tb_matmul_plan_destroy(p);
    return s;
}

extern "C" TB_API tb_status tb_matmul(tb_context* ctx, const tb_matmul_desc* d, const tb_rescale_attr* rescale,
                                      const void* a, const void* b, void* out, void* stream) {
    tb_matmul_plan* p = nullptr;
    TB_TRY(tb_matmul_plan_create(ctx, d, rescale, &p));
    tb_status s = tb_matmul_plan_run(p, a, b, out, stream);
    // The plan's device buffers may still be read by queued kernels.
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    tb_matmul_plan_destroy(p);
    return s;
}

// ===========================================================================
// CONV2D / DEPTHWISE_CONV2D
// ===========================================================================

struct tb_conv2d_plan {
    tb_context* ctx = nullptr;
    tb_conv2d_desc d{};
    bool depthwise = false;
    int oh = 0, ow = 0;
    int path = 0;  // 0 TC int8, 1 TC f16/bf16, 2 direct int, 3 direct float, 4 dw int vec4, 5 dw int, 6 dw float,
                   // 7 direct INT16 x INT8 -> INT48 (conv or depthwise), 8 im2col rows + 1x1 TC int8,
                   // 9 dw int8 on dp2a (depthwise_i8_dp2a)
    const void* weight = nullptr;
    const void* bias = nullptr;
    RescalePlan rs;
    SmallRange sr;                  // tensor-core int8 path: small-range RESCALE constants
    int bn = 64, bk = 128;
    bool tap2 = false;              // int8 tensor-core path: two filter taps per stage (64 input channels)
    int32_t* d_colterm = nullptr;   // [n_classes][ct_ld] column terms of each border class
    int32_t* d_ctdelta = nullptr;   // [n_classes][ct_ld] class terms minus the base class's
    long long ct_ld = 0;            // output channels padded to whole 256-column tiles
    int base_class = 0;             // the interior class (all taps valid) when there is one
    uint8_t* d_rowclass = nullptr;
    uint8_t* d_colclass = nullptr;
    int n_cx = 1;
    int n_classes = 1;              // border classes (1: every output pixel sees every tap, e.g. a 1x1)
    const void* in_cached = nullptr;
    const void* o_cached = nullptr;  // output the TMA-store map tmO was made for
    CUtensorMap tmA, tmB, tmO;
    float* d_fbias = nullptr;  // float bias widened to f32
    // path 8: im2col rows + a 1x1 tensor-core convolution over them
    tb_conv2d_plan* inner = nullptr;
    tb_conv3d_desc d3{};            // path 11 (CONV3D, direct kernels): the 3-D descriptor
    int od = 0;                     // path 11: output depth
    bool transpose = false;         // TRANSPOSE_CONV2D: d.pad holds out_pad; path 10 runs `inner` (stride 1,
                                    // int8) over the tap-reversed weights in d_wpad, else a direct kernel
    int8_t* d_rows = nullptr;       // [n*oh*ow][kp]
    int8_t* d_wpad = nullptr;       // [oc][kp]
    int kp = 0;
    int segp = 0;                   // path 8: bytes per filter-row segment of a row (KW * IC rounded up to words)
    // path 9 (depthwise int8 on dp2a): [taps][ic] masked weight words, then bias2 [ic]
    uint32_t* d_dw = nullptr;
    int strip_rows = 0;             // output rows per block of the 3x3 strip kernel (0: chosen per launch)
    int dw_k = 0;                   // path 9: the table's weights and bias pre-scaled by 2^dw_k (small-range RESCALE in sr)
};

// Path 9 tables (depthwise_i8_dp2a): the masked 16-bit weight words and the bias with the
// input zero point's terms taken out, from the weight and bias contents at plan creation.
// Leaves the plan on path 4 when the input zero point does not fit a signed byte.
static tb_status prepare_dw_dp2a(tb_conv2d_plan* p, const tb_rescale_attr* rescale) {
    const tb_conv2d_desc& d = p->d;
    const int c = d.ic;
    const long long taps = static_cast<long long>(d.kh) * d.kw;
    if (d.input_zp < -128 || d.input_zp > 127) return TB_OK;
    std::vector<int8_t> w(static_cast<size_t>(taps * c));
    std::vector<int32_t> bias(static_cast<size_t>(d.bias_len));
    TB_CUDA(cudaMemcpy(w.data(), p->weight, w.size(), cudaMemcpyDeviceToHost));
    TB_CUDA(cudaMemcpy(bias.data(), p->bias, sizeof(int32_t) * bias.size(), cudaMemcpyDeviceToHost));
    std::vector<long long> wsum(c, 0), wabs(c, 0);
    int wmax = 1;
    for (long long t = 0; t < taps; ++t)
        for (int ch = 0; ch < c; ++ch) {
            const int wv = w[static_cast<size_t>(t * c + ch)] - d.weight_zp;
            if (wv < -32768 || wv > 32767) return TB_OK;
            wsum[ch] += wv;
            wabs[ch] += std::abs(wv);
            wmax = std::max(wmax, std::abs(wv));
        }
    // The 3x3 strip kernel's small-range RESCALE: weights and bias pre-scaled by 2^k, so the
    // accumulator is v * 2^k and the epilogue is one mad.hi and a shift (as in the GEMM). k is
    // bounded by the 16-bit weight lanes (|w - zw| * 2^k <= 32767) and by |v| * 2^k < 2^31 over
    // |v| <= (128 + |zx|) * sum |w - zw| + |bias| (the host bound; the substituted zero-point
    // taps are inside it).
    const bool strip = d.kh == 3 && d.kw == 3 && d.stride[0] == d.stride[1] && d.stride[0] <= 2 &&
                       d.dilation[0] == 1 && d.dilation[1] == 1;
    int k = 0;
    if (strip && rescale != nullptr && p->rs.fast && p->rs.out_dtype == TB_DT_INT8) {
        int kcap = 0;
        while (kcap < 15 && (static_cast<long long>(wmax) << (kcap + 1)) <= 32767) ++kcap;
        long long bound = 0;
        for (int ch = 0; ch < c; ++ch)
            bound = std::max(bound, (128ll + std::abs(d.input_zp)) * wabs[ch] +
                                        std::llabs(static_cast<long long>(bias[d.bias_len == 1 ? 0 : ch])));
        // a bound of at least 2^(30 - kcap) keeps prepare_small_range's k at or below kcap
        bound = std::max(bound, 1ll << (30 - kcap));
        tb_status s = make_small_range(*rescale, p->rs, bound, &p->sr);
        if (s != TB_OK) return s;
        if (p->sr.ok && p->sr.k >= 1) k = p->sr.k;
        else free_small_range(&p->sr);
    }
    p->dw_k = k;
    std::vector<uint32_t> blob(static_cast<size_t>(taps * c + c), 0);
    for (long long t = 0; t < taps; ++t)
        for (int ch = 0; ch < c; ++ch) {
            const int wv = (w[static_cast<size_t>(t * c + ch)] - d.weight_zp) * (1 << k);
            blob[static_cast<size_t>(t * c + ch)] = static_cast<uint32_t>(static_cast<uint16_t>(wv)) << (16 * (ch & 1));
        }
    for (int ch = 0; ch < c; ++ch) {
        const long long b = bias[d.bias_len == 1 ? 0 : ch];
        blob[static_cast<size_t>(taps * c + ch)] = static_cast<uint32_t>(
            static_cast<unsigned long long>(b - static_cast<long long>(d.input_zp) * wsum[ch]) << k);
    }
    TB_CUDA(cudaMalloc(&p->d_dw, sizeof(uint32_t) * blob.size()));
    TB_CUDA(cudaMemcpy(p->d_dw, blob.data(), sizeof(uint32_t) * blob.size(), cudaMemcpyHostToDevice));
    // strip height override (tests use it to run several rows per block on small shapes)
    if (const char* ev = std::getenv("TB_DEPTHWISE_STRIP_ROWS")) p->strip_rows = std::max(0, std::atoi(ev));
    p->path = 9;
    return TB_OK;
}

template <int K, int SW>
static void launch_dw_dp2a(int ek, dim3 grid, dim3 block, cudaStream_t st, const DwGeom& g, const uint32_t* x,
                           const uint4* wm, const int32_t* b2, uint32_t zxw, const DwEpi& e, void* out,
                           uint32_t* err) {
    if (ek == 2) depthwise_i8_dp2a<K, SW, 2><<<grid, block, 0, st>>>(g, x, wm, b2, zxw, e, out, err);
    else if (ek == 1) depthwise_i8_dp2a<K, SW, 1><<<grid, block, 0, st>>>(g, x, wm, b2, zxw, e, out, err);
    else depthwise_i8_dp2a<K, SW, 0><<<grid, block, 0, st>>>(g, x, wm, b2, zxw, e, out, err);
}

static tb_status conv_extent(const char* op, int in, int pb, int pa, int k, int dil, int stride, int* out) {
    // src/ops/conv.rs:54-75
    const long long full = static_cast<long long>(in) - 1 + pb + pa - static_cast<long long>(k - 1) * dil;
    if (full % stride != 0) return fail(TB_ERR_GRAPH, "%s: parameters must yield exact integer output dimensions", op);
    const long long o = full / stride + 1;
    if (o < 1) return fail(TB_ERR_GRAPH, "%s: output dimension %lld must be positive", op, o);
    *out = static_cast<int>(o);
    return TB_OK;
}

// Valid tap range [lo, hi] of output position o (possibly empty: lo > hi).
static void tap_range(int o, int stride, int pad, int dil, int k, int in, int* lo, int* hi) {
    int l = 0, h = k - 1;
    while (l <= h && o * stride + l * dil - pad < 0) ++l;
    while (h >= l && o * stride + h * dil - pad >= in) --h;
    *lo = l;
    *hi = h;
}

// The (input, weight, acc, output) combinations the reference admits:
// conv2d_types (src/ops/conv.rs:375-385) and standard_types (:388-396).
static bool conv_types_valid(bool depthwise, int i, int w, int a, int o) {
    auto fp8 = [](int t) { return t == TB_DT_FP8E4M3 || t == TB_DT_FP8E5M2; };
    if (i == TB_DT_INT8 && (w == TB_DT_INT8 || w == TB_DT_INT4) && a == TB_DT_INT32 && o == TB_DT_INT32) return true;
    if (i == TB_DT_INT16 && w == TB_DT_INT8 && a == TB_DT_INT48 && o == TB_DT_INT48) return true;
    if (!depthwise) {
        auto any = [&](int t) { return fp8(t) || t == TB_DT_FP16 || t == TB_DT_BF16 || t == TB_DT_FP32; };
        if (a == TB_DT_FP32 && o == TB_DT_FP32) return any(i) && any(w);
        if ((a == TB_DT_FP16 || a == TB_DT_FP32) && o == TB_DT_FP16)
            return (fp8(i) || i == TB_DT_FP16) && (fp8(w) || w == TB_DT_FP16);
        if ((a == TB_DT_BF16 || a == TB_DT_FP32) && o == TB_DT_BF16)
            return (fp8(i) || i == TB_DT_BF16) && (fp8(w) || w == TB_DT_BF16);
        return false;
    }
    if (i == TB_DT_FP16 && w == TB_DT_FP16 && (a == TB_DT_FP16 || a == TB_DT_FP32) && o == TB_DT_FP16) return true;
    if (i == TB_DT_BF16 && w == TB_DT_BF16 && a == TB_DT_FP32 && o == TB_DT_BF16) return true;
    if (i == TB_DT_FP32 && w == TB_DT_FP32 && a == TB_DT_FP32 && o == TB_DT_FP32) return true;
    if ((i == TB_DT_FP8E4M3 && w == TB_DT_FP8E4M3) || (i == TB_DT_FP8E5M2 && w == TB_DT_FP8E5M2))
        return (a == TB_DT_FP16 && o == TB_DT_FP16) || (a == TB_DT_FP32 && o == TB_DT_FP32);
    return false;
}

static tb_status conv_plan_create(tb_context* ctx, const tb_conv2d_desc* d, const void* weight, const void* bias,
                                  const tb_rescale_attr* rescale, bool depthwise, tb_conv2d_plan** out) {
    if (!ctx || !d || !out || !weight || !bias) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    TB_CUDA(cudaSetDevice(ctx->device));
    const char* op = depthwise ? "DEPTHWISE_CONV2D" : "CONV2D";
    // conv.rs:77-92 attribute checks
    for (int i = 0; i < 4; ++i)
        if (d->pad[i] < 0) return fail(TB_ERR_GRAPH, "%s: pad must be non-negative", op);
    for (int i = 0; i < 2; ++i) {
        if (d->stride[i] < 1) return fail(TB_ERR_GRAPH, "%s: stride must be at least 1", op);
        if (d->dilation[i] < 1) return fail(TB_ERR_GRAPH, "%s: dilation must be at least 1", op);
    }
    const int oc = depthwise ? d->ic * d->m : d->oc;
    if (depthwise && d->m < 1) return fail(TB_ERR_SHAPE_MISMATCH, "%s: channel multiplier must be positive", op);
    int oh = 0, ow = 0;
    TB_TRY(conv_extent(op, d->ih, d->pad[0], d->pad[1], d->kh, d->dilation[0], d->stride[0], &oh));
    TB_TRY(conv_extent(op, d->iw, d->pad[2], d->pad[3], d->kw, d->dilation[1], d->stride[1], &ow));
    if (d->bias_len != oc && d->bias_len != 1)
        return fail(TB_ERR_SHAPE_MISMATCH, "%s: bias channels %d must be 1 or match output channels %d", op,
                    d->bias_len, oc);
    const int it = d->in_dtype, wt = d->w_dtype, at = d->acc_dtype, ot = d->out_dtype;
    const bool int8 = it == TB_DT_INT8 && (wt == TB_DT_INT8 || wt == TB_DT_INT4) && at == TB_DT_INT32 &&
                      ot == TB_DT_INT32;
    const bool int16 = it == TB_DT_INT16 && wt == TB_DT_INT8 && at == TB_DT_INT48 && ot == TB_DT_INT48;
    // every type combination of the reference's tables runs: int8 and BF16/F16 pairs with
    // fp32 accumulation on tensor cores where the layout allows, the rest (fp8 operands,
    // mixed float types, f16/bf16 accumulators, INT16 x INT8 -> INT48) on the direct
    // kernels in the reference's accumulation order
    if (!conv_types_valid(depthwise, it, wt, at, ot))
        return fail(TB_ERR_DTYPE_MISMATCH, "%s: unsupported types input=%d weight=%d acc=%d output=%d", op, it, wt, at,
                    ot);
    const bool fl = !int8 && !int16;
    const bool tc_float = fl && it == wt && (it == TB_DT_FP16 || it == TB_DT_BF16) && at == TB_DT_FP32;
    if (int8 || int16) {
        if (d->input_zp != 0 && it != TB_DT_INT8)
            return fail(TB_ERR_GRAPH, "%s: input zero point must be zero for non-int8 input", op);
        if (d->weight_zp != 0 && wt != TB_DT_INT8)
            return fail(TB_ERR_GRAPH, "%s: weight zero point must be zero for non-int8 weight", op);
    } else if (d->input_zp != 0 || d->weight_zp != 0) {
        return fail(TB_ERR_GRAPH, "%s: zero points must be zero for floating-point operands", op);
    }
    if (rescale && !int8) return fail(TB_ERR_DTYPE_MISMATCH, "%s: RESCALE needs an int32 result", op);

    tb_conv2d_plan* p = new tb_conv2d_plan;
    p->ctx = ctx;
    p->d = *d;
    p->d.oc = oc;
    p->depthwise = depthwise;
    p->oh = oh;
    p->ow = ow;
    p->weight = weight;
    p->bias = bias;
    auto bail = [&](tb_status s) {
        tb_conv2d_plan_destroy(p);
        return s;
    };
    if (rescale) {
        tb_status s = make_rescale_plan(ctx, rescale, TB_DT_INT32, oc, &p->rs);
        if (s != TB_OK) return bail(s);
    }
    if (int16) {
        p->path = 7;
        *out = p;
        return TB_OK;
    }
    if (depthwise) {
        p->path = int8 ? ((d->m == 1 && d->ic % 4 == 0) ? 4 : 5) : 6;
        if (p->path == 4 && d->dilation[1] == 1 && (d->kw == 3 || d->kw == 5) && d->kh == d->kw &&
            (d->stride[1] == 1 || d->stride[1] == 2) && d->n <= 65535 && oh <= 65535) {
            tb_status s = prepare_dw_dp2a(p, rescale);
            if (s != TB_OK) return bail(s);
        }
        *out = p;
        return TB_OK;
    }
    const int e = int8 ? 1 : 2;
    const long long taps = static_cast<long long>(d->kh) * d->kw;
    const bool tma_ok = (static_cast<long long>(d->ic) * e) % 16 == 0 && d->n > 0 && oh > 0 && ow > 0 &&
                        d->pad[0] <= 127 && d->pad[2] <= 127 && d->kw * d->dilation[1] < 256 &&
                        d->kh * d->dilation[0] < 256 && (taps * d->ic * e) % 16 == 0 && oh <= 255 && ow <= 255 &&
                        aligned16(weight);
    p->path = tma_ok && (int8 || tc_float) ? (int8 ? 0 : 1) : (int8 ? 2 : 3);
    // Few input channels (an RGB stem): gather im2col rows once and run them as a 1x1
    // tensor-core convolution when the contraction is long enough to pay for the rows.
    const long long kfull = taps * d->ic;
    const long long m_rows = static_cast<long long>(d->n) * oh * ow;
    // rows of KH segments (one per filter row, KW * IC bytes padded to whole words)
    const int seg = d->kw * d->ic, segp = (seg + 3) / 4 * 4;
    const long long kpad = (static_cast<long long>(d->kh) * segp + 15) / 16 * 16;
    if (p->path == 2 && wt == TB_DT_INT8 && kfull >= 16 && m_rows >= 4096 && aligned16(weight) &&
        m_rows * kpad <= (4ll << 30) && kpad <= 384) {
        p->path = 8;
        p->kp = static_cast<int>(kpad);
        p->segp = segp;
        cudaError_t ce = cudaMalloc(&p->d_rows, static_cast<size_t>(m_rows) * p->kp);
        if (ce == cudaSuccess) ce = cudaMalloc(&p->d_wpad, static_cast<size_t>(oc) * p->kp);
        if (ce != cudaSuccess) return bail(fail(TB_ERR_CUDA, "im2col buffer allocation failed: %s", cudaGetErrorString(ce)));
        pad_weight_segments_i8<<<grid_for(ctx, static_cast<long long>(oc) * p->kp), 256>>>(
            oc, d->kh, seg, segp, p->kp, static_cast<const int8_t*>(weight), p->d_wpad);
        ce = cudaGetLastError();
        if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
        if (ce != cudaSuccess) return bail(fail(TB_ERR_CUDA, "weight padding failed: %s", cudaGetErrorString(ce)));
        ctx->launches++;
        tb_conv2d_desc in = *d;
        in.ih = oh;
        in.iw = ow;
        in.ic = p->kp;
        in.kh = in.kw = 1;
        for (int i = 0; i < 4; ++i) in.pad[i] = 0;
        in.stride[0] = in.stride[1] = in.dilation[0] = in.dilation[1] = 1;
        tb_status s2 = conv_plan_create(ctx, &in, p->d_wpad, bias, rescale, false, &p->inner);
        if (s2 != TB_OK) return bail(s2);
        if (p->inner->path != 0) return bail(fail(TB_ERR_NOT_ACCELERATED, "%s: im2col rows did not take the tensor cores", op));
        *out = p;
        return TB_OK;
    }
    if (p->path == 1) {
        // float bias widened once (the epilogue adds it in f32)
        cudaError_t ce = cudaMalloc(&p->d_fbias, sizeof(float) * d->bias_len);
        if (ce != cudaSuccess) return bail(fail(TB_ERR_CUDA, "bias alloc failed"));
    }
    if (p->path >= 2) { *out = p; return TB_OK; }

    p->bn = oc <= 64 ? 64 : oc <= 128 ? 128 : 256;
    {
        // Up to 512 output channels over many pixels (int8): 128-column tiles, which the three
        // epilogue groups take whole in turn, instead of 256-column tiles split 64 / 96 / 96
        // columns between them (ResNet-50's 64->256 and 128->512, MobileNetV2's 32->192 and
        // 64->384 layers at 64 images: 4-18 % faster; at 14x14 the 256-column form is faster)
        const long long m_tiles = (static_cast<long long>(d->n) * oh * ow + 127) / 128;
        const long long n128 = (oc + 127) / 128;
        if (int8 && p->bn == 256 && n128 <= 4 && m_tiles * n128 >= 4ll * ctx->num_sms) p->bn = 128;
    }
    {
        // Few tiles (small maps, few images): narrower tiles while their count stays within one
        // wave of the SMs, so more SMs share the contraction (a 7x7 map of 64 images has 25 row
        // tiles: 50 tiles of 256 output channels, 100 of 128)
        const long long m_tiles = (static_cast<long long>(d->n) * oh * ow + 127) / 128;
        auto tiles = [&](int bn) { return m_tiles * ((oc + bn - 1) / bn); };
        while (p->bn > 64 && tiles(p->bn / 2) <= ctx->num_sms) p->bn /= 2;
    }
    // TB_CONV_MAX_BN (read at plan creation) caps the tile width of the tensor-core convolutions
    if (const char* ev = std::getenv("TB_CONV_MAX_BN")) {
        const int cap = std::atoi(ev);
        if ((cap == 64 || cap == 128) && p->bn > cap) p->bn = cap;
    }
    // K block of one stage: the channel run of a tap, rounded up to 32, 64 or 128 bytes
    p->bk = (int8 && d->ic <= 32) ? 32 : (int8 && d->ic <= 64) ? 64 : 128;
    p->tap2 = p->path == 0 && int8 && d->ic == 64 && taps >= 2 && p->bn <= 128;
    const int bke = p->bk / e;
    // Weight tensor map: [OC][KH*KW*IC], K-major.
    {
        const uint64_t K = static_cast<uint64_t>(taps) * d->ic;
        const uint64_t dims[3] = {K, static_cast<uint64_t>(oc), 1};
        const uint64_t str[2] = {K * e, K * e * oc};
        // two taps per stage: one 128-byte box covers both taps' weights (adjacent in K)
        const uint32_t box[3] = {static_cast<uint32_t>(p->tap2 ? 2 * bke : bke), static_cast<uint32_t>(p->bn), 1};
        tb_status s = encode_tiled(&p->tmB, tmap_dtype(wt), 3, weight, dims, str, box,
                                   (p->bk == 128 || p->tap2) ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : p->bk == 64            ? CU_TENSOR_MAP_SWIZZLE_64B
                                                            : CU_TENSOR_MAP_SWIZZLE_32B);
        if (s != TB_OK) return bail(s);
    }
    if (p->path == 1) {
        // bias of the output type -> f32 table (exact)
        std::vector<float> fb(d->bias_len);
        std::vector<uint16_t> raw(d->bias_len);
        std::vector<float> raw32(d->bias_len);
        cudaError_t ce;
        if (ot == TB_DT_FP32) ce = cudaMemcpy(fb.data(), bias, sizeof(float) * d->bias_len, cudaMemcpyDeviceToHost);
        else {
            ce = cudaMemcpy(raw.data(), bias, sizeof(uint16_t) * d->bias_len, cudaMemcpyDeviceToHost);
            for (int i = 0; i < d->bias_len; ++i) {
                if (ot == TB_DT_BF16) {
                    uint32_t u = static_cast<uint32_t>(raw[i]) << 16;
                    memcpy(&fb[i], &u, 4);
                } else {
                    __half h;
                    memcpy(&h, &raw[i], 2);
                    fb[i] = __half2float(h);
                }
            }
        }
        if (ce == cudaSuccess) ce = cudaMemcpy(p->d_fbias, fb.data(), sizeof(float) * d->bias_len, cudaMemcpyHostToDevice);
        if (ce != cudaSuccess) return bail(fail(TB_ERR_CUDA, "bias upload failed"));
        *out = p;
        return TB_OK;
    }
    // Small-range RESCALE: |v| <= (128 + |zx|) * sum_k |w - zw| + |bias| per output channel.
    if (rescale && int8) {
        const size_t kk = static_cast<size_t>(taps) * d->ic;
        std::vector<int8_t> hw(static_cast<size_t>(oc) * kk);
        std::vector<int32_t> hb(d->bias_len);
        cudaError_t ce = cudaMemcpy(hw.data(), weight, hw.size(), cudaMemcpyDeviceToHost);
        if (ce == cudaSuccess) ce = cudaMemcpy(hb.data(), bias, sizeof(int32_t) * hb.size(), cudaMemcpyDeviceToHost);
        if (ce != cudaSuccess) return bail(fail(TB_ERR_CUDA, "weight read failed: %s", cudaGetErrorString(ce)));
        long long bound = 0;
        for (int o = 0; o < oc; ++o) {
            long long sw = 0;
            for (size_t k = 0; k < kk; ++k) sw += std::abs(static_cast<int>(hw[o * kk + k]) - d->weight_zp);
            const long long b = std::llabs(static_cast<long long>(hb[d->bias_len == 1 ? 0 : o]));
            bound = std::max(bound, (128ll + std::abs(d->input_zp)) * sw + b);
        }
        tb_status s2 = make_small_range(*rescale, p->rs, bound, &p->sr);
        if (s2 != TB_OK) return bail(s2);
    }
    // Integer: border classes and the per-class column terms.
    std::vector<int> ky_r, kx_r;
    std::vector<uint8_t> rowc(oh), colc(ow);
    auto classify = [](int n_out, int stride, int pad, int dil, int k, int in, std::vector<int>& ranges,
                       std::vector<uint8_t>& cls) {
        for (int o = 0; o < n_out; ++o) {
            int lo, hi;
            tap_range(o, stride, pad, dil, k, in, &lo, &hi);
            int found = -1;
            for (size_t c = 0; c < ranges.size() / 2; ++c)
                if (ranges[2 * c] == lo && ranges[2 * c + 1] == hi) { found = static_cast<int>(c); break; }
            if (found < 0) {
                found = static_cast<int>(ranges.size() / 2);
                ranges.push_back(lo);
                ranges.push_back(hi);
            }
            cls[o] = static_cast<uint8_t>(found);
        }
    };
    classify(oh, d->stride[0], d->pad[0], d->dilation[0], d->kh, d->ih, ky_r, rowc);
    classify(ow, d->stride[1], d->pad[2], d->dilation[1], d->kw, d->iw, kx_r, colc);
    const int n_ry = static_cast<int>(ky_r.size() / 2), n_rx = static_cast<int>(kx_r.size() / 2);
    if (n_ry > 255 || n_rx > 255) return bail(fail(TB_ERR_NOT_ACCELERATED, "%s: too many border classes", op));
    p->n_cx = n_rx;
    p->n_classes = n_ry * n_rx;
    int ry_full = 0, rx_full = 0;
    for (int c = 0; c < n_ry; ++c)
        if (ky_r[2 * c] == 0 && ky_r[2 * c + 1] == d->kh - 1) ry_full = c;
    for (int c = 0; c < n_rx; ++c)
        if (kx_r[2 * c] == 0 && kx_r[2 * c + 1] == d->kw - 1) rx_full = c;
    p->base_class = ry_full * n_rx + rx_full;
    p->ct_ld = (static_cast<long long>(oc) + 255) / 256 * 256;
    int32_t* d_wsum = nullptr;
    int* d_ranges = nullptr;
    const size_t tab = sizeof(int32_t) * static_cast<size_t>(n_ry) * n_rx * p->ct_ld;
    cudaError_t ce = cudaMalloc(&p->d_colterm, tab);
    if (ce == cudaSuccess) ce = cudaMalloc(&p->d_ctdelta, tab);
    if (ce == cudaSuccess) ce = cudaMalloc(&p->d_rowclass, oh);
    if (ce == cudaSuccess) ce = cudaMalloc(&p->d_colclass, ow);
    if (ce == cudaSuccess) ce = cudaMalloc(&d_wsum, sizeof(int32_t) * oc * taps);
    if (ce == cudaSuccess) ce = cudaMalloc(&d_ranges, sizeof(int) * (ky_r.size() + kx_r.size()));
    if (ce == cudaSuccess) ce = cudaMemcpy(p->d_rowclass, rowc.data(), oh, cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(p->d_colclass, colc.data(), ow, cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemcpy(d_ranges, ky_r.data(), sizeof(int) * ky_r.size(), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess)
        ce = cudaMemcpy(d_ranges + ky_r.size(), kx_r.data(), sizeof(int) * kx_r.size(), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        if (d_wsum) cudaFree(d_wsum);
        if (d_ranges) cudaFree(d_ranges);
        return bail(fail(TB_ERR_CUDA, "conv plan allocation failed: %s", cudaGetErrorString(ce)));
    }
    conv_weight_tap_sums<<<grid_for(ctx, oc * taps), 256>>>(oc, static_cast<int>(taps), d->ic,
                                                            static_cast<const int8_t*>(weight), d_wsum);
    conv_colterm<<<grid_for(ctx, static_cast<long long>(n_ry) * n_rx * p->ct_ld), 256>>>(
        oc, p->ct_ld, d->kh, d->kw, d->ic, n_ry, n_rx, p->base_class, d_ranges, d_ranges + ky_r.size(), d_wsum,
        static_cast<const int32_t*>(bias), d->bias_len, d->input_zp, d->weight_zp,
        p->sr.ok ? static_cast<uint32_t>(p->sr.mul) : 1u, p->d_colterm, p->d_ctdelta);
    ce = cudaDeviceSynchronize();
    cudaFree(d_wsum);
    cudaFree(d_ranges);
    ctx->launches += 2;
    if (ce != cudaSuccess) return bail(fail(TB_ERR_CUDA, "conv plan kernels failed: %s", cudaGetErrorString(ce)));
    *out = p;
    return TB_OK;
}

extern "C" TB_API tb_status tb_conv2d_plan_create(tb_context* ctx, const tb_conv2d_desc* d, const void* weight,
                                                  const void* bias, const tb_rescale_attr* rescale,
                                                  tb_conv2d_plan** out) {
    return conv_plan_create(ctx, d, weight, bias, rescale, false, out);
}

extern "C" TB_API tb_status tb_depthwise_conv2d_plan_create(tb_context* ctx, const tb_conv2d_desc* d,
                                                            const void* weight, const void* bias,
                                                            const tb_rescale_attr* rescale, tb_conv2d_plan** out) {
    return conv_plan_create(ctx, d, weight, bias, rescale, true, out);
}

extern "C" TB_API tb_status tb_transpose_conv2d_plan_create(tb_context* ctx, const tb_conv2d_desc* d,
                                                            const void* weight, const void* bias,
                                                            const tb_rescale_attr* rescale, tb_conv2d_plan** out) {
    if (!ctx || !d || !out || !weight || !bias) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    TB_CUDA(cudaSetDevice(ctx->device));
    const char* op = "TRANSPOSE_CONV2D";
    // Transpose::new (src/ops/conv.rs:286-329)
    if (d->stride[0] < 1 || d->stride[1] < 1) return fail(TB_ERR_GRAPH, "%s: stride must be at least 1", op);
    for (int i = 0; i < 4; ++i)
        if (d->pad[i] <= -(i < 2 ? d->kh : d->kw))
            return fail(TB_ERR_GRAPH, "%s: out_pad must be greater than -kernel size", op);
    const long long oh = (static_cast<long long>(d->ih) - 1) * d->stride[0] + d->pad[0] + d->pad[1] + d->kh;
    const long long ow = (static_cast<long long>(d->iw) - 1) * d->stride[1] + d->pad[2] + d->pad[3] + d->kw;
    if (oh < 1 || ow < 1) return fail(TB_ERR_GRAPH, "%s: output size %lldx%lld must be positive", op, oh, ow);
    if (oh > INT32_MAX || ow > INT32_MAX) return fail(TB_ERR_NOT_ACCELERATED, "%s: output above int32", op);
    if (d->bias_len != d->oc && d->bias_len != 1)
        return fail(TB_ERR_SHAPE_MISMATCH, "%s: bias channels %d must be 1 or match output channels %d", op,
                    d->bias_len, d->oc);
    // standard_types (conv.rs:388-396), the table conv_types_valid applies to depthwise
    const int it = d->in_dtype, wt = d->w_dtype, at = d->acc_dtype, ot = d->out_dtype;
    if (!conv_types_valid(true, it, wt, at, ot))
        return fail(TB_ERR_DTYPE_MISMATCH, "%s: unsupported types input=%d weight=%d acc=%d output=%d", op, it, wt, at,
                    ot);
    const bool int8 = it == TB_DT_INT8 && at == TB_DT_INT32;
    const bool int16 = it == TB_DT_INT16;
    if (int8 || int16) {
        if (d->input_zp != 0 && it != TB_DT_INT8)
            return fail(TB_ERR_GRAPH, "%s: input zero point must be zero for non-int8 input", op);
        if (d->weight_zp != 0 && wt != TB_DT_INT8)
            return fail(TB_ERR_GRAPH, "%s: weight zero point must be zero for non-int8 weight", op);
    } else if (d->input_zp != 0 || d->weight_zp != 0) {
        return fail(TB_ERR_GRAPH, "%s: zero points must be zero for floating-point operands", op);
    }
    if (rescale && !int8) return fail(TB_ERR_DTYPE_MISMATCH, "%s: RESCALE needs an int32 result", op);
    tb_conv2d_plan* p = new tb_conv2d_plan;
    p->ctx = ctx;
    p->d = *d;
    p->transpose = true;
    p->oh = static_cast<int>(oh);
    p->ow = static_cast<int>(ow);
    p->weight = weight;
    p->bias = bias;
    auto bail = [&](tb_status s) {
        tb_conv2d_plan_destroy(p);
        return s;
    };
    // (the CONV2D's padding k - 1 + out_pad stays inside the im2col corner range of its TMA path)
    const bool small_pad = d->pad[0] <= 100 && d->pad[1] <= 100 && d->pad[2] <= 100 && d->pad[3] <= 100 &&
                           d->kh <= 28 && d->kw <= 28;
    if (int8 && small_pad && d->stride[0] == 1 && d->stride[1] == 1) {
        // stride 1: out[oy] = sum_ky x[oy - out_pad_top - ky] w[ky] is the CONV2D with the taps
        // reversed and padding k - 1 + out_pad on each side (all >= 0: out_pad > -k)
        const size_t wbytes = static_cast<size_t>(d->oc) * d->kh * d->kw * d->ic;
        if (wbytes) {
            if (cudaMalloc(&p->d_wpad, wbytes) != cudaSuccess) return bail(fail(TB_ERR_CUDA, "%s: weight alloc failed", op));
            flip_taps_i8<<<grid_for(ctx, static_cast<long long>(wbytes)), 256>>>(
                d->oc, d->kh, d->kw, d->ic, static_cast<const int8_t*>(weight), p->d_wpad);
            TB_LAUNCHED(ctx);
            if (cudaStreamSynchronize(nullptr) != cudaSuccess) return bail(fail(TB_ERR_CUDA, "%s: weight flip failed", op));
        }
        tb_conv2d_desc cd = *d;
        cd.pad[0] = d->kh - 1 + d->pad[0];
        cd.pad[1] = d->kh - 1 + d->pad[1];
        cd.pad[2] = d->kw - 1 + d->pad[2];
        cd.pad[3] = d->kw - 1 + d->pad[3];
        cd.dilation[0] = cd.dilation[1] = 1;
        tb_status s = conv_plan_create(ctx, &cd, p->d_wpad ? static_cast<const void*>(p->d_wpad) : weight, bias,
                                       rescale, false, &p->inner);
        if (s != TB_OK) return bail(s);
        p->path = 10;
        *out = p;
        return TB_OK;
    }
    if (rescale) {
        tb_status s = make_rescale_plan(ctx, rescale, TB_DT_INT32, d->oc, &p->rs);
        if (s != TB_OK) return bail(s);
    }
    p->path = int16 ? 7 : int8 ? 2 : 3;  // direct kernels in the reference's gather order
    *out = p;
    return TB_OK;
}

extern "C" TB_API tb_status tb_conv2d_plan_run(tb_conv2d_plan* p, const void* input, void* out, void* stream_) {
    if (!p || !input || !out) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    tb_context* ctx = p->ctx;
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    const tb_conv2d_desc& d = p->d;
    if (p->path == 10) return tb_conv2d_plan_run(p->inner, input, out, stream_);
    if (p->path == 11) {
        const tb_conv3d_desc& e = p->d3;
        Conv3GeomDev g3{e.n, e.id, e.ih, e.iw, e.ic, e.oc, e.kd, e.kh, e.kw, p->od, p->oh, p->ow,
                        e.pad[0], e.pad[2], e.pad[4], e.stride[0], e.stride[1], e.stride[2],
                        e.dilation[0], e.dilation[1], e.dilation[2]};
        const long long total3 = static_cast<long long>(e.n) * p->od * p->oh * p->ow * e.oc;
        if (total3 == 0) return TB_OK;
        cudaStream_t st3 = static_cast<cudaStream_t>(stream_);
        if (e.in_dtype == TB_DT_INT8)
            conv3d_direct_int<<<grid_for(ctx, total3), 256, 0, st3>>>(
                g3, static_cast<const int8_t*>(input), static_cast<const int8_t*>(p->weight),
                static_cast<const int32_t*>(p->bias), e.bias_len, e.input_zp, e.weight_zp, int_epi(p->rs), out,
                ctx->dev_err);
        else if (e.in_dtype == TB_DT_INT16)
            conv3d_direct_i48<<<grid_for(ctx, total3), 256, 0, st3>>>(
                g3, static_cast<const int16_t*>(input), static_cast<const int8_t*>(p->weight),
                static_cast<const int64_t*>(p->bias), e.bias_len, e.input_zp, e.weight_zp, static_cast<int64_t*>(out));
        else
            conv3d_direct_float<<<grid_for(ctx, total3), 256, 0, st3>>>(g3, input, p->weight, p->bias, e.bias_len,
                                                                        e.in_dtype, e.w_dtype, e.acc_dtype,
                                                                        e.out_dtype, out);
        TB_LAUNCHED(ctx);
        return TB_OK;
    }
    ConvGeomDev g;
    g.tr = p->transpose ? 1 : 0;
    g.n = d.n; g.ih = d.ih; g.iw = d.iw; g.ic = d.ic; g.oc = d.oc; g.kh = d.kh; g.kw = d.kw;
    g.oh = p->oh; g.ow = p->ow; g.m = d.m;
    g.pad_t = d.pad[0]; g.pad_l = d.pad[2]; g.sh = d.stride[0]; g.sw = d.stride[1];
    g.dh = d.dilation[0]; g.dw = d.dilation[1];
    const long long total = static_cast<long long>(d.n) * p->oh * p->ow * d.oc;
    if (total == 0) return TB_OK;
    int path = p->path;
    if (path <= 1 && !aligned16(input)) path = path == 0 ? 2 : 3;
    // word loads and stores of the vectorised depthwise kernels
    if ((path == 4 || path == 9) && ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(out)) & 3u))
        path = 5;
    switch (path) {
    case 2:
        conv2d_direct_int<<<grid_for(ctx, total), 256, 0, st>>>(g, static_cast<const int8_t*>(input),
                                                                static_cast<const int8_t*>(p->weight),
                                                                static_cast<const int32_t*>(p->bias), d.bias_len,
                                                                d.input_zp, d.weight_zp, int_epi(p->rs), out,
                                                                ctx->dev_err);
        TB_LAUNCHED(ctx);
        return TB_OK;
    case 3:
        conv2d_direct_float<<<grid_for(ctx, total), 256, 0, st>>>(g, input, p->weight, p->bias, d.bias_len, d.in_dtype,
                                                                  d.w_dtype, d.acc_dtype, d.out_dtype, out);
        TB_LAUNCHED(ctx);
        return TB_OK;
    case 4:
        depthwise_int_vec4<<<grid_for(ctx, total / 4), 256, 0, st>>>(g, static_cast<const int8_t*>(input),
                                                                    static_cast<const int8_t*>(p->weight),
                                                                    static_cast<const int32_t*>(p->bias), d.bias_len,
                                                                    d.input_zp, d.weight_zp, int_epi(p->rs), out,
                                                                    ctx->dev_err);
        TB_LAUNCHED(ctx);
        return TB_OK;
    case 9: {
        DwGeom dg;
        dg.ih = d.ih; dg.iw = d.iw; dg.c4 = d.ic / 4; dg.oh = p->oh; dg.ow = p->ow; dg.kh = d.kh;
        dg.pad_t = d.pad[0]; dg.pad_l = d.pad[2]; dg.sh = d.stride[0]; dg.dh = d.dilation[0];
        dg.rows = 1;
        const int cx = std::min(dg.c4, 256);
        dg.chunks = (dg.c4 + cx - 1) / cx;
        const int groups = (p->ow + kDwPix - 1) / kDwPix;
        const int ng = std::min(std::max(1, 256 / cx), groups);
        const dim3 block(cx, ng);
        const dim3 grid(dg.chunks * ((groups + ng - 1) / ng), p->oh, d.n);
        DwEpi e{};
        e.gen = int_epi(p->rs);
        e.fq_m = p->rs.fq_m;
        e.fq_sh = p->rs.fq_sh;
        e.fq_hz = p->rs.fq_hz;
        e.per_channel = p->rs.per_channel;
        e.zp_add = p->rs.zp_folded ? 0 : p->rs.out_zp;
        e.lo = p->rs.lo;
        e.hi = p->rs.hi;
        int ek = (p->rs.enabled && p->rs.fast && p->rs.out_dtype == TB_DT_INT8)
                     ? (p->rs.rounding == ROUND_DOUBLE ? 2 : 1)
                     : 0;
        if (p->dw_k > 0) {  // pre-scaled table: the small-range RESCALE (3x3 strip kernel only)
            ek += 2;
            e.sr_sh = p->sr.d_sh;
            e.sr_c = p->sr.d_c;
            e.k2 = p->sr.k2;
            e.zp_add = p->sr.zp_folded ? 0 : p->rs.out_zp;
        }
        const uint32_t zxw = static_cast<uint32_t>(static_cast<uint8_t>(d.input_zp)) * 0x01010101u;
        auto x = static_cast<const uint32_t*>(input);
        auto wm = reinterpret_cast<const uint4*>(p->d_dw);
        const int32_t* b2 = reinterpret_cast<const int32_t*>(p->d_dw) + static_cast<long long>(d.kh) * d.kw * d.ic;
        if (d.kh == 3 && d.stride[0] == d.stride[1] && d.stride[0] <= 2 && d.dilation[0] == 1) {
            // strips of output rows: about four blocks per SM, at most 16 rows each (longer
            // strips load fewer rows twice; measured on B200, shorter ones were not faster)
            const long long row_blocks = static_cast<long long>(grid.x) * d.n;
            const long long want = 4ll * ctx->num_sms;
            long long rows = (static_cast<long long>(p->oh) * row_blocks) / std::max(want, 1ll);
            rows = std::max(1ll, std::min<long long>(rows, std::min(16, p->oh)));
            if (p->strip_rows > 0) rows = std::min(p->strip_rows, p->oh);
            dg.rows = static_cast<int>(rows);
            const dim3 sgrid(grid.x, (p->oh + dg.rows - 1) / dg.rows, d.n);
            auto x4 = x;
            if (d.stride[0] == 1) {
                if (ek == 4) depthwise_i8_dp2a_strip<1, 4><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else if (ek == 3) depthwise_i8_dp2a_strip<1, 3><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else if (ek == 2) depthwise_i8_dp2a_strip<1, 2><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else if (ek == 1) depthwise_i8_dp2a_strip<1, 1><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else depthwise_i8_dp2a_strip<1, 0><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
            } else {
                if (ek == 4) depthwise_i8_dp2a_strip<2, 4><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else if (ek == 3) depthwise_i8_dp2a_strip<2, 3><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else if (ek == 2) depthwise_i8_dp2a_strip<2, 2><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else if (ek == 1) depthwise_i8_dp2a_strip<2, 1><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
                else depthwise_i8_dp2a_strip<2, 0><<<sgrid, block, 0, st>>>(dg, x4, wm, b2, zxw, e, out, ctx->dev_err);
            }
            TB_LAUNCHED(ctx);
            return TB_OK;
        }
        if (ek >= 3) return fail(TB_ERR_INVALID_ARGUMENT, "DEPTHWISE_CONV2D: pre-scaled weights outside the 3x3 strip kernel");
        const int key = d.kw * 10 + d.stride[1];
        if (key == 31) launch_dw_dp2a<3, 1>(ek, grid, block, st, dg, x, wm, b2, zxw, e, out, ctx->dev_err);
        else if (key == 32) launch_dw_dp2a<3, 2>(ek, grid, block, st, dg, x, wm, b2, zxw, e, out, ctx->dev_err);
        else if (key == 51) launch_dw_dp2a<5, 1>(ek, grid, block, st, dg, x, wm, b2, zxw, e, out, ctx->dev_err);
        else launch_dw_dp2a<5, 2>(ek, grid, block, st, dg, x, wm, b2, zxw, e, out, ctx->dev_err);
        TB_LAUNCHED(ctx);
        return TB_OK;
    }
    case 5:
        depthwise_int_generic<<<grid_for(ctx, total), 256, 0, st>>>(g, static_cast<const int8_t*>(input),
                                                                   static_cast<const int8_t*>(p->weight),
                                                                   static_cast<const int32_t*>(p->bias), d.bias_len,
                                                                   d.input_zp, d.weight_zp, int_epi(p->rs), out,
                                                                   ctx->dev_err);
        TB_LAUNCHED(ctx);
        return TB_OK;
    case 6:
        depthwise_float<<<grid_for(ctx, total), 256, 0, st>>>(g, input, p->weight, p->bias, d.bias_len, d.in_dtype,
                                                              d.w_dtype, d.acc_dtype, d.out_dtype, out);
        TB_LAUNCHED(ctx);
        return TB_OK;
    case 8: {
        const long long m_rows = static_cast<long long>(d.n) * p->oh * p->ow;
        const int threads = 128;
        long long blocks = (m_rows + threads - 1) / threads;
        blocks = std::min<long long>(blocks, static_cast<long long>(ctx->num_sms) * 64);
        const size_t smem = static_cast<size_t>(threads) * p->kp;
        auto x = static_cast<const int8_t*>(input);
        const int8_t zx = static_cast<int8_t>(d.input_zp);
        const int bl = static_cast<int>(blocks);
        // unrolled taps for the common stem shapes (3 or 4 channels, square windows of 3, 5 or 7)
        const long long x_bytes = static_cast<long long>(d.n) * d.ih * d.iw * d.ic;
#define TB_IM2COL(IC_, KW_)                                                                               \
    else if (d.ic == IC_ && d.kw == KW_ && d.kh == KW_ && d.dilation[1] == 1 && p->kp == im2col_t_kp(IC_, KW_)) \
        im2col_rows_i8_t<IC_, KW_><<<bl, threads, smem, st>>>(g, x, x_bytes, zx, p->d_rows)
        if (d.kh == 1 && d.kw == 1 && d.ic % 4 == 0 && (reinterpret_cast<uintptr_t>(input) & 3) == 0) {
            // 1x1 (channel counts that are not 16-byte multiples): each row is the pixel's channels
            // padded with the input zero point, one 16-byte chunk per thread
            const long long chunks = m_rows * (p->kp / 16);
            const uint32_t zxw = 0x01010101u * static_cast<uint8_t>(zx);
            im2col_rows_1x1_i8<<<grid_for(ctx, chunks), 256, 0, st>>>(g, static_cast<const uint32_t*>(input), p->kp,
                                                                    zxw, reinterpret_cast<uint4*>(p->d_rows));
        }
        TB_IM2COL(3, 7); TB_IM2COL(3, 5); TB_IM2COL(3, 3); TB_IM2COL(4, 7); TB_IM2COL(4, 5); TB_IM2COL(4, 3);
        else im2col_rows_i8<<<bl, threads, smem, st>>>(g, x, p->segp, p->kp, zx, p->d_rows);
#undef TB_IM2COL
        TB_LAUNCHED(ctx);
        return tb_conv2d_plan_run(p->inner, p->d_rows, out, stream_);
    }
    case 7:
        conv2d_direct_i48<<<grid_for(ctx, total), 256, 0, st>>>(g, static_cast<const int16_t*>(input),
                                                                static_cast<const int8_t*>(p->weight),
                                                                static_cast<const int64_t*>(p->bias), d.bias_len,
                                                                d.input_zp, d.weight_zp, p->depthwise ? 1 : 0,
                                                                static_cast<int64_t*>(out));
        TB_LAUNCHED(ctx);
        return TB_OK;
    default: break;
    }
    const int e = path == 0 ? 1 : 2;
    const int bke = p->bk / e;
    if (input != p->in_cached) {
        const uint64_t dims[4] = {static_cast<uint64_t>(d.ic), static_cast<uint64_t>(d.iw), static_cast<uint64_t>(d.ih),
                                  static_cast<uint64_t>(d.n)};
        const uint64_t str[3] = {static_cast<uint64_t>(d.ic) * e, static_cast<uint64_t>(d.ic) * d.iw * e,
                                 static_cast<uint64_t>(d.ic) * d.iw * d.ih * e};
        const int lower[2] = {-d.pad[2], -d.pad[0]};
        const int upper[2] = {d.pad[3] - (d.kw - 1) * d.dilation[1], d.pad[1] - (d.kh - 1) * d.dilation[0]};
        const uint32_t es[4] = {1, static_cast<uint32_t>(d.stride[1]), static_cast<uint32_t>(d.stride[0]), 1};
        TB_TRY(encode_im2col(&p->tmA, tmap_dtype(d.in_dtype), input, dims, str, lower, upper,
                             static_cast<uint32_t>(bke), 128, es,
                             p->bk == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                             : p->bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                           : CU_TENSOR_MAP_SWIZZLE_32B));
        p->in_cached = input;
    }
    GemmParams gp{};
    gp.M = d.n * p->oh * p->ow;
    gp.N = d.oc;
    gp.K = d.kh * d.kw * d.ic;
    gp.batch = 1;
    gp.in_bf16 = d.in_dtype == TB_DT_BF16;
    gp.c_blocks = (d.ic + bke - 1) / bke;
    gp.taps = d.kh * d.kw;
    gp.k_blocks = p->tap2 ? (gp.taps + 1) / 2 : gp.taps * gp.c_blocks;
    gp.conv_OW = p->ow;
    gp.conv_OHOW = p->oh * p->ow;
    gp.stride_h = d.stride[0];
    gp.stride_w = d.stride[1];
    gp.pad_t = d.pad[0];
    gp.pad_l = d.pad[2];
    gp.KW = d.kw;
    gp.dil_h = d.dilation[0];
    gp.dil_w = d.dilation[1];
    gp.IC = d.ic;
    gp.out = out;
    gp.out_batch_stride = 0;
    gp.ldo = d.oc;
    GemmEpilogue& ep = gp.epi;
    if (path == 1) {
        ep.mode = EPI_FCONV;
        ep.out_dtype = d.out_dtype;
        ep.fbias = p->d_fbias;
        ep.fbias_len = d.bias_len;
        return launch_f16_conv(ctx, p->bn, p->tmA, p->tmB, gp, st);
    }
    ep.colterm = p->d_colterm + static_cast<long long>(p->base_class) * p->ct_ld;
    ep.colterm_bstride = 0;
    ep.ct_delta = p->d_ctdelta;
    ep.ct_ld = p->ct_ld;
    ep.base_class = p->base_class;
    // one border class (no padding reaches a window), or classes that differ only through the
    // input zero point when it is 0: the base column terms are the whole story, and the kernel
    // without border-class code runs
    // (with input zero point 0 every class has the same terms: bias + 0)
    const bool classes = p->n_classes > 1 && d.input_zp != 0;
    ep.rowclass = classes ? p->d_rowclass : nullptr;
    ep.colclass = classes ? p->d_colclass : nullptr;
    ep.n_col_classes = p->n_cx;
    ep.row_zp_neg = static_cast<int32_t>(static_cast<uint32_t>(-d.weight_zp) *
                                         (p->sr.ok ? static_cast<uint32_t>(p->sr.mul) : 1u));
    if (p->rs.enabled) {
        ep.mode = EPI_RESCALE;
        ep.rs = rescale_args(p->rs);
        set_fast_epilogue(&ep, p->rs, p->sr);
        ep.out_dtype = p->rs.out_dtype;
    } else {
        ep.mode = EPI_I32;
        ep.out_dtype = TB_DT_INT32;
    }
    prepare_tma_out(&gp, p->bn, &p->tmO, &p->o_cached);
    if (p->tap2) return launch_i8_conv_tap2(ctx, p->bn, epilogue_kind(ep), p->tmA, p->tmB, gp, st);
    return launch_i8_conv(ctx, p->bn, p->bk, epilogue_kind(ep), p->tmA, p->tmB, gp, st);
}

extern "C" TB_API void tb_conv2d_plan_destroy(tb_conv2d_plan* p) {
    if (!p) return;
    if (p->inner) tb_conv2d_plan_destroy(p->inner);
    if (p->d_rows) cudaFree(p->d_rows);
    if (p->d_wpad) cudaFree(p->d_wpad);
    free_rescale_plan(&p->rs);
    free_small_range(&p->sr);
    if (p->d_colterm) cudaFree(p->d_colterm);
    if (p->d_ctdelta) cudaFree(p->d_ctdelta);
    if (p->d_rowclass) cudaFree(p->d_rowclass);
    if (p->d_colclass) cudaFree(p->d_colclass);
    if (p->d_fbias) cudaFree(p->d_fbias);
    if (p->d_dw) cudaFree(p->d_dw);
    delete p;
}

extern "C" TB_API tb_status tb_conv3d_plan_create(tb_context* ctx, const tb_conv3d_desc* d, const void* weight,
                                                  const void* bias, const tb_rescale_attr* rescale,
                                                  tb_conv2d_plan** out) {
    if (!ctx || !d || !out || !weight || !bias) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    TB_CUDA(cudaSetDevice(ctx->device));
    const char* op = "CONV3D";
    // check_conv_attributes (src/ops/conv.rs:77-92), ConvNd::new (:107-139)
    for (int i = 0; i < 6; ++i)
        if (d->pad[i] < 0) return fail(TB_ERR_GRAPH, "%s: pad must be non-negative", op);
    for (int i = 0; i < 3; ++i) {
        if (d->stride[i] < 1) return fail(TB_ERR_GRAPH, "%s: stride must be at least 1", op);
        if (d->dilation[i] < 1) return fail(TB_ERR_GRAPH, "%s: dilation must be at least 1", op);
    }
    int od = 0, oh = 0, ow = 0;
    TB_TRY(conv_extent(op, d->id, d->pad[0], d->pad[1], d->kd, d->dilation[0], d->stride[0], &od));
    TB_TRY(conv_extent(op, d->ih, d->pad[2], d->pad[3], d->kh, d->dilation[1], d->stride[1], &oh));
    TB_TRY(conv_extent(op, d->iw, d->pad[4], d->pad[5], d->kw, d->dilation[2], d->stride[2], &ow));
    if (d->bias_len != d->oc && d->bias_len != 1)
        return fail(TB_ERR_SHAPE_MISMATCH, "%s: bias channels %d must be 1 or match output channels %d", op,
                    d->bias_len, d->oc);
    const int it = d->in_dtype, wt = d->w_dtype, at = d->acc_dtype, ot = d->out_dtype;
    if (!conv_types_valid(true, it, wt, at, ot))  // standard_types (conv.rs:388-396)
        return fail(TB_ERR_DTYPE_MISMATCH, "%s: unsupported types input=%d weight=%d acc=%d output=%d", op, it, wt, at,
                    ot);
    const bool integer = it == TB_DT_INT8 || it == TB_DT_INT16;
    if (integer) {
        if (d->input_zp != 0 && it != TB_DT_INT8)
            return fail(TB_ERR_GRAPH, "%s: input zero point must be zero for non-int8 input", op);
        if (d->weight_zp != 0 && wt != TB_DT_INT8)
            return fail(TB_ERR_GRAPH, "%s: weight zero point must be zero for non-int8 weight", op);
    } else if (d->input_zp != 0 || d->weight_zp != 0) {
        return fail(TB_ERR_GRAPH, "%s: zero points must be zero for floating-point operands", op);
    }
    if (rescale && it != TB_DT_INT8) return fail(TB_ERR_DTYPE_MISMATCH, "%s: RESCALE needs an int32 result", op);
    // one depth tap, no depth padding, depth stride 1: each output depth slice is the CONV2D of
    // its input slice, so the whole op is one CONV2D over n * id images (int8: exact on the
    // tensor cores)
    const long long n2 = static_cast<long long>(d->n) * d->id;
    if (it == TB_DT_INT8 && d->kd == 1 && d->pad[0] == 0 && d->pad[1] == 0 && d->stride[0] == 1 && n2 <= INT32_MAX) {
        tb_conv2d_desc cd{};
        cd.n = static_cast<int32_t>(n2);
        cd.ih = d->ih;
        cd.iw = d->iw;
        cd.ic = d->ic;
        cd.oc = d->oc;
        cd.kh = d->kh;
        cd.kw = d->kw;
        cd.m = 1;
        for (int i = 0; i < 4; ++i) cd.pad[i] = d->pad[2 + i];
        for (int i = 0; i < 2; ++i) {
            cd.stride[i] = d->stride[1 + i];
            cd.dilation[i] = d->dilation[1 + i];
        }
        cd.in_dtype = it;
        cd.w_dtype = wt;
        cd.acc_dtype = at;
        cd.out_dtype = ot;
        cd.input_zp = d->input_zp;
        cd.weight_zp = d->weight_zp;
        cd.bias_len = d->bias_len;
        tb_conv2d_plan* p = new tb_conv2d_plan;
        p->ctx = ctx;
        p->d3 = *d;
        p->d.oc = d->oc;
        p->od = od;
        p->oh = oh;
        p->ow = ow;
        p->path = 10;
        tb_status s = conv_plan_create(ctx, &cd, weight, bias, rescale, false, &p->inner);
        if (s != TB_OK) {
            tb_conv2d_plan_destroy(p);
            return s;
        }
        *out = p;
        return TB_OK;
    }
    tb_conv2d_plan* p = new tb_conv2d_plan;
    p->ctx = ctx;
    p->d3 = *d;
    p->d.oc = d->oc;
    p->od = od;
    p->oh = oh;
    p->ow = ow;
    p->weight = weight;
    p->bias = bias;
    p->path = 11;
    if (rescale) {
        tb_status s = make_rescale_plan(ctx, rescale, TB_DT_INT32, d->oc, &p->rs);
        if (s != TB_OK) {
            tb_conv2d_plan_destroy(p);
            return s;
        }
    }
    *out = p;
    return TB_OK;
}

extern "C" TB_API tb_status tb_conv3d(tb_context* ctx, const tb_conv3d_desc* d, const tb_rescale_attr* rescale,
                                     const void* input, const void* weight, const void* bias, void* out,
                                     void* stream) {
    tb_conv2d_plan* p = nullptr;
    TB_TRY(tb_conv3d_plan_create(ctx, d, weight, bias, rescale, &p));
    tb_status s = tb_conv2d_plan_run(p, input, out, stream);
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    tb_conv2d_plan_destroy(p);
    return s;
}

extern "C" TB_API tb_status tb_transpose_conv2d(tb_context* ctx, const tb_conv2d_desc* d,
                                                const tb_rescale_attr* rescale, const void* input, const void* weight,
                                                const void* bias, void* out, void* stream) {
    tb_conv2d_plan* p = nullptr;
    TB_TRY(tb_transpose_conv2d_plan_create(ctx, d, weight, bias, rescale, &p));
    tb_status s = tb_conv2d_plan_run(p, input, out, stream);
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    tb_conv2d_plan_destroy(p);
    return s;
}

extern "C" TB_API tb_status tb_conv2d(tb_context* ctx, const tb_conv2d_desc* d, const tb_rescale_attr* rescale,
                                      const void* input, const void* weight, const void* bias, void* out,
                                      void* stream) {
    tb_conv2d_plan* p = nullptr;
    TB_TRY(tb_conv2d_plan_create(ctx, d, weight, bias, rescale, &p));
    tb_status s = tb_conv2d_plan_run(p, input, out, stream);
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    tb_conv2d_plan_destroy(p);
    return s;
}

extern "C" TB_API tb_status tb_depthwise_conv2d(tb_context* ctx, const tb_conv2d_desc* d,
                                                const tb_rescale_attr* rescale, const void* input,
                                                const void* weight, const void* bias, void* out, void* stream) {
    tb_conv2d_plan* p = nullptr;
    TB_TRY(tb_depthwise_conv2d_plan_create(ctx, d, weight, bias, rescale, &p));
    tb_status s = tb_conv2d_plan_run(p, input, out, stream);
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    tb_conv2d_plan_destroy(p);
    return s;
}

// ===========================================================================
// Elementwise and pooling
// ===========================================================================

extern "C" TB_API tb_status tb_rescale(tb_context* ctx, const tb_rescale_attr* attr, int32_t in_dtype,
                                       const void* input, int64_t count, void* out, void* stream_) {
    if (!ctx || !attr || (count > 0 && (!input || !out))) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    TB_CUDA(cudaSetDevice(ctx->device));
    RescalePlan r;
    int64_t izp = 0, ozp = 0;
    int32_t lo, hi;
    TB_TRY(check_rescale(attr, in_dtype, attr->channels, &izp, &ozp, &lo, &hi));
    TB_TRY(make_rescale_plan(ctx, attr, in_dtype, attr->channels, &r));
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    if (count > 0) {
        rescale_elementwise<<<grid_for(ctx, count), 256, 0, st>>>(input, in_dtype, attr->input_unsigned,
                                                                  static_cast<int32_t>(izp), count, attr->channels,
                                                                  rescale_args(r), attr->out_dtype, out, ctx->dev_err);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) { free_rescale_plan(&r); return fail(TB_ERR_CUDA, "rescale launch: %s", cudaGetErrorString(e)); }
        ctx->launches++;
    }
    cudaStreamSynchronize(st);
    free_rescale_plan(&r);
    return TB_OK;
}

extern "C" TB_API tb_status tb_clamp(tb_context* ctx, int32_t dtype, const void* input, int64_t count, int64_t min_i,
                                     int64_t max_i, float min_f, float max_f, int32_t nan_mode, void* out,
                                     void* stream_) {
    if (!ctx || (count > 0 && (!input || !out))) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    if (nan_mode != TB_NAN_PROPAGATE && nan_mode != TB_NAN_IGNORE)
        return fail(TB_ERR_GRAPH, "CLAMP: nan_mode must be PROPAGATE or IGNORE");
    if (dtype == TB_DT_INT8 || dtype == TB_DT_INT16) {
        if (max_i < min_i) return fail(TB_ERR_GRAPH, "CLAMP: max_val must not be smaller than min_val");
        if (count == 0) return TB_OK;
        clamp_int<<<grid_for(ctx, count), 256, 0, st>>>(input, dtype, count, static_cast<int32_t>(min_i),
                                                       static_cast<int32_t>(max_i), out);
    } else if (dtype == TB_DT_FP16 || dtype == TB_DT_BF16 || dtype == TB_DT_FP32) {
        if (min_f != min_f || max_f != max_f || max_f < min_f)
            return fail(TB_ERR_GRAPH, "CLAMP: min_val/max_val must be ordered and not NaN");
        if (count == 0) return TB_OK;
        clamp_float<<<grid_for(ctx, count), 256, 0, st>>>(input, dtype, count, min_f, max_f, nan_mode, out);
    } else {
        return fail(TB_ERR_DTYPE_MISMATCH, "CLAMP: unsupported dtype %d", dtype);
    }
    TB_LAUNCHED(ctx);
    return TB_OK;
}

extern "C" TB_API tb_status tb_add(tb_context* ctx, int32_t dtype, const void* a, const void* b, int64_t count,
                                   void* out, void* stream_) {
    if (!ctx || (count > 0 && (!a || !b || !out))) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    if (!(dtype == TB_DT_INT32 || dtype == TB_DT_FP32 || dtype == TB_DT_FP16 || dtype == TB_DT_BF16))
        return fail(TB_ERR_NOT_ACCELERATED, "ADD dtype %d is not accelerated", dtype);
    if (count == 0) return TB_OK;
    add_elementwise<<<grid_for(ctx, count), 256, 0, static_cast<cudaStream_t>(stream_)>>>(a, b, dtype, count, out);
    TB_LAUNCHED(ctx);
    return TB_OK;
}

static tb_status pool_geom(const char* op, const tb_pool2d_desc* d, PoolGeomDev* g) {
    // src/ops/pool.rs:31-70
    for (int i = 0; i < 4; ++i)
        if (d->pad[i] < 0) return fail(TB_ERR_GRAPH, "%s: pad must be non-negative", op);
    for (int i = 0; i < 2; ++i)
        if (d->kernel[i] < 1 || d->stride[i] < 1) return fail(TB_ERR_GRAPH, "%s: kernel and stride must be at least 1", op);
    if (d->pad[0] >= d->kernel[0] || d->pad[1] >= d->kernel[0] || d->pad[2] >= d->kernel[1] || d->pad[3] >= d->kernel[1])
        return fail(TB_ERR_GRAPH, "%s: pad must be smaller than kernel", op);
    if (d->ih == 0 || d->iw == 0) return fail(TB_ERR_GRAPH, "%s: input height and width must be positive", op);
    auto extent = [&](int size, int a, int b, int k, int s, int* o) -> tb_status {
        const long long full = static_cast<long long>(size) + a + b - k;
        if (full < 0 || full % s != 0) return fail(TB_ERR_GRAPH, "%s: parameters must yield exact integer output dimensions", op);
        *o = static_cast<int>(full / s + 1);
        return TB_OK;
    };
    g->n = d->n; g->ih = d->ih; g->iw = d->iw; g->c = d->c;
    TB_TRY(extent(d->ih, d->pad[0], d->pad[1], d->kernel[0], d->stride[0], &g->oh));
    TB_TRY(extent(d->iw, d->pad[2], d->pad[3], d->kernel[1], d->stride[1], &g->ow));
    g->ky = d->kernel[0]; g->kx = d->kernel[1]; g->sy = d->stride[0]; g->sx = d->stride[1];
    g->pad_t = d->pad[0]; g->pad_l = d->pad[2];
    return TB_OK;
}

namespace tb {
tb_status pool_check(const char* op, const tb_pool2d_desc* d, int* oh, int* ow) {
    PoolGeomDev g;
    TB_TRY(pool_geom(op, d, &g));
    *oh = g.oh;
    *ow = g.ow;
    return TB_OK;
}
}  // namespace tb

extern "C" TB_API tb_status tb_avg_pool2d(tb_context* ctx, const tb_pool2d_desc* d, const void* input, void* out,
                                          void* stream_) {
    if (!ctx || !d) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    PoolGeomDev g;
    TB_TRY(pool_geom("AVG_POOL2D", d, &g));
    const int dt = d->dtype, at = d->acc_dtype;
    // (src/ops/pool.rs:182-187)
    const bool ok = ((dt == TB_DT_INT8 || dt == TB_DT_INT16) && at == TB_DT_INT32) ||
                    (dt == TB_DT_FP16 && (at == TB_DT_FP16 || at == TB_DT_FP32)) ||
                    ((dt == TB_DT_BF16 || dt == TB_DT_FP32) && at == TB_DT_FP32) ||
                    ((dt == TB_DT_FP8E4M3 || dt == TB_DT_FP8E5M2) && at == TB_DT_FP16);
    if (!ok) return fail(TB_ERR_DTYPE_MISMATCH, "AVG_POOL2D: unsupported types input=%d acc=%d", dt, at);
    if (dt != TB_DT_INT8 && (d->input_zp != 0 || d->output_zp != 0))
        return fail(TB_ERR_GRAPH, "AVG_POOL2D: zero points must be zero for non-int8 data");
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.c;
    if (total == 0) return TB_OK;
    if (!input || !out) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    if (dt == TB_DT_INT8 && g.c % 16 == 0 && aligned16(input) && aligned16(out) && g.kx * g.ky <= 64 &&
        g.oh <= 65535 && g.n <= 65535) {
        static RecipTable table = [] {
            RecipTable t{};
            for (int c = 1; c <= 64; ++c) {  // reciprocal_scale (src/ops/quant.rs:6-11)
                const uint32_t v = static_cast<uint32_t>(c) - 1u;
                const int k = v == 0 ? 0 : 32 - __builtin_clz(v);
                const long long numerator = ((1ll << 30) + 1) << k;
                t.m[c] = static_cast<int32_t>(numerator / c);
                t.s[c] = 30 + k;
            }
            return t;
        }();
        const PoolTile pt = pool_tile(g.c, g.ow);
        const dim3 grid((g.ow + pt.ppb - 1) / pt.ppb, g.oh, g.n);
        const long long items = static_cast<long long>(g.n) * g.oh * g.ow * pt.cg;
        // wide windows over fewer outputs than two 256-thread blocks per SM would cover (global
        // pools): eight lanes per output group; otherwise taps in flight per thread: a window of up
        // to 4 taps in one batch, eight at a time for wide windows, one at a time in between
        // (measured on B200: batches of 8 over a 3x3 window cost more occupancy than they hide
        // latency)
        if (g.kx * g.ky >= 16 && items < 2ll * ctx->num_sms * 256) {
            constexpr int kLanes = 8;
            const dim3 sgrid((g.ow * pt.cg + 256 / kLanes - 1) / (256 / kLanes), g.oh, g.n);
            avg_pool_i8_vec16_split<kLanes><<<sgrid, 256, 0, st>>>(g, pt.cg, static_cast<const int8_t*>(input),
                                                                  d->input_zp, d->output_zp, table,
                                                                  static_cast<int8_t*>(out));
        } else if (g.kx * g.ky <= 4)
            avg_pool_i8_vec16<4><<<grid, pool_block(pt), 0, st>>>(g, pt, static_cast<const int8_t*>(input), d->input_zp,
                                                                  d->output_zp, table, static_cast<int8_t*>(out));
        else if (g.kx >= 6)
            avg_pool_i8_vec16<8><<<grid, pool_block(pt), 0, st>>>(g, pt, static_cast<const int8_t*>(input), d->input_zp,
                                                                  d->output_zp, table, static_cast<int8_t*>(out));
        else
            avg_pool_i8_vec16<1><<<grid, pool_block(pt), 0, st>>>(g, pt, static_cast<const int8_t*>(input), d->input_zp,
                                                                  d->output_zp, table, static_cast<int8_t*>(out));
    } else if (dt == TB_DT_INT8 && g.c % 4 == 0 && aligned16(input))
        avg_pool_i8_vec4<<<grid_for(ctx, total / 4), 256, 0, st>>>(g, static_cast<const int8_t*>(input), d->input_zp,
                                                                  d->output_zp, static_cast<int8_t*>(out), ctx->dev_err);
    else if (dt == TB_DT_INT8 || dt == TB_DT_INT16)
        avg_pool_int<<<grid_for(ctx, total), 256, 0, st>>>(g, input, dt, d->input_zp, d->output_zp, out, ctx->dev_err);
    else
        avg_pool_float<<<grid_for(ctx, total), 256, 0, st>>>(g, input, dt, at, out);
    TB_LAUNCHED(ctx);
    return TB_OK;
}

extern "C" TB_API tb_status tb_max_pool2d(tb_context* ctx, const tb_pool2d_desc* d, const void* input, void* out,
                                          void* stream_) {
    if (!ctx || !d) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    if (d->nan_mode != TB_NAN_PROPAGATE && d->nan_mode != TB_NAN_IGNORE)
        return fail(TB_ERR_GRAPH, "MAX_POOL2D: nan_mode must be PROPAGATE or IGNORE");
    PoolGeomDev g;
    TB_TRY(pool_geom("MAX_POOL2D", d, &g));
    const int dt = d->dtype;
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.c;
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    if (!(dt == TB_DT_INT8 || dt == TB_DT_INT16 || dt == TB_DT_FP16 || dt == TB_DT_BF16 || dt == TB_DT_FP32 ||
          dt == TB_DT_FP8E4M3 || dt == TB_DT_FP8E5M2))
        return fail(TB_ERR_DTYPE_MISMATCH, "MAX_POOL2D: unsupported dtype %d", dt);
    if (total == 0) return TB_OK;
    if (!input || !out) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    if (dt == TB_DT_INT8 && g.c % 16 == 0 && aligned16(input) && aligned16(out) && g.oh <= 65535 && g.n <= 65535) {
        const PoolTile pt = pool_tile(g.c, g.ow);
        const dim3 grid((g.ow + pt.ppb - 1) / pt.ppb, g.oh, g.n);
        // taps in flight per thread, as for AVG_POOL2D
        if (g.kx * g.ky <= 4)
            max_pool_i8_vec16<4><<<grid, pool_block(pt), 0, st>>>(g, pt, static_cast<const int8_t*>(input),
                                                                  static_cast<int8_t*>(out));
        else if (g.kx >= 6)
            max_pool_i8_vec16<8><<<grid, pool_block(pt), 0, st>>>(g, pt, static_cast<const int8_t*>(input),
                                                                  static_cast<int8_t*>(out));
        else
            max_pool_i8_vec16<1><<<grid, pool_block(pt), 0, st>>>(g, pt, static_cast<const int8_t*>(input),
                                                                  static_cast<int8_t*>(out));
    }
    else if (dt == TB_DT_INT8 && g.c % 4 == 0 && aligned16(input))
        max_pool_i8_vec4<<<grid_for(ctx, total / 4), 256, 0, st>>>(g, static_cast<const int8_t*>(input),
                                                                  static_cast<int8_t*>(out));
    else if (dt == TB_DT_INT8 || dt == TB_DT_INT16)
        max_pool_int<<<grid_for(ctx, total), 256, 0, st>>>(g, input, dt, out);
    else
        max_pool_float<<<grid_for(ctx, total), 256, 0, st>>>(g, input, dt, d->nan_mode, out);
    TB_LAUNCHED(ctx);
    return TB_OK;
}
