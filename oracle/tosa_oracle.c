/*
 * CPU oracle: C restatement of the reference interpreter's arithmetic for the
 * dense-contraction path. TEST INFRASTRUCTURE ONLY -- see tosa_oracle.h.
 *
 * Every function cites the reference source (tosa-interp, path:line) whose
 * loop order and integer/float arithmetic it restates. Compile with
 * -ffp-contract=off: the reference's `acc + a * b` rounds the product and the
 * sum separately (src/ops/accum.rs:58-71), so no FMA may be formed.
 */
#include "tosa_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------------
 * Float rounding helpers (src/ops/common.rs:100-108; half 2.7.1 from_f32 is
 * round-to-nearest-even with NaN kept NaN; src/float8.rs:69-113 for FP8).
 * ------------------------------------------------------------------------- */

static uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* f32 -> bf16 -> f32, round to nearest even. */
static float round_bf16(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return u2f((u | 0x00400000u) & 0xffff0000u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return u2f(u & 0xffff0000u);
}

/* f32 -> f16 -> f32, round to nearest even, with subnormals and overflow to
 * infinity. Written from the IEEE-754 binary16 definition. */
static float round_f16(float x) {
    if (isnan(x)) return x;
    float a = fabsf(x);
    if (a >= 65520.0f) return copysignf(INFINITY, x); /* halfway to 2^16 rounds up */
    if (a < 6.103515625e-05f) {
        /* subnormal range: multiples of 2^-24 */
        float q = rintf(a * 16777216.0f);
        return copysignf(q / 16777216.0f, x);
    }
    int e;
    frexpf(a, &e);                 /* a = f * 2^e, f in [0.5, 1) */
    float scale = ldexpf(1.0f, 11 - e); /* keep 11 significant bits */
    float q = rintf(a * scale);
    return copysignf(q / scale, x);
}

typedef struct { int man_bits, bias, has_inf; } fp8_fmt;
static fp8_fmt fp8_format(int dtype) {
    fp8_fmt f;
    if (dtype == ORC_FP8E4M3) { f.man_bits = 3; f.bias = 7; f.has_inf = 0; }
    else { f.man_bits = 2; f.bias = 15; f.has_inf = 1; }
    return f;
}

float orc_fp8_decode(int dtype, uint8_t bits) {
    fp8_fmt f = fp8_format(dtype);
    int exp_bits = 7 - f.man_bits;
    unsigned maxe = (1u << exp_bits) - 1u, manm = (1u << f.man_bits) - 1u;
    unsigned e = (bits >> f.man_bits) & maxe, m = bits & manm;
    int nan = f.has_inf ? (e == maxe && m != 0) : (e == maxe && m == manm);
    if (nan) return NAN;
    double sign = (bits & 0x80) ? -1.0 : 1.0;
    if (f.has_inf && e == maxe) return (float)(sign * INFINITY);
    double scale = (double)(1u << f.man_bits);
    double mag = e == 0 ? (double)m / scale * ldexp(1.0, 1 - f.bias)
                        : (1.0 + (double)m / scale) * ldexp(1.0, (int)e - f.bias);
    return (float)(sign * mag);
}

uint8_t orc_fp8_encode(int dtype, float x) {
    fp8_fmt f = fp8_format(dtype);
    int exp_bits = 7 - f.man_bits;
    unsigned maxe = (1u << exp_bits) - 1u, manm = (1u << f.man_bits) - 1u;
    uint8_t nanv = (uint8_t)((maxe << f.man_bits) | manm);
    if (isnan(x)) return nanv;
    uint8_t sign = signbit(x) ? 0x80 : 0;
    uint8_t overflow = f.has_inf ? (uint8_t)(sign | (maxe << f.man_bits)) : (uint8_t)(sign | nanv);
    if (isinf(x)) return overflow;
    double a = fabs((double)x);
    if (a == 0.0) return sign;
    double man_scale = (double)(1u << f.man_bits);
    int min_normal_exp = 1 - f.bias;
    int fe;
    frexp(a, &fe);
    int e = fe - 1; /* unbiased exponent */
    unsigned exp_field, man;
    if (e < min_normal_exp) {
        unsigned q = (unsigned)rint(a / ldexp(1.0, min_normal_exp) * man_scale);
        exp_field = q >> f.man_bits;
        man = q & manm;
    } else {
        unsigned q = (unsigned)rint(a / ldexp(1.0, e) * man_scale);
        if (q == (2u << f.man_bits)) { e += 1; q = 1u << f.man_bits; }
        exp_field = (unsigned)(e + f.bias);
        man = q & manm;
    }
    int exceeded = f.has_inf ? (exp_field >= maxe)
                             : (exp_field > maxe || (exp_field == maxe && man == manm));
    if (exceeded) return overflow;
    return (uint8_t)(sign | ((exp_field << f.man_bits) | man));
}

float orc_round_to(int dtype, float x) {
    switch (dtype) {
    case ORC_F16: return round_f16(x);
    case ORC_BF16: return round_bf16(x);
    case ORC_FP8E4M3:
    case ORC_FP8E5M2: return orc_fp8_decode(dtype, orc_fp8_encode(dtype, x));
    default: return x;
    }
}

/* ---------------------------------------------------------------------------
 * Fixed-point scaling (src/ops/quant.rs:6-32, src/ops/type_conv.rs:86-92)
 * ------------------------------------------------------------------------- */

void orc_reciprocal_scale(int32_t value, int32_t *multiplier, int32_t *shift) {
    uint32_t v = (uint32_t)value - 1u;
    int lz = v == 0 ? 32 : __builtin_clz(v);
    int k = 32 - lz;
    int64_t numerator = (((int64_t)1 << 30) + 1) << k;
    *multiplier = (int32_t)(numerator / (int64_t)value);
    *shift = 30 + k;
}

int orc_apply_scale_32(int32_t value, int32_t multiplier, int32_t shift, int double_round, int32_t *out) {
    if (multiplier < 0 || shift < 2 || shift > 62) return ORC_ERR_GRAPH;
    int64_t low = -((int64_t)1 << (shift - 1)), high = (int64_t)1 << (shift - 1);
    int64_t v = value;
    if (v < low || v >= high) return ORC_ERR_GRAPH;
    int64_t round = (int64_t)1 << (shift - 1);
    if (double_round && shift > 31) round += v >= 0 ? ((int64_t)1 << 30) : -((int64_t)1 << 30);
    int64_t r = (v * (int64_t)multiplier + round) >> shift;
    if (r < INT32_MIN || r > INT32_MAX) return ORC_ERR_GRAPH;
    *out = (int32_t)r;
    return ORC_OK;
}

int orc_apply_scale_16(int64_t value, int16_t multiplier, int32_t shift, int32_t *out) {
    if (multiplier < 0 || shift < 2 || shift > 62) return ORC_ERR_GRAPH;
    int64_t r = (value * (int64_t)multiplier + ((int64_t)1 << (shift - 1))) >> shift;
    if (r < INT32_MIN || r > INT32_MAX) return ORC_ERR_GRAPH;
    *out = (int32_t)r;
    return ORC_OK;
}

/* ---------------------------------------------------------------------------
 * Accumulators (src/ops/accum.rs:20-139). ACC_* select the mac rule.
 * ------------------------------------------------------------------------- */

enum { ACC_F32, ACC_F16, ACC_BF16, ACC_F16_UNROUNDED, ACC_BF16_UNROUNDED };

static inline float fmac(int kind, float acc, float a, float b) {
    float p = a * b;
    switch (kind) {
    case ACC_F32: return acc + p;                                         /* accum.rs:68-70 */
    case ACC_F16: return round_f16(acc + round_f16(p));                   /* accum.rs:84-87 */
    case ACC_BF16: return round_bf16(acc + round_bf16(p));                /* accum.rs:135-138 */
    case ACC_F16_UNROUNDED: return round_f16(acc + p);                    /* accum.rs:103-105 */
    default: return round_bf16(acc + p);                                  /* accum.rs:119-121 */
    }
}

static int acc_kind_for(int acc_type) {
    return acc_type == ORC_F16 ? ACC_F16 : acc_type == ORC_BF16 ? ACC_BF16 : ACC_F32;
}

static const int64_t INT48_MIN = -((int64_t)1 << 47);
static const int64_t INT48_MAX = ((int64_t)1 << 47) - 1;
static int64_t clamp48(int64_t v) { return v < INT48_MIN ? INT48_MIN : v > INT48_MAX ? INT48_MAX : v; }

/* ---------------------------------------------------------------------------
 * CONV2D (src/ops/conv.rs:147-181 loop; :457-497 operand handling)
 * ------------------------------------------------------------------------- */

/* Visit the output elements of rows [b0, b1) of the batch in reference order:
 * batch, output position (row-major), oc, then taps (ky,kx) and ic. The
 * template-like macro keeps the integer and float loops textually identical. */
#define CONV_LOOP(G, B0, B1, ACC_T, ZERO, MAC, EMIT)                                        \
    do {                                                                                     \
        const orc_conv_geom *g_ = (G);                                                       \
        for (int64_t b = (B0); b < (B1); ++b)                                                \
            for (int64_t oy = 0; oy < g_->oh; ++oy)                                          \
                for (int64_t ox = 0; ox < g_->ow; ++ox)                                      \
                    for (int64_t oc = 0; oc < g_->oc; ++oc) {                                \
                        ACC_T acc = ZERO;                                                    \
                        for (int64_t ky = 0; ky < g_->kh; ++ky) {                            \
                            int64_t y = oy * g_->stride[0] + ky * g_->dilation[0] - g_->pad[0]; \
                            if (y < 0 || y >= g_->ih) continue;                              \
                            for (int64_t kx = 0; kx < g_->kw; ++kx) {                        \
                                int64_t x = ox * g_->stride[1] + kx * g_->dilation[1] - g_->pad[2]; \
                                if (x < 0 || x >= g_->iw) continue;                          \
                                int64_t ib = ((b * g_->ih + y) * g_->iw + x) * g_->ic;       \
                                int64_t wb = ((oc * g_->kh + ky) * g_->kw + kx) * g_->ic;    \
                                for (int64_t c = 0; c < g_->ic; ++c) { MAC(ib + c, wb + c); } \
                            }                                                                \
                        }                                                                    \
                        int64_t oi = ((b * g_->oh + oy) * g_->ow + ox) * g_->oc + oc;       \
                        EMIT(oi, oc);                                                        \
                    }                                                                        \
    } while (0)

static void conv2d_i32_rows(const orc_conv_geom *g, const int32_t *in, const int32_t *w,
                            const int64_t *bias, int64_t bias_len, int64_t b0, int64_t b1,
                            int64_t *out) {
#define MAC_I32(i, j) acc = (int32_t)((uint32_t)acc + (uint32_t)in[i] * (uint32_t)w[j])
#define EMIT_I32(o, oc) out[o] = (int32_t)((uint32_t)acc + (uint32_t)(int32_t)bias[bias_len == 1 ? 0 : oc])
    CONV_LOOP(g, b0, b1, int32_t, 0, MAC_I32, EMIT_I32);
#undef MAC_I32
#undef EMIT_I32
}

static int32_t *sub_zp_i32(const int64_t *v, int64_t count, int64_t zp) {
    /* conv.rs:457-462: values minus zero point in i64, then `as i32`. */
    int32_t *r = (int32_t *)malloc((size_t)(count ? count : 1) * sizeof(int32_t));
    for (int64_t i = 0; i < count; ++i) r[i] = (int32_t)(v[i] - zp);
    return r;
}

void orc_conv2d_int(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                    const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                    int acc_i48, int64_t *out) {
    int64_t in_count = g->n * g->ih * g->iw * g->ic;
    int64_t w_count = g->oc * g->kh * g->kw * g->ic;
    if (!acc_i48) {
        int32_t *in = sub_zp_i32(input, in_count, input_zp);
        int32_t *w = sub_zp_i32(weight, w_count, weight_zp);
        conv2d_i32_rows(g, in, w, bias, bias_len, 0, g->n, out);
        free(in);
        free(w);
        return;
    }
    /* AccI64 path (I16 x I8 -> I48), conv.rs:466-473 */
#define MAC_I64(i, j) acc = (int64_t)((uint64_t)acc + (uint64_t)(input[i] - input_zp) * (uint64_t)(weight[j] - weight_zp))
#define EMIT_I64(o, oc) out[o] = clamp48((int64_t)((uint64_t)acc + (uint64_t)bias[bias_len == 1 ? 0 : oc]))
    CONV_LOOP(g, 0, g->n, int64_t, 0, MAC_I64, EMIT_I64);
#undef MAC_I64
#undef EMIT_I64
}

void orc_conv2d_float(const orc_conv_geom *g, const float *input, const float *weight,
                      const float *bias, int64_t bias_len, float input_zp, float weight_zp,
                      int acc_type, int out_type, float *out) {
    int64_t in_count = g->n * g->ih * g->iw * g->ic;
    int64_t w_count = g->oc * g->kh * g->kw * g->ic;
    float *in = (float *)malloc((size_t)(in_count ? in_count : 1) * sizeof(float));
    float *w = (float *)malloc((size_t)(w_count ? w_count : 1) * sizeof(float));
    for (int64_t i = 0; i < in_count; ++i) in[i] = input[i] - input_zp;
    for (int64_t i = 0; i < w_count; ++i) w[i] = weight[i] - weight_zp;
    int kind = acc_kind_for(acc_type);
    /* conv.rs:493-495: out = round(round(acc) + bias) */
#define MAC_F(i, j) acc = fmac(kind, acc, in[i], w[j])
#define EMIT_F(o, oc) out[o] = orc_round_to(out_type, orc_round_to(out_type, acc) + bias[bias_len == 1 ? 0 : oc])
    CONV_LOOP(g, 0, g->n, float, 0.0f, MAC_F, EMIT_F);
#undef MAC_F
#undef EMIT_F
    free(in);
    free(w);
}

/* ---------------------------------------------------------------------------
 * DEPTHWISE_CONV2D (src/ops/conv.rs:234-266)
 * ------------------------------------------------------------------------- */

#define DW_LOOP(G, ACC_T, ZERO, MAC, EMIT)                                                   \
    do {                                                                                     \
        const orc_conv_geom *g_ = (G);                                                       \
        int64_t cm = g_->ic * g_->m;                                                         \
        for (int64_t b = 0; b < g_->n; ++b)                                                  \
            for (int64_t oy = 0; oy < g_->oh; ++oy) {                                        \
                int64_t iy = oy * g_->stride[0] - g_->pad[0];                                \
                for (int64_t ox = 0; ox < g_->ow; ++ox) {                                    \
                    int64_t ix = ox * g_->stride[1] - g_->pad[2];                            \
                    for (int64_t c = 0; c < g_->ic; ++c)                                     \
                        for (int64_t mm = 0; mm < g_->m; ++mm) {                             \
                            ACC_T acc = ZERO;                                                \
                            for (int64_t ky = 0; ky < g_->kh; ++ky) {                        \
                                int64_t y = iy + ky * g_->dilation[0];                       \
                                if (y < 0 || y >= g_->ih) continue;                          \
                                for (int64_t kx = 0; kx < g_->kw; ++kx) {                    \
                                    int64_t x = ix + kx * g_->dilation[1];                   \
                                    if (x < 0 || x >= g_->iw) continue;                      \
                                    int64_t ii = ((b * g_->ih + y) * g_->iw + x) * g_->ic + c; \
                                    int64_t wi = ((ky * g_->kw + kx) * g_->ic + c) * g_->m + mm; \
                                    MAC(ii, wi);                                             \
                                }                                                            \
                            }                                                                \
                            int64_t oi = ((b * g_->oh + oy) * g_->ow + ox) * cm + c * g_->m + mm; \
                            EMIT(oi, c * g_->m + mm);                                        \
                        }                                                                    \
                }                                                                            \
            }                                                                                \
    } while (0)

void orc_depthwise_int(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                       const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                       int acc_i48, int64_t *out) {
    int64_t in_count = g->n * g->ih * g->iw * g->ic;
    int64_t w_count = g->kh * g->kw * g->ic * g->m;
    if (!acc_i48) {
        int32_t *in = sub_zp_i32(input, in_count, input_zp);
        int32_t *w = sub_zp_i32(weight, w_count, weight_zp);
#define MAC_I32(i, j) acc = (int32_t)((uint32_t)acc + (uint32_t)in[i] * (uint32_t)w[j])
#define EMIT_I32(o, oc) out[o] = (int32_t)((uint32_t)acc + (uint32_t)(int32_t)bias[bias_len == 1 ? 0 : oc])
        DW_LOOP(g, int32_t, 0, MAC_I32, EMIT_I32);
#undef MAC_I32
#undef EMIT_I32
        free(in);
        free(w);
        return;
    }
#define MAC_I64(i, j) acc = (int64_t)((uint64_t)acc + (uint64_t)(input[i] - input_zp) * (uint64_t)(weight[j] - weight_zp))
#define EMIT_I64(o, oc) out[o] = clamp48((int64_t)((uint64_t)acc + (uint64_t)bias[bias_len == 1 ? 0 : oc]))
    DW_LOOP(g, int64_t, 0, MAC_I64, EMIT_I64);
#undef MAC_I64
#undef EMIT_I64
}

void orc_depthwise_float(const orc_conv_geom *g, const float *input, const float *weight,
                         const float *bias, int64_t bias_len, float input_zp, float weight_zp,
                         int acc_type, int out_type, float *out) {
    int kind = acc_kind_for(acc_type);
#define MAC_F(i, j) acc = fmac(kind, acc, input[i] - input_zp, weight[j] - weight_zp)
#define EMIT_F(o, oc) out[o] = orc_round_to(out_type, orc_round_to(out_type, acc) + bias[bias_len == 1 ? 0 : oc])
    DW_LOOP(g, float, 0.0f, MAC_F, EMIT_F);
#undef MAC_F
#undef EMIT_F
}

/* ---------------------------------------------------------------------------
 * CONV3D (src/ops/conv.rs:147-181 ConvNd::accumulate, dims = 3): batch, output
 * position (d, h, w row-major), oc, then taps (kd, kh, kw row-major), ic
 * innermost; taps reading outside the input are skipped.
 * ------------------------------------------------------------------------- */
#define CONV3D_LOOP(G, ACC_T, ZERO, MAC, EMIT)                                              \
    do {                                                                                     \
        const orc_conv3d_geom *g_ = (G);                                                     \
        for (int64_t b = 0; b < g_->n; ++b)                                                  \
            for (int64_t oz = 0; oz < g_->od; ++oz)                                          \
                for (int64_t oy = 0; oy < g_->oh; ++oy)                                      \
                    for (int64_t ox = 0; ox < g_->ow; ++ox)                                  \
                        for (int64_t oc = 0; oc < g_->oc; ++oc) {                            \
                            ACC_T acc = ZERO;                                                \
                            for (int64_t kz = 0; kz < g_->kd; ++kz) {                        \
                                int64_t z = oz * g_->stride[0] + kz * g_->dilation[0] - g_->pad[0]; \
                                if (z < 0 || z >= g_->id) continue;                          \
                                for (int64_t ky = 0; ky < g_->kh; ++ky) {                    \
                                    int64_t y = oy * g_->stride[1] + ky * g_->dilation[1] - g_->pad[2]; \
                                    if (y < 0 || y >= g_->ih) continue;                      \
                                    for (int64_t kx = 0; kx < g_->kw; ++kx) {                \
                                        int64_t x = ox * g_->stride[2] + kx * g_->dilation[2] - g_->pad[4]; \
                                        if (x < 0 || x >= g_->iw) continue;                  \
                                        int64_t ib = (((b * g_->id + z) * g_->ih + y) * g_->iw + x) * g_->ic; \
                                        int64_t wb = (((oc * g_->kd + kz) * g_->kh + ky) * g_->kw + kx) * g_->ic; \
                                        for (int64_t c = 0; c < g_->ic; ++c) { MAC(ib + c, wb + c); } \
                                    }                                                        \
                                }                                                            \
                            }                                                                \
                            int64_t oi = (((b * g_->od + oz) * g_->oh + oy) * g_->ow + ox) * g_->oc + oc; \
                            EMIT(oi, oc);                                                    \
                        }                                                                    \
    } while (0)

void orc_conv3d_int(const orc_conv3d_geom *g, const int64_t *input, const int64_t *weight, const int64_t *bias,
                    int64_t bias_len, int64_t input_zp, int64_t weight_zp, int acc_i48, int64_t *out) {
    if (!acc_i48) {
        int32_t *in = sub_zp_i32(input, g->n * g->id * g->ih * g->iw * g->ic, input_zp);
        int32_t *w = sub_zp_i32(weight, g->oc * g->kd * g->kh * g->kw * g->ic, weight_zp);
#define MAC_I32(i, j) acc = (int32_t)((uint32_t)acc + (uint32_t)in[i] * (uint32_t)w[j])
#define EMIT_I32(o, oc) out[o] = (int32_t)((uint32_t)acc + (uint32_t)(int32_t)bias[bias_len == 1 ? 0 : oc])
        CONV3D_LOOP(g, int32_t, 0, MAC_I32, EMIT_I32);
#undef MAC_I32
#undef EMIT_I32
        free(in);
        free(w);
        return;
    }
#define MAC_I64(i, j) acc = (int64_t)((uint64_t)acc + (uint64_t)(input[i] - input_zp) * (uint64_t)(weight[j] - weight_zp))
#define EMIT_I64(o, oc) out[o] = clamp48((int64_t)((uint64_t)acc + (uint64_t)bias[bias_len == 1 ? 0 : oc]))
    CONV3D_LOOP(g, int64_t, 0, MAC_I64, EMIT_I64);
#undef MAC_I64
#undef EMIT_I64
}

void orc_conv3d_float(const orc_conv3d_geom *g, const float *input, const float *weight, const float *bias,
                      int64_t bias_len, float input_zp, float weight_zp, int acc_type, int out_type, float *out) {
    int64_t in_count = g->n * g->id * g->ih * g->iw * g->ic;
    int64_t w_count = g->oc * g->kd * g->kh * g->kw * g->ic;
    float *in = (float *)malloc((size_t)(in_count ? in_count : 1) * sizeof(float));
    float *w = (float *)malloc((size_t)(w_count ? w_count : 1) * sizeof(float));
    for (int64_t i = 0; i < in_count; ++i) in[i] = input[i] - input_zp;
    for (int64_t i = 0; i < w_count; ++i) w[i] = weight[i] - weight_zp;
    int kind = acc_kind_for(acc_type);
#define MAC_F(i, j) acc = fmac(kind, acc, in[i], w[j])
#define EMIT_F(o, oc) out[o] = orc_round_to(out_type, orc_round_to(out_type, acc) + bias[bias_len == 1 ? 0 : oc])
    CONV3D_LOOP(g, float, 0.0f, MAC_F, EMIT_F);
#undef MAC_F
#undef EMIT_F
    free(in);
    free(w);
}

/* ---------------------------------------------------------------------------
 * TRANSPOSE_CONV2D (src/ops/conv.rs:337-371 Transpose::accumulate, gather form):
 * output (oy, ox) reads input ((oy - out_pad_top - ky) / stride_y, ...) where
 * the division is exact and in range; taps (ky, kx) row-major, ic innermost.
 * g->pad[0] / g->pad[2] hold out_pad_top / out_pad_left (may be negative);
 * the weight is OHWI as for CONV2D.
 * ------------------------------------------------------------------------- */
#define TCONV_LOOP(G, ACC_T, ZERO, MAC, EMIT)                                               \
    do {                                                                                     \
        const orc_conv_geom *g_ = (G);                                                       \
        int64_t sy_ = g_->stride[0], sx_ = g_->stride[1];                                    \
        for (int64_t b = 0; b < g_->n; ++b)                                                  \
            for (int64_t oy = 0; oy < g_->oh; ++oy)                                          \
                for (int64_t ox = 0; ox < g_->ow; ++ox)                                      \
                    for (int64_t oc = 0; oc < g_->oc; ++oc) {                                \
                        ACC_T acc = ZERO;                                                    \
                        for (int64_t ky = 0; ky < g_->kh; ++ky) {                            \
                            int64_t y = oy - g_->pad[0] - ky;                                \
                            if (y < 0 || y >= g_->ih * sy_ || y % sy_ != 0) continue;        \
                            for (int64_t kx = 0; kx < g_->kw; ++kx) {                        \
                                int64_t x = ox - g_->pad[2] - kx;                            \
                                if (x < 0 || x >= g_->iw * sx_ || x % sx_ != 0) continue;    \
                                int64_t ib = ((b * g_->ih + y / sy_) * g_->iw + x / sx_) * g_->ic; \
                                int64_t wb = ((oc * g_->kh + ky) * g_->kw + kx) * g_->ic;    \
                                for (int64_t c = 0; c < g_->ic; ++c) { MAC(ib + c, wb + c); } \
                            }                                                                \
                        }                                                                    \
                        int64_t oi = ((b * g_->oh + oy) * g_->ow + ox) * g_->oc + oc;       \
                        EMIT(oi, oc);                                                        \
                    }                                                                        \
    } while (0)

void orc_transpose_conv2d_int(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                              const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                              int acc_i48, int64_t *out) {
    if (!acc_i48) {
        int32_t *in = sub_zp_i32(input, g->n * g->ih * g->iw * g->ic, input_zp);
        int32_t *w = sub_zp_i32(weight, g->oc * g->kh * g->kw * g->ic, weight_zp);
#define MAC_I32(i, j) acc = (int32_t)((uint32_t)acc + (uint32_t)in[i] * (uint32_t)w[j])
#define EMIT_I32(o, oc) out[o] = (int32_t)((uint32_t)acc + (uint32_t)(int32_t)bias[bias_len == 1 ? 0 : oc])
        TCONV_LOOP(g, int32_t, 0, MAC_I32, EMIT_I32);
#undef MAC_I32
#undef EMIT_I32
        free(in);
        free(w);
        return;
    }
#define MAC_I64(i, j) acc = (int64_t)((uint64_t)acc + (uint64_t)(input[i] - input_zp) * (uint64_t)(weight[j] - weight_zp))
#define EMIT_I64(o, oc) out[o] = clamp48((int64_t)((uint64_t)acc + (uint64_t)bias[bias_len == 1 ? 0 : oc]))
    TCONV_LOOP(g, int64_t, 0, MAC_I64, EMIT_I64);
#undef MAC_I64
#undef EMIT_I64
}

void orc_transpose_conv2d_float(const orc_conv_geom *g, const float *input, const float *weight,
                                const float *bias, int64_t bias_len, float input_zp, float weight_zp,
                                int acc_type, int out_type, float *out) {
    int64_t in_count = g->n * g->ih * g->iw * g->ic;
    int64_t w_count = g->oc * g->kh * g->kw * g->ic;
    float *in = (float *)malloc((size_t)(in_count ? in_count : 1) * sizeof(float));
    float *w = (float *)malloc((size_t)(w_count ? w_count : 1) * sizeof(float));
    for (int64_t i = 0; i < in_count; ++i) in[i] = input[i] - input_zp;
    for (int64_t i = 0; i < w_count; ++i) w[i] = weight[i] - weight_zp;
    int kind = acc_kind_for(acc_type);
#define MAC_F(i, j) acc = fmac(kind, acc, in[i], w[j])
#define EMIT_F(o, oc) out[o] = orc_round_to(out_type, orc_round_to(out_type, acc) + bias[bias_len == 1 ? 0 : oc])
    TCONV_LOOP(g, float, 0.0f, MAC_F, EMIT_F);
#undef MAC_F
#undef EMIT_F
    free(in);
    free(w);
}

/* ---------------------------------------------------------------------------
 * MATMUL (src/ops/matmul.rs:75-95 Dims::run, :137-171 operand handling)
 * ------------------------------------------------------------------------- */

static void matmul_i32_rows(int64_t h, int64_t c, int64_t w, const int32_t *a, const int32_t *b,
                            int64_t r0, int64_t r1, int64_t *out) {
    /* rows r = bn*h + row, matmul.rs:82-93 with b_index (n*c + k)*w + col */
    for (int64_t r = r0; r < r1; ++r) {
        int64_t bn = r / h;
        const int32_t *arow = a + r * c;
        for (int64_t col = 0; col < w; ++col) {
            int32_t acc = 0;
            for (int64_t k = 0; k < c; ++k)
                acc = (int32_t)((uint32_t)acc + (uint32_t)arow[k] * (uint32_t)b[(bn * c + k) * w + col]);
            out[r * w + col] = acc;
        }
    }
}

void orc_matmul_int(int64_t n, int64_t h, int64_t c, int64_t w, const int64_t *a, const int64_t *b,
                    int64_t a_zp, int64_t b_zp, int out_i48, int64_t *out) {
    if (!out_i48) {
        int32_t *av = sub_zp_i32(a, n * h * c, a_zp);
        int32_t *bv = sub_zp_i32(b, n * c * w, b_zp);
        matmul_i32_rows(h, c, w, av, bv, 0, n * h, out);
        free(av);
        free(bv);
        return;
    }
    for (int64_t bn = 0; bn < n; ++bn)
        for (int64_t row = 0; row < h; ++row)
            for (int64_t col = 0; col < w; ++col) {
                int64_t acc = 0;
                for (int64_t k = 0; k < c; ++k)
                    acc = (int64_t)((uint64_t)acc + (uint64_t)(a[(bn * h + row) * c + k] - a_zp) *
                                                        (uint64_t)(b[(bn * c + k) * w + col] - b_zp));
                out[(bn * h + row) * w + col] = clamp48(acc);
            }
}

/* MATMUL_T (matmul.rs:75-78 b_index with b_transposed): b [d,w,c], its batch
 * index 0 for every bn when d == 1 (b_broadcast); otherwise as MATMUL. */
static int64_t mt_b_index(int64_t bn, int64_t k, int64_t col, int64_t c, int64_t w, int bcast) {
    int64_t nb = bcast ? 0 : bn;
    return (nb * w + col) * c + k;
}

void orc_matmul_t_int(int64_t n, int64_t h, int64_t c, int64_t w, int64_t d, const int64_t *a, const int64_t *b,
                      int64_t a_zp, int64_t b_zp, int out_i48, int64_t *out) {
    int bcast = d != n;
    for (int64_t bn = 0; bn < n; ++bn)
        for (int64_t row = 0; row < h; ++row)
            for (int64_t col = 0; col < w; ++col) {
                uint64_t acc = 0;
                for (int64_t k = 0; k < c; ++k) {
                    int64_t x = a[(bn * h + row) * c + k] - a_zp;
                    int64_t y = b[mt_b_index(bn, k, col, c, w, bcast)] - b_zp;
                    if (out_i48) acc += (uint64_t)x * (uint64_t)y;
                    else acc = (uint32_t)((uint32_t)acc + (uint32_t)(int32_t)x * (uint32_t)(int32_t)y);
                }
                out[(bn * h + row) * w + col] = out_i48 ? clamp48((int64_t)acc) : (int64_t)(int32_t)(uint32_t)acc;
            }
}

void orc_matmul_t_float(int64_t n, int64_t h, int64_t c, int64_t w, int64_t d, const float *a, const float *b,
                        int out_type, float *out) {
    int kind = out_type == ORC_F16 ? ACC_F16_UNROUNDED : out_type == ORC_BF16 ? ACC_BF16_UNROUNDED : ACC_F32;
    int bcast = d != n;
    for (int64_t bn = 0; bn < n; ++bn)
        for (int64_t row = 0; row < h; ++row)
            for (int64_t col = 0; col < w; ++col) {
                float acc = 0.0f;
                for (int64_t k = 0; k < c; ++k)
                    acc = fmac(kind, acc, orc_round_to(out_type, a[(bn * h + row) * c + k]),
                               orc_round_to(out_type, b[mt_b_index(bn, k, col, c, w, bcast)]));
                out[(bn * h + row) * w + col] = orc_round_to(out_type, acc);
            }
}

/* Rows r0..r1 of the flattened [n*h] output rows of a float MATMUL. */
static void matmul_float_rows(int64_t h, int64_t c, int64_t w, const float *a, const float *b, int out_type,
                              int64_t r0, int64_t r1, float *out) {
    /* matmul.rs:160-170: operands rounded to the output type; accumulator per
     * output type (F32: AccF32, F16/BF16: rounded sum, unrounded product). */
    int kind = out_type == ORC_F16 ? ACC_F16_UNROUNDED : out_type == ORC_BF16 ? ACC_BF16_UNROUNDED : ACC_F32;
    for (int64_t r = r0; r < r1; ++r) {
        const int64_t bn = r / h;
        for (int64_t col = 0; col < w; ++col) {
            float acc = 0.0f;
            for (int64_t k = 0; k < c; ++k)
                acc = fmac(kind, acc, orc_round_to(out_type, a[r * c + k]),
                           orc_round_to(out_type, b[(bn * c + k) * w + col]));
            out[r * w + col] = orc_round_to(out_type, acc);
        }
    }
}

void orc_matmul_float(int64_t n, int64_t h, int64_t c, int64_t w, const float *a, const float *b,
                      int out_type, float *out) {
    matmul_float_rows(h, c, w, a, b, out_type, 0, n * h, out);
}

/* Multi-threaded drivers for the timed reference arm: rows are split into
 * contiguous chunks; each output element is computed exactly as above. */
typedef struct {
    int kind; /* 0 int matmul, 1 int conv, 2 float matmul */
    int64_t h, c, w;
    const int32_t *a, *b;
    const orc_conv_geom *g;
    const int64_t *bias;
    int64_t bias_len;
    int64_t r0, r1;
    int64_t *out;
    const float *fa, *fb;
    int out_type;
    float *fout;
} mt_job;

static void *mt_worker(void *p) {
    mt_job *j = (mt_job *)p;
    if (j->kind == 0) matmul_i32_rows(j->h, j->c, j->w, j->a, j->b, j->r0, j->r1, j->out);
    else if (j->kind == 1) conv2d_i32_rows(j->g, j->a, j->b, j->bias, j->bias_len, j->r0, j->r1, j->out);
    else matmul_float_rows(j->h, j->c, j->w, j->fa, j->fb, j->out_type, j->r0, j->r1, j->fout);
    return NULL;
}

static void run_mt(mt_job *proto, int64_t rows, int threads) {
    if (threads < 1) threads = 1;
    if (threads > rows) threads = (int)(rows ? rows : 1);
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    mt_job *jobs = (mt_job *)malloc(sizeof(mt_job) * (size_t)threads);
    for (int t = 0; t < threads; ++t) {
        jobs[t] = *proto;
        jobs[t].r0 = rows * t / threads;
        jobs[t].r1 = rows * (t + 1) / threads;
        pthread_create(&tid[t], NULL, mt_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
}

void orc_matmul_int_mt(int64_t n, int64_t h, int64_t c, int64_t w, const int64_t *a,
                       const int64_t *b, int64_t a_zp, int64_t b_zp, int64_t *out, int threads) {
    int32_t *av = sub_zp_i32(a, n * h * c, a_zp);
    int32_t *bv = sub_zp_i32(b, n * c * w, b_zp);
    mt_job proto;
    memset(&proto, 0, sizeof proto);
    proto.kind = 0; proto.h = h; proto.c = c; proto.w = w; proto.a = av; proto.b = bv; proto.out = out;
    run_mt(&proto, n * h, threads);
    free(av);
    free(bv);
}

void orc_matmul_float_mt(int64_t n, int64_t h, int64_t c, int64_t w, const float *a, const float *b,
                         int out_type, float *out, int threads) {
    mt_job proto;
    memset(&proto, 0, sizeof proto);
    proto.kind = 2; proto.h = h; proto.c = c; proto.w = w; proto.fa = a; proto.fb = b;
    proto.out_type = out_type; proto.fout = out;
    run_mt(&proto, n * h, threads);
}

void orc_conv2d_int_mt(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                       const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                       int64_t *out, int threads) {
    int32_t *in = sub_zp_i32(input, g->n * g->ih * g->iw * g->ic, input_zp);
    int32_t *w = sub_zp_i32(weight, g->oc * g->kh * g->kw * g->ic, weight_zp);
    mt_job proto;
    memset(&proto, 0, sizeof proto);
    proto.kind = 1; proto.g = g; proto.a = in; proto.b = w; proto.bias = bias; proto.bias_len = bias_len;
    proto.out = out;
    run_mt(&proto, g->n, threads);
    free(in);
    free(w);
}

/* ---------------------------------------------------------------------------
 * RESCALE (src/ops/type_conv.rs:94-190)
 * ------------------------------------------------------------------------- */

static int bit_width(int dtype) {
    return dtype == ORC_I8 ? 8 : dtype == ORC_I16 ? 16 : dtype == ORC_I32 ? 32 : 48;
}
static int64_t extend(int dtype, int64_t v, int uns) {
    return uns ? (v & (((int64_t)1 << bit_width(dtype)) - 1)) : v;
}
static void int_range(int dtype, int64_t *lo, int64_t *hi) {
    switch (dtype) {
    case ORC_I4: *lo = -8; *hi = 7; break;
    case ORC_I8: *lo = -128; *hi = 127; break;
    case ORC_I16: *lo = -32768; *hi = 32767; break;
    case ORC_I32: *lo = INT32_MIN; *hi = INT32_MAX; break;
    case ORC_I48: *lo = INT48_MIN; *hi = INT48_MAX; break;
    default: *lo = INT64_MIN; *hi = INT64_MAX;
    }
}
/* int_data packing (common.rs:112-122): wrap to the dtype's width. */
static int64_t wrap_to(int dtype, int64_t v) {
    switch (dtype) {
    case ORC_I4: return (int64_t)(int8_t)((int8_t)(v << 4) >> 4);
    case ORC_I8: return (int8_t)v;
    case ORC_I16: return (int16_t)v;
    case ORC_I32: return (int32_t)v;
    case ORC_I48: return (int64_t)((uint64_t)v << 16) >> 16;
    default: return v;
    }
}

/* Rust `f32 as i32`: saturating, NaN -> 0. */
static int32_t f32_to_i32_sat(float x) {
    if (isnan(x)) return 0;
    if (x >= 2147483648.0f) return INT32_MAX;
    if (x < -2147483648.0f) return INT32_MIN;
    return (int32_t)x;
}

int orc_rescale(const int64_t *input, int64_t count, int in_type, int out_type,
                const int64_t *multiplier, const int64_t *shift, int64_t channels,
                int64_t in_zp_raw, int64_t out_zp_raw, int scale32, int rounding_mode,
                int per_channel, int input_unsigned, int output_unsigned, int64_t *out) {
    int64_t in_zp = extend(in_type, in_zp_raw, input_unsigned);
    int64_t out_zp = extend(out_type, out_zp_raw, output_unsigned);
    int64_t lo, hi;
    if (output_unsigned) { lo = 0; hi = ((int64_t)1 << bit_width(out_type)) - 1; }
    else int_range(out_type, &lo, &hi);
    for (int64_t i = 0; i < count; ++i) {
        int64_t ch = per_channel ? i % channels : 0;
        int32_t m = (int32_t)multiplier[ch], s = (int32_t)shift[ch];
        int64_t x = extend(in_type, input[i], input_unsigned) - in_zp;
        int32_t scaled;
        if (rounding_mode == ORC_ROUND_INEXACT) {
            float t = (float)x * (float)m;
            t = t * ldexpf(1.0f, -s);
            scaled = f32_to_i32_sat(rintf(t));
        } else if (scale32) {
            if (orc_apply_scale_32((int32_t)x, m, s, rounding_mode == ORC_ROUND_DOUBLE, &scaled)) return ORC_ERR_GRAPH;
        } else {
            if (orc_apply_scale_16(x, (int16_t)m, s, &scaled)) return ORC_ERR_GRAPH;
        }
        int64_t result = (int64_t)scaled + out_zp;
        if (result < INT32_MIN || result > INT32_MAX) return ORC_ERR_GRAPH;
        int64_t c = result < lo ? lo : result > hi ? hi : result;
        out[i] = wrap_to(out_type, c);
    }
    return ORC_OK;
}

/* ---------------------------------------------------------------------------
 * Pooling (src/ops/pool.rs:77-104 window order; :186-227 AVG; :262-284 MAX)
 * ------------------------------------------------------------------------- */

#define POOL_LOOP(G, ...)                                                                    \
    do {                                                                                     \
        const orc_pool_geom *g_ = (G);                                                       \
        int64_t widx[1024];                                                                  \
        int64_t o_ = 0;                                                                      \
        for (int64_t b = 0; b < g_->n; ++b)                                                  \
            for (int64_t oy = 0; oy < g_->oh; ++oy) {                                        \
                int64_t iy = oy * g_->stride[0] - g_->pad_top;                               \
                for (int64_t ox = 0; ox < g_->ow; ++ox) {                                    \
                    int64_t ix = ox * g_->stride[1] - g_->pad_left;                          \
                    for (int64_t c = 0; c < g_->c; ++c) {                                    \
                        int64_t nw = 0;                                                      \
                        for (int64_t ky = 0; ky < g_->kernel[0]; ++ky) {                     \
                            int64_t y = iy + ky;                                             \
                            if (y < 0 || y >= g_->ih) continue;                              \
                            for (int64_t kx = 0; kx < g_->kernel[1]; ++kx) {                 \
                                int64_t x = ix + kx;                                         \
                                if (x < 0 || x >= g_->iw) continue;                          \
                                if (nw < 1024) widx[nw] = ((b * g_->ih + y) * g_->iw + x) * g_->c + c; \
                                ++nw;                                                        \
                            }                                                                \
                        }                                                                    \
                        __VA_ARGS__;                                                         \
                        ++o_;                                                                \
                    }                                                                        \
                }                                                                            \
            }                                                                                \
    } while (0)

/* Windows above 1024 in-bounds taps fall back to recomputing indices. */
static int64_t window_index(const orc_pool_geom *g, int64_t b, int64_t iy, int64_t ix, int64_t c,
                            int64_t k) {
    int64_t seen = 0;
    for (int64_t ky = 0; ky < g->kernel[0]; ++ky) {
        int64_t y = iy + ky;
        if (y < 0 || y >= g->ih) continue;
        for (int64_t kx = 0; kx < g->kernel[1]; ++kx) {
            int64_t x = ix + kx;
            if (x < 0 || x >= g->iw) continue;
            if (seen++ == k) return ((b * g->ih + y) * g->iw + x) * g->c + c;
        }
    }
    return -1;
}
#define WIDX(k) ((k) < 1024 ? widx[k] : window_index(g_, b, iy, ix, c, (k)))

int orc_avg_pool_int(const orc_pool_geom *g, const int64_t *input, int in_type,
                     int64_t in_zp, int64_t out_zp, int64_t *out) {
    int64_t lo, hi;
    int_range(in_type, &lo, &hi);
    int status = ORC_OK;
    POOL_LOOP(g, {
        int32_t acc = 0;
        for (int64_t k = 0; k < nw; ++k) acc = (int32_t)((uint32_t)acc + (uint32_t)(int32_t)(input[WIDX(k)] - in_zp));
        int32_t m, s, v;
        orc_reciprocal_scale((int32_t)nw, &m, &s);
        if (orc_apply_scale_32(acc, m, s, 0, &v)) status = ORC_ERR_GRAPH;
        else {
            int64_t r = (int64_t)v + out_zp;
            out[o_] = wrap_to(in_type, r < lo ? lo : r > hi ? hi : r);
        }
    });
    return status;
}

void orc_avg_pool_float(const orc_pool_geom *g, const float *input, int in_type, int acc_type,
                        float *out) {
    POOL_LOOP(g, {
        float acc = 0.0f;
        for (int64_t k = 0; k < nw; ++k) acc = orc_round_to(acc_type, acc + input[WIDX(k)]);
        out[o_] = orc_round_to(in_type, orc_round_to(acc_type, acc / (float)nw));
    });
}

void orc_max_pool_int(const orc_pool_geom *g, const int64_t *input, int in_type, int64_t *out) {
    int64_t lo, hi;
    int_range(in_type, &lo, &hi);
    POOL_LOOP(g, {
        int64_t m = lo;
        for (int64_t k = 0; k < nw; ++k) { int64_t v = input[WIDX(k)]; if (v > m) m = v; }
        out[o_] = m;
    });
}

/* nan_max / nan_pick (src/ops/common.rs:153-177) */
static float nan_pick(float a, float b, int mode) {
    if (mode == ORC_NAN_IGNORE) return isnan(a) ? b : a;
    return NAN;
}
static float nan_max(float a, float b, int mode) {
    if (isnan(a) || isnan(b)) return nan_pick(a, b, mode);
    return a >= b ? a : b;
}
static float nan_min(float a, float b, int mode) {
    if (isnan(a) || isnan(b)) return nan_pick(a, b, mode);
    return a < b ? a : b;
}
static float float_lowest(int dtype) { return dtype == ORC_FP8E4M3 ? -448.0f : -INFINITY; }

void orc_max_pool_float(const orc_pool_geom *g, const float *input, int in_type, int nan_mode,
                        float *out) {
    float init = nan_mode == ORC_NAN_IGNORE ? NAN : float_lowest(in_type);
    POOL_LOOP(g, {
        float m = init;
        for (int64_t k = 0; k < nw; ++k) m = nan_max(m, input[WIDX(k)], nan_mode);
        out[o_] = orc_round_to(in_type, m);
    });
}

/* ---------------------------------------------------------------------------
 * CLAMP (src/ops/elementwise.rs:319-343) and ADD (:395-397)
 * ------------------------------------------------------------------------- */

void orc_clamp_int(const int64_t *input, int64_t count, int64_t lo, int64_t hi, int64_t *out) {
    for (int64_t i = 0; i < count; ++i) {
        int64_t x = input[i];
        x = x > lo ? x : lo;
        out[i] = x < hi ? x : hi;
    }
}

void orc_clamp_float(const float *input, int64_t count, float lo, float hi, int nan_mode,
                     int dtype, float *out) {
    for (int64_t i = 0; i < count; ++i)
        out[i] = orc_round_to(dtype, nan_min(nan_max(input[i], lo, nan_mode), hi, nan_mode));
}

void orc_add_int(const int64_t *a, const int64_t *b, int64_t count, int dtype, int64_t *out) {
    for (int64_t i = 0; i < count; ++i) out[i] = wrap_to(dtype, (int64_t)((uint64_t)a[i] + (uint64_t)b[i]));
}
