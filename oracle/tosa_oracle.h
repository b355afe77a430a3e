/*
 * CPU oracle for the tosa_b200 dense-contraction path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a single-threaded C restatement of the
 * reference interpreter's (tosa-interp, Rust) arithmetic for CONV2D, CONV3D,
 * DEPTHWISE_CONV2D, TRANSPOSE_CONV2D, MATMUL, MATMUL_T, RESCALE, AVG_POOL2D,
 * MAX_POOL2D and CLAMP. It is
 * linked only by tests/, by __graft_entry__.smoke() and by bench.py's CPU
 * baseline legs, where it is the checker or the timed reference arm. The
 * product library (libtosa_b200) never links or calls it.
 *
 * Parity is pinned: tests/test_oracle_golden.py replays every positive and
 * negative conformance case of these operators that the reference ships
 * (golden vectors produced by the TOSA reference model, committed under
 * tests/golden/) through this oracle and requires bit-exact agreement.
 *
 * Integer operands are passed widened to int64 (the reference's
 * `int_values`, src/ops/common.rs:63-71); float operands are passed widened to
 * f32 (`float_values`, src/ops/common.rs:75-84). Validation of shapes,
 * attributes and dtypes (the ERROR_IF rules) lives in oracle/oracle.py.
 */
#ifndef TOSA_ORACLE_H
#define TOSA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (mirroring the reference's Error variants that the hot path
 * can raise at run time). */
enum {
    ORC_OK = 0,
    ORC_ERR_GRAPH = 1, /* Error::GraphError (apply_scale range, int32 overflow) */
};

/* DType codes: the serialized TOSA DType enum (schema/tosa.fbs:26-46). */
enum {
    ORC_BOOL = 1,
    ORC_I4 = 2,
    ORC_I8 = 3,
    ORC_I16 = 4,
    ORC_I32 = 5,
    ORC_I48 = 6,
    ORC_F32 = 7,
    ORC_F16 = 8,
    ORC_BF16 = 9,
    ORC_FP8E4M3 = 11,
    ORC_FP8E5M2 = 12,
    ORC_I64 = 17,
};

/* Rounding modes of RESCALE (src/ir.rs:75-85). */
enum { ORC_ROUND_SINGLE = 1, ORC_ROUND_INEXACT = 2, ORC_ROUND_DOUBLE = 3 };
/* NaN modes (src/ir.rs:103-111). */
enum { ORC_NAN_PROPAGATE = 1, ORC_NAN_IGNORE = 2 };

/* Round an f32 to the nearest value of `dtype` (common.rs:100-108). */
float orc_round_to(int dtype, float x);
/* Decode an 8-bit float (float8.rs:48-67). */
float orc_fp8_decode(int dtype, uint8_t bits);
uint8_t orc_fp8_encode(int dtype, float x);

/* quant.rs:6-11 and :17-32. Returns ORC_OK or ORC_ERR_GRAPH. */
void orc_reciprocal_scale(int32_t value, int32_t *multiplier, int32_t *shift);
int orc_apply_scale_32(int32_t value, int32_t multiplier, int32_t shift, int double_round, int32_t *out);
/* type_conv.rs:86-92 */
int orc_apply_scale_16(int64_t value, int16_t multiplier, int32_t shift, int32_t *out);

/* Convolution geometry. pad = [top, bottom, left, right]. */
typedef struct {
    int64_t n, ih, iw, ic;   /* input  NHWC */
    int64_t oc, kh, kw;      /* weight OHWI (CONV2D) */
    int64_t oh, ow;          /* output NHWC */
    int64_t pad[4];
    int64_t stride[2];
    int64_t dilation[2];
    int64_t m;               /* DEPTHWISE channel multiplier (weight [KH,KW,C,M]) */
} orc_conv_geom;

/* CONV2D integer path, conv.rs:398-500 (eval_conv, int branch) with
 * ConvNd::accumulate conv.rs:147-181. acc_i48 selects AccI64 + 48-bit clamp. */
void orc_conv2d_int(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                    const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                    int acc_i48, int64_t *out);
/* CONV2D float path: acc_type F32/F16/BF16, output rounded to out_type. */
void orc_conv2d_float(const orc_conv_geom *g, const float *input, const float *weight,
                      const float *bias, int64_t bias_len, float input_zp, float weight_zp,
                      int acc_type, int out_type, float *out);
/* DEPTHWISE_CONV2D, Depthwise::accumulate conv.rs:225-266. */
void orc_depthwise_int(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                       const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                       int acc_i48, int64_t *out);
void orc_depthwise_float(const orc_conv_geom *g, const float *input, const float *weight,
                         const float *bias, int64_t bias_len, float input_zp, float weight_zp,
                         int acc_type, int out_type, float *out);

/* CONV3D geometry: input NDHWC, weight [oc, kd, kh, kw, ic], pad = [front, back,
 * top, bottom, left, right], stride / dilation [d, h, w]. */
typedef struct {
    int64_t n, id, ih, iw, ic, oc, kd, kh, kw, od, oh, ow;
    int64_t pad[6];
    int64_t stride[3];
    int64_t dilation[3];
} orc_conv3d_geom;
/* CONV3D, ConvNd::accumulate conv.rs:147-181 with three spatial dimensions. */
void orc_conv3d_int(const orc_conv3d_geom *g, const int64_t *input, const int64_t *weight, const int64_t *bias,
                    int64_t bias_len, int64_t input_zp, int64_t weight_zp, int acc_i48, int64_t *out);
void orc_conv3d_float(const orc_conv3d_geom *g, const float *input, const float *weight, const float *bias,
                      int64_t bias_len, float input_zp, float weight_zp, int acc_type, int out_type, float *out);

/* TRANSPOSE_CONV2D, Transpose::accumulate conv.rs:337-371 (gather form); the
 * geometry's pad[0] / pad[2] are out_pad_top / out_pad_left, weight OHWI. */
void orc_transpose_conv2d_int(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                              const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                              int acc_i48, int64_t *out);
void orc_transpose_conv2d_float(const orc_conv_geom *g, const float *input, const float *weight,
                                const float *bias, int64_t bias_len, float input_zp, float weight_zp,
                                int acc_type, int out_type, float *out);

/* MATMUL, matmul.rs:80-95 + :137-171. a [N,H,C], b [N,C,W]. */
void orc_matmul_int(int64_t n, int64_t h, int64_t c, int64_t w, const int64_t *a, const int64_t *b,
                    int64_t a_zp, int64_t b_zp, int out_i48, int64_t *out);
void orc_matmul_float(int64_t n, int64_t h, int64_t c, int64_t w, const float *a, const float *b,
                      int out_type, float *out);
/* MATMUL_T, matmul.rs:75-95 with b_transposed: b [d,w,c], d == n, or 1 broadcast. */
void orc_matmul_t_int(int64_t n, int64_t h, int64_t c, int64_t w, int64_t d, const int64_t *a, const int64_t *b,
                      int64_t a_zp, int64_t b_zp, int out_i48, int64_t *out);
void orc_matmul_t_float(int64_t n, int64_t h, int64_t c, int64_t w, int64_t d, const float *a, const float *b,
                        int out_type, float *out);
/* MATMUL int path split over `threads` POSIX threads by (batch,row): used only
 * as the timed CPU reference arm, same arithmetic and loop order per row. */
void orc_matmul_int_mt(int64_t n, int64_t h, int64_t c, int64_t w, const int64_t *a,
                       const int64_t *b, int64_t a_zp, int64_t b_zp, int64_t *out, int threads);
void orc_matmul_float_mt(int64_t n, int64_t h, int64_t c, int64_t w, const float *a, const float *b,
                         int out_type, float *out, int threads);
void orc_conv2d_int_mt(const orc_conv_geom *g, const int64_t *input, const int64_t *weight,
                       const int64_t *bias, int64_t bias_len, int64_t input_zp, int64_t weight_zp,
                       int64_t *out, int threads);

/* RESCALE element loop, type_conv.rs:168-190 (validation is in oracle.py). */
int orc_rescale(const int64_t *input, int64_t count, int in_type, int out_type,
                const int64_t *multiplier, const int64_t *shift, int64_t channels,
                int64_t in_zp_raw, int64_t out_zp_raw, int scale32, int rounding_mode,
                int per_channel, int input_unsigned, int output_unsigned, int64_t *out);

/* Pool geometry (pool.rs:17-105). pad = [top, bottom, left, right]. */
typedef struct {
    int64_t n, ih, iw, c, oh, ow;
    int64_t kernel[2], stride[2];
    int64_t pad_top, pad_left;
} orc_pool_geom;

/* AVG_POOL2D int path pool.rs:186-214. Returns ORC_ERR_GRAPH on an
 * apply_scale_32 failure. */
int orc_avg_pool_int(const orc_pool_geom *g, const int64_t *input, int in_type,
                     int64_t in_zp, int64_t out_zp, int64_t *out);
/* AVG_POOL2D float path pool.rs:215-227: values rounded to acc_type, output
 * rounded to in_type. */
void orc_avg_pool_float(const orc_pool_geom *g, const float *input, int in_type, int acc_type,
                        float *out);
/* MAX_POOL2D pool.rs:262-284. */
void orc_max_pool_int(const orc_pool_geom *g, const int64_t *input, int in_type, int64_t *out);
void orc_max_pool_float(const orc_pool_geom *g, const float *input, int in_type, int nan_mode,
                        float *out);

/* CLAMP elementwise.rs:319-343. */
void orc_clamp_int(const int64_t *input, int64_t count, int64_t lo, int64_t hi, int64_t *out);
void orc_clamp_float(const float *input, int64_t count, float lo, float hi, int nan_mode,
                     int dtype, float *out);

/* ADD (int32 wrap) elementwise.rs:395-397 with `wrap` :138. */
void orc_add_int(const int64_t *a, const int64_t *b, int64_t count, int dtype, int64_t *out);

#ifdef __cplusplus
}
#endif
#endif
