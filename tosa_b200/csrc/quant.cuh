// Device-side TOSA fixed-point arithmetic: RESCALE (scale32 single/double
// rounding, scale16, inexact) and the float rounding used by the float
// convolution epilogue. Semantics follow the reference interpreter:
//   apply_scale_32   src/ops/quant.rs:17-32
//   apply_scale_16   src/ops/type_conv.rs:86-92
//   RESCALE element  src/ops/type_conv.rs:174-188
//   round_to         src/ops/common.rs:100-108 (round to nearest even)
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace tb {

// Error bits of the per-context device error word.
enum : uint32_t {
    DEV_ERR_SCALE = 1u,    // apply_scale range / int32 overflow (Error::GraphError)
    DEV_ERR_TIMEOUT = 2u,  // a bounded wait gave up
    DEV_ERR_INTERNAL = 4u,
};

// Rounding modes (schema RoundingMode enum).
enum : int { ROUND_SINGLE = 1, ROUND_INEXACT = 2, ROUND_DOUBLE = 3 };

// DType codes (schema DType enum).
enum : int {
    DT_BOOL = 1, DT_INT4 = 2, DT_INT8 = 3, DT_INT16 = 4, DT_INT32 = 5, DT_INT48 = 6,
    DT_FP32 = 7, DT_FP16 = 8, DT_BF16 = 9, DT_SHAPE = 10, DT_FP8E4M3 = 11, DT_FP8E5M2 = 12, DT_INT64 = 17,
};

// FP8 formats (src/float8.rs): E4M3 (bias 7, no infinities, NaN = exponent and
// mantissa all ones, overflow -> NaN) and E5M2 (bias 15, IEEE-style infinities
// and NaNs, overflow -> infinity). Decoding is exact.
__device__ __forceinline__ float fp8_decode(uint8_t bits, int dt) {
    const int man_bits = dt == DT_FP8E4M3 ? 3 : 2;
    const int bias = dt == DT_FP8E4M3 ? 7 : 15;
    const unsigned maxe = (1u << (7 - man_bits)) - 1u, manm = (1u << man_bits) - 1u;
    const unsigned e = (bits >> man_bits) & maxe, m = bits & manm;
    const bool has_inf = dt == DT_FP8E5M2;
    if (has_inf ? (e == maxe && m != 0) : (e == maxe && m == manm)) return __int_as_float(0x7fc00000);
    const float sign = (bits & 0x80) ? -1.f : 1.f;
    if (has_inf && e == maxe) return sign * __int_as_float(0x7f800000);
    // value = m * 2^(1 - bias - man_bits) (subnormal) or (2^man_bits + m) * 2^(e - bias - man_bits)
    const int expo = (e == 0 ? 1 : static_cast<int>(e)) - bias - man_bits;
    const float mant = static_cast<float>(e == 0 ? m : ((1u << man_bits) | m));
    return sign * mant * __int_as_float((127 + expo) << 23);
}

// Round-to-nearest-even encode with the format's overflow rule.
__device__ __forceinline__ uint8_t fp8_encode(float x, int dt) {
    const int man_bits = dt == DT_FP8E4M3 ? 3 : 2;
    const int bias = dt == DT_FP8E4M3 ? 7 : 15;
    const bool has_inf = dt == DT_FP8E5M2;
    const unsigned maxe = (1u << (7 - man_bits)) - 1u, manm = (1u << man_bits) - 1u;
    const uint8_t nanv = static_cast<uint8_t>((maxe << man_bits) | manm);
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return nanv;
    const uint8_t sign = (u >> 31) ? 0x80 : 0;
    const uint8_t overflow = has_inf ? static_cast<uint8_t>(sign | (maxe << man_bits)) : static_cast<uint8_t>(sign | nanv);
    if ((u & 0x7fffffffu) == 0x7f800000u) return overflow;
    const float a = __uint_as_float(u & 0x7fffffffu);
    if (a == 0.f) return sign;
    const int min_normal = 1 - bias;
    int e = static_cast<int>((u >> 23) & 0xff) - 127;  // f32 subnormals fall in the fp8 subnormal branch
    unsigned exp_field, man;
    if (e < min_normal) {
        // q = rint(a / 2^min_normal * 2^man_bits), exact scaling by a power of two
        const unsigned q = static_cast<unsigned>(rintf(a * __int_as_float((127 - min_normal + man_bits) << 23)));
        exp_field = q >> man_bits;
        man = q & manm;
    } else {
        unsigned q = static_cast<unsigned>(rintf(a * __int_as_float((127 - e + man_bits) << 23)));
        if (q == (2u << man_bits)) {
            e += 1;
            q = 1u << man_bits;
        }
        exp_field = static_cast<unsigned>(e + bias);
        man = q & manm;
    }
    const bool exceeded = has_inf ? (exp_field >= maxe) : (exp_field > maxe || (exp_field == maxe && man == manm));
    if (exceeded) return overflow;
    return static_cast<uint8_t>(sign | ((exp_field << man_bits) | man));
}

struct RescaleArgs {
    const int32_t* multiplier;  // [channels] (scale32: int32 values; scale16: int16 values widened)
    const int32_t* shift;       // [channels], widened from int8
    int per_channel;
    int scale32;
    int rounding;               // ROUND_*
    int32_t out_zp;             // already extended for an unsigned output
    int32_t lo, hi;             // output clamp range, intersected with a fused CLAMP
};

// General RESCALE of one value x = extend(v) - in_zp. Returns the clamped
// result; sets *err on the conditions where the reference returns Err.
__device__ __forceinline__ int64_t rescale_value(int64_t x, int32_t m, int32_t s, int rounding, int scale32,
                                                 int32_t out_zp, int32_t lo, int32_t hi, uint32_t* err) {
    int64_t scaled;
    if (rounding == ROUND_INEXACT) {
        // (f32(x) * f32(m)) * 2^-s, each product rounded to nearest, then
        // round-half-even to int32 with saturation (NaN -> 0).
        float t = __fmul_rn(__ll2float_rn(x), __int2float_rn(m));
        float p2 = __int_as_float((127 - s) << 23);  // exact 2^-s for s in [2, 62]
        t = __fmul_rn(t, p2);
        scaled = static_cast<int64_t>(__float2int_rn(t));
    } else if (scale32) {
        if (m < 0 || s < 2 || s > 62) { *err |= DEV_ERR_SCALE; return 0; }
        const int64_t half = static_cast<int64_t>(1) << (s - 1);
        const int32_t xv = static_cast<int32_t>(x);
        if (static_cast<int64_t>(xv) < -half || static_cast<int64_t>(xv) >= half) { *err |= DEV_ERR_SCALE; return 0; }
        int64_t round = half;
        if (rounding == ROUND_DOUBLE && s > 31) round += xv >= 0 ? (1ll << 30) : -(1ll << 30);
        scaled = (static_cast<int64_t>(xv) * m + round) >> s;
        if (scaled < INT32_MIN || scaled > INT32_MAX) { *err |= DEV_ERR_SCALE; return 0; }
    } else {
        const int16_t m16 = static_cast<int16_t>(m);
        if (m16 < 0 || s < 2 || s > 62) { *err |= DEV_ERR_SCALE; return 0; }
        scaled = (x * m16 + (static_cast<int64_t>(1) << (s - 1))) >> s;
        if (scaled < INT32_MIN || scaled > INT32_MAX) { *err |= DEV_ERR_SCALE; return 0; }
    }
    int64_t r = scaled + out_zp;
    if (r < INT32_MIN || r > INT32_MAX) { *err |= DEV_ERR_SCALE; return 0; }
    r = r < lo ? lo : r;
    r = r > hi ? hi : r;
    return r;
}

// Fast path for scale32 single/double rounding when the host has verified
// that every shift is >= 32 and every multiplier is non-negative: then every
// int32 input is in range and no intermediate can overflow, so the result is
// ((v * m + round) >> s) + out_zp, clamped.
__device__ __forceinline__ int32_t rescale_fast(int32_t v, int32_t m, int32_t s, int64_t round_pos, int double_round,
                                                int32_t out_zp, int32_t lo, int32_t hi) {
    int64_t round = round_pos;
    if (double_round && v < 0) round -= (1ll << 31);  // +2^30 for v >= 0, -2^30 otherwise
    int32_t r = static_cast<int32_t>((static_cast<int64_t>(v) * m + round) >> s) + out_zp;
    r = max(r, lo);
    r = min(r, hi);
    return r;
}

// Four int32 -> four saturated int8 in one word, v0 in the lowest byte
// (cvt.pack.sat: d = c << 16 | sat(a) << 8 | sat(b)).
__device__ __forceinline__ uint32_t pack4_sat_i8(int32_t v0, int32_t v1, int32_t v2, int32_t v3) {
    uint32_t t, d;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(t) : "r"(v3), "r"(v2), "r"(0));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(v1), "r"(v0), "r"(t));
    return d;
}

// The fast RESCALE of one value (every shift s in [33, 62], m >= 0, checked on the
// host): apply_scale_32's (v*m + 2^(s-1) [+-2^30]) >> s as the high word of
// v*m [+-2^30 by the sign of v] plus hz = 2^(s-33) (+ zp * 2^(s-32)), shifted by
// s - 32; |high word| <= 2^30 and |hz| < 2^30 keep the sum inside int32.
template <bool DBL>
__device__ __forceinline__ int32_t rescale_f2(int32_t v, int32_t m, int32_t sh, int32_t hz) {
    int32_t h;
    if (DBL) {
        // R = +2^30, or -2^30 for v < 0, as the 64-bit pair {lo, hi}:
        // hi = v >> 31 (sign), lo = (v & 2^31) ^ 2^30; then one wide multiply-add.
        asm("{\n\t"
            ".reg .b32 s, lo, dlo;\n\t"
            ".reg .b64 r, t;\n\t"
            "shr.s32 s, %1, 31;\n\t"
            "lop3.b32 lo, %1, 0x80000000, 0x40000000, 0x6a;\n\t"
            "mov.b64 r, {lo, s};\n\t"
            "mad.wide.s32 t, %1, %2, r;\n\t"
            "mov.b64 {dlo, %0}, t;\n\t"
            "}"
            : "=r"(h)
            : "r"(v), "r"(m));
    } else {
        h = __mulhi(v, m);
    }
    return (h + hz) >> sh;
}

// f32 -> dtype -> f32 rounding (round to nearest even).
__device__ __forceinline__ float round_to_dtype(float x, int dtype) {
    if (dtype == DT_BF16) return __bfloat162float(__float2bfloat16_rn(x));
    if (dtype == DT_FP16) return __half2float(__float2half_rn(x));
    if (dtype == DT_FP8E4M3 || dtype == DT_FP8E5M2) return fp8_decode(fp8_encode(x, dtype), dtype);
    return x;
}

}  // namespace tb
