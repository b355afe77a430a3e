// CUDA-core kernels of the backend:
//   * HBM-bound operators: DEPTHWISE_CONV2D, AVG_POOL2D, MAX_POOL2D, RESCALE,
//     CLAMP, ADD (vectorised over 4 channels where the layout allows);
//   * helpers of the tensor-core path: zero-point sums of weights / B columns
//     and the per-border-class column-term tables of a convolution plan;
//   * direct CONV2D / MATMUL for shapes the TMA tiles cannot address (channel
//     counts that are not multiples of 16 bytes, e.g. the conformance shapes
//     and RGB stems). These follow the reference's loop order, so the float
//     variants reproduce AccF32 bit for bit.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"
#include "quant.cuh"

namespace tb {

struct ConvGeomDev {
    int n, ih, iw, ic, oc, kh, kw, oh, ow, m;
    int pad_t, pad_l, sh, sw, dh, dw;
    int tr;  // TRANSPOSE_CONV2D: pad_t / pad_l are out_pad_top / out_pad_left
};

// Input row (or column) that output position o reads through tap k, or -1 when the tap
// reads nothing. CONV2D: o*s + k*d - pad inside [0, in) (src/ops/conv.rs:160-170).
// TRANSPOSE_CONV2D (tr; conv.rs:345-362, gather form): (o - out_pad - k) / s when the
// division is exact and the quotient lies inside [0, in).
__device__ __forceinline__ int tap_src(int o, int k, int s, int d, int pad, int in, int tr) {
    if (tr) {
        const int v = o - pad - k;
        return (v < 0 || v >= in * s || v % s != 0) ? -1 : v / s;
    }
    const int v = o * s + k * d - pad;
    return (v < 0 || v >= in) ? -1 : v;
}

// TRANSPOSE_CONV2D with stride 1 as a CONV2D: weights [oc][kh][kw][ic] with the taps
// reversed in both spatial dimensions (one byte per value: INT8, or INT4 held in bytes).
__global__ void flip_taps_i8(int oc, int kh, int kw, int ic, const int8_t* __restrict__ w, int8_t* __restrict__ out) {
    const long long total = static_cast<long long>(oc) * kh * kw * ic;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % ic);
        long long r = i / ic;
        const int kx = static_cast<int>(r % kw);
        r /= kw;
        const int ky = static_cast<int>(r % kh);
        const long long o = r / kh;
        out[i] = w[((o * kh + (kh - 1 - ky)) * kw + (kw - 1 - kx)) * ic + c];
    }
}

// Integer result of a contraction -> optional RESCALE -> store.
struct IntEpiDev {
    int rescale;          // 0: store int32, 1: RESCALE
    RescaleArgs rs;
    int out_dtype;
};

__device__ __forceinline__ void store_int(void* out, long long idx, int dtype, int32_t v) {
    if (dtype == DT_INT8) static_cast<int8_t*>(out)[idx] = static_cast<int8_t>(v);
    else if (dtype == DT_INT16) static_cast<int16_t*>(out)[idx] = static_cast<int16_t>(v);
    else static_cast<int32_t*>(out)[idx] = v;
}

__device__ __forceinline__ void finish_int(const IntEpiDev& e, int32_t v, int ch, void* out, long long idx,
                                           uint32_t* err) {
    if (!e.rescale) {
        static_cast<int32_t*>(out)[idx] = v;
        return;
    }
    const int c = e.rs.per_channel ? ch : 0;
    const int64_t r = rescale_value(v, e.rs.multiplier[c], e.rs.shift[c], e.rs.rounding, e.rs.scale32, e.rs.out_zp,
                                    e.rs.lo, e.rs.hi, err);
    store_int(out, idx, e.out_dtype, static_cast<int32_t>(r));
}

__device__ __forceinline__ float load_f(const void* p, long long i, int dt) {
    if (dt == DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    if (dt == DT_FP16) return __half2float(static_cast<const __half*>(p)[i]);
    if (dt == DT_FP8E4M3 || dt == DT_FP8E5M2) return fp8_decode(static_cast<const uint8_t*>(p)[i], dt);
    return static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_f(void* p, long long i, int dt, float v) {
    if (dt == DT_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else if (dt == DT_FP16) static_cast<__half*>(p)[i] = __float2half_rn(v);
    else if (dt == DT_FP8E4M3 || dt == DT_FP8E5M2) static_cast<uint8_t*>(p)[i] = fp8_encode(v, dt);
    else static_cast<float*>(p)[i] = v;
}

// One multiply-accumulate in the reference's accumulator types (src/ops/accum.rs):
// acc_dt FP32 -> acc + a*b (product and sum each rounded to f32, no fused
// multiply-add); FP16 / BF16 -> the product rounded to the accumulator type, then
// the sum rounded to it (`acc += a * b`); with unrounded_product (MATMUL's
// `acc = acc + a * b`) only the sum is rounded.
__device__ __forceinline__ float mac_acc(float acc, float a, float b, int acc_dt, bool unrounded_product = false) {
    if (acc_dt == DT_FP32) return __fadd_rn(acc, __fmul_rn(a, b));
    const float p = unrounded_product ? __fmul_rn(a, b) : round_to_dtype(__fmul_rn(a, b), acc_dt);
    return round_to_dtype(__fadd_rn(acc, p), acc_dt);
}

// ---------------------------------------------------------------------------
// Direct CONV2D (one thread per output element), reference loop order
// (src/ops/conv.rs:147-181): taps row-major, ic innermost.
// ---------------------------------------------------------------------------
__global__ void conv2d_direct_int(ConvGeomDev g, const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                  const int32_t* __restrict__ bias, int bias_len, int32_t zx, int32_t zw,
                                  IntEpiDev e, void* out, uint32_t* err) {
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.oc;
    uint32_t lerr = 0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int oc = static_cast<int>(i % g.oc);
        long long r = i / g.oc;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        uint32_t acc = 0;
        for (int ky = 0; ky < g.kh; ++ky) {
            const int y = tap_src(oy, ky, g.sh, g.dh, g.pad_t, g.ih, g.tr);
            if (y < 0) continue;
            for (int kx = 0; kx < g.kw; ++kx) {
                const int xx = tap_src(ox, kx, g.sw, g.dw, g.pad_l, g.iw, g.tr);
                if (xx < 0) continue;
                const int8_t* xp = x + ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.ic;
                const int8_t* wp = w + ((static_cast<long long>(oc) * g.kh + ky) * g.kw + kx) * g.ic;
                for (int c = 0; c < g.ic; ++c)
                    acc += static_cast<uint32_t>(static_cast<int32_t>(xp[c]) - zx) *
                           static_cast<uint32_t>(static_cast<int32_t>(wp[c]) - zw);
            }
        }
        acc += static_cast<uint32_t>(bias[bias_len == 1 ? 0 : oc]);
        finish_int(e, static_cast<int32_t>(acc), oc, out, i, &lerr);
    }
    if (lerr) atomicOr(err, lerr);
}

__global__ void conv2d_direct_float(ConvGeomDev g, const void* __restrict__ x, const void* __restrict__ w,
                                    const void* __restrict__ bias, int bias_len, int in_dt, int w_dt, int acc_dt,
                                    int out_dt, void* out) {
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.oc;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int oc = static_cast<int>(i % g.oc);
        long long r = i / g.oc;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        float acc = 0.f;
        for (int ky = 0; ky < g.kh; ++ky) {
            const int y = tap_src(oy, ky, g.sh, g.dh, g.pad_t, g.ih, g.tr);
            if (y < 0) continue;
            for (int kx = 0; kx < g.kw; ++kx) {
                const int xx = tap_src(ox, kx, g.sw, g.dw, g.pad_l, g.iw, g.tr);
                if (xx < 0) continue;
                const long long xb = ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.ic;
                const long long wb = ((static_cast<long long>(oc) * g.kh + ky) * g.kw + kx) * g.ic;
                for (int c = 0; c < g.ic; ++c)
                    acc = mac_acc(acc, load_f(x, xb + c, in_dt), load_f(w, wb + c, w_dt), acc_dt);
            }
        }
        const float bv = load_f(bias, bias_len == 1 ? 0 : oc, out_dt);
        store_f(out, i, out_dt, round_to_dtype(__fadd_rn(round_to_dtype(acc, out_dt), bv), out_dt));
    }
}

// ---------------------------------------------------------------------------
// im2col for convolutions whose input channels are too few for the im2col TMA
// boxes (an RGB stem): rows [N*OH*OW][kp], one segment of segp bytes per filter
// row ky (its KW taps x IC channels in weight order, padded to whole 32-bit
// words), padded taps and all padding filled with the input zero point, so that
// (x - zx) is 0 there and a 1x1 tensor-core convolution over the rows yields the
// reference's sum over valid taps. The weights are laid out to match
// (pad_weight_segments_i8).
// ---------------------------------------------------------------------------
__global__ void im2col_rows_i8(ConvGeomDev g, const int8_t* __restrict__ x, int segp, int kp, int8_t zx,
                               int8_t* __restrict__ rows) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    // One thread per output pixel assembles its row in shared memory, then the
    // block writes its rows out with 16-byte stores.
    extern __shared__ __align__(16) int8_t srow[];
    const long long m_total = static_cast<long long>(g.n) * g.oh * g.ow;
    const int chunks = kp >> 4;
    for (long long m0 = static_cast<long long>(blockIdx.x) * blockDim.x; m0 < m_total;
         m0 += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long m = m0 + threadIdx.x;
        int8_t* my = srow + threadIdx.x * kp;
        if (m < m_total) {
            const int ox = static_cast<int>(m % g.ow);
            const long long r = m / g.ow;
            const int oy = static_cast<int>(r % g.oh);
            const int b = static_cast<int>(r / g.oh);
            const int8_t* xb = x + static_cast<long long>(b) * g.ih * g.iw * g.ic;
            for (int k = 0; k < kp; ++k) my[k] = zx;
            for (int ky = 0; ky < g.kh; ++ky) {
                const int y = oy * g.sh + ky * g.dh - g.pad_t;
                if (y < 0 || y >= g.ih) continue;
                for (int kx = 0; kx < g.kw; ++kx) {
                    const int xx = ox * g.sw + kx * g.dw - g.pad_l;
                    if (xx < 0 || xx >= g.iw) continue;
                    const int8_t* src = xb + (static_cast<long long>(y) * g.iw + xx) * g.ic;
                    for (int c = 0; c < g.ic; ++c) my[ky * segp + kx * g.ic + c] = __ldg(src + c);
                }
            }
        }
        __syncthreads();
        // cooperative copy of the block's rows: rows are contiguous in global memory
        const long long rows_here = m_total - m0 < blockDim.x ? m_total - m0 : blockDim.x;
        const int vecs = static_cast<int>(rows_here) * chunks;
        uint4* dst = reinterpret_cast<uint4*>(rows + m0 * kp);
        const uint4* s4 = reinterpret_cast<const uint4*>(srow);
        for (int v = threadIdx.x; v < vecs; v += blockDim.x) dst[v] = s4[v];
        __syncthreads();
    }
}

// The rows of a 1x1 convolution (IC % 4 == 0, kp a multiple of 16): the pixel's IC channels
// then the input zero point up to kp bytes; a pixel outside the input (padding) is a row of
// the zero point. One thread per 16-byte chunk of a row: word loads of the pixel, one 16-byte
// store, both contiguous across the threads of a warp.
__global__ void im2col_rows_1x1_i8(ConvGeomDev g, const uint32_t* __restrict__ x, int kp, uint32_t zxw,
                                   uint4* __restrict__ rows) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    const int icw = g.ic >> 2, chunks = kp >> 4;
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * chunks;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long m = i / chunks;
        const int q = static_cast<int>(i - m * chunks);
        const int ox = static_cast<int>(m % g.ow);
        const long long r = m / g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const long long b = r / g.oh;
        const int y = oy * g.sh - g.pad_t, xx = ox * g.sw - g.pad_l;
        uint32_t w[4] = {zxw, zxw, zxw, zxw};
        if (static_cast<unsigned>(y) < static_cast<unsigned>(g.ih) && static_cast<unsigned>(xx) < static_cast<unsigned>(g.iw)) {
            const uint32_t* src = x + ((b * g.ih + y) * g.iw + xx) * icw;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (4 * q + k < icw) w[k] = __ldg(src + 4 * q + k);
        }
        rows[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// The same rows for the common stems (IC channels, a square K x K window known at compile
// time, no horizontal dilation): a filter row's K * IC input bytes are contiguous, so an
// interior segment is read as the aligned 32-bit words covering it and funnel-shifted into
// place (word loads instead of byte ones); segments touching the image border take bytes
// one by one. The row (kp = KPW * 4 bytes, fixed by IC and K) is assembled in registers with
// the filter rows unrolled, so all of a pixel's loads are in flight together, and staged in
// shared memory with 16-byte stores: rows of 11 such chunks (the 7x7 RGB stem) put the 8
// lanes of each store phase in 8 distinct bank groups, where word stores were 4-way
// conflicts.

// Row bytes of im2col_rows_i8_t<IC, K>: K segments of whole words, rounded up to 16 bytes
// (the plan's kp for these shapes).
__host__ __device__ constexpr int im2col_t_kp(int ic, int k) { return (k * ((k * ic + 3) / 4) + 3) / 4 * 16; }

template <int IC, int KW>
__global__ void __launch_bounds__(128) im2col_rows_i8_t(ConvGeomDev g, const int8_t* __restrict__ x,
                                                         long long x_bytes, int8_t zx, int8_t* __restrict__ rows) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    constexpr int L = KW * IC, LW = (L + 3) / 4;      // segment bytes and words (the segment pitch)
    constexpr int KPW = (KW * LW + 3) / 4 * 4;        // words per row: whole 16-byte chunks
    constexpr int kp = KPW * 4;
    static_assert(kp == im2col_t_kp(IC, KW), "row layout");
    extern __shared__ __align__(16) int8_t srow[];
    const long long m_total = static_cast<long long>(g.n) * g.oh * g.ow;
    const uint32_t fill = static_cast<uint8_t>(zx) * 0x01010101u;
    for (long long m0 = static_cast<long long>(blockIdx.x) * blockDim.x; m0 < m_total;
         m0 += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long m = m0 + threadIdx.x;
        if (m < m_total) {
            const int ox = static_cast<int>(m % g.ow);
            const long long r = m / g.ow;
            const int oy = static_cast<int>(r % g.oh);
            const int b = static_cast<int>(r / g.oh);
            const long long xb = static_cast<long long>(b) * g.ih * g.iw * IC;
            const int x0 = ox * g.sw - g.pad_l;
            const bool x_in = x0 >= 0 && x0 + KW <= g.iw;
            uint32_t row[KPW];
#pragma unroll
            for (int k = KW * LW; k < KPW; ++k) row[k] = fill;
#pragma unroll
            for (int ky = 0; ky < KW; ++ky) {
                const int y = oy * g.sh + ky * g.dh - g.pad_t;
                const long long a = xb + (static_cast<long long>(y) * g.iw + x0) * IC;  // first byte
                const long long a0 = a & ~3ll;
                if (y >= 0 && y < g.ih && x_in && a0 + 4 * (LW + 1) <= x_bytes) {
                    const uint32_t* w = reinterpret_cast<const uint32_t*>(x + a0);
                    uint32_t in[LW + 1];
#pragma unroll
                    for (int j = 0; j <= LW; ++j) in[j] = __ldg(w + j);
                    const uint32_t sh = static_cast<uint32_t>(a - a0) * 8;
#pragma unroll
                    for (int j = 0; j < LW; ++j) {
                        uint32_t v = __funnelshift_r(in[j], in[j + 1], sh);
                        if (4 * j + 4 > L) {  // the segment's last word: bytes past it hold zx
                            const uint32_t keep = 0xffffffffu >> (8 * (4 * j + 4 - L));
                            v = (v & keep) | (fill & ~keep);
                        }
                        row[ky * LW + j] = v;
                    }
                } else {
                    const bool yok = y >= 0 && y < g.ih;
#pragma unroll
                    for (int j = 0; j < LW; ++j) {
                        uint32_t v = 0;
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int i = 4 * j + q, kx = i / IC;
                            const bool ok = i < L && yok && x0 + kx >= 0 && x0 + kx < g.iw;
                            const uint32_t byte = ok ? static_cast<uint8_t>(__ldg(x + a + i)) : static_cast<uint8_t>(zx);
                            v |= byte << (8 * q);
                        }
                        row[ky * LW + j] = v;
                    }
                }
            }
            uint4* my = reinterpret_cast<uint4*>(srow + threadIdx.x * kp);
#pragma unroll
            for (int c = 0; c < KPW / 4; ++c) my[c] = make_uint4(row[4 * c], row[4 * c + 1], row[4 * c + 2], row[4 * c + 3]);
        }
        __syncthreads();
        const long long rows_here = m_total - m0 < blockDim.x ? m_total - m0 : blockDim.x;
        const int vecs = static_cast<int>(rows_here) * (KPW / 4);
        uint4* dst = reinterpret_cast<uint4*>(rows + m0 * kp);
        const uint4* s4 = reinterpret_cast<const uint4*>(srow);
        for (int v = threadIdx.x; v < vecs; v += blockDim.x) dst[v] = s4[v];
        __syncthreads();
    }
}

// Weights [oc][KH][KW*IC] -> [oc][kp] in the rows' layout: segment ky at ky * segp,
// zeros in the padding (the rows hold the input zero point there, so any weight
// value gives (x - zx) * (w - zw) = 0).
__global__ void pad_weight_segments_i8(int oc, int kh, int seg, int segp, int kp, const int8_t* __restrict__ w,
                                       int8_t* __restrict__ out) {
    const long long total = static_cast<long long>(oc) * kp;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(i % kp);
        const long long o = i / kp;
        const int ky = col / segp, j = col - ky * segp;
        out[i] = (ky < kh && j < seg) ? w[(o * kh + ky) * seg + j] : 0;
    }
}

// Weights [OC][K] -> [OC][kp], zero-padded.
__global__ void pad_weight_rows_i8(int oc, int k, int kp, const int8_t* __restrict__ w, int8_t* __restrict__ out) {
    const long long total = static_cast<long long>(oc) * kp;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(i % kp);
        const long long row = i / kp;
        out[i] = col < k ? w[row * k + col] : 0;
    }
}

// Column terms of a constant MATMUL B [n][c][w]: out[bn][x] = scale * sum_c B[bn][c][x] + add
// (int32 wrap-around, as the in-GEMM column-sum job). Block (32, 8): 32 columns, 8 row
// slices reduced in shared memory; grid (ceil(w / 32), n).
__global__ void colterm_const_i8(int c, int w, const int8_t* __restrict__ b, int32_t scale, int32_t add,
                                 int32_t* __restrict__ out) {
    __shared__ int32_t part[8][33];
    const int x = blockIdx.x * 32 + threadIdx.x, bn = blockIdx.y;
    int32_t sum = 0;
    if (x < w)
        for (int k = threadIdx.y; k < c; k += 8) sum += b[(static_cast<long long>(bn) * c + k) * w + x];
    part[threadIdx.y][threadIdx.x] = sum;
    __syncthreads();
    if (threadIdx.y == 0 && x < w) {
        int32_t t = 0;
#pragma unroll
        for (int r = 0; r < 8; ++r) t += part[r][threadIdx.x];
        out[static_cast<long long>(bn) * w + x] =
            static_cast<int32_t>(static_cast<uint32_t>(scale) * static_cast<uint32_t>(t) + static_cast<uint32_t>(add));
    }
}

// Column terms of MATMUL_T's B [d][w][c] (K-major rows, c % 16 == 0): out[r] = scale *
// sum_k B[r][k] + add for the d*w rows r. One warp per row, 16-byte loads. Releases its
// dependent launch at once: the GEMM reading `out` waits for it only in its epilogue.
__global__ void __launch_bounds__(256) colterm_rows_i8(long long rows, int c, const int8_t* __restrict__ b,
                                                       int32_t scale, int32_t add, int32_t* __restrict__ out) {
    grid_launch_dependents();
    const int lane = threadIdx.x & 31;
    const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
        const int4* row = reinterpret_cast<const int4*>(b + r * c);
        int sum = 0;
        for (int j = lane; j < (c >> 4); j += 32) {
            const int4 v = row[j];
            sum = __dp4a(v.x, 0x01010101, sum);
            sum = __dp4a(v.y, 0x01010101, sum);
            sum = __dp4a(v.z, 0x01010101, sum);
            sum = __dp4a(v.w, 0x01010101, sum);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0)
            out[r] = static_cast<int32_t>(static_cast<uint32_t>(scale) * static_cast<uint32_t>(sum) +
                                          static_cast<uint32_t>(add));
    }
}

// ---------------------------------------------------------------------------
// CONV3D (src/ops/conv.rs:147-181, ConvNd with three spatial dimensions), one thread per
// output element in the reference's order: taps (kd, kh, kw) row-major, ic innermost.
// Input NDHWC, weight [oc, kd, kh, kw, ic]. INT16 x INT8 -> INT48 needs clamp48 (below).
// ---------------------------------------------------------------------------
struct Conv3GeomDev {
    int n, id, ih, iw, ic, oc, kd, kh, kw, od, oh, ow;
    int pd, pt, pl, sd, sh, sw, dd, dh, dw;  // front / top / left pad, strides, dilations
};

// Visits the taps of output element i that read inside the input: f(input offset, weight
// offset) per tap, in the reference's order; returns the output channel.
template <class F>
__device__ __forceinline__ int conv3_taps(const Conv3GeomDev& g, long long i, F f) {
    const int oc = static_cast<int>(i % g.oc);
    long long r = i / g.oc;
    const int ox = static_cast<int>(r % g.ow);
    r /= g.ow;
    const int oy = static_cast<int>(r % g.oh);
    r /= g.oh;
    const int oz = static_cast<int>(r % g.od);
    const long long b = r / g.od;
    for (int kz = 0; kz < g.kd; ++kz) {
        const int z = oz * g.sd + kz * g.dd - g.pd;
        if (z < 0 || z >= g.id) continue;
        for (int ky = 0; ky < g.kh; ++ky) {
            const int y = oy * g.sh + ky * g.dh - g.pt;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kw; ++kx) {
                const int x = ox * g.sw + kx * g.dw - g.pl;
                if (x < 0 || x >= g.iw) continue;
                f((((b * g.id + z) * g.ih + y) * g.iw + x) * g.ic,
                  (((static_cast<long long>(oc) * g.kd + kz) * g.kh + ky) * g.kw + kx) * g.ic);
            }
        }
    }
    return oc;
}

__global__ void conv3d_direct_int(Conv3GeomDev g, const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                  const int32_t* __restrict__ bias, int bias_len, int32_t zx, int32_t zw,
                                  IntEpiDev e, void* out, uint32_t* err) {
    const long long total = static_cast<long long>(g.n) * g.od * g.oh * g.ow * g.oc;
    uint32_t lerr = 0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        uint32_t acc = 0;
        const int oc = conv3_taps(g, i, [&](long long xb, long long wb) {
            for (int c = 0; c < g.ic; ++c)
                acc += static_cast<uint32_t>(static_cast<int32_t>(x[xb + c]) - zx) *
                       static_cast<uint32_t>(static_cast<int32_t>(w[wb + c]) - zw);
        });
        acc += static_cast<uint32_t>(bias[bias_len == 1 ? 0 : oc]);
        finish_int(e, static_cast<int32_t>(acc), oc, out, i, &lerr);
    }
    if (lerr) atomicOr(err, lerr);
}

__global__ void conv3d_direct_float(Conv3GeomDev g, const void* __restrict__ x, const void* __restrict__ w,
                                    const void* __restrict__ bias, int bias_len, int in_dt, int w_dt, int acc_dt,
                                    int out_dt, void* out) {
    const long long total = static_cast<long long>(g.n) * g.od * g.oh * g.ow * g.oc;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        float acc = 0.f;
        const int oc = conv3_taps(g, i, [&](long long xb, long long wb) {
            for (int c = 0; c < g.ic; ++c) acc = mac_acc(acc, load_f(x, xb + c, in_dt), load_f(w, wb + c, w_dt), acc_dt);
        });
        const float bv = load_f(bias, bias_len == 1 ? 0 : oc, out_dt);
        store_f(out, i, out_dt, round_to_dtype(__fadd_rn(round_to_dtype(acc, out_dt), bv), out_dt));
    }
}

// INT16 x INT8 -> INT48 (AccI64, src/ops/accum.rs:43-56): int64 accumulation,
// bias added with wrap-around, then clamped to 48 bits (src/ops/conv.rs:466-470).
// INT48 values are stored as int64. depthwise: weight [KH,KW,C,M].
__device__ __forceinline__ int64_t clamp48(int64_t v) {
    const int64_t lo = -(1ll << 47), hi = (1ll << 47) - 1;
    return v < lo ? lo : (v > hi ? hi : v);
}

__global__ void conv3d_direct_i48(Conv3GeomDev g, const int16_t* __restrict__ x, const int8_t* __restrict__ w,
                                  const int64_t* __restrict__ bias, int bias_len, int32_t zx, int32_t zw,
                                  int64_t* __restrict__ out) {
    const long long total = static_cast<long long>(g.n) * g.od * g.oh * g.ow * g.oc;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        uint64_t acc = 0;
        const int oc = conv3_taps(g, i, [&](long long xb, long long wb) {
            for (int c = 0; c < g.ic; ++c)
                acc += static_cast<uint64_t>((static_cast<int64_t>(x[xb + c]) - zx) *
                                             (static_cast<int64_t>(w[wb + c]) - zw));
        });
        acc += static_cast<uint64_t>(bias[bias_len == 1 ? 0 : oc]);
        out[i] = clamp48(static_cast<int64_t>(acc));
    }
}

__global__ void conv2d_direct_i48(ConvGeomDev g, const int16_t* __restrict__ x, const int8_t* __restrict__ w,
                                  const int64_t* __restrict__ bias, int bias_len, int32_t zx, int32_t zw,
                                  int depthwise, int64_t* __restrict__ out) {
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.oc;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int oc = static_cast<int>(i % g.oc);
        long long r = i / g.oc;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        uint64_t acc = 0;
        for (int ky = 0; ky < g.kh; ++ky) {
            const int y = tap_src(oy, ky, g.sh, g.dh, g.pad_t, g.ih, g.tr);
            if (y < 0) continue;
            for (int kx = 0; kx < g.kw; ++kx) {
                const int xx = tap_src(ox, kx, g.sw, g.dw, g.pad_l, g.iw, g.tr);
                if (xx < 0) continue;
                const int16_t* xp = x + ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.ic;
                if (depthwise) {
                    const int c = oc / g.m, mm = oc % g.m;
                    const int64_t wv = w[((ky * g.kw + kx) * g.ic + c) * g.m + mm] - zw;
                    acc += static_cast<uint64_t>((static_cast<int64_t>(xp[c]) - zx) * wv);
                } else {
                    const int8_t* wp = w + ((static_cast<long long>(oc) * g.kh + ky) * g.kw + kx) * g.ic;
                    for (int c = 0; c < g.ic; ++c)
                        acc += static_cast<uint64_t>((static_cast<int64_t>(xp[c]) - zx) *
                                                     (static_cast<int64_t>(wp[c]) - zw));
                }
            }
        }
        acc += static_cast<uint64_t>(bias[bias_len == 1 ? 0 : oc]);
        out[i] = clamp48(static_cast<int64_t>(acc));
    }
}

// Offset of B's element (k, col) for batch bn: MATMUL's B is [n,c,w]; MATMUL_T's (bt) is
// [d,w,c] (src/ops/matmul.rs:75-78), its one batch broadcast over every bn when bb.
__device__ __forceinline__ long long mm_b_index(int bn, int k, int col, int c, int w, int bt, int bb) {
    const long long nb = bb ? 0 : bn;
    return bt ? (nb * w + col) * c + k : (nb * c + k) * w + col;
}

__global__ void matmul_direct_i48(int n, int h, int c, int w, const int16_t* __restrict__ a,
                                  const int16_t* __restrict__ bm, int bt, int bb, int64_t* __restrict__ out) {
    const long long total = static_cast<long long>(n) * h * w;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(i % w);
        const long long rowi = i / w;
        const int bn = static_cast<int>(rowi / h);
        uint64_t acc = 0;
        for (int k = 0; k < c; ++k)
            acc += static_cast<uint64_t>(static_cast<int64_t>(a[rowi * c + k]) * bm[mm_b_index(bn, k, col, c, w, bt, bb)]);
        out[i] = clamp48(static_cast<int64_t>(acc));
    }
}

// ---------------------------------------------------------------------------
// DEPTHWISE_CONV2D (src/ops/conv.rs:234-266). HBM-bound: one thread computes
// 4 consecutive output channels of one output pixel when m == 1 and c % 4 == 0
// (char4 loads of activations and weights), else one channel.
// ---------------------------------------------------------------------------
__global__ void depthwise_int_vec4(ConvGeomDev g, const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                   const int32_t* __restrict__ bias, int bias_len, int32_t zx, int32_t zw,
                                   IntEpiDev e, void* out, uint32_t* err) {
    const int cg = g.ic >> 2;
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * cg;
    uint32_t lerr = 0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c4 = static_cast<int>(i % cg) * 4;
        long long r = i / cg;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        uint32_t acc[4] = {0, 0, 0, 0};
        const int iy0 = oy * g.sh - g.pad_t, ix0 = ox * g.sw - g.pad_l;
        for (int ky = 0; ky < g.kh; ++ky) {
            const int y = iy0 + ky * g.dh;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kw; ++kx) {
                const int xx = ix0 + kx * g.dw;
                if (xx < 0 || xx >= g.iw) continue;
                const char4 xv = __ldg(reinterpret_cast<const char4*>(
                    x + ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.ic + c4));
                const char4 wv = __ldg(reinterpret_cast<const char4*>(w + (ky * g.kw + kx) * g.ic + c4));
                acc[0] += static_cast<uint32_t>(xv.x - zx) * static_cast<uint32_t>(wv.x - zw);
                acc[1] += static_cast<uint32_t>(xv.y - zx) * static_cast<uint32_t>(wv.y - zw);
                acc[2] += static_cast<uint32_t>(xv.z - zx) * static_cast<uint32_t>(wv.z - zw);
                acc[3] += static_cast<uint32_t>(xv.w - zx) * static_cast<uint32_t>(wv.w - zw);
            }
        }
        const long long o = ((static_cast<long long>(b) * g.oh + oy) * g.ow + ox) * g.ic + c4;
        if (e.rescale && e.out_dtype == DT_INT8) {
            char4 ov;
            int32_t rv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ch = c4 + k;
                const int32_t v = static_cast<int32_t>(acc[k] + static_cast<uint32_t>(bias[bias_len == 1 ? 0 : ch]));
                const int pc = e.rs.per_channel ? ch : 0;
                rv[k] = static_cast<int32_t>(rescale_value(v, e.rs.multiplier[pc], e.rs.shift[pc], e.rs.rounding,
                                                           e.rs.scale32, e.rs.out_zp, e.rs.lo, e.rs.hi, &lerr));
            }
            ov.x = static_cast<signed char>(rv[0]);
            ov.y = static_cast<signed char>(rv[1]);
            ov.z = static_cast<signed char>(rv[2]);
            ov.w = static_cast<signed char>(rv[3]);
            *reinterpret_cast<char4*>(static_cast<int8_t*>(out) + o) = ov;
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ch = c4 + k;
                const int32_t v = static_cast<int32_t>(acc[k] + static_cast<uint32_t>(bias[bias_len == 1 ? 0 : ch]));
                finish_int(e, v, ch, out, o + k, &lerr);
            }
        }
    }
    if (lerr) atomicOr(err, lerr);
}

// DEPTHWISE_CONV2D int8 with multiplier 1, channels a multiple of 4 and no horizontal
// dilation: one thread computes 4 channels (one input word) of kDwPix consecutive output
// pixels of a row, with dp2a (two 16-bit x 8-bit products) doing the multiplies. The weight
// table wm is built on the host when the plan is created: for tap t and channel c, word
// (t, c) holds w[t][c] - weight_zp (up to 9 bits) as a 16-bit lane, lane c % 2, the other
// lane zero; dp2a.lo against an input word then adds exactly channel c's product for
// c % 4 < 2 (input bytes 0 and 1) and dp2a.hi for c % 4 >= 2. Taps that fall outside the input
// read the input zero point zx instead of being skipped, and
// bias2[c] = bias[c] - zx * sum_t (w[t][c] - weight_zp) takes those terms back out:
//   sum over valid taps of (x - zx)(w - zw) = sum over all taps of x~ (w - zw) - zx sum_t (w - zw).
struct DwGeom {
    int ih, iw, c4, oh, ow, kh;
    int pad_t, pad_l, sh, dh;
    int chunks;  // channel chunks of blockDim.x words per pixel group
    int rows;    // output rows per block (strip kernel)
};

// Epilogue of the dp2a depthwise kernel: the general RESCALE (per value) or the fast form
// of rescale_f2 with the plan's fq arrays (per channel when per_channel, else entry 0).
struct DwEpi {
    IntEpiDev gen;
    const int32_t* fq_m;
    const int32_t* fq_sh;
    const int32_t* fq_hz;
    int per_channel;
    int32_t zp_add;  // the output zero point when it is not folded into fq_hz (or sr_c)
    int32_t lo, hi;
    // small-range form (strip kernel, epilogue kinds 3 and 4; the table pre-scaled by 2^k):
    // r = (mad.hi(v, m, c [- k2 if v < 0])) >> sh, per channel sh and c (padded to 256)
    const int32_t* sr_sh;
    const int32_t* sr_c;
    int32_t k2;
};

constexpr int kDwPix = 4;

// Multiply-accumulates of one thread's K x K window (rows ky, columns kx) into acc. CHECK:
// the window may cross the input's border (positions outside read the zero-point word).
template <int K, int SW, bool CHECK>
__device__ __forceinline__ void dw_window(int (&acc)[kDwPix][4], const uint32_t* __restrict__ xb,
                                          const uint4* __restrict__ wb, long long row_step, int cw, int iy0,
                                          int dh, int ih, uint32_t colmask, uint32_t zxw) {
    constexpr int P = kDwPix;
    constexpr int NC = (P - 1) * SW + K;
    int coff[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) coff[j] = j * cw;
#pragma unroll
    for (int ky = 0; ky < K; ++ky) {
        const uint32_t* xr = xb + ky * row_step;
        const bool row_ok = !CHECK || static_cast<unsigned>(iy0 + ky * dh) < static_cast<unsigned>(ih);
        uint32_t xw[NC];
#pragma unroll
        for (int j = 0; j < NC; ++j) {
            if (CHECK) xw[j] = (row_ok && ((colmask >> j) & 1u)) ? __ldg(xr + coff[j]) : zxw;
            else xw[j] = __ldg(xr + coff[j]);
        }
        uint4 wq[K];
#pragma unroll
        for (int kx = 0; kx < K; ++kx) wq[kx] = __ldg(wb + (ky * K + kx) * cw);
#pragma unroll
        for (int p = 0; p < P; ++p)
#pragma unroll
            for (int kx = 0; kx < K; ++kx) {
                const int xv = static_cast<int>(xw[p * SW + kx]);
                acc[p][0] = __dp2a_lo(static_cast<int>(wq[kx].x), xv, acc[p][0]);
                acc[p][1] = __dp2a_lo(static_cast<int>(wq[kx].y), xv, acc[p][1]);
                acc[p][2] = __dp2a_hi(static_cast<int>(wq[kx].z), xv, acc[p][2]);
                acc[p][3] = __dp2a_hi(static_cast<int>(wq[kx].w), xv, acc[p][3]);
            }
    }
}

// K x K window (K = 3 or 5), horizontal stride SW. EK: 0 general epilogue (any output type),
// 1 fast RESCALE to int8 with single rounding, 2 fast RESCALE to int8 with double rounding.
template <int K, int SW, int EK>
__global__ void depthwise_i8_dp2a(DwGeom g, const uint32_t* __restrict__ x, const uint4* __restrict__ wm,
                                  const int32_t* __restrict__ bias2, uint32_t zxw, DwEpi e, void* out,
                                  uint32_t* err) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    constexpr int P = kDwPix;
    constexpr int NC = (P - 1) * SW + K;  // input columns under P output pixels
    const int c4 = (blockIdx.x % g.chunks) * blockDim.x + threadIdx.x;
    const int ox0 = ((blockIdx.x / g.chunks) * blockDim.y + threadIdx.y) * P;
    if (c4 >= g.c4 || ox0 >= g.ow) return;
    const int oy = blockIdx.y, b = blockIdx.z;
    const int cw = g.c4;
    const int iy0 = oy * g.sh - g.pad_t, ix0 = ox0 * SW - g.pad_l;
    // the accumulators start from the bias (with the input zero point's terms taken out)
    const int4 bz = __ldg(reinterpret_cast<const int4*>(bias2) + c4);
    int acc[P][4];
#pragma unroll
    for (int p = 0; p < P; ++p) {
        acc[p][0] = bz.x;
        acc[p][1] = bz.y;
        acc[p][2] = bz.z;
        acc[p][3] = bz.w;
    }
    // word (b, iy0, ix0, c4); only positions inside the input are read through it
    const long long base = ((static_cast<long long>(b) * g.ih + iy0) * g.iw + ix0) * cw + c4;
    const long long row_step = static_cast<long long>(g.dh) * g.iw * cw;
    const uint4* wb = wm + c4;
    const bool interior = iy0 >= 0 && iy0 + (K - 1) * g.dh < g.ih && ix0 >= 0 && ix0 + NC <= g.iw;
    if (interior) {
        dw_window<K, SW, false>(acc, x + base, wb, row_step, cw, iy0, g.dh, g.ih, 0u, zxw);
    } else {
        uint32_t colmask = 0;
#pragma unroll
        for (int j = 0; j < NC; ++j)
            colmask |= static_cast<uint32_t>(static_cast<unsigned>(ix0 + j) < static_cast<unsigned>(g.iw)) << j;
        dw_window<K, SW, true>(acc, x + base, wb, row_step, cw, iy0, g.dh, g.ih, colmask, zxw);
    }
    const long long pix0 = (static_cast<long long>(b) * g.oh + oy) * g.ow + ox0;
    if (EK == 0) {
        uint32_t lerr = 0;
        const int c0 = c4 * 4;
        const long long cn = static_cast<long long>(cw) * 4;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            if (ox0 + p >= g.ow) break;
            const long long o = (pix0 + p) * cn + c0;
#pragma unroll
            for (int q = 0; q < 4; ++q) finish_int(e.gen, acc[p][q], c0 + q, out, o + q, &lerr);
        }
        if (lerr) atomicOr(err, lerr);
    } else {
        const int pc = e.per_channel ? c4 : 0;
        const int4 m = __ldg(reinterpret_cast<const int4*>(e.fq_m) + pc);
        const int4 sh = __ldg(reinterpret_cast<const int4*>(e.fq_sh) + pc);
        const int4 hz = __ldg(reinterpret_cast<const int4*>(e.fq_hz) + pc);
        uint32_t* o = static_cast<uint32_t*>(out) + pix0 * cw + c4;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            if (ox0 + p >= g.ow) break;
            int32_t r[4];
            r[0] = rescale_f2<EK == 2>(acc[p][0], m.x, sh.x, hz.x);
            r[1] = rescale_f2<EK == 2>(acc[p][1], m.y, sh.y, hz.y);
            r[2] = rescale_f2<EK == 2>(acc[p][2], m.z, sh.z, hz.z);
            r[3] = rescale_f2<EK == 2>(acc[p][3], m.w, sh.w, hz.w);
#pragma unroll
            for (int q = 0; q < 4; ++q) r[q] = min(max(r[q] + e.zp_add, e.lo), e.hi);
            o[p * cw] = pack4_sat_i8(r[0], r[1], r[2], r[3]);
        }
    }
}

// 3x3 windows with equal strides S (1 or 2) and no dilation: a thread keeps its 4 channels'
// 9 weight words in registers and walks down a strip of g.rows output rows, loading per
// output row only the S input rows that enter the window. The three row buffers rotate
// roles with period 3, written out as one call per role so that no buffer is ever copied.
// EK: 0 general epilogue, 1/2 fast RESCALE (single/double rounding, rescale_f2), 3/4 the
// small-range form of a table pre-scaled by 2^k at plan time (single/double rounding).
template <int S>
struct DwStrip {
    static constexpr int P = kDwPix;
    static constexpr int NC = (P - 1) * S + 3;
};

template <int S>
__device__ __forceinline__ void dw_load_row(uint32_t (&r)[DwStrip<S>::NC], const uint32_t* __restrict__ xc, int iy,
                                            const DwGeom& g, long long row_words, bool cols_ok, uint32_t colmask,
                                            uint32_t zxw) {
    constexpr int NC = DwStrip<S>::NC;
    if (static_cast<unsigned>(iy) < static_cast<unsigned>(g.ih)) {
        const uint32_t* xr = xc + iy * row_words;
        if (cols_ok) {
#pragma unroll
            for (int j = 0; j < NC; ++j) r[j] = __ldg(xr + j * g.c4);
        } else {
#pragma unroll
            for (int j = 0; j < NC; ++j) r[j] = ((colmask >> j) & 1u) ? __ldg(xr + j * g.c4) : zxw;
        }
    } else {
#pragma unroll
        for (int j = 0; j < NC; ++j) r[j] = zxw;
    }
}

// One window row's taps (weights w0, w1, w2) into the P pixels' accumulators.
template <int S>
__device__ __forceinline__ void dw_row_mac(int (&acc)[kDwPix][4], const uint32_t (&r)[DwStrip<S>::NC],
                                           const uint4& w0, const uint4& w1, const uint4& w2) {
#pragma unroll
    for (int p = 0; p < kDwPix; ++p)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            const int xv = static_cast<int>(r[p * S + kx]);
            const uint4& wq = kx == 0 ? w0 : (kx == 1 ? w1 : w2);
            acc[p][0] = __dp2a_lo(static_cast<int>(wq.x), xv, acc[p][0]);
            acc[p][1] = __dp2a_lo(static_cast<int>(wq.y), xv, acc[p][1]);
            acc[p][2] = __dp2a_hi(static_cast<int>(wq.z), xv, acc[p][2]);
            acc[p][3] = __dp2a_hi(static_cast<int>(wq.w), xv, acc[p][3]);
        }
}

template <int S, int EK>
__device__ __forceinline__ void dw_strip_row(const uint32_t (&top)[DwStrip<S>::NC], const uint32_t (&mid)[DwStrip<S>::NC],
                                             const uint32_t (&bot)[DwStrip<S>::NC], const uint4 (&w)[9],
                                             const int4& bz, const DwEpi& e, const DwGeom& g, int c4, int ox0,
                                             long long pix0, void* out, uint32_t* lerr) {
    constexpr int P = DwStrip<S>::P;
    int acc[P][4];
#pragma unroll
    for (int p = 0; p < P; ++p) {
        acc[p][0] = bz.x;
        acc[p][1] = bz.y;
        acc[p][2] = bz.z;
        acc[p][3] = bz.w;
    }
    dw_row_mac<S>(acc, top, w[0], w[1], w[2]);
    dw_row_mac<S>(acc, mid, w[3], w[4], w[5]);
    dw_row_mac<S>(acc, bot, w[6], w[7], w[8]);
    if (EK == 0) {
        const int c0 = c4 * 4;
        const long long cn = static_cast<long long>(g.c4) * 4;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            if (ox0 + p >= g.ow) break;
            const long long o = (pix0 + p) * cn + c0;
#pragma unroll
            for (int q = 0; q < 4; ++q) finish_int(e.gen, acc[p][q], c0 + q, out, o + q, lerr);
        }
    } else if (EK >= 3) {
        const int pc = e.per_channel ? c4 : 0;
        const int4 m = __ldg(reinterpret_cast<const int4*>(e.fq_m) + pc);
        const int4 sh = __ldg(reinterpret_cast<const int4*>(e.sr_sh) + pc);
        const int4 c = __ldg(reinterpret_cast<const int4*>(e.sr_c) + pc);
        auto small = [&](int32_t x, int32_t mm, int32_t s, int32_t cc) -> int32_t {
            int32_t add = cc;
            if (EK == 4) add += (x >> 31) * e.k2;  // -2^(31-d) for a negative value (double rounding)
            int32_t h;
            asm("mad.hi.s32 %0, %1, %2, %3;" : "=r"(h) : "r"(x), "r"(mm), "r"(add));
            return h >> s;
        };
        uint32_t* o = static_cast<uint32_t*>(out) + pix0 * g.c4 + c4;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            if (ox0 + p >= g.ow) break;
            int32_t v[4];
            v[0] = small(acc[p][0], m.x, sh.x, c.x);
            v[1] = small(acc[p][1], m.y, sh.y, c.y);
            v[2] = small(acc[p][2], m.z, sh.z, c.z);
            v[3] = small(acc[p][3], m.w, sh.w, c.w);
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = min(max(v[q] + e.zp_add, e.lo), e.hi);
            o[p * g.c4] = pack4_sat_i8(v[0], v[1], v[2], v[3]);
        }
    } else {
        const int pc = e.per_channel ? c4 : 0;
        const int4 m = __ldg(reinterpret_cast<const int4*>(e.fq_m) + pc);
        const int4 sh = __ldg(reinterpret_cast<const int4*>(e.fq_sh) + pc);
        const int4 hz = __ldg(reinterpret_cast<const int4*>(e.fq_hz) + pc);
        uint32_t* o = static_cast<uint32_t*>(out) + pix0 * g.c4 + c4;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            if (ox0 + p >= g.ow) break;
            int32_t v[4];
            v[0] = rescale_f2<EK == 2>(acc[p][0], m.x, sh.x, hz.x);
            v[1] = rescale_f2<EK == 2>(acc[p][1], m.y, sh.y, hz.y);
            v[2] = rescale_f2<EK == 2>(acc[p][2], m.z, sh.z, hz.z);
            v[3] = rescale_f2<EK == 2>(acc[p][3], m.w, sh.w, hz.w);
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = min(max(v[q] + e.zp_add, e.lo), e.hi);
            o[p * g.c4] = pack4_sat_i8(v[0], v[1], v[2], v[3]);
        }
    }
}

template <int S, int EK>
__global__ void depthwise_i8_dp2a_strip(DwGeom g, const uint32_t* __restrict__ x, const uint4* __restrict__ wm,
                                        const int32_t* __restrict__ bias2, uint32_t zxw, DwEpi e, void* out,
                                        uint32_t* err) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    constexpr int NC = DwStrip<S>::NC;
    const int c4 = (blockIdx.x % g.chunks) * blockDim.x + threadIdx.x;
    const int ox0 = ((blockIdx.x / g.chunks) * blockDim.y + threadIdx.y) * DwStrip<S>::P;
    if (c4 >= g.c4 || ox0 >= g.ow) return;
    const int b = blockIdx.z;
    const int oy0 = blockIdx.y * g.rows;
    const int oy1 = min(oy0 + g.rows, g.oh);
    const int ix0 = ox0 * S - g.pad_l;
    uint32_t colmask = 0;
#pragma unroll
    for (int j = 0; j < NC; ++j)
        colmask |= static_cast<uint32_t>(static_cast<unsigned>(ix0 + j) < static_cast<unsigned>(g.iw)) << j;
    const bool cols_ok = colmask == (1u << NC) - 1;
    uint4 w[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) w[t] = __ldg(wm + t * g.c4 + c4);
    const int4 bz = __ldg(reinterpret_cast<const int4*>(bias2) + c4);
    const long long row_words = static_cast<long long>(g.iw) * g.c4;
    // column ix0 of row 0 of image b, channel word c4 (read only at columns inside the input)
    const uint32_t* xc = x + static_cast<long long>(b) * g.ih * row_words + static_cast<long long>(ix0) * g.c4 + c4;
    long long pix0 = (static_cast<long long>(b) * g.oh + oy0) * g.ow + ox0;
    int iy = oy0 * S - g.pad_t;  // top input row of the window
    uint32_t lerr = 0;
    // window rows (top, mid, bot) rotate with period 3: stride 1 brings one new row per
    // output row, stride 2 two
    uint32_t r0[NC], r1[NC], r2[NC];
    dw_load_row<S>(r0, xc, iy, g, row_words, cols_ok, colmask, zxw);
    if (S == 1) dw_load_row<S>(r1, xc, iy + 1, g, row_words, cols_ok, colmask, zxw);
    for (int oy = oy0;;) {
        // (r0, r1, r2)
        if (S == 2) dw_load_row<S>(r1, xc, iy + 1, g, row_words, cols_ok, colmask, zxw);
        dw_load_row<S>(r2, xc, iy + 2, g, row_words, cols_ok, colmask, zxw);
        dw_strip_row<S, EK>(r0, r1, r2, w, bz, e, g, c4, ox0, pix0, out, &lerr);
        if (++oy >= oy1) break;
        iy += S;
        pix0 += g.ow;
        if (S == 1) {  // (r1, r2, r0)
            dw_load_row<S>(r0, xc, iy + 2, g, row_words, cols_ok, colmask, zxw);
            dw_strip_row<S, EK>(r1, r2, r0, w, bz, e, g, c4, ox0, pix0, out, &lerr);
        } else {  // (r2, r0, r1)
            dw_load_row<S>(r0, xc, iy + 1, g, row_words, cols_ok, colmask, zxw);
            dw_load_row<S>(r1, xc, iy + 2, g, row_words, cols_ok, colmask, zxw);
            dw_strip_row<S, EK>(r2, r0, r1, w, bz, e, g, c4, ox0, pix0, out, &lerr);
        }
        if (++oy >= oy1) break;
        iy += S;
        pix0 += g.ow;
        if (S == 1) {  // (r2, r0, r1)
            dw_load_row<S>(r1, xc, iy + 2, g, row_words, cols_ok, colmask, zxw);
            dw_strip_row<S, EK>(r2, r0, r1, w, bz, e, g, c4, ox0, pix0, out, &lerr);
        } else {  // (r1, r2, r0)
            dw_load_row<S>(r2, xc, iy + 1, g, row_words, cols_ok, colmask, zxw);
            dw_load_row<S>(r0, xc, iy + 2, g, row_words, cols_ok, colmask, zxw);
            dw_strip_row<S, EK>(r1, r2, r0, w, bz, e, g, c4, ox0, pix0, out, &lerr);
        }
        if (++oy >= oy1) break;
        iy += S;
        pix0 += g.ow;
    }
    if (EK == 0 && lerr) atomicOr(err, lerr);
}

__global__ void depthwise_int_generic(ConvGeomDev g, const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                      const int32_t* __restrict__ bias, int bias_len, int32_t zx, int32_t zw,
                                      IntEpiDev e, void* out, uint32_t* err) {
    const int cm = g.ic * g.m;
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * cm;
    uint32_t lerr = 0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int oc = static_cast<int>(i % cm);
        const int c = oc / g.m, mm = oc % g.m;
        long long r = i / cm;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        uint32_t acc = 0;
        for (int ky = 0; ky < g.kh; ++ky) {
            const int y = oy * g.sh - g.pad_t + ky * g.dh;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kw; ++kx) {
                const int xx = ox * g.sw - g.pad_l + kx * g.dw;
                if (xx < 0 || xx >= g.iw) continue;
                const int32_t xv = x[((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.ic + c];
                const int32_t wv = w[((ky * g.kw + kx) * g.ic + c) * g.m + mm];
                acc += static_cast<uint32_t>(xv - zx) * static_cast<uint32_t>(wv - zw);
            }
        }
        acc += static_cast<uint32_t>(bias[bias_len == 1 ? 0 : oc]);
        finish_int(e, static_cast<int32_t>(acc), oc, out, i, &lerr);
    }
    if (lerr) atomicOr(err, lerr);
}

__global__ void depthwise_float(ConvGeomDev g, const void* __restrict__ x, const void* __restrict__ w,
                                const void* __restrict__ bias, int bias_len, int in_dt, int w_dt, int acc_dt,
                                int out_dt, void* out) {
    const int cm = g.ic * g.m;
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * cm;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int oc = static_cast<int>(i % cm);
        const int c = oc / g.m, mm = oc % g.m;
        long long r = i / cm;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        float acc = 0.f;
        for (int ky = 0; ky < g.kh; ++ky) {
            const int y = oy * g.sh - g.pad_t + ky * g.dh;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kw; ++kx) {
                const int xx = ox * g.sw - g.pad_l + kx * g.dw;
                if (xx < 0 || xx >= g.iw) continue;
                const float xv = load_f(x, ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.ic + c, in_dt);
                const float wv = load_f(w, ((ky * g.kw + kx) * g.ic + c) * g.m + mm, w_dt);
                acc = mac_acc(acc, xv, wv, acc_dt);
            }
        }
        const float bv = load_f(bias, bias_len == 1 ? 0 : oc, out_dt);
        store_f(out, i, out_dt, round_to_dtype(__fadd_rn(round_to_dtype(acc, out_dt), bv), out_dt));
    }
}

// ---------------------------------------------------------------------------
// Direct MATMUL (src/ops/matmul.rs:80-95), one thread per output element.
// ---------------------------------------------------------------------------
__global__ void matmul_direct_int(int n, int h, int c, int w, const int8_t* __restrict__ a,
                                  const int8_t* __restrict__ bm, int bt, int bb, int32_t za, int32_t zb, IntEpiDev e,
                                  void* out, uint32_t* err) {
    const long long total = static_cast<long long>(n) * h * w;
    uint32_t lerr = 0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(i % w);
        const long long rowi = i / w;  // bn*h + row
        const int bn = static_cast<int>(rowi / h);
        const int8_t* ar = a + rowi * c;
        const int8_t* bc = bm + mm_b_index(bn, 0, col, c, w, bt, bb);
        const long long kstep = bt ? 1 : w;
        uint32_t acc = 0;
        for (int k = 0; k < c; ++k)
            acc += static_cast<uint32_t>(ar[k] - za) * static_cast<uint32_t>(bc[k * kstep] - zb);
        finish_int(e, static_cast<int32_t>(acc), col, out, i, &lerr);
    }
    if (lerr) atomicOr(err, lerr);
}

__global__ void matmul_direct_float(int n, int h, int c, int w, const void* __restrict__ a, const void* __restrict__ bm,
                                    int bt, int bb, int in_dt, int b_dt, int out_dt, void* out) {
    const long long total = static_cast<long long>(n) * h * w;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int col = static_cast<int>(i % w);
        const long long rowi = i / w;
        const int bn = static_cast<int>(rowi / h);
        float acc = 0.f;
        // operands are first converted to the output type (matmul.rs:160-162; this rounds only
        // the F16 / F32 operands of a BF16 MATMUL_T)
        for (int k = 0; k < c; ++k)
            acc = mac_acc(acc, round_to_dtype(load_f(a, rowi * c + k, in_dt), out_dt),
                          round_to_dtype(load_f(bm, mm_b_index(bn, k, col, c, w, bt, bb), b_dt), out_dt), out_dt, true);
        store_f(out, i, out_dt, acc);
    }
}

// ---------------------------------------------------------------------------
// Zero-point helpers of the tensor-core path
// ---------------------------------------------------------------------------

// Column terms of MATMUL's B [n][c][w] (w % 16 == 0, 16-byte aligned rows):
// out[bn][x] = scale * sum_k B[bn][k][x] + add (int32 wrap-around); with scale = -a_zp and
// add = c * a_zp * b_zp (both x 2^k for the small-range epilogue) the epilogue's column term.
// Block of 384 threads per 64 columns of one batch: 4 groups of 16 columns x 96 row slices,
// every thread's loads 8 rows at a time in flight. Bytes are biased to unsigned (x ^ 0x80 is
// x + 128) and summed in 16-bit lanes, even and odd bytes of each word apart (8 rows x 255
// fits a lane), widened per batch of 8 rows; the bias comes off at the end. The 96 slices
// are reduced in shared memory in two steps. The kernel releases its dependent launch at
// once: the GEMM that reads `out` waits for it only in its epilogue (griddepcontrol.wait).
constexpr int kColtermThreads = 384;
__global__ void __launch_bounds__(kColtermThreads) colterm_cols_i8(int c, int w, const int8_t* __restrict__ b,
                                                                  int32_t scale, int32_t add,
                                                                  int32_t* __restrict__ out) {
    grid_launch_dependents();
    constexpr int kSlices = kColtermThreads / 4;
    constexpr int kPitch = 68;  // 64 sums + 4 ints of padding: conflict-free 16-byte writes
    __shared__ __align__(16) int32_t red[kSlices * kPitch];
    __shared__ int32_t red2[6][64];
    const int t = threadIdx.x, g = t & 3, slice = t >> 2;
    const int bn = blockIdx.y, col0 = blockIdx.x * 64;
    const int col = col0 + g * 16;
    int s[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) s[j] = 0;
    int rows = 0;
    if (col < w) {
        const long long step = static_cast<long long>(kSlices) * w;
        const int8_t* src = b + (static_cast<long long>(bn) * c + slice) * w + col;
#pragma unroll 1
        for (int k = slice; k < c; k += 8 * kSlices, src += 8 * step) {
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                v[j] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // biased zeros past c
                if (k + kSlices * j < c) v[j] = __ldg(reinterpret_cast<const uint4*>(src + j * step));
            }
            rows += min(8, (c - k + kSlices - 1) / kSlices);
            uint32_t ev[4] = {0, 0, 0, 0}, od[4] = {0, 0, 0, 0};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t wv[4] = {v[j].x ^ 0x80808080u, v[j].y ^ 0x80808080u, v[j].z ^ 0x80808080u,
                                        v[j].w ^ 0x80808080u};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    ev[q] += wv[q] & 0x00ff00ffu;
                    od[q] += (wv[q] >> 8) & 0x00ff00ffu;
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                s[4 * q + 0] += static_cast<int>(ev[q] & 0xffffu);
                s[4 * q + 1] += static_cast<int>(od[q] & 0xffffu);
                s[4 * q + 2] += static_cast<int>(ev[q] >> 16);
                s[4 * q + 3] += static_cast<int>(od[q] >> 16);
            }
        }
    }
    int4* r4 = reinterpret_cast<int4*>(red + slice * kPitch + g * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q)
        r4[q] = make_int4(s[4 * q] - 128 * rows, s[4 * q + 1] - 128 * rows, s[4 * q + 2] - 128 * rows,
                          s[4 * q + 3] - 128 * rows);
    __syncthreads();
    {
        // 6 parts of 16 slices per column
        const int cc = t & 63, part = t >> 6;
        int sum = 0;
#pragma unroll
        for (int sl = 0; sl < kSlices / 6; ++sl) sum += red[(part * (kSlices / 6) + sl) * kPitch + cc];
        red2[part][cc] = sum;
    }
    __syncthreads();
    if (t < 64 && col0 + t < w) {
        int sum = 0;
#pragma unroll
        for (int part = 0; part < 6; ++part) sum += red2[part][t];
        out[static_cast<long long>(bn) * w + col0 + t] =
            static_cast<int32_t>(static_cast<uint32_t>(scale) * static_cast<uint32_t>(sum) + static_cast<uint32_t>(add));
    }
}

// wsum[oc][tap] = sum_ic w[oc][tap][ic]  (CONV2D weights OHWI, taps = kh*kw).
__global__ void conv_weight_tap_sums(int oc, int taps, int ic, const int8_t* __restrict__ w, int32_t* __restrict__ wsum) {
    const long long total = static_cast<long long>(oc) * taps;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int8_t* p = w + i * ic;
        int32_t s = 0;
        for (int c = 0; c < ic; ++c) s += p[c];
        wsum[i] = s;
    }
}

// colterm[cls][o] = bias[o] - zx * sum_{valid taps of cls} wsum[o][tap]
//                  + n_valid(cls) * ic * zx * zw     (all mod 2^32)
// Class cls = ry * n_rx + rx; row class ry admits taps ky in [ky_lo, ky_hi],
// column class rx admits kx in [kx_lo, kx_hi]. Rows are `ld` long (padded with
// zeros past oc); delta[cls][o] = colterm[cls][o] - colterm[base][o].
__device__ __forceinline__ uint32_t conv_class_term(int o, int cls, int n_rx, int kh, int kw, int ic,
                                                    const int* ky_range, const int* kx_range, const int32_t* wsum,
                                                    const int32_t* bias, int bias_len, int32_t zx, int32_t zw) {
    const int ry = cls / n_rx, rx = cls % n_rx;
    const int ky0 = ky_range[2 * ry], ky1 = ky_range[2 * ry + 1];
    const int kx0 = kx_range[2 * rx], kx1 = kx_range[2 * rx + 1];
    uint32_t ws = 0, nvalid = 0;
    for (int ky = ky0; ky <= ky1; ++ky)
        for (int kx = kx0; kx <= kx1; ++kx) {
            ws += static_cast<uint32_t>(wsum[static_cast<long long>(o) * kh * kw + ky * kw + kx]);
            ++nvalid;
        }
    const uint32_t b = static_cast<uint32_t>(bias[bias_len == 1 ? 0 : o]);
    return b - static_cast<uint32_t>(zx) * ws +
           nvalid * static_cast<uint32_t>(ic) * static_cast<uint32_t>(zx) * static_cast<uint32_t>(zw);
}

__global__ void conv_colterm(int oc, long long ld, int kh, int kw, int ic, int n_ry, int n_rx, int base,
                             const int* __restrict__ ky_range, const int* __restrict__ kx_range,
                             const int32_t* __restrict__ wsum, const int32_t* __restrict__ bias, int bias_len,
                             int32_t zx, int32_t zw, uint32_t mul, int32_t* __restrict__ colterm,
                             int32_t* __restrict__ delta) {
    const long long total = static_cast<long long>(n_ry) * n_rx * ld;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int o = static_cast<int>(i % ld);
        const int cls = static_cast<int>(i / ld);
        if (o >= oc) {
            colterm[i] = 0;
            delta[i] = 0;
            continue;
        }
        const uint32_t t = conv_class_term(o, cls, n_rx, kh, kw, ic, ky_range, kx_range, wsum, bias, bias_len, zx, zw);
        const uint32_t tb = conv_class_term(o, base, n_rx, kh, kw, ic, ky_range, kx_range, wsum, bias, bias_len, zx, zw);
        // mul: 2^k of the small-range epilogue (1 otherwise), wrap-around
        colterm[i] = static_cast<int32_t>(t * mul);
        delta[i] = static_cast<int32_t>((t - tb) * mul);
    }
}

}  // namespace tb
