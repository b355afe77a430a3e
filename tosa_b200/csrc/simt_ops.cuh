// HBM-bound pooling and elementwise kernels (CUDA cores).
//   AVG_POOL2D   src/ops/pool.rs:164-231 (int: wrapping i32 sum of x - zp over
//                in-bounds taps, then apply_scale_32 by reciprocal_scale(count))
//   MAX_POOL2D   src/ops/pool.rs:251-286
//   RESCALE      src/ops/type_conv.rs:168-190
//   CLAMP        src/ops/elementwise.rs:319-343
//   ADD          src/ops/elementwise.rs:395-397
// Every thread walks a grid-stride loop; int8 NHWC pooling handles 4
// channels per thread with char4 loads when C % 4 == 0.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "quant.cuh"
#include "simt_kernels.cuh"

namespace tb {

struct PoolGeomDev {
    int n, ih, iw, c, oh, ow, ky, kx, sy, sx, pad_t, pad_l;
};

// quant.rs:6-11
__device__ __forceinline__ void reciprocal_scale_dev(int32_t value, int32_t* m, int32_t* s) {
    const int k = 32 - __clz(static_cast<uint32_t>(value) - 1u);
    const int64_t numerator = ((1ll << 30) + 1) << k;
    *m = static_cast<int32_t>(numerator / value);
    *s = 30 + k;
}

__device__ __forceinline__ int32_t int_lo(int dt) { return dt == DT_INT8 ? -128 : dt == DT_INT16 ? -32768 : INT32_MIN; }
__device__ __forceinline__ int32_t int_hi(int dt) { return dt == DT_INT8 ? 127 : dt == DT_INT16 ? 32767 : INT32_MAX; }

__device__ __forceinline__ int32_t load_int(const void* p, long long i, int dt) {
    if (dt == DT_INT8) return static_cast<const int8_t*>(p)[i];
    if (dt == DT_INT16) return static_cast<const int16_t*>(p)[i];
    return static_cast<const int32_t*>(p)[i];
}

// One AVG_POOL2D output (integer), channel c of pixel (b, oy, ox).
__device__ __forceinline__ int32_t avg_pool_int_one(const PoolGeomDev& g, const void* x, int dt, int b, int oy, int ox,
                                                    int c, int32_t zi, int32_t zo, uint32_t* err) {
    const int iy0 = oy * g.sy - g.pad_t, ix0 = ox * g.sx - g.pad_l;
    uint32_t acc = 0;
    int count = 0;
    for (int ky = 0; ky < g.ky; ++ky) {
        const int y = iy0 + ky;
        if (y < 0 || y >= g.ih) continue;
        for (int kx = 0; kx < g.kx; ++kx) {
            const int xx = ix0 + kx;
            if (xx < 0 || xx >= g.iw) continue;
            acc += static_cast<uint32_t>(load_int(x, ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.c + c, dt) - zi);
            ++count;
        }
    }
    int32_t m, s;
    reciprocal_scale_dev(count, &m, &s);
    const int64_t r = rescale_value(static_cast<int32_t>(acc), m, s, ROUND_SINGLE, 1, zo, int_lo(dt), int_hi(dt), err);
    return static_cast<int32_t>(r);
}

__global__ void avg_pool_int(PoolGeomDev g, const void* __restrict__ x, int dt, int32_t zi, int32_t zo, void* out,
                             uint32_t* err) {
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.c;
    uint32_t lerr = 0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % g.c);
        long long r = i / g.c;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        store_int(out, i, dt, avg_pool_int_one(g, x, dt, b, oy, ox, c, zi, zo, &lerr));
    }
    if (lerr) atomicOr(err, lerr);
}

// int8, C % 4 == 0: four channels per thread.
__global__ void avg_pool_i8_vec4(PoolGeomDev g, const int8_t* __restrict__ x, int32_t zi, int32_t zo, int8_t* out,
                                 uint32_t* err) {
    const int cg = g.c >> 2;
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
        const int iy0 = oy * g.sy - g.pad_t, ix0 = ox * g.sx - g.pad_l;
        uint32_t acc[4] = {0, 0, 0, 0};
        int count = 0;
        for (int ky = 0; ky < g.ky; ++ky) {
            const int y = iy0 + ky;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kx; ++kx) {
                const int xx = ix0 + kx;
                if (xx < 0 || xx >= g.iw) continue;
                const char4 v = __ldg(reinterpret_cast<const char4*>(
                    x + ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.c + c4));
                acc[0] += static_cast<uint32_t>(v.x - zi);
                acc[1] += static_cast<uint32_t>(v.y - zi);
                acc[2] += static_cast<uint32_t>(v.z - zi);
                acc[3] += static_cast<uint32_t>(v.w - zi);
                ++count;
            }
        }
        int32_t m, s;
        reciprocal_scale_dev(count, &m, &s);
        char4 o;
        o.x = static_cast<signed char>(rescale_value(static_cast<int32_t>(acc[0]), m, s, ROUND_SINGLE, 1, zo, -128, 127, &lerr));
        o.y = static_cast<signed char>(rescale_value(static_cast<int32_t>(acc[1]), m, s, ROUND_SINGLE, 1, zo, -128, 127, &lerr));
        o.z = static_cast<signed char>(rescale_value(static_cast<int32_t>(acc[2]), m, s, ROUND_SINGLE, 1, zo, -128, 127, &lerr));
        o.w = static_cast<signed char>(rescale_value(static_cast<int32_t>(acc[3]), m, s, ROUND_SINGLE, 1, zo, -128, 127, &lerr));
        reinterpret_cast<char4*>(out)[i] = o;
    }
    if (lerr) atomicOr(err, lerr);
}

// reciprocal_scale of every window size up to 64, computed once on the host.
struct RecipTable {
    int32_t m[65];
    int32_t s[65];
};

// int8 pooling, C % 16 == 0: sixteen channels (one 16-byte word) per work item. A block
// covers ppb = max(1, 256 / (C/16)) consecutive output pixels of one output row:
// grid (ceil(OW / ppb), OH, N), so pixel coordinates come from the block index.
struct PoolTile {
    int cg;   // 16-channel groups per pixel
    int ppb;  // output pixels per block
};

__host__ __device__ inline PoolTile pool_tile(int c, int ow) {
    const int cg = c >> 4;
    const int ppb = cg >= 256 ? 1 : 256 / cg;
    return PoolTile{cg, ppb < ow ? ppb : ow};
}

// Threads of a pooling block: the tile's work items rounded up to whole warps, at most 256.
__host__ __device__ inline int pool_block(const PoolTile& pt) {
    const int items = pt.ppb * pt.cg;
    return items >= 256 ? 256 : (items + 31) / 32 * 32;
}

// AVG_POOL2D int8 with at most 64 taps: the window is summed as biased bytes (x + 128)
// in 16-bit lanes of 32-bit registers (at most 64 * 255 per lane, no carry between
// lanes), and sum(x - zi) = sum(x + 128) - count * (128 + zi). apply_scale_32 with
// single rounding of |sum| < 2^14 by the reciprocal (m, s = 30 + k), exactly:
// floor((sum * m + 2^(s-1)) / 2^s) + zo = (mulhi(sum * 2^16, m) + 2^(s-17) + zo * 2^(s-16))
// >> (s - 16), the inner floor division being exact for whole multiples; no
// apply_scale_32 range check can fail for these inputs. Saturating packs give the int8 clamp.
template <int BATCH>
__global__ void avg_pool_i8_vec16(PoolGeomDev g, PoolTile pt, const int8_t* __restrict__ x, int32_t zi, int32_t zo,
                                  RecipTable rt, int8_t* out) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    const int oy = blockIdx.y, b = blockIdx.z;
    const int iy0 = oy * g.sy - g.pad_t;
    const int ky0 = max(0, -iy0), ky1 = min(g.ky, g.ih - iy0);
    for (int item = threadIdx.x; item < pt.ppb * pt.cg; item += blockDim.x) {
        const int px = item / pt.cg, c16 = (item - px * pt.cg) * 16;
        const int ox = blockIdx.x * pt.ppb + px;
        if (ox >= g.ow) break;
        const int ix0 = ox * g.sx - g.pad_l;
        const int kx0 = max(0, -ix0), kx1 = min(g.kx, g.iw - ix0);
        uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
        const uint4* xb = reinterpret_cast<const uint4*>(x + static_cast<long long>(b) * g.ih * g.iw * g.c + c16);
        const int nkx = kx1 - kx0, ntaps = (ky1 - ky0) * nkx;
        int ky = ky0, kx = kx0;
        for (int t0 = 0; t0 < ntaps; t0 += BATCH) {
            uint4 v[BATCH];  // BATCH taps of the window in flight, across its rows
#pragma unroll
            for (int j = 0; j < BATCH; ++j)
                if (t0 + j < ntaps) {
                    v[j] = __ldg(xb + static_cast<long long>((iy0 + ky) * g.iw + ix0 + kx) * pt.cg);
                    if (++kx == kx1) {
                        kx = kx0;
                        ++ky;
                    }
                }
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                if (t0 + j >= ntaps) break;
                const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    lo[q] += (w[q] ^ 0x80808080u) & 0x00ff00ffu;
                    hi[q] += ((w[q] >> 8) ^ 0x00808080u) & 0x00ff00ffu;
                }
            }
        }
        const int count = (ky1 - ky0) * (kx1 - kx0);
        if (count <= 0) break;  // cannot happen for a valid geometry (pads smaller than the kernel)
        const int32_t m = rt.m[count], sh = rt.s[count] - 16;
        const int32_t bias16 = count * (128 + zi) * 65536;
        const int32_t cst = (1 << (sh - 1)) + zo * (1 << sh);
        int32_t r[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int32_t s0 = static_cast<int32_t>(lo[q] << 16) - bias16;          // byte 0
            const int32_t s2 = static_cast<int32_t>(lo[q] & 0xffff0000u) - bias16;  // byte 2
            const int32_t s1 = static_cast<int32_t>(hi[q] << 16) - bias16;          // byte 1
            const int32_t s3 = static_cast<int32_t>(hi[q] & 0xffff0000u) - bias16;  // byte 3
            r[4 * q + 0] = (__mulhi(s0, m) + cst) >> sh;
            r[4 * q + 1] = (__mulhi(s1, m) + cst) >> sh;
            r[4 * q + 2] = (__mulhi(s2, m) + cst) >> sh;
            r[4 * q + 3] = (__mulhi(s3, m) + cst) >> sh;
        }
        reinterpret_cast<uint4*>(out)[((static_cast<long long>(b) * g.oh + oy) * g.ow + ox) * pt.cg + (c16 >> 4)] =
            make_uint4(pack4_sat_i8(r[0], r[1], r[2], r[3]), pack4_sat_i8(r[4], r[5], r[6], r[7]),
                       pack4_sat_i8(r[8], r[9], r[10], r[11]), pack4_sat_i8(r[12], r[13], r[14], r[15]));
    }
}

// The same AVG_POOL2D for wide windows over few outputs (global pools: 64 images x 128
// channel groups of a 7x7 window would be 8192 threads walking 49 taps each): S adjacent
// lanes of a warp share one output group, each summing every S-th tap of the window, and
// their 16-bit-lane partial sums are added with shuffles inside the S lanes (the lanes'
// sums add without carries for the same reason the whole window's does). Block b.x covers
// blockDim.x / S consecutive (pixel, channel group) items of output row b.y of image b.z.
template <int S>
__global__ void avg_pool_i8_vec16_split(PoolGeomDev g, int cg, const int8_t* __restrict__ x, int32_t zi, int32_t zo,
                                        RecipTable rt, int8_t* out) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    static_assert(S >= 2 && S <= 32 && (S & (S - 1)) == 0, "S lanes of one warp");
    const int oy = blockIdx.y, b = blockIdx.z;
    const int s = threadIdx.x % S;
    const int item = blockIdx.x * (blockDim.x / S) + threadIdx.x / S;
    const int ox = item / cg, c16 = (item - ox * cg) * 16;
    if (ox >= g.ow) return;  // the whole group of S lanes
    const unsigned lane = threadIdx.x & 31u;
    const unsigned mask = ((S == 32) ? 0xffffffffu : ((1u << S) - 1u)) << (lane & ~static_cast<unsigned>(S - 1));
    const int iy0 = oy * g.sy - g.pad_t, ix0 = ox * g.sx - g.pad_l;
    const int ky0 = max(0, -iy0), ky1 = min(g.ky, g.ih - iy0);
    const int kx0 = max(0, -ix0), kx1 = min(g.kx, g.iw - ix0);
    const int nkx = kx1 - kx0, ntaps = (ky1 - ky0) * nkx;
    const int count = ntaps;
    if (count <= 0) return;  // cannot happen for a valid geometry (pads smaller than the kernel)
    const uint4* xb = reinterpret_cast<const uint4*>(x + static_cast<long long>(b) * g.ih * g.iw * g.c + c16);
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    int ky = ky0 + s / nkx, kx = kx0 + s % nkx;  // tap s of the window, row-major
#pragma unroll 4
    for (int t = s; t < ntaps; t += S) {
        const uint4 v = __ldg(xb + static_cast<long long>((iy0 + ky) * g.iw + ix0 + kx) * cg);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            lo[q] += (w[q] ^ 0x80808080u) & 0x00ff00ffu;
            hi[q] += ((w[q] >> 8) ^ 0x00808080u) & 0x00ff00ffu;
        }
        kx += S;
        while (kx >= kx1) {
            kx -= nkx;
            ++ky;
        }
    }
#pragma unroll
    for (int o = S / 2; o > 0; o >>= 1)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            lo[q] += __shfl_xor_sync(mask, lo[q], o);
            hi[q] += __shfl_xor_sync(mask, hi[q], o);
        }
    if (s != 0) return;
    const int32_t m = rt.m[count], sh = rt.s[count] - 16;
    const int32_t bias16 = count * (128 + zi) * 65536;
    const int32_t cst = (1 << (sh - 1)) + zo * (1 << sh);
    int32_t r[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int32_t s0 = static_cast<int32_t>(lo[q] << 16) - bias16;          // byte 0
        const int32_t s2 = static_cast<int32_t>(lo[q] & 0xffff0000u) - bias16;  // byte 2
        const int32_t s1 = static_cast<int32_t>(hi[q] << 16) - bias16;          // byte 1
        const int32_t s3 = static_cast<int32_t>(hi[q] & 0xffff0000u) - bias16;  // byte 3
        r[4 * q + 0] = (__mulhi(s0, m) + cst) >> sh;
        r[4 * q + 1] = (__mulhi(s1, m) + cst) >> sh;
        r[4 * q + 2] = (__mulhi(s2, m) + cst) >> sh;
        r[4 * q + 3] = (__mulhi(s3, m) + cst) >> sh;
    }
    reinterpret_cast<uint4*>(out)[((static_cast<long long>(b) * g.oh + oy) * g.ow + ox) * cg + (c16 >> 4)] =
        make_uint4(pack4_sat_i8(r[0], r[1], r[2], r[3]), pack4_sat_i8(r[4], r[5], r[6], r[7]),
                   pack4_sat_i8(r[8], r[9], r[10], r[11]), pack4_sat_i8(r[12], r[13], r[14], r[15]));
}

__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// MAX_POOL2D int8, C % 16 == 0 (same tiling): the bytes, biased to unsigned (x + 128),
// are split into even and odd bytes held in 16-bit lanes, and the lanes take packed
// unsigned 16-bit maxima; the bytes are rejoined and unbiased at the end.
template <int BATCH>
__global__ void max_pool_i8_vec16(PoolGeomDev g, PoolTile pt, const int8_t* __restrict__ x, int8_t* out) {
    grid_launch_dependents();  // a programmatic dependent launch of the next kernel may start
    const int oy = blockIdx.y, b = blockIdx.z;
    const int iy0 = oy * g.sy - g.pad_t;
    const int ky0 = max(0, -iy0), ky1 = min(g.ky, g.ih - iy0);
    for (int item = threadIdx.x; item < pt.ppb * pt.cg; item += blockDim.x) {
        const int px = item / pt.cg, c16 = (item - px * pt.cg) * 16;
        const int ox = blockIdx.x * pt.ppb + px;
        if (ox >= g.ow) break;
        const int ix0 = ox * g.sx - g.pad_l;
        const int kx0 = max(0, -ix0), kx1 = min(g.kx, g.iw - ix0);
        uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};  // biased -128
        const uint4* xb = reinterpret_cast<const uint4*>(x + static_cast<long long>(b) * g.ih * g.iw * g.c + c16);
        const int nkx = kx1 - kx0, ntaps = (ky1 - ky0) * nkx;
        int ky = ky0, kx = kx0;
        for (int t0 = 0; t0 < ntaps; t0 += BATCH) {
            uint4 v[BATCH];  // BATCH taps of the window in flight, across its rows
#pragma unroll
            for (int j = 0; j < BATCH; ++j)
                if (t0 + j < ntaps) {
                    v[j] = __ldg(xb + static_cast<long long>((iy0 + ky) * g.iw + ix0 + kx) * pt.cg);
                    if (++kx == kx1) {
                        kx = kx0;
                        ++ky;
                    }
                }
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                if (t0 + j >= ntaps) break;
                const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    lo[q] = max_u16x2(lo[q], (w[q] ^ 0x80808080u) & 0x00ff00ffu);
                    hi[q] = max_u16x2(hi[q], ((w[q] >> 8) ^ 0x00808080u) & 0x00ff00ffu);
                }
            }
        }
        reinterpret_cast<uint4*>(out)[((static_cast<long long>(b) * g.oh + oy) * g.ow + ox) * pt.cg + (c16 >> 4)] =
            make_uint4((lo[0] | (hi[0] << 8)) ^ 0x80808080u, (lo[1] | (hi[1] << 8)) ^ 0x80808080u,
                       (lo[2] | (hi[2] << 8)) ^ 0x80808080u, (lo[3] | (hi[3] << 8)) ^ 0x80808080u);
    }
}

// Float AVG_POOL2D: every add and the division rounded to acc_dt, the result
// rounded to the data type (pool.rs:215-227).
__global__ void avg_pool_float(PoolGeomDev g, const void* __restrict__ x, int dt, int acc_dt, void* out) {
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.c;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % g.c);
        long long r = i / g.c;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        const int iy0 = oy * g.sy - g.pad_t, ix0 = ox * g.sx - g.pad_l;
        float acc = 0.f;
        int count = 0;
        for (int ky = 0; ky < g.ky; ++ky) {
            const int y = iy0 + ky;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kx; ++kx) {
                const int xx = ix0 + kx;
                if (xx < 0 || xx >= g.iw) continue;
                acc = round_to_dtype(__fadd_rn(acc, load_f(x, ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.c + c, dt)),
                                     acc_dt);
                ++count;
            }
        }
        const float v = round_to_dtype(__fdiv_rn(acc, static_cast<float>(count)), acc_dt);
        store_f(out, i, dt, round_to_dtype(v, dt));
    }
}

__global__ void max_pool_int(PoolGeomDev g, const void* __restrict__ x, int dt, void* out) {
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.c;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % g.c);
        long long r = i / g.c;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        const int iy0 = oy * g.sy - g.pad_t, ix0 = ox * g.sx - g.pad_l;
        int32_t m = int_lo(dt);
        for (int ky = 0; ky < g.ky; ++ky) {
            const int y = iy0 + ky;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kx; ++kx) {
                const int xx = ix0 + kx;
                if (xx < 0 || xx >= g.iw) continue;
                m = max(m, load_int(x, ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.c + c, dt));
            }
        }
        store_int(out, i, dt, m);
    }
}

// int8, C % 4 == 0: byte-wise signed max over char4 words (__vmaxs4).
__global__ void max_pool_i8_vec4(PoolGeomDev g, const int8_t* __restrict__ x, int8_t* out) {
    const int cg = g.c >> 2;
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * cg;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c4 = static_cast<int>(i % cg) * 4;
        long long r = i / cg;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        const int iy0 = oy * g.sy - g.pad_t, ix0 = ox * g.sx - g.pad_l;
        unsigned m = 0x80808080u;
        for (int ky = 0; ky < g.ky; ++ky) {
            const int y = iy0 + ky;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kx; ++kx) {
                const int xx = ix0 + kx;
                if (xx < 0 || xx >= g.iw) continue;
                const unsigned v = __ldg(reinterpret_cast<const unsigned*>(
                    x + ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.c + c4));
                m = __vmaxs4(m, v);
            }
        }
        reinterpret_cast<unsigned*>(out)[i] = m;
    }
}

// NaN-aware max / min of the reference (common.rs:153-177): ties keep a (max)
// or b (min); with IGNORE a NaN operand yields the other one.
__device__ __forceinline__ float nan_pick(float a, float b, int mode) {
    if (mode == 2) return isnan(a) ? b : a;
    return __int_as_float(0x7fc00000);
}
// The most negative finite value of a float type (the reference's float_lowest).
__device__ __forceinline__ float float_lowest(int dt) {
    switch (dt) {
    case DT_FP16: return -65504.f;
    case DT_BF16: return __uint_as_float(0xff7f0000u);
    case DT_FP8E4M3: return -448.f;
    case DT_FP8E5M2: return -57344.f;
    default: return __uint_as_float(0xff7fffffu);
    }
}

__device__ __forceinline__ float nan_max(float a, float b, int mode) {
    if (isnan(a) || isnan(b)) return nan_pick(a, b, mode);
    return a >= b ? a : b;
}
__device__ __forceinline__ float nan_min(float a, float b, int mode) {
    if (isnan(a) || isnan(b)) return nan_pick(a, b, mode);
    return a < b ? a : b;
}

__global__ void max_pool_float(PoolGeomDev g, const void* __restrict__ x, int dt, int nan_mode, void* out) {
    const long long total = static_cast<long long>(g.n) * g.oh * g.ow * g.c;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % g.c);
        long long r = i / g.c;
        const int ox = static_cast<int>(r % g.ow);
        r /= g.ow;
        const int oy = static_cast<int>(r % g.oh);
        const int b = static_cast<int>(r / g.oh);
        const int iy0 = oy * g.sy - g.pad_t, ix0 = ox * g.sx - g.pad_l;
        float m = nan_mode == 2 ? __int_as_float(0x7fc00000) : float_lowest(dt);
        for (int ky = 0; ky < g.ky; ++ky) {
            const int y = iy0 + ky;
            if (y < 0 || y >= g.ih) continue;
            for (int kx = 0; kx < g.kx; ++kx) {
                const int xx = ix0 + kx;
                if (xx < 0 || xx >= g.iw) continue;
                m = nan_max(m, load_f(x, ((static_cast<long long>(b) * g.ih + y) * g.iw + xx) * g.c + c, dt), nan_mode);
            }
        }
        store_f(out, i, dt, m);
    }
}

// ---------------------------------------------------------------------------
// Elementwise
// ---------------------------------------------------------------------------

// RESCALE: x = extend(v) - in_zp (extend masks to the width when unsigned).
__global__ void rescale_elementwise(const void* __restrict__ in, int in_dt, int in_unsigned, int32_t in_zp_ext,
                                    long long count, int channels, RescaleArgs rs, int out_dt, void* out,
                                    uint32_t* err) {
    uint32_t lerr = 0;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        int64_t v = in_dt == DT_INT48 ? static_cast<const int64_t*>(in)[i] : load_int(in, i, in_dt);
        if (in_unsigned) v &= in_dt == DT_INT8 ? 0xff : 0xffff;
        const int64_t x = v - in_zp_ext;
        const int ch = rs.per_channel ? static_cast<int>(i % channels) : 0;
        const int64_t r = rescale_value(x, rs.multiplier[ch], rs.shift[ch], rs.rounding, rs.scale32, rs.out_zp, rs.lo,
                                        rs.hi, &lerr);
        store_int(out, i, out_dt, static_cast<int32_t>(r));
    }
    if (lerr) atomicOr(err, lerr);
}

__global__ void clamp_int(const void* __restrict__ in, int dt, long long count, int32_t lo, int32_t hi, void* out) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        int32_t v = load_int(in, i, dt);
        v = max(v, lo);
        v = min(v, hi);
        store_int(out, i, dt, v);
    }
}

__global__ void clamp_float(const void* __restrict__ in, int dt, long long count, float lo, float hi, int nan_mode,
                            void* out) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float v = nan_min(nan_max(load_f(in, i, dt), lo, nan_mode), hi, nan_mode);
        store_f(out, i, dt, v);
    }
}

__global__ void add_elementwise(const void* __restrict__ a, const void* __restrict__ b, int dt, long long count,
                                void* out) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        if (dt == DT_INT32) {
            static_cast<int32_t*>(out)[i] = static_cast<int32_t>(static_cast<uint32_t>(static_cast<const int32_t*>(a)[i]) +
                                                                 static_cast<uint32_t>(static_cast<const int32_t*>(b)[i]));
        } else {
            store_f(out, i, dt, round_to_dtype(__fadd_rn(load_f(a, i, dt), load_f(b, i, dt)), dt));
        }
    }
}

}  // namespace tb
