"""Shared helpers for the GPU parity tests: oracle calls on numpy arrays and
torch device tensors for the C-ABI calls."""

from __future__ import annotations

import ctypes

import numpy as np

from oracle import oracle as O


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def oracle_matmul_int(a, b, za, zb):
    n, h, c = a.shape
    w = b.shape[2]
    out = np.zeros(n * h * w, dtype=np.int64)
    O.lib().orc_matmul_int(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                           _p(np.ascontiguousarray(a, np.int64)), _p(np.ascontiguousarray(b, np.int64)),
                           ctypes.c_int64(za), ctypes.c_int64(zb), ctypes.c_int(0), _p(out))
    return out.reshape(n, h, w)


def oracle_matmul_float(a, b, out_type):
    n, h, c = a.shape
    w = b.shape[2]
    out = np.zeros(n * h * w, dtype=np.float32)
    O.lib().orc_matmul_float(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                             _p(np.ascontiguousarray(a, np.float32)), _p(np.ascontiguousarray(b, np.float32)),
                             ctypes.c_int(out_type), _p(out))
    return out.reshape(n, h, w)


def conv_geom(x_shape, w_shape, pad, stride, dil, depthwise=False):
    n, ih, iw, ic = x_shape
    if depthwise:
        kh, kw, _, m = w_shape
        oc = ic * m
    else:
        oc, kh, kw, _ = w_shape
        m = 1
    oh = (ih - 1 + pad[0] + pad[1] - (kh - 1) * dil[0]) // stride[0] + 1
    ow = (iw - 1 + pad[2] + pad[3] - (kw - 1) * dil[1]) // stride[1] + 1
    g = O.ConvGeom(n=n, ih=ih, iw=iw, ic=ic, oc=oc, kh=kh, kw=kw, oh=oh, ow=ow, m=m)
    for i in range(4):
        g.pad[i] = pad[i]
    for i in range(2):
        g.stride[i] = stride[i]
        g.dilation[i] = dil[i]
    return g


def oracle_conv_int(x, w, bias, zx, zw, pad, stride, dil, depthwise=False):
    g = conv_geom(x.shape, w.shape, pad, stride, dil, depthwise)
    out = np.zeros(g.n * g.oh * g.ow * g.oc, dtype=np.int64)
    fn = O.lib().orc_depthwise_int if depthwise else O.lib().orc_conv2d_int
    fn(ctypes.byref(g), _p(np.ascontiguousarray(x, np.int64)), _p(np.ascontiguousarray(w, np.int64)),
       _p(np.ascontiguousarray(bias, np.int64)), ctypes.c_int64(len(bias)), ctypes.c_int64(zx),
       ctypes.c_int64(zw), ctypes.c_int(0), _p(out))
    return out.reshape(g.n, g.oh, g.ow, g.oc)


def oracle_conv_float(x, w, bias, acc_type, out_type, pad, stride, dil, depthwise=False):
    g = conv_geom(x.shape, w.shape, pad, stride, dil, depthwise)
    out = np.zeros(g.n * g.oh * g.ow * g.oc, dtype=np.float32)
    fn = O.lib().orc_depthwise_float if depthwise else O.lib().orc_conv2d_float
    fn(ctypes.byref(g), _p(np.ascontiguousarray(x, np.float32)), _p(np.ascontiguousarray(w, np.float32)),
       _p(np.ascontiguousarray(bias, np.float32)), ctypes.c_int64(len(bias)), ctypes.c_float(0.0),
       ctypes.c_float(0.0), ctypes.c_int(acc_type), ctypes.c_int(out_type), _p(out))
    return out.reshape(g.n, g.oh, g.ow, g.oc)


def oracle_rescale(x, in_type, out_type, mult, shift, in_zp, out_zp, scale32, rounding, per_channel,
                   in_uns=False, out_uns=False):
    x = np.ascontiguousarray(x, np.int64).reshape(-1)
    out = np.zeros(x.size, dtype=np.int64)
    ch = len(mult)
    rc = O.lib().orc_rescale(_p(x), ctypes.c_int64(x.size), ctypes.c_int(in_type), ctypes.c_int(out_type),
                             _p(np.asarray(mult, np.int64)), _p(np.asarray(shift, np.int64)), ctypes.c_int64(ch),
                             ctypes.c_int64(in_zp), ctypes.c_int64(out_zp), ctypes.c_int(scale32),
                             ctypes.c_int(rounding), ctypes.c_int(per_channel), ctypes.c_int(in_uns),
                             ctypes.c_int(out_uns), _p(out))
    return rc, out


def pool_geom(x_shape, kernel, stride, pad):
    n, ih, iw, c = x_shape
    oh = (ih + pad[0] + pad[1] - kernel[0]) // stride[0] + 1
    ow = (iw + pad[2] + pad[3] - kernel[1]) // stride[1] + 1
    g = O.PoolGeom(n=n, ih=ih, iw=iw, c=c, oh=oh, ow=ow, pad_top=pad[0], pad_left=pad[2])
    g.kernel[0], g.kernel[1] = kernel
    g.stride[0], g.stride[1] = stride
    return g


def bf16_round(x):
    """f32 -> nearest bf16 (as f32)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def ulp_bf16(x):
    """Spacing of bf16 values at |x| (2^(e-7))."""
    a = np.abs(np.asarray(x, np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return 2.0 ** (e - 7)


def float_matmul_within_tolerance(got, exp, a, b):
    """The float MATMUL bound of the parity tests: |got - exp| <= 2 bf16 ULP of exp plus
    2^-16 * sum_k |a_k * b_k| (an absolute floor near zero, where the tensor cores' and the
    reference's different accumulation orders make a relative bound meaningless). a [n,h,c],
    b [n,c,w]. Returns (all within, worst error / tolerance)."""
    absab = np.einsum("nhc,ncw->nhw", np.abs(a.astype(np.float64)), np.abs(b.astype(np.float64)))
    tol = 2 * ulp_bf16(exp) + 2.0 ** -16 * absab
    err = np.abs(got.astype(np.float64) - exp.astype(np.float64))
    return bool(np.all(err <= tol)), float(np.max(err / np.maximum(tol, 1e-30)))
