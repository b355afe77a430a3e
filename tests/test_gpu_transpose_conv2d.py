"""TRANSPOSE_CONV2D on the GPU against the CPU oracle (src/ops/conv.rs:526-532,
Transpose :286-371, gather form).

INT8 with stride 1 runs as a CONV2D over tap-reversed weights on the tensor
cores; everything else (other strides, INT4 weights stored one per byte,
INT16 x INT8 -> INT48, the float types) runs the direct gather kernel in the
reference's order. Every result must be bit-exact, zero points, negative
out_pad and a fused RESCALE included.
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tosa_b200 import _lib as L  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


def _geom(n, ih, iw, ic, oc, kh, kw, out_pad, stride):
    oh = (ih - 1) * stride[0] + out_pad[0] + out_pad[1] + kh
    ow = (iw - 1) * stride[1] + out_pad[2] + out_pad[3] + kw
    g = O.ConvGeom(n=n, ih=ih, iw=iw, ic=ic, oc=oc, kh=kh, kw=kw, oh=oh, ow=ow, m=1)
    for i in range(4):
        g.pad[i] = out_pad[i]
    for i in range(2):
        g.stride[i] = stride[i]
        g.dilation[i] = 1
    return g


def oracle_int(x, w, bias, zx, zw, out_pad, stride, i48=False):
    n, ih, iw, ic = x.shape
    oc, kh, kw, _ = w.shape
    g = _geom(n, ih, iw, ic, oc, kh, kw, out_pad, stride)
    out = np.zeros(n * g.oh * g.ow * oc, dtype=np.int64)
    O.lib().orc_transpose_conv2d_int(ctypes.byref(g), O._p(O._i64(x.reshape(-1))), O._p(O._i64(w.reshape(-1))),
                                     O._p(O._i64(bias)), ctypes.c_int64(bias.size), ctypes.c_int64(zx),
                                     ctypes.c_int64(zw), ctypes.c_int(int(i48)), O._p(out))
    return out.reshape(n, g.oh, g.ow, oc)


def oracle_float(x, w, bias, acc_t, out_t, out_pad, stride):
    n, ih, iw, ic = x.shape
    oc, kh, kw, _ = w.shape
    g = _geom(n, ih, iw, ic, oc, kh, kw, out_pad, stride)
    out = np.zeros(n * g.oh * g.ow * oc, dtype=np.float32)
    O.lib().orc_transpose_conv2d_float(ctypes.byref(g), O._p(O._f32(x.reshape(-1))), O._p(O._f32(w.reshape(-1))),
                                       O._p(O._f32(bias)), ctypes.c_int64(bias.size), ctypes.c_float(0.0),
                                       ctypes.c_float(0.0), ctypes.c_int(acc_t), ctypes.c_int(out_t), O._p(out))
    return out.reshape(n, g.oh, g.ow, oc)


def run(ctx, x, w, bias, dts, out_pad, stride, zx=0, zw=0, rescale=None):
    it, wt, at, ot = dts
    n, ih, iw, ic = x.shape
    oc, kh, kw, _ = w.shape
    d = L.conv_desc(n, ih, iw, ic, oc, kh, kw, out_pad, stride, (1, 1), it, wt, at, ot, zx, zw, bias.size)
    oh = (ih - 1) * stride[0] + out_pad[0] + out_pad[1] + kh
    ow = (iw - 1) * stride[1] + out_pad[2] + out_pad[3] + kw
    tdt = {L.DT_INT8: torch.int8, L.DT_INT4: torch.int8, L.DT_INT16: torch.int16, L.DT_INT32: torch.int32,
           L.DT_INT48: torch.int64, L.DT_FP32: torch.float32, L.DT_FP16: torch.float16, L.DT_BF16: torch.bfloat16}

    def dev(a, dt):
        if dt in (L.DT_FP32, L.DT_FP16, L.DT_BF16):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(tdt[dt]).cuda()
        return torch.from_numpy(np.ascontiguousarray(a)).to(tdt[dt]).cuda()

    tx, tw, tb = dev(x, it), dev(w, wt), dev(bias, ot)
    out = torch.empty((n, oh, ow, oc), dtype=tdt[rescale.out_dtype if rescale is not None else ot], device="cuda")
    L.check(L.load().tb_transpose_conv2d(ctx.h, d, rescale, L.ptr(tx), L.ptr(tw), L.ptr(tb), L.ptr(out),
                                         L.stream_ptr()))
    ctx.synchronize()
    return out.float().cpu().numpy() if out.dtype == torch.bfloat16 else out.cpu().numpy()


INT8_CASES = [
    # n, ih, iw, ic, oc, kh, kw, out_pad, stride, zx, zw
    (2, 14, 14, 64, 64, 3, 3, (0, 0, 0, 0), (1, 1), -3, 2),     # tensor cores (stride 1)
    (1, 9, 11, 32, 40, 3, 3, (-1, 1, 0, -2), (1, 1), 5, 0),     # negative out_pad
    (2, 8, 8, 128, 96, 1, 1, (0, 0, 0, 0), (1, 1), 0, -4),
    (1, 7, 5, 16, 24, 5, 3, (2, 0, 1, 1), (1, 1), -128, 127),
    (2, 8, 8, 64, 32, 4, 4, (-1, -1, -1, -1), (2, 2), -3, 1),  # stride 2: direct gather
    (1, 6, 7, 12, 10, 3, 2, (0, 1, 1, 0), (2, 3), 4, -2),
]


@pytest.mark.parametrize("n,ih,iw,ic,oc,kh,kw,out_pad,stride,zx,zw", INT8_CASES)
def test_transpose_conv2d_int8(ctx, n, ih, iw, ic, oc, kh, kw, out_pad, stride, zx, zw):
    rng = np.random.default_rng(ih * 100 + ic + oc + kh)
    x = rng.integers(-128, 128, (n, ih, iw, ic), dtype=np.int64)
    w = rng.integers(-128, 128, (oc, kh, kw, ic), dtype=np.int64)
    bias = rng.integers(-50000, 50000, oc)
    dts = (L.DT_INT8, L.DT_INT8, L.DT_INT32, L.DT_INT32)
    got = run(ctx, x, w, bias, dts, out_pad, stride, zx, zw)
    assert np.array_equal(got.astype(np.int64), oracle_int(x, w, bias, zx, zw, out_pad, stride))


@pytest.mark.parametrize("stride", [(1, 1), (2, 2)])
def test_transpose_conv2d_int8_fused_rescale(ctx, stride):
    rng = np.random.default_rng(11 + stride[0])
    n, ih, iw, ic, oc, kh, kw = 2, 10, 10, 64, 48, 3, 3
    out_pad = (0, 0, 0, 0) if stride == (1, 1) else (-1, 0, -1, 0)
    x = rng.integers(-128, 128, (n, ih, iw, ic), dtype=np.int64)
    w = rng.integers(-128, 128, (oc, kh, kw, ic), dtype=np.int64)
    bias = rng.integers(-30000, 30000, oc)
    mult = rng.integers(1 << 30, (1 << 31) - 1, oc)
    shift = rng.integers(34, 40, oc)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, per_channel=True, output_zp=-2,
                          out_dtype=L.DT_INT8, clamp=(-128, 127))
    dts = (L.DT_INT8, L.DT_INT8, L.DT_INT32, L.DT_INT32)
    got = run(ctx, x, w, bias, dts, out_pad, stride, -3, 2, rescale=attr)
    acc = oracle_int(x, w, bias, -3, 2, out_pad, stride).reshape(-1)
    rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, -2, 1, L.ROUND_DOUBLE, 1)
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), exp)


@pytest.mark.parametrize("stride", [(1, 1), (2, 1)])
def test_transpose_conv2d_int4_weights(ctx, stride):
    rng = np.random.default_rng(3 + stride[0])
    x = rng.integers(-128, 128, (2, 6, 5, 16), dtype=np.int64)
    w = rng.integers(-8, 8, (8, 3, 2, 16), dtype=np.int64)
    bias = rng.integers(-1000, 1000, 8)
    dts = (L.DT_INT8, L.DT_INT4, L.DT_INT32, L.DT_INT32)
    got = run(ctx, x, w, bias, dts, (0, 1, 1, 0), stride, 7, 0)
    assert np.array_equal(got.astype(np.int64), oracle_int(x, w, bias, 7, 0, (0, 1, 1, 0), stride))


def test_transpose_conv2d_int16(ctx):
    rng = np.random.default_rng(8)
    x = rng.integers(-32768, 32768, (2, 4, 3, 6), dtype=np.int64)
    w = rng.integers(-128, 128, (5, 2, 2, 6), dtype=np.int64)
    bias = rng.integers(-(1 << 40), 1 << 40, 5)
    dts = (L.DT_INT16, L.DT_INT8, L.DT_INT48, L.DT_INT48)
    got = run(ctx, x, w, bias, dts, (0, 1, 1, 1), (2, 2))
    assert np.array_equal(got.astype(np.int64), oracle_int(x, w, bias, 0, 0, (0, 1, 1, 1), (2, 2), i48=True))


@pytest.mark.parametrize("dts", [(L.DT_FP32, L.DT_FP32, L.DT_FP32, L.DT_FP32),
                                 (L.DT_FP16, L.DT_FP16, L.DT_FP16, L.DT_FP16),
                                 (L.DT_FP16, L.DT_FP16, L.DT_FP32, L.DT_FP16),
                                 (L.DT_BF16, L.DT_BF16, L.DT_FP32, L.DT_BF16)])
@pytest.mark.parametrize("stride", [(1, 1), (2, 2)])
def test_transpose_conv2d_float(ctx, dts, stride):
    rng = np.random.default_rng(dts[0] * 10 + dts[2] + stride[0])
    x = rng.standard_normal((1, 5, 6, 3)).astype(np.float32)
    w = rng.standard_normal((8, 3, 3, 3)).astype(np.float32)
    bias = rng.standard_normal(8).astype(np.float32)
    if dts[0] == L.DT_FP16:
        x, w, bias = (v.astype(np.float16).astype(np.float32) for v in (x, w, bias))
    elif dts[0] == L.DT_BF16:
        x, w, bias = (torch.from_numpy(v).to(torch.bfloat16).float().numpy() for v in (x, w, bias))
    got = run(ctx, x, w, bias, dts, (1, 1, 0, 1), stride)
    exp = oracle_float(x, w, bias, dts[2], dts[3], (1, 1, 0, 1), stride)
    ot = dts[3]
    assert np.array_equal(O.to_bits(ot, got.reshape(-1).astype(np.float32)), O.to_bits(ot, exp.reshape(-1)))


def test_transpose_conv2d_rejects(ctx):
    """Transpose::new's checks (conv.rs:286-329) and the type table."""
    lib = L.load()
    plan = ctypes.c_void_p()
    w = torch.zeros(64, dtype=torch.int8, device="cuda")
    b = torch.zeros(4, dtype=torch.int32, device="cuda")
    i8 = (L.DT_INT8, L.DT_INT8, L.DT_INT32, L.DT_INT32)
    graph_error, dtype_mismatch = 7, 4  # tb_status codes
    bad_pad = L.conv_desc(1, 4, 4, 4, 4, 2, 2, (-2, 0, 0, 0), (1, 1), (1, 1), *i8)
    assert lib.tb_transpose_conv2d_plan_create(ctx.h, bad_pad, L.ptr(w), L.ptr(b), None,
                                               ctypes.byref(plan)) == graph_error
    bad_stride = L.conv_desc(1, 4, 4, 4, 4, 2, 2, (0, 0, 0, 0), (0, 1), (1, 1), *i8)
    assert lib.tb_transpose_conv2d_plan_create(ctx.h, bad_stride, L.ptr(w), L.ptr(b), None,
                                               ctypes.byref(plan)) == graph_error
    mixed = L.conv_desc(1, 4, 4, 4, 4, 2, 2, (0, 0, 0, 0), (1, 1), (1, 1), L.DT_FP16, L.DT_BF16, L.DT_FP32, L.DT_FP32)
    assert lib.tb_transpose_conv2d_plan_create(ctx.h, mixed, L.ptr(w), L.ptr(b), None,
                                               ctypes.byref(plan)) == dtype_mismatch
