"""CONV3D on the GPU against the CPU oracle (src/ops/conv.rs:510-516, ConvNd
:107-181 with three spatial dimensions).

The direct kernel follows the reference's order (taps kd, kh, kw row-major,
ic innermost), so every type is compared bit for bit: INT8 x INT8 / INT4 with
zero points and a fused RESCALE, INT16 x INT8 -> INT48, and the float types.
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tosa_b200 import _lib as L  # noqa: E402

_T = {L.DT_INT8: torch.int8, L.DT_INT4: torch.int8, L.DT_INT16: torch.int16, L.DT_INT32: torch.int32,
      L.DT_INT48: torch.int64, L.DT_FP32: torch.float32, L.DT_FP16: torch.float16, L.DT_BF16: torch.bfloat16}


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


def _geom(x_shape, w_shape, pad, stride, dil):
    n, idd, ih, iw, ic = x_shape
    oc, kd, kh, kw, _ = w_shape
    sp = [((idd, ih, iw)[d] - 1 + pad[2 * d] + pad[2 * d + 1] - ((kd, kh, kw)[d] - 1) * dil[d]) // stride[d] + 1
          for d in range(3)]
    g = O.Conv3dGeom(n=n, id=idd, ih=ih, iw=iw, ic=ic, oc=oc, kd=kd, kh=kh, kw=kw, od=sp[0], oh=sp[1], ow=sp[2])
    for i in range(6):
        g.pad[i] = pad[i]
    for i in range(3):
        g.stride[i] = stride[i]
        g.dilation[i] = dil[i]
    return g, [n] + sp + [oc]


def run(ctx, x, w, bias, dts, pad, stride, dil, zx=0, zw=0, rescale=None):
    it, wt, at, ot = dts
    d = L.Conv3dDesc()
    d.n, d.id, d.ih, d.iw, d.ic = x.shape
    d.oc, d.kd, d.kh, d.kw = w.shape[:4]
    for i in range(6):
        d.pad[i] = pad[i]
    for i in range(3):
        d.stride[i], d.dilation[i] = stride[i], dil[i]
    d.in_dtype, d.w_dtype, d.acc_dtype, d.out_dtype = it, wt, at, ot
    d.input_zp, d.weight_zp, d.bias_len = zx, zw, bias.size
    _, shape = _geom(x.shape, w.shape, pad, stride, dil)

    def dev(a, dt):
        if dt in (L.DT_FP32, L.DT_FP16, L.DT_BF16):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(_T[dt]).cuda()
        return torch.from_numpy(np.ascontiguousarray(a)).to(_T[dt]).cuda()

    tx, tw, tb = dev(x, it), dev(w, wt), dev(bias, ot)
    out = torch.empty(shape, dtype=_T[rescale.out_dtype if rescale is not None else ot], device="cuda")
    L.check(L.load().tb_conv3d(ctx.h, d, rescale, L.ptr(tx), L.ptr(tw), L.ptr(tb), L.ptr(out), L.stream_ptr()))
    ctx.synchronize()
    return out.float().cpu().numpy() if out.dtype == torch.bfloat16 else out.cpu().numpy()


def oracle_int(x, w, bias, zx, zw, pad, stride, dil, i48=False):
    g, shape = _geom(x.shape, w.shape, pad, stride, dil)
    out = np.zeros(int(np.prod(shape)), dtype=np.int64)
    O.lib().orc_conv3d_int(ctypes.byref(g), O._p(O._i64(x.reshape(-1))), O._p(O._i64(w.reshape(-1))),
                           O._p(O._i64(bias)), ctypes.c_int64(bias.size), ctypes.c_int64(zx), ctypes.c_int64(zw),
                           ctypes.c_int(int(i48)), O._p(out))
    return out.reshape(shape)


def oracle_float(x, w, bias, acc_t, out_t, pad, stride, dil):
    g, shape = _geom(x.shape, w.shape, pad, stride, dil)
    out = np.zeros(int(np.prod(shape)), dtype=np.float32)
    O.lib().orc_conv3d_float(ctypes.byref(g), O._p(O._f32(x.reshape(-1))), O._p(O._f32(w.reshape(-1))),
                             O._p(O._f32(bias)), ctypes.c_int64(bias.size), ctypes.c_float(0.0), ctypes.c_float(0.0),
                             ctypes.c_int(acc_t), ctypes.c_int(out_t), O._p(out))
    return out.reshape(shape)


I8 = (L.DT_INT8, L.DT_INT8, L.DT_INT32, L.DT_INT32)
INT8_CASES = [
    # x shape, w shape, pad, stride, dilation, zx, zw
    ((2, 6, 7, 8, 16), (12, 3, 3, 3, 16), (1, 1, 1, 1, 1, 1), (1, 1, 1), (1, 1, 1), -3, 2),
    ((1, 5, 9, 6, 8), (6, 2, 3, 1, 8), (0, 1, 2, 0, 0, 0), (1, 2, 1), (2, 1, 1), 5, 0),
    ((2, 5, 4, 4, 3), (5, 1, 2, 2, 3), (0, 0, 0, 1, 1, 0), (2, 1, 3), (1, 2, 1), -128, 127),
    # one depth tap, depth stride 1: one CONV2D over n * id images (tensor cores)
    ((2, 4, 14, 14, 64), (64, 1, 3, 3, 64), (0, 0, 1, 1, 1, 1), (1, 1, 1), (3, 1, 1), -3, 2),
    ((1, 3, 9, 7, 32), (48, 1, 1, 3, 32), (0, 0, 0, 0, 1, 1), (1, 2, 1), (1, 1, 2), 4, 0),
]


@pytest.mark.parametrize("xs,ws,pad,stride,dil,zx,zw", INT8_CASES)
def test_conv3d_int8(ctx, xs, ws, pad, stride, dil, zx, zw):
    rng = np.random.default_rng(sum(xs) + sum(ws))
    x = rng.integers(-128, 128, xs, dtype=np.int64)
    w = rng.integers(-128, 128, ws, dtype=np.int64)
    bias = rng.integers(-50000, 50000, ws[0])
    got = run(ctx, x, w, bias, I8, pad, stride, dil, zx, zw)
    assert np.array_equal(got.astype(np.int64), oracle_int(x, w, bias, zx, zw, pad, stride, dil))


@pytest.mark.parametrize("kd", [3, 1])
def test_conv3d_int8_fused_rescale(ctx, kd):
    rng = np.random.default_rng(21 + kd)
    x = rng.integers(-128, 128, (2, 5, 6, 6, 16), dtype=np.int64)
    w = rng.integers(-128, 128, (10, kd, 3, 3, 16), dtype=np.int64)
    bias = rng.integers(-30000, 30000, 10)
    mult = rng.integers(1 << 30, (1 << 31) - 1, 10)
    shift = rng.integers(34, 40, 10)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, per_channel=True, output_zp=1, out_dtype=L.DT_INT8)
    pad, stride, dil = ((1, 1) if kd == 3 else (0, 0)) + (1, 1, 1, 1), (1, 1, 1), (1, 1, 1)
    got = run(ctx, x, w, bias, I8, pad, stride, dil, -3, 2, rescale=attr)
    acc = oracle_int(x, w, bias, -3, 2, pad, stride, dil).reshape(-1)
    rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, 1, 1, L.ROUND_DOUBLE, 1)
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), exp)


def test_conv3d_int4_and_int16(ctx):
    rng = np.random.default_rng(4)
    pad, stride, dil = (0, 1, 1, 0, 1, 1), (1, 1, 1), (1, 1, 1)
    x = rng.integers(-128, 128, (1, 4, 5, 6, 4), dtype=np.int64)
    w = rng.integers(-8, 8, (3, 2, 2, 3, 4), dtype=np.int64)
    bias = rng.integers(-500, 500, 3)
    got = run(ctx, x, w, bias, (L.DT_INT8, L.DT_INT4, L.DT_INT32, L.DT_INT32), pad, stride, dil, 6, 0)
    assert np.array_equal(got.astype(np.int64), oracle_int(x, w, bias, 6, 0, pad, stride, dil))
    x16 = rng.integers(-32768, 32768, (1, 4, 5, 6, 4), dtype=np.int64)
    w8 = rng.integers(-128, 128, (3, 2, 2, 3, 4), dtype=np.int64)
    b48 = rng.integers(-(1 << 40), 1 << 40, 3)
    got = run(ctx, x16, w8, b48, (L.DT_INT16, L.DT_INT8, L.DT_INT48, L.DT_INT48), pad, stride, dil, 0, -5)
    assert np.array_equal(got.astype(np.int64), oracle_int(x16, w8, b48, 0, -5, pad, stride, dil, i48=True))


@pytest.mark.parametrize("dts", [(L.DT_FP32, L.DT_FP32, L.DT_FP32, L.DT_FP32),
                                 (L.DT_FP16, L.DT_FP16, L.DT_FP16, L.DT_FP16),
                                 (L.DT_BF16, L.DT_BF16, L.DT_FP32, L.DT_BF16)])
def test_conv3d_float(ctx, dts):
    rng = np.random.default_rng(dts[0] + dts[2])
    x = rng.standard_normal((1, 4, 5, 5, 3)).astype(np.float32)
    w = rng.standard_normal((6, 2, 3, 3, 3)).astype(np.float32)
    bias = rng.standard_normal(6).astype(np.float32)
    if dts[0] == L.DT_FP16:
        x, w, bias = (v.astype(np.float16).astype(np.float32) for v in (x, w, bias))
    elif dts[0] == L.DT_BF16:
        x, w, bias = (torch.from_numpy(v).to(torch.bfloat16).float().numpy() for v in (x, w, bias))
    pad, stride, dil = (1, 0, 1, 1, 0, 2), (1, 2, 1), (1, 1, 2)
    got = run(ctx, x, w, bias, dts, pad, stride, dil)
    exp = oracle_float(x, w, bias, dts[2], dts[3], pad, stride, dil)
    assert np.array_equal(O.to_bits(dts[3], got.reshape(-1).astype(np.float32)), O.to_bits(dts[3], exp.reshape(-1)))
