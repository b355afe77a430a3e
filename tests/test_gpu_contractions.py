"""GPU parity of the tensor-core contractions against the CPU oracle.

Integer results must be bit-exact (the reference's AccI32 wraps mod 2^32, so
any summation order gives the same bits). Float MATMUL / CONV2D results
accumulate in fp32 on the tensor core in a different order than the
reference's sequential AccF32 loop; they must lie within

    |gpu - ref| <= 2 * ulp_bf16(ref) + 2^-16 * sum_k |a_k * b_k|

(2 bf16 ULP of the reference value, plus an absolute floor scaled by the
dot product's magnitude for results near zero, where cancellation makes a
relative bound meaningless).
"""

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


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a).astype(dtype)).cuda()


def run_matmul(ctx, a, b, za, zb, rescale=None, a_dtype=L.DT_INT8, out_dtype=L.DT_INT32):
    n, h, c = a.shape
    w = b.shape[2]
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=a_dtype, b_dtype=a_dtype, out_dtype=out_dtype, a_zp=za, b_zp=zb)
    if a_dtype == L.DT_INT8:
        ta, tb = dev(a, np.int8), dev(b, np.int8)
        odt = {L.DT_INT8: torch.int8, L.DT_INT16: torch.int16, L.DT_INT32: torch.int32}[
            rescale.out_dtype if rescale is not None else L.DT_INT32]
    else:
        tdt = torch.bfloat16 if a_dtype == L.DT_BF16 else torch.float16
        ta = torch.from_numpy(a.astype(np.float32)).to(tdt).cuda()
        tb = torch.from_numpy(b.astype(np.float32)).to(tdt).cuda()
        odt = torch.float32
    out = torch.empty((n, h, w), dtype=odt, device="cuda")
    L.check(L.load().tb_matmul(ctx.h, d, rescale, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
    ctx.synchronize()
    return out.cpu().numpy()


MATMUL_SHAPES = [
    (1, 128, 128, 128, 0, 0),
    (2, 200, 96, 160, -5, 7),      # M tail, K < BK, N tail with BN=256
    (3, 130, 256, 64, 3, 0),       # a_zp only
    (1, 64, 1024, 384, 0, -8),     # b_zp only, N spans 2 tiles
    (2, 257, 528, 272, -128, 127), # extreme zero points
    # B rows not 16-byte multiples: copied into padded rows, then tensor cores
    (1, 64, 2048, 1000, 5, -3),    # a classifier head: 1000 classes
    (2, 96, 128, 20, -7, 0),
]


@pytest.mark.parametrize("n,h,c,w,za,zb", MATMUL_SHAPES)
def test_matmul_int8_tensor_core(ctx, n, h, c, w, za, zb):
    rng = np.random.default_rng(n * 1000 + h + c + w)
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    b = rng.integers(-128, 128, (n, c, w), dtype=np.int64)
    got = run_matmul(ctx, a, b, za, zb)
    exp = H.oracle_matmul_int(a, b, za, zb)
    assert np.array_equal(got.astype(np.int64), exp)


@pytest.mark.parametrize("rounding", [L.ROUND_SINGLE, L.ROUND_DOUBLE])
@pytest.mark.parametrize("per_channel", [False, True])
def test_matmul_int8_fused_rescale(ctx, rounding, per_channel):
    rng = np.random.default_rng(7 + rounding + per_channel)
    n, h, c, w = 2, 160, 256, 192
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    b = rng.integers(-128, 128, (n, c, w), dtype=np.int64)
    za, zb = int(rng.integers(-8, 9)), int(rng.integers(-8, 9))
    ch = w if per_channel else 1
    mult = rng.integers(1 << 30, (1 << 31) - 1, ch)
    shift = rng.integers(32, 40, ch)
    attr = L.rescale_attr(mult, shift, rounding=rounding, output_zp=5, out_dtype=L.DT_INT8)
    got = run_matmul(ctx, a, b, za, zb, rescale=attr)
    acc = H.oracle_matmul_int(a, b, za, zb)
    rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, 5, 1, rounding, int(per_channel))
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), exp)


def test_matmul_int8_padded_b_fused_rescale(ctx):
    """The padded-B path with a fused per-channel RESCALE to int8 (rows of 1000
    bytes: the epilogue stores unaligned chunks element by element)."""
    rng = np.random.default_rng(99)
    n, h, c, w = 1, 128, 256, 1000
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    b = rng.integers(-128, 128, (n, c, w), dtype=np.int64)
    mult = rng.integers(1 << 30, (1 << 31) - 1, w)
    shift = rng.integers(32, 40, w)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=-3, out_dtype=L.DT_INT8)
    got = run_matmul(ctx, a, b, 4, -2, rescale=attr)
    acc = H.oracle_matmul_int(a, b, 4, -2)
    rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, -3, 1, L.ROUND_DOUBLE, 1)
    assert rc == 0 and np.array_equal(got.reshape(-1).astype(np.int64), exp)


@pytest.mark.parametrize("w", [256, 1000])
def test_matmul_int8_constant_b(ctx, w):
    """A plan told that B is constant (graph CONST weights) keeps B's column terms
    (and padded rows): runs with that B are exact, a run with another B computes
    its own (and discards the kept ones), and B is prepared again afterwards."""
    import ctypes
    rng = np.random.default_rng(w)
    n, h, c = 1, 64, 512
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    bs = [rng.integers(-128, 128, (n, c, w), dtype=np.int64) for _ in range(2)]
    mult = rng.integers(1 << 30, (1 << 31) - 1, w)
    shift = rng.integers(33, 40, w)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=4, out_dtype=L.DT_INT8)
    za, zb = -5, 3
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32, a_zp=za, b_zp=zb)
    plan = ctypes.c_void_p()
    L.check(L.load().tb_matmul_plan_create(ctx.h, d, attr, ctypes.byref(plan)))
    try:
        ta = torch.from_numpy(a.astype(np.int8)).cuda()
        tb = [torch.from_numpy(b.astype(np.int8)).cuda() for b in bs]
        out = torch.empty((n, h, w), dtype=torch.int8, device="cuda")
        L.check(L.load().tb_matmul_plan_set_constant_b(plan, L.ptr(tb[0]), L.stream_ptr()))
        for k in (0, 0, 1, 0, -1, 0):
            if k < 0:
                L.check(L.load().tb_matmul_plan_set_constant_b(plan, L.ptr(tb[0]), L.stream_ptr()))
                continue
            L.check(L.load().tb_matmul_plan_run(plan, L.ptr(ta), L.ptr(tb[k]), L.ptr(out), L.stream_ptr()))
            ctx.synchronize()
            acc = H.oracle_matmul_int(a, bs[k], za, zb)
            rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, 4, 1, L.ROUND_DOUBLE, 1)
            assert rc == 0 and np.array_equal(out.cpu().numpy().reshape(-1).astype(np.int64), exp), k
    finally:
        L.load().tb_matmul_plan_destroy(plan)


def test_matmul_int8_rescale_small_shift_checks(ctx):
    """Shifts below 32 take the checked epilogue: in-range values are exact,
    out-of-range values are reported as GraphError (quant.rs:21-25)."""
    rng = np.random.default_rng(11)
    n, h, c, w = 1, 128, 64, 128
    a = rng.integers(-4, 5, (n, h, c), dtype=np.int64)
    b = rng.integers(-4, 5, (n, c, w), dtype=np.int64)
    mult = [1 << 20] * w
    shift = [24] * w
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_SINGLE, out_dtype=L.DT_INT16)
    got = run_matmul(ctx, a, b, 0, 0, rescale=attr)
    acc = H.oracle_matmul_int(a, b, 0, 0)
    rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT16, mult, shift, 0, 0, 1, L.ROUND_SINGLE, 1)
    assert rc == 0 and np.array_equal(got.reshape(-1).astype(np.int64), exp)
    # value out of range for shift 4: |v| >= 2^3
    attr2 = L.rescale_attr([1 << 20] * w, [4] * w, rounding=L.ROUND_SINGLE, out_dtype=L.DT_INT16)
    with pytest.raises(L.TbError) as ei:
        run_matmul(ctx, a * 0 + 100, b * 0 + 100, 0, 0, rescale=attr2)
    assert ei.value.kind == "GraphError"


@pytest.mark.parametrize("n,h,c,w", [(33, 7, 9, 32), (3, 5, 17, 13)])
def test_matmul_int8_direct_path(ctx, n, h, c, w):
    """Rows not a multiple of 16 bytes take the CUDA-core kernel."""
    rng = np.random.default_rng(n + h)
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    b = rng.integers(-128, 128, (n, c, w), dtype=np.int64)
    got = run_matmul(ctx, a, b, -80, -9)
    assert np.array_equal(got.astype(np.int64), H.oracle_matmul_int(a, b, -80, -9))


float_tolerance_ok = H.float_matmul_within_tolerance


@pytest.mark.parametrize("dt", [L.DT_BF16, L.DT_FP16])
@pytest.mark.parametrize("n,h,c,w", [(1, 128, 128, 128), (2, 192, 320, 200), (4, 64, 512, 256)])
def test_matmul_float_tensor_core(ctx, dt, n, h, c, w):
    rng = np.random.default_rng(c + w)
    a = rng.normal(0, 1, (n, h, c)).astype(np.float32)
    b = rng.normal(0, 1, (n, c, w)).astype(np.float32)
    if dt == L.DT_BF16:
        a, b = H.bf16_round(a), H.bf16_round(b)
    else:
        a, b = a.astype(np.float16).astype(np.float32), b.astype(np.float16).astype(np.float32)
    got = run_matmul(ctx, a, b, 0, 0, a_dtype=dt, out_dtype=L.DT_FP32)
    exp = H.oracle_matmul_float(a, b, O.D["FP32"])
    ok, worst = float_tolerance_ok(got, exp, a, b)
    assert ok, f"worst error / tolerance = {worst}"


# ---------------------------------------------------------------------------
# CONV2D
# ---------------------------------------------------------------------------


def run_conv(ctx, x, w, bias, zx, zw, pad, stride, dil, rescale=None, depthwise=False,
             in_dtype=L.DT_INT8, acc=L.DT_INT32, out_dtype=L.DT_INT32):
    n, ih, iw, ic = x.shape
    if depthwise:
        kh, kw, _, m = w.shape
        oc = ic * m
    else:
        oc, kh, kw, _ = w.shape
        m = 1
    d = L.conv_desc(n, ih, iw, ic, oc, kh, kw, pad, stride, dil, in_dtype, in_dtype, acc, out_dtype, zx, zw,
                    len(bias), m)
    oh, ow = L.conv_out_hw(ih, iw, kh, kw, pad, stride, dil)
    if in_dtype == L.DT_INT8:
        tx, tw, tbias = dev(x, np.int8), dev(w, np.int8), dev(bias, np.int32)
        odt = {L.DT_INT8: torch.int8, L.DT_INT16: torch.int16, L.DT_INT32: torch.int32}[
            rescale.out_dtype if rescale is not None else L.DT_INT32]
    else:
        tdt = torch.bfloat16 if in_dtype == L.DT_BF16 else torch.float16
        tx = torch.from_numpy(x.astype(np.float32)).to(tdt).cuda()
        tw = torch.from_numpy(w.astype(np.float32)).to(tdt).cuda()
        odt = {L.DT_BF16: torch.bfloat16, L.DT_FP16: torch.float16, L.DT_FP32: torch.float32}[out_dtype]
        tbias = torch.from_numpy(bias.astype(np.float32)).to(odt).cuda()
    out = torch.empty((n, oh, ow, oc), dtype=odt, device="cuda")
    fn = L.load().tb_depthwise_conv2d if depthwise else L.load().tb_conv2d
    L.check(fn(ctx.h, d, rescale, L.ptr(tx), L.ptr(tw), L.ptr(tbias), L.ptr(out), L.stream_ptr()))
    ctx.synchronize()
    return out.float().cpu().numpy() if in_dtype != L.DT_INT8 else out.cpu().numpy()


CONV_CASES = [
    # (n, ih, iw, ic, oc, kh, kw, pad, stride, dil, zx, zw)
    (1, 8, 8, 64, 64, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), -3, 0),
    (2, 14, 14, 128, 96, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 5, -2),
    (2, 10, 11, 32, 40, 3, 3, (1, 0, 2, 1), (2, 1), (2, 1), -49, 1),
    (1, 16, 16, 64, 256, 1, 1, (0, 0, 0, 0), (1, 1), (1, 1), 7, 3),
    (2, 15, 15, 64, 128, 1, 1, (0, 0, 0, 0), (2, 2), (1, 1), -8, 8),
    (1, 13, 13, 16, 64, 5, 5, (2, 2, 2, 2), (2, 2), (1, 1), 4, -4),
    (1, 7, 7, 256, 320, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 0, 0),
    (1, 5, 200, 16, 32, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 3, -2),     # wide rows
    (2, 23, 19, 48, 64, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), -7, 2),     # odd extents, a partial last tile
    (3, 31, 29, 32, 48, 1, 1, (0, 0, 0, 0), (2, 2), (1, 1), 11, 0),     # strided 1x1
    # few input channels: im2col rows + 1x1 tensor-core convolution (RGB stems)
    (4, 64, 64, 3, 64, 7, 7, (2, 3, 2, 3), (2, 2), (1, 1), -5, 3),
    (3, 96, 80, 3, 32, 3, 3, (0, 1, 0, 1), (2, 2), (1, 1), 6, 0),
    (8, 57, 45, 3, 64, 7, 7, (2, 2, 2, 2), (2, 2), (1, 1), 127, -128),   # odd input extents
    (11, 40, 40, 4, 32, 5, 5, (2, 1, 2, 1), (2, 2), (1, 1), -128, 5),
    (5, 64, 66, 1, 16, 4, 4, (0, 0, 2, 2), (2, 2), (1, 1), 9, -7),      # even kernel, one channel
    (1, 72, 72, 4, 48, 5, 5, (2, 2, 1, 3), (1, 1), (1, 2), -128, -2),
    (7, 50, 50, 3, 32, 7, 7, (3, 2, 3, 2), (2, 2), (1, 1), 2, 1),       # odd pads
    # the other unrolled stem shapes (4 channels x 7 and 3, 3 channels x 5), borders on every side
    (2, 94, 98, 4, 16, 7, 7, (3, 2, 3, 2), (2, 2), (1, 1), -3, 0),
    (4, 40, 40, 4, 24, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 100, 2),
    (3, 40, 40, 3, 40, 5, 5, (2, 2, 2, 2), (1, 1), (1, 1), -100, -1),
    # 64 input channels: two filter taps per stage (odd tap counts end on a one-tap stage)
    (2, 14, 14, 64, 96, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 5, -2),     # weight zero point: row sums of both taps
    (1, 13, 13, 64, 64, 5, 5, (2, 2, 2, 2), (2, 2), (1, 1), 4, -4),
    (2, 10, 11, 64, 40, 3, 3, (1, 0, 2, 1), (2, 1), (2, 1), -49, 1),    # vertical dilation, asymmetric pads
    (1, 9, 12, 64, 64, 1, 3, (0, 0, 1, 1), (1, 1), (1, 1), 2, 3),       # three taps in one row
]


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv2d_int8_tensor_core(ctx, case):
    n, ih, iw, ic, oc, kh, kw, pad, stride, dil, zx, zw = case
    rng = np.random.default_rng(ih * 31 + ic + oc)
    x = rng.integers(-128, 128, (n, ih, iw, ic), dtype=np.int64)
    w = rng.integers(-127, 128, (oc, kh, kw, ic), dtype=np.int64)
    bias = rng.integers(-32768, 32768, oc, dtype=np.int64)
    got = run_conv(ctx, x, w, bias, zx, zw, pad, stride, dil)
    exp = H.oracle_conv_int(x, w, bias, zx, zw, pad, stride, dil)
    assert got.shape == exp.shape
    assert np.array_equal(got.astype(np.int64), exp)


def test_conv2d_config1_fused_rescale(ctx):
    """[1,56,56,64] x [64,3,3,64], pad 1, zx=-3, zw=0,
    per-channel double-round RESCALE to int8 with output_zp 5."""
    rng = np.random.default_rng(20261201)
    x = rng.integers(-128, 128, (1, 56, 56, 64), dtype=np.int64)
    w = rng.integers(-127, 128, (64, 3, 3, 64), dtype=np.int64)
    bias = rng.integers(-32768, 32768, 64, dtype=np.int64)
    mult = rng.integers(1 << 30, (1 << 31) - 1, 64, endpoint=True)
    shift = rng.integers(30, 39, 64)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=5, out_dtype=L.DT_INT8)
    got = run_conv(ctx, x, w, bias, -3, 0, (1, 1, 1, 1), (1, 1), (1, 1), rescale=attr)
    acc = H.oracle_conv_int(x, w, bias, -3, 0, (1, 1, 1, 1), (1, 1), (1, 1))
    rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, 5, 1, L.ROUND_DOUBLE, 1)
    if rc != 0:
        with pytest.raises(L.TbError):
            run_conv(ctx, x, w, bias, -3, 0, (1, 1, 1, 1), (1, 1), (1, 1), rescale=attr)
        return
    assert np.array_equal(got.reshape(-1).astype(np.int64), exp)


def test_conv2d_int8_rescale_clamp(ctx):
    rng = np.random.default_rng(99)
    x = rng.integers(-128, 128, (2, 11, 11, 64), dtype=np.int64)
    w = rng.integers(-127, 128, (128, 3, 3, 64), dtype=np.int64)
    bias = rng.integers(-1000, 1000, 128, dtype=np.int64)
    mult = rng.integers(1 << 30, (1 << 31) - 1, 128)
    shift = rng.integers(36, 42, 128)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=-4, out_dtype=L.DT_INT8, clamp=(0, 127))
    got = run_conv(ctx, x, w, bias, 2, -3, (1, 1, 1, 1), (2, 2), (1, 1), rescale=attr)
    acc = H.oracle_conv_int(x, w, bias, 2, -3, (1, 1, 1, 1), (2, 2), (1, 1))
    rc, r = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, -4, 1, L.ROUND_DOUBLE, 1)
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), np.clip(r, 0, 127))


@pytest.mark.parametrize("case", [
    (2, 10, 5, 3, 7, 3, 3, (1, 0, 2, 1), (2, 1), (2, 1), -49, 1),  # ic=3: direct kernel
    (2, 8, 8, 24, 16, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 3, 2),
])
def test_conv2d_int8_direct_path(ctx, case):
    n, ih, iw, ic, oc, kh, kw, pad, stride, dil, zx, zw = case
    rng = np.random.default_rng(ic)
    x = rng.integers(-128, 128, (n, ih, iw, ic), dtype=np.int64)
    w = rng.integers(-127, 128, (oc, kh, kw, ic), dtype=np.int64)
    bias = rng.integers(-2 ** 31, 2 ** 31, 1, dtype=np.int64)
    got = run_conv(ctx, x, w, bias, zx, zw, pad, stride, dil)
    assert np.array_equal(got.astype(np.int64), H.oracle_conv_int(x, w, bias, zx, zw, pad, stride, dil))


@pytest.mark.parametrize("dt,out_dt", [(L.DT_BF16, L.DT_BF16), (L.DT_BF16, L.DT_FP32), (L.DT_FP16, L.DT_FP16)])
def test_conv2d_float_tensor_core(ctx, dt, out_dt):
    rng = np.random.default_rng(dt * 10 + out_dt)
    x = rng.normal(0, 1, (2, 12, 12, 64)).astype(np.float32)
    w = rng.normal(0, 0.1, (96, 3, 3, 64)).astype(np.float32)
    bias = rng.normal(0, 1, 96).astype(np.float32)
    rnd = H.bf16_round if dt == L.DT_BF16 else (lambda v: v.astype(np.float16).astype(np.float32))
    x, w = rnd(x), rnd(w)
    bias = H.bf16_round(bias) if out_dt == L.DT_BF16 else (
        bias.astype(np.float16).astype(np.float32) if out_dt == L.DT_FP16 else bias)
    pad, stride, dil = (1, 1, 1, 1), (1, 1), (1, 1)
    got = run_conv(ctx, x, w, bias, 0, 0, pad, stride, dil, in_dtype=dt, acc=L.DT_FP32, out_dtype=out_dt)
    exp = H.oracle_conv_float(x, w, bias, O.D["FP32"], out_dt, pad, stride, dil)
    # |x*w| summed over the window, for the absolute floor
    absx = np.abs(x.astype(np.float64))
    xp = np.pad(absx, ((0, 0), (1, 1), (1, 1), (0, 0)))
    absw = np.abs(w.astype(np.float64))
    mag = np.zeros(exp.shape)
    for ky in range(3):
        for kx in range(3):
            mag += np.einsum("nhwc,oc->nhwo", xp[:, ky:ky + 12, kx:kx + 12, :], absw[:, ky, kx, :])
    out_ulp = H.ulp_bf16(exp) if out_dt != L.DT_FP16 else 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exp), 2.0 ** -14))) - 10)
    tol = 2 * np.maximum(out_ulp, H.ulp_bf16(exp)) + 2.0 ** -16 * mag
    err = np.abs(got.astype(np.float64) - exp)
    assert np.all(err <= tol), float(np.max(err / tol))


# ---------------------------------------------------------------------------
# DEPTHWISE_CONV2D
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", [
    (2, 28, 28, 96, 1, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), -5, 3),
    (1, 16, 16, 64, 1, 3, 3, (0, 1, 0, 1), (2, 2), (1, 1), 7, 0),
    (2, 5, 6, 2, 3, 3, 3, (1, 1, 0, 1), (2, 2), (1, 2), 53, 39),
    # dp2a kernel: 4 pixels x 4 channels per thread, 3- and 5-wide rows, strides 1 and 2
    (3, 19, 23, 32, 1, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), -128, 0),   # a partial last pixel group
    (2, 21, 17, 48, 1, 5, 5, (2, 2, 2, 2), (1, 1), (1, 1), 127, -1),
    (2, 22, 26, 80, 1, 5, 5, (1, 2, 2, 1), (2, 2), (1, 1), 9, 2),       # asymmetric pads
    (1, 13, 13, 1040, 1, 3, 3, (1, 1, 1, 1), (2, 1), (1, 1), -3, 0),   # 260 channel words: two chunks
    (2, 14, 15, 16, 1, 3, 3, (2, 2, 1, 1), (1, 2), (2, 1), 4, 1),       # vertical dilation
    (1, 9, 9, 24, 1, 3, 3, (0, 0, 0, 0), (1, 1), (1, 1), 6, -100),     # w - zw beyond a byte (9 bits)
    (1, 9, 11, 8, 1, 3, 5, (1, 1, 2, 2), (1, 1), (1, 2), -1, 1),       # horizontal dilation: vec4 kernel
    # 3x3 strip kernel block shapes: two channel chunks of 130 and of 120 words, 9 words x 10 groups
    (1, 9, 10, 1040, 1, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 3, 0),
    (2, 12, 30, 960, 1, 3, 3, (1, 0, 1, 0), (2, 2), (1, 1), -7, 1),
    (1, 11, 37, 36, 1, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), 0, 2),
])
def test_depthwise_int8(ctx, case):
    n, ih, iw, c, m, kh, kw, pad, stride, dil, zx, zw = case
    rng = np.random.default_rng(c * 7 + m)
    x = rng.integers(-128, 128, (n, ih, iw, c), dtype=np.int64)
    w = rng.integers(-127, 128, (kh, kw, c, m), dtype=np.int64)
    bias = rng.integers(-5000, 5000, c * m, dtype=np.int64)
    got = run_conv(ctx, x, w, bias, zx, zw, pad, stride, dil, depthwise=True)
    exp = H.oracle_conv_int(x, w, bias, zx, zw, pad, stride, dil, depthwise=True)
    assert np.array_equal(got.astype(np.int64), exp)


def test_depthwise_int8_fused_rescale_clamp(ctx):
    rng = np.random.default_rng(5)
    n, ih, iw, c = 2, 15, 15, 144
    x = rng.integers(-128, 128, (n, ih, iw, c), dtype=np.int64)
    w = rng.integers(-127, 128, (3, 3, c, 1), dtype=np.int64)
    bias = rng.integers(-5000, 5000, c, dtype=np.int64)
    mult = rng.integers(1 << 30, (1 << 31) - 1, c)
    shift = rng.integers(34, 40, c)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=3, out_dtype=L.DT_INT8, clamp=(0, 127))
    got = run_conv(ctx, x, w, bias, -2, 1, (1, 1, 1, 1), (2, 2), (1, 1), rescale=attr, depthwise=True)
    acc = H.oracle_conv_int(x, w, bias, -2, 1, (1, 1, 1, 1), (2, 2), (1, 1), depthwise=True)
    rc, r = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, 3, 1, L.ROUND_DOUBLE, 1)
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), np.clip(r, 0, 127))


@pytest.mark.parametrize("case", [
    # (n, ih, iw, c, k, stride, pad, zx, zw, per_channel, rounding, shift range, out_dtype, bias_len)
    (2, 30, 30, 96, 3, 1, 1, -128, 0, True, L.ROUND_DOUBLE, (33, 38), L.DT_INT8, 96),
    (1, 27, 29, 64, 5, 2, 2, 17, 0, False, L.ROUND_SINGLE, (35, 36), L.DT_INT8, 1),
    (2, 17, 19, 32, 3, 2, 1, 3, -2, True, L.ROUND_SINGLE, (40, 46), L.DT_INT8, 32),
    (1, 13, 14, 40, 3, 1, 1, -7, 0, True, L.ROUND_DOUBLE, (20, 30), L.DT_INT8, 40),   # shifts below 33: general form
    (1, 12, 11, 24, 5, 1, 2, 5, 1, True, L.ROUND_DOUBLE, (33, 40), L.DT_INT16, 24),
])
def test_depthwise_int8_rescale_forms(ctx, case):
    n, ih, iw, c, k, st, pd, zx, zw, pc, rnd, srange, odt, blen = case
    rng = np.random.default_rng(n * 1000 + c + k)
    x = rng.integers(-128, 128, (n, ih, iw, c), dtype=np.int64)
    w = rng.integers(-127, 128, (k, k, c, 1), dtype=np.int64)
    bias = rng.integers(-20000, 20000, blen, dtype=np.int64)
    nch = c if pc else 1
    mult = rng.integers(1 << 30, (1 << 31) - 1, nch)
    shift = rng.integers(srange[0], srange[1] + 1, nch)
    ozp = -4 if odt == L.DT_INT8 else 0  # RESCALE allows an output zero point on int8 only
    lo, hi = (-120, 110) if odt == L.DT_INT8 else (-32768, 32767)
    attr = L.rescale_attr(mult, shift, rounding=rnd, output_zp=ozp, out_dtype=odt, clamp=(lo, hi))
    pad, stride = (pd, pd, pd, pd), (st, st)
    got = run_conv(ctx, x, w, bias, zx, zw, pad, stride, (1, 1), rescale=attr, depthwise=True)
    acc = H.oracle_conv_int(x, w, bias, zx, zw, pad, stride, (1, 1), depthwise=True)
    rc, r = H.oracle_rescale(acc, L.DT_INT32, odt, mult, shift, 0, ozp, 1, rnd, int(pc))
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), np.clip(r, lo, hi))


@pytest.mark.parametrize("rows", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("stride", [1, 2])
def test_depthwise_int8_strips(ctx, monkeypatch, rows, stride):
    """3x3 strips of several output rows per block: every phase of the row-buffer rotation,
    loop-back and a remainder strip, against the oracle (int32 and fused int8 RESCALE)."""
    monkeypatch.setenv("TB_DEPTHWISE_STRIP_ROWS", str(rows))
    rng = np.random.default_rng(rows * 10 + stride)
    n, ih, iw, c = 2, 19, 21, 40
    pad = (1, 1, 1, 1)
    x = rng.integers(-128, 128, (n, ih, iw, c), dtype=np.int64)
    w = rng.integers(-127, 128, (3, 3, c, 1), dtype=np.int64)
    bias = rng.integers(-20000, 20000, c, dtype=np.int64)
    got = run_conv(ctx, x, w, bias, -9, 4, pad, (stride, stride), (1, 1), depthwise=True)
    acc = H.oracle_conv_int(x, w, bias, -9, 4, pad, (stride, stride), (1, 1), depthwise=True)
    assert np.array_equal(got.astype(np.int64), acc)
    mult = rng.integers(1 << 30, (1 << 31) - 1, c)
    shift = rng.integers(34, 39, c)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=-2, out_dtype=L.DT_INT8, clamp=(-100, 127))
    got = run_conv(ctx, x, w, bias, -9, 4, pad, (stride, stride), (1, 1), rescale=attr, depthwise=True)
    rc, r = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, -2, 1, L.ROUND_DOUBLE, 1)
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), np.clip(r, -100, 127))


POOL_CASES = [
    # (n, ih, iw, c, kernel, stride, pad)
    (2, 17, 19, 32, (3, 3), (2, 2), (1, 1, 1, 1)),   # 16 channels per thread, borders
    (1, 56, 56, 64, (2, 2), (2, 2), (0, 0, 0, 0)),   # a strided 2x2 shortcut pool
    (2, 7, 7, 48, (7, 7), (1, 1), (0, 0, 0, 0)),     # global pool
    (1, 9, 10, 12, (3, 2), (1, 2), (1, 0, 0, 0)),    # 4 channels per thread
    (1, 6, 5, 7, (2, 3), (2, 1), (0, 0, 1, 1)),      # scalar
    (1, 8, 8, 4096, (3, 3), (1, 1), (1, 1, 1, 1)),   # 256 channel groups: one pixel per block
    (2, 10, 10, 32, (8, 8), (2, 2), (3, 3, 3, 3)),   # 64 taps (the widest 16-bit-lane window), borders
    (1, 8, 8, 1024, (3, 3), (1, 1), (1, 1, 1, 1)),   # max pool rows staged in shared memory, 64 channel groups
    (3, 15, 13, 16, (4, 3), (1, 2), (2, 1, 0, 2)),   # four-row windows, uneven padding
    (3, 9, 9, 512, (5, 5), (2, 2), (2, 2, 2, 2)),    # wide windows over few outputs: 8 lanes per group, borders
]


def _pool_desc(n, ih, iw, c, kernel, stride, pad, dtype, zi=0, zo=0):
    d = L.Pool2dDesc()
    d.n, d.ih, d.iw, d.c = n, ih, iw, c
    d.kernel[0], d.kernel[1] = kernel
    d.stride[0], d.stride[1] = stride
    for i in range(4):
        d.pad[i] = pad[i]
    d.dtype, d.acc_dtype, d.input_zp, d.output_zp, d.nan_mode = dtype, L.DT_INT32, zi, zo, L.NAN_PROPAGATE
    return d


@pytest.mark.parametrize("case", POOL_CASES)
def test_pool2d_int8(ctx, case):
    """AVG_POOL2D (zero points, reciprocal_scale rounding) and MAX_POOL2D on int8
    NHWC against the oracle, bit for bit."""
    import ctypes as C
    from oracle import oracle as O
    n, ih, iw, c, kernel, stride, pad = case
    rng = np.random.default_rng(ih * 7 + c)
    x = rng.integers(-128, 128, (n, ih, iw, c), dtype=np.int8)
    g = H.pool_geom(x.shape, kernel, stride, pad)
    tx = torch.from_numpy(x).cuda()
    out = torch.empty((n, g.oh, g.ow, c), dtype=torch.int8, device="cuda")
    xi = np.ascontiguousarray(x, np.int64)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    for zi, zo in ((0, 0), (-7, 5), (-128, 127), (127, -128)):
        d = _pool_desc(n, ih, iw, c, kernel, stride, pad, L.DT_INT8, zi, zo)
        L.check(L.load().tb_avg_pool2d(ctx.h, d, L.ptr(tx), L.ptr(out), L.stream_ptr()))
        ctx.synchronize()
        exp = np.zeros(out.numel(), dtype=np.int64)
        assert O.lib().orc_avg_pool_int(C.byref(g), p(xi), C.c_int(L.DT_INT8), C.c_int64(zi), C.c_int64(zo),
                                        p(exp)) == 0
        assert np.array_equal(out.cpu().numpy().reshape(-1).astype(np.int64), exp)
    d = _pool_desc(n, ih, iw, c, kernel, stride, pad, L.DT_INT8)
    L.check(L.load().tb_max_pool2d(ctx.h, d, L.ptr(tx), L.ptr(out), L.stream_ptr()))
    ctx.synchronize()
    exp = np.zeros(out.numel(), dtype=np.int64)
    O.lib().orc_max_pool_int(C.byref(g), p(xi), C.c_int(L.DT_INT8), p(exp))
    assert np.array_equal(out.cpu().numpy().reshape(-1).astype(np.int64), exp)
