"""MATMUL_T on the GPU against the CPU oracle (src/ops/matmul.rs:180-182, :98-174).

b is [d, w, c] with d == n, or d == 1 broadcast over every batch of a. INT8
runs on the tensor cores with B K-major (c % 16 == 0) and must be bit-exact,
with zero points, a fused RESCALE and a constant B; INT8 with other c, INT16 ->
INT48 and the mixed float types run the direct kernels in the reference's
order and must be bit-exact too. BF16 x BF16 / FP16 x FP16 -> FP32 on the
tensor cores must lie within

    |gpu - ref| <= 2 * ulp_bf16(ref) + 2^-16 * sum_k |a_k * b_k|

(fp32 accumulation in another order than the reference's sequential loop).
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tosa_b200 import _lib as L  # noqa: E402

_TORCH = {L.DT_INT8: torch.int8, L.DT_INT16: torch.int16, L.DT_INT32: torch.int32, L.DT_INT48: torch.int64,
          L.DT_FP32: torch.float32, L.DT_FP16: torch.float16, L.DT_BF16: torch.bfloat16}


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


def _dev(x, dt):
    """Device tensor of dtype code dt holding x (float values already exact in dt)."""
    if dt in (L.DT_FP8E4M3, L.DT_FP8E5M2):
        lut = O.fp8_lut(dt)
        codes = np.array([int(np.nonzero(lut == v)[0][0]) for v in x.reshape(-1)], dtype=np.uint8)
        return torch.from_numpy(codes.reshape(x.shape)).cuda()
    if dt in (L.DT_FP32, L.DT_FP16, L.DT_BF16):
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(_TORCH[dt]).cuda()
    return torch.from_numpy(np.ascontiguousarray(x).astype({L.DT_INT8: np.int8, L.DT_INT16: np.int16}[dt])).cuda()


def _values(rng, dt, shape):
    if dt == L.DT_INT8:
        return rng.integers(-128, 128, shape, dtype=np.int64)
    if dt == L.DT_INT16:
        return rng.integers(-32768, 32768, shape, dtype=np.int64)
    if dt in (L.DT_FP8E4M3, L.DT_FP8E5M2):
        lut = O.fp8_lut(dt)
        ok = lut[np.isfinite(lut) & (np.abs(lut) <= 16)]
        return rng.choice(ok, shape).astype(np.float32)
    x = rng.standard_normal(shape).astype(np.float32)
    if dt == L.DT_BF16:
        return torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    if dt == L.DT_FP16:
        return x.astype(np.float16).astype(np.float32)
    return x


def run_t(ctx, a, b, at, bt, ot, za=0, zb=0, rescale=None, plan_const=False):
    n, h, c = a.shape
    d_, w, _ = b.shape
    desc = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=at, b_dtype=bt, out_dtype=ot, a_zp=za, b_zp=zb)
    ta, tb = _dev(a, at), _dev(b, bt)
    odt = _TORCH[rescale.out_dtype if rescale is not None else ot]
    out = torch.empty((n, h, w), dtype=odt, device="cuda")
    lib = L.load()
    if plan_const:
        plan = ctypes.c_void_p()
        L.check(lib.tb_matmul_t_plan_create(ctx.h, desc, d_, rescale, ctypes.byref(plan)))
        try:
            L.check(lib.tb_matmul_plan_set_constant_b(plan, L.ptr(tb), L.stream_ptr()))
            for _ in range(2):
                L.check(lib.tb_matmul_plan_run(plan, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
            ctx.synchronize()
        finally:
            lib.tb_matmul_plan_destroy(plan)
    else:
        L.check(lib.tb_matmul_t(ctx.h, desc, d_, rescale, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
        ctx.synchronize()
    if odt == torch.bfloat16:
        return out.float().cpu().numpy()
    return out.cpu().numpy()


def oracle_t_int(a, b, za, zb, i48=False):
    n, h, c = a.shape
    d_, w, _ = b.shape
    out = np.zeros(n * h * w, dtype=np.int64)
    O.lib().orc_matmul_t_int(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                             ctypes.c_int64(d_), O._p(O._i64(a.reshape(-1))), O._p(O._i64(b.reshape(-1))),
                             ctypes.c_int64(za), ctypes.c_int64(zb), ctypes.c_int(int(i48)), O._p(out))
    return out.reshape(n, h, w)


def oracle_t_float(a, b, ot):
    n, h, c = a.shape
    d_, w, _ = b.shape
    out = np.zeros(n * h * w, dtype=np.float32)
    O.lib().orc_matmul_t_float(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                               ctypes.c_int64(d_), O._p(O._f32(a.reshape(-1))), O._p(O._f32(b.reshape(-1))),
                               ctypes.c_int(ot), O._p(out))
    return out.reshape(n, h, w)


INT8_SHAPES = [
    # n, h, c, w, d, za, zb
    (1, 128, 128, 128, 1, 0, 0),
    (2, 200, 96, 160, 2, -5, 7),      # M tail, K < BK, N tail with BN=256
    (3, 130, 256, 64, 1, 3, 0),       # broadcast B, a_zp only
    (2, 64, 1024, 384, 2, 0, -8),     # b_zp only, N spans 2 tiles
    (4, 257, 528, 272, 1, -128, 127), # broadcast, extreme zero points
    (1, 64, 2048, 1000, 1, 5, -3),    # w = 1000: K-major B needs no padding
    (2, 96, 128, 20, 2, -7, 0),
    (2, 33, 40, 24, 1, 2, -1),        # c % 16 != 0: direct kernel
]


@pytest.mark.parametrize("n,h,c,w,d,za,zb", INT8_SHAPES)
def test_matmul_t_int8(ctx, n, h, c, w, d, za, zb):
    rng = np.random.default_rng(n * 1000 + h + c + w + d)
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    b = rng.integers(-128, 128, (d, w, c), dtype=np.int64)
    got = run_t(ctx, a, b, L.DT_INT8, L.DT_INT8, L.DT_INT32, za, zb)
    assert np.array_equal(got.astype(np.int64), oracle_t_int(a, b, za, zb))


@pytest.mark.parametrize("d", [1, 2])
@pytest.mark.parametrize("per_channel", [False, True])
def test_matmul_t_int8_fused_rescale(ctx, d, per_channel):
    rng = np.random.default_rng(17 + d + per_channel)
    n, h, c, w = 2, 160, 256, 192
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    b = rng.integers(-128, 128, (d, w, c), dtype=np.int64)
    za, zb = int(rng.integers(-8, 9)), int(rng.integers(-8, 9))
    ch = w if per_channel else 1
    mult = rng.integers(1 << 30, (1 << 31) - 1, ch)
    shift = rng.integers(32, 40, ch)
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, per_channel=per_channel, output_zp=5,
                          out_dtype=L.DT_INT8)
    got = run_t(ctx, a, b, L.DT_INT8, L.DT_INT8, L.DT_INT32, za, zb, rescale=attr)
    acc = oracle_t_int(a, b, za, zb).reshape(-1)
    rc, exp = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, 5, 1, L.ROUND_DOUBLE, int(per_channel))
    assert rc == 0
    assert np.array_equal(got.reshape(-1).astype(np.int64), exp)


@pytest.mark.parametrize("d", [1, 3])
def test_matmul_t_int8_constant_b(ctx, d):
    """set_constant_b computes the a_zp column terms of a K-major B once; runs reuse them."""
    rng = np.random.default_rng(40 + d)
    n, h, c, w = 3, 100, 320, 136
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
    b = rng.integers(-128, 128, (d, w, c), dtype=np.int64)
    got = run_t(ctx, a, b, L.DT_INT8, L.DT_INT8, L.DT_INT32, -9, 4, plan_const=True)
    assert np.array_equal(got.astype(np.int64), oracle_t_int(a, b, -9, 4))


def test_matmul_t_int16(ctx):
    rng = np.random.default_rng(5)
    a = rng.integers(-32768, 32768, (2, 12, 40), dtype=np.int64)
    b = rng.integers(-32768, 32768, (1, 23, 40), dtype=np.int64)
    got = run_t(ctx, a, b, L.DT_INT16, L.DT_INT16, L.DT_INT48)
    assert np.array_equal(got.astype(np.int64), oracle_t_int(a, b, 0, 0, i48=True))


FLOAT_DIRECT = [
    (L.DT_FP16, L.DT_FP32, L.DT_FP32),
    (L.DT_BF16, L.DT_FP8E4M3, L.DT_BF16),
    (L.DT_FP16, L.DT_BF16, L.DT_BF16),   # F16 operand rounded to BF16 first
    (L.DT_FP8E5M2, L.DT_FP16, L.DT_FP32),
    (L.DT_FP16, L.DT_FP16, L.DT_FP16),
    (L.DT_BF16, L.DT_BF16, L.DT_BF16),
    (L.DT_FP32, L.DT_FP32, L.DT_FP32),
]


@pytest.mark.parametrize("at,bt,ot", FLOAT_DIRECT)
@pytest.mark.parametrize("d", [1, 2])
def test_matmul_t_float_direct(ctx, at, bt, ot, d):
    """Direct kernels in the reference's loop order: bit-exact."""
    rng = np.random.default_rng(at * 100 + bt * 10 + ot + d)
    n, h, c, w = 2, 19, 37, 23
    a = _values(rng, at, (n, h, c))
    b = _values(rng, bt, (d, w, c))
    got = run_t(ctx, a, b, at, bt, ot)
    exp = oracle_t_float(a, b, ot)
    assert np.array_equal(O.to_bits(ot, got.reshape(-1).astype(np.float32)), O.to_bits(ot, exp.reshape(-1)))


@pytest.mark.parametrize("dt", [L.DT_BF16, L.DT_FP16])
@pytest.mark.parametrize("d", [1, 2])
def test_matmul_t_float_tensor_core(ctx, dt, d):
    rng = np.random.default_rng(dt + d)
    n, h, c, w = 2, 200, 192, 144
    a = _values(rng, dt, (n, h, c))
    b = _values(rng, dt, (d, w, c))
    got = run_t(ctx, a, b, dt, dt, L.DT_FP32).astype(np.float64)
    exp = oracle_t_float(a, b, L.DT_FP32).astype(np.float64)
    bb = np.broadcast_to(b, (n, w, c)) if d == 1 else b
    floor = np.einsum("nhc,nwc->nhw", np.abs(a.astype(np.float64)), np.abs(bb.astype(np.float64)))
    e = np.floor(np.log2(np.maximum(np.abs(exp), 2.0 ** -126)))
    tol = 2 * 2.0 ** (e - 7) + 2.0 ** -16 * floor
    assert np.all(np.abs(got - exp) <= tol)


def test_matmul_t_rejects(ctx):
    """Shape and type errors of matmul.rs:117-137 are reported, not run."""
    shape_mismatch, dtype_mismatch, graph_error = 5, 4, 7  # tb_status codes
    lib = L.load()
    plan = ctypes.c_void_p()
    bad_batch = L.MatmulDesc(n=3, h=4, c=16, w=8, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32)
    assert lib.tb_matmul_t_plan_create(ctx.h, bad_batch, 2, None, ctypes.byref(plan)) == shape_mismatch
    f16_f16_bf16 = L.MatmulDesc(n=1, h=4, c=16, w=8, a_dtype=L.DT_FP16, b_dtype=L.DT_FP16, out_dtype=L.DT_BF16)
    assert lib.tb_matmul_t_plan_create(ctx.h, f16_f16_bf16, 1, None, ctypes.byref(plan)) == dtype_mismatch
    zp_float = L.MatmulDesc(n=1, h=4, c=16, w=8, a_dtype=L.DT_BF16, b_dtype=L.DT_BF16, out_dtype=L.DT_FP32, a_zp=1)
    assert lib.tb_matmul_t_plan_create(ctx.h, zp_float, 1, None, ctypes.byref(plan)) == graph_error
