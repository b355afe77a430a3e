"""GEMMs whose output tiles would leave SMs idle: narrower tiles.

A contraction with few 128-row output tiles (a classifier over one batch of images, the 7x7
and 14x14 layers of ResNet-50 at 64 images) takes 128- or 64-column tiles instead of 256
while their count still fits one wave of the SMs. These shapes take that path: int8 MATMULs
of 64-256 rows over K = 1536-2048 into 384-1024 columns (partial row tiles included), a
MATMUL_T with a B shared by both batches, and a 3x3 convolution of 6400 output pixels into
256 channels (100 tiles of 128 columns rather than 50 of 256). Each runs twice through one
plan with per-tensor and per-channel RESCALE, single and double rounding, an A / input zero
point and a clamp, bit-exact against the oracle.
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tests import helpers as H  # noqa: E402
from tosa_b200 import _lib as L  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


def _rescale(rng, channels, rounding, out_zp, clamp=None):
    mult = rng.integers(1 << 30, (1 << 31) - 1, channels)
    shift = rng.integers(36, 41, channels)
    attr = L.rescale_attr(mult, shift, rounding=rounding, per_channel=channels > 1, output_zp=out_zp,
                          out_dtype=L.DT_INT8, clamp=clamp)
    return attr, mult, shift


def _oracle_rescale(acc, mult, shift, rounding, out_zp, clamp=None):
    rc, q = H.oracle_rescale(acc, 5, 3, list(mult), list(shift), 0, out_zp, 1, rounding, int(len(mult) > 1))
    assert rc == 0
    q = q.reshape(acc.shape)
    if clamp is not None:
        q = np.clip(q, clamp[0], clamp[1])
    return q


MM_CASES = [
    # (n, h, c, w, a_zp, per_channel, rounding, clamp)
    (1, 256, 2048, 512, 0, False, L.ROUND_SINGLE, None),
    (1, 256, 2048, 512, 3, True, L.ROUND_DOUBLE, (-20, 127)),
    (1, 64, 2048, 1024, -5, True, L.ROUND_DOUBLE, None),
    (2, 130, 1536, 384, 2, False, L.ROUND_DOUBLE, None),
]


@pytest.mark.parametrize("case", MM_CASES, ids=lambda c: "x".join(map(str, c[:4])) + f"_za{c[4]}")
def test_few_tile_matmul_twice(ctx, case):
    n, h, c, w, za, pc, rounding, clamp = case
    lib = L.load()
    rng = np.random.default_rng(h + c + w)
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32, a_zp=za, b_zp=0)
    attr, mult, shift = _rescale(rng, w if pc else 1, rounding, 4, clamp)
    plan = ctypes.c_void_p()
    L.check(lib.tb_matmul_plan_create(ctx.h, d, attr, ctypes.byref(plan)))
    try:
        for run in range(2):
            a = rng.integers(-128, 128, (n, h, c), dtype=np.int8)
            b = rng.integers(-128, 128, (n, c, w), dtype=np.int8)
            ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
            out = torch.full((n, h, w), 99, dtype=torch.int8, device="cuda")
            L.check(lib.tb_matmul_plan_run(plan, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
            ctx.synchronize()
            acc = H.oracle_matmul_int(a.astype(np.int64), b.astype(np.int64), za, 0)
            want = _oracle_rescale(acc, mult, shift, rounding, 4, clamp)
            assert np.array_equal(out.cpu().numpy().astype(np.int64), want), f"run {run}"
    finally:
        lib.tb_matmul_plan_destroy(plan)


def test_few_tile_matmul_t(ctx):
    """MATMUL_T: A [2,128,2048] x B [1,384,2048] shared by both batches (6 tiles of 128)."""
    lib = L.load()
    rng = np.random.default_rng(77)
    n, h, c, w = 2, 128, 2048, 384
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32, a_zp=-3, b_zp=0)
    attr, mult, shift = _rescale(rng, w, L.ROUND_DOUBLE, -2)
    plan = ctypes.c_void_p()
    L.check(lib.tb_matmul_t_plan_create(ctx.h, d, 1, attr, ctypes.byref(plan)))
    try:
        for run in range(2):
            a = rng.integers(-128, 128, (n, h, c), dtype=np.int8)
            bt = rng.integers(-128, 128, (1, w, c), dtype=np.int8)
            ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(bt).cuda()
            out = torch.full((n, h, w), 99, dtype=torch.int8, device="cuda")
            L.check(lib.tb_matmul_plan_run(plan, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
            ctx.synchronize()
            b = np.broadcast_to(np.transpose(bt, (0, 2, 1)), (n, c, w)).astype(np.int64)
            acc = H.oracle_matmul_int(a.astype(np.int64), b, -3, 0)
            want = _oracle_rescale(acc, mult, shift, L.ROUND_DOUBLE, -2)
            assert np.array_equal(out.cpu().numpy().astype(np.int64), want), f"run {run}"
    finally:
        lib.tb_matmul_plan_destroy(plan)


def _conv_plan(ctx, n, hw, ic, oc, rounding, rng):
    d = L.conv_desc(n, hw, hw, ic, oc, 3, 3, (1, 1, 1, 1), (1, 1), (1, 1), L.DT_INT8, L.DT_INT8, L.DT_INT32,
                    L.DT_INT32, -3, 0, oc)
    w = rng.integers(-127, 128, (oc, 3, 3, ic), dtype=np.int8)
    bias = rng.integers(-40000, 40000, oc).astype(np.int32)
    attr, mult, shift = _rescale(rng, oc, rounding, 5, (5, 127))
    tw, tbias = torch.from_numpy(w).cuda(), torch.from_numpy(bias).cuda()
    plan = ctypes.c_void_p()
    L.check(L.load().tb_conv2d_plan_create(ctx.h, d, L.ptr(tw), L.ptr(tbias), attr, ctypes.byref(plan)))
    return plan, (w, bias, mult, shift, tw, tbias, attr)


def test_few_tile_conv3x3_twice(ctx):
    """[4,40,40,128] 3x3 -> 256: 50 row tiles x 2 column tiles of 128, K = 9 x 128 channels."""
    lib = L.load()
    rng = np.random.default_rng(5)
    n, hw, ic, oc = 4, 40, 128, 256
    plan, (w, bias, mult, shift, *_keep) = _conv_plan(ctx, n, hw, ic, oc, L.ROUND_DOUBLE, rng)
    try:
        for run in range(2):
            x = rng.integers(-128, 128, (n, hw, hw, ic), dtype=np.int8)
            tx = torch.from_numpy(x).cuda()
            out = torch.full((n, hw, hw, oc), 99, dtype=torch.int8, device="cuda")
            L.check(lib.tb_conv2d_plan_run(plan, L.ptr(tx), L.ptr(out), L.stream_ptr()))
            ctx.synchronize()
            acc = H.oracle_conv_int(x.astype(np.int64), w.astype(np.int64), bias.astype(np.int64), -3, 0,
                                    (1, 1, 1, 1), (1, 1), (1, 1))
            want = _oracle_rescale(acc, mult, shift, L.ROUND_DOUBLE, 5, (5, 127))
            assert np.array_equal(out.cpu().numpy().astype(np.int64), want), f"run {run}"
    finally:
        lib.tb_conv2d_plan_destroy(plan)
