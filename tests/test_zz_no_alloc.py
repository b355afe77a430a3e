"""The allocation-free MATMUL entry point (tb_matmul_i8_noalloc).

It serves callers that cannot call cudaMalloc themselves or through this
library -- for example code whose device memory is owned by another
allocator, or code running where allocation is not allowed -- by keeping the
kernel's scratch (column sums for the a zero point, a cross-CTA counter, the
packed RESCALE constants, the error word) in a fixed file-scope device array.

The checks: its results equal the regular entry point's (tb_matmul, which
allocates per-plan scratch) bit for bit -- integer results, so the tolerance
is exact -- on two calls in a row with different inputs, zero points and
rescale constants (the array keeps the previous call's contents, so stale
scratch would show), and shapes beyond the array's limit are rejected.

This file is collected last so a run that stops at the first failure has run
every other test; it also passes on its own in a fresh process.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tosa_b200 import _lib as L  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


def _inputs(seed, n, h, c, w):
    rng = np.random.default_rng(seed)
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int8)
    b = rng.integers(-128, 128, (n, c, w), dtype=np.int8)
    za, zb = int(rng.integers(-8, 9)), int(rng.integers(-8, 9))
    mult = rng.integers(1 << 30, (1 << 31) - 1, w)
    shift = rng.integers(32, 40, w)
    return a, b, za, zb, mult, shift


def _run(fn_name, ctx, a, b, za, zb, attr):
    n, h, c = a.shape
    w = b.shape[2]
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32,
                     a_zp=za, b_zp=zb)
    ta = torch.from_numpy(a).cuda()
    tb = torch.from_numpy(b).cuda()
    odt = torch.int8 if attr is not None else torch.int32
    out = torch.full((n, h, w), 77, dtype=odt, device="cuda")
    lib = L.load()
    if fn_name == "noalloc":
        L.check(lib.tb_matmul_i8_noalloc(d, attr, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
    else:
        L.check(lib.tb_matmul(ctx.h, d, attr, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
        ctx.synchronize()
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("shape", [(2, 192, 256, 320), (3, 130, 128, 96)])
def test_noalloc_matches_regular_entry_point_twice(ctx, shape):
    n, h, c, w = shape
    for call, seed in enumerate((101, 202)):
        a, b, za, zb, mult, shift = _inputs(seed + n, n, h, c, w)
        rounding = L.ROUND_DOUBLE if call == 0 else L.ROUND_SINGLE
        attr = L.rescale_attr(mult, shift, rounding=rounding, output_zp=3 - call, out_dtype=L.DT_INT8)
        want = _run("regular", ctx, a, b, za, zb, attr)
        got = _run("noalloc", ctx, a, b, za, zb, attr)
        assert np.array_equal(got, want), f"call {call}"
        # the int32 result without RESCALE too
        want32 = _run("regular", ctx, a, b, za, zb, None)
        got32 = _run("noalloc", ctx, a, b, za, zb, None)
        assert np.array_equal(got32, want32), f"call {call} (int32)"


def test_noalloc_rejects_shapes_beyond_its_array(ctx):
    n, h, c, w = 2, 16, 64, 131072 // 2 + 16  # n*w above the 131072 limit, a_zp != 0
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32,
                     a_zp=1, b_zp=0)
    dummy = torch.zeros(16, dtype=torch.int8, device="cuda")
    status = L.load().tb_matmul_i8_noalloc(d, None, L.ptr(dummy), L.ptr(dummy), L.ptr(dummy), L.stream_ptr())
    assert status == 66  # TB_ERR_INVALID_ARGUMENT
    assert b"scratch limit" in L.load().tb_last_error()
