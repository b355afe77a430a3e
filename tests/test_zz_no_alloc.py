"""The allocation-free MATMUL entry point (tb_matmul_i8_noalloc).

It serves callers that cannot call cudaMalloc themselves or through this
library -- for example code whose device memory is owned by another
allocator, or code running where allocation is not allowed -- by keeping the
kernel's scratch (column terms for the a zero point, the packed RESCALE
constants, the error word) in a fixed file-scope device array.

The checks: its results equal the regular entry point's (tb_matmul, which
allocates per-plan scratch) and the oracle's bit for bit -- integer results,
so the tolerance is exact -- on two calls in a row with different inputs,
zero points and rescale constants (the array keeps the previous call's
contents, so stale scratch would show). The shapes reach every path the entry
point takes: the tensor cores (w % 16 == 0, aligned operands), and the direct
kernel for B rows that are not 16-byte multiples (an odd w, and 1000 classes,
which the regular entry point pads) and for an A that starts one byte past an
aligned address; the rescale runs at its 16384-channel limit. Shapes beyond
the array's limits are rejected.

This file is collected last so a run that stops at the first failure has run
every other test; it also passes on its own in a fresh process.
"""

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


def _inputs(seed, n, h, c, w):
    rng = np.random.default_rng(seed)
    a = rng.integers(-128, 128, (n, h, c), dtype=np.int8)
    b = rng.integers(-128, 128, (n, c, w), dtype=np.int8)
    za = int(rng.integers(-8, 9)) or 5
    zb = int(rng.integers(-8, 9))
    mult = rng.integers(1 << 30, (1 << 31) - 1, w)
    shift = rng.integers(32, 40, w)
    return a, b, za, zb, mult, shift


def _device(arr, offset=0):
    """A device copy of `arr` that starts `offset` bytes past a 256-byte-aligned address."""
    flat = torch.zeros(arr.nbytes + 256, dtype=torch.int8, device="cuda")
    view = flat[offset:offset + arr.nbytes]
    view.copy_(torch.from_numpy(np.ascontiguousarray(arr).reshape(-1)).cuda())
    return flat, view


def _run(fn_name, ctx, a, b, za, zb, attr, a_offset=0):
    n, h, c = a.shape
    w = b.shape[2]
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32,
                     a_zp=za, b_zp=zb)
    _keep, ta = _device(a, a_offset)
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


def _oracle(a, b, za, zb, mult, shift, rounding, out_zp):
    acc = H.oracle_matmul_int(a, b, za, zb)
    if mult is None:
        return acc
    rc, q = H.oracle_rescale(acc, 5, 3, list(mult), list(shift), 0, out_zp, 1, rounding, int(len(mult) > 1))
    assert rc == 0
    return q.reshape(acc.shape)


# (n, h, c, w, A byte offset): tensor cores; 1000 classes (B rows not 16-byte multiples, padded by
# the regular entry point, direct here); an odd w (direct in both); A one byte off alignment (direct)
SHAPES = [(2, 192, 256, 320, 0), (3, 130, 128, 96, 0), (1, 64, 256, 1000, 0), (2, 37, 48, 23, 0),
          (2, 70, 64, 96, 1)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_noalloc_matches_regular_entry_point_twice(ctx, shape):
    n, h, c, w, off = shape
    for call, seed in enumerate((101, 202)):
        a, b, za, zb, mult, shift = _inputs(seed + n + w, n, h, c, w)
        rounding = L.ROUND_DOUBLE if call == 0 else L.ROUND_SINGLE
        out_zp = 3 - call
        attr = L.rescale_attr(mult, shift, rounding=rounding, output_zp=out_zp, out_dtype=L.DT_INT8)
        want = _run("regular", ctx, a, b, za, zb, attr)
        got = _run("noalloc", ctx, a, b, za, zb, attr, a_offset=off)
        assert np.array_equal(got, want), f"call {call}"
        assert np.array_equal(got.astype(np.int64), _oracle(a, b, za, zb, mult, shift, rounding, out_zp)), \
            f"call {call} (oracle)"
        # the int32 result without RESCALE too
        want32 = _run("regular", ctx, a, b, za, zb, None)
        got32 = _run("noalloc", ctx, a, b, za, zb, None, a_offset=off)
        assert np.array_equal(got32, want32), f"call {call} (int32)"
        assert np.array_equal(got32.astype(np.int64), _oracle(a, b, za, zb, None, None, 0, 0)), \
            f"call {call} (int32, oracle)"


def test_noalloc_rescale_at_channel_limit(ctx):
    """16384 per-channel multipliers and shifts: the largest RESCALE the array holds."""
    n, h, c, w = 1, 64, 64, 16384
    for call, seed in enumerate((7, 8)):
        a, b, za, zb, mult, shift = _inputs(seed, n, h, c, w)
        attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=-2 + call, out_dtype=L.DT_INT8)
        want = _run("regular", ctx, a, b, za, zb, attr)
        got = _run("noalloc", ctx, a, b, za, zb, attr)
        assert np.array_equal(got, want), f"call {call}"
        assert np.array_equal(got.astype(np.int64), _oracle(a, b, za, zb, mult, shift, L.ROUND_DOUBLE, -2 + call))


def test_noalloc_rejects_shapes_beyond_its_array(ctx):
    lib = L.load()
    dummy = torch.zeros(16, dtype=torch.int8, device="cuda")
    n, h, c, w = 2, 16, 64, 131072 // 2 + 16  # n*w above the 131072 limit, a_zp != 0
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32,
                     a_zp=1, b_zp=0)
    status = lib.tb_matmul_i8_noalloc(d, None, L.ptr(dummy), L.ptr(dummy), L.ptr(dummy), L.stream_ptr())
    assert status == 66  # TB_ERR_INVALID_ARGUMENT
    assert b"scratch limit" in lib.tb_last_error()
    # one rescale channel more than the array holds
    w = 16384 + 16
    d = L.MatmulDesc(n=1, h=16, c=64, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32,
                     a_zp=0, b_zp=0)
    attr = L.rescale_attr([1 << 30] * w, [35] * w, out_dtype=L.DT_INT8)
    status = lib.tb_matmul_i8_noalloc(d, attr, L.ptr(dummy), L.ptr(dummy), L.ptr(dummy), L.stream_ptr())
    assert status == 66
    assert b"scratch limit" in lib.tb_last_error()
