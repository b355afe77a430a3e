"""Parity at the benchmark sizes, and under both forms of the GEMM epilogue.

The tensor-core GEMM gives each tile's epilogue to its three groups of four
warps in one of two ways: by column thirds (few tiles per CTA, or tiles of 256
columns), or whole tiles to the groups in turn (tiles of at most 128 columns,
several per CTA, i.e. only at large batch). Small parity shapes never reach
the second form on their own, so the first
test forces each form (TB_GEMM_EPI_GROUPS at context creation) over the
output widths and epilogue variants the benchmark graphs use: 32 to 256
output channels, the fused per-channel RESCALE + CLAMP and the int32 result,
weight zero points (row terms) and border classes, two taps per stage,
strided windows and the im2col-row stem.

The rest run the benchmark shapes themselves at 64 images with the library's
own choices, and compare the first and the last image bit for bit with the
oracle (the convolutions, pools and graphs are per image, so two whole images
cover every border class): the layers of the ResNet-50-shaped graph
(7x7/s2 stem, 3x3 convolutions over 64 channels with two taps per stage, the
1x1 expansions and projections, the strided 3x3, the 3x3/s2 max pool, the
1000-class classifier with a constant, padded B replayed from a CUDA graph),
and the whole ResNet-50- and MobileNetV2-shaped graphs of BASELINE configs 3
and 4 in fused and CUDA-graph modes (conv.rs:147-181, type_conv.rs:174-188,
pool.rs:164-286, matmul.rs:80-95, composed by interpreter.rs:154-245).
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tests.test_gpu_contractions import run_conv  # noqa: E402
from tosa_b200 import _lib as L  # noqa: E402
from tosa_b200 import graphs  # noqa: E402
from tosa_b200 import interpreter as I  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


def _same(size, k, s):
    """TF 'SAME' padding (before, after), as the benchmark graphs use."""
    pb, pa, _ = graphs.GraphBuilder.same_pads(size, k, s)
    return pb, pa


def _conv_case(rng, n, ih, iw, ic, oc, k, stride, zx, zw):
    """Uniform int8 activations and weights; per-channel multipliers in [2^30, 2^31) with
    shifts around the one that maps the accumulator's spread to about 24 int8 steps, so the
    outputs span the int8 range instead of saturating."""
    pt, pb = _same(ih, k, stride)
    pl, pr = _same(iw, k, stride)
    x = rng.integers(-128, 128, (n, ih, iw, ic), dtype=np.int64)
    w = rng.integers(-127, 128, (oc, k, k, ic), dtype=np.int64)
    bias = rng.integers(-40000, 40000, oc, dtype=np.int64)
    mult = rng.integers(1 << 30, (1 << 31) - 1, oc)
    spread = 74.0 * 74.0 * np.sqrt(k * k * ic)
    base = int(np.round(np.log2(spread / 24.0))) + 31
    shift = rng.integers(base - 1, base + 2, oc)
    return x, w, bias, (pt, pb, pl, pr), (stride, stride), mult, shift


def _oracle_fused(x, w, bias, zx, zw, pad, stride, mult, shift, out_zp, clamp):
    acc = H.oracle_conv_int(x, w, bias, zx, zw, pad, stride, (1, 1))
    rc, q = H.oracle_rescale(acc, L.DT_INT32, L.DT_INT8, mult, shift, 0, out_zp, 1, L.ROUND_DOUBLE, 1)
    assert rc == 0
    q = q.reshape(acc.shape)
    return acc, (np.clip(q, *clamp) if clamp is not None else q)


# (n, ih, iw, ic, oc, k, stride, zx, zw)
EPI_CASES = [
    (2, 14, 14, 64, 64, 1, 1, 3, 0),     # BN 64, one 32-column staging group per pass
    (2, 14, 14, 64, 64, 3, 1, -5, 0),    # BN 64, two taps per stage, border classes
    (2, 14, 14, 64, 32, 3, 1, 4, 0),     # 32 channels: the second half of BN 64 is empty
    (2, 14, 14, 32, 96, 1, 1, -2, 4),    # BN 128 with a partial last group and row terms
    (2, 14, 14, 64, 256, 1, 1, 6, 0),    # BN 256
    (2, 15, 15, 64, 128, 3, 2, 1, -2),   # strided, border classes and row terms
    (2, 30, 30, 3, 64, 7, 2, -4, 0),     # few-channel stem: im2col rows, then a 1x1 GEMM
]


@pytest.mark.parametrize("groups", [0, 1], ids=["column_thirds", "whole_tiles"])
@pytest.mark.parametrize("case", EPI_CASES, ids=lambda c: "x".join(map(str, c)))
def test_conv_epilogue_forms(monkeypatch, case, groups):
    n, ih, iw, ic, oc, k, stride, zx, zw = case
    monkeypatch.setenv("TB_GEMM_EPI_GROUPS", str(groups))
    c = L.Context(0)
    try:
        rng = np.random.default_rng(ih * 1000 + ic * 10 + oc + k)
        x, w, bias, pad, st, mult, shift = _conv_case(rng, n, ih, iw, ic, oc, k, stride, zx, zw)
        out_zp = -3
        acc, want = _oracle_fused(x, w, bias, zx, zw, pad, st, mult, shift, out_zp, (out_zp, 127))
        attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=out_zp, out_dtype=L.DT_INT8,
                              clamp=(out_zp, 127))
        got = run_conv(c, x, w, bias, zx, zw, pad, st, (1, 1), rescale=attr)
        assert np.array_equal(got.astype(np.int64), want)
        got32 = run_conv(c, x, w, bias, zx, zw, pad, st, (1, 1))
        assert np.array_equal(got32.astype(np.int64), acc)
    finally:
        c.close()


# ---------------------------------------------------------------------------
# ResNet-50 layers at 64 images
# ---------------------------------------------------------------------------

# (name, ih, ic, oc, k, stride, zx): the shapes of the ResNet-50-shaped graph (tosa_b200/graphs.py)
R50_LAYERS = [
    ("stem_7x7s2", 224, 3, 64, 7, 2, -4),
    ("conv3x3_64", 56, 64, 64, 3, 1, 5),
    ("conv1x1_64_256", 56, 64, 256, 1, 1, -7),
    ("conv1x1_256_64", 56, 256, 64, 1, 1, 2),
    ("conv3x3s2_128", 56, 128, 128, 3, 2, -1),
    ("conv1x1_2048_512", 7, 2048, 512, 1, 1, 3),
]
IMAGES = [0, 63]


@pytest.mark.parametrize("layer", R50_LAYERS, ids=lambda l: l[0])
def test_resnet50_layer_batch64(ctx, layer):
    _, ih, ic, oc, k, stride, zx = layer
    rng = np.random.default_rng(ih + ic + oc + k)
    x, w, bias, pad, st, mult, shift = _conv_case(rng, 64, ih, ih, ic, oc, k, stride, zx, 0)
    out_zp = 4
    attr = L.rescale_attr(mult, shift, rounding=L.ROUND_DOUBLE, output_zp=out_zp, out_dtype=L.DT_INT8,
                          clamp=(out_zp, 127))
    got = run_conv(ctx, x, w, bias, zx, 0, pad, st, (1, 1), rescale=attr)
    _, want = _oracle_fused(x[IMAGES], w, bias, zx, 0, pad, st, mult, shift, out_zp, (out_zp, 127))
    assert np.array_equal(got[IMAGES].astype(np.int64), want)


def test_resnet50_max_pool_batch64(ctx):
    """MAX_POOL2D 3x3/s2 (SAME padding) over [64, 112, 112, 64]."""
    rng = np.random.default_rng(112)
    x = rng.integers(-128, 128, (64, 112, 112, 64), dtype=np.int8)
    pt, pb = _same(112, 3, 2)
    pad = (pt, pb, pt, pb)
    d = L.Pool2dDesc()
    d.n, d.ih, d.iw, d.c = 64, 112, 112, 64
    d.kernel[0] = d.kernel[1] = 3
    d.stride[0] = d.stride[1] = 2
    for i in range(4):
        d.pad[i] = pad[i]
    d.dtype, d.acc_dtype, d.nan_mode = L.DT_INT8, L.DT_INT32, L.NAN_PROPAGATE
    tx = torch.from_numpy(x).cuda()
    out = torch.empty((64, 56, 56, 64), dtype=torch.int8, device="cuda")
    L.check(L.load().tb_max_pool2d(ctx.h, d, L.ptr(tx), L.ptr(out), L.stream_ptr()))
    ctx.synchronize()
    xs = np.ascontiguousarray(x[IMAGES], np.int64)
    g = H.pool_geom(xs.shape, (3, 3), (2, 2), pad)
    exp = np.zeros(2 * 56 * 56 * 64, dtype=np.int64)
    O.lib().orc_max_pool_int(ctypes.byref(g), xs.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(L.DT_INT8),
                             exp.ctypes.data_as(ctypes.c_void_p))
    assert np.array_equal(out.cpu().numpy()[IMAGES].reshape(-1).astype(np.int64), exp)


@pytest.mark.parametrize("zb", [0, -3])
def test_classifier_constant_padded_b_cuda_graph(ctx, zb):
    """The 1000-class classifier [1,64,2048] x [1,2048,1000]: B rows are not 16-byte
    multiples (padded once, as a constant B), the launch is captured into a CUDA graph
    and replayed with new activations; both replays exact."""
    rng = np.random.default_rng(1000 - zb)
    n, h, c, w = 1, 64, 2048, 1000
    za = 3
    b = rng.integers(-127, 128, (n, c, w), dtype=np.int64)
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32, a_zp=za, b_zp=zb)
    lib = L.load()
    plan = ctypes.c_void_p()
    L.check(lib.tb_matmul_plan_create(ctx.h, d, None, ctypes.byref(plan)))
    try:
        tb = torch.from_numpy(b.astype(np.int8)).cuda()
        ta = torch.empty((n, h, c), dtype=torch.int8, device="cuda")
        out = torch.empty((n, h, w), dtype=torch.int32, device="cuda")
        s = torch.cuda.Stream()
        L.check(lib.tb_matmul_plan_set_constant_b(plan, L.ptr(tb), L.stream_ptr(s)))
        ta.copy_(torch.from_numpy(rng.integers(-128, 128, (n, h, c), dtype=np.int8)))
        L.check(lib.tb_matmul_plan_run(plan, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr(s)))  # warm-up
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            L.check(lib.tb_matmul_plan_run(plan, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr(s)))
        for rep in range(2):
            a = rng.integers(-128, 128, (n, h, c), dtype=np.int64)
            ta.copy_(torch.from_numpy(a.astype(np.int8)))
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            ctx.synchronize()
            assert np.array_equal(out.cpu().numpy().astype(np.int64), H.oracle_matmul_int(a, b, za, zb)), rep
        del graph
    finally:
        lib.tb_matmul_plan_destroy(plan)


# ---------------------------------------------------------------------------
# The benchmark graphs at 64 images
# ---------------------------------------------------------------------------

_ORACLE = {}


def _oracle_images(name, images):
    """Logits of the given images through the oracle's batch-1 graph (cached per graph)."""
    if name not in _ORACLE:
        d1, info = getattr(graphs, name + "_int8")(1)
        block = O.read_graph(d1).main_block
        res = []
        for i in IMAGES:
            r = O.run_block(block, {info["input"]: O.T(3, [1, 224, 224, 3], images[i].astype(np.int64).reshape(-1))})
            res.append(next(iter(r.values())).values)
        _ORACLE[name] = res
    return _ORACLE[name]


@pytest.mark.parametrize("mode", ["fused", "cuda_graph"])
@pytest.mark.parametrize("name", ["resnet50", "mobilenetv2"])
def test_benchmark_graph_batch64(ctx, name, mode):
    data, info = getattr(graphs, name + "_int8")(64)
    rng = np.random.default_rng(21)
    images = rng.integers(-128, 128, (64, 224, 224, 3), dtype=np.int8)
    want = _oracle_images(name, images)
    it = I.Interpreter(data, context=ctx, cuda_graph=mode == "cuda_graph")
    try:
        it.bind({info["input"]: I.Tensor.from_numpy(info["input"], images, L.DT_INT8)})
        s = torch.cuda.Stream()
        for _ in range(2 if mode == "cuda_graph" else 1):
            it.execute(stream=s)
            s.synchronize()
        got = it.output(info["output"]).data.reshape(64, -1).astype(np.int64)
    finally:
        it.close()
    for k, i in enumerate(IMAGES):
        bad = np.nonzero(got[i] != want[k])[0]
        assert bad.size == 0, f"image {i}: {bad.size}/{got.shape[1]} logits differ, first at {bad[:5]}"
