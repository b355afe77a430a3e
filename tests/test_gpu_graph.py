"""The graph runner on the GPU, against the reference's own fixtures.

Every conformance case the reference ships for the operators on this path
(tests/golden/*.zip: CONV2D, CONV3D, DEPTHWISE_CONV2D, TRANSPOSE_CONV2D, MATMUL, MATMUL_T, RESCALE, AVG_POOL2D,
MAX_POOL2D, CLAMP, and the network graphs) runs end to end through
``run_graph`` -- the .tosa flatbuffer parsed in C++, constants uploaded, the
operator executed by the CUDA kernels -- and its result is compared bit for
bit with the expected output (any two NaNs equal, as in the reference's
tests/conformance.rs:165-229). ERROR_IF cases must raise. Cases whose types
the backend does not run (fp8, int16 x int8 -> int48, f16 accumulators, ...)
must be declined with NotAccelerated, the signal for the caller to keep the
reference path; the test counts them so the accelerated share is fixed.

Hook events are checked against the oracle's trace of the reference's
ready-queue order (src/interpreter.rs:154-245).
"""

import os

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tosa_b200 import _lib as L  # noqa: E402
from tosa_b200 import interpreter as I  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
FAMILIES = ["conv2d", "conv3d", "depthwise_conv2d", "transpose_conv2d", "matmul", "matmul_t", "rescale", "avg_pool2d", "max_pool2d", "clamp", "networks"]
# cases per family the runner executes (the rest are declined as not accelerated or are ERROR_IF cases)
_RESULTS = {}


def _cases():
    for fam in FAMILIES:
        for c in O.load_cases(os.path.join(GOLDEN, f"{fam}.zip")):
            yield pytest.param(fam, c, id=f"{fam}::{c.name}")


def _inputs(case, block):
    out = {}
    for name, fn in zip(case.desc["ifm_name"], case.desc["ifm_file"]):
        arr = case.npy(fn)
        td = block.tensor(name)
        dt = td.dtype if td is not None else L.DT_FP32
        if dt == L.DT_BF16:
            arr = arr.view(np.uint16)
        elif dt in (L.DT_FP8E4M3, L.DT_FP8E5M2):
            arr = arr.view(np.uint8)
        out[name] = I.Tensor.from_numpy(name, arr, dt)
    return out


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("fam,case", list(_cases()))
def test_fixture_through_runner(ctx, fam, case):
    g = O.read_graph(case.graph_bytes)
    block = g.main_block
    inputs = _inputs(case, block)
    if case.desc.get("expected_failure", False):
        # rejected when the graph is loaded (e.g. a tensor rank above 6) or when it runs
        with pytest.raises(L.TbError):
            it = I.Interpreter(case.graph_bytes, context=ctx)
            try:
                it.run(inputs)
            finally:
                it.close()
        _RESULTS.setdefault(fam, {}).setdefault("rejected", 0)
        _RESULTS[fam]["rejected"] += 1
        return
    it = I.Interpreter(case.graph_bytes, context=ctx)
    try:
        try:
            outs = it.run(inputs)
        except L.TbError as e:
            if e.kind == "NotAccelerated":
                _RESULTS.setdefault(fam, {}).setdefault("declined", 0)
                _RESULTS[fam]["declined"] += 1
                pytest.skip(f"declined: {e}")
            raise
    finally:
        it.close()
    for name, fn in zip(case.desc["ofm_name"], case.desc["ofm_file"]):
        exp = case.npy(fn)
        td = block.tensor(name)
        got = outs[name]
        assert list(exp.shape) == got.shape, name
        exp_bits = O.to_bits(td.dtype, O.from_npy(exp, td.dtype)).reshape(-1)
        if td.dtype == L.DT_BF16:
            got_vals = I.bf16_bits_to_f32(got.data)
        elif td.dtype in (L.DT_FP16, L.DT_FP32):
            got_vals = got.data.astype(np.float32)
        elif td.dtype in (L.DT_FP8E4M3, L.DT_FP8E5M2):
            got_vals = O.fp8_lut(td.dtype)[got.data.astype(np.uint8)]
        else:
            got_vals = got.data.astype(np.int64)
        got_bits = O.to_bits(td.dtype, got_vals.reshape(-1))
        bad = np.nonzero(exp_bits != got_bits)[0]
        if bad.size and td.dtype in (L.DT_BF16, L.DT_FP16, L.DT_FP32) and fam in TOLERANT:
            # tensor-core accumulation order: within 2 ULP of the output type plus
            # 2^-16 * sum |a*b| (the same bound as the direct GPU tests)
            ref = O.from_npy(exp, td.dtype).astype(np.float64).reshape(-1)
            floor = _abs_dot(case, block).reshape(-1)
            tol = 2 * _ulp(ref, td.dtype) + 2.0 ** -16 * floor
            err = np.abs(got_vals.astype(np.float64).reshape(-1) - ref)
            over = np.nonzero(~(err <= tol) & ~(np.isnan(ref) & np.isnan(got_vals.reshape(-1))))[0]
            assert over.size == 0, f"{name}: {over.size}/{ref.size} beyond tolerance, first at {over[:5]}"
            _RESULTS.setdefault(fam, {}).setdefault("within_tolerance", 0)
            _RESULTS[fam]["within_tolerance"] += 1
            return
        assert bad.size == 0, f"{name}: {bad.size}/{exp_bits.size} differ, first at {bad[:5]}"
    _RESULTS.setdefault(fam, {}).setdefault("exact", 0)
    _RESULTS[fam]["exact"] += 1


TOLERANT = {"conv2d", "conv3d", "depthwise_conv2d", "transpose_conv2d", "matmul", "matmul_t"}


def _ulp(x, dtype):
    bits = {L.DT_BF16: 7, L.DT_FP16: 10, L.DT_FP32: 23}[dtype]
    a = np.abs(x)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    if dtype == L.DT_FP16:
        e = np.maximum(e, -14)
    return 2.0 ** (e - bits)


def _abs_dot(case, block):
    """sum |a*b| per output of the case's contraction (bias zero), through the oracle."""
    st = O.State(block, {k: O.T(v.dtype, v.shape, np.abs(v.values)) for k, v in O.case_inputs(case, block).items()})
    main = [o for o in block.operators if o.name not in ("CONST", "CONST_SHAPE")][0]
    bias = main.inputs[2] if main.name in ("CONV2D", "DEPTHWISE_CONV2D") else None
    for op in block.operators:
        if op is main:
            continue
        r = O.EVAL[op.name](st, op)
        vals = np.abs(r.values) if r.values.dtype.kind == "f" else r.values
        if op.outputs[0] == bias:
            vals = np.zeros_like(vals)
        st.tensors[op.outputs[0]] = O.T(r.dtype, r.shape, vals)
    return np.asarray(O.EVAL[main.name](st, main).values, np.float64)


def _net(name):
    for c in O.load_cases(os.path.join(GOLDEN, "networks.zip")):
        if c.name == name:
            return c
    raise KeyError(name)


@pytest.mark.parametrize("net", ["mobilenet_like", "conv_matmul", "tflite_conv2d_qi8", "tf_conv2d_f32"])
@pytest.mark.parametrize("fuse", [True, False])
def test_hook_events_follow_reference_order(ctx, net, fuse):
    """OpTrace/StatsCollector/FlopCounter see one event per graph operator, in the
    reference's order and with its shapes, fused or not."""
    case = _net(net)
    g = O.read_graph(case.graph_bytes)
    block = g.main_block
    inputs = _inputs(case, block)
    expected = []
    O.run_block(block, O.case_inputs(case, block), trace=expected)
    trace, stats, flops = I.OpTrace(), I.StatsCollector(), I.FlopCounter()
    hooks = I.HookSet([trace, stats, flops])
    it = I.Interpreter(case.graph_bytes, context=ctx, fuse=fuse)
    try:
        it.run(inputs, hooks)
    finally:
        it.close()
    got = [(e.op_index, e.op, e.input_shapes, e.output_shapes) for e in trace.entries]
    assert got == expected
    assert stats.total_ops_executed == len(block.operators)
    assert sum(s.count for s in stats.op_stats.values()) == len(block.operators)
    want_flops = 0
    for (_, op, ins, outs) in expected:
        if op == "CONV2D":
            n, oh, ow, oc = outs[0]
            _, kh, kw, ic = ins[1]
            want_flops += 2 * n * oh * ow * oc * kh * kw * ic
        elif op == "MATMUL":
            n, h, c = ins[0]
            want_flops += 2 * n * h * ins[1][2] * c
        elif op == "ADD":
            want_flops += int(np.prod(outs[0]))
    assert flops.total_flops == want_flops


def test_fused_intermediates_are_not_materialised(ctx):
    """tflite_conv2d_qi8 is CONV2D -> RESCALE: fused, the int32 accumulator never
    reaches memory, so its hook view has no data; unfused it does, and both runs
    give the same output."""
    case = _net("tflite_conv2d_qi8")
    block = O.read_graph(case.graph_bytes).main_block
    inputs = _inputs(case, block)
    seen = {}

    class Grab(I.InterpreterHook):
        def post_op(self, op, ins, outs):
            for t in outs:
                seen[(op.name(), fuse)] = t.data

    results = {}
    for fuse in (True, False):
        it = I.Interpreter(case.graph_bytes, context=ctx, fuse=fuse)
        results[fuse] = it.run(inputs, Grab())
        launches = it.last_launches
        it.close()
        assert launches == (1 if fuse else 2)
    assert seen[("CONV2D", True)] is None
    assert seen[("CONV2D", False)] is not None and seen[("CONV2D", False)].dtype == np.int32
    for name in results[True]:
        assert np.array_equal(results[True][name].data, results[False][name].data)


def test_cuda_graph_replay_matches_eager(ctx):
    case = _net("mobilenet_like")
    block = O.read_graph(case.graph_bytes).main_block
    inputs = _inputs(case, block)
    eager = I.Interpreter(case.graph_bytes, context=ctx)
    want = eager.run(inputs)
    eager.close()
    s = torch.cuda.Stream()
    it = I.Interpreter(case.graph_bytes, context=ctx, cuda_graph=True)
    try:
        for _ in range(3):  # capture, then two replays
            it.bind(inputs)
            with torch.cuda.stream(s):
                it.execute(stream=s)
            s.synchronize()
            for name in want:
                got = it.output(name)
                assert np.array_equal(np.asarray(got.data).view(np.uint8), np.asarray(want[name].data).view(np.uint8))
    finally:
        it.close()


def test_missing_input_reports_stuck_ops(ctx):
    """An unbound graph input leaves its consumers unexecuted: GraphError after
    the rest ran (src/interpreter.rs:233-242)."""
    case = _net("tflite_add_f32")
    block = O.read_graph(case.graph_bytes).main_block
    inputs = _inputs(case, block)
    first = next(iter(inputs))
    it = I.Interpreter(case.graph_bytes, context=ctx)
    try:
        with pytest.raises(L.TbError) as e:
            it.run({first: inputs[first]})
        assert e.value.kind == "GraphError"
        assert "stuck on" in str(e.value)
    finally:
        it.close()


def test_unsupported_operator_is_declined_at_load(ctx):
    from tosa_b200 import tosa_graph as TG
    g = TG.Graph(regions=[("main", [TG.Block(
        name="main",
        operators=[TG.Operator(op=TG.OP["SIN"], inputs=["x"], outputs=["y"])],
        tensors=[TG.TensorDef("x", [4], TG.DTYPE["FP32"]), TG.TensorDef("y", [4], TG.DTYPE["FP32"])],
        inputs=["x"], outputs=["y"])])])
    with pytest.raises(L.TbError) as e:
        I.Interpreter(TG.write_graph(g), context=ctx)
    assert e.value.kind == "UnsupportedOp"


def test_malformed_buffer_is_a_deserialize_error(ctx):
    case = _net("mobilenet_like")
    with pytest.raises(L.TbError) as e:
        I.Interpreter(case.graph_bytes[:40], context=ctx)
    assert e.value.kind == "Deserialize"


def test_zz_accelerated_share():
    """Most positive fixtures run on the GPU (printed for the record)."""
    print({k: v for k, v in sorted(_RESULTS.items())})
    if not _RESULTS:
        pytest.skip("fixture tests did not run in this session")
    ran = sum(v.get("exact", 0) + v.get("within_tolerance", 0) for v in _RESULTS.values())
    declined = sum(v.get("declined", 0) for v in _RESULTS.values())
    assert ran >= 280 and declined == 0


def _synthetic(name):
    from tosa_b200 import graphs
    return {"residual": lambda: graphs.residual_block_int8(),
            "mobilenetv2": lambda: graphs.mobilenetv2_int8(1),
            "resnet50": lambda: graphs.resnet50_int8(1)}[name]()


def _oracle_run(data, inputs):
    block = O.read_graph(data).main_block
    ins = {k: O.T(t.dtype, list(t.shape), np.asarray(t.data).astype(np.int64).reshape(-1)) for k, t in inputs.items()}
    return O.run_block(block, ins)


@pytest.mark.parametrize("rounding", ["SINGLE_ROUND", "DOUBLE_ROUND"])
@pytest.mark.parametrize("clamp", [None, "relu", (-20, 90)])
def test_residual_chain_int8(ctx, rounding, clamp):
    """The fused residual chain (two int8 -> int32 RESCALEs, ADD, int32 -> int8
    RESCALE, optional CLAMP) against the oracle, both roundings of the output RESCALE."""
    from tosa_b200 import graphs
    g = graphs.GraphBuilder(5, 2)
    shape = [2, 12, 10, 48]
    x = g.input("x", shape)
    y = g.input("y", shape)
    q, _ = g.residual(x, -3, y, 6, relu=clamp == "relu", clamp=None if clamp in (None, "relu") else clamp,
                      rounding=rounding)
    g.outputs.append(q)
    data = g.build()
    block = O.read_graph(data).main_block
    rng = np.random.default_rng(3)
    inputs = {nm: I.Tensor.from_numpy(nm, rng.integers(-128, 128, shape).astype(np.int8), block.tensor(nm).dtype)
              for nm in block.inputs}
    want = _oracle_run(data, inputs)
    it = I.Interpreter(data, context=ctx)
    try:
        got = it.run(inputs)
        assert it.last_launches == 1  # the whole chain in one kernel
    finally:
        it.close()
    for nm in block.outputs:
        assert np.array_equal(np.asarray(got[nm].data).astype(np.int64).reshape(-1), want[nm].values)


@pytest.mark.parametrize("name", ["residual", "mobilenetv2", "resnet50"])
@pytest.mark.parametrize("mode", ["fused", "unfused", "cuda_graph"])
def test_synthetic_int8_graph_bit_exact(ctx, name, mode):
    """The benchmark graphs (and a small graph with every fusion pattern) at batch
    1-2 against the oracle, bit for bit, in every execution mode."""
    data, info = _synthetic(name)
    block = O.read_graph(data).main_block
    rng = np.random.default_rng(11)
    inputs = {}
    for nm in block.inputs:
        td = block.tensor(nm)
        inputs[nm] = I.Tensor.from_numpy(nm, rng.integers(-128, 128, td.shape).astype(np.int8), td.dtype)
    want = _oracle_run(data, inputs)
    kw = {"fuse": mode != "unfused", "cuda_graph": mode == "cuda_graph"}
    it = I.Interpreter(data, context=ctx, **kw)
    try:
        if mode == "cuda_graph":
            s = torch.cuda.Stream()
            for _ in range(2):
                it.bind(inputs)
                it.execute(stream=s)
                s.synchronize()
            got = {nm: it.output(nm) for nm in block.outputs}
        else:
            got = it.run(inputs)
    finally:
        it.close()
    for nm in block.outputs:
        g = np.asarray(got[nm].data).astype(np.int64).reshape(-1)
        assert got[nm].shape == want[nm].shape
        bad = np.nonzero(g != want[nm].values)[0]
        assert bad.size == 0, f"{nm}: {bad.size}/{g.size} differ, first at {bad[:5]}"


def test_sharded_interpreter_matches_whole_batch():
    """ShardedInterpreter: the batch split over two replicas (two GPUs when the
    box has them, else two contexts on one), one host thread each; the gathered
    outputs equal the oracle's whole-batch run bit for bit."""
    from tosa_b200 import graphs
    from tosa_b200 import parallel as P
    devices = [0, 1] if torch.cuda.device_count() >= 2 else [0, 0]
    per, world = 2, 2
    data1, _ = graphs.residual_block_int8(batch=per)
    dataw, _ = graphs.residual_block_int8(batch=per * world)
    rng = np.random.default_rng(9)
    x = rng.integers(-128, 128, (per * world, 14, 14, 64)).astype(np.int8)
    inputs = {"x": I.Tensor.from_numpy("x", x, L.DT_INT8)}
    want = _oracle_run(dataw, inputs)
    si = P.ShardedInterpreter(data1, devices)
    try:
        for _ in range(2):
            got = si.run(inputs)
            for nm, w in want.items():
                assert got[nm].shape == w.shape, nm
                assert np.array_equal(np.asarray(got[nm].data).astype(np.int64).reshape(-1), w.values), nm
    finally:
        si.close()


def test_external_constant_data(ctx):
    """A graph whose constants lie after the flatbuffer (TosaTensor.offset / .size,
    schema/tosa.fbs:711-716) runs bit-exact like the same graph with inline data; an
    offset past the end of the file is rejected when the graph is loaded."""
    from tosa_b200 import graphs
    from tosa_b200 import tosa_graph as TG
    data, _ = graphs.residual_block_int8(batch=2)
    g = TG.read_graph(data)
    for t in g.main_block.tensors:
        if t.data is not None and len(t.data) > 64 and t.dtype != TG.DTYPE["SHAPE"]:
            t.external = True
    ext = TG.write_graph(g)
    x = np.random.default_rng(12).integers(-128, 128, (2, 14, 14, 64)).astype(np.int8)
    inputs = {"x": I.Tensor.from_numpy("x", x, L.DT_INT8)}
    want = _oracle_run(data, inputs)
    it = I.Interpreter(ext, context=ctx)
    try:
        got = it.run(inputs)
    finally:
        it.close()
    for nm, w in want.items():
        assert np.array_equal(np.asarray(got[nm].data).astype(np.int64).reshape(-1), w.values), nm
    with pytest.raises(L.TbError) as ei:
        I.Interpreter(ext[:-16], context=ctx)
    assert ei.value.kind == "Deserialize"
