"""Failure detection on the GPU, in forms that fault, trap or hang nothing.

* A bounded wait that runs out: the context's wait bound is set to zero, so the
  first wait of an ordinary int8 MATMUL that is not satisfied at once (for
  example the MMA warp's wait for the first stage's copies) gives up. The kernel unwinds by design -- its TMA loads and MMAs
  drain under their own bound, tensor memory is released -- and the next
  synchronize reports Timeout (TB_ERR_TIMEOUT). With the bound restored, the
  same context runs the same product and a convolution exactly (a leaked
  tensor-memory allocation would stall every later GEMM on that SM).
* An allocation that fails: TB_FAULT_ALLOC_FAIL makes one device buffer
  allocation of a graph fail as if the device were out of memory; the run
  returns an error of the CUDA kind, and the next run of the same graph
  allocates the rest and is exact.
* A shard that fails: TB_FAULT_SHARD makes one shard of a ShardedInterpreter
  raise before its run; the run reports ShardError for that shard after the
  other shard finished, and the next run without the injection is exact.
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers as H

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tosa_b200 import _lib as L  # noqa: E402
from tosa_b200 import graphs  # noqa: E402
from tosa_b200 import interpreter as I  # noqa: E402
from tosa_b200 import parallel as P  # noqa: E402


def _matmul(ctx, a, b, za, zb):
    n, h, c = a.shape
    w = b.shape[2]
    d = L.MatmulDesc(n=n, h=h, c=c, w=w, a_dtype=L.DT_INT8, b_dtype=L.DT_INT8, out_dtype=L.DT_INT32, a_zp=za, b_zp=zb)
    ta = torch.from_numpy(a.astype(np.int8)).cuda()
    tb = torch.from_numpy(b.astype(np.int8)).cuda()
    out = torch.zeros((n, h, w), dtype=torch.int32, device="cuda")
    L.check(L.load().tb_matmul(ctx.h, d, None, L.ptr(ta), L.ptr(tb), L.ptr(out), L.stream_ptr()))
    return out


def test_wait_timeout_reports_and_context_stays_usable():
    lib = L.load()
    ctx = L.Context(0)
    try:
        rng = np.random.default_rng(65)
        a = rng.integers(-128, 128, (8, 1024, 1024), dtype=np.int64)
        b = rng.integers(-128, 128, (8, 1024, 1024), dtype=np.int64)
        L.check(lib.tb_context_set_wait_timeout_ms(ctx.h, ctypes.c_double(0.0)))
        _matmul(ctx, a, b, 3, -2)
        with pytest.raises(L.TbError) as ei:
            ctx.synchronize()
        assert ei.value.kind == "Timeout"
        # the bound back to two seconds: the same context, the same product, exact
        L.check(lib.tb_context_set_wait_timeout_ms(ctx.h, ctypes.c_double(2000.0)))
        out = _matmul(ctx, a, b, 3, -2)
        ctx.synchronize()
        got = out.cpu().numpy().astype(np.int64)
        for bi, r0 in ((0, 0), (7, 1008)):
            want = H.oracle_matmul_int(a[bi:bi + 1, r0:r0 + 16], b[bi:bi + 1], 3, -2)
            assert np.array_equal(got[bi:bi + 1, r0:r0 + 16], want), (bi, r0)
        # a convolution on every SM of the same context
        x = rng.integers(-128, 128, (4, 28, 28, 64), dtype=np.int64)
        w = rng.integers(-127, 128, (128, 3, 3, 64), dtype=np.int64)
        bias = rng.integers(-1000, 1000, 128, dtype=np.int64)
        from tests.test_gpu_contractions import run_conv
        got = run_conv(ctx, x, w, bias, -3, 0, (1, 1, 1, 1), (1, 1), (1, 1))
        assert np.array_equal(got.astype(np.int64), H.oracle_conv_int(x, w, bias, -3, 0, (1, 1, 1, 1), (1, 1), (1, 1)))
    finally:
        ctx.close()


def test_wait_timeout_rejects_bad_bounds():
    ctx = L.Context(0)
    try:
        assert L.load().tb_context_set_wait_timeout_ms(ctx.h, ctypes.c_double(-1.0)) == 66
        assert L.load().tb_context_set_wait_timeout_ms(ctx.h, ctypes.c_double(float("nan"))) == 66
    finally:
        ctx.close()


def _residual_inputs(batch):
    data, _ = graphs.residual_block_int8(batch=batch)
    x = np.random.default_rng(9).integers(-128, 128, (batch, 14, 14, 64)).astype(np.int8)
    return data, {"x": I.Tensor.from_numpy("x", x, L.DT_INT8)}


def _oracle(data, inputs):
    block = O.read_graph(data).main_block
    ins = {k: O.T(t.dtype, list(t.shape), np.asarray(t.data).astype(np.int64).reshape(-1)) for k, t in inputs.items()}
    return O.run_block(block, ins)


def test_injected_allocation_failure(monkeypatch):
    data, inputs = _residual_inputs(2)
    want = _oracle(data, inputs)
    ctx = L.Context(0)
    monkeypatch.setenv("TB_FAULT_ALLOC_FAIL", "2")
    it = I.Interpreter(data, context=ctx)
    try:
        with pytest.raises(L.TbError) as ei:
            it.run(inputs)
        assert ei.value.kind == "Cuda" and "TB_FAULT_ALLOC_FAIL" in str(ei.value)
        got = it.run(inputs)  # the next run allocates the rest
        for nm, w in want.items():
            assert np.array_equal(np.asarray(got[nm].data).astype(np.int64).reshape(-1), w.values), nm
    finally:
        it.close()
        ctx.close()


def test_sharded_interpreter_reports_a_failed_shard(monkeypatch):
    devices = [0, 1] if torch.cuda.device_count() >= 2 else [0, 0]
    data1, _ = graphs.residual_block_int8(batch=2)
    dataw, inputs = _residual_inputs(4)
    want = _oracle(dataw, inputs)
    si = P.ShardedInterpreter(data1, devices)
    try:
        monkeypatch.setenv("TB_FAULT_SHARD", "1")
        with pytest.raises(P.ShardError) as ei:
            si.run(inputs)
        assert ei.value.shard == 1 and isinstance(ei.value.__cause__, P.InjectedFault)
        monkeypatch.delenv("TB_FAULT_SHARD")
        got = si.run(inputs)
        for nm, w in want.items():
            assert np.array_equal(np.asarray(got[nm].data).astype(np.int64).reshape(-1), w.values), nm
    finally:
        si.close()
