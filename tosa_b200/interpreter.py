"""Python face of the graph runner, mirroring the reference interpreter's API.

Names and behaviour follow tosa-interp:

* ``run_graph``, ``run_graph_with_stats``, ``run_graph_with_hooks``
  (src/lib.rs:20-43);
* ``Interpreter.from_flatbuffer`` / ``Interpreter.run`` (src/interpreter.rs:108-147);
* ``InterpreterHook``, ``HookSet``, ``NoopHook``, ``StatsCollector``,
  ``FlopCounter``, ``OpTrace``, ``OpInfo`` (src/stats.rs);
* errors raise ``TbError`` whose ``kind`` is the reference's Error variant
  (src/error.rs:4-31).

Every operator runs on the GPU through libtosa_b200 (tb_graph_*); there is no
CPU path. Hooks receive ``HookTensor`` views (name, shape, dtype, size) whose
``data`` property copies the device tensor to the host on demand (``None``
for tensors a fused kernel never wrote).
"""

from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L
from .tosa_graph import DTYPE_NAMES, OP_NAMES

TbError = L.TbError

# numpy storage of each dtype in host buffers (the C ABI's one-element-per-slot layout)
_NP = {
    L.DT_BOOL: np.uint8, L.DT_INT4: np.int8, L.DT_INT8: np.int8, L.DT_INT16: np.int16, L.DT_INT32: np.int32,
    L.DT_INT48: np.int64, L.DT_FP32: np.float32, L.DT_FP16: np.float16, L.DT_BF16: np.uint16,
    L.DT_SHAPE: np.int64, L.DT_INT64: np.int64, L.DT_FP8E4M3: np.uint8, L.DT_FP8E5M2: np.uint8,
}
_ELEM = {L.DT_BOOL: 1, L.DT_INT4: 1, L.DT_INT8: 1, L.DT_INT16: 2, L.DT_INT32: 4, L.DT_INT48: 8, L.DT_FP32: 4,
         L.DT_FP16: 2, L.DT_BF16: 2, L.DT_SHAPE: 8, L.DT_INT64: 8, L.DT_FP8E4M3: 1, L.DT_FP8E5M2: 1}


def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (NaN stays NaN)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    return np.where(nan, np.uint16(0x7FC0), r)


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class Tensor:
    """A host tensor (src/tensor.rs:228-249). ``data`` is a numpy array in the
    dtype's storage form (BF16 as uint16 bit patterns, INT4 one int8 per
    element, INT48 as int64)."""

    name: str
    shape: list
    dtype: int
    data: np.ndarray

    @staticmethod
    def from_numpy(name: str, arr, dtype: int) -> "Tensor":
        a = np.asarray(arr)
        if dtype == L.DT_BF16 and a.dtype != np.uint16:
            a = f32_to_bf16_bits(a)
        else:
            a = a.astype(_NP[dtype], copy=False)
        return Tensor(name, list(a.shape), dtype, np.ascontiguousarray(a))

    def element_count(self) -> int:
        return max(int(np.prod(self.shape)) if self.shape else 1, 1)

    def size_bytes(self) -> int:
        return self.element_count() * _ELEM.get(self.dtype, 0)

    def as_float(self) -> np.ndarray:
        if self.dtype == L.DT_BF16:
            return bf16_bits_to_f32(self.data)
        return self.data.astype(np.float32)


@dataclass
class OpInfo:
    """src/stats.rs:6-9"""
    op: int
    op_index: int

    def name(self) -> str:
        return OP_NAMES[self.op] if 0 <= self.op < len(OP_NAMES) else "UNKNOWN"


class HookTensor:
    """What a hook sees of a tensor: metadata, plus device data on demand."""

    __slots__ = ("name", "shape", "dtype", "_bytes", "_ptr", "_ctx")

    def __init__(self, info: L.TensorInfo, ctx=None):
        self.name = info.name.decode()
        self.shape = [int(info.shape[i]) for i in range(info.rank)]
        self.dtype = int(info.dtype)
        self._bytes = int(info.bytes)
        self._ptr = info.data
        self._ctx = ctx

    def element_count(self) -> int:
        return max(int(np.prod(self.shape)) if self.shape else 1, 1)

    def size_bytes(self) -> int:
        return self._bytes

    @property
    def data(self):
        if not self._ptr:
            return None
        n = int(np.prod(self.shape)) if self.shape else 1
        out = np.empty(n, dtype=_NP[self.dtype])
        if n:
            import torch
            torch.cuda.synchronize()
            L.check(L.load().tb_memcpy_d2h(self._ctx, out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(self._ptr),
                                           out.nbytes, None))
            torch.cuda.synchronize()
        return out.reshape(self.shape)


class InterpreterHook:
    """src/stats.rs:11-16 -- override any of the four callbacks."""

    def pre_op(self, op: OpInfo, inputs: list) -> None:
        pass

    def post_op(self, op: OpInfo, inputs: list, outputs: list) -> None:
        pass

    def on_tensor_alloc(self, name: str, shape: list, dtype: int, size_bytes: int) -> None:
        pass

    def on_tensor_free(self, name: str, size_bytes: int) -> None:
        pass


class NoopHook(InterpreterHook):
    pass


class HookSet(InterpreterHook):
    """Dispatches every event to its hooks in order (src/stats.rs:19-75)."""

    def __init__(self, hooks=None):
        self._hooks = list(hooks or [])

    def add(self, hook: InterpreterHook) -> None:
        self._hooks.append(hook)

    def hooks(self) -> list:
        return self._hooks

    def into_hooks(self) -> list:
        return self._hooks

    def pre_op(self, op, inputs):
        for h in self._hooks:
            h.pre_op(op, inputs)

    def post_op(self, op, inputs, outputs):
        for h in self._hooks:
            h.post_op(op, inputs, outputs)

    def on_tensor_alloc(self, name, shape, dtype, size_bytes):
        for h in self._hooks:
            h.on_tensor_alloc(name, shape, dtype, size_bytes)

    def on_tensor_free(self, name, size_bytes):
        for h in self._hooks:
            h.on_tensor_free(name, size_bytes)


@dataclass
class OpStats:
    count: int = 0
    total_time: float = 0.0  # seconds
    total_input_elements: int = 0
    total_output_elements: int = 0


class StatsCollector(InterpreterHook):
    """Op counts, time and element throughput, peak memory (src/stats.rs:98-189).
    Times are host wall-clock between pre_op and post_op; run the graph with
    ``sync_each_op=True`` for them to include device execution."""

    def __init__(self):
        self.op_stats: dict = {}
        self.peak_memory_bytes = 0
        self.current_memory_bytes = 0
        self.total_ops_executed = 0
        self._start = None

    def pre_op(self, op, inputs):
        self._start = time.perf_counter()

    def post_op(self, op, inputs, outputs):
        elapsed = time.perf_counter() - self._start if self._start is not None else 0.0
        e = self.op_stats.setdefault(op.name(), OpStats())
        e.count += 1
        e.total_time += elapsed
        e.total_input_elements += sum(t.element_count() for t in inputs)
        e.total_output_elements += sum(t.element_count() for t in outputs)
        self.total_ops_executed += 1

    def on_tensor_alloc(self, name, shape, dtype, size_bytes):
        self.current_memory_bytes += size_bytes
        self.peak_memory_bytes = max(self.peak_memory_bytes, self.current_memory_bytes)

    def on_tensor_free(self, name, size_bytes):
        self.current_memory_bytes = max(self.current_memory_bytes - size_bytes, 0)

    def summary(self) -> str:
        lines = [f"Total ops executed: {self.total_ops_executed}", f"Peak memory: {self.peak_memory_bytes} bytes", ""]
        for name in sorted(self.op_stats):
            s = self.op_stats[name]
            lines.append(f"  {name:<16} count={s.count:<6} time={s.total_time * 1000:>8.3f}ms  "
                         f"elements_in={s.total_input_elements:<10} elements_out={s.total_output_elements:<10}")
        return "\n".join(lines)


_ELEMENTWISE = {"ADD", "SUB", "MUL", "ABS", "NEGATE", "MAXIMUM", "MINIMUM"}
_TRANSCENDENTAL = {"EXP", "LOG", "SIN", "COS", "TANH", "SIGMOID", "ERF", "RSQRT", "RECIPROCAL", "POW"}


def estimate_flops(op: OpInfo, inputs: list, outputs: list) -> int:
    """src/stats.rs:218-260"""
    name = op.name()
    if name in _ELEMENTWISE:
        return outputs[0].element_count() if outputs else 0
    if name in _TRANSCENDENTAL:
        return outputs[0].element_count() * 10 if outputs else 0
    if name == "MATMUL":
        if len(inputs) >= 2 and len(inputs[0].shape) == 3:
            n, h, c = inputs[0].shape
            return 2 * n * h * inputs[1].shape[2] * c
        return 0
    if name == "CONV2D" and len(inputs) >= 2 and outputs:
        o = outputs[0]
        if len(o.shape) == 4 and len(inputs[1].shape) == 4:
            n, oh, ow, oc = o.shape
            _, kh, kw, ic = inputs[1].shape
            return 2 * n * oh * ow * oc * kh * kw * ic
    return 0


class FlopCounter(InterpreterHook):
    """src/stats.rs:193-216"""

    def __init__(self):
        self.total_flops = 0
        self.flops_by_op: dict = {}

    def post_op(self, op, inputs, outputs):
        f = estimate_flops(op, inputs, outputs)
        self.total_flops += f
        self.flops_by_op[op.name()] = self.flops_by_op.get(op.name(), 0) + f


@dataclass
class TraceEntry:
    op: str
    op_index: int
    input_shapes: list = field(default_factory=list)
    output_shapes: list = field(default_factory=list)
    elapsed: float = 0.0


class OpTrace(InterpreterHook):
    """src/stats.rs:262-299"""

    def __init__(self):
        self.entries: list = []

    def post_op(self, op, inputs, outputs):
        self.entries.append(TraceEntry(op.name(), op.op_index, [list(t.shape) for t in inputs],
                                       [list(t.shape) for t in outputs]))


class Interpreter:
    """A parsed graph bound to one GPU (src/interpreter.rs:108-147)."""

    def __init__(self, data: bytes, device: int = 0, *, fuse: bool = True, sync_each_op: bool = False,
                 cuda_graph: bool = False, time_ops: bool = False, context: L.Context | None = None):
        self._ctx = context or L.Context(device)
        self._own_ctx = context is None
        self._data = bytes(data)
        flags = 0
        if not fuse:
            flags |= L.GRAPH_NO_FUSION
        if sync_each_op:
            flags |= L.GRAPH_SYNC_EACH_OP
        if cuda_graph:
            flags |= L.GRAPH_CUDA_GRAPH
        if time_ops:
            flags |= L.GRAPH_TIME_OPS
        h = ctypes.c_void_p()
        L.check(L.load().tb_graph_load(self._ctx.h, self._data, len(self._data), flags, ctypes.byref(h)))
        self._h = h
        self._stream = None

    @classmethod
    def from_flatbuffer(cls, data: bytes, **kw) -> "Interpreter":
        return cls(data, **kw)

    def close(self):
        if getattr(self, "_h", None):
            L.load().tb_graph_destroy(self._h)
            self._h = None
        if getattr(self, "_own_ctx", False) and self._ctx is not None:
            self._ctx.close()
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _decl(self, fn, n):
        out = []
        for i in range(n):
            info = L.TensorInfo()
            L.check(fn(self._h, i, ctypes.byref(info)))
            out.append((info.name.decode(), int(info.dtype), [int(info.shape[k]) for k in range(info.rank)]))
        return out

    def inputs(self) -> list:
        """Declared (name, dtype, shape) of the main block's inputs."""
        return self._decl(L.load().tb_graph_input_info, L.load().tb_graph_num_inputs(self._h))

    def outputs(self) -> list:
        return self._decl(L.load().tb_graph_output_info, L.load().tb_graph_num_outputs(self._h))

    def op_time_ms(self, op_index: int) -> float:
        """Device time of an operator's kernels in the last run (time_ops=True); -1 if none."""
        return float(L.load().tb_graph_op_time_ms(self._h, op_index))

    @property
    def last_launches(self) -> int:
        return int(L.load().tb_graph_last_launches(self._h))

    def bind(self, inputs: dict, stream=None) -> None:
        """Copy host tensors to the device (the reference's `inputs` map)."""
        lib = L.load()
        sp = L.stream_ptr(stream) if stream is not None else None
        for name, t in inputs.items():
            arr = np.ascontiguousarray(t.data)
            shape = (ctypes.c_int64 * max(len(t.shape), 1))(*[int(v) for v in t.shape])
            L.check(lib.tb_graph_set_input(self._h, name.encode(), t.dtype, shape, len(t.shape),
                                           arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes, 0, sp))

    def bind_device(self, name: str, dtype: int, shape, ptr: int) -> None:
        """Bind a device buffer in place (no copy)."""
        sh = (ctypes.c_int64 * max(len(shape), 1))(*[int(v) for v in shape])
        n = int(np.prod(shape)) if len(shape) else 1
        L.check(L.load().tb_graph_set_input(self._h, name.encode(), dtype, sh, len(shape), ctypes.c_void_p(ptr),
                                            n * _ELEM[dtype], 1, None))

    def execute(self, hook: InterpreterHook | None = None, stream=None) -> None:
        """Run with the bound inputs; hooks as in Interpreter::run."""
        keep = []
        hooks_p = None
        if hook is not None and not isinstance(hook, NoopHook):
            ctx = self._ctx.h

            def pre(_u, op, ins, n):
                hook.pre_op(OpInfo(op[0].op, op[0].op_index), [HookTensor(ins[i], ctx) for i in range(n)])

            def post(_u, op, ins, ni, outs, no):
                hook.post_op(OpInfo(op[0].op, op[0].op_index), [HookTensor(ins[i], ctx) for i in range(ni)],
                             [HookTensor(outs[i], ctx) for i in range(no)])

            def alloc(_u, name, shape, rank, dtype, nbytes):
                hook.on_tensor_alloc(name.decode(), [int(shape[i]) for i in range(rank)], int(dtype), int(nbytes))

            def free(_u, name, nbytes):
                hook.on_tensor_free(name.decode(), int(nbytes))

            hs = L.Hooks(None, L.PRE_OP(pre), L.POST_OP(post), L.ON_ALLOC(alloc), L.ON_FREE(free))
            keep.append(hs)
            hooks_p = ctypes.byref(hs)
        sp = L.stream_ptr(stream) if stream is not None else None
        L.check(L.load().tb_graph_run(self._h, hooks_p, sp))

    def output(self, name: str) -> Tensor:
        lib = L.load()
        info = L.TensorInfo()
        L.check(lib.tb_graph_get_output(self._h, name.encode(), ctypes.byref(info)))
        shape = [int(info.shape[i]) for i in range(info.rank)]
        dtype = int(info.dtype)
        n = int(np.prod(shape)) if shape else 1
        arr = np.empty(n, dtype=_NP[dtype])
        L.check(lib.tb_graph_read_output(self._h, name.encode(), arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes,
                                         None))
        return Tensor(name, shape, dtype, arr.reshape(shape))

    def run(self, inputs: dict, hook: InterpreterHook | None = None) -> dict:
        """Interpreter::run: bind `inputs`, execute, return the main block's outputs."""
        self.bind(inputs)
        self.execute(hook)
        out = {}
        for name, _, _ in self.outputs():
            try:
                out[name] = self.output(name)
            except TbError as e:
                if e.kind != "TensorNotFound":
                    raise
        return out


def run_graph(data: bytes, inputs: dict, **kw) -> dict:
    """src/lib.rs:20-24"""
    it = Interpreter.from_flatbuffer(data, **kw)
    try:
        return it.run(inputs, NoopHook())
    finally:
        it.close()


def run_graph_with_stats(data: bytes, inputs: dict, **kw):
    """src/lib.rs:26-34"""
    it = Interpreter.from_flatbuffer(data, **kw)
    try:
        hook = StatsCollector()
        return it.run(inputs, hook), hook
    finally:
        it.close()


def run_graph_with_hooks(data: bytes, inputs: dict, hooks: InterpreterHook, **kw) -> dict:
    """src/lib.rs:36-43"""
    it = Interpreter.from_flatbuffer(data, **kw)
    try:
        return it.run(inputs, hooks)
    finally:
        it.close()


def dtype_name(dt: int) -> str:
    return DTYPE_NAMES[dt] if 0 <= dt < len(DTYPE_NAMES) else str(dt)
