"""CPU oracle for the tosa_b200 dense-contraction path -- TEST INFRASTRUCTURE.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU legs.
It restates the reference interpreter (tosa-interp) on the CPU:

* arithmetic: oracle/tosa_oracle.c (loaded here with ctypes), a C restatement
  of the reference's loops and accumulators;
* validation: the ERROR_IF rules of each operator, restated below in Python
  with the reference file:line they follow;
* graph flow: a small dataflow runner over the main block in the reference's
  ready-queue order (src/interpreter.rs:154-245) for the operators that the
  conformance and network fixtures use.

Parity is pinned: tests/test_oracle_golden.py requires this oracle to match
every checked-in conformance vector of CONV2D, CONV3D, DEPTHWISE_CONV2D, TRANSPOSE_CONV2D,
MATMUL, MATMUL_T,
RESCALE, AVG_POOL2D, MAX_POOL2D and CLAMP bit for bit, to reject every
ERROR_IF case, and to reproduce the network fixtures.

Tensors are (dtype, shape, values): integer values widened to int64, float
values widened to float32 (the reference's int_values / float_values,
src/ops/common.rs:63-84).
"""

from __future__ import annotations

import ctypes
import io
import json
import os
import subprocess
import zipfile
from collections import deque
from dataclasses import dataclass

import numpy as np

from tosa_b200.tosa_graph import DTYPE, DTYPE_NAMES, OP_NAMES, read_graph

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

D = DTYPE
INT_TYPES = {D["INT4"], D["INT8"], D["INT16"], D["INT32"], D["INT48"], D["INT64"]}
FP8_TYPES = {D["FP8E4M3"], D["FP8E5M2"]}
FLOAT_TYPES = {D["FP16"], D["BF16"], D["FP32"]} | FP8_TYPES
ELEM_BYTES = {D["BOOL"]: 1, D["INT4"]: 1, D["INT8"]: 1, D["INT16"]: 2, D["INT32"]: 4,
              D["INT48"]: 8, D["INT64"]: 8, D["FP32"]: 4, D["FP16"]: 2, D["BF16"]: 2,
              D["SHAPE"]: 8, D["FP8E4M3"]: 1, D["FP8E5M2"]: 1}


class OracleError(Exception):
    """An Err(...) of the reference; `kind` names the Error variant
    (src/error.rs:4-31)."""

    def __init__(self, kind: str, msg: str):
        super().__init__(f"{kind}: {msg}")
        self.kind = kind


def graph_error(op, msg):
    return OracleError("GraphError", f"{op}: {msg}")


# ---------------------------------------------------------------------------
# C library
# ---------------------------------------------------------------------------

_lib = None


def build(force: bool = False) -> str:
    """Compile tosa_oracle.c into oracle/_build/liboracle.so."""
    if force or not os.path.exists(LIB_PATH) or (
            os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "tosa_oracle.c"))):
        subprocess.check_call(["make", "-s", "-C", HERE])
    return LIB_PATH


class ConvGeom(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int64), ("ih", ctypes.c_int64), ("iw", ctypes.c_int64),
                ("ic", ctypes.c_int64), ("oc", ctypes.c_int64), ("kh", ctypes.c_int64),
                ("kw", ctypes.c_int64), ("oh", ctypes.c_int64), ("ow", ctypes.c_int64),
                ("pad", ctypes.c_int64 * 4), ("stride", ctypes.c_int64 * 2),
                ("dilation", ctypes.c_int64 * 2), ("m", ctypes.c_int64)]


class PoolGeom(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int64), ("ih", ctypes.c_int64), ("iw", ctypes.c_int64),
                ("c", ctypes.c_int64), ("oh", ctypes.c_int64), ("ow", ctypes.c_int64),
                ("kernel", ctypes.c_int64 * 2), ("stride", ctypes.c_int64 * 2),
                ("pad_top", ctypes.c_int64), ("pad_left", ctypes.c_int64)]


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.orc_round_to.restype = ctypes.c_float
        _lib.orc_round_to.argtypes = [ctypes.c_int, ctypes.c_float]
        _lib.orc_fp8_decode.restype = ctypes.c_float
        _lib.orc_fp8_decode.argtypes = [ctypes.c_int, ctypes.c_uint8]
        _lib.orc_fp8_encode.restype = ctypes.c_uint8
        _lib.orc_fp8_encode.argtypes = [ctypes.c_int, ctypes.c_float]
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# Data conversion (src/tensor.rs:86-167, src/npy.rs, src/ops/common.rs)
# ---------------------------------------------------------------------------

_FP8_LUT = {}


def fp8_lut(dtype):
    if dtype not in _FP8_LUT:
        L = lib()
        _FP8_LUT[dtype] = np.array([L.orc_fp8_decode(dtype, b) for b in range(256)], dtype=np.float32)
    return _FP8_LUT[dtype]


def bf16_bits_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def round_to(dtype, values):
    """common.rs:100-108, elementwise through the C oracle."""
    v = _f32(values).copy()
    if dtype == D["FP32"]:
        return v
    L = lib()
    flat = v.reshape(-1)
    if dtype == D["BF16"]:
        u = flat.view(np.uint32).astype(np.uint64)
        nan = (u & 0x7FFFFFFF) > 0x7F800000
        r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
        r = np.where(nan, ((u | 0x00400000) & 0xFFFF0000).astype(np.uint32), r)
        return r.view(np.float32).reshape(v.shape)
    if dtype == D["FP16"]:
        return flat.astype(np.float16).astype(np.float32).reshape(v.shape)
    for i in range(flat.size):
        flat[i] = L.orc_round_to(dtype, float(flat[i]))
    return v


def decode_raw(dtype, data: bytes | None, count: int):
    """TensorData::from_raw_bytes (tensor.rs:86-167) widened to int64/f32."""
    if data is None:
        return np.zeros(count, dtype=np.float32 if dtype in FLOAT_TYPES else np.int64)
    if dtype == D["INT4"]:
        needed = (count + 1) // 2
    elif dtype == D["INT48"]:
        needed = count * 6
    else:
        needed = count * ELEM_BYTES[dtype]
    if len(data) < needed:
        raise OracleError("Deserialize", f"{DTYPE_NAMES[dtype]} tensor of {count} elements needs "
                                         f"{needed} bytes, got {len(data)}")
    b = np.frombuffer(data[:needed], dtype=np.uint8)
    if dtype == D["BOOL"]:
        return (b != 0).astype(np.int64)
    if dtype == D["INT4"]:
        nib = np.stack([b & 0xF, b >> 4], axis=1).reshape(-1)[:count].astype(np.int64)
        return np.where(nib >= 8, nib - 16, nib)
    if dtype == D["INT8"]:
        return b.view(np.int8).astype(np.int64)
    if dtype == D["INT16"]:
        return b.view("<i2").astype(np.int64)
    if dtype == D["INT32"]:
        return b.view("<i4").astype(np.int64)
    if dtype in (D["INT64"], D["SHAPE"]):
        return b.view("<i8").astype(np.int64)
    if dtype == D["INT48"]:
        q = b.reshape(-1, 6).astype(np.int64)
        v = sum(q[:, i] << (8 * i) for i in range(6))
        return np.where(v >= (1 << 47), v - (1 << 48), v)
    if dtype == D["FP32"]:
        return b.view("<f4").astype(np.float32)
    if dtype == D["FP16"]:
        return b.view("<f2").astype(np.float32)
    if dtype == D["BF16"]:
        return bf16_bits_to_f32(b.view("<u2"))
    if dtype in FP8_TYPES:
        return fp8_lut(dtype)[b]
    raise OracleError("DTypeMismatch", f"cannot deserialize raw bytes for {DTYPE_NAMES[dtype]}")


def from_npy(arr: np.ndarray, dtype: int):
    """npy array (as the reference's npy.rs stores each dtype) -> widened values."""
    flat = arr.reshape(-1)
    if dtype == D["BF16"]:
        return bf16_bits_to_f32(flat.view(np.uint16))
    if dtype in FP8_TYPES:
        return fp8_lut(dtype)[flat.view(np.uint8)]
    if dtype in (D["FP16"], D["FP32"]):
        return flat.astype(np.float32)
    if dtype == D["BOOL"]:
        return flat.astype(np.int64)
    return flat.astype(np.int64)


def to_bits(dtype, values):
    """Canonical comparison form: ints as int64, floats as the bit pattern of
    the dtype with every NaN mapped to one value (the harness treats any two
    NaNs as equal, tests/conformance.rs:165-229)."""
    v = np.asarray(values)
    if dtype in INT_TYPES or dtype == D["BOOL"]:
        return v.astype(np.int64)
    f = _f32(v)
    nan = np.isnan(f)
    if dtype == D["FP32"]:
        bits = f.view(np.uint32).astype(np.int64)
    elif dtype == D["FP16"]:
        bits = f.astype(np.float16).view(np.uint16).astype(np.int64)
    elif dtype == D["BF16"]:
        bits = (f.view(np.uint32) >> 16).astype(np.int64)
    else:
        bits = np.array([lib().orc_fp8_encode(dtype, float(x)) for x in f.reshape(-1)],
                        dtype=np.int64).reshape(f.shape)
    return np.where(nan, -1, bits)


@dataclass
class T:
    dtype: int
    shape: list
    values: np.ndarray  # flat int64 or float32

    @property
    def is_int(self):
        return self.dtype in INT_TYPES

    def count(self):
        return int(np.prod(self.shape)) if self.shape else 1


# ---------------------------------------------------------------------------
# Validation helpers (src/ops/common.rs)
# ---------------------------------------------------------------------------


class State:
    def __init__(self, block, tensors):
        self.block = block
        self.tensors = dict(tensors)
        self.defs = {t.name: t for t in block.tensors}

    def get(self, name) -> T:
        if name not in self.tensors:
            raise OracleError("TensorNotFound", name)
        return self.tensors[name]

    def declared(self, op, name, shape):
        """check_declared_output (common.rs:46-60)."""
        d = self.defs.get(name)
        if d is None:
            return None
        if all(s >= 0 for s in d.shape) and list(d.shape) != list(shape):
            raise OracleError("ShapeMismatch", f"{op}: output shape {shape} does not match declared {d.shape}")
        return d.dtype


def expect_operands(op, name, ni, no):
    if len(op.inputs) != ni or len(op.outputs) != no:
        raise graph_error(name, f"expected {ni} inputs and {no} outputs")


def expect_rank(name, what, t: T, rank):
    if len(t.shape) != rank:
        raise OracleError("ShapeMismatch", f"{name}: {what} must have rank {rank}, got {t.shape}")


def single_value(name, what, t: T) -> T:
    expect_rank(name, what, t, 1)
    if t.values.size != 1:
        raise OracleError("ShapeMismatch", f"{name}: {what} must have exactly one element")
    return t


# ---------------------------------------------------------------------------
# Operators
# ---------------------------------------------------------------------------


def output_extent(name, size, pb, pa, k, d, s):
    """conv.rs:54-75"""
    full = size - 1 + pb + pa - (k - 1) * d
    if full % s != 0:
        raise graph_error(name, "parameters must yield exact integer output dimensions")
    out = full // s + 1
    if out < 1:
        raise graph_error(name, f"output dimension {out} must be positive")
    return out


def check_conv_attributes(name, dims, pad, stride, dil):
    """conv.rs:77-92"""
    if len(pad) != 2 * dims or len(stride) != dims or len(dil) != dims:
        raise graph_error(name, "bad attribute lengths")
    if any(p < 0 for p in pad):
        raise graph_error(name, "pad must be non-negative")
    if any(s < 1 for s in stride):
        raise graph_error(name, "stride must be at least 1")
    if any(d < 1 for d in dil):
        raise graph_error(name, "dilation must be at least 1")


def conv2d_types(i, w, acc, out):
    """conv.rs:375-385"""
    ok = lambda t, s: t in FP8_TYPES or t in s  # noqa: E731
    if (i, acc, out) == (D["INT8"], D["INT32"], D["INT32"]) and w in (D["INT8"], D["INT4"]):
        return True
    if (i, w, acc, out) == (D["INT16"], D["INT8"], D["INT48"], D["INT48"]):
        return True
    if acc == D["FP32"] and out == D["FP32"]:
        return all(ok(t, {D["FP16"], D["BF16"], D["FP32"]}) for t in (i, w))
    if acc in (D["FP16"], D["FP32"]) and out == D["FP16"]:
        return all(ok(t, {D["FP16"]}) for t in (i, w))
    if acc in (D["BF16"], D["FP32"]) and out == D["BF16"]:
        return all(ok(t, {D["BF16"]}) for t in (i, w))
    return False


def standard_types(i, w, acc, out):
    """conv.rs:388-396"""
    if (i, acc, out) == (D["INT8"], D["INT32"], D["INT32"]) and w in (D["INT8"], D["INT4"]):
        return True
    if (i, w, acc, out) == (D["INT16"], D["INT8"], D["INT48"], D["INT48"]):
        return True
    if (i, w, out) == (D["FP16"], D["FP16"], D["FP16"]) and acc in (D["FP16"], D["FP32"]):
        return True
    if (i, w, acc, out) in ((D["BF16"], D["BF16"], D["FP32"], D["BF16"]),
                            (D["FP32"], D["FP32"], D["FP32"], D["FP32"])):
        return True
    if i == w and i in FP8_TYPES:
        return (acc, out) in ((D["FP16"], D["FP16"]), (D["FP32"], D["FP32"]))
    return False


class Conv3dGeom(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int64) for k in ("n", "id", "ih", "iw", "ic", "oc", "kd", "kh", "kw", "od", "oh",
                                               "ow")] + \
               [("pad", ctypes.c_int64 * 6), ("stride", ctypes.c_int64 * 3), ("dilation", ctypes.c_int64 * 3)]


def eval_conv3d(st: State, op):
    """conv.rs:510-516 (eval_conv3d): eval_conv :398-500 with ConvNd::new :107-139, dims = 3."""
    name = "CONV3D"
    a = op.attr
    if not a:
        raise graph_error(name, "missing attribute")
    expect_operands(op, name, 5, 1)
    x = st.get(op.inputs[0])
    w = st.get(op.inputs[1])
    bias = st.get(op.inputs[2])
    izp = single_value(name, "input_zp", st.get(op.inputs[3]))
    wzp = single_value(name, "weight_zp", st.get(op.inputs[4]))
    expect_rank(name, "bias", bias, 1)
    expect_rank(name, "input", x, 5)
    expect_rank(name, "weight", w, 5)
    pad, stride, dil = a["pad"], a["stride"], a["dilation"]
    check_conv_attributes(name, 3, pad, stride, dil)
    n, idd, ih, iw, ic = x.shape
    oc, kd, kh, kw, kc = w.shape
    if kc != ic:
        raise OracleError("ShapeMismatch", f"{name}: weight input channels {kc} != input channels {ic}")
    sp = [output_extent(name, (idd, ih, iw)[d], pad[2 * d], pad[2 * d + 1], (kd, kh, kw)[d], dil[d], stride[d])
          for d in range(3)]
    out_shape = [n] + sp + [oc]
    bc = bias.shape[0]
    if bc != oc and bc != 1:
        raise OracleError("ShapeMismatch", f"{name}: bias channels {bc} must be 1 or {oc}")
    in_t, w_t, out_t, acc_t = x.dtype, w.dtype, bias.dtype, a["acc_type"]
    declared = st.declared(name, op.outputs[0], out_shape)
    if declared is not None and declared != out_t:
        raise OracleError("DTypeMismatch", f"{name}: output dtype does not match bias dtype")
    if not standard_types(in_t, w_t, acc_t, out_t):
        raise OracleError("DTypeMismatch", f"{name}: unsupported types")
    if izp.dtype != in_t or wzp.dtype != w_t:
        raise OracleError("DTypeMismatch", f"{name}: zero points must match input/weight dtypes")
    g = Conv3dGeom(n=n, id=idd, ih=ih, iw=iw, ic=ic, oc=oc, kd=kd, kh=kh, kw=kw, od=sp[0], oh=sp[1], ow=sp[2])
    for i in range(6):
        g.pad[i] = pad[i]
    for i in range(3):
        g.stride[i] = stride[i]
        g.dilation[i] = dil[i]
    L = lib()
    count = int(np.prod(out_shape))
    if acc_t in INT_TYPES:
        zx, zw = int(izp.values[0]), int(wzp.values[0])
        if zx != 0 and in_t != D["INT8"]:
            raise graph_error(name, "input zero point must be zero for non-int8 input")
        if zw != 0 and w_t != D["INT8"]:
            raise graph_error(name, "weight zero point must be zero for non-int8 weight")
        out = np.zeros(count, dtype=np.int64)
        L.orc_conv3d_int(ctypes.byref(g), _p(_i64(x.values)), _p(_i64(w.values)), _p(_i64(bias.values)),
                         ctypes.c_int64(bc), ctypes.c_int64(zx), ctypes.c_int64(zw),
                         ctypes.c_int(acc_t == D["INT48"]), _p(out))
        return T(out_t, out_shape, out)
    zx, zw = float(izp.values[0]), float(wzp.values[0])
    if zx != 0.0 or zw != 0.0:
        raise graph_error(name, "zero points must be zero for floating-point operands")
    out = np.zeros(count, dtype=np.float32)
    L.orc_conv3d_float(ctypes.byref(g), _p(_f32(x.values)), _p(_f32(w.values)), _p(_f32(bias.values)),
                       ctypes.c_int64(bc), ctypes.c_float(zx), ctypes.c_float(zw), ctypes.c_int(acc_t),
                       ctypes.c_int(out_t), _p(out))
    return T(out_t, out_shape, out)


def eval_conv(st: State, op, depthwise: bool, transpose: bool = False):
    """conv.rs:398-500 (eval_conv) with ConvNd::new :107-139 / Depthwise::new :201-223 /
    Transpose::new :286-329."""
    name = "TRANSPOSE_CONV2D" if transpose else "DEPTHWISE_CONV2D" if depthwise else "CONV2D"
    a = op.attr
    if not a:
        raise graph_error(name, "missing attribute")
    expect_operands(op, name, 5, 1)
    x = st.get(op.inputs[0])
    w = st.get(op.inputs[1])
    bias = st.get(op.inputs[2])
    izp = single_value(name, "input_zp", st.get(op.inputs[3]))
    wzp = single_value(name, "weight_zp", st.get(op.inputs[4]))
    expect_rank(name, "bias", bias, 1)
    expect_rank(name, "input", x, 4)
    expect_rank(name, "weight", w, 4)
    n, ih, iw, ic = x.shape
    if transpose:
        pad, stride, dil = a["out_pad"], a["stride"], [1, 1]
        if len(pad) != 4 or len(stride) != 2:
            raise graph_error(name, "out_pad must have 4 elements and stride 2")
        if any(v < 1 for v in stride):
            raise graph_error(name, "stride must be at least 1")
    else:
        pad, stride, dil = a["pad"], a["stride"], a["dilation"]
        check_conv_attributes(name, 2, pad, stride, dil)
    if depthwise:
        kh, kw, kc, m = w.shape
        if kc != ic:
            raise OracleError("ShapeMismatch", f"{name}: weight channels {kc} != input channels {ic}")
        oc = ic * m
    else:
        oc, kh, kw, kc = w.shape
        m = 1
        if kc != ic:
            raise OracleError("ShapeMismatch", f"{name}: weight input channels {kc} != input channels {ic}")
    if transpose:
        for i, p_ in enumerate(pad):
            if p_ <= -(kh if i < 2 else kw):
                raise graph_error(name, "out_pad must be greater than -kernel size")
        oh = (ih - 1) * stride[0] + pad[0] + pad[1] + kh
        ow = (iw - 1) * stride[1] + pad[2] + pad[3] + kw
        if oh < 1 or ow < 1:
            raise graph_error(name, "output size must be positive")
    else:
        oh = output_extent(name, ih, pad[0], pad[1], kh, dil[0], stride[0])
        ow = output_extent(name, iw, pad[2], pad[3], kw, dil[1], stride[1])
    out_shape = [n, oh, ow, oc]
    bc = bias.shape[0]
    if bc != oc and bc != 1:
        raise OracleError("ShapeMismatch", f"{name}: bias channels {bc} must be 1 or {oc}")
    in_t, w_t, out_t, acc_t = x.dtype, w.dtype, bias.dtype, a["acc_type"]
    declared = st.declared(name, op.outputs[0], out_shape)
    if declared is not None and declared != out_t:
        raise OracleError("DTypeMismatch", f"{name}: output dtype does not match bias dtype")
    types_ok = standard_types if depthwise or transpose else conv2d_types
    if not types_ok(in_t, w_t, acc_t, out_t):
        raise OracleError("DTypeMismatch", f"{name}: unsupported types")
    if izp.dtype != in_t or wzp.dtype != w_t:
        raise OracleError("DTypeMismatch", f"{name}: zero points must match input/weight dtypes")
    g = ConvGeom(n=n, ih=ih, iw=iw, ic=ic, oc=oc, kh=kh, kw=kw, oh=oh, ow=ow, m=m)
    for i in range(4):
        g.pad[i] = pad[i]
    for i in range(2):
        g.stride[i] = stride[i]
        g.dilation[i] = dil[i]
    L = lib()
    count = n * oh * ow * oc
    if acc_t in INT_TYPES:
        zx, zw = int(izp.values[0]), int(wzp.values[0])
        if zx != 0 and in_t != D["INT8"]:
            raise graph_error(name, "input zero point must be zero for non-int8 input")
        if zw != 0 and w_t != D["INT8"]:
            raise graph_error(name, "weight zero point must be zero for non-int8 weight")
        xi, wi, bi = _i64(x.values), _i64(w.values), _i64(bias.values)
        out = np.zeros(count, dtype=np.int64)
        fn = L.orc_transpose_conv2d_int if transpose else L.orc_depthwise_int if depthwise else L.orc_conv2d_int
        fn(ctypes.byref(g), _p(xi), _p(wi), _p(bi), ctypes.c_int64(bc), ctypes.c_int64(zx),
           ctypes.c_int64(zw), ctypes.c_int(acc_t == D["INT48"]), _p(out))
        return T(out_t, out_shape, out)
    zx, zw = float(izp.values[0]), float(wzp.values[0])
    if zx != 0.0 or zw != 0.0:
        raise graph_error(name, "zero points must be zero for floating-point operands")
    xf, wf, bf = _f32(x.values), _f32(w.values), _f32(bias.values)
    out = np.zeros(count, dtype=np.float32)
    fn = (L.orc_transpose_conv2d_float if transpose else L.orc_depthwise_float if depthwise
          else L.orc_conv2d_float)
    fn(ctypes.byref(g), _p(xf), _p(wf), _p(bf), ctypes.c_int64(bc), ctypes.c_float(zx),
       ctypes.c_float(zw), ctypes.c_int(acc_t), ctypes.c_int(out_t), _p(out))
    return T(out_t, out_shape, out)


def matmul_types(a, b, out):
    """matmul.rs:30-38"""
    if (a, b, out) in ((D["INT8"], D["INT8"], D["INT32"]), (D["INT16"], D["INT16"], D["INT48"])):
        return True
    if (a, b) == (D["FP16"], D["FP16"]) and out in (D["FP16"], D["FP32"]):
        return True
    if (a, b, out) in ((D["BF16"], D["BF16"], D["FP32"]), (D["FP32"], D["FP32"], D["FP32"])):
        return True
    if out in (D["FP16"], D["FP32"]):
        return a in FP8_TYPES and b in FP8_TYPES
    return False


def matmul_t_types(a, b, out):
    """matmul.rs:42-51"""
    fl = set(FP8_TYPES) | {D["FP16"], D["BF16"], D["FP32"]}
    if (a, b, out) in ((D["INT8"], D["INT8"], D["INT32"]), (D["INT16"], D["INT16"], D["INT48"]),
                       (D["FP16"], D["FP16"], D["FP16"])):
        return True
    if out == D["FP32"]:
        return a in fl and b in fl
    if out == D["BF16"]:
        return a in fl and b in fl and D["FP32"] not in (a, b) and (a, b) != (D["FP16"], D["FP16"])
    return False


def default_output(a):
    """matmul.rs:54-61"""
    if a == D["INT8"]:
        return D["INT32"]
    if a == D["INT16"]:
        return D["INT48"]
    if a in (D["FP16"],) or a in FP8_TYPES:
        return D["FP16"]
    return D["FP32"]


def eval_matmul(st: State, op):
    """matmul.rs:176-178"""
    return _eval_matmul(st, op, "MATMUL", False, matmul_types)


def eval_matmul_t(st: State, op):
    """matmul.rs:180-182: b [D,W,C], D == N or 1 (broadcast)"""
    return _eval_matmul(st, op, "MATMUL_T", True, matmul_t_types)


def _eval_matmul(st: State, op, name, transposed, types_ok):
    """matmul.rs:98-174"""
    expect_operands(op, name, 4, 1)
    a = st.get(op.inputs[0])
    b = st.get(op.inputs[1])
    azp = single_value(name, "a_zp", st.get(op.inputs[2]))
    bzp = single_value(name, "b_zp", st.get(op.inputs[3]))
    expect_rank(name, "a", a, 3)
    expect_rank(name, "b", b, 3)
    n, h, c = a.shape
    if transposed:
        bn, w, bc = b.shape
    else:
        bn, bc, w = b.shape
    if bc != c or (bn != n and not (transposed and bn == 1)):
        raise OracleError("ShapeMismatch", f"{name}: b shape {b.shape} incompatible with a {a.shape}")
    out_shape = [n, h, w]
    out_t = st.declared(name, op.outputs[0], out_shape)
    if out_t is None:
        out_t = default_output(a.dtype)
    if not types_ok(a.dtype, b.dtype, out_t):
        raise OracleError("DTypeMismatch", f"{name}: unsupported types")
    if azp.dtype != a.dtype or bzp.dtype != b.dtype:
        raise OracleError("DTypeMismatch", f"{name}: zero points must match input dtypes")
    L = lib()
    if out_t in INT_TYPES:
        za, zb = int(azp.values[0]), int(bzp.values[0])
        if (za != 0 and a.dtype != D["INT8"]) or (zb != 0 and b.dtype != D["INT8"]):
            raise graph_error(name, "zero points must be zero for non-int8 inputs")
        out = np.zeros(n * h * w, dtype=np.int64)
        if transposed:
            L.orc_matmul_t_int(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                               ctypes.c_int64(bn), _p(_i64(a.values)), _p(_i64(b.values)), ctypes.c_int64(za),
                               ctypes.c_int64(zb), ctypes.c_int(out_t == D["INT48"]), _p(out))
        else:
            L.orc_matmul_int(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                             _p(_i64(a.values)), _p(_i64(b.values)), ctypes.c_int64(za), ctypes.c_int64(zb),
                             ctypes.c_int(out_t == D["INT48"]), _p(out))
        return T(out_t, out_shape, out)
    if float(azp.values[0]) != 0.0 or float(bzp.values[0]) != 0.0:
        raise graph_error(name, "zero points must be zero for floating-point inputs")
    out = np.zeros(n * h * w, dtype=np.float32)
    if transposed:
        L.orc_matmul_t_float(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                             ctypes.c_int64(bn), _p(_f32(a.values)), _p(_f32(b.values)), ctypes.c_int(out_t), _p(out))
    else:
        L.orc_matmul_float(ctypes.c_int64(n), ctypes.c_int64(h), ctypes.c_int64(c), ctypes.c_int64(w),
                           _p(_f32(a.values)), _p(_f32(b.values)), ctypes.c_int(out_t), _p(out))
    return T(out_t, out_shape, out)


def eval_rescale(st: State, op):
    """type_conv.rs:111-191"""
    name = "RESCALE"
    a = op.attr
    if not a:
        raise graph_error(name, "missing attribute")
    expect_operands(op, name, 5, 1)
    x = st.get(op.inputs[0])
    mult = st.get(op.inputs[1])
    shift = st.get(op.inputs[2])
    izp = st.get(op.inputs[3])
    ozp = st.get(op.inputs[4])
    shape = list(x.shape)
    in_t = x.dtype
    out_t = st.declared(name, op.outputs[0], shape)
    if out_t is None:
        out_t = D["INT32"]
    scale32, rm, pc = a["scale32"], a["rounding_mode"], a["per_channel"]
    iu, ou = a["input_unsigned"], a["output_unsigned"]
    if in_t not in (D["INT8"], D["INT16"], D["INT32"], D["INT48"]) or \
            out_t not in (D["INT8"], D["INT16"], D["INT32"]):
        raise OracleError("DTypeMismatch", f"{name}: unsupported types")
    if rm not in (1, 2, 3):
        raise graph_error(name, "unsupported rounding mode")
    if scale32 and in_t == D["INT48"]:
        raise graph_error(name, "scale32 is not allowed for INT48 input")
    if not scale32 and rm == 3:
        raise graph_error(name, "double rounding requires scale32")
    has32 = in_t in (D["INT32"], D["INT48"]) or out_t == D["INT32"]
    if (iu and ou) or ((iu or ou) and has32):
        raise graph_error(name, "invalid combination of input_unsigned/output_unsigned and types")
    em = D["INT32"] if scale32 else D["INT16"]
    if mult.dtype != em or shift.dtype != D["INT8"]:
        raise OracleError("DTypeMismatch", f"{name}: multiplier/shift dtypes")
    if izp.dtype != in_t or ozp.dtype != out_t or izp.values.size != 1 or ozp.values.size != 1:
        raise graph_error(name, "zero points must be single elements of the input/output types")
    if pc:
        if not shape:
            raise graph_error(name, "per_channel requires rank >= 1")
        channels = shape[-1]
    else:
        channels = 1
    if mult.values.size != channels or shift.values.size != channels:
        raise graph_error(name, f"multiplier and shift must have {channels} elements")
    bw = {D["INT8"]: 8, D["INT16"]: 16, D["INT32"]: 32}.get

    def extend(t, v, uns):
        return v & ((1 << bw(t, 48)) - 1) if uns else v

    izp_v = extend(in_t, int(izp.values[0]), iu)
    ozp_v = extend(out_t, int(ozp.values[0]), ou)

    def zp_ok(t, zp, uns):
        return t == D["INT8"] or zp == 0 or (t == D["INT16"] and uns and zp == 32768)

    if not zp_ok(in_t, izp_v, iu) or not zp_ok(out_t, ozp_v, ou):
        raise graph_error(name, "zero point not allowed for this type")
    out = np.zeros(x.values.size, dtype=np.int64)
    rc = lib().orc_rescale(_p(_i64(x.values)), ctypes.c_int64(x.values.size), ctypes.c_int(in_t),
                           ctypes.c_int(out_t), _p(_i64(mult.values)), _p(_i64(shift.values)),
                           ctypes.c_int64(channels), ctypes.c_int64(int(izp.values[0])),
                           ctypes.c_int64(int(ozp.values[0])), ctypes.c_int(scale32),
                           ctypes.c_int(rm), ctypes.c_int(pc), ctypes.c_int(iu), ctypes.c_int(ou),
                           _p(out))
    if rc:
        raise graph_error(name, "apply_scale / int32 range failure")
    return T(out_t, shape, out)


def pool_geometry(name, x: T, kernel, stride, pad):
    """pool.rs:31-70"""
    expect_rank(name, "input", x, 4)
    if len(pad) != 4 or len(kernel) != 2 or len(stride) != 2:
        raise graph_error(name, "pad must have 4 elements, kernel and stride 2")
    if any(p < 0 for p in pad):
        raise graph_error(name, "pad must be non-negative")
    if any(k < 1 for k in list(kernel) + list(stride)):
        raise graph_error(name, "kernel and stride must be at least 1")
    if pad[0] >= kernel[0] or pad[1] >= kernel[0] or pad[2] >= kernel[1] or pad[3] >= kernel[1]:
        raise graph_error(name, "pad must be smaller than kernel")
    n, ih, iw, c = x.shape
    if ih == 0 or iw == 0:
        raise graph_error(name, "input height and width must be positive")

    def extent(size, a, b, k, s):
        full = size + a + b - k
        if full < 0 or full % s != 0:
            raise graph_error(name, "parameters must yield exact integer output dimensions")
        return full // s + 1

    oh = extent(ih, pad[0], pad[1], kernel[0], stride[0])
    ow = extent(iw, pad[2], pad[3], kernel[1], stride[1])
    g = PoolGeom(n=n, ih=ih, iw=iw, c=c, oh=oh, ow=ow, pad_top=pad[0], pad_left=pad[2])
    g.kernel[0], g.kernel[1] = kernel
    g.stride[0], g.stride[1] = stride
    return g, [n, oh, ow, c]


def check_output_dtype(name, declared, in_t):
    if declared is not None and declared != in_t:
        raise OracleError("DTypeMismatch", f"{name}: output dtype must match input dtype")


def eval_avg_pool(st: State, op):
    """pool.rs:146-231"""
    name = "AVG_POOL2D"
    a = op.attr
    if not a:
        raise graph_error(name, "missing attribute")
    expect_operands(op, name, 3, 1)
    x = st.get(op.inputs[0])
    izp = single_value(name, "input_zp", st.get(op.inputs[1]))
    ozp = single_value(name, "output_zp", st.get(op.inputs[2]))
    g, out_shape = pool_geometry(name, x, a["kernel"], a["stride"], a["pad"])
    in_t, acc_t = x.dtype, a["acc_type"]
    check_output_dtype(name, st.declared(name, op.outputs[0], out_shape), in_t)
    ok = ((in_t in (D["INT8"], D["INT16"]) and acc_t == D["INT32"])
          or (in_t == D["FP16"] and acc_t in (D["FP16"], D["FP32"]))
          or ((in_t, acc_t) in ((D["BF16"], D["FP32"]), (D["FP32"], D["FP32"])))
          or (in_t in FP8_TYPES and acc_t == D["FP16"]))
    if not ok:
        raise OracleError("DTypeMismatch", f"{name}: unsupported types")
    if izp.dtype != in_t or ozp.dtype != in_t:
        raise OracleError("DTypeMismatch", f"{name}: zero points must have the input dtype")
    count = int(np.prod(out_shape))
    if in_t in INT_TYPES:
        zi, zo = int(izp.values[0]), int(ozp.values[0])
        if in_t != D["INT8"] and (zi != 0 or zo != 0):
            raise graph_error(name, "zero points must be zero for non-int8 data")
        out = np.zeros(count, dtype=np.int64)
        if lib().orc_avg_pool_int(ctypes.byref(g), _p(_i64(x.values)), ctypes.c_int(in_t),
                                  ctypes.c_int64(zi), ctypes.c_int64(zo), _p(out)):
            raise graph_error(name, "apply_scale_32 failure")
        return T(in_t, out_shape, out)
    if float(izp.values[0]) != 0.0 or float(ozp.values[0]) != 0.0:
        raise graph_error(name, "zero points must be zero for floating-point data")
    out = np.zeros(count, dtype=np.float32)
    lib().orc_avg_pool_float(ctypes.byref(g), _p(_f32(x.values)), ctypes.c_int(in_t),
                             ctypes.c_int(acc_t), _p(out))
    return T(in_t, out_shape, out)


def eval_max_pool(st: State, op):
    """pool.rs:233-286"""
    name = "MAX_POOL2D"
    a = op.attr
    if not a:
        raise graph_error(name, "missing attribute")
    expect_operands(op, name, 1, 1)
    nan_mode = a["nan_mode"]
    if nan_mode not in (1, 2):
        raise graph_error(name, "nan_mode must be PROPAGATE or IGNORE")
    x = st.get(op.inputs[0])
    g, out_shape = pool_geometry(name, x, a["kernel"], a["stride"], a["pad"])
    in_t = x.dtype
    check_output_dtype(name, st.declared(name, op.outputs[0], out_shape), in_t)
    count = int(np.prod(out_shape))
    if in_t in (D["INT8"], D["INT16"]):
        out = np.zeros(count, dtype=np.int64)
        lib().orc_max_pool_int(ctypes.byref(g), _p(_i64(x.values)), ctypes.c_int(in_t), _p(out))
        return T(in_t, out_shape, out)
    if in_t in FLOAT_TYPES:
        out = np.zeros(count, dtype=np.float32)
        lib().orc_max_pool_float(ctypes.byref(g), _p(_f32(x.values)), ctypes.c_int(in_t),
                                 ctypes.c_int(nan_mode), _p(out))
        return T(in_t, out_shape, out)
    raise OracleError("DTypeMismatch", f"{name}: unsupported dtype")


def eval_clamp(st: State, op):
    """elementwise.rs:319-343"""
    name = "CLAMP"
    a = op.attr
    if not a:
        raise graph_error(name, "missing attribute")
    nan_mode = a["nan_mode"]
    if nan_mode not in (1, 2):
        raise graph_error(name, "nan_mode must be PROPAGATE or IGNORE")
    x = st.get(op.inputs[0] if op.inputs else "")
    dt = x.dtype
    try:
        lo_v = decode_raw(dt, a["min_val"], 1)
        hi_v = decode_raw(dt, a["max_val"], 1)
    except OracleError:
        raise graph_error(name, "malformed min/max")
    expect_operands(op, name, 1, 1)
    if dt not in (D["FP16"], D["BF16"], D["FP32"], D["INT8"], D["INT16"]):
        raise OracleError("DTypeMismatch", f"{name}: unsupported dtype")
    n = x.values.size
    if dt in INT_TYPES:
        lo, hi = int(lo_v[0]), int(hi_v[0])
        if hi < lo:
            raise graph_error(name, "max_val must not be smaller than min_val")
        out = np.zeros(n, dtype=np.int64)
        lib().orc_clamp_int(_p(_i64(x.values)), ctypes.c_int64(n), ctypes.c_int64(lo),
                            ctypes.c_int64(hi), _p(out))
    else:
        lo, hi = float(lo_v[0]), float(hi_v[0])
        if np.isnan(lo) or np.isnan(hi) or hi < lo:
            raise graph_error(name, "min_val/max_val must be ordered and not NaN")
        out = np.zeros(n, dtype=np.float32)
        lib().orc_clamp_float(_p(_f32(x.values)), ctypes.c_int64(n), ctypes.c_float(lo),
                              ctypes.c_float(hi), ctypes.c_int(nan_mode), ctypes.c_int(dt), _p(out))
    finish(st, op, name, list(x.shape), dt)
    return T(dt, list(x.shape), out)


def finish(st, op, name, shape, dtype):
    declared = st.declared(name, op.outputs[0], shape)
    if declared is not None and declared != dtype:
        raise OracleError("DTypeMismatch", f"{name}: output dtype mismatch")


def eval_add(st: State, op):
    """elementwise.rs:395-397 with broadcasting (elementwise.rs:346-360)."""
    name = "ADD"
    expect_operands(op, name, 2, 1)
    a, b = st.get(op.inputs[0]), st.get(op.inputs[1])
    if a.dtype != b.dtype:
        raise OracleError("DTypeMismatch", f"{name}: input dtypes differ")
    try:  # broadcast.rs:3-26 (numpy's right-aligned rule)
        shape = list(np.broadcast_shapes(tuple(a.shape), tuple(b.shape)))
    except ValueError:
        raise OracleError("Broadcast", f"{name}: shapes {a.shape} and {b.shape} are not compatible")
    if a.dtype not in (D["FP16"], D["BF16"], D["FP32"], D["INT32"], D["INT64"]):
        raise OracleError("DTypeMismatch", f"{name}: unsupported dtype")
    av = np.broadcast_to(a.values.reshape(a.shape), shape).reshape(-1)
    bv = np.broadcast_to(b.values.reshape(b.shape), shape).reshape(-1)
    if a.dtype in INT_TYPES:
        out = np.zeros(av.size, dtype=np.int64)
        lib().orc_add_int(_p(_i64(av)), _p(_i64(bv)), ctypes.c_int64(av.size),
                          ctypes.c_int(a.dtype), _p(out))
    else:
        out = round_to(a.dtype, _f32(av) + _f32(bv))
    finish(st, op, name, shape, a.dtype)
    return T(a.dtype, shape, out)


def eval_reshape(st: State, op):
    """data_layout.rs:163-177"""
    name = "RESHAPE"
    expect_operands(op, name, 2, 1)
    x = st.get(op.inputs[0])
    s = st.get(op.inputs[1])
    if s.dtype not in INT_TYPES and s.dtype != D["SHAPE"]:
        raise graph_error(name, "shape operand must be a shape")
    new_shape = [int(v) for v in s.values]
    if any(d < 0 for d in new_shape):
        raise graph_error(name, "shape must be non-negative")
    if int(np.prod(new_shape)) != int(np.prod(x.shape)):
        raise OracleError("ShapeMismatch", f"{name}: cannot reshape {x.shape} to {new_shape}")
    finish(st, op, name, new_shape, x.dtype)
    return T(x.dtype, new_shape, x.values)


def eval_transpose(st: State, op):
    name = "TRANSPOSE"
    expect_operands(op, name, 1, 1)
    x = st.get(op.inputs[0])
    perms = op.attr["perms"]
    v = x.values.reshape(x.shape).transpose(perms)
    return T(x.dtype, list(v.shape), np.ascontiguousarray(v).reshape(-1))


def eval_const(st: State, op):
    """data_nodes.rs:6-22"""
    name = op.outputs[0] if op.outputs else None
    if name is None:
        raise graph_error("CONST", "CONST op has no output")
    d = st.defs.get(name)
    if d is None:
        raise OracleError("TensorNotFound", name)
    shape = [max(s, 0) for s in d.shape]
    count = int(np.prod(shape)) if shape else 1
    if d.dtype == D["SHAPE"]:
        count = shape[0] if shape else 0
    return T(d.dtype, shape, decode_raw(d.dtype, d.data, count))


def eval_identity(st: State, op):
    x = st.get(op.inputs[0])
    return T(x.dtype, list(x.shape), x.values)


EVAL = {
    "CONST": eval_const, "CONST_SHAPE": eval_const, "IDENTITY": eval_identity,
    "CONV2D": lambda s, o: eval_conv(s, o, False),
    "DEPTHWISE_CONV2D": lambda s, o: eval_conv(s, o, True),
    "TRANSPOSE_CONV2D": lambda s, o: eval_conv(s, o, False, transpose=True),
    "CONV3D": eval_conv3d,
    "MATMUL": eval_matmul, "MATMUL_T": eval_matmul_t, "RESCALE": eval_rescale, "AVG_POOL2D": eval_avg_pool,
    "MAX_POOL2D": eval_max_pool, "CLAMP": eval_clamp, "ADD": eval_add,
    "RESHAPE": eval_reshape, "TRANSPOSE": eval_transpose,
}


def run_block(block, inputs: dict, trace: list | None = None):
    """Dataflow execution in the reference's ready-queue order
    (src/interpreter.rs:154-245). Returns {output name: T}. With `trace`, appends
    (op_index, op name, input shapes, output shapes) per executed operator --
    the post_op events the reference's hooks see (src/interpreter.rs:199-216)."""
    st = State(block, inputs)
    available = set(st.tensors)
    ready = deque(i for i, op in enumerate(block.operators)
                  if op.name in ("CONST",) or all(n in available for n in op.inputs))
    executed = [False] * len(block.operators)
    while ready:
        i = ready.popleft()
        if executed[i]:
            continue
        op = block.operators[i]
        fn = EVAL.get(op.name)
        if fn is None:
            raise OracleError("UnsupportedOp", op.name)
        res = fn(st, op)
        st.tensors[op.outputs[0]] = res
        if trace is not None:
            trace.append((i, op.name, [list(st.tensors[n].shape) for n in op.inputs if n in st.tensors],
                          [list(res.shape)]))
        executed[i] = True
        available.update(op.outputs)
        for j, nxt in enumerate(block.operators):
            if not executed[j] and j not in ready and (
                    nxt.name == "CONST" or all(n in available for n in nxt.inputs)):
                ready.append(j)
    if not all(executed):
        raise graph_error("graph", "could not execute all ops")
    return {n: st.tensors[n] for n in block.outputs if n in st.tensors}


# ---------------------------------------------------------------------------
# Fixture cases (tests/golden/*.zip)
# ---------------------------------------------------------------------------


@dataclass
class Case:
    name: str
    desc: dict
    graph_bytes: bytes
    files: dict  # filename -> bytes

    def npy(self, fn):
        return np.load(io.BytesIO(self.files[fn]), allow_pickle=False)


def load_cases(zip_path):
    z = zipfile.ZipFile(zip_path)
    by_case = {}
    for n in z.namelist():
        case, fn = n.split("/", 1)
        by_case.setdefault(case, {})[fn] = z.read(n)
    out = []
    for case in sorted(by_case):
        files = by_case[case]
        desc = json.loads(files["desc.json"])
        out.append(Case(case, desc, files[desc["tosa_file"]], files))
    return out


def case_inputs(case: Case, block):
    inputs = {}
    for name, fn in zip(case.desc["ifm_name"], case.desc["ifm_file"]):
        arr = case.npy(fn)
        td = block.tensor(name)
        dt = td.dtype if td is not None else D["FP32"]
        inputs[name] = T(dt, list(arr.shape), from_npy(arr, dt))
    return inputs


def run_case(case: Case):
    """Run one fixture through the oracle; returns {name: (expected_bits, actual_bits)}.
    Raises OracleError where the reference returns Err."""
    g = read_graph(case.graph_bytes)
    block = g.main_block
    outs = run_block(block, case_inputs(case, block))
    result = {}
    for name, fn in zip(case.desc["ofm_name"], case.desc["ofm_file"]):
        exp = case.npy(fn)
        td = block.tensor(name)
        got = outs[name]
        exp_vals = from_npy(exp, td.dtype)
        result[name] = (to_bits(td.dtype, exp_vals).reshape(-1), to_bits(td.dtype, got.values).reshape(-1),
                        list(exp.shape), list(got.shape))
    return result
