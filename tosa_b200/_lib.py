"""ctypes binding of libtosa_b200.so (the C ABI declared in include/tosa_b200.h).

Device memory comes from PyTorch tensors (their data_ptr()); streams are
torch.cuda streams. The library is loaded from this package directory and must
have been built for sm_100a (tosa_b200/build.py); there is no fallback: if the
library or a CUDA device is missing every call raises.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtosa_b200.so")

# DType codes (schema/tosa.fbs:26-46), as in tosa_b200.h
DT_BOOL, DT_INT4, DT_INT8, DT_INT16, DT_INT32, DT_INT48 = 1, 2, 3, 4, 5, 6
DT_FP32, DT_FP16, DT_BF16, DT_SHAPE, DT_FP8E4M3, DT_FP8E5M2, DT_INT64 = 7, 8, 9, 10, 11, 12, 17
ROUND_SINGLE, ROUND_INEXACT, ROUND_DOUBLE = 1, 2, 3
NAN_PROPAGATE, NAN_IGNORE = 1, 2

STATUS_NAMES = {
    0: "OK", 1: "Deserialize", 2: "UnsupportedOp", 3: "TensorNotFound", 4: "DTypeMismatch",
    5: "ShapeMismatch", 6: "Broadcast", 7: "GraphError", 8: "ControlFlow", 9: "Io",
    64: "Cuda", 65: "Timeout", 66: "InvalidArgument", 67: "NotAccelerated",
}
TB_ERR_NOT_ACCELERATED = 67


class TbError(RuntimeError):
    """A non-OK tb_status; `.kind` is the reference Error variant name."""

    def __init__(self, status: int, msg: str):
        self.status = status
        self.kind = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.kind}: {msg}")


class RescaleAttr(ctypes.Structure):
    _fields_ = [("scale32", ctypes.c_int32), ("rounding_mode", ctypes.c_int32),
                ("per_channel", ctypes.c_int32), ("input_unsigned", ctypes.c_int32),
                ("output_unsigned", ctypes.c_int32), ("input_zp", ctypes.c_int32),
                ("output_zp", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
                ("channels", ctypes.c_int32), ("multiplier", ctypes.POINTER(ctypes.c_int32)),
                ("shift", ctypes.POINTER(ctypes.c_int8)), ("clamp_enabled", ctypes.c_int32),
                ("clamp_min", ctypes.c_int32), ("clamp_max", ctypes.c_int32)]


class MatmulDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("n", "h", "c", "w", "a_dtype", "b_dtype", "out_dtype",
                                              "a_zp", "b_zp")]


class Conv2dDesc(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32), ("ih", ctypes.c_int32), ("iw", ctypes.c_int32), ("ic", ctypes.c_int32),
                ("oc", ctypes.c_int32), ("kh", ctypes.c_int32), ("kw", ctypes.c_int32), ("m", ctypes.c_int32),
                ("pad", ctypes.c_int32 * 4), ("stride", ctypes.c_int32 * 2), ("dilation", ctypes.c_int32 * 2),
                ("in_dtype", ctypes.c_int32), ("w_dtype", ctypes.c_int32), ("acc_dtype", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("input_zp", ctypes.c_int32), ("weight_zp", ctypes.c_int32),
                ("bias_len", ctypes.c_int32)]


class Conv3dDesc(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int32) for k in ("n", "id", "ih", "iw", "ic", "oc", "kd", "kh", "kw")] + \
               [("pad", ctypes.c_int32 * 6), ("stride", ctypes.c_int32 * 3), ("dilation", ctypes.c_int32 * 3)] + \
               [(k, ctypes.c_int32) for k in ("in_dtype", "w_dtype", "acc_dtype", "out_dtype", "input_zp",
                                              "weight_zp", "bias_len")]


class Pool2dDesc(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32), ("ih", ctypes.c_int32), ("iw", ctypes.c_int32), ("c", ctypes.c_int32),
                ("kernel", ctypes.c_int32 * 2), ("stride", ctypes.c_int32 * 2), ("pad", ctypes.c_int32 * 4),
                ("dtype", ctypes.c_int32), ("acc_dtype", ctypes.c_int32), ("input_zp", ctypes.c_int32),
                ("output_zp", ctypes.c_int32), ("nan_mode", ctypes.c_int32)]


class TensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("shape", ctypes.POINTER(ctypes.c_int64)), ("bytes", ctypes.c_uint64), ("data", ctypes.c_void_p)]


class OpInfoC(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("op_index", ctypes.c_int32)]


PRE_OP = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.POINTER(OpInfoC), ctypes.POINTER(TensorInfo), ctypes.c_int32)
POST_OP = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.POINTER(OpInfoC), ctypes.POINTER(TensorInfo), ctypes.c_int32,
                           ctypes.POINTER(TensorInfo), ctypes.c_int32)
ON_ALLOC = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int32,
                            ctypes.c_int32, ctypes.c_uint64)
ON_FREE = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_uint64)


class Hooks(ctypes.Structure):
    _fields_ = [("user", ctypes.c_void_p), ("pre_op", PRE_OP), ("post_op", POST_OP), ("on_tensor_alloc", ON_ALLOC),
                ("on_tensor_free", ON_FREE)]


GRAPH_NO_FUSION, GRAPH_SYNC_EACH_OP, GRAPH_CUDA_GRAPH, GRAPH_TIME_OPS = 1, 2, 4, 8

_V = ctypes.c_void_p
_P = ctypes.POINTER
_I = ctypes.c_int32
_L = ctypes.c_int64

# (name, restype, argtypes) for every entry point declared in tosa_b200.h
SIGNATURES = [
    ("tb_context_create", _I, [ctypes.c_int, _P(_V)]),
    ("tb_context_destroy", None, [_V]),
    ("tb_last_error", ctypes.c_char_p, []),
    ("tb_synchronize", _I, [_V, _V]),
    ("tb_malloc", _I, [_V, ctypes.c_size_t, _P(_V)]),
    ("tb_free", _I, [_V, _V]),
    ("tb_memcpy_h2d", _I, [_V, _V, _V, ctypes.c_size_t, _V]),
    ("tb_memcpy_d2h", _I, [_V, _V, _V, ctypes.c_size_t, _V]),
    ("tb_launch_count", ctypes.c_uint64, [_V]),
    ("tb_debug_trace", _I, [_V, _P(ctypes.c_longlong)]),
    ("tb_context_set_wait_timeout_ms", _I, [_V, ctypes.c_double]),
    ("tb_matmul_plan_create", _I, [_V, _P(MatmulDesc), _P(RescaleAttr), _P(_V)]),
    ("tb_matmul_plan_run", _I, [_V, _V, _V, _V, _V]),
    ("tb_matmul_plan_set_constant_b", _I, [_V, _V, _V]),
    ("tb_matmul_plan_destroy", None, [_V]),
    ("tb_matmul", _I, [_V, _P(MatmulDesc), _P(RescaleAttr), _V, _V, _V, _V]),
    ("tb_matmul_i8_noalloc", _I, [_P(MatmulDesc), _P(RescaleAttr), _V, _V, _V, _V]),
    ("tb_matmul_t_plan_create", _I, [_V, _P(MatmulDesc), ctypes.c_int32, _P(RescaleAttr), _P(_V)]),
    ("tb_matmul_t", _I, [_V, _P(MatmulDesc), ctypes.c_int32, _P(RescaleAttr), _V, _V, _V, _V]),
    ("tb_conv2d_plan_create", _I, [_V, _P(Conv2dDesc), _V, _V, _P(RescaleAttr), _P(_V)]),
    ("tb_depthwise_conv2d_plan_create", _I, [_V, _P(Conv2dDesc), _V, _V, _P(RescaleAttr), _P(_V)]),
    ("tb_conv2d_plan_run", _I, [_V, _V, _V, _V]),
    ("tb_conv2d_plan_destroy", None, [_V]),
    ("tb_conv2d", _I, [_V, _P(Conv2dDesc), _P(RescaleAttr), _V, _V, _V, _V, _V]),
    ("tb_depthwise_conv2d", _I, [_V, _P(Conv2dDesc), _P(RescaleAttr), _V, _V, _V, _V, _V]),
    ("tb_conv3d_plan_create", _I, [_V, _P(Conv3dDesc), _V, _V, _P(RescaleAttr), _P(_V)]),
    ("tb_conv3d", _I, [_V, _P(Conv3dDesc), _P(RescaleAttr), _V, _V, _V, _V, _V]),
    ("tb_transpose_conv2d_plan_create", _I, [_V, _P(Conv2dDesc), _V, _V, _P(RescaleAttr), _P(_V)]),
    ("tb_transpose_conv2d", _I, [_V, _P(Conv2dDesc), _P(RescaleAttr), _V, _V, _V, _V, _V]),
    ("tb_rescale", _I, [_V, _P(RescaleAttr), _I, _V, _L, _V, _V]),
    ("tb_clamp", _I, [_V, _I, _V, _L, _L, _L, ctypes.c_float, ctypes.c_float, _I, _V, _V]),
    ("tb_add", _I, [_V, _I, _V, _V, _L, _V, _V]),
    ("tb_avg_pool2d", _I, [_V, _P(Pool2dDesc), _V, _V, _V]),
    ("tb_max_pool2d", _I, [_V, _P(Pool2dDesc), _V, _V, _V]),
    ("tb_graph_load", _I, [_V, _V, ctypes.c_size_t, ctypes.c_uint32, _P(_V)]),
    ("tb_graph_destroy", None, [_V]),
    ("tb_graph_num_inputs", _I, [_V]),
    ("tb_graph_num_outputs", _I, [_V]),
    ("tb_graph_input_info", _I, [_V, _I, _P(TensorInfo)]),
    ("tb_graph_output_info", _I, [_V, _I, _P(TensorInfo)]),
    ("tb_graph_set_input", _I, [_V, ctypes.c_char_p, _I, _P(_L), _I, _V, ctypes.c_uint64, _I, _V]),
    ("tb_graph_run", _I, [_V, _P(Hooks), _V]),
    ("tb_graph_get_output", _I, [_V, ctypes.c_char_p, _P(TensorInfo)]),
    ("tb_graph_read_output", _I, [_V, ctypes.c_char_p, _V, ctypes.c_uint64, _V]),
    ("tb_graph_last_launches", ctypes.c_uint64, [_V]),
    ("tb_graph_op_time_ms", ctypes.c_float, [_V, _I]),
]

_lib = None


def load(path: str = LIB_PATH):
    """Load the library and declare every entry point's signature."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise OSError(f"{path} is missing: build it with `python -m tosa_b200.build`")
        lib = ctypes.CDLL(path)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int):
    if status != 0:
        raise TbError(status, (load().tb_last_error() or b"").decode(errors="replace"))


def stream_ptr(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


class Context:
    """One tb_context on a CUDA device."""

    def __init__(self, device: int = 0):
        lib = load()
        h = ctypes.c_void_p()
        check(lib.tb_context_create(device, ctypes.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            load().tb_context_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self, stream=None):
        check(load().tb_synchronize(self.h, stream_ptr(stream)))

    @property
    def launches(self) -> int:
        return int(load().tb_launch_count(self.h))


def rescale_attr(multiplier, shift, *, scale32=True, rounding=ROUND_SINGLE, per_channel=None,
                 input_zp=0, output_zp=0, out_dtype=DT_INT8, input_unsigned=False,
                 output_unsigned=False, clamp=None):
    """Build a RescaleAttr; keeps the host arrays alive on the returned object."""
    m = (ctypes.c_int32 * len(multiplier))(*[int(v) for v in multiplier])
    s = (ctypes.c_int8 * len(shift))(*[int(v) for v in shift])
    a = RescaleAttr()
    a.scale32 = int(bool(scale32))
    a.rounding_mode = rounding
    a.per_channel = int(len(multiplier) > 1 if per_channel is None else bool(per_channel))
    a.input_unsigned = int(bool(input_unsigned))
    a.output_unsigned = int(bool(output_unsigned))
    a.input_zp = int(input_zp)
    a.output_zp = int(output_zp)
    a.out_dtype = out_dtype
    a.channels = len(multiplier)
    a.multiplier = ctypes.cast(m, ctypes.POINTER(ctypes.c_int32))
    a.shift = ctypes.cast(s, ctypes.POINTER(ctypes.c_int8))
    a.clamp_enabled = 0 if clamp is None else 1
    if clamp is not None:
        a.clamp_min, a.clamp_max = int(clamp[0]), int(clamp[1])
    a._keep = (m, s)
    return a


def conv_desc(n, ih, iw, ic, oc, kh, kw, pad, stride, dilation, in_dtype, w_dtype, acc_dtype, out_dtype,
              input_zp=0, weight_zp=0, bias_len=None, m=1):
    d = Conv2dDesc()
    d.n, d.ih, d.iw, d.ic, d.oc, d.kh, d.kw, d.m = n, ih, iw, ic, oc, kh, kw, m
    for i in range(4):
        d.pad[i] = pad[i]
    for i in range(2):
        d.stride[i] = stride[i]
        d.dilation[i] = dilation[i]
    d.in_dtype, d.w_dtype, d.acc_dtype, d.out_dtype = in_dtype, w_dtype, acc_dtype, out_dtype
    d.input_zp, d.weight_zp = input_zp, weight_zp
    d.bias_len = oc if bias_len is None else bias_len
    return d


def conv_out_hw(ih, iw, kh, kw, pad, stride, dilation):
    oh = (ih - 1 + pad[0] + pad[1] - (kh - 1) * dilation[0]) // stride[0] + 1
    ow = (iw - 1 + pad[2] + pad[3] - (kw - 1) * dilation[1]) // stride[1] + 1
    return oh, ow
