"""`.npy` files in the encodings the TOSA reference model writes for every TOSA
element type (the reference's reader/writer: src/npy.rs:1-7, parse :73-98,
write :200-229).

NumPy has no BF16 or FP8 types, so those are stored as raw bit patterns: BF16
as '<V2', FP8E4M3 as '<V1', FP8E5M2 as '|u1'; INT48 is stored as '<i8' and INT4
as '|i1' (one value per byte). Reading therefore needs the TOSA dtype as well
as the file. Tensors are the interpreter's host ``Tensor`` (storage form: BF16
as uint16 bits, FP8 as uint8 bits, INT4 one int8 per element, INT48 as int64).

The writer's header is the reference's: version 1.0, ``{'descr': ..,
'fortran_order': False, 'shape': (..), }`` padded with spaces so the data
starts on a 64-byte boundary, ending in a newline.
"""

from __future__ import annotations

import numpy as np

from . import _lib as L
from .interpreter import Tensor

MAGIC = b"\x93NUMPY"

# TOSA dtype -> (descr, numpy storage of the body)
_WRITE = {
    L.DT_BOOL: ("|b1", np.uint8), L.DT_INT4: ("|i1", np.int8), L.DT_INT8: ("|i1", np.int8),
    L.DT_INT16: ("<i2", "<i2"), L.DT_INT32: ("<i4", "<i4"), L.DT_INT48: ("<i8", "<i8"),
    L.DT_INT64: ("<i8", "<i8"), L.DT_SHAPE: ("<i8", "<i8"),
    L.DT_FP8E4M3: ("<V1", np.uint8), L.DT_FP8E5M2: ("|u1", np.uint8),
    L.DT_FP16: ("<f2", "<f2"), L.DT_BF16: ("<V2", "<u2"), L.DT_FP32: ("<f4", "<f4"),
}


class NpyError(ValueError):
    """A malformed or unsupported .npy file (the reference's Error::Deserialize), or
    one whose element encoding does not fit the requested dtype (Error::DTypeMismatch:
    ``kind`` says which)."""

    def __init__(self, msg: str, kind: str = "Deserialize"):
        super().__init__(f"npy: {msg}")
        self.kind = kind


def _header_value(header: str, key: str) -> str:
    pat = f"'{key}':"
    i = header.find(pat)
    if i < 0:
        raise NpyError(f"missing '{key}' in header")
    return header[i + len(pat):].lstrip()


def parse(data: bytes):
    """(kind, size, shape, raw little-endian body) of an .npy file."""
    if len(data) < 10 or data[:6] != MAGIC:
        raise NpyError("not an npy file")
    if data[6] == 1:
        hlen, start = int.from_bytes(data[8:10], "little"), 10
    elif data[6] in (2, 3):
        if len(data) < 12:
            raise NpyError("truncated header")
        hlen, start = int.from_bytes(data[8:12], "little"), 12
    else:
        raise NpyError(f"unsupported version {data[6]}")
    if start + hlen > len(data):
        raise NpyError("truncated header")
    try:
        header = data[start:start + hlen].decode("utf-8")
    except UnicodeDecodeError:
        raise NpyError("header is not UTF-8") from None
    if "'fortran_order': True" in header:
        raise NpyError("fortran-ordered arrays are not supported")
    v = _header_value(header, "descr")
    if not v or v[0] not in "'\"":
        raise NpyError("structured dtypes are not supported")
    end = v.find(v[0], 1)
    if end < 0:
        raise NpyError("unterminated descr")
    s = v[1:end]
    if not s:
        raise NpyError("empty descr")
    if s[0] == ">":
        raise NpyError(f"big-endian data is not supported ({s})")
    kind, size = (s[1], s[2:]) if s[0] in "<|=" else (s[0], s[1:])
    if kind not in "biufV" or not size.isdigit():
        raise NpyError(f"unsupported descr {s}")
    size = int(size)
    sv = _header_value(header, "shape")
    if not sv.startswith("(") or ")" not in sv:
        raise NpyError("bad shape")
    dims = [d.strip() for d in sv[1:sv.index(")")].split(",") if d.strip()]
    if not all(d.isdigit() for d in dims):
        raise NpyError("bad shape dimension")
    shape = [int(d) for d in dims]
    n = int(np.prod(shape)) if shape else 1
    body = data[start + hlen:start + hlen + n * size]
    if len(body) != n * size:
        raise NpyError(f"expected {n * size} bytes of data")
    return kind, size, shape, body


def _uint_bits(body: bytes, size: int) -> np.ndarray:
    if size in (1, 2, 4, 8):
        return np.frombuffer(body, dtype=f"<u{size}").astype(np.uint64)
    raise NpyError(f"{size}-byte elements are not supported")


def _ints(kind, size, body) -> np.ndarray:
    if kind == "i" and size <= 8:
        return np.frombuffer(body, dtype=f"<i{size}").astype(np.int64)
    if kind in "ub" and size <= 8:
        return _uint_bits(body, size).astype(np.int64)
    raise NpyError(f"expected an integer, file holds '{kind}{size}'", "DTypeMismatch")


def _floats(kind, size, body) -> np.ndarray:
    if kind == "f" and size in (2, 4, 8):
        return np.frombuffer(body, dtype=f"<f{size}").astype(np.float64)
    raise NpyError(f"expected a float, file holds '{kind}{size}'", "DTypeMismatch")


def _bits(kind, size, body, want) -> np.ndarray:
    if kind in "Vui" and size == want:
        return _uint_bits(body, size)
    raise NpyError(f"expected {want}-byte raw bits, file holds '{kind}{size}'", "DTypeMismatch")


def read(data: bytes, dtype: int, name: str = "") -> Tensor:
    """Decode an .npy file as elements of TOSA type `dtype` (NpyArray::to_tensor_data)."""
    kind, size, shape, body = parse(data)
    if dtype == L.DT_BOOL:
        vals = (_ints(kind, size, body) != 0).astype(np.uint8)
    elif dtype in (L.DT_INT4, L.DT_INT8):
        vals = _ints(kind, size, body).astype(np.int8)
    elif dtype == L.DT_INT16:
        vals = _ints(kind, size, body).astype(np.int16)
    elif dtype == L.DT_INT32:
        vals = _ints(kind, size, body).astype(np.int32)
    elif dtype in (L.DT_INT48, L.DT_INT64, L.DT_SHAPE):
        vals = _ints(kind, size, body)
    elif dtype == L.DT_FP32:
        vals = _floats(kind, size, body).astype(np.float32)
    elif dtype == L.DT_FP16:
        if kind == "f" and size == 2:
            vals = np.frombuffer(body, dtype="<f2").astype(np.float16)
        else:
            vals = _bits(kind, size, body, 2).astype(np.uint16).view(np.float16)
    elif dtype == L.DT_BF16:
        vals = _bits(kind, size, body, 2).astype(np.uint16)
    elif dtype in (L.DT_FP8E4M3, L.DT_FP8E5M2):
        vals = _bits(kind, size, body, 1).astype(np.uint8)
    else:
        raise NpyError(f"cannot decode dtype {dtype} tensors", "DTypeMismatch")
    return Tensor(name, list(shape), dtype, np.ascontiguousarray(vals.reshape(shape)))


def write(t: Tensor) -> bytes:
    """Serialize a tensor with the reference model's encoding for its dtype."""
    if t.dtype not in _WRITE:
        raise NpyError(f"cannot encode dtype {t.dtype} tensors", "DTypeMismatch")
    descr, store = _WRITE[t.dtype]
    body = np.ascontiguousarray(np.asarray(t.data).reshape(-1).astype(store)).tobytes()
    dims = [str(int(d)) for d in t.shape]
    shape = f"({dims[0]},)" if len(dims) == 1 else f"({', '.join(dims)})"
    header = f"{{'descr': '{descr}', 'fortran_order': False, 'shape': {shape}, }}"
    unpadded = len(MAGIC) + 4 + len(header) + 1
    header += " " * ((64 - unpadded % 64) % 64) + "\n"
    return MAGIC + bytes([1, 0]) + len(header).to_bytes(2, "little") + header.encode() + body
