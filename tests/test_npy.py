"""tosa_b200.npy against the reference's .npy encodings (src/npy.rs): every TOSA
dtype round-trips, scalar and multi-dimensional shapes keep their shape, and
every .npy file the reference ships with its conformance and network cases
(written by the TOSA reference model) is read and written back byte for byte."""

import zipfile
import os

import numpy as np
import pytest

from tosa_b200 import _lib as L
from tosa_b200 import npy
from tosa_b200.interpreter import Tensor

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DESCR_DTYPE = {"|b1": L.DT_BOOL, "|i1": L.DT_INT8, "<i2": L.DT_INT16, "<i4": L.DT_INT32, "<i8": L.DT_INT48,
               "<f2": L.DT_FP16, "<f4": L.DT_FP32, "<V2": L.DT_BF16, "<V1": L.DT_FP8E4M3, "|u1": L.DT_FP8E5M2}


@pytest.mark.parametrize("dtype,vals", [
    (L.DT_BOOL, [1, 0, 1]), (L.DT_INT4, [-7, 0, 7]), (L.DT_INT8, [-128, 0, 127]),
    (L.DT_INT16, [-32768, 1, 32767]), (L.DT_INT32, [-2 ** 31, 2, 2 ** 31 - 1]),
    (L.DT_INT48, [-(1 << 47), 3, (1 << 47) - 1]), (L.DT_FP8E4M3, [0x7E, 1, 0x80]),
    (L.DT_FP8E5M2, [0x7C, 1, 0xFD]), (L.DT_FP16, [1.5, 1.5, 1.5]), (L.DT_BF16, [0xC010, 0xC010, 0xC010]),
    (L.DT_FP32, [1.0, -np.inf, -0.0]),
])
def test_round_trip_every_dtype(dtype, vals):
    t = Tensor.from_numpy("t", np.array(vals), dtype)
    back = npy.read(npy.write(t), dtype)
    assert back.shape == [3] and back.data.dtype == t.data.dtype
    assert np.array_equal(back.data.view(np.uint8), t.data.view(np.uint8))


def test_scalar_and_multi_dim_shapes():
    b = npy.read(npy.write(Tensor("s", [], L.DT_INT32, np.array(5, np.int32))), L.DT_INT32)
    assert b.shape == [] and int(b.data) == 5
    b = npy.read(npy.write(Tensor("m", [2, 3], L.DT_INT8, np.zeros((2, 3), np.int8))), L.DT_INT8)
    assert b.shape == [2, 3]


def test_header_is_numpy_readable_and_64_byte_aligned():
    t = Tensor.from_numpy("x", np.arange(12, dtype=np.int32).reshape(3, 4), L.DT_INT32)
    data = npy.write(t)
    hlen = int.from_bytes(data[8:10], "little")
    assert (10 + hlen) % 64 == 0 and data[10 + hlen - 1:10 + hlen] == b"\n"
    import io
    assert np.array_equal(np.load(io.BytesIO(data)), t.data)


def _raw(header: str, body: bytes) -> bytes:
    h = header.encode()
    return npy.MAGIC + b"\x01\x00" + len(h).to_bytes(2, "little") + h + body


@pytest.mark.parametrize("bad,why", [
    (b"NOTNPY" + b"\x00" * 10, "not an npy file"),
    (_raw("{'descr': '>i4', 'fortran_order': False, 'shape': (1,), }\n", b"\x00" * 4), "big-endian"),
    (_raw("{'descr': '<i4', 'fortran_order': True, 'shape': (1,), }\n", b"\x00" * 4), "fortran"),
    (_raw("{'descr': '<i4', 'fortran_order': False, 'shape': (4,), }\n", b"\x00" * 5), "expected 16 bytes"),
    (_raw("{'descr': [('a', '<i4')], 'fortran_order': False, 'shape': (1,), }\n", b"\x00" * 4), "structured"),
    (_raw("{'fortran_order': False, 'shape': (1,), }\n", b"\x00" * 4), "missing 'descr'"),
])
def test_malformed_files_rejected(bad, why):
    with pytest.raises(npy.NpyError, match=why):
        npy.parse(bad)


def test_dtype_mismatch():
    data = npy.write(Tensor.from_numpy("x", np.array([1.0, 2.0]), L.DT_FP32))
    with pytest.raises(npy.NpyError) as ei:
        npy.read(data, L.DT_INT8)
    assert ei.value.kind == "DTypeMismatch"


def test_reference_fixture_files_byte_identical():
    n = 0
    for fam in sorted(f for f in os.listdir(GOLDEN) if f.endswith(".zip")):
        with zipfile.ZipFile(os.path.join(GOLDEN, fam)) as z:
            for name in z.namelist():
                if not name.endswith(".npy"):
                    continue
                data = z.read(name)
                kind, size, shape, _ = npy.parse(data)
                dtype = DESCR_DTYPE[data[10:].split(b"'descr': '")[1][:3].decode()]
                assert npy.write(npy.read(data, dtype)) == data, f"{fam}:{name}"
                n += 1
    assert n > 1000  # every .npy member of the fixture archives
