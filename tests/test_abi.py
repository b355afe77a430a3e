"""The C ABI on CPU: the library builds, loads without a GPU, and exports every
entry point include/tosa_b200.h declares; the ctypes binding declares the
same set; no compute call is made here."""

import ctypes
import os
import re

import pytest

from tosa_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tosa_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"TB_API\s+[\w\s\*]+?\b(tb_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    from tosa_b200 import build
    build.build()
    return L.load()


def test_header_declares_the_entry_points():
    names = _declared()
    for required in ("tb_context_create", "tb_conv2d", "tb_depthwise_conv2d", "tb_matmul", "tb_rescale",
                     "tb_clamp", "tb_avg_pool2d", "tb_max_pool2d", "tb_synchronize", "tb_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_matches_header():
    assert {n for n, _, _ in L.SIGNATURES} == _declared()


def test_struct_layout_matches_the_c_compiler(tmp_path):
    """sizeof/offsetof of every descriptor as gcc lays it out from the header."""
    structs = {"tb_matmul_desc": L.MatmulDesc, "tb_conv2d_desc": L.Conv2dDesc,
               "tb_pool2d_desc": L.Pool2dDesc, "tb_rescale_attr": L.RescaleAttr}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    import subprocess
    subprocess.check_call(["gcc", "-std=c99", "-o", str(exe), str(src)])
    got = dict(line.split() for line in subprocess.check_output([str(exe)]).decode().splitlines())
    for cname, py in structs.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, f"{cname}.{fname}"


def test_last_error_is_empty_or_text(lib):
    msg = lib.tb_last_error()
    assert msg is None or isinstance(msg, bytes)


def test_no_device_reports_a_cuda_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    h = ctypes.c_void_p()
    status = lib.tb_context_create(0, ctypes.byref(h))
    assert status == 64  # TB_ERR_CUDA: there is no CPU fallback
    assert lib.tb_last_error()
