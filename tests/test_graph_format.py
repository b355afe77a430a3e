"""The `.tosa` flatbuffer readers and writer, on CPU.

* The C++ reader the graph runner uses (tosa_b200/csrc/tosa_fb.hpp) parses
  every fixture graph the reference ships to the same structure as the Python
  reader (operators with their attribute fields, tensors with shapes, dtypes
  and data, block inputs/outputs).
* The Python writer round-trips every fixture graph and the synthetic
  benchmark graphs.
* Truncated buffers are rejected by the C++ reader (Error::Deserialize).
"""

import os
import subprocess
import zipfile

import numpy as np
import pytest

from oracle import oracle as O
from tosa_b200 import graphs
from tosa_b200 import tosa_graph as TG

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
FAMILIES = ["conv2d", "depthwise_conv2d", "matmul", "rescale", "avg_pool2d", "max_pool2d", "clamp", "networks"]

HARNESS = r"""
#include <cstdio>
#include <fstream>
#include <iterator>
#include "tosa_fb.hpp"
using namespace tb::fb;
static void vec(const char* k, const std::vector<int32_t>& v) {
    std::printf(" %s=", k);
    for (size_t i = 0; i < v.size(); ++i) std::printf("%s%d", i ? "," : "", v[i]);
}
int main(int argc, char** argv) {
    for (int f = 1; f < argc; ++f) {
        std::ifstream in(argv[f], std::ios::binary);
        std::vector<uint8_t> buf((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
        Graph g;
        std::string err;
        if (!parse_graph(buf.data(), buf.size(), &g, &err)) { std::printf("ERROR %s\n", err.c_str()); continue; }
        for (const auto& r : g.regions) for (const auto& b : r.blocks) {
            std::printf("block %s in=%zu out=%zu\n", b.name.c_str(), b.inputs.size(), b.outputs.size());
            for (const auto& s : b.inputs) std::printf("input %s\n", s.c_str());
            for (const auto& s : b.outputs) std::printf("output %s\n", s.c_str());
            for (const auto& t : b.tensors) {
                std::printf("tensor %s dtype=%d data=%d:%zu", t.name.c_str(), t.dtype, (int)t.has_data, t.data.size());
                vec("shape", t.shape);
                std::printf("\n");
            }
            for (const auto& o : b.operators) {
                std::printf("op %d attr=%d", o.op, o.attr.type);
                for (const auto& s : o.inputs) std::printf(" <%s", s.c_str());
                for (const auto& s : o.outputs) std::printf(" >%s", s.c_str());
                const Attr& a = o.attr;
                vec("pad", a.pad); vec("stride", a.stride); vec("dilation", a.dilation); vec("kernel", a.kernel);
                vec("perms", a.perms);
                std::printf(" acc=%d nan=%d round=%d flags=%d%d%d%d min=%zu max=%zu\n", a.acc_type, a.nan_mode,
                            a.rounding_mode, (int)a.scale32, (int)a.per_channel, (int)a.input_unsigned,
                            (int)a.output_unsigned, a.min_val.size(), a.max_val.size());
            }
        }
    }
    return 0;
}
"""

ATTR_TAGS = {TG.OP[n] for n in ("AVG_POOL2D", "CONV2D", "DEPTHWISE_CONV2D", "MAX_POOL2D", "CLAMP", "RESCALE",
                                "TRANSPOSE")}


def _py_dump(data: bytes) -> str:
    g = TG.read_graph(data)
    out = []
    for _, blocks in g.regions:
        for b in blocks:
            out.append(f"block {b.name} in={len(b.inputs)} out={len(b.outputs)}")
            out += [f"input {s}" for s in b.inputs]
            out += [f"output {s}" for s in b.outputs]
            for t in b.tensors:
                n = len(t.data) if t.data is not None else 0
                out.append(f"tensor {t.name} dtype={t.dtype} data={int(t.data is not None)}:{n} shape="
                           + ",".join(str(v) for v in t.shape))
            for o in b.operators:
                # the C++ reader decodes the attribute tables of the runner's operators
                a = o.attr if o.attr_type in ATTR_TAGS else {}
                s = f"op {o.op} attr={o.attr_type}"
                s += "".join(f" <{x}" for x in o.inputs) + "".join(f" >{x}" for x in o.outputs)
                for k in ("pad", "stride", "dilation", "kernel", "perms"):
                    s += f" {k}=" + ",".join(str(v) for v in a.get(k, []))
                flags = "".join(str(int(bool(a.get(k, False)))) for k in
                                ("scale32", "per_channel", "input_unsigned", "output_unsigned"))
                s += (f" acc={a.get('acc_type', 0)} nan={a.get('nan_mode', 0)} round={a.get('rounding_mode', 0)}"
                      f" flags={flags} min={len(a.get('min_val', b''))} max={len(a.get('max_val', b''))}")
                out.append(s)
    return "\n".join(out)


def _fixture_graphs():
    for fam in FAMILIES:
        z = zipfile.ZipFile(os.path.join(GOLDEN, f"{fam}.zip"))
        for n in sorted(z.namelist()):
            if n.endswith(".tosa"):
                yield n, z.read(n)


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    d = tmp_path_factory.mktemp("fb")
    src = d / "fbdump.cpp"
    src.write_text(HARNESS)
    exe = d / "fbdump"
    subprocess.check_call(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "tosa_b200", "csrc"), "-o", str(exe),
                           str(src)])
    return exe, d


def test_cpp_reader_matches_python_reader(harness):
    exe, d = harness
    files, expected = [], []
    for i, (name, data) in enumerate(_fixture_graphs()):
        p = d / f"g{i}.tosa"
        p.write_bytes(data)
        files.append(str(p))
        expected.append(_py_dump(data))
    got = subprocess.check_output([str(exe), *files]).decode()
    assert got.strip() == "\n".join(expected).strip()
    assert len(files) == 531


def test_cpp_reader_rejects_truncated_buffers(harness):
    exe, d = harness
    name, data = next(_fixture_graphs())
    paths = []
    for cut in (3, 16, len(data) // 3, len(data) - 9):
        p = d / f"cut{cut}.tosa"
        p.write_bytes(data[:cut])
        paths.append(str(p))
    out = subprocess.check_output([str(exe), *paths]).decode().splitlines()
    assert sum(line.startswith("ERROR") for line in out) == len(paths)


def test_writer_round_trips_fixture_graphs():
    for name, data in _fixture_graphs():
        g = TG.read_graph(data)
        again = TG.read_graph(TG.write_graph(g))
        assert _py_dump(TG.write_graph(g)) == _py_dump(TG.write_graph(again)), name
        assert [(t.name, t.shape, t.dtype, t.data) for t in g.main_block.tensors] == \
               [(t.name, t.shape, t.dtype, t.data) for t in again.main_block.tensors], name


def test_synthetic_graph_shapes():
    data, info = graphs.resnet50_int8(2)
    g = TG.read_graph(data)
    ops = [o.name for o in g.main_block.operators]
    assert ops.count("CONV2D") == 53 and ops.count("MATMUL") == 1 and ops.count("MAX_POOL2D") == 1
    assert ops.count("ADD") == 16
    assert info["ops_per_image"] == pytest.approx(8.178e9, rel=1e-3)
    data, info = graphs.mobilenetv2_int8(2)
    ops = [o.name for o in TG.read_graph(data).main_block.operators]
    assert ops.count("DEPTHWISE_CONV2D") == 17 and ops.count("CONV2D") == 2 + 2 * 17
    assert ops.count("ADD") == 10


def _externalize(data, min_bytes=64):
    """The same graph with every constant of more than `min_bytes` stored after the
    flatbuffer (TosaTensor.offset / .size)."""
    g = TG.read_graph(data)
    n = 0
    for t in g.main_block.tensors:
        if t.data is not None and len(t.data) > min_bytes and t.dtype != TG.DTYPE["SHAPE"]:
            t.external = True
            n += 1
    return TG.write_graph(g), n


def test_external_tensor_data_round_trip():
    """Constants stored outside the flatbuffer (schema/tosa.fbs:711-716, the form of
    models above 2 GB) read back to the same tensors, and the oracle computes the
    same outputs from either file."""
    from tosa_b200 import graphs
    data, _ = graphs.residual_block_int8(batch=2)
    ext, n = _externalize(data)
    assert n >= 5
    a, b = TG.read_graph(data).main_block, TG.read_graph(ext).main_block
    for ta, tb in zip(a.tensors, b.tensors):
        assert (ta.name, ta.shape, ta.dtype, ta.data) == (tb.name, tb.shape, tb.dtype, tb.data)
    assert sum(t.external for t in b.tensors) == n
    x = np.random.default_rng(4).integers(-128, 128, (2, 14, 14, 64)).astype(np.int64)
    outs = [O.run_block(TG.read_graph(d).main_block, {"x": O.T(3, [2, 14, 14, 64], x.reshape(-1))})
            for d in (data, ext)]
    for nm in outs[0]:
        assert np.array_equal(outs[0][nm].values, outs[1][nm].values)


def test_external_tensor_data_outside_the_file():
    from tosa_b200 import graphs
    data, _ = graphs.residual_block_int8(batch=2)
    ext, _ = _externalize(data)
    with pytest.raises(TG.TosaFormatError):  # the last constant's bytes cut off the end of the file
        TG.read_graph(ext[:-16])
