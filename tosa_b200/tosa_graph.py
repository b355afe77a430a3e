"""Reader and writer for serialized TOSA graphs (`.tosa` flatbuffers).

The file format is the one the reference interpreter parses
(schema/tosa.fbs:702-768, parsed by src/ir.rs:592-885): a `TosaGraph` root
table holding regions, each holding basic blocks of operators and tensor
definitions. The main block is the first block of the first region
(src/ir.rs:886-888).

This is host tooling (tests, the synthetic graph generator, the bench driver).
The C++ runner in tosa_b200/csrc has its own reader for the product path.
The writer emits standard flatbuffers: little-endian, tables referenced by
32-bit forward offsets, vtables of 16-bit field offsets, vectors prefixed by
their 32-bit length, byte vectors 8-byte aligned (the schema's force_align).
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field

# schema/tosa.fbs:26-46
DTYPE_NAMES = [
    "UNKNOWN", "BOOL", "INT4", "INT8", "INT16", "INT32", "INT48", "FP32", "FP16",
    "BF16", "SHAPE", "FP8E4M3", "FP8E5M2", "FP6E2M3", "FP6E3M2", "FP4E2M1",
    "FP8UE8M0", "INT64", "MXINT8",
]
DTYPE = {n: i for i, n in enumerate(DTYPE_NAMES)}

# schema/tosa.fbs:88-201 (the Attribute union uses the same order)
OP_NAMES = [
    "UNKNOWN", "ARGMAX", "AVG_POOL2D", "CONV2D", "CONV3D", "DEPTHWISE_CONV2D", "FFT2D",
    "MATMUL", "MAX_POOL2D", "RFFT2D", "TRANSPOSE_CONV2D", "CLAMP", "ERF", "SIGMOID", "TANH",
    "ADD", "ARITHMETIC_RIGHT_SHIFT", "BITWISE_AND", "BITWISE_OR", "BITWISE_XOR", "INTDIV",
    "LOGICAL_AND", "LOGICAL_LEFT_SHIFT", "LOGICAL_RIGHT_SHIFT", "LOGICAL_OR", "LOGICAL_XOR",
    "MAXIMUM", "MINIMUM", "MUL", "POW", "SUB", "TABLE", "ABS", "BITWISE_NOT", "CEIL", "CLZ",
    "COS", "EXP", "FLOOR", "LOG", "LOGICAL_NOT", "NEGATE", "RECIPROCAL", "RSQRT", "SIN",
    "SELECT", "EQUAL", "GREATER", "GREATER_EQUAL", "REDUCE_ALL", "REDUCE_ANY", "REDUCE_MAX",
    "REDUCE_MIN", "REDUCE_PRODUCT", "REDUCE_SUM", "CONCAT", "PAD", "RESHAPE", "REVERSE",
    "SLICE", "TILE", "TRANSPOSE", "GATHER", "SCATTER", "RESIZE", "CAST", "RESCALE", "CONST",
    "IDENTITY", "CUSTOM", "COND_IF", "WHILE_LOOP", "VARIABLE", "VARIABLE_WRITE",
    "VARIABLE_READ", "CONST_SHAPE", "MATMUL_T_BLOCK_SCALED", "CAST_FROM_BLOCK_SCALED",
    "CAST_TO_BLOCK_SCALED", "DIM", "CONCAT_SHAPE", "ADD_SHAPE", "SUB_SHAPE", "MUL_SHAPE",
    "SLICE_SHAPE", "EXP2_SHAPE", "LOG2_CEIL_SHAPE", "LOG2_FLOOR_SHAPE", "MAX_SHAPE",
    "MIN_SHAPE", "MOD_SHAPE", "DIV_CEIL_SHAPE", "DIV_FLOOR_SHAPE", "ASSERT_EQUAL_SHAPE",
    "CONV2D_BLOCK_SCALED", "MAX_POOL2D_ADAPTIVE", "AVG_POOL2D_ADAPTIVE",
    "RESHAPE_BLOCK_SCALED", "ROW_GATHER_BLOCK_SCALED", "ROW_GATHER", "MATMUL_T", "ARGMIN",
]
OP = {n: i for i, n in enumerate(OP_NAMES)}

ROUNDING = {"UNKNOWN": 0, "SINGLE_ROUND": 1, "INEXACT_ROUND": 2, "DOUBLE_ROUND": 3}
NAN_MODE = {"UNKNOWN": 0, "PROPAGATE": 1, "IGNORE": 2}

# Attribute table layouts: (field name, kind) in schema field order. Kinds:
# "i32v" [int32], "u8v" [ubyte], "bool", "u32" (enum), "i32", "str".
ATTR_FIELDS = {
    "AVG_POOL2D": [("kernel", "i32v"), ("stride", "i32v"), ("pad", "i32v"), ("acc_type", "u32")],
    "CONV2D": [("pad", "i32v"), ("stride", "i32v"), ("dilation", "i32v"), ("local_bound", "bool"),
               ("acc_type", "u32")],
    "CONV3D": [("pad", "i32v"), ("stride", "i32v"), ("dilation", "i32v"), ("local_bound", "bool"),
               ("acc_type", "u32")],
    "DEPTHWISE_CONV2D": [("pad", "i32v"), ("stride", "i32v"), ("dilation", "i32v"),
                         ("local_bound", "bool"), ("acc_type", "u32")],
    "TRANSPOSE_CONV2D": [("out_pad", "i32v"), ("stride", "i32v"), ("local_bound", "bool"),
                         ("acc_type", "u32")],
    "MAX_POOL2D": [("kernel", "i32v"), ("stride", "i32v"), ("pad", "i32v"), ("nan_mode", "u32")],
    "CLAMP": [("min_val", "u8v"), ("max_val", "u8v"), ("nan_mode", "u32")],
    "RESCALE": [("scale32", "bool"), ("rounding_mode", "u32"), ("per_channel", "bool"),
                ("input_unsigned", "bool"), ("output_unsigned", "bool")],
    "ARGMAX": [("axis", "i32"), ("nan_mode", "u32")],
    "MAXIMUM": [("nan_mode", "u32")],
    "MINIMUM": [("nan_mode", "u32")],
    "CONCAT": [("axis", "i32")],
    "TRANSPOSE": [("perms", "i32v")],
    "CAST": [("input_unsigned", "bool")],
}


class TosaFormatError(ValueError):
    """Malformed flatbuffer (the reference's Error::Deserialize)."""


@dataclass
class TensorDef:
    name: str
    shape: list
    dtype: int
    data: bytes | None = None
    variable: bool = False
    # write the data outside the flatbuffer, at an offset from the start of the file
    # (TosaTensor.offset / .size, schema/tosa.fbs:711-716); a read sets it when it found them
    external: bool = False


@dataclass
class Operator:
    op: int
    inputs: list
    outputs: list
    attr: dict = field(default_factory=dict)
    attr_type: int = 0

    @property
    def name(self) -> str:
        return OP_NAMES[self.op] if 0 <= self.op < len(OP_NAMES) else "UNKNOWN"


@dataclass
class Block:
    name: str
    operators: list
    tensors: list
    inputs: list
    outputs: list

    def tensor(self, name):
        for t in self.tensors:
            if t.name == name:
                return t
        return None


@dataclass
class Graph:
    regions: list  # list of (name, [Block])
    version: tuple = (1, 0, 0, False)

    @property
    def main_block(self) -> Block:
        if not self.regions or not self.regions[0][1]:
            raise TosaFormatError("no main block found")
        return self.regions[0][1][0]


# ---------------------------------------------------------------------------
# Reader
# ---------------------------------------------------------------------------


class _Buf:
    def __init__(self, data: bytes):
        self.d = memoryview(bytes(data))
        self.n = len(data)

    def need(self, pos, size):
        if pos < 0 or size < 0 or pos + size > self.n:
            raise TosaFormatError(f"offset {pos}+{size} outside buffer of {self.n} bytes")

    def u8(self, p):
        self.need(p, 1)
        return self.d[p]

    def u16(self, p):
        self.need(p, 2)
        return struct.unpack_from("<H", self.d, p)[0]

    def i32(self, p):
        self.need(p, 4)
        return struct.unpack_from("<i", self.d, p)[0]

    def u32(self, p):
        self.need(p, 4)
        return struct.unpack_from("<I", self.d, p)[0]

    def u64(self, p):
        self.need(p, 8)
        return struct.unpack_from("<Q", self.d, p)[0]


class _Table:
    def __init__(self, buf: _Buf, pos: int):
        self.b = buf
        self.pos = pos
        vt = pos - buf.i32(pos)
        self.vt = vt
        self.vt_size = buf.u16(vt)
        if self.vt_size < 4 or self.vt_size % 2:
            raise TosaFormatError("bad vtable")
        buf.need(vt, self.vt_size)

    def off(self, fid):
        o = 4 + 2 * fid
        if o >= self.vt_size:
            return 0
        return self.b.u16(self.vt + o)

    def scalar(self, fid, kind, default=0):
        o = self.off(fid)
        if not o:
            return default
        p = self.pos + o
        return {"u8": self.b.u8, "u32": self.b.u32, "i32": self.b.i32, "u64": self.b.u64}[kind](p)

    def _ref(self, fid):
        o = self.off(fid)
        if not o:
            return None
        p = self.pos + o
        return p + self.b.u32(p)

    def table(self, fid):
        p = self._ref(fid)
        return None if p is None else _Table(self.b, p)

    def string(self, fid):
        p = self._ref(fid)
        if p is None:
            return None
        n = self.b.u32(p)
        self.b.need(p + 4, n)
        return bytes(self.b.d[p + 4:p + 4 + n]).decode("utf-8", errors="replace")

    def _vec(self, fid):
        p = self._ref(fid)
        if p is None:
            return None, 0
        return p + 4, self.b.u32(p)

    def bytes_vec(self, fid):
        p, n = self._vec(fid)
        if p is None:
            return None
        self.b.need(p, n)
        return bytes(self.b.d[p:p + n])

    def i32_vec(self, fid):
        p, n = self._vec(fid)
        if p is None:
            return []
        self.b.need(p, 4 * n)
        return list(struct.unpack_from(f"<{n}i", self.b.d, p))

    def table_vec(self, fid):
        p, n = self._vec(fid)
        if p is None:
            return []
        self.b.need(p, 4 * n)
        return [_Table(self.b, p + 4 * i + self.b.u32(p + 4 * i)) for i in range(n)]

    def string_vec(self, fid):
        p, n = self._vec(fid)
        if p is None:
            return []
        out = []
        for i in range(n):
            q = p + 4 * i
            s = q + self.b.u32(q)
            ln = self.b.u32(s)
            self.b.need(s + 4, ln)
            out.append(bytes(self.b.d[s + 4:s + 4 + ln]).decode("utf-8", errors="replace"))
        return out


def _parse_attr(opname: str, t: _Table | None) -> dict:
    if t is None:
        return {}
    fields = ATTR_FIELDS.get(opname)
    if not fields:
        return {}
    out = {}
    for fid, (name, kind) in enumerate(fields):
        if kind == "i32v":
            out[name] = t.i32_vec(fid)
        elif kind == "u8v":
            out[name] = t.bytes_vec(fid) or b""
        elif kind == "bool":
            out[name] = bool(t.scalar(fid, "u8"))
        elif kind == "u32":
            out[name] = t.scalar(fid, "u32")
        elif kind == "i32":
            out[name] = t.scalar(fid, "i32")
    return out


def read_graph(data: bytes) -> Graph:
    """Parse a `.tosa` flatbuffer (src/ir.rs:592-614)."""
    if len(data) < 8:
        raise TosaFormatError("buffer too small")
    b = _Buf(data)
    root = _Table(b, b.u32(0))
    regions = []
    for rt in root.table_vec(1):
        blocks = []
        for bt in rt.table_vec(1):
            tensors = []
            for tt in bt.table_vec(2):
                tdata = tt.bytes_vec(3)
                ext = False
                off = tt.scalar(7, "u64")
                if tdata is None and off > 1:
                    # data outside the flatbuffer: `size` bytes at `offset` from the start of the file
                    size = tt.scalar(8, "u64")
                    b.need(off, size)
                    tdata = bytes(data[off:off + size])
                    ext = True
                tensors.append(TensorDef(
                    name=tt.string(0) or "",
                    shape=tt.i32_vec(1),
                    dtype=tt.scalar(2, "u32"),
                    data=tdata,
                    variable=bool(tt.scalar(4, "u8")),
                    external=ext,
                ))
            for st in bt.table_vec(5):  # shapes: SHAPE tensors of rank `rank`
                tensors.append(TensorDef(name=st.string(0) or "", shape=[st.scalar(1, "u32")],
                                         dtype=DTYPE["SHAPE"], data=st.bytes_vec(2)))
            ops = []
            for ot in bt.table_vec(1):
                opc = ot.scalar(0, "u32")
                opname = OP_NAMES[opc] if opc < len(OP_NAMES) else "UNKNOWN"
                atype = ot.scalar(1, "u8")
                ops.append(Operator(op=opc, inputs=ot.string_vec(3), outputs=ot.string_vec(4),
                                    attr=_parse_attr(opname, ot.table(2)) if atype else {},
                                    attr_type=atype))
            blocks.append(Block(name=bt.string(0) or "", operators=ops, tensors=tensors,
                                inputs=bt.string_vec(3), outputs=bt.string_vec(4)))
        regions.append((rt.string(0) or "", blocks))
    return Graph(regions=regions)


# ---------------------------------------------------------------------------
# Writer
# ---------------------------------------------------------------------------


class _Builder:
    """Minimal back-to-front flatbuffer builder (standard wire format).

    The buffer grows at the front; pieces are kept in a list (last piece =
    frontmost) and joined once at the end, so building is linear in size.
    Offsets are measured from the end, as in the flatbuffers implementations."""

    def __init__(self):
        self.chunks: list = []
        self.size = 0
        self.minalign = 1

    def off(self):
        return self.size

    def _front(self, data: bytes):
        self.chunks.append(data)
        self.size += len(data)

    def pad(self, n):
        if n:
            self._front(b"\x00" * n)

    def prep(self, size, additional):
        if size > self.minalign:
            self.minalign = size
        align = (-(self.size + additional)) % size
        self.pad(align)

    def put(self, fmt, v):
        self._front(struct.pack("<" + fmt, v))

    def add_scalar(self, fmt, v):
        sz = struct.calcsize(fmt)
        self.prep(sz, 0)
        self.put(fmt, v)
        return self.off()

    def add_uoffset(self, target):
        self.prep(4, 0)
        rel = self.off() + 4 - target
        self.put("I", rel)
        return self.off()

    def create_bytes(self, data: bytes, align=8):
        self.prep(max(4, align), len(data))
        self.prep(4, len(data))
        self._front(bytes(data))
        self.put("I", len(data))
        return self.off()

    def create_string(self, s: str):
        data = s.encode()
        self.prep(4, len(data) + 1)
        self._front(data + b"\x00")
        self.put("I", len(data))
        return self.off()

    def create_i32_vec(self, vals):
        self.prep(4, 4 * len(vals))
        self._front(struct.pack(f"<{len(vals)}i", *[int(v) for v in vals]))
        self.put("I", len(vals))
        return self.off()

    def create_offset_vec(self, offs):
        self.prep(4, 4 * len(offs))
        for o in reversed(offs):
            self.add_uoffset(o)
        self.prep(4, 0)
        self.put("I", len(offs))
        return self.off()

    def table(self, fields):
        """fields: list indexed by field id of None or (kind, value). Scalars
        are written inline; "ref" values are offsets returned by create_*."""
        # Write fields largest first for alignment, recording their offsets.
        sizes = {"u8": 1, "bool": 1, "u16": 2, "u32": 4, "i32": 4, "u64": 8, "ref": 4}
        order = sorted([i for i, f in enumerate(fields) if f is not None],
                       key=lambda i: -sizes[fields[i][0]])
        start = self.off()
        pos = {}
        for i in order:
            kind, v = fields[i]
            if kind == "ref":
                pos[i] = self.add_uoffset(v)
            elif kind in ("u8", "bool"):
                pos[i] = self.add_scalar("B", int(v))
            elif kind == "u32":
                pos[i] = self.add_scalar("I", int(v))
            elif kind == "i32":
                pos[i] = self.add_scalar("i", int(v))
            elif kind == "u64":
                pos[i] = self.add_scalar("Q", int(v))
        # soffset to the vtable, which is written immediately in front of the table
        self.prep(4, 0)
        table_off = self.off() + 4
        nf = len(fields)
        while nf and fields[nf - 1] is None:
            nf -= 1
        vt = [0] * nf
        for i, p in pos.items():
            vt[i] = table_off - p
        table_size = table_off - start
        vbytes = struct.pack(f"<HH{nf}H", 4 + 2 * nf, table_size, *vt)
        # vtable position = table position - soffset (the vtable precedes the table)
        self.put("i", len(vbytes))
        self._front(vbytes)
        return table_off

    def finish(self, root, ident=b"TOSA"):
        self.prep(max(self.minalign, 8), 8)
        self._front(ident)
        self.add_uoffset(root)
        return b"".join(reversed(self.chunks))


def _attr_fields(opname, attr, b: _Builder):
    spec = ATTR_FIELDS.get(opname, [])
    fields = []
    for name, kind in spec:
        v = attr.get(name)
        if v is None:
            fields.append(None)
        elif kind == "i32v":
            fields.append(("ref", b.create_i32_vec(v)))
        elif kind == "u8v":
            fields.append(("ref", b.create_bytes(bytes(v))))
        elif kind == "bool":
            fields.append(("bool", bool(v)))
        elif kind == "u32":
            fields.append(("u32", int(v)))
        elif kind == "i32":
            fields.append(("i32", int(v)))
    return fields


def write_graph(g: Graph) -> bytes:
    """Serialize a Graph to `.tosa` bytes. Tensors marked `external` keep their data after
    the flatbuffer, 16-byte aligned, addressed by TosaTensor.offset / .size (the layout the
    schema defines for models above 2 GB)."""
    ext = [t for _, blocks in g.regions for blk in blocks for t in blk.tensors
           if t.external and t.data is not None and t.dtype != DTYPE["SHAPE"]]
    if not ext:
        return _write_graph(g, {})
    # the flatbuffer's size does not depend on the offset values (fixed-size scalars), so a
    # first pass with placeholders gives the position of the appended data
    head = len(_write_graph(g, {id(t): (2, len(t.data)) for t in ext}))
    offs, pos = {}, (head + 15) // 16 * 16
    for t in ext:
        offs[id(t)] = (pos, len(t.data))
        pos = (pos + len(t.data) + 15) // 16 * 16
    out = bytearray(_write_graph(g, offs))
    assert len(out) == head
    for t in ext:
        p, n = offs[id(t)]
        out.extend(b"\0" * (p - len(out)))
        out.extend(t.data)
    return bytes(out)


def _write_graph(g: Graph, external: dict) -> bytes:
    b = _Builder()
    region_offs = []
    for rname, blocks in g.regions:
        block_offs = []
        for blk in blocks:
            op_offs = []
            for op in blk.operators:
                attr_off = b.table(_attr_fields(op.name, op.attr, b))
                ins = b.create_offset_vec([b.create_string(s) for s in op.inputs])
                outs = b.create_offset_vec([b.create_string(s) for s in op.outputs])
                atype = op.attr_type or (op.op if attr_off is not None else 0)
                op_offs.append(b.table([
                    ("u32", op.op),
                    ("u8", atype) if attr_off is not None else None,
                    ("ref", attr_off) if attr_off is not None else None,
                    ("ref", ins), ("ref", outs),
                ]))
            ten_offs = []
            for t in blk.tensors:
                if t.dtype == DTYPE["SHAPE"]:
                    continue
                name = b.create_string(t.name)
                shape = b.create_i32_vec(t.shape)
                where = external.get(id(t))
                data = b.create_bytes(t.data) if t.data is not None and where is None else None
                ten_offs.append(b.table([
                    ("ref", name), ("ref", shape), ("u32", t.dtype),
                    ("ref", data) if data is not None else None,
                    ("bool", t.variable) if t.variable else None,
                    None, None,
                    ("u64", where[0]) if where else None,
                    ("u64", where[1]) if where else None,
                ]))
            shape_offs = []
            for t in blk.tensors:
                if t.dtype != DTYPE["SHAPE"]:
                    continue
                name = b.create_string(t.name)
                data = b.create_bytes(t.data) if t.data is not None else None
                shape_offs.append(b.table([("ref", name), ("u32", t.shape[0] if t.shape else 0),
                                           ("ref", data) if data is not None else None]))
            name = b.create_string(blk.name)
            opv = b.create_offset_vec(op_offs)
            tv = b.create_offset_vec(ten_offs)
            iv = b.create_offset_vec([b.create_string(s) for s in blk.inputs])
            ov = b.create_offset_vec([b.create_string(s) for s in blk.outputs])
            sv = b.create_offset_vec(shape_offs) if shape_offs else None
            block_offs.append(b.table([("ref", name), ("ref", opv), ("ref", tv), ("ref", iv),
                                       ("ref", ov), ("ref", sv) if sv is not None else None]))
        rn = b.create_string(rname)
        bv = b.create_offset_vec(block_offs)
        region_offs.append(b.table([("ref", rn), ("ref", bv)]))
    rv = b.create_offset_vec(region_offs)
    maj, mnr, pat, draft = g.version
    ver = b.table([("i32", maj), ("i32", mnr), ("i32", pat), ("bool", draft)])
    root = b.table([("ref", ver), ("ref", rv)])
    return b.finish(root)
