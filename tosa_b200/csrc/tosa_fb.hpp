// Reader for serialized TOSA graphs (`.tosa` flatbuffers, schema/tosa.fbs).
//
// Produces the same in-memory graph the reference builds in
// Graph::from_flatbuffer (src/ir.rs:592-614) and parse_block (:616-680):
// regions -> blocks -> {operators, tensors (+ SHAPE values from `shapes`),
// inputs, outputs}, with the attribute tables of the operators this backend
// runs. Every offset is bounds-checked; a malformed buffer yields
// TB_ERR_DESERIALIZE (the reference's Error::Deserialize).
#pragma once

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace tb {
namespace fb {

// Serialized Op enum values (schema/tosa.fbs:88-201) used by the runner.
enum Op : int {
    OP_AVG_POOL2D = 2, OP_CONV2D = 3, OP_DEPTHWISE_CONV2D = 5, OP_MATMUL = 7, OP_MAX_POOL2D = 8,
    OP_CLAMP = 11, OP_ADD = 15, OP_RESHAPE = 57, OP_TRANSPOSE = 61, OP_RESCALE = 66, OP_CONST = 67,
    OP_IDENTITY = 68, OP_CONST_SHAPE = 75, OP_MATMUL_T = 100,
    OP_TRANSPOSE_CONV2D = 10, OP_CONV3D = 4,
};

// Attribute union members (schema/tosa.fbs: the Attribute union repeats the Op order).
struct Attr {
    int type = 0;                       // union type tag; 0 = none
    std::vector<int32_t> pad, stride, dilation, kernel, perms;
    int32_t acc_type = 0;
    bool local_bound = false;
    std::vector<uint8_t> min_val, max_val;
    int32_t nan_mode = 0;
    bool scale32 = false, per_channel = false, input_unsigned = false, output_unsigned = false;
    int32_t rounding_mode = 0;
};

struct TensorDef {
    std::string name;
    std::vector<int32_t> shape;
    int32_t dtype = 0;
    bool has_data = false;
    std::vector<uint8_t> data;
    bool variable = false;
};

struct Operator {
    int32_t op = 0;
    Attr attr;
    std::vector<std::string> inputs, outputs;
};

struct Block {
    std::string name;
    std::vector<Operator> operators;
    std::vector<TensorDef> tensors;
    std::vector<std::string> inputs, outputs;
};

struct Region {
    std::string name;
    std::vector<Block> blocks;
};

struct Graph {
    std::vector<Region> regions;
    const Block* main_block() const {
        if (regions.empty() || regions[0].blocks.empty()) return nullptr;
        return &regions[0].blocks[0];
    }
};

class Reader {
  public:
    Reader(const uint8_t* d, size_t n) : d_(d), n_(n) {}
    bool ok() const { return ok_; }
    const std::string& error() const { return err_; }

    struct Table {
        size_t pos = 0, vt = 0;
        uint16_t vt_size = 0;
        bool valid = false;
    };

    Table root() {
        Table t;
        if (n_ < 8) { bad("buffer too small"); return t; }
        return table_at(u32(0));
    }

    Table table_at(size_t pos) {
        Table t;
        if (!need(pos, 4)) return t;
        const int64_t vt = static_cast<int64_t>(pos) - i32(pos);
        if (vt < 0 || !need(static_cast<size_t>(vt), 4)) { bad("vtable outside the buffer"); return t; }
        t.pos = pos;
        t.vt = static_cast<size_t>(vt);
        t.vt_size = u16(t.vt);
        if (t.vt_size < 4 || (t.vt_size & 1) || !need(t.vt, t.vt_size)) { bad("malformed vtable"); return t; }
        t.valid = true;
        return t;
    }

    uint16_t field(const Table& t, int id) {
        if (!t.valid) return 0;
        const size_t o = 4 + 2 * static_cast<size_t>(id);
        if (o >= t.vt_size) return 0;
        return u16(t.vt + o);
    }

    uint32_t scalar_u32(const Table& t, int id, uint32_t def = 0) {
        const uint16_t o = field(t, id);
        return o ? u32(t.pos + o) : def;
    }
    int32_t scalar_i32(const Table& t, int id, int32_t def = 0) {
        const uint16_t o = field(t, id);
        return o ? i32(t.pos + o) : def;
    }
    uint8_t scalar_u8(const Table& t, int id, uint8_t def = 0) {
        const uint16_t o = field(t, id);
        return o ? u8(t.pos + o) : def;
    }
    uint64_t scalar_u64(const Table& t, int id, uint64_t def = 0) {
        const uint16_t o = field(t, id);
        if (!o || !need(t.pos + o, 8)) return def;
        uint64_t v;
        std::memcpy(&v, d_ + t.pos + o, 8);
        return v;
    }
    // `size` bytes at file offset `off` (tensor data stored outside the flatbuffer).
    std::vector<uint8_t> span(uint64_t off, uint64_t size) {
        if (off > n_ || size > n_ - off) { bad("external tensor data outside the file"); return {}; }
        return std::vector<uint8_t>(d_ + off, d_ + off + size);
    }

    // Position of the referenced object (table, string, vector) or 0 if absent.
    size_t ref(const Table& t, int id) {
        const uint16_t o = field(t, id);
        if (!o) return 0;
        const size_t p = t.pos + o;
        if (!need(p, 4)) return 0;
        const size_t q = p + u32(p);
        return need(q, 4) ? q : 0;
    }

    Table table(const Table& t, int id) {
        const size_t p = ref(t, id);
        return p ? table_at(p) : Table{};
    }

    std::string string(const Table& t, int id) {
        const size_t p = ref(t, id);
        if (!p) return std::string();
        return string_at(p);
    }

    std::vector<uint8_t> bytes(const Table& t, int id, bool* present = nullptr) {
        const size_t p = ref(t, id);
        if (present) *present = p != 0;
        if (!p) return {};
        const uint32_t n = u32(p);
        if (!need(p + 4, n)) return {};
        return std::vector<uint8_t>(d_ + p + 4, d_ + p + 4 + n);
    }

    std::vector<int32_t> i32_vec(const Table& t, int id) {
        const size_t p = ref(t, id);
        if (!p) return {};
        const uint32_t n = u32(p);
        if (!need(p + 4, static_cast<size_t>(n) * 4)) return {};
        std::vector<int32_t> v(n);
        for (uint32_t i = 0; i < n; ++i) v[i] = i32(p + 4 + 4 * static_cast<size_t>(i));
        return v;
    }

    std::vector<Table> table_vec(const Table& t, int id) {
        const size_t p = ref(t, id);
        if (!p) return {};
        const uint32_t n = u32(p);
        if (!need(p + 4, static_cast<size_t>(n) * 4)) return {};
        std::vector<Table> v;
        v.reserve(n);
        for (uint32_t i = 0; i < n && ok_; ++i) {
            const size_t q = p + 4 + 4 * static_cast<size_t>(i);
            v.push_back(table_at(q + u32(q)));
        }
        return v;
    }

    std::vector<std::string> string_vec(const Table& t, int id) {
        const size_t p = ref(t, id);
        if (!p) return {};
        const uint32_t n = u32(p);
        if (!need(p + 4, static_cast<size_t>(n) * 4)) return {};
        std::vector<std::string> v;
        v.reserve(n);
        for (uint32_t i = 0; i < n && ok_; ++i) {
            const size_t q = p + 4 + 4 * static_cast<size_t>(i);
            v.push_back(string_at(q + u32(q)));
        }
        return v;
    }

  private:
    bool need(size_t pos, size_t size) {
        if (!ok_) return false;
        if (pos > n_ || size > n_ - pos) { bad("offset outside the buffer"); return false; }
        return true;
    }
    void bad(const char* why) {
        if (ok_) err_ = why;
        ok_ = false;
    }
    uint8_t u8(size_t p) { return need(p, 1) ? d_[p] : 0; }
    uint16_t u16(size_t p) {
        if (!need(p, 2)) return 0;
        return static_cast<uint16_t>(d_[p] | (d_[p + 1] << 8));
    }
    uint32_t u32(size_t p) {
        if (!need(p, 4)) return 0;
        uint32_t v;
        std::memcpy(&v, d_ + p, 4);
        return v;
    }
    int32_t i32(size_t p) { return static_cast<int32_t>(u32(p)); }
    std::string string_at(size_t p) {
        const uint32_t n = u32(p);
        if (!need(p + 4, n)) return std::string();
        return std::string(reinterpret_cast<const char*>(d_ + p + 4), n);
    }

    const uint8_t* d_;
    size_t n_;
    bool ok_ = true;
    std::string err_;
};

// Attribute tables, fields in schema order (schema/tosa.fbs:313-420), chosen by the union tag.
inline void parse_attr(Reader& r, int tag, const Reader::Table& t, Attr* a) {
    switch (tag) {
    case OP_AVG_POOL2D:
        a->kernel = r.i32_vec(t, 0); a->stride = r.i32_vec(t, 1); a->pad = r.i32_vec(t, 2);
        a->acc_type = static_cast<int32_t>(r.scalar_u32(t, 3));
        break;
    case OP_CONV2D:
    case OP_CONV3D:
    case OP_DEPTHWISE_CONV2D:
        a->pad = r.i32_vec(t, 0); a->stride = r.i32_vec(t, 1); a->dilation = r.i32_vec(t, 2);
        a->local_bound = r.scalar_u8(t, 3) != 0; a->acc_type = static_cast<int32_t>(r.scalar_u32(t, 4));
        break;
    case OP_TRANSPOSE_CONV2D:  // out_pad, stride, local_bound, acc_type
        a->pad = r.i32_vec(t, 0); a->stride = r.i32_vec(t, 1);
        a->local_bound = r.scalar_u8(t, 2) != 0; a->acc_type = static_cast<int32_t>(r.scalar_u32(t, 3));
        break;
    case OP_MAX_POOL2D:
        a->kernel = r.i32_vec(t, 0); a->stride = r.i32_vec(t, 1); a->pad = r.i32_vec(t, 2);
        a->nan_mode = static_cast<int32_t>(r.scalar_u32(t, 3));
        break;
    case OP_CLAMP:
        a->min_val = r.bytes(t, 0); a->max_val = r.bytes(t, 1);
        a->nan_mode = static_cast<int32_t>(r.scalar_u32(t, 2));
        break;
    case OP_RESCALE:
        a->scale32 = r.scalar_u8(t, 0) != 0; a->rounding_mode = static_cast<int32_t>(r.scalar_u32(t, 1));
        a->per_channel = r.scalar_u8(t, 2) != 0; a->input_unsigned = r.scalar_u8(t, 3) != 0;
        a->output_unsigned = r.scalar_u8(t, 4) != 0;
        break;
    case OP_TRANSPOSE:
        a->perms = r.i32_vec(t, 0);
        break;
    default: break;
    }
}

// TosaGraph {version:0, regions:1}; TosaRegion {name:0, blocks:1};
// TosaBasicBlock {name:0, operators:1, tensors:2, inputs:3, outputs:4, shapes:5};
// TosaTensor {name:0, shape:1, type:2, data:3, variable:4, is_unranked:5, variable_name:6, offset:7,
//             size:8}; TosaShape {name:0, rank:1, data:2};
// A tensor without inline data whose offset is above 1 keeps `size` bytes at that offset from the
// start of the file (models above 2 GB; schema/tosa.fbs:711-716). The reference reads only the
// inline data (src/ir.rs parses no offset): such constants fail there and load here.
// TosaOperator {op:0, attribute_type:1, attribute:2, inputs:3, outputs:4}.
inline bool parse_graph(const uint8_t* data, size_t len, Graph* g, std::string* err) {
    Reader r(data, len);
    Reader::Table root = r.root();
    for (const auto& rt : r.table_vec(root, 1)) {
        Region reg;
        reg.name = r.string(rt, 0);
        for (const auto& bt : r.table_vec(rt, 1)) {
            Block b;
            b.name = r.string(bt, 0);
            for (const auto& tt : r.table_vec(bt, 2)) {
                TensorDef td;
                td.name = r.string(tt, 0);
                td.shape = r.i32_vec(tt, 1);
                td.dtype = static_cast<int32_t>(r.scalar_u32(tt, 2));
                td.data = r.bytes(tt, 3, &td.has_data);
                td.variable = r.scalar_u8(tt, 4) != 0;
                const uint64_t off = r.scalar_u64(tt, 7);
                if (!td.has_data && off > 1) {
                    td.data = r.span(off, r.scalar_u64(tt, 8));
                    td.has_data = true;
                }
                b.tensors.push_back(std::move(td));
            }
            for (const auto& st : r.table_vec(bt, 5)) {
                TensorDef td;
                td.name = r.string(st, 0);
                td.shape = {static_cast<int32_t>(r.scalar_u32(st, 1))};
                td.dtype = 10;  // SHAPE
                td.data = r.bytes(st, 2, &td.has_data);
                b.tensors.push_back(std::move(td));
            }
            for (const auto& ot : r.table_vec(bt, 1)) {
                Operator op;
                op.op = static_cast<int32_t>(r.scalar_u32(ot, 0));
                op.attr.type = r.scalar_u8(ot, 1);
                if (op.attr.type) {
                    Reader::Table at = r.table(ot, 2);
                    // The union tag repeats the Op enum order, so the tag names the op whose
                    // attribute table follows; an op reads its attribute only when the tags agree.
                    if (at.valid) parse_attr(r, op.attr.type, at, &op.attr);
                }
                op.inputs = r.string_vec(ot, 3);
                op.outputs = r.string_vec(ot, 4);
                b.operators.push_back(std::move(op));
            }
            b.inputs = r.string_vec(bt, 3);
            b.outputs = r.string_vec(bt, 4);
            reg.blocks.push_back(std::move(b));
        }
        g->regions.push_back(std::move(reg));
    }
    if (!r.ok()) {
        *err = r.error();
        return false;
    }
    return true;
}

}  // namespace fb
}  // namespace tb
