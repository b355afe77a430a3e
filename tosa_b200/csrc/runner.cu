// Graph runner: executes the main block of a serialized TOSA graph on the
// device, in the reference interpreter's operator order and with its hook
// events, its validation and its error kinds.
//
//   tb_graph_load  ~ Interpreter::from_flatbuffer (src/interpreter.rs:115-118)
//   tb_graph_run   ~ Interpreter::run + execute_block_inner (src/interpreter.rs:122-245)
//
// Design. A run is compiled once per set of bound input shapes: operator
// order (the reference's ready queue, computed once instead of rescanned per
// operator), shape/dtype inference with the reference's checks, device
// buffers for every materialised tensor, CONST tensors decoded and uploaded
// once, and one prepared plan per operator (contraction plans precompute their
// zero-point tables, RESCALE plans their packed constants). A compile error is
// recorded on the operator where the reference would raise it; the run then
// executes (and reports to hooks) every operator before it and returns that
// error. Fusion groups a contraction with the RESCALE (+ CLAMP) consuming it,
// and the residual chain RESCALE, RESCALE -> ADD -> RESCALE (+ CLAMP), into
// single kernels. With TB_GRAPH_CUDA_GRAPH the launch sequence is captured
// once and replayed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.hpp"
#include "tosa_fb.hpp"

using namespace tb;
using tb::fb::Attr;

namespace {

// Element size the reference reports (DType::element_size_bytes, src/ir.rs:55-64).
int ref_elem_bytes(int dt) {
    switch (dt) {
    case TB_DT_BOOL: case TB_DT_INT4: case TB_DT_INT8: case TB_DT_FP8E4M3: case TB_DT_FP8E5M2: return 1;
    case TB_DT_INT16: case TB_DT_FP16: case TB_DT_BF16: return 2;
    case TB_DT_INT32: case TB_DT_FP32: return 4;
    case TB_DT_INT48: case TB_DT_INT64: case TB_DT_SHAPE: return 8;
    default: return dt >= 13 && dt <= 18 ? 1 : 0;
    }
}

// Bytes per element on the device: INT4 is stored one per byte (sign-extended),
// INT48 as int64.
int dev_elem_bytes(int dt) { return ref_elem_bytes(dt); }

bool is_int_dt(int dt) {
    return dt == TB_DT_INT4 || dt == TB_DT_INT8 || dt == TB_DT_INT16 || dt == TB_DT_INT32 || dt == TB_DT_INT48 ||
           dt == TB_DT_INT64;
}
bool is_float_dt(int dt) {
    return dt == TB_DT_FP32 || dt == TB_DT_FP16 || dt == TB_DT_BF16 || dt == TB_DT_FP8E4M3 || dt == TB_DT_FP8E5M2;
}

const char* op_name(int op) {
    switch (op) {
    case fb::OP_AVG_POOL2D: return "AVG_POOL2D";
    case fb::OP_CONV2D: return "CONV2D";
    case fb::OP_DEPTHWISE_CONV2D: return "DEPTHWISE_CONV2D";
    case fb::OP_MATMUL: return "MATMUL";
    case fb::OP_MATMUL_T: return "MATMUL_T";
    case fb::OP_TRANSPOSE_CONV2D: return "TRANSPOSE_CONV2D";
    case fb::OP_CONV3D: return "CONV3D";
    case fb::OP_MAX_POOL2D: return "MAX_POOL2D";
    case fb::OP_CLAMP: return "CLAMP";
    case fb::OP_ADD: return "ADD";
    case fb::OP_RESHAPE: return "RESHAPE";
    case fb::OP_TRANSPOSE: return "TRANSPOSE";
    case fb::OP_RESCALE: return "RESCALE";
    case fb::OP_CONST: return "CONST";
    case fb::OP_IDENTITY: return "IDENTITY";
    case fb::OP_CONST_SHAPE: return "CONST_SHAPE";
    default: return "UNSUPPORTED";
    }
}

bool runner_supports(int op) { return std::strcmp(op_name(op), "UNSUPPORTED") != 0; }

float bf16_to_f32(uint16_t b) {
    uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    float v;
    if (exp == 0) v = std::ldexp(static_cast<float>(man), -24);
    else if (exp == 31) v = man ? NAN : INFINITY;
    else v = std::ldexp(static_cast<float>(man | 0x400), static_cast<int>(exp) - 25);
    return sign ? -v : v;
}

// FP8 E4M3 / E5M2 byte -> float (exact; src/float8.rs).
float fp8_to_f32(uint8_t bits, int dt) {
    const int man_bits = dt == TB_DT_FP8E4M3 ? 3 : 2, bias = dt == TB_DT_FP8E4M3 ? 7 : 15;
    const unsigned maxe = (1u << (7 - man_bits)) - 1u, manm = (1u << man_bits) - 1u;
    const unsigned e = (bits >> man_bits) & maxe, m = bits & manm;
    const bool has_inf = dt == TB_DT_FP8E5M2;
    if (has_inf ? (e == maxe && m != 0) : (e == maxe && m == manm)) return NAN;
    const float sign = (bits & 0x80) ? -1.f : 1.f;
    if (has_inf && e == maxe) return sign * INFINITY;
    const int expo = (e == 0 ? 1 : static_cast<int>(e)) - bias - man_bits;
    return sign * std::ldexp(static_cast<float>(e == 0 ? m : ((1u << man_bits) | m)), expo);
}

struct Tensor {
    std::string name;
    int dtype = 0;
    std::vector<int64_t> shape;
    int64_t count = 0;             // product of the shape (0 for an empty tensor)
    void* dev = nullptr;           // device data (owned buffer, alias, or bound input)
    bool owned = false;
    bool materialized = true;      // false: produced inside a fused group, never written
    bool is_static = false;        // value fixed at compile (CONST-derived)
    bool host = false;             // host values below are valid
    std::vector<int64_t> hi;       // integer values (static tensors)
    std::vector<float> hf;         // float values (static tensors)
    int64_t ref_bytes() const { return std::max<int64_t>(count, 1) * ref_elem_bytes(dtype); }
    size_t dev_bytes() const { return static_cast<size_t>(count) * dev_elem_bytes(dtype); }
};

enum Kind {
    K_NONE, K_CONST, K_ALIAS, K_TRANSPOSE, K_CONV, K_MATMUL, K_RESCALE, K_CLAMP, K_ADD, K_AVGPOOL, K_MAXPOOL,
    K_RESIDUAL, K_FUSED
};

struct Step {
    int op_index = 0;
    int op = 0;
    int kind = K_NONE;
    tb_status status = TB_OK;
    std::string err;
    std::vector<int> in, out;       // tensor ids of the operator's operands (in) and result (out)
    int exec_out = -1;              // tensor the group's kernel writes (fusion leader)
    std::vector<int> group;         // fused op indices led by this step (RESCALE, CLAMP / chain members)
    // contraction
    bool depthwise = false;
    bool transpose = false;         // TRANSPOSE_CONV2D (cdesc.pad holds out_pad)
    bool conv3d = false;            // CONV3D: c3desc instead of cdesc
    tb_conv3d_desc c3desc{};
    tb_conv2d_desc cdesc{};
    tb_matmul_desc mdesc{};
    int mt_batch = 0;               // MATMUL_T: batch of b [mt_batch, w, c] (n or 1); 0 for MATMUL
    tb_conv2d_plan* conv = nullptr;
    tb_matmul_plan* mm = nullptr;
    tb_rescale_attr rattr{};        // fused or standalone RESCALE attribute (host arrays below)
    std::vector<int32_t> rmult;
    std::vector<int8_t> rshift;
    bool has_rescale = false;
    // standalone RESCALE / residual chain
    RescalePlan rs, ra, rb;
    ResidualFast rfast;
    int in_dtype = 0, in_uns = 0, b_dtype = 0, b_uns = 0;
    int32_t izp = 0, bzp = 0;
    int channels = 1;
    // CLAMP
    int64_t cmin_i = 0, cmax_i = 0;
    float cmin_f = 0, cmax_f = 0;
    int nan_mode = 1;
    // pools
    tb_pool2d_desc pool{};
    // TRANSPOSE / ADD
    NdMap map{};
    int rank = 0;
    bool same_shape = false;
};

struct StatusError {
    tb_status st;
    std::string msg;
};

}  // namespace

struct tb_graph {
    tb_context* ctx = nullptr;
    uint32_t flags = 0;
    fb::Graph g;
    const fb::Block* block = nullptr;
    std::unordered_map<std::string, const fb::TensorDef*> defs;

    struct Bound {
        int dtype;
        std::vector<int64_t> shape;
        void* dev = nullptr;        // device data (owned copy or caller pointer)
        size_t cap = 0;             // owned capacity
        bool owned = false;
    };
    std::unordered_map<std::string, Bound> inputs;

    // compiled state
    bool compiled = false;
    std::string signature;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int> tid;
    std::vector<int> order;          // op indices in execution order
    std::vector<Step> steps;         // indexed by op index
    std::vector<int> unexecuted;     // ops the order never reaches
    int stop_at = -1;                // position in `order` of the first compile error
    std::vector<void*> buffers;
    int fault_alloc = 0;             // TB_FAULT_ALLOC_FAIL: fail this buffer allocation (1-based), 0 = never
    int allocs = 0;                  // buffer allocations attempted so far

    std::vector<cudaEvent_t> op_events;   // TB_GRAPH_TIME_OPS: start/stop pair per operator
    std::vector<float> op_ms;             // device time per operator index of the last run (-1: no kernel)

    cudaGraph_t cgraph = nullptr;
    cudaGraphExec_t cexec = nullptr;
    uint64_t graph_launches = 0;
    uint64_t last_launches = 0;

    ~tb_graph() {
        release();
        for (cudaEvent_t e : op_events) cudaEventDestroy(e);
    }

    void release() {
        if (cexec) cudaGraphExecDestroy(cexec);
        if (cgraph) cudaGraphDestroy(cgraph);
        cexec = nullptr;
        cgraph = nullptr;
        for (auto& s : steps) {
            if (s.conv) tb_conv2d_plan_destroy(s.conv);
            if (s.mm) tb_matmul_plan_destroy(s.mm);
            free_rescale_plan(&s.rs);
            free_rescale_plan(&s.ra);
            free_rescale_plan(&s.rb);
            free_residual_table(&s.rfast);
        }
        steps.clear();
        for (void* p : buffers) cudaFree(p);
        buffers.clear();
        tensors.clear();
        tid.clear();
        order.clear();
        unexecuted.clear();
        compiled = false;
    }
};

namespace {

[[noreturn]] void raise(tb_status st, const char* fmt, ...) {
    char buf[768];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    throw StatusError{st, buf};
}

std::string shape_str(const std::vector<int64_t>& s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
    return r + "]";
}

class Compiler {
  public:
    explicit Compiler(tb_graph* g) : G(*g) {}

    Tensor& T(int id) { return G.tensors[id]; }

    int get(const std::string& name) {
        auto it = G.tid.find(name);
        if (it == G.tid.end()) raise(TB_ERR_TENSOR_NOT_FOUND, "%s", name.c_str());
        return it->second;
    }

    int add_tensor(Tensor t) {
        const int id = static_cast<int>(G.tensors.size());
        G.tid[t.name] = id;
        G.tensors.push_back(std::move(t));
        return id;
    }

    const fb::TensorDef* def(const std::string& name) {
        auto it = G.defs.find(name);
        return it == G.defs.end() ? nullptr : it->second;
    }

    // check_declared_output (src/ops/common.rs:46-60): returns the declared dtype or 0.
    int declared(const char* op, const std::string& name, const std::vector<int64_t>& shape) {
        const fb::TensorDef* d = def(name);
        if (!d) return 0;
        bool stat = true;
        for (int v : d->shape) stat &= v >= 0;
        if (stat) {
            std::vector<int64_t> dec(d->shape.begin(), d->shape.end());
            if (dec != shape)
                raise(TB_ERR_SHAPE_MISMATCH, "%s: output shape %s does not match declared shape %s", op,
                      shape_str(shape).c_str(), shape_str(dec).c_str());
        }
        return d->dtype;
    }

    void expect_operands(const fb::Operator& o, const char* op, size_t ni, size_t no) {
        if (o.inputs.size() != ni || o.outputs.size() != no)
            raise(TB_ERR_GRAPH, "%s: expected %zu inputs and %zu outputs, got %zu and %zu", op, ni, no, o.inputs.size(),
                  o.outputs.size());
    }

    void expect_rank(const char* op, const char* what, const Tensor& t, size_t rank) {
        if (t.shape.size() != rank)
            raise(TB_ERR_SHAPE_MISMATCH, "%s: %s must have rank %zu, got shape %s", op, what, rank,
                  shape_str(t.shape).c_str());
    }

    // single_value (src/ops/common.rs:31-40) + host value (static operands only).
    const Tensor& single(const char* op, const char* what, int id) {
        const Tensor& t = T(id);
        expect_rank(op, what, t, 1);
        if (t.count != 1)
            raise(TB_ERR_SHAPE_MISMATCH, "%s: %s must have exactly one element, got shape %s", op, what,
                  shape_str(t.shape).c_str());
        if (!t.host) raise(TB_ERR_NOT_ACCELERATED, "%s: %s must be a constant for this backend", op, what);
        return t;
    }

    static int64_t ival(const Tensor& t, size_t i = 0) {
        return t.hi.empty() ? static_cast<int64_t>(t.hf[i]) : t.hi[i];
    }

    // Result tensor of an operator.
    int make_out(const std::string& name, int dtype, std::vector<int64_t> shape) {
        Tensor t;
        t.name = name;
        t.dtype = dtype;
        t.shape = std::move(shape);
        t.count = 1;
        for (int64_t v : t.shape) t.count *= v;
        return add_tensor(std::move(t));
    }

    int make_alias(const std::string& name, int src, std::vector<int64_t> shape) {
        Tensor t = T(src);
        t.name = name;
        t.shape = std::move(shape);
        t.owned = false;
        const int id = add_tensor(std::move(t));
        alias_of[id] = src;
        return id;
    }

    std::unordered_map<int, int> alias_of;

    // ---- per-operator inference and validation -----------------------------------------

    void c_const(const fb::Operator& o, Step& s) {
        if (o.outputs.empty()) raise(TB_ERR_GRAPH, "CONST op has no output");
        const fb::TensorDef* d = def(o.outputs[0]);
        if (!d) raise(TB_ERR_TENSOR_NOT_FOUND, "%s", o.outputs[0].c_str());
        Tensor t;
        t.name = o.outputs[0];
        t.dtype = d->dtype == TB_DT_SHAPE ? TB_DT_INT64 : d->dtype;
        t.count = 1;
        for (int v : d->shape) {
            t.shape.push_back(std::max(v, 0));
            t.count *= std::max(v, 0);
        }
        decode(d, &t);
        t.is_static = true;
        s.kind = K_CONST;
        s.out = {add_tensor(std::move(t))};
    }

    // TensorData::from_raw_bytes (src/tensor.rs:86-167).
    void decode(const fb::TensorDef* d, Tensor* t) {
        const int dt = d->dtype;
        const int64_t n = t->count;
        const bool keep_host = n <= (1 << 16);
        if (ref_elem_bytes(dt) == 0) raise(TB_ERR_DTYPE_MISMATCH, "cannot deserialize raw bytes for dtype %d", dt);
        int64_t needed = dt == TB_DT_INT4 ? (n + 1) / 2 : dt == TB_DT_INT48 ? n * 6 : n * ref_elem_bytes(dt);
        std::vector<uint8_t> zeros;
        const uint8_t* src;
        if (!d->has_data) {
            zeros.assign(static_cast<size_t>(std::max<int64_t>(needed, 0)), 0);
            src = zeros.data();
        } else {
            if (static_cast<int64_t>(d->data.size()) < needed)
                raise(TB_ERR_DESERIALIZE, "dtype %d tensor of %lld elements needs %lld bytes, got %zu", dt,
                      static_cast<long long>(n), static_cast<long long>(needed), d->data.size());
            src = d->data.data();
        }
        if (!(is_int_dt(dt) || is_float_dt(dt) || dt == TB_DT_BOOL || dt == TB_DT_SHAPE))
            raise(TB_ERR_DTYPE_MISMATCH, "cannot deserialize raw bytes for dtype %d", dt);
        // device image
        std::vector<uint8_t>& img = t_img;
        img.assign(static_cast<size_t>(n) * dev_elem_bytes(t->dtype), 0);
        if (dt == TB_DT_INT4) {
            for (int64_t i = 0; i < n; ++i) {
                const int nib = (src[i / 2] >> (4 * (i % 2))) & 0xF;
                img[i] = static_cast<uint8_t>(static_cast<int8_t>(nib << 4) >> 4);
            }
        } else if (dt == TB_DT_INT48) {
            for (int64_t i = 0; i < n; ++i) {
                int64_t v = 0;
                for (int k = 0; k < 6; ++k) v |= static_cast<int64_t>(src[6 * i + k]) << (8 * k);
                if (v & (1ll << 47)) v -= 1ll << 48;
                std::memcpy(&img[8 * i], &v, 8);
            }
        } else if (dt == TB_DT_BOOL) {
            for (int64_t i = 0; i < n; ++i) img[i] = src[i] != 0;
        } else {
            std::memcpy(img.data(), src, img.size());
        }
        if (keep_host) {
            t->host = true;
            for (int64_t i = 0; i < n; ++i) {
                const uint8_t* p = &img[static_cast<size_t>(i) * dev_elem_bytes(t->dtype)];
                switch (t->dtype) {
                case TB_DT_BOOL: case TB_DT_INT4: case TB_DT_INT8: t->hi.push_back(static_cast<int8_t>(*p)); break;
                case TB_DT_INT16: { int16_t v; std::memcpy(&v, p, 2); t->hi.push_back(v); break; }
                case TB_DT_INT32: { int32_t v; std::memcpy(&v, p, 4); t->hi.push_back(v); break; }
                case TB_DT_INT48: case TB_DT_INT64: { int64_t v; std::memcpy(&v, p, 8); t->hi.push_back(v); break; }
                case TB_DT_FP32: { float v; std::memcpy(&v, p, 4); t->hf.push_back(v); break; }
                case TB_DT_FP16: { uint16_t v; std::memcpy(&v, p, 2); t->hf.push_back(f16_to_f32(v)); break; }
                case TB_DT_BF16: { uint16_t v; std::memcpy(&v, p, 2); t->hf.push_back(bf16_to_f32(v)); break; }
                case TB_DT_FP8E4M3: case TB_DT_FP8E5M2: t->hf.push_back(fp8_to_f32(*p, t->dtype)); break;
                default: t->host = false; break;
                }
                if (!t->host) break;
            }
            if (t->dtype == TB_DT_BOOL)
                for (auto& v : t->hi) v = v != 0;
        }
        uploads.emplace_back(static_cast<int>(G.tensors.size()), std::move(img));
    }
    std::vector<uint8_t> t_img;
    std::vector<std::pair<int, std::vector<uint8_t>>> uploads;  // tensor id -> device image

    void c_identity(const fb::Operator& o, Step& s) {
        if (o.inputs.empty()) raise(TB_ERR_GRAPH, "IDENTITY op has no input");
        if (o.outputs.empty()) raise(TB_ERR_GRAPH, "IDENTITY op has no output");
        const int x = get(o.inputs[0]);
        s.in = {x};
        s.kind = K_ALIAS;
        s.out = {make_alias(o.outputs[0], x, T(x).shape)};
    }

    void c_reshape(const fb::Operator& o, Step& s) {
        const char* op = "RESHAPE";
        expect_operands(o, op, 2, 1);
        const int x = get(o.inputs[0]);
        const int sh = get(o.inputs[1]);
        const Tensor& st = T(sh);
        if (!is_int_dt(st.dtype)) raise(TB_ERR_GRAPH, "%s: operand '%s' must be a shape", op, o.inputs[1].c_str());
        if (!st.host) raise(TB_ERR_NOT_ACCELERATED, "%s: the new shape must be a constant for this backend", op);
        std::vector<int64_t> ns(st.hi.begin(), st.hi.end());
        for (int64_t v : ns)
            if (v < 0) raise(TB_ERR_GRAPH, "%s: shape %s must be non-negative", op, shape_str(ns).c_str());
        int64_t a = 1, b = 1;
        for (int64_t v : ns) a *= v;
        for (int64_t v : T(x).shape) b *= v;
        if (a != b)
            raise(TB_ERR_SHAPE_MISMATCH, "%s: cannot reshape %s to %s", op, shape_str(T(x).shape).c_str(),
                  shape_str(ns).c_str());
        const int decl = declared(op, o.outputs[0], ns);
        if (decl && decl != T(x).dtype) raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype must match input dtype", op);
        s.in = {x, sh};
        s.kind = K_ALIAS;
        s.out = {make_alias(o.outputs[0], x, ns)};
    }

    void c_transpose(const fb::Operator& o, Step& s) {
        const char* op = "TRANSPOSE";
        if (o.attr.type != fb::OP_TRANSPOSE) raise(TB_ERR_GRAPH, "%s: missing attribute", op);
        expect_operands(o, op, 1, 1);
        const int x = get(o.inputs[0]);
        const Tensor& t = T(x);
        if (t.shape.empty()) raise(TB_ERR_SHAPE_MISMATCH, "%s: input must have rank at least 1", op);
        const size_t rank = t.shape.size();
        std::vector<bool> used(rank, false);
        for (int p : o.attr.perms) {
            if (p < 0 || static_cast<size_t>(p) >= rank || used[p])
                raise(TB_ERR_GRAPH, "%s: perms must be a permutation of 0..%zu", op, rank);
            used[p] = true;
        }
        if (o.attr.perms.size() != rank) raise(TB_ERR_GRAPH, "%s: perms must have %zu entries", op, rank);
        if (rank > 6) raise(TB_ERR_NOT_ACCELERATED, "%s: rank above 6", op);
        std::vector<int64_t> out_shape(rank);
        std::vector<int64_t> in_stride(rank);
        int64_t acc = 1;
        for (size_t d = rank; d-- > 0;) {
            in_stride[d] = acc;
            acc *= t.shape[d];
        }
        for (size_t d = 0; d < rank; ++d) {
            out_shape[d] = t.shape[o.attr.perms[d]];
            s.map.dims[d] = out_shape[d];
            s.map.a_stride[d] = in_stride[o.attr.perms[d]];
        }
        const int decl = declared(op, o.outputs[0], out_shape);
        if (decl && decl != t.dtype) raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype must match input dtype", op);
        s.rank = static_cast<int>(rank);
        s.in = {x};
        s.kind = K_TRANSPOSE;
        const int y = make_out(o.outputs[0], t.dtype, out_shape);
        if (t.is_static && t.host) {  // a transposed constant stays a constant
            Tensor& ty = T(y);
            ty.is_static = true;
        }
        s.out = {y};
    }

    // CONV2D, DEPTHWISE_CONV2D, and TRANSPOSE_CONV2D (transpose: attribute out_pad in a.pad,
    // no dilation; Transpose::new src/ops/conv.rs:286-329)
    void c_conv(const fb::Operator& o, Step& s, bool depthwise, bool transpose = false) {
        const char* op = transpose ? "TRANSPOSE_CONV2D" : depthwise ? "DEPTHWISE_CONV2D" : "CONV2D";
        if (o.attr.type != o.op) raise(TB_ERR_GRAPH, "%s: missing attribute", op);
        expect_operands(o, op, 5, 1);
        const int x = get(o.inputs[0]), w = get(o.inputs[1]), b = get(o.inputs[2]);
        const Tensor& zx = single(op, "input_zp", get(o.inputs[3]));
        const Tensor& zw = single(op, "weight_zp", get(o.inputs[4]));
        const Tensor &X = T(x), &W = T(w), &B = T(b);
        expect_rank(op, "bias", B, 1);
        expect_rank(op, "input", X, 4);
        expect_rank(op, "weight", W, 4);
        Attr a = o.attr;
        if (transpose) {
            if (a.pad.size() != 4 || a.stride.size() != 2)
                raise(TB_ERR_GRAPH, "%s: out_pad must have 4 elements and stride 2", op);
            for (int v : a.stride) if (v < 1) raise(TB_ERR_GRAPH, "%s: stride must be at least 1", op);
            a.dilation = {1, 1};
        } else {
            if (a.pad.size() != 4 || a.stride.size() != 2 || a.dilation.size() != 2)
                raise(TB_ERR_GRAPH, "%s: pad must have 4 elements, stride and dilation 2", op);
            for (int p : a.pad) if (p < 0) raise(TB_ERR_GRAPH, "%s: pad must be non-negative", op);
            for (int v : a.stride) if (v < 1) raise(TB_ERR_GRAPH, "%s: stride must be at least 1", op);
            for (int v : a.dilation) if (v < 1) raise(TB_ERR_GRAPH, "%s: dilation must be at least 1", op);
        }
        const int64_t ic = X.shape[3];
        const int64_t kic = depthwise ? W.shape[2] : W.shape[3];
        if (kic != ic)
            raise(TB_ERR_SHAPE_MISMATCH, "%s: weight input channels %lld != input channels %lld", op,
                  static_cast<long long>(kic), static_cast<long long>(ic));
        const int64_t kh = depthwise ? W.shape[0] : W.shape[1], kw = depthwise ? W.shape[1] : W.shape[2];
        auto extent = [&](int64_t in, int pb, int pa, int64_t k, int dil, int st) -> int64_t {
            const int64_t full = in - 1 + pb + pa - (k - 1) * dil;
            if (full % st != 0) raise(TB_ERR_GRAPH, "%s: parameters must yield exact integer output dimensions", op);
            const int64_t out = full / st + 1;
            if (out < 1) raise(TB_ERR_GRAPH, "%s: output dimension %lld must be positive", op, static_cast<long long>(out));
            return out;
        };
        int64_t oh, ow;
        if (transpose) {
            for (int i = 0; i < 4; ++i)
                if (a.pad[i] <= -(i < 2 ? kh : kw))
                    raise(TB_ERR_GRAPH, "%s: out_pad must be greater than -kernel size", op);
            oh = (X.shape[1] - 1) * a.stride[0] + a.pad[0] + a.pad[1] + kh;
            ow = (X.shape[2] - 1) * a.stride[1] + a.pad[2] + a.pad[3] + kw;
            if (oh < 1 || ow < 1) raise(TB_ERR_GRAPH, "%s: output size must be positive", op);
        } else {
            oh = extent(X.shape[1], a.pad[0], a.pad[1], kh, a.dilation[0], a.stride[0]);
            ow = extent(X.shape[2], a.pad[2], a.pad[3], kw, a.dilation[1], a.stride[1]);
        }
        const int64_t m = depthwise ? W.shape[3] : 1;
        const int64_t oc = depthwise ? ic * m : W.shape[0];
        const int64_t bc = B.shape[0];
        if (bc != oc && bc != 1)
            raise(TB_ERR_SHAPE_MISMATCH, "%s: bias channels %lld must be 1 or match output channels %lld", op,
                  static_cast<long long>(bc), static_cast<long long>(oc));
        const std::vector<int64_t> out_shape = {X.shape[0], oh, ow, oc};
        const int decl = declared(op, o.outputs[0], out_shape);
        if (decl && decl != B.dtype)
            raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype %d does not match bias dtype %d", op, decl, B.dtype);
        if (zx.dtype != X.dtype || zw.dtype != W.dtype)
            raise(TB_ERR_DTYPE_MISMATCH, "%s: zero points must match input/weight dtypes", op);
        for (int64_t v : {X.shape[0], X.shape[1], X.shape[2], ic, oc, kh, kw, m})
            if (v > INT32_MAX) raise(TB_ERR_NOT_ACCELERATED, "%s: dimension above int32", op);
        tb_conv2d_desc& d = s.cdesc;
        d.n = static_cast<int32_t>(X.shape[0]);
        d.ih = static_cast<int32_t>(X.shape[1]);
        d.iw = static_cast<int32_t>(X.shape[2]);
        d.ic = static_cast<int32_t>(ic);
        d.oc = static_cast<int32_t>(oc);
        d.kh = static_cast<int32_t>(kh);
        d.kw = static_cast<int32_t>(kw);
        d.m = static_cast<int32_t>(m);
        for (int i = 0; i < 4; ++i) d.pad[i] = a.pad[i];
        for (int i = 0; i < 2; ++i) { d.stride[i] = a.stride[i]; d.dilation[i] = a.dilation[i]; }
        d.in_dtype = X.dtype;
        d.w_dtype = W.dtype;
        d.acc_dtype = a.acc_type;
        d.out_dtype = B.dtype;
        d.bias_len = static_cast<int32_t>(bc);
        const int64_t izp = ival(zx), wzp = ival(zw);
        if (is_float_dt(X.dtype)) {
            if (zx.hf.empty() ? izp != 0 : zx.hf[0] != 0.f) raise(TB_ERR_GRAPH, "%s: zero points must be zero", op);
            if (zw.hf.empty() ? wzp != 0 : zw.hf[0] != 0.f) raise(TB_ERR_GRAPH, "%s: zero points must be zero", op);
        } else {
            if (izp != 0 && X.dtype != TB_DT_INT8)
                raise(TB_ERR_GRAPH, "%s: input zero point must be zero for non-int8 input", op);
            if (wzp != 0 && W.dtype != TB_DT_INT8)
                raise(TB_ERR_GRAPH, "%s: weight zero point must be zero for non-int8 weight", op);
            d.input_zp = static_cast<int32_t>(izp);
            d.weight_zp = static_cast<int32_t>(wzp);
        }
        s.depthwise = depthwise;
        s.transpose = transpose;
        s.kind = K_CONV;
        s.in = {x, w, b, get(o.inputs[3]), get(o.inputs[4])};
        s.out = {make_out(o.outputs[0], B.dtype, out_shape)};
    }

    // CONV3D (src/ops/conv.rs:510-516; eval_conv :398-500 with ConvNd::new :107-139, dims 3)
    void c_conv3d(const fb::Operator& o, Step& s) {
        const char* op = "CONV3D";
        if (o.attr.type != o.op) raise(TB_ERR_GRAPH, "%s: missing attribute", op);
        expect_operands(o, op, 5, 1);
        const int x = get(o.inputs[0]), w = get(o.inputs[1]), b = get(o.inputs[2]);
        const Tensor& zx = single(op, "input_zp", get(o.inputs[3]));
        const Tensor& zw = single(op, "weight_zp", get(o.inputs[4]));
        const Tensor &X = T(x), &W = T(w), &B = T(b);
        expect_rank(op, "bias", B, 1);
        expect_rank(op, "input", X, 5);
        expect_rank(op, "weight", W, 5);
        const Attr& a = o.attr;
        if (a.pad.size() != 6 || a.stride.size() != 3 || a.dilation.size() != 3)
            raise(TB_ERR_GRAPH, "%s: pad must have 6 elements, stride and dilation 3", op);
        for (int p : a.pad) if (p < 0) raise(TB_ERR_GRAPH, "%s: pad must be non-negative", op);
        for (int v : a.stride) if (v < 1) raise(TB_ERR_GRAPH, "%s: stride must be at least 1", op);
        for (int v : a.dilation) if (v < 1) raise(TB_ERR_GRAPH, "%s: dilation must be at least 1", op);
        if (W.shape[4] != X.shape[4])
            raise(TB_ERR_SHAPE_MISMATCH, "%s: weight input channels %lld != input channels %lld", op,
                  static_cast<long long>(W.shape[4]), static_cast<long long>(X.shape[4]));
        std::vector<int64_t> out_shape = {X.shape[0]};
        for (int d = 0; d < 3; ++d) {
            const int64_t full = X.shape[1 + d] - 1 + a.pad[2 * d] + a.pad[2 * d + 1] - (W.shape[1 + d] - 1) * a.dilation[d];
            if (full % a.stride[d] != 0)
                raise(TB_ERR_GRAPH, "%s: parameters must yield exact integer output dimensions", op);
            const int64_t e = full / a.stride[d] + 1;
            if (e < 1) raise(TB_ERR_GRAPH, "%s: output dimension %lld must be positive", op, static_cast<long long>(e));
            out_shape.push_back(e);
        }
        const int64_t oc = W.shape[0], bc = B.shape[0];
        out_shape.push_back(oc);
        if (bc != oc && bc != 1)
            raise(TB_ERR_SHAPE_MISMATCH, "%s: bias channels %lld must be 1 or match output channels %lld", op,
                  static_cast<long long>(bc), static_cast<long long>(oc));
        const int decl = declared(op, o.outputs[0], out_shape);
        if (decl && decl != B.dtype)
            raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype %d does not match bias dtype %d", op, decl, B.dtype);
        if (zx.dtype != X.dtype || zw.dtype != W.dtype)
            raise(TB_ERR_DTYPE_MISMATCH, "%s: zero points must match input/weight dtypes", op);
        for (int64_t v : X.shape) if (v > INT32_MAX) raise(TB_ERR_NOT_ACCELERATED, "%s: dimension above int32", op);
        for (int64_t v : W.shape) if (v > INT32_MAX) raise(TB_ERR_NOT_ACCELERATED, "%s: dimension above int32", op);
        tb_conv3d_desc& d = s.c3desc;
        d.n = static_cast<int32_t>(X.shape[0]);
        d.id = static_cast<int32_t>(X.shape[1]);
        d.ih = static_cast<int32_t>(X.shape[2]);
        d.iw = static_cast<int32_t>(X.shape[3]);
        d.ic = static_cast<int32_t>(X.shape[4]);
        d.oc = static_cast<int32_t>(oc);
        d.kd = static_cast<int32_t>(W.shape[1]);
        d.kh = static_cast<int32_t>(W.shape[2]);
        d.kw = static_cast<int32_t>(W.shape[3]);
        for (int i = 0; i < 6; ++i) d.pad[i] = a.pad[i];
        for (int i = 0; i < 3; ++i) { d.stride[i] = a.stride[i]; d.dilation[i] = a.dilation[i]; }
        d.in_dtype = X.dtype;
        d.w_dtype = W.dtype;
        d.acc_dtype = a.acc_type;
        d.out_dtype = B.dtype;
        d.bias_len = static_cast<int32_t>(bc);
        const int64_t izp = ival(zx), wzp = ival(zw);
        if (is_float_dt(X.dtype)) {
            if (zx.hf.empty() ? izp != 0 : zx.hf[0] != 0.f) raise(TB_ERR_GRAPH, "%s: zero points must be zero", op);
            if (zw.hf.empty() ? wzp != 0 : zw.hf[0] != 0.f) raise(TB_ERR_GRAPH, "%s: zero points must be zero", op);
        } else {
            if (izp != 0 && X.dtype != TB_DT_INT8)
                raise(TB_ERR_GRAPH, "%s: input zero point must be zero for non-int8 input", op);
            if (wzp != 0 && W.dtype != TB_DT_INT8)
                raise(TB_ERR_GRAPH, "%s: weight zero point must be zero for non-int8 weight", op);
            d.input_zp = static_cast<int32_t>(izp);
            d.weight_zp = static_cast<int32_t>(wzp);
        }
        s.conv3d = true;
        s.kind = K_CONV;
        s.in = {x, w, b, get(o.inputs[3]), get(o.inputs[4])};
        s.out = {make_out(o.outputs[0], B.dtype, out_shape)};
    }

    // MATMUL, and MATMUL_T (transposed) with b [d,w,c], d == n or 1 (src/ops/matmul.rs:98-174)
    void c_matmul(const fb::Operator& o, Step& s, bool transposed) {
        const char* op = transposed ? "MATMUL_T" : "MATMUL";
        expect_operands(o, op, 4, 1);
        const int a = get(o.inputs[0]), b = get(o.inputs[1]);
        const Tensor& za = single(op, "a_zp", get(o.inputs[2]));
        const Tensor& zb = single(op, "b_zp", get(o.inputs[3]));
        const Tensor &A = T(a), &B = T(b);
        expect_rank(op, "a", A, 3);
        expect_rank(op, "b", B, 3);
        const int64_t bc = transposed ? B.shape[2] : B.shape[1], bw = transposed ? B.shape[1] : B.shape[2];
        if (bc != A.shape[2] || (B.shape[0] != A.shape[0] && !(transposed && B.shape[0] == 1)))
            raise(TB_ERR_SHAPE_MISMATCH, "%s: b shape %s incompatible with a shape %s", op, shape_str(B.shape).c_str(),
                  shape_str(A.shape).c_str());
        const std::vector<int64_t> out_shape = {A.shape[0], A.shape[1], bw};
        int out_t = declared(op, o.outputs[0], out_shape);
        if (!out_t) {
            const int at = A.dtype;
            out_t = at == TB_DT_INT8 ? TB_DT_INT32 : at == TB_DT_INT16 ? TB_DT_INT48
                    : (at == TB_DT_FP16 || at == TB_DT_FP8E4M3 || at == TB_DT_FP8E5M2) ? TB_DT_FP16 : TB_DT_FP32;
        }
        if (za.dtype != A.dtype || zb.dtype != B.dtype)
            raise(TB_ERR_DTYPE_MISMATCH, "%s: zero points must match input dtypes", op);
        tb_matmul_desc& d = s.mdesc;
        d.n = static_cast<int32_t>(A.shape[0]);
        d.h = static_cast<int32_t>(A.shape[1]);
        d.c = static_cast<int32_t>(A.shape[2]);
        d.w = static_cast<int32_t>(bw);
        d.a_dtype = A.dtype;
        d.b_dtype = B.dtype;
        d.out_dtype = out_t;
        if (is_int_dt(out_t)) {
            d.a_zp = static_cast<int32_t>(ival(za));
            d.b_zp = static_cast<int32_t>(ival(zb));
        } else {
            const bool nz = (za.hf.empty() ? ival(za) != 0 : za.hf[0] != 0.f) ||
                            (zb.hf.empty() ? ival(zb) != 0 : zb.hf[0] != 0.f);
            if (nz) raise(TB_ERR_GRAPH, "%s: zero points must be zero for floating-point inputs", op);
        }
        s.mt_batch = transposed ? static_cast<int>(B.shape[0]) : 0;
        int path = 0, bn = 0;
        tb_status st = matmul_validate(&d, false, &path, &bn, s.mt_batch);
        if (st != TB_OK) raise(st, "%s", tb_last_error());
        s.kind = K_MATMUL;
        s.in = {a, b, get(o.inputs[2]), get(o.inputs[3])};
        s.out = {make_out(o.outputs[0], out_t, out_shape)};
    }

    void c_rescale(const fb::Operator& o, Step& s) {
        const char* op = "RESCALE";
        if (o.attr.type != fb::OP_RESCALE) raise(TB_ERR_GRAPH, "%s: missing attribute", op);
        expect_operands(o, op, 5, 1);
        const int x = get(o.inputs[0]);
        const Tensor& X = T(x);
        const Tensor& M = T(get(o.inputs[1]));
        const Tensor& S = T(get(o.inputs[2]));
        const Tensor& IZ = T(get(o.inputs[3]));
        const Tensor& OZ = T(get(o.inputs[4]));
        int out_t = declared(op, o.outputs[0], X.shape);
        if (!out_t) out_t = TB_DT_INT32;
        const int in_t = X.dtype;
        const Attr& a = o.attr;
        auto in_ok = in_t == TB_DT_INT8 || in_t == TB_DT_INT16 || in_t == TB_DT_INT32 || in_t == TB_DT_INT48;
        auto out_ok = out_t == TB_DT_INT8 || out_t == TB_DT_INT16 || out_t == TB_DT_INT32;
        if (!in_ok || !out_ok) raise(TB_ERR_DTYPE_MISMATCH, "%s: unsupported types %d -> %d", op, in_t, out_t);
        if (a.rounding_mode < 1 || a.rounding_mode > 3) raise(TB_ERR_GRAPH, "%s: unsupported rounding mode", op);
        if (a.scale32 && in_t == TB_DT_INT48) raise(TB_ERR_GRAPH, "%s: scale32 is not allowed for INT48 input", op);
        if (!a.scale32 && a.rounding_mode == TB_ROUND_DOUBLE)
            raise(TB_ERR_GRAPH, "%s: double rounding requires scale32", op);
        const bool has32 = in_t == TB_DT_INT32 || in_t == TB_DT_INT48 || out_t == TB_DT_INT32;
        if ((a.input_unsigned && a.output_unsigned) || ((a.input_unsigned || a.output_unsigned) && has32))
            raise(TB_ERR_GRAPH, "%s: invalid combination of input_unsigned/output_unsigned and types", op);
        const int want_m = a.scale32 ? TB_DT_INT32 : TB_DT_INT16;
        if (M.dtype != want_m || S.dtype != TB_DT_INT8)
            raise(TB_ERR_DTYPE_MISMATCH, "%s: multiplier must be %s and shift INT8", op, a.scale32 ? "INT32" : "INT16");
        if (IZ.dtype != in_t || OZ.dtype != out_t || IZ.count != 1 || OZ.count != 1)
            raise(TB_ERR_GRAPH, "%s: zero points must be single elements of the input/output types", op);
        if (a.per_channel && X.shape.empty()) raise(TB_ERR_GRAPH, "%s: per_channel requires rank >= 1", op);
        const int64_t channels = a.per_channel ? X.shape.back() : 1;
        if (M.count != channels || S.count != channels)
            raise(TB_ERR_GRAPH, "%s: multiplier and shift must have %lld elements", op, static_cast<long long>(channels));
        if (!M.host || !S.host || !IZ.host || !OZ.host)
            raise(TB_ERR_NOT_ACCELERATED, "%s: multiplier, shift and zero points must be constants for this backend", op);
        s.rmult.assign(M.hi.begin(), M.hi.end());
        s.rshift.assign(S.hi.begin(), S.hi.end());
        tb_rescale_attr& r = s.rattr;
        r.scale32 = a.scale32;
        r.rounding_mode = a.rounding_mode;
        r.per_channel = a.per_channel;
        r.input_unsigned = a.input_unsigned;
        r.output_unsigned = a.output_unsigned;
        r.input_zp = static_cast<int32_t>(IZ.hi[0]);
        r.output_zp = static_cast<int32_t>(OZ.hi[0]);
        r.out_dtype = out_t;
        r.channels = static_cast<int32_t>(channels);
        r.multiplier = s.rmult.data();
        r.shift = s.rshift.data();
        int64_t ize, oze;
        int32_t lo, hi;
        tb_status st = check_rescale(&r, in_t, X.shape.empty() ? 1 : X.shape.back(), &ize, &oze, &lo, &hi);
        if (st != TB_OK) raise(st, "%s", tb_last_error());
        s.in_dtype = in_t;
        s.in_uns = a.input_unsigned;
        s.izp = static_cast<int32_t>(ize);
        s.channels = static_cast<int>(X.shape.empty() ? 1 : X.shape.back());
        s.kind = K_RESCALE;
        s.in = {x, get(o.inputs[1]), get(o.inputs[2]), get(o.inputs[3]), get(o.inputs[4])};
        s.out = {make_out(o.outputs[0], out_t, X.shape)};
    }

    void c_clamp(const fb::Operator& o, Step& s) {
        const char* op = "CLAMP";
        if (o.attr.type != fb::OP_CLAMP) raise(TB_ERR_GRAPH, "%s: missing attribute", op);
        if (o.attr.nan_mode != TB_NAN_PROPAGATE && o.attr.nan_mode != TB_NAN_IGNORE)
            raise(TB_ERR_GRAPH, "%s: nan_mode must be PROPAGATE or IGNORE", op);
        const int x = get(o.inputs.empty() ? std::string() : o.inputs[0]);
        const Tensor& X = T(x);
        const int dt = X.dtype;
        auto decode1 = [&](const std::vector<uint8_t>& raw, int64_t* iv, float* fv) {
            const int eb = dt == TB_DT_INT4 ? 1 : ref_elem_bytes(dt);
            if (eb == 0 || static_cast<int>(raw.size()) < eb) raise(TB_ERR_GRAPH, "%s: malformed min/max", op);
            switch (dt) {
            case TB_DT_INT8: *iv = static_cast<int8_t>(raw[0]); break;
            case TB_DT_INT16: { int16_t v; std::memcpy(&v, raw.data(), 2); *iv = v; break; }
            case TB_DT_INT32: { int32_t v; std::memcpy(&v, raw.data(), 4); *iv = v; break; }
            case TB_DT_FP32: std::memcpy(fv, raw.data(), 4); break;
            case TB_DT_FP16: { uint16_t v; std::memcpy(&v, raw.data(), 2); *fv = f16_to_f32(v); break; }
            case TB_DT_BF16: { uint16_t v; std::memcpy(&v, raw.data(), 2); *fv = bf16_to_f32(v); break; }
            default: break;
            }
        };
        int64_t lo_i = 0, hi_i = 0;
        float lo_f = 0, hi_f = 0;
        decode1(o.attr.min_val, &lo_i, &lo_f);
        decode1(o.attr.max_val, &hi_i, &hi_f);
        expect_operands(o, op, 1, 1);
        if (!(dt == TB_DT_FP16 || dt == TB_DT_BF16 || dt == TB_DT_FP32 || dt == TB_DT_INT8 || dt == TB_DT_INT16))
            raise(TB_ERR_DTYPE_MISMATCH, "%s: unsupported dtype", op);
        if (is_int_dt(dt)) {
            if (hi_i < lo_i) raise(TB_ERR_GRAPH, "%s: max_val must not be smaller than min_val", op);
        } else if (std::isnan(lo_f) || std::isnan(hi_f) || hi_f < lo_f) {
            raise(TB_ERR_GRAPH, "%s: min_val/max_val must be ordered and not NaN", op);
        }
        const int decl = declared(op, o.outputs[0], X.shape);
        if (decl && decl != dt) raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype mismatch", op);
        s.cmin_i = lo_i;
        s.cmax_i = hi_i;
        s.cmin_f = lo_f;
        s.cmax_f = hi_f;
        s.nan_mode = o.attr.nan_mode;
        s.kind = K_CLAMP;
        s.in = {x};
        s.out = {make_out(o.outputs[0], dt, X.shape)};
    }

    void c_add(const fb::Operator& o, Step& s) {
        const char* op = "ADD";
        expect_operands(o, op, 2, 1);
        const int a = get(o.inputs[0]), b = get(o.inputs[1]);
        const Tensor &A = T(a), &B = T(b);
        if (A.dtype != B.dtype) raise(TB_ERR_DTYPE_MISMATCH, "%s: input dtypes differ", op);
        // broadcast.rs: right-aligned, each pair equal or one of them 1
        const size_t rank = std::max(A.shape.size(), B.shape.size());
        std::vector<int64_t> out(rank);
        for (size_t i = 0; i < rank; ++i) {
            const int64_t da = i < rank - A.shape.size() ? 1 : A.shape[i - (rank - A.shape.size())];
            const int64_t db = i < rank - B.shape.size() ? 1 : B.shape[i - (rank - B.shape.size())];
            if (da != db && da != 1 && db != 1)
                raise(TB_ERR_BROADCAST, "%s: shapes %s and %s are not compatible", op, shape_str(A.shape).c_str(),
                      shape_str(B.shape).c_str());
            out[i] = da == 1 ? db : da;
        }
        const int dt = A.dtype;
        if (!(dt == TB_DT_FP16 || dt == TB_DT_BF16 || dt == TB_DT_FP32 || dt == TB_DT_INT32 || dt == TB_DT_INT64))
            raise(TB_ERR_DTYPE_MISMATCH, "%s: unsupported dtype", op);
        if (dt == TB_DT_INT64) raise(TB_ERR_NOT_ACCELERATED, "%s: INT64 is not accelerated", op);
        if (rank > 6) raise(TB_ERR_NOT_ACCELERATED, "%s: rank above 6", op);
        const int decl = declared(op, o.outputs[0], out);
        if (decl && decl != dt) raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype mismatch", op);
        auto strides = [&](const std::vector<int64_t>& sh, long long* st) {
            long long acc = 1;
            for (size_t i = rank; i-- > 0;) {
                const size_t off = rank - sh.size();
                const int64_t d = i < off ? 1 : sh[i - off];
                st[i] = d == 1 ? 0 : acc;
                acc *= d;
            }
        };
        for (size_t i = 0; i < rank; ++i) s.map.dims[i] = out[i];
        strides(A.shape, s.map.a_stride);
        strides(B.shape, s.map.b_stride);
        s.rank = static_cast<int>(rank);
        s.same_shape = A.shape == B.shape;
        s.kind = K_ADD;
        s.in = {a, b};
        s.out = {make_out(o.outputs[0], dt, out)};
    }

    void pool_common(const fb::Operator& o, Step& s, const char* op, const Tensor& X) {
        expect_rank(op, "input", X, 4);
        const Attr& a = o.attr;
        if (a.pad.size() != 4 || a.kernel.size() != 2 || a.stride.size() != 2)
            raise(TB_ERR_GRAPH, "%s: pad must have 4 elements, kernel and stride 2", op);
        tb_pool2d_desc& d = s.pool;
        d.n = static_cast<int32_t>(X.shape[0]);
        d.ih = static_cast<int32_t>(X.shape[1]);
        d.iw = static_cast<int32_t>(X.shape[2]);
        d.c = static_cast<int32_t>(X.shape[3]);
        for (int i = 0; i < 2; ++i) { d.kernel[i] = a.kernel[i]; d.stride[i] = a.stride[i]; }
        for (int i = 0; i < 4; ++i) d.pad[i] = a.pad[i];
        d.dtype = X.dtype;
    }

    void c_avgpool(const fb::Operator& o, Step& s) {
        const char* op = "AVG_POOL2D";
        if (o.attr.type != fb::OP_AVG_POOL2D) raise(TB_ERR_GRAPH, "%s: missing attribute", op);
        expect_operands(o, op, 3, 1);
        const int x = get(o.inputs[0]);
        const Tensor& iz = single(op, "input_zp", get(o.inputs[1]));
        const Tensor& oz = single(op, "output_zp", get(o.inputs[2]));
        const Tensor& X = T(x);
        pool_common(o, s, op, X);
        int oh = 0, ow = 0;
        tb_status st = pool_check(op, &s.pool, &oh, &ow);
        if (st != TB_OK) raise(st, "%s", tb_last_error());
        const std::vector<int64_t> out = {X.shape[0], oh, ow, X.shape[3]};
        const int decl = declared(op, o.outputs[0], out);
        if (decl && decl != X.dtype) raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype must match input dtype", op);
        const int dt = X.dtype, at = o.attr.acc_type;
        const bool sup = ((dt == TB_DT_INT8 || dt == TB_DT_INT16) && at == TB_DT_INT32) ||
                         (dt == TB_DT_FP16 && (at == TB_DT_FP16 || at == TB_DT_FP32)) ||
                         ((dt == TB_DT_BF16 || dt == TB_DT_FP32) && at == TB_DT_FP32) ||
                         ((dt == TB_DT_FP8E4M3 || dt == TB_DT_FP8E5M2) && at == TB_DT_FP16);
        if (!sup) raise(TB_ERR_DTYPE_MISMATCH, "%s: unsupported types input=%d acc=%d", op, dt, at);
        if (iz.dtype != dt || oz.dtype != dt) raise(TB_ERR_DTYPE_MISMATCH, "%s: zero points must have the input dtype", op);
        if (is_int_dt(dt)) {
            s.pool.input_zp = static_cast<int32_t>(ival(iz));
            s.pool.output_zp = static_cast<int32_t>(ival(oz));
            if (dt != TB_DT_INT8 && (s.pool.input_zp != 0 || s.pool.output_zp != 0))
                raise(TB_ERR_GRAPH, "%s: zero points must be zero for non-int8 data", op);
        } else {
            if ((!iz.hf.empty() && iz.hf[0] != 0.f) || (!oz.hf.empty() && oz.hf[0] != 0.f))
                raise(TB_ERR_GRAPH, "%s: zero points must be zero for float data", op);
        }
        s.pool.acc_dtype = at;
        s.kind = K_AVGPOOL;
        s.in = {x, get(o.inputs[1]), get(o.inputs[2])};
        s.out = {make_out(o.outputs[0], dt, out)};
    }

    void c_maxpool(const fb::Operator& o, Step& s) {
        const char* op = "MAX_POOL2D";
        if (o.attr.type != fb::OP_MAX_POOL2D) raise(TB_ERR_GRAPH, "%s: missing attribute", op);
        expect_operands(o, op, 1, 1);
        if (o.attr.nan_mode != TB_NAN_PROPAGATE && o.attr.nan_mode != TB_NAN_IGNORE)
            raise(TB_ERR_GRAPH, "%s: nan_mode must be PROPAGATE or IGNORE", op);
        const int x = get(o.inputs[0]);
        const Tensor& X = T(x);
        pool_common(o, s, op, X);
        int oh = 0, ow = 0;
        tb_status st = pool_check(op, &s.pool, &oh, &ow);
        if (st != TB_OK) raise(st, "%s", tb_last_error());
        const std::vector<int64_t> out = {X.shape[0], oh, ow, X.shape[3]};
        const int dt = X.dtype;
        const int decl = declared(op, o.outputs[0], out);
        if (decl && decl != dt) raise(TB_ERR_DTYPE_MISMATCH, "%s: output dtype must match input dtype", op);
        if (!(dt == TB_DT_INT8 || dt == TB_DT_INT16 || dt == TB_DT_FP16 || dt == TB_DT_BF16 || dt == TB_DT_FP32 ||
              dt == TB_DT_FP8E4M3 || dt == TB_DT_FP8E5M2))
            raise(TB_ERR_DTYPE_MISMATCH, "%s: unsupported dtype", op);
        s.pool.nan_mode = o.attr.nan_mode;
        s.kind = K_MAXPOOL;
        s.in = {x};
        s.out = {make_out(o.outputs[0], dt, out)};
    }

    void compile_op(int idx) {
        const fb::Operator& o = G.block->operators[idx];
        Step& s = G.steps[idx];
        s.op_index = idx;
        s.op = o.op;
        switch (o.op) {
        case fb::OP_CONST: case fb::OP_CONST_SHAPE: c_const(o, s); break;
        case fb::OP_IDENTITY: c_identity(o, s); break;
        case fb::OP_RESHAPE: c_reshape(o, s); break;
        case fb::OP_TRANSPOSE: c_transpose(o, s); break;
        case fb::OP_CONV2D: c_conv(o, s, false); break;
        case fb::OP_DEPTHWISE_CONV2D: c_conv(o, s, true); break;
        case fb::OP_TRANSPOSE_CONV2D: c_conv(o, s, false, true); break;
        case fb::OP_CONV3D: c_conv3d(o, s); break;
        case fb::OP_MATMUL: c_matmul(o, s, false); break;
        case fb::OP_MATMUL_T: c_matmul(o, s, true); break;
        case fb::OP_RESCALE: c_rescale(o, s); break;
        case fb::OP_CLAMP: c_clamp(o, s); break;
        case fb::OP_ADD: c_add(o, s); break;
        case fb::OP_AVG_POOL2D: c_avgpool(o, s); break;
        case fb::OP_MAX_POOL2D: c_maxpool(o, s); break;
        default: raise(TB_ERR_UNSUPPORTED_OP, "%d", o.op);
        }
    }

    tb_graph& G;
};

// The reference's execution order (src/interpreter.rs:175-231): a FIFO of
// ready operators, seeded in index order; after each operator, every
// not-yet-executed operator that became ready is appended in index order.
void ready_order(const fb::Block& b, const std::vector<std::string>& available_names, std::vector<int>* order,
                 std::vector<int>* left) {
    const int n = static_cast<int>(b.operators.size());
    std::unordered_map<std::string, int> idx;
    auto id_of = [&](const std::string& s) {
        auto it = idx.find(s);
        if (it != idx.end()) return it->second;
        const int k = static_cast<int>(idx.size());
        idx.emplace(s, k);
        return k;
    };
    std::vector<std::vector<int>> ins(n), outs(n);
    for (int i = 0; i < n; ++i) {
        for (const auto& s : b.operators[i].inputs) ins[i].push_back(id_of(s));
        for (const auto& s : b.operators[i].outputs) outs[i].push_back(id_of(s));
    }
    std::vector<int> avail_ids;
    for (const auto& s : available_names) avail_ids.push_back(id_of(s));
    const int n_names = static_cast<int>(idx.size());
    std::vector<char> avail(n_names, 0);
    for (int k : avail_ids) avail[k] = 1;
    // consumers of each tensor, to update only the operators a new tensor can make ready
    std::vector<std::vector<int>> consumers(n_names);
    for (int i = 0; i < n; ++i)
        for (int t : ins[i]) consumers[t].push_back(i);
    std::vector<int> missing(n, 0);  // input listings not yet available (CONST: always ready)
    for (int i = 0; i < n; ++i) {
        if (b.operators[i].op == fb::OP_CONST) continue;
        for (int t : ins[i]) missing[i] += !avail[t];
    }
    std::vector<char> executed(n, 0), queued(n, 0);
    std::deque<int> q;
    for (int i = 0; i < n; ++i)
        if (missing[i] == 0) { q.push_back(i); queued[i] = 1; }
    while (!q.empty()) {
        const int i = q.front();
        q.pop_front();
        queued[i] = 0;
        if (executed[i]) continue;
        executed[i] = 1;
        order->push_back(i);
        for (int t : outs[i]) {
            if (avail[t]) continue;
            avail[t] = 1;
            for (int c : consumers[t])
                if (b.operators[c].op != fb::OP_CONST) missing[c] -= 1;  // one per listing of t
        }
        // append, in index order, every operator that is ready, not executed and not queued
        for (int c = 0; c < n; ++c)
            if (!executed[c] && !queued[c] && missing[c] <= 0) { q.push_back(c); queued[c] = 1; }
    }
    for (int i = 0; i < n; ++i)
        if (!executed[i]) left->push_back(i);
}

// Count consumers of each tensor name among the block's operators.
std::unordered_map<std::string, int> consumer_counts(const fb::Block& b) {
    std::unordered_map<std::string, int> c;
    for (const auto& o : b.operators)
        for (const auto& s : o.inputs) c[s]++;
    return c;
}

tb_status do_compile(tb_graph* G) {
    G->release();
    const fb::Block& b = *G->block;
    G->steps.assign(b.operators.size(), Step());
    std::vector<std::string> names;
    for (auto& kv : G->inputs) names.push_back(kv.first);
    std::sort(names.begin(), names.end());
    ready_order(b, names, &G->order, &G->unexecuted);
    Compiler C(G);
    // every tensor is created once: reserve so references into the table stay valid
    size_t n_tensors = names.size() + 1;
    for (const auto& o : b.operators) n_tensors += o.outputs.size();
    G->tensors.reserve(n_tensors);
    for (const auto& name : names) {
        const tb_graph::Bound& in = G->inputs[name];
        Tensor t;
        t.name = name;
        t.dtype = in.dtype;
        t.shape = in.shape;
        t.count = 1;
        for (int64_t v : t.shape) t.count *= v;
        t.dev = in.dev;
        C.add_tensor(std::move(t));
    }
    G->stop_at = -1;
    for (size_t k = 0; k < G->order.size(); ++k) {
        const int idx = G->order[k];
        try {
            C.compile_op(idx);
        } catch (const StatusError& e) {
            G->steps[idx].status = e.st;
            G->steps[idx].err = e.msg;
            G->stop_at = static_cast<int>(k);
            break;
        }
    }
    const size_t n_ok = G->stop_at < 0 ? G->order.size() : static_cast<size_t>(G->stop_at);

    // ---- fusion ------------------------------------------------------------------------
    tb_context* ctx = G->ctx;
    auto cons = consumer_counts(b);
    std::unordered_map<std::string, bool> is_block_out;
    for (const auto& s : b.outputs) is_block_out[s] = true;
    auto private_to = [&](int tensor_id) {
        const std::string& nm = G->tensors[tensor_id].name;
        return cons[nm] == 1 && !is_block_out.count(nm);
    };
    std::unordered_map<int, int> producer;  // tensor id -> op index
    std::unordered_map<int, int> consumer_op;  // tensor id -> the single consuming op index (compiled ones)
    for (size_t k = 0; k < n_ok; ++k) {
        const Step& s = G->steps[G->order[k]];
        for (int t : s.out) producer[t] = s.op_index;
        for (size_t j = 0; j < s.in.size(); ++j) consumer_op[s.in[j]] = s.op_index;
    }
    auto pos_of = [&](int op_index) {
        for (size_t k = 0; k < n_ok; ++k)
            if (G->order[k] == op_index) return static_cast<int>(k);
        return -1;
    };
    const bool fuse = !(G->flags & TB_GRAPH_NO_FUSION);
    if (fuse) {
        for (size_t k = 0; k < n_ok; ++k) {
            Step& s = G->steps[G->order[k]];
            // contraction (int32 result) -> RESCALE [-> CLAMP]
            if ((s.kind == K_CONV || s.kind == K_MATMUL) && G->tensors[s.out[0]].dtype == TB_DT_INT32 &&
                private_to(s.out[0])) {
                auto it = consumer_op.find(s.out[0]);
                if (it == consumer_op.end()) continue;
                Step& r = G->steps[it->second];
                if (r.kind != K_RESCALE || r.in[0] != s.out[0] || pos_of(r.op_index) < 0) continue;
                if (s.kind == K_MATMUL && (s.mdesc.a_dtype != TB_DT_INT8)) continue;
                if (s.kind == K_CONV && s.cdesc.in_dtype != TB_DT_INT8) continue;
                s.has_rescale = true;
                s.rattr = r.rattr;
                s.rmult = r.rmult;
                s.rshift = r.rshift;
                s.rattr.multiplier = s.rmult.data();
                s.rattr.shift = s.rshift.data();
                r.kind = K_FUSED;
                s.group.push_back(r.op_index);
                G->tensors[s.out[0]].materialized = false;
                s.exec_out = r.out[0];
                // CLAMP of the RESCALE result
                if (private_to(r.out[0]) && !s.rattr.output_unsigned) {
                    auto ic = consumer_op.find(r.out[0]);
                    if (ic != consumer_op.end()) {
                        Step& c = G->steps[ic->second];
                        if (c.kind == K_CLAMP && pos_of(c.op_index) >= 0 && is_int_dt(G->tensors[c.in[0]].dtype)) {
                            s.rattr.clamp_enabled = 1;
                            s.rattr.clamp_min = static_cast<int32_t>(c.cmin_i);
                            s.rattr.clamp_max = static_cast<int32_t>(c.cmax_i);
                            c.kind = K_FUSED;
                            s.group.push_back(c.op_index);
                            G->tensors[r.out[0]].materialized = false;
                            s.exec_out = c.out[0];
                        }
                    }
                }
            }
            // residual chain: ADD(int32) of two RESCALEs (8/16-bit -> int32) of equal shapes, then RESCALE [-> CLAMP]
            if (s.kind == K_ADD && G->tensors[s.out[0]].dtype == TB_DT_INT32 && s.same_shape && private_to(s.out[0])) {
                auto pa = producer.find(s.in[0]);
                auto pb = producer.find(s.in[1]);
                auto po = consumer_op.find(s.out[0]);
                if (pa == producer.end() || pb == producer.end() || po == consumer_op.end()) continue;
                Step& ra = G->steps[pa->second];
                Step& rb = G->steps[pb->second];
                Step& ro = G->steps[po->second];
                if (ra.kind != K_RESCALE || rb.kind != K_RESCALE || ro.kind != K_RESCALE || &ra == &rb) continue;
                if (!private_to(ra.out[0]) || !private_to(rb.out[0]) || ro.in[0] != s.out[0]) continue;
                if (ra.in_dtype == TB_DT_INT32 || rb.in_dtype == TB_DT_INT32) continue;
                // the chain runs where the ADD runs: both RESCALE inputs exist by then
                s.kind = K_RESIDUAL;
                s.ra.enabled = false;
                s.rattr = ro.rattr;
                s.rmult = ro.rmult;
                s.rshift = ro.rshift;
                s.rattr.multiplier = s.rmult.data();
                s.rattr.shift = s.rshift.data();
                s.in_dtype = ra.in_dtype; s.in_uns = ra.in_uns; s.izp = ra.izp;
                s.b_dtype = rb.in_dtype; s.b_uns = rb.in_uns; s.bzp = rb.izp;
                s.channels = ro.channels;
                // borrow the members' attributes (plans are built below)
                s.group = {ra.op_index, rb.op_index, ro.op_index};
                ra.kind = rb.kind = ro.kind = K_FUSED;
                G->tensors[ra.out[0]].materialized = false;
                G->tensors[rb.out[0]].materialized = false;
                G->tensors[s.out[0]].materialized = false;
                s.exec_out = ro.out[0];
                if (private_to(ro.out[0]) && !s.rattr.output_unsigned) {
                    auto ic = consumer_op.find(ro.out[0]);
                    if (ic != consumer_op.end()) {
                        Step& c = G->steps[ic->second];
                        if (c.kind == K_CLAMP && pos_of(c.op_index) >= 0 && is_int_dt(G->tensors[c.in[0]].dtype)) {
                            s.rattr.clamp_enabled = 1;
                            s.rattr.clamp_min = static_cast<int32_t>(c.cmin_i);
                            s.rattr.clamp_max = static_cast<int32_t>(c.cmax_i);
                            c.kind = K_FUSED;
                            s.group.push_back(c.op_index);
                            G->tensors[ro.out[0]].materialized = false;
                            s.exec_out = c.out[0];
                        }
                    }
                }
            }
        }
    }

    // ---- device buffers ----------------------------------------------------------------
    // aliases (RESHAPE, IDENTITY) share their source's buffer
    for (size_t id = 0; id < G->tensors.size(); ++id) {
        Tensor& t = G->tensors[id];
        if (t.dev || !t.materialized) continue;
        auto al = C.alias_of.find(static_cast<int>(id));
        if (al != C.alias_of.end()) continue;
        const size_t bytes = std::max<size_t>(t.dev_bytes(), 16);
        void* p = nullptr;
        if (++G->allocs == G->fault_alloc)
            return fail(TB_ERR_CUDA, "graph buffer allocation (%zu bytes) failed: injected by TB_FAULT_ALLOC_FAIL", bytes);
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return fail(TB_ERR_CUDA, "graph buffer allocation (%zu bytes) failed: %s", bytes,
                                          cudaGetErrorString(e));
        G->buffers.push_back(p);
        t.dev = p;
        t.owned = true;
    }
    for (size_t id = 0; id < G->tensors.size(); ++id) {
        auto al = C.alias_of.find(static_cast<int>(id));
        if (al == C.alias_of.end()) continue;
        int src = al->second;
        while (C.alias_of.count(src)) src = C.alias_of[src];
        G->tensors[id].dev = G->tensors[src].dev;
        G->tensors[id].materialized = G->tensors[src].materialized;
    }
    for (auto& up : C.uploads) {
        Tensor& t = G->tensors[up.first];
        if (!up.second.empty()) {
            cudaError_t e = cudaMemcpy(t.dev, up.second.data(), up.second.size(), cudaMemcpyHostToDevice);
            if (e != cudaSuccess) return fail(TB_ERR_CUDA, "constant upload failed: %s", cudaGetErrorString(e));
        }
    }

    // ---- plans -------------------------------------------------------------------------
    for (size_t k = 0; k < n_ok; ++k) {
        Step& s = G->steps[G->order[k]];
        tb_status st = TB_OK;
        switch (s.kind) {
        case K_CONV: {
            const Tensor& W = G->tensors[s.in[1]];
            const Tensor& B = G->tensors[s.in[2]];
            if (s.conv3d)
                st = tb_conv3d_plan_create(ctx, &s.c3desc, W.dev, B.dev, nullptr, &s.conv);
            else if (s.transpose)
                st = tb_transpose_conv2d_plan_create(ctx, &s.cdesc, W.dev, B.dev, s.has_rescale ? &s.rattr : nullptr,
                                                     &s.conv);
            else if (s.depthwise)
                st = tb_depthwise_conv2d_plan_create(ctx, &s.cdesc, W.dev, B.dev, s.has_rescale ? &s.rattr : nullptr,
                                                     &s.conv);
            else
                st = tb_conv2d_plan_create(ctx, &s.cdesc, W.dev, B.dev, s.has_rescale ? &s.rattr : nullptr, &s.conv);
            break;
        }
        case K_MATMUL:
            st = s.mt_batch ? tb_matmul_t_plan_create(ctx, &s.mdesc, s.mt_batch, s.has_rescale ? &s.rattr : nullptr, &s.mm)
                            : tb_matmul_plan_create(ctx, &s.mdesc, s.has_rescale ? &s.rattr : nullptr, &s.mm);
            if (st == TB_OK && G->tensors[s.in[1]].is_static && G->tensors[s.in[1]].dev != nullptr)
                st = tb_matmul_plan_set_constant_b(s.mm, G->tensors[s.in[1]].dev, nullptr);  // e.g. FC weights
            break;
        case K_RESCALE:
            st = make_rescale_plan(ctx, &s.rattr, s.in_dtype, s.channels, &s.rs);
            break;
        case K_RESIDUAL: {
            const Step& a = G->steps[s.group[0]];
            const Step& bb = G->steps[s.group[1]];
            st = make_rescale_plan(ctx, &a.rattr, a.in_dtype, a.channels, &s.ra);
            if (st == TB_OK) st = make_rescale_plan(ctx, &bb.rattr, bb.in_dtype, bb.channels, &s.rb);
            if (st == TB_OK) st = make_rescale_plan(ctx, &s.rattr, TB_DT_INT32, s.channels, &s.rs);
            residual_fast_constants(a.rattr, a.in_dtype, bb.rattr, bb.in_dtype, s.rattr, &s.rfast);
            if (st == TB_OK) st = make_residual_table(s.rattr, s.rs, &s.rfast);
            break;
        }
        default: break;
        }
        if (st != TB_OK) {
            // a plan that cannot be built: the error belongs to this operator
            s.status = st;
            s.err = tb_last_error();
            G->stop_at = static_cast<int>(k);
            break;
        }
    }
    G->compiled = true;
    return TB_OK;
}

void fill_info(const Tensor& t, tb_tensor_info* info) {
    info->name = t.name.c_str();
    info->dtype = t.dtype;
    info->rank = static_cast<int32_t>(t.shape.size());
    info->shape = t.shape.data();
    info->bytes = static_cast<uint64_t>(t.ref_bytes());
    info->data = t.materialized ? t.dev : nullptr;
}

tb_status exec_step(tb_graph* G, Step& s, cudaStream_t st) {
    tb_context* ctx = G->ctx;
    auto dev = [&](int id) { return G->tensors[id].dev; };
    switch (s.kind) {
    case K_CONST: case K_ALIAS: case K_FUSED: case K_NONE: return TB_OK;
    case K_TRANSPOSE: {
        const Tensor& x = G->tensors[s.in[0]];
        return launch_transpose(ctx, x.dev, dev(s.out[0]), dev_elem_bytes(x.dtype), G->tensors[s.out[0]].count, s.rank,
                                s.map, st);
    }
    case K_CONV: {
        void* out = dev(s.exec_out >= 0 ? s.exec_out : s.out[0]);
        return tb_conv2d_plan_run(s.conv, dev(s.in[0]), out, st);
    }
    case K_MATMUL: {
        void* out = dev(s.exec_out >= 0 ? s.exec_out : s.out[0]);
        return tb_matmul_plan_run(s.mm, dev(s.in[0]), dev(s.in[1]), out, st);
    }
    case K_RESCALE: {
        const Tensor& x = G->tensors[s.in[0]];
        return launch_rescale(ctx, s.rs, s.in_dtype, s.in_uns, s.izp, x.dev, x.count, s.channels, dev(s.out[0]), st);
    }
    case K_RESIDUAL: {
        const Step& ra = G->steps[s.group[0]];
        const Step& rb = G->steps[s.group[1]];
        const Tensor& a = G->tensors[ra.in[0]];
        const Tensor& b = G->tensors[rb.in[0]];
        return launch_residual(ctx, a.dev, s.in_dtype, s.in_uns, s.izp, s.ra, b.dev, s.b_dtype, s.b_uns, s.bzp, s.rb,
                               s.rs, s.rfast, a.count, s.channels, dev(s.exec_out), st);
    }
    case K_CLAMP: {
        const Tensor& x = G->tensors[s.in[0]];
        return tb_clamp(ctx, x.dtype, x.dev, x.count, s.cmin_i, s.cmax_i, s.cmin_f, s.cmax_f, s.nan_mode,
                        dev(s.out[0]), st);
    }
    case K_ADD: {
        const Tensor& a = G->tensors[s.in[0]];
        if (s.same_shape) return tb_add(ctx, a.dtype, a.dev, dev(s.in[1]), a.count, dev(s.out[0]), st);
        return launch_add_broadcast(ctx, a.dtype, a.dev, dev(s.in[1]), G->tensors[s.out[0]].count, s.rank, s.map,
                                    dev(s.out[0]), st);
    }
    case K_AVGPOOL: return tb_avg_pool2d(ctx, &s.pool, dev(s.in[0]), dev(s.out[0]), st);
    case K_MAXPOOL: return tb_max_pool2d(ctx, &s.pool, dev(s.in[0]), dev(s.out[0]), st);
    default: return fail(TB_ERR_INVALID_ARGUMENT, "internal: unknown step kind %d", s.kind);
    }
}

struct HookCtx {
    std::vector<tb_tensor_info> ins, outs;
};

void gather(tb_graph* G, const fb::Operator& o, std::vector<tb_tensor_info>* v, bool outputs) {
    v->clear();
    const auto& names = outputs ? o.outputs : o.inputs;
    for (const auto& nm : names) {
        auto it = G->tid.find(nm);
        if (it == G->tid.end()) continue;  // the reference skips names it cannot find
        tb_tensor_info ti;
        fill_info(G->tensors[it->second], &ti);
        v->push_back(ti);
    }
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================

extern "C" TB_API tb_status tb_graph_load(tb_context* ctx, const void* data, size_t len, uint32_t flags,
                                          tb_graph** out) {
    if (!ctx || !data || !out) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    std::unique_ptr<tb_graph> g(new tb_graph);
    g->ctx = ctx;
    g->flags = flags;
    if (const char* ev = std::getenv("TB_FAULT_ALLOC_FAIL")) g->fault_alloc = std::max(0, std::atoi(ev));
    std::string err;
    if (!fb::parse_graph(static_cast<const uint8_t*>(data), len, &g->g, &err))
        return fail(TB_ERR_DESERIALIZE, "%s", err.c_str());
    g->block = g->g.main_block();
    if (!g->block) return fail(TB_ERR_GRAPH, "no main block found");
    for (const auto& op : g->block->operators)
        if (!runner_supports(op.op))
            return fail(TB_ERR_UNSUPPORTED_OP, "operator code %d is not run by this backend (it stays on the reference path)",
                        op.op);
    for (const auto& t : g->block->tensors) {
        if (t.dtype != TB_DT_SHAPE && t.shape.size() > 6)
            return fail(TB_ERR_SHAPE_MISMATCH, "tensor '%s' has rank %zu, above the maximum of 6", t.name.c_str(),
                        t.shape.size());
        g->defs.emplace(t.name, &t);
    }
    *out = g.release();
    return TB_OK;
}

extern "C" TB_API void tb_graph_destroy(tb_graph* g) {
    if (!g) return;
    cudaSetDevice(g->ctx->device);
    cudaDeviceSynchronize();
    for (auto& kv : g->inputs)
        if (kv.second.owned && kv.second.dev) cudaFree(kv.second.dev);
    delete g;
}

extern "C" TB_API int32_t tb_graph_num_inputs(const tb_graph* g) {
    return g ? static_cast<int32_t>(g->block->inputs.size()) : 0;
}
extern "C" TB_API int32_t tb_graph_num_outputs(const tb_graph* g) {
    return g ? static_cast<int32_t>(g->block->outputs.size()) : 0;
}

static thread_local std::vector<int64_t> g_info_shape;

static tb_status decl_info(const tb_graph* g, const std::string& name, tb_tensor_info* info) {
    auto it = g->defs.find(name);
    g_info_shape.clear();
    info->name = name.c_str();
    info->data = nullptr;
    if (it == g->defs.end()) {
        info->dtype = 0;
        info->rank = 0;
        info->shape = nullptr;
        info->bytes = 0;
        return TB_OK;
    }
    const fb::TensorDef* d = it->second;
    int64_t n = 1;
    for (int v : d->shape) {
        g_info_shape.push_back(v);
        n *= std::max(v, 0);
    }
    info->dtype = d->dtype;
    info->rank = static_cast<int32_t>(d->shape.size());
    info->shape = g_info_shape.data();
    info->bytes = static_cast<uint64_t>(std::max<int64_t>(n, 1) * ref_elem_bytes(d->dtype));
    return TB_OK;
}

extern "C" TB_API tb_status tb_graph_input_info(const tb_graph* g, int32_t i, tb_tensor_info* info) {
    if (!g || !info || i < 0 || i >= static_cast<int32_t>(g->block->inputs.size()))
        return fail(TB_ERR_INVALID_ARGUMENT, "bad input index");
    return decl_info(g, g->block->inputs[i], info);
}

extern "C" TB_API tb_status tb_graph_output_info(const tb_graph* g, int32_t i, tb_tensor_info* info) {
    if (!g || !info || i < 0 || i >= static_cast<int32_t>(g->block->outputs.size()))
        return fail(TB_ERR_INVALID_ARGUMENT, "bad output index");
    return decl_info(g, g->block->outputs[i], info);
}

extern "C" TB_API tb_status tb_graph_set_input(tb_graph* g, const char* name, int32_t dtype, const int64_t* shape,
                                               int32_t rank, const void* data, uint64_t bytes, int32_t on_device,
                                               void* stream) {
    if (!g || !name || (rank > 0 && !shape) || rank < 0) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    TB_CUDA(cudaSetDevice(g->ctx->device));
    std::vector<int64_t> sh(shape, shape + rank);
    int64_t n = 1;
    for (int64_t v : sh) {
        if (v < 0) return fail(TB_ERR_SHAPE_MISMATCH, "input '%s': negative dimension", name);
        n *= v;
    }
    const size_t need = static_cast<size_t>(n) * dev_elem_bytes(dtype);
    if (ref_elem_bytes(dtype) == 0) return fail(TB_ERR_DTYPE_MISMATCH, "input '%s': unknown dtype %d", name, dtype);
    if (bytes < need) return fail(TB_ERR_INVALID_ARGUMENT, "input '%s' needs %zu bytes, got %llu", name, need,
                                  static_cast<unsigned long long>(bytes));
    auto& b = g->inputs[name];
    const bool same_sig = b.dtype == dtype && b.shape == sh && ((b.owned && !on_device) || (!b.owned && on_device && b.dev == data));
    if (!same_sig) g->compiled = false;  // recompile for new shapes or buffers
    if (on_device) {
        if (b.owned && b.dev) cudaFree(b.dev);
        b.owned = false;
        b.cap = 0;
        b.dev = const_cast<void*>(data);
    } else {
        if (!b.owned || b.cap < std::max<size_t>(need, 16)) {
            if (b.owned && b.dev) cudaFree(b.dev);
            b.dev = nullptr;
            TB_CUDA(cudaMalloc(&b.dev, std::max<size_t>(need, 16)));
            b.cap = std::max<size_t>(need, 16);
            b.owned = true;
            g->compiled = false;
        }
        if (need) TB_CUDA(cudaMemcpyAsync(b.dev, data, need, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
        TB_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    }
    b.dtype = dtype;
    b.shape = sh;
    return TB_OK;
}

extern "C" TB_API tb_status tb_graph_run(tb_graph* g, const tb_hooks* hooks, void* stream_) {
    if (!g) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    tb_context* ctx = g->ctx;
    TB_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream_);
    if (!g->compiled) {
        tb_status s = do_compile(g);
        if (s != TB_OK) return s;
    }
    const uint64_t launches0 = ctx->launches;
    const fb::Block& b = *g->block;
    const size_t n_run = g->stop_at < 0 ? g->order.size() : static_cast<size_t>(g->stop_at) + 1;
    const bool use_graph = (g->flags & TB_GRAPH_CUDA_GRAPH) && g->stop_at < 0;
    HookCtx hc;
    std::vector<int> timed_ops;
    if (g->flags & TB_GRAPH_TIME_OPS) {
        if (use_graph) return fail(TB_ERR_INVALID_ARGUMENT, "TB_GRAPH_TIME_OPS and TB_GRAPH_CUDA_GRAPH exclude each other");
        const size_t need = 2 * b.operators.size();
        while (g->op_events.size() < need) {
            cudaEvent_t e;
            TB_CUDA(cudaEventCreate(&e));
            g->op_events.push_back(e);
        }
        g->op_ms.assign(b.operators.size(), -1.f);
    }

    // Launch everything first when a CUDA graph replays the run; hooks then follow in order.
    if (use_graph) {
        if (!st) return fail(TB_ERR_INVALID_ARGUMENT, "TB_GRAPH_CUDA_GRAPH needs a non-default stream");
        if (!g->cexec) {
            TB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            tb_status s = TB_OK;
            for (size_t k = 0; k < g->order.size() && s == TB_OK; ++k) s = exec_step(g, g->steps[g->order[k]], st);
            cudaGraph_t graph = nullptr;
            cudaError_t ce = cudaStreamEndCapture(st, &graph);
            if (s != TB_OK) {
                if (graph) cudaGraphDestroy(graph);
                return s;
            }
            if (ce != cudaSuccess) return fail(TB_ERR_CUDA, "stream capture of the graph failed: %s", cudaGetErrorString(ce));
            g->cgraph = graph;
            ce = cudaGraphInstantiate(&g->cexec, graph, 0);
            if (ce != cudaSuccess) return fail(TB_ERR_CUDA, "cudaGraphInstantiate failed: %s", cudaGetErrorString(ce));
            g->graph_launches = ctx->launches - launches0;
        }
        TB_CUDA(cudaGraphLaunch(g->cexec, st));
    }
    for (size_t k = 0; k < n_run; ++k) {
        Step& s = g->steps[g->order[k]];
        const fb::Operator& o = b.operators[s.op_index];
        tb_op_info info{o.op, s.op_index};
        if (hooks && hooks->pre_op) {
            gather(g, o, &hc.ins, false);
            hooks->pre_op(hooks->user, &info, hc.ins.data(), static_cast<int32_t>(hc.ins.size()));
        }
        if (s.status != TB_OK) {
            cudaStreamSynchronize(st);
            g->last_launches = ctx->launches - launches0;
            return fail(s.status, "%s", s.err.c_str());
        }
        if (!use_graph) {
            const bool timed = (g->flags & TB_GRAPH_TIME_OPS) && s.kind != K_CONST && s.kind != K_ALIAS &&
                               s.kind != K_FUSED && s.kind != K_NONE;
            if (timed) TB_CUDA(cudaEventRecord(g->op_events[2 * s.op_index], st));
            tb_status r = exec_step(g, s, st);
            if (r != TB_OK) return r;
            if (timed) {
                TB_CUDA(cudaEventRecord(g->op_events[2 * s.op_index + 1], st));
                timed_ops.push_back(s.op_index);
            }
            if (g->flags & TB_GRAPH_SYNC_EACH_OP) TB_CUDA(cudaStreamSynchronize(st));
        }
        if (hooks && (hooks->on_tensor_alloc || hooks->post_op)) {
            gather(g, o, &hc.outs, true);
            if (hooks->on_tensor_alloc)
                for (const auto& t : hc.outs)
                    hooks->on_tensor_alloc(hooks->user, t.name, t.shape, t.rank, t.dtype, t.bytes);
            if (hooks->post_op) {
                gather(g, o, &hc.ins, false);
                hooks->post_op(hooks->user, &info, hc.ins.data(), static_cast<int32_t>(hc.ins.size()), hc.outs.data(),
                               static_cast<int32_t>(hc.outs.size()));
            }
        }
    }
    g->last_launches = use_graph ? g->graph_launches : ctx->launches - launches0;
    if (!timed_ops.empty()) {
        TB_CUDA(cudaStreamSynchronize(st));
        for (int i : timed_ops)
            TB_CUDA(cudaEventElapsedTime(&g->op_ms[i], g->op_events[2 * i], g->op_events[2 * i + 1]));
    }
    if (!g->unexecuted.empty()) {
        std::string names = "[";
        for (size_t i = 0; i < g->unexecuted.size(); ++i)
            names += std::string(i ? ", \"" : "\"") + op_name(b.operators[g->unexecuted[i]].op) + "\"";
        names += "]";
        cudaStreamSynchronize(st);
        return fail(TB_ERR_GRAPH, "could not execute all ops, stuck on: %s", names.c_str());
    }
    return tb_synchronize(ctx, stream_);
}

extern "C" TB_API tb_status tb_graph_get_output(tb_graph* g, const char* name, tb_tensor_info* info) {
    if (!g || !name || !info) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    auto it = g->tid.find(name);
    if (!g->compiled || it == g->tid.end()) return fail(TB_ERR_TENSOR_NOT_FOUND, "%s", name);
    fill_info(g->tensors[it->second], info);
    return TB_OK;
}

extern "C" TB_API tb_status tb_graph_read_output(tb_graph* g, const char* name, void* dst, uint64_t bytes,
                                                 void* stream) {
    if (!g || !name || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    auto it = g->tid.find(name);
    if (!g->compiled || it == g->tid.end()) return fail(TB_ERR_TENSOR_NOT_FOUND, "%s", name);
    const Tensor& t = g->tensors[it->second];
    if (!t.materialized || !t.dev) return fail(TB_ERR_TENSOR_NOT_FOUND, "%s was fused away", name);
    const size_t need = t.dev_bytes();
    if (bytes < need) return fail(TB_ERR_INVALID_ARGUMENT, "output '%s' needs %zu bytes", name, need);
    if (need) {
        TB_CUDA(cudaMemcpyAsync(dst, t.dev, need, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
        TB_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    }
    return TB_OK;
}

extern "C" TB_API uint64_t tb_graph_last_launches(const tb_graph* g) { return g ? g->last_launches : 0; }

extern "C" TB_API float tb_graph_op_time_ms(const tb_graph* g, int32_t op_index) {
    if (!g || op_index < 0 || static_cast<size_t>(op_index) >= g->op_ms.size()) return -1.f;
    return g->op_ms[op_index];
}
