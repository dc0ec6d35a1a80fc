// Protobuf wire-format decoder for mlvc.wire.Graph (proto/mlvc_model.proto:30-83)
// with the validation rules of the reference loader
// (runtime/src/aot_graph.cpp:110-283), written without libprotobuf: the
// schema is small (varints, length-delimited submessages, packed repeated
// scalars, one fixed32 float) and the deployment image has no protobuf C++
// runtime.
#include "graph.hpp"

#include <cmath>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <unordered_set>

namespace mlvc_b200 {
namespace {

[[noreturn]] void invalid(const char* what)
{
    throw std::runtime_error(std::string("invalid AOT graph: ") + what);
}

inline void require(bool ok, const char* what)
{
    if (!ok)
        invalid(what);
}

class Wire {
public:
    Wire(const uint8_t* b, const uint8_t* e) : p_(b), e_(e) {}
    bool more() const { return p_ < e_; }

    uint64_t varint()
    {
        uint64_t v = 0;
        for (int s = 0; s < 64; s += 7) {
            require(p_ < e_, "truncated varint");
            const uint8_t b = *p_++;
            v |= static_cast<uint64_t>(b & 0x7fu) << s;
            if (!(b & 0x80u))
                return v;
        }
        invalid("overlong varint");
    }

    Wire message()
    {
        const uint64_t n = varint();
        require(n <= static_cast<uint64_t>(e_ - p_), "truncated field");
        Wire w(p_, p_ + n);
        p_ += n;
        return w;
    }

    std::string bytes()
    {
        Wire w = message();
        return std::string(reinterpret_cast<const char*>(w.p_), w.e_ - w.p_);
    }

    uint32_t fixed32()
    {
        require(e_ - p_ >= 4, "truncated fixed32");
        uint32_t v;
        std::memcpy(&v, p_, 4);
        p_ += 4;
        return v;
    }

    void skip(int wire)
    {
        if (wire == 0)
            varint();
        else if (wire == 1) {
            require(e_ - p_ >= 8, "truncated fixed64");
            p_ += 8;
        } else if (wire == 2)
            message();
        else if (wire == 5)
            fixed32();
        else
            invalid("unsupported wire type");
    }

    template <typename T>
    void repeated(int wire, std::vector<T>& out)
    {
        if (wire == 2) {
            Wire w = message();
            while (w.more())
                out.push_back(static_cast<T>(w.varint()));
        } else {
            require(wire == 0, "bad repeated scalar");
            out.push_back(static_cast<T>(varint()));
        }
    }

private:
    const uint8_t* p_;
    const uint8_t* e_;
};

struct RawNode {
    uint32_t op = 0;
    std::vector<uint32_t> inputs, outputs;
    int attr = 0;
    std::vector<uint32_t> strides, pads, dilations;
    uint32_t groups = 0;
    int32_t axis = 0;
    float alpha = 0.0f;
    uint32_t block = 0;
};

struct RawTensor {
    uint32_t id = 0;
    TensorDesc desc;
    int storage_field = 0;
};

RawTensor read_tensor(Wire w)
{
    RawTensor t;
    uint32_t dtype = 0;
    while (w.more()) {
        const uint64_t key = w.varint();
        const int f = static_cast<int>(key >> 3), wt = static_cast<int>(key & 7);
        if (f == 1 && wt == 0)
            t.id = static_cast<uint32_t>(w.varint());
        else if (f == 2 && wt == 2)
            t.desc.name = w.bytes();
        else if (f == 3 && wt == 0)
            dtype = static_cast<uint32_t>(w.varint());
        else if (f == 4)
            w.repeated(wt, t.desc.shape);
        else if ((f == 5 || f == 6) && wt == 2) {
            t.storage_field = f;
            Wire s = w.message();
            while (s.more()) {
                const uint64_t k = s.varint();
                const int sf = static_cast<int>(k >> 3), sw = static_cast<int>(k & 7);
                if (sf == 1 && sw == 0)
                    t.desc.offset = s.varint();
                else if (sf == 2 && sw == 0)
                    t.desc.bytes = s.varint();
                else if (f == 5 && sf == 3 && sw == 0)
                    t.desc.birth = static_cast<uint32_t>(s.varint());
                else if (f == 5 && sf == 4 && sw == 0)
                    t.desc.death = static_cast<uint32_t>(s.varint());
                else
                    s.skip(sw);
            }
        } else
            w.skip(wt);
    }
    require(dtype >= 1 && dtype <= 3, "unsupported dtype");
    t.desc.dtype = static_cast<DType>(dtype);
    t.desc.storage = t.storage_field == 5 ? Storage::kArena : t.storage_field == 6 ? Storage::kWeight : Storage::kNone;
    return t;
}

RawNode read_node(Wire w)
{
    RawNode n;
    while (w.more()) {
        const uint64_t key = w.varint();
        const int f = static_cast<int>(key >> 3), wt = static_cast<int>(key & 7);
        if (f == 1 && wt == 0)
            n.op = static_cast<uint32_t>(w.varint());
        else if (f == 2)
            w.repeated(wt, n.inputs);
        else if (f == 3)
            w.repeated(wt, n.outputs);
        else if (f >= 4 && f <= 7 && wt == 2) {
            n.attr = f;
            Wire s = w.message();
            while (s.more()) {
                const uint64_t k = s.varint();
                const int sf = static_cast<int>(k >> 3), sw = static_cast<int>(k & 7);
                if (f == 4 && sf == 1)
                    s.repeated(sw, n.strides);
                else if (f == 4 && sf == 2)
                    s.repeated(sw, n.pads);
                else if (f == 4 && sf == 3)
                    s.repeated(sw, n.dilations);
                else if (f == 4 && sf == 4 && sw == 0)
                    n.groups = static_cast<uint32_t>(s.varint());
                else if (f == 5 && sf == 1 && sw == 0) {
                    const uint64_t z = s.varint();
                    n.axis = static_cast<int32_t>((z >> 1) ^ (~(z & 1) + 1));
                } else if (f == 6 && sf == 1 && sw == 5) {
                    const uint32_t b = s.fixed32();
                    std::memcpy(&n.alpha, &b, 4);
                } else if (f == 7 && sf == 1 && sw == 0)
                    n.block = static_cast<uint32_t>(s.varint());
                else
                    s.skip(sw);
            }
        } else
            w.skip(wt);
    }
    return n;
}

template <size_t N>
std::array<int, N> dims_of(const std::vector<uint32_t>& v, bool positive)
{
    require(v.size() == N, "attribute dimension count");
    std::array<int, N> out{};
    for (size_t i = 0; i < N; ++i) {
        require(v[i] <= static_cast<uint32_t>(std::numeric_limits<int>::max()) && (!positive || v[i] > 0),
                "invalid attribute dimension");
        out[i] = static_cast<int>(v[i]);
    }
    return out;
}

}  // namespace

size_t dtype_size(DType t)
{
    return t == DType::kFp16 ? 2 : t == DType::kInt32 ? 4 : 8;
}

int64_t element_count(const std::vector<int64_t>& shape)
{
    int64_t n = 1;
    for (auto d : shape)
        n *= d;
    return n;
}

GraphDesc decode_graph(const uint8_t* data, size_t size)
{
    require(data && size > 0 && size <= 64u * 1024u * 1024u, "message size");
    Wire w(data, data + size);
    uint32_t schema = 0, alignment = 0;
    size_t checkpoint_len = 0, weights_sha_len = 0;
    std::vector<RawTensor> raw_tensors;
    std::vector<RawNode> raw_nodes;
    GraphDesc g;
    while (w.more()) {
        const uint64_t key = w.varint();
        const int f = static_cast<int>(key >> 3), wt = static_cast<int>(key & 7);
        if (f == 1 && wt == 0)
            schema = static_cast<uint32_t>(w.varint());
        else if (f == 2 && wt == 2)
            checkpoint_len = w.bytes().size();
        else if (f == 3 && wt == 2)
            raw_tensors.push_back(read_tensor(w.message()));
        else if (f == 4)
            w.repeated(wt, g.inputs);
        else if (f == 5)
            w.repeated(wt, g.outputs);
        else if (f == 6 && wt == 2)
            raw_nodes.push_back(read_node(w.message()));
        else if (f == 7 && wt == 0)
            g.arena_bytes = w.varint();
        else if (f == 8 && wt == 0)
            alignment = static_cast<uint32_t>(w.varint());
        else if (f == 9 && wt == 0)
            g.weights_bytes = w.varint();
        else if (f == 10 && wt == 2)
            weights_sha_len = w.bytes().size();
        else
            w.skip(wt);
    }
    require(schema == 3, "unsupported schema");
    require(checkpoint_len == 32 && weights_sha_len == 32, "missing SHA-256 provenance");
    require(!raw_tensors.empty() && raw_tensors.size() <= 1000000, "tensor count");
    require(!raw_nodes.empty() && !g.inputs.empty() && !g.outputs.empty(), "empty graph");
    require(alignment == 256 && g.arena_bytes > 0, "arena configuration");

    g.tensors.resize(raw_tensors.size() + 1);
    std::unordered_set<std::string> names;
    std::unordered_set<uint32_t> available;
    for (auto& rt : raw_tensors) {
        require(rt.id > 0 && rt.id < g.tensors.size(), "tensor ID range");
        TensorDesc& d = g.tensors[rt.id];
        require(!d.present && !rt.desc.name.empty() && names.insert(rt.desc.name).second,
                "duplicate tensor ID or name");
        d = std::move(rt.desc);
        d.present = true;
        require(d.shape.size() <= 4, "tensor rank");
        uint64_t bytes = dtype_size(d.dtype);
        for (auto e : d.shape) {
            require(e > 0 && static_cast<uint64_t>(e) < (1ull << 40), "tensor extent overflow");
            bytes *= static_cast<uint64_t>(e);
        }
        if (d.storage == Storage::kWeight) {
            require(d.dtype != DType::kInt32 && d.offset % 256 == 0 && d.bytes == bytes &&
                        d.offset <= g.weights_bytes && d.bytes <= g.weights_bytes - d.offset,
                    "weight extent");
            available.insert(rt.id);
        } else {
            require(d.dtype != DType::kInt64, "runtime int64 tensor");
            if (d.storage == Storage::kArena)
                require(d.offset % 256 == 0 && d.bytes >= bytes && d.offset <= g.arena_bytes &&
                            d.bytes <= g.arena_bytes - d.offset && d.birth <= d.death &&
                            d.death <= raw_nodes.size(),
                        "arena extent");
        }
    }
    auto valid = [&](uint32_t id) { return id > 0 && id < g.tensors.size() && g.tensors[id].present; };
    for (auto id : g.inputs)
        require(valid(id) && g.tensors[id].storage == Storage::kNone && available.insert(id).second,
                "input ID or storage");
    for (auto& rn : raw_nodes) {
        NodeDesc n;
        require(rn.op >= 1 && rn.op <= 14, "unknown operator");
        n.op = static_cast<Op>(rn.op);
        n.inputs = rn.inputs;
        const size_t count = n.inputs.size();
        switch (n.op) {
        case Op::kConv: {
            require(rn.attr == 4 && (count == 2 || count == 3), "convolution contract");
            n.strides = dims_of<2>(rn.strides, true);
            n.pads = dims_of<4>(rn.pads, false);
            const auto dil = dims_of<2>(rn.dilations, true);
            require(rn.groups > 0 && rn.groups <= static_cast<uint32_t>(std::numeric_limits<int>::max()),
                    "invalid positive attribute");
            n.groups = static_cast<int>(rn.groups);
            require(dil[0] == 1 && dil[1] == 1, "unsupported dilation");
            require(n.pads[0] == n.pads[2] && n.pads[1] == n.pads[3], "asymmetric convolution padding");
            break;
        }
        case Op::kConcat:
        case Op::kGather:
            require(rn.attr == 5 && (n.op == Op::kConcat ? count > 0 : count == 2), "axis contract");
            n.axis = rn.axis;
            break;
        case Op::kLeakyRelu:
            require(rn.attr == 6 && count == 1 && std::isfinite(rn.alpha), "activation contract");
            n.alpha = rn.alpha;
            break;
        case Op::kSpaceToDepth:
        case Op::kDepthToSpace:
            require(rn.attr == 7 && count == 1 && rn.block > 0 && rn.block < 65536, "pixel layout contract");
            n.block = static_cast<int>(rn.block);
            break;
        case Op::kAdd:
        case Op::kSub:
        case Op::kMul:
            require(rn.attr == 0 && count == 2, "binary contract");
            break;
        case Op::kClip:
            require(rn.attr == 0 && count >= 1 && count <= 3, "clip contract");
            break;
        case Op::kSlice:
            require(rn.attr == 0 && count >= 3 && count <= 5, "slice contract");
            break;
        default:
            require(rn.attr == 0 && count == 1, "unary contract");
        }
        for (size_t i = 0; i < count; ++i) {
            if (n.inputs[i] == 0)
                require((n.op == Op::kConv && i == 2) || (n.op == Op::kClip && i > 0) ||
                            (n.op == Op::kSlice && i > 2),
                        "absent required operand");
            else
                require(valid(n.inputs[i]) && available.count(n.inputs[i]), "unresolved operand");
        }
        require(rn.outputs.size() == 1 && valid(rn.outputs[0]), "output ID");
        n.output = rn.outputs[0];
        const TensorDesc& out = g.tensors[n.output];
        require(out.storage == Storage::kArena && available.insert(n.output).second,
                "duplicate output or missing arena");
        require(out.birth == g.nodes.size(), "tensor birth");
        g.nodes.push_back(std::move(n));
    }
    std::unordered_set<uint32_t> seen;
    for (auto id : g.outputs)
        require(valid(id) && available.count(id) && seen.insert(id).second, "graph output");
    return g;
}

}  // namespace mlvc_b200
