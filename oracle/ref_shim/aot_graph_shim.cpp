// Test infrastructure only (oracle side). Never linked into the product.
//
// The reference's CPU backend (backends/cpu/src/*.cpp, compiled unchanged
// from the reference tree) calls mlvc::aot::load_aot_graph(), which upstream
// lives in runtime/src/aot_graph.cpp:291-317 and needs libprotobuf.  No
// libprotobuf C++ runtime exists in this image, so this file supplies a
// protobuf-free implementation with the same contract: it decodes the
// mlvc.wire.Graph message (proto/mlvc_model.proto:30-83) from raw wire bytes
// and applies the validation rules of runtime/src/aot_graph.cpp:110-283
// (schema 3, 256-byte arena alignment, SHA-256 provenance, tensor extents,
// per-op operand contracts, birth order).  The metadata.pb checksum cross
// check (aot_graph.cpp:299-305) is skipped when metadata.pb is absent, since
// the synthetic test bundles carry only aot/<part>/{graph.pb,weights.bin}.
#include "mlvc/runtime/aot_graph.hpp"

#include <cmath>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>
#include <unordered_set>

namespace mlvc::aot {
namespace {

[[noreturn]] void fail(const char* what)
{
    throw std::runtime_error(std::string("invalid AOT Protobuf graph: ") + what);
}

void require(bool ok, const char* what)
{
    if (!ok)
        fail(what);
}

struct Reader {
    const std::uint8_t* p;
    const std::uint8_t* end;

    bool done() const { return p >= end; }

    std::uint64_t varint()
    {
        std::uint64_t value = 0;
        for (int shift = 0; shift < 64; shift += 7) {
            require(p < end, "truncated varint");
            const std::uint8_t byte = *p++;
            value |= static_cast<std::uint64_t>(byte & 0x7f) << shift;
            if ((byte & 0x80) == 0)
                return value;
        }
        fail("overlong varint");
    }

    Reader sub()
    {
        const std::uint64_t n = varint();
        require(n <= static_cast<std::uint64_t>(end - p), "truncated field");
        Reader r{p, p + n};
        p += n;
        return r;
    }

    std::uint32_t fixed32()
    {
        require(end - p >= 4, "truncated fixed32");
        std::uint32_t v;
        std::memcpy(&v, p, 4);
        p += 4;
        return v;
    }

    void skip(int wire)
    {
        switch (wire) {
        case 0: varint(); break;
        case 1: require(end - p >= 8, "truncated fixed64"); p += 8; break;
        case 2: sub(); break;
        case 5: fixed32(); break;
        default: fail("unsupported wire type");
        }
    }
};

// Repeated scalar fields may arrive packed (wire type 2) or unpacked.
template <typename T>
void repeated_varint(Reader& r, int wire, std::vector<T>& out)
{
    if (wire == 2) {
        Reader s = r.sub();
        while (!s.done())
            out.push_back(static_cast<T>(s.varint()));
    } else {
        require(wire == 0, "bad repeated varint");
        out.push_back(static_cast<T>(r.varint()));
    }
}

std::int32_t zigzag32(std::uint64_t v)
{
    return static_cast<std::int32_t>((v >> 1) ^ (~(v & 1) + 1));
}

struct WireTensor {
    std::uint32_t id = 0;
    std::string name;
    std::uint32_t dtype = 0;
    std::vector<std::int64_t> shape;
    int storage = 0;  // 5 arena, 6 weight
    std::uint64_t offset = 0, size = 0;
    std::uint32_t birth = 0, death = 0;
};

struct WireNode {
    std::uint32_t op = 0;
    std::vector<std::uint32_t> inputs, outputs;
    int attr = 0;  // 4 conv, 5 axis, 6 activation, 7 pixel
    std::vector<std::uint32_t> strides, pads, dilations;
    std::uint32_t groups = 0;
    std::int32_t axis = 0;
    float alpha = 0.0F;
    std::uint32_t block = 0;
};

WireTensor parse_tensor(Reader r)
{
    WireTensor t;
    while (!r.done()) {
        const std::uint64_t key = r.varint();
        const int field = static_cast<int>(key >> 3), wire = static_cast<int>(key & 7);
        if (field == 1 && wire == 0) t.id = static_cast<std::uint32_t>(r.varint());
        else if (field == 2 && wire == 2) { Reader s = r.sub(); t.name.assign(reinterpret_cast<const char*>(s.p), s.end - s.p); }
        else if (field == 3 && wire == 0) t.dtype = static_cast<std::uint32_t>(r.varint());
        else if (field == 4) repeated_varint(r, wire, t.shape);
        else if ((field == 5 || field == 6) && wire == 2) {
            t.storage = field;
            Reader s = r.sub();
            while (!s.done()) {
                const std::uint64_t k = s.varint();
                const int f = static_cast<int>(k >> 3), w = static_cast<int>(k & 7);
                if (f == 1 && w == 0) t.offset = s.varint();
                else if (f == 2 && w == 0) t.size = s.varint();
                else if (f == 3 && w == 0 && field == 5) t.birth = static_cast<std::uint32_t>(s.varint());
                else if (f == 4 && w == 0 && field == 5) t.death = static_cast<std::uint32_t>(s.varint());
                else s.skip(w);
            }
        } else r.skip(wire);
    }
    return t;
}

WireNode parse_node(Reader r)
{
    WireNode n;
    while (!r.done()) {
        const std::uint64_t key = r.varint();
        const int field = static_cast<int>(key >> 3), wire = static_cast<int>(key & 7);
        if (field == 1 && wire == 0) n.op = static_cast<std::uint32_t>(r.varint());
        else if (field == 2) repeated_varint(r, wire, n.inputs);
        else if (field == 3) repeated_varint(r, wire, n.outputs);
        else if (field >= 4 && field <= 7 && wire == 2) {
            n.attr = field;
            Reader s = r.sub();
            while (!s.done()) {
                const std::uint64_t k = s.varint();
                const int f = static_cast<int>(k >> 3), w = static_cast<int>(k & 7);
                if (field == 4 && f == 1) repeated_varint(s, w, n.strides);
                else if (field == 4 && f == 2) repeated_varint(s, w, n.pads);
                else if (field == 4 && f == 3) repeated_varint(s, w, n.dilations);
                else if (field == 4 && f == 4 && w == 0) n.groups = static_cast<std::uint32_t>(s.varint());
                else if (field == 5 && f == 1 && w == 0) n.axis = zigzag32(s.varint());
                else if (field == 6 && f == 1 && w == 5) { const std::uint32_t b = s.fixed32(); std::memcpy(&n.alpha, &b, 4); }
                else if (field == 7 && f == 1 && w == 0) n.block = static_cast<std::uint32_t>(s.varint());
                else s.skip(w);
            }
        } else r.skip(wire);
    }
    return n;
}

template <std::size_t N>
std::array<int, N> dims(const std::vector<std::uint32_t>& v, bool positive)
{
    require(v.size() == N, "attribute dimension count");
    std::array<int, N> out{};
    for (std::size_t i = 0; i < N; ++i) {
        require(v[i] <= static_cast<std::uint32_t>(std::numeric_limits<int>::max()) &&
                    (!positive || v[i] > 0),
                "invalid attribute dimension");
        out[i] = static_cast<int>(v[i]);
    }
    return out;
}

}  // namespace

GraphDescriptor decode_graph_binary(std::span<const std::byte> bytes)
{
    require(!bytes.empty() && bytes.size() <= 64U * 1024U * 1024U, "message size");
    Reader r{reinterpret_cast<const std::uint8_t*>(bytes.data()),
             reinterpret_cast<const std::uint8_t*>(bytes.data()) + bytes.size()};
    std::uint32_t schema = 0, alignment = 0;
    std::size_t ck_len = 0, wsha_len = 0;
    std::uint64_t arena_bytes = 0, weights_bytes = 0;
    std::vector<WireTensor> tensors;
    std::vector<WireNode> nodes;
    std::vector<std::uint32_t> inputs, outputs;
    while (!r.done()) {
        const std::uint64_t key = r.varint();
        const int field = static_cast<int>(key >> 3), wire = static_cast<int>(key & 7);
        if (field == 1 && wire == 0) schema = static_cast<std::uint32_t>(r.varint());
        else if (field == 2 && wire == 2) { Reader s = r.sub(); ck_len = s.end - s.p; }
        else if (field == 3 && wire == 2) tensors.push_back(parse_tensor(r.sub()));
        else if (field == 4) repeated_varint(r, wire, inputs);
        else if (field == 5) repeated_varint(r, wire, outputs);
        else if (field == 6 && wire == 2) nodes.push_back(parse_node(r.sub()));
        else if (field == 7 && wire == 0) arena_bytes = r.varint();
        else if (field == 8 && wire == 0) alignment = static_cast<std::uint32_t>(r.varint());
        else if (field == 9 && wire == 0) weights_bytes = r.varint();
        else if (field == 10 && wire == 2) { Reader s = r.sub(); wsha_len = s.end - s.p; }
        else r.skip(wire);
    }
    require(schema == 3, "unsupported schema");
    require(ck_len == 32 && wsha_len == 32, "missing SHA-256 provenance");
    require(!tensors.empty() && tensors.size() <= 1000000, "tensor count");
    require(!nodes.empty() && !inputs.empty() && !outputs.empty(), "empty graph");
    require(alignment == 256 && arena_bytes > 0, "arena configuration");

    GraphDescriptor g;
    g.arena_bytes = arena_bytes;
    g.weights_bytes = weights_bytes;
    g.tensors.resize(tensors.size() + 1);
    std::unordered_set<std::string> names;
    std::unordered_set<TensorId> available;
    for (const auto& t : tensors) {
        require(t.id > 0 && t.id < g.tensors.size(), "tensor ID range");
        auto& d = g.tensors[t.id];
        require(d.name.empty() && !t.name.empty() && names.insert(t.name).second,
                "duplicate tensor ID or name");
        d.name = t.name;
        require(t.dtype >= 1 && t.dtype <= 3, "unsupported dtype");
        d.dtype = static_cast<DataType>(t.dtype);
        d.shape = t.shape;
        require(d.shape.size() <= 4, "tensor rank");
        std::uint64_t bytes = t.dtype == 1 ? 2 : t.dtype == 2 ? 4 : 8;
        for (auto e : d.shape) {
            require(e > 0 && static_cast<std::uint64_t>(e) < (1ULL << 40), "tensor extent overflow");
            bytes *= static_cast<std::uint64_t>(e);
        }
        if (t.storage == 6) {
            require(d.dtype != DataType::INT32 && t.offset % 256 == 0 && t.size == bytes &&
                        t.offset <= weights_bytes && t.size <= weights_bytes - t.offset,
                    "weight extent");
            d.storage = WeightLocation{t.offset, t.size};
            available.insert(t.id);
        } else {
            require(d.dtype != DataType::INT64, "runtime int64 tensor");
            if (t.storage == 5) {
                require(t.offset % 256 == 0 && t.size >= bytes && t.offset <= arena_bytes &&
                            t.size <= arena_bytes - t.offset && t.birth <= t.death &&
                            t.death <= nodes.size(),
                        "arena extent");
                d.storage = ArenaSlot{t.offset, t.size, t.birth, t.death};
            }
        }
    }
    auto valid = [&](TensorId id) {
        return id > 0 && id < g.tensors.size() && !g.tensors[id].name.empty();
    };
    for (auto id : inputs) {
        require(valid(id) && std::holds_alternative<std::monostate>(g.tensors[id].storage) &&
                    available.insert(id).second,
                "input ID or storage");
        g.inputs.push_back(id);
    }
    for (const auto& w : nodes) {
        Node n;
        n.index = g.nodes.size();
        require(w.op >= 1 && w.op <= 14, "unknown operator");
        n.op = static_cast<Op>(w.op);
        n.inputs.assign(w.inputs.begin(), w.inputs.end());
        n.outputs.assign(w.outputs.begin(), w.outputs.end());
        const std::size_t count = n.inputs.size();
        switch (n.op) {
        case Op::CONV:
            require(w.attr == 4 && (count == 2 || count == 3), "convolution contract");
            require(w.groups > 0, "invalid positive attribute");
            n.attributes = ConvAttributes{dims<2>(w.strides, true), dims<4>(w.pads, false),
                                          dims<2>(w.dilations, true), static_cast<int>(w.groups)};
            require(n.conv().dilations == std::array<int, 2>{1, 1}, "unsupported dilation");
            require(n.conv().pads[0] == n.conv().pads[2] && n.conv().pads[1] == n.conv().pads[3],
                    "asymmetric convolution padding");
            break;
        case Op::CONCAT:
        case Op::GATHER:
            require(w.attr == 5 && (n.op == Op::CONCAT ? count > 0 : count == 2), "axis contract");
            n.attributes = AxisAttributes{w.axis};
            break;
        case Op::LEAKY_RELU:
            require(w.attr == 6 && count == 1 && std::isfinite(w.alpha), "activation contract");
            n.attributes = ActivationAttributes{w.alpha};
            break;
        case Op::SPACE_TO_DEPTH:
        case Op::DEPTH_TO_SPACE:
            require(w.attr == 7 && count == 1 && w.block > 0, "pixel layout contract");
            n.attributes = PixelAttributes{static_cast<int>(w.block)};
            break;
        case Op::ADD:
        case Op::SUB:
        case Op::MUL:
            require(w.attr == 0 && count == 2, "binary contract");
            break;
        case Op::CLIP:
            require(w.attr == 0 && count >= 1 && count <= 3, "clip contract");
            break;
        case Op::SLICE:
            require(w.attr == 0 && count >= 3 && count <= 5, "slice contract");
            break;
        default:
            require(w.attr == 0 && count == 1, "unary contract");
        }
        for (std::size_t i = 0; i < count; ++i) {
            if (n.inputs[i] == 0)
                require((n.op == Op::CONV && i == 2) || (n.op == Op::CLIP && i > 0) ||
                            (n.op == Op::SLICE && i > 2),
                        "absent required operand");
            else
                require(valid(n.inputs[i]) && available.count(n.inputs[i]), "unresolved operand");
        }
        require(n.outputs.size() == 1 && valid(n.outputs[0]), "output ID");
        const auto id = n.outputs[0];
        require(std::holds_alternative<ArenaSlot>(g.tensors[id].storage) &&
                    available.insert(id).second,
                "duplicate output or missing arena");
        require(std::get<ArenaSlot>(g.tensors[id].storage).birth == n.index, "tensor birth");
        g.nodes.push_back(std::move(n));
    }
    std::unordered_set<TensorId> seen;
    for (auto id : outputs) {
        require(valid(id) && available.count(id) && seen.insert(id).second, "graph output");
        g.outputs.push_back(id);
    }
    return g;
}

LoadedGraph load_aot_graph(const ModelAssetReader& assets, const std::string& model_name)
{
    const std::filesystem::path dir = std::filesystem::path("aot") / model_name;
    const auto bytes = assets.read_binary(dir / "graph.pb");
    LoadedGraph loaded;
    loaded.descriptor = decode_graph_binary(bytes);
    loaded.weights = assets.read_binary(dir / "weights.bin");
    if (loaded.weights.size() != loaded.descriptor.weights_bytes)
        throw std::runtime_error("AOT weights size does not match graph (" +
                                 assets.location_label() + ")");
    return loaded;
}

LoadedGraph load_aot_graph(const std::filesystem::path& model_dir, const std::string& model_name)
{
    const auto assets = make_model_asset_reader(model_dir);
    return load_aot_graph(*assets, model_name);
}

}  // namespace mlvc::aot
