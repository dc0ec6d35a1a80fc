// In-memory form of one AOT graph part (mlvc.wire.Graph, schema 3).
//
// Mirrors the reference's runtime contract (runtime/include/mlvc/runtime/
// aot_graph.hpp:18-123): dense tensor IDs from 1, 14 operators, NCHW logical
// shapes, weights at 256-byte aligned offsets of weights.bin, runtime values
// with arena slots planned by the AOT compiler.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace mlvc_b200 {

enum class Op : int {
    kUnspecified = 0,
    kAdd = 1,
    kSub = 2,
    kMul = 3,
    kClip = 4,
    kConcat = 5,
    kConv = 6,
    kDepthToSpace = 7,
    kGather = 8,
    kLeakyRelu = 9,
    kReciprocal = 10,
    kRound = 11,
    kSigmoid = 12,
    kSlice = 13,
    kSpaceToDepth = 14,
};

enum class DType : int { kUnspecified = 0, kFp16 = 1, kInt32 = 2, kInt64 = 3 };

enum class Storage : int { kNone = 0, kArena = 1, kWeight = 2 };

struct TensorDesc {
    std::string name;
    DType dtype = DType::kUnspecified;
    std::vector<int64_t> shape;
    Storage storage = Storage::kNone;
    uint64_t offset = 0;  // arena or weights byte offset
    uint64_t bytes = 0;   // slot / weight size
    uint32_t birth = 0, death = 0;
    bool present = false;
};

struct NodeDesc {
    Op op = Op::kUnspecified;
    std::vector<uint32_t> inputs;
    uint32_t output = 0;
    // Conv
    std::array<int, 2> strides{1, 1};
    std::array<int, 4> pads{0, 0, 0, 0};
    int groups = 1;
    // Concat / Gather
    int axis = 0;
    // LeakyRelu
    float alpha = 0.01f;
    // DepthToSpace / SpaceToDepth
    int block = 1;
};

struct GraphDesc {
    std::vector<TensorDesc> tensors;  // index = tensor ID, [0] unused
    std::vector<NodeDesc> nodes;
    std::vector<uint32_t> inputs;
    std::vector<uint32_t> outputs;
    uint64_t arena_bytes = 0;
    uint64_t weights_bytes = 0;
};

// Decodes and validates graph.pb bytes; throws std::runtime_error with an
// "invalid AOT graph: ..." message on any contract violation.
GraphDesc decode_graph(const uint8_t* data, size_t size);

size_t dtype_size(DType t);
int64_t element_count(const std::vector<int64_t>& shape);

}  // namespace mlvc_b200
