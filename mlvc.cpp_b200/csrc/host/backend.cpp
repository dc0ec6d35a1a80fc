// B200 backend: graph planning (layout, fusion, arena), weight preparation,
// kernel-parameter construction, CUDA-graph capture and replay.
//
// Layout: every rank-4 FP16 runtime tensor is stored channels-last (NHWC) on
// the device; weights keep their NCHW/OIHW layout and conv weights get a
// one-time prepared copy in the order each kernel reads.  Graph inputs and
// outputs keep NCHW on the host; conversion kernels sit at the boundary (the
// CPU backend of the reference makes the same choice,
// backends/cpu/src/execution_plan.cpp:646-650,1324-1360).
//
// Fusion: the same chains the reference recognises
// (backends/driver_cubin/src/execution_plan.cpp:16-41,
//  fusion_registry.cpp:711-1036): Conv+LeakyReLU, Conv+Add (residual),
// Conv+Slice+Slice+Clip+Mul (ReGLU), Slice+Slice+Clip+Mul.  Fused chains write
// only their final tensor; the backend plans its own arena over the tensors it
// actually materialises, so inputs and outputs of one step never overlap.
#include "backend.hpp"

#include "../kernels/params.h"

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <limits>
#include <map>
#include <sstream>
#include <stdexcept>

extern "C" const unsigned char mlvc_b200_cubin_start[];
extern "C" const unsigned char mlvc_b200_cubin_end[];

namespace mlvc_b200 {

namespace {

uint16_t float_to_half_bits(float f)
{
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const int exp = static_cast<int>((u >> 23) & 0xff) - 127 + 15;
    uint32_t man = u & 0x7fffffu;
    if (((u >> 23) & 0xff) == 0xff)
        return static_cast<uint16_t>(sign | 0x7c00u | (man ? 0x200u : 0u));
    if (exp >= 31)
        return static_cast<uint16_t>(sign | 0x7c00u);
    if (exp <= 0) {
        if (exp < -10)
            return static_cast<uint16_t>(sign);
        man |= 0x800000u;
        const unsigned shift = static_cast<unsigned>(14 - exp);
        uint32_t q = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u)))
            ++q;
        return static_cast<uint16_t>(sign | q);
    }
    uint32_t q = man >> 13;
    const uint32_t rem = man & 0x1fffu;
    uint32_t e = static_cast<uint32_t>(exp);
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) {
        if (++q == 0x400u) {
            q = 0;
            if (++e >= 31)
                return static_cast<uint16_t>(sign | 0x7c00u);
        }
    }
    return static_cast<uint16_t>(sign | (e << 10) | q);
}

float half_bits_to_float(uint16_t h)
{
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    if (exp == 0) {
        const float mag = static_cast<float>(man) * 5.9604644775390625e-08f;  // 2^-24
        return sign ? -mag : mag;
    }
    uint32_t bits;
    if (exp == 31)
        bits = sign | 0x7f800000u | (man << 13);
    else
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Output / residual tile view of a tensor-core epilogue on an NHWC tensor:
// 1x1 (w == 0): {channels, pixels} with {64, 128} boxes; otherwise {channels,
// w, h} with {64, box_w, box_h} boxes (k x k: one 128-pixel row segment,
// fused depthwise: 16 x 8 pixels); 128-byte swizzle.  Boxes are clipped (stores)
// or zero-filled (loads) at the tensor edges.
void encode_tile_map(CUtensorMap* map, CUdeviceptr addr, int channels, int pixels, int w, int h, const char* what,
                     int box_w = 128, int box_h = 1)
{
    const cuuint32_t elem[3] = {1, 1, 1};
    const cuuint64_t c = static_cast<cuuint64_t>(channels);
    if (w == 0) {
        const cuuint64_t dims[2] = {c, static_cast<cuuint64_t>(pixels)};
        const cuuint64_t strides[1] = {c * 2};
        const cuuint32_t box[2] = {64, 128};
        check(cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, reinterpret_cast<void*>(addr), dims,
                                     strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
              what);
    } else {
        const cuuint64_t dims[3] = {c, static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h)};
        const cuuint64_t strides[2] = {c * 2, static_cast<cuuint64_t>(w) * c * 2};
        const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_w), static_cast<cuuint32_t>(box_h)};
        check(cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, reinterpret_cast<void*>(addr), dims,
                                     strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
              what);
    }
}

std::vector<int64_t> dims4(const std::vector<int64_t>& s)
{
    std::vector<int64_t> d(4 - std::min<size_t>(4, s.size()), 1);
    d.insert(d.end(), s.begin(), s.end());
    return d;
}

unsigned blocks_for(long long work, int threads, int sm_count)
{
    const long long b = (work + threads - 1) / threads;
    return static_cast<unsigned>(std::max<long long>(1, std::min<long long>(b, static_cast<long long>(sm_count) * 16)));
}

}  // namespace

// ------------------------------------------------------------------ types
struct Backend::Value {
    bool present = false;
    DType dtype = DType::kFp16;
    std::vector<int64_t> shape;
    bool nhwc = false;
    enum Kind { kNone, kWeight, kInput, kArena, kState } kind = kNone;
    CUdeviceptr addr = 0;
    size_t bytes = 0;
    long first = -1, last = -1;  // arena liveness in step indices
    size_t arena_off = 0;
    int consumers = 0;
    bool graph_output = false;
    size_t weight_off = 0;  // weights.bin offset for kWeight
    // A Slice whose result is one contiguous byte range of its source is not
    // materialised: the value lives inside the source's buffer, alias_off bytes
    // in (alias_of = the source, never itself an alias; 0 = not an alias).
    uint32_t alias_of = 0;
    size_t alias_off = 0;

    // Physical element strides for logical (n, c, h, w).
    std::array<long long, 4> strides() const
    {
        const auto d = dims4(shape);
        if (nhwc)
            return {d[1] * d[2] * d[3], 1, d[3] * d[1], d[1]};
        return {d[1] * d[2] * d[3], d[2] * d[3], d[3], 1};
    }
};

struct Backend::Step {
    enum Type { kKernel, kCopy, kMemset } type = kKernel;
    std::string kernel;
    std::string symbol;  // cubin entry point when it is a variant of `kernel` (empty: `kernel` itself)
    CUfunction f = nullptr;
    unsigned grid = 1, block = 256, smem = 0;
    unsigned grid_y = 1, grid_z = 1, block_y = 1;
    std::vector<uint8_t> params;
    std::function<void(Step&)> build;
    std::vector<uint32_t> reads, writes;  // value IDs (for liveness)
    CUdeviceptr src = 0, dst = 0;
    size_t bytes = 0;
    StepInfo info;

    template <typename P>
    void set(const P& p)
    {
        params.resize(sizeof(P));
        std::memcpy(params.data(), &p, sizeof(P));
    }
};

// One buffered frame of the slot pipeline (reference: the two codec slots of
// backends/driver_cubin/src/cuda_graph_executor.cpp:205-290).  Pinned host
// buffers for the caller, device staging of its own, and a CUDA graph that
// moves the staged inputs into the schedule's input buffers, runs the
// schedule and copies the outputs out to the staging: the host->device copy
// of one slot and the device->host copy of another overlap the schedule of a
// third on separate copy streams.
struct Backend::Slot {
    std::vector<PinnedBuffer> in, out;
    std::vector<DeviceBuffer> din, dout;
    Event in_done{CU_EVENT_DISABLE_TIMING}, computed{CU_EVENT_DISABLE_TIMING}, done{CU_EVENT_DISABLE_TIMING};
    CUgraph graph = nullptr;
    CUgraphExec exec = nullptr;
    bool pending = false;
    Slot() = default;
    Slot(const Slot&) = delete;
    Slot& operator=(const Slot&) = delete;
    ~Slot()
    {
        if (exec)
            cuGraphExecDestroy(exec);
        if (graph)
            cuGraphDestroy(graph);
    }
};

// ------------------------------------------------------------ lifecycle
Backend::Backend(int device_id) : device_(device_id)
{
    check(cuInit(0), "cuInit");
    int count = 0;
    check(cuDeviceGetCount(&count), "cuDeviceGetCount");
    if (device_id < 0 || device_id >= count)
        throw std::runtime_error("mlvc-b200: device id " + std::to_string(device_id) + " out of range");
    check(cuDeviceGet(&dev_, device_id), "cuDeviceGet");
    int major = 0, minor = 0;
    check(cuDeviceGetAttribute(&major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, dev_), "cuDeviceGetAttribute");
    check(cuDeviceGetAttribute(&minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, dev_), "cuDeviceGetAttribute");
    if (major != 10 || minor != 0)
        throw std::runtime_error("mlvc-b200: requires an sm_100 (B200) device, found sm_" + std::to_string(major) +
                                 std::to_string(minor));
    check(cuDevicePrimaryCtxRetain(&ctx_, dev_), "cuDevicePrimaryCtxRetain");
    ContextGuard guard(ctx_);
    check(cuDeviceGetAttribute(&sm_count_, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev_), "cuDeviceGetAttribute");
    check(cuDeviceGetAttribute(&max_smem_optin_, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, dev_),
          "cuDeviceGetAttribute");
    check(cuStreamCreate(&stream_, CU_STREAM_NON_BLOCKING), "cuStreamCreate");
    check(cuModuleLoadData(&module_, mlvc_b200_cubin_start), "cuModuleLoadData");
    size_t sz = 0;
    check(cuModuleGetGlobal(&status_ptr_, &sz, module_, "mlvc_b200_status"), "cuModuleGetGlobal(mlvc_b200_status)");
}

Backend::Backend(int sm_count, int smem_optin, bool) : sm_count_(sm_count), max_smem_optin_(smem_optin), offline_(true)
{
}

Backend::~Backend()
{
    if (!ctx_)
        return;
    cuCtxSetCurrent(ctx_);
    if (stream_)
        cuStreamSynchronize(stream_);
    for (CUstream s : {copy_in_, copy_out_})
        if (s)
            cuStreamSynchronize(s);
    if (graph_exec_)
        cuGraphExecDestroy(graph_exec_);
    if (graph_handle_)
        cuGraphDestroy(graph_handle_);
    slots_.clear();
    weights_dev_.reset();
    prepped_dev_.reset();
    arena_dev_.reset();
    flush_dev_.reset();
    entropy_scratch_.reset();
    input_dev_.clear();
    input_stage_dev_.clear();
    output_stage_dev_.clear();
    state_dev_.clear();
    if (module_)
        cuModuleUnload(module_);
    for (CUstream s : {copy_in_, copy_out_})
        if (s) {
            cuStreamSynchronize(s);
            cuStreamDestroy(s);
        }
    if (stream_)
        cuStreamDestroy(stream_);
    cuDevicePrimaryCtxRelease(dev_);
}

CUfunction Backend::fn(const char* name)
{
    CUfunction f = nullptr;
    check(cuModuleGetFunction(&f, module_, name), name);
    return f;
}

const TensorDesc& Backend::input_desc(size_t i) const { return graph_.tensors.at(graph_.inputs.at(ext_inputs_.at(i))); }
const TensorDesc& Backend::output_desc(size_t i) const
{
    return graph_.tensors.at(graph_.outputs.at(ext_outputs_.at(i)));
}

void Backend::load(const std::string& model_dir, const std::string& part, const std::vector<StateBinding>& bindings)
{
    auto read = [](const std::string& path) {
        std::ifstream f(path, std::ios::binary);
        if (!f)
            throw std::runtime_error("mlvc-b200: cannot read " + path);
        return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    };
    const std::string dir = model_dir + "/aot/" + part + "/";
    const auto g = read(dir + "graph.pb");
    const auto w = read(dir + "weights.bin");
    load_bytes(g.data(), g.size(), w.data(), w.size(), bindings);
}

void Backend::load_bytes(const uint8_t* graph, size_t graph_size, const uint8_t* weights, size_t weights_size,
                         const std::vector<StateBinding>& bindings)
{
    if (loaded_)
        throw std::runtime_error("mlvc-b200: load() may be called once per backend instance");
    graph_ = decode_graph(graph, graph_size);
    if (weights_size != graph_.weights_bytes)
        throw std::runtime_error("mlvc-b200: AOT weights size does not match graph");
    weights_host_.assign(weights, weights + weights_size);
    bindings_ = bindings;
    std::vector<bool> in_bound(graph_.inputs.size()), out_bound(graph_.outputs.size());
    for (const auto& b : bindings_) {
        if (b.input_index >= graph_.inputs.size() || b.output_index >= graph_.outputs.size() ||
            in_bound[b.input_index] || out_bound[b.output_index])
            throw std::runtime_error("mlvc-b200: invalid state binding");
        const auto& ti = graph_.tensors[graph_.inputs[b.input_index]];
        const auto& to = graph_.tensors[graph_.outputs[b.output_index]];
        if (ti.shape != to.shape || ti.dtype != DType::kFp16 || to.dtype != DType::kFp16)
            throw std::runtime_error("mlvc-b200: state binding shape or dtype mismatch");
        in_bound[b.input_index] = out_bound[b.output_index] = true;
    }
    for (size_t i = 0; i < graph_.inputs.size(); ++i)
        if (!in_bound[i])
            ext_inputs_.push_back(i);
    for (size_t i = 0; i < graph_.outputs.size(); ++i)
        if (!out_bound[i])
            ext_outputs_.push_back(i);
    plan();
    if (offline_) {
        step_info_.clear();
        for (auto& st : steps_) {
            st.info.kernel = st.kernel;
            st.info.grid = st.grid * st.grid_y * st.grid_z;
            st.info.block = st.block * st.block_y;
            st.info.smem = st.smem;
            step_info_.push_back(st.info);
        }
        loaded_ = true;
        return;
    }
    ContextGuard guard(ctx_);
    build_schedule();
    capture();
    state_ready_ = bindings_.empty();
    loaded_ = true;
}

// ---------------------------------------------------------------- planning
void Backend::plan()
{
    {
        const char* env = std::getenv("MLVC_B200_FFN_FUSION");
        ffn_fusion_ = !(env && env[0] == '0');
        env = std::getenv("MLVC_B200_DW_FUSION");
        dw_fusion_ = !(env && env[0] == '0');
        env = std::getenv("MLVC_B200_MB_FUSION");
        mb_fusion_ = !(env && env[0] == '0');
        env = std::getenv("MLVC_B200_TAIL_FUSION");
        tail_fusion_ = !(env && env[0] == '0');
        env = std::getenv("MLVC_B200_D2S_FUSION");
        d2s_fusion_ = !(env && env[0] == '0');
    }
    const size_t nt = graph_.tensors.size();
    values_.assign(nt, Value{});
    for (size_t id = 1; id < nt; ++id) {
        const auto& t = graph_.tensors[id];
        if (!t.present)
            continue;
        Value& v = values_[id];
        v.present = true;
        v.dtype = t.dtype;
        v.shape = t.shape;
        v.bytes = static_cast<size_t>(element_count(t.shape)) * dtype_size(t.dtype);
        if (t.storage == Storage::kWeight) {
            v.kind = Value::kWeight;
            v.weight_off = t.offset;
        } else {
            v.nhwc = t.shape.size() == 4 && t.dtype == DType::kFp16;
        }
    }
    for (const auto& n : graph_.nodes)
        for (auto id : n.inputs)
            if (id)
                values_[id].consumers++;
    for (auto id : graph_.outputs)
        values_[id].graph_output = true;
    for (size_t i = 0; i < graph_.inputs.size(); ++i)
        values_[graph_.inputs[i]].kind = Value::kInput;
    for (const auto& b : bindings_)
        values_[graph_.inputs[b.input_index]].kind = Value::kState;

    steps_.clear();
    prepped_host_.clear();
    auto prep = [&](const void* data, size_t bytes) {
        const size_t off = align_up(prepped_host_.size(), 256);
        prepped_host_.resize(off + bytes);
        std::memcpy(prepped_host_.data() + off, data, bytes);
        return off;
    };
    auto wdata = [&](uint32_t id) -> const uint16_t* {
        return reinterpret_cast<const uint16_t*>(weights_host_.data() + values_[id].weight_off);
    };
    auto scalar = [&](uint32_t id, float dflt) -> float {
        if (id == 0)
            return dflt;
        const Value& v = values_.at(id);
        if (v.kind != Value::kWeight || v.dtype != DType::kFp16)
            throw std::runtime_error("mlvc-b200: Clip bound must be an FP16 initializer");
        return half_bits_to_float(wdata(id)[0]);
    };
    auto int64s = [&](uint32_t id) {
        const Value& v = values_.at(id);
        if (v.kind != Value::kWeight || v.dtype != DType::kInt64)
            throw std::runtime_error("mlvc-b200: Slice parameters must be INT64 initializers");
        std::vector<int64_t> out(static_cast<size_t>(element_count(v.shape)));
        std::memcpy(out.data(), weights_host_.data() + v.weight_off, out.size() * 8);
        return out;
    };
    std::vector<size_t> prepped_for_weight;  // not used yet
    (void)prepped_for_weight;

    // ---- operand extents of the data-movement and elementwise operators.
    // Their kernels index operands by the output's extents, so a graph whose
    // declared shapes disagree would read or write past a buffer: reject it.
    for (const auto& n : graph_.nodes) {
        const auto od = dims4(values_[n.output].shape);
        const int rank = static_cast<int>(values_[n.output].shape.size());
        if (n.op == Op::kConcat) {
            int axis = n.axis < 0 ? n.axis + rank : n.axis;
            if (axis < 0 || axis >= rank)
                throw std::runtime_error("mlvc-b200: Concat axis out of range");
            axis += 4 - rank;
            long long sum = 0;
            for (auto id : n.inputs) {
                const auto d = dims4(values_[id].shape);
                for (int l = 0; l < 4; ++l)
                    if (l != axis && d[l] != od[l])
                        throw std::runtime_error("mlvc-b200: Concat operand shapes do not match its output");
                sum += d[axis];
            }
            if (sum != od[axis])
                throw std::runtime_error("mlvc-b200: Concat operand shapes do not match its output");
        } else if (n.op == Op::kSlice) {
            const Value& av = values_[n.inputs[0]];
            const int arank = static_cast<int>(av.shape.size());
            if (arank != rank)
                throw std::runtime_error("mlvc-b200: Slice changes the tensor rank");
            const auto id4 = dims4(av.shape);
            const auto starts = int64s(n.inputs[1]);
            const auto axes = n.inputs.size() > 3 && n.inputs[3] ? int64s(n.inputs[3]) : std::vector<int64_t>{};
            const auto stepv = n.inputs.size() > 4 && n.inputs[4] ? int64s(n.inputs[4]) : std::vector<int64_t>{};
            std::array<long long, 4> start4{0, 0, 0, 0}, step4{1, 1, 1, 1};
            for (size_t k = 0; k < starts.size(); ++k) {
                long long axis = axes.empty() ? static_cast<long long>(k) : axes.at(k);
                if (axis < 0)
                    axis += arank;
                if (axis < 0 || axis >= arank)
                    throw std::runtime_error("mlvc-b200: Slice axis out of range");
                axis += 4 - arank;
                long long st0 = starts[k];
                if (st0 < 0)
                    st0 += id4[axis];
                // clamped to [0, dim] like the reference CPU plan
                // (backends/cpu/src/execution_plan.cpp:596-599)
                start4[axis] = std::clamp<long long>(st0, 0, id4[axis]);
                if (!stepv.empty())
                    step4[axis] = stepv.at(k);
            }
            for (int l = 0; l < 4; ++l) {
                const long long last = start4[l] + (od[l] - 1) * step4[l];
                if (start4[l] < 0 || start4[l] >= id4[l] || last < 0 || last >= id4[l])
                    throw std::runtime_error("mlvc-b200: Slice output exceeds its input");
            }
        } else if (n.op == Op::kAdd || n.op == Op::kSub || n.op == Op::kMul) {
            for (auto id : n.inputs) {
                const auto d = dims4(values_[id].shape);
                for (int l = 0; l < 4; ++l)
                    if (d[l] != 1 && d[l] != od[l])
                        throw std::runtime_error("mlvc-b200: binary operand does not broadcast to the output shape");
            }
        } else if (n.op == Op::kLeakyRelu || n.op == Op::kClip || n.op == Op::kSigmoid || n.op == Op::kReciprocal ||
                   n.op == Op::kRound) {
            if (dims4(values_[n.inputs[0]].shape) != od)
                throw std::runtime_error("mlvc-b200: elementwise operator changes the tensor shape");
        } else if (n.op == Op::kGather) {
            // one row of the table per index; the kernel copies one row
            const auto& dshape = values_[n.inputs[0]].shape;
            const long long idx = element_count(values_[n.inputs[1]].shape);
            const long long row = dshape.empty() || dshape[0] <= 0 ? 0 : element_count(dshape) / dshape[0];
            if (idx != 1 || element_count(values_[n.output].shape) != row)
                throw std::runtime_error("mlvc-b200: Gather takes one index and produces one table row");
        } else if (n.op == Op::kConv) {
            const auto& x = values_[n.inputs[0]].shape;
            const auto& w = values_[n.inputs[1]].shape;
            const auto& o = values_[n.output].shape;
            // the conv kernels index NCHW / OIHW operands: every Conv is rank 4
            // (the reference's exporter emits nothing else, aot.py:161-168)
            if (x.size() != 4 || w.size() != 4 || o.size() != 4)
                throw std::runtime_error("mlvc-b200: Conv input, weights and output must be rank 4");
            {
                const long long g = n.groups, sh = n.strides[0], sw = n.strides[1], ph = n.pads[0], pw = n.pads[1];
                const long long oh = (x[2] + 2 * ph - w[2]) / sh + 1, ow = (x[3] + 2 * pw - w[3]) / sw + 1;
                const bool bias_ok = n.inputs.size() < 3 || !n.inputs[2] ||
                                     element_count(values_[n.inputs[2]].shape) == w[0];
                if (sh <= 0 || sw <= 0 || x[2] + 2 * ph < w[2] || x[3] + 2 * pw < w[3] || o[0] != x[0] ||
                    o[1] != w[0] || x[1] != w[1] * g || w[0] % g || o[2] != oh || o[3] != ow || !bias_ok)
                    throw std::runtime_error("mlvc-b200: Conv shapes do not match its input, weights and attributes");
            }
        } else if (n.op == Op::kDepthToSpace || n.op == Op::kSpaceToDepth) {
            const auto d = dims4(values_[n.inputs[0]].shape);
            const long long r = n.block, rr = r * r;
            const std::array<long long, 4> want =
                n.op == Op::kDepthToSpace ? std::array<long long, 4>{d[0], d[1] / rr, d[2] * r, d[3] * r}
                                          : std::array<long long, 4>{d[0], d[1] * rr, d[2] / r, d[3] / r};
            const bool divisible = n.op == Op::kDepthToSpace ? d[1] % rr == 0 : d[2] % r == 0 && d[3] % r == 0;
            if (!divisible || want[0] != od[0] || want[1] != od[1] || want[2] != od[2] || want[3] != od[3])
                throw std::runtime_error("mlvc-b200: pixel (un)shuffle output shape does not match its input");
        }
    }

    // ---- boundary: NCHW host layout <-> NHWC device layout.  A SpaceToDepth
    // that is the only consumer of a graph input, and a DepthToSpace that
    // produces a graph output from a private tensor, are folded into the
    // conversion kernel (one pass over the data instead of two).
    std::vector<bool> absorbed(graph_.nodes.size(), false);
    auto needs_conversion = [&](const Value& v) {
        const auto d = dims4(v.shape);
        return v.nhwc && d[1] > 1 && d[2] * d[3] > 1;
    };
    auto boundary_step = [&](uint32_t host_id, uint32_t dev_id, int r, bool to_host, size_t k) {
        Step s;
        s.kernel = "mlvc_boundary_f16";
        s.info.kernel = s.kernel;
        s.info.nodes = std::string(to_host ? "output:" : "input:") + graph_.tensors[host_id].name +
                       (r > 1 ? (to_host ? "+depth_to_space" : "+space_to_depth") : "");
        s.info.bytes = 2.0 * values_[host_id].bytes;
        if (to_host)
            s.reads = {dev_id};
        else
            s.writes = {dev_id};
        const auto dd = dims4(values_[dev_id].shape);  // device tensor, logical NCHW extents
        const int tiles_x = static_cast<int>((dd[3] + 31) / 32);
        s.grid = static_cast<unsigned>(dd[0] * dd[2] * tiles_x);
        s.block = 256;
        // tile of host rows: scalar path pitch 32r+1, vector path 32r+8 halfs
        s.smem = static_cast<unsigned>((dd[1] / (r * r)) * r * (32 * r + 8) * 2);
        s.build = [this, dev_id, dd, r, to_host, k](Step& st) {
            BoundaryParams p{};
            const CUdeviceptr stage = to_host ? output_stage_dev_.at(k).get() : input_stage_dev_.at(k).get();
            p.src = reinterpret_cast<const mlvc_half*>(to_host ? values_[dev_id].addr : stage);
            p.dst = reinterpret_cast<mlvc_half*>(to_host ? stage : values_[dev_id].addr);
            p.n = static_cast<int>(dd[0]);
            p.c = static_cast<int>(dd[1]);
            p.h = static_cast<int>(dd[2]);
            p.w = static_cast<int>(dd[3]);
            p.r = r;
            p.to_host = to_host ? 1 : 0;
            st.set(p);
        };
        return s;
    };
    for (size_t k = 0; k < ext_inputs_.size(); ++k) {
        const uint32_t id = graph_.inputs[ext_inputs_[k]];
        const Value& v = values_[id];
        if (!needs_conversion(v))
            continue;
        uint32_t dev_id = id;
        int r = 1;
        if (v.consumers == 1 && !v.graph_output) {
            for (size_t j = 0; j < graph_.nodes.size(); ++j) {
                const NodeDesc& n = graph_.nodes[j];
                if (n.op == Op::kSpaceToDepth && n.inputs[0] == id && v.shape[2] % n.block == 0 &&
                    v.shape[3] % n.block == 0) {
                    absorbed[j] = true;
                    dev_id = n.output;
                    r = n.block;
                }
            }
        }
        steps_.push_back(boundary_step(id, dev_id, r, false, k));
    }
    std::vector<std::pair<uint32_t, int>> output_source(ext_outputs_.size(), {0, 1});
    for (size_t k = 0; k < ext_outputs_.size(); ++k) {
        const uint32_t id = graph_.outputs[ext_outputs_[k]];
        output_source[k] = {id, 1};
        if (!needs_conversion(values_[id]))
            continue;
        for (size_t j = 0; j < graph_.nodes.size(); ++j) {
            const NodeDesc& n = graph_.nodes[j];
            if (n.output != id || n.op != Op::kDepthToSpace)
                continue;
            const uint32_t t = n.inputs[0];
            if (values_[t].nhwc && values_[t].consumers == 1 && !values_[t].graph_output &&
                values_[t].kind != Value::kInput && values_[t].kind != Value::kState && values_[id].consumers == 0) {
                absorbed[j] = true;
                output_source[k] = {t, n.block};
                absorbed_outputs_.push_back(id);
            }
        }
    }

    auto& nodes = graph_.nodes;
    auto only_consumer = [&](uint32_t id) { return values_[id].consumers == 1 && !values_[id].graph_output; };
    auto is_channel_slice = [&](const NodeDesc& n, uint32_t src, int64_t begin, int64_t end) {
        if (n.op != Op::kSlice || n.inputs[0] != src)
            return false;
        const auto starts = int64s(n.inputs[1]);
        const auto axes = n.inputs.size() > 3 && n.inputs[3] ? int64s(n.inputs[3]) : std::vector<int64_t>{0};
        const auto steps = n.inputs.size() > 4 && n.inputs[4] ? int64s(n.inputs[4]) : std::vector<int64_t>{1};
        const auto& in = values_[src].shape;
        const auto& out = values_[n.output].shape;
        if (starts.size() != 1 || axes.size() != 1 || steps.size() != 1 || in.size() != 4)
            return false;
        const int64_t axis = axes[0] < 0 ? axes[0] + 4 : axes[0];
        return axis == 1 && steps[0] == 1 && starts[0] == begin && out[1] == end - begin && out[0] == in[0] &&
               out[2] == in[2] && out[3] == in[3];
    };
    // ReGLU tail at nodes [i, i+3]: Slice(T, 0:C), Slice(T, C:2C), Clip(first), Mul(clip, second).
    auto match_reglu_tail = [&](size_t i, uint32_t t_id, float& lo, float& hi) -> bool {
        if (i + 3 >= nodes.size())
            return false;
        const auto &s1 = nodes[i], &s2 = nodes[i + 1], &cl = nodes[i + 2], &mu = nodes[i + 3];
        if (s1.op != Op::kSlice || s2.op != Op::kSlice || cl.op != Op::kClip || mu.op != Op::kMul)
            return false;
        const Value& t = values_[t_id];
        if (t.shape.size() != 4 || t.shape[1] % 2 || values_[t_id].graph_output || t.consumers != 2)
            return false;
        const int64_t c = t.shape[1] / 2;
        if (!is_channel_slice(s1, t_id, 0, c) || !is_channel_slice(s2, t_id, c, 2 * c))
            return false;
        if (cl.inputs[0] != s1.output || mu.inputs.size() != 2 || mu.inputs[0] != cl.output ||
            mu.inputs[1] != s2.output)
            return false;
        if (!only_consumer(s1.output) || !only_consumer(s2.output) || !only_consumer(cl.output))
            return false;
        lo = cl.inputs.size() > 1 ? scalar(cl.inputs[1], -INFINITY) : -INFINITY;
        hi = cl.inputs.size() > 2 ? scalar(cl.inputs[2], INFINITY) : INFINITY;
        return values_[mu.output].shape == values_[s1.output].shape;
    };

    // Conv at node ci followed by LeakyRelu or Add of a same-shape NHWC tensor:
    // sets the fused epilogue and returns the number of nodes the step covers.
    auto conv_epilogue = [&](size_t ci, int& epi, float& alpha, uint32_t& out_id, uint32_t& res_id) -> size_t {
        const NodeDesc& n = nodes[ci];
        const auto& oshape = values_[n.output].shape;
        epi = kEpiBias;
        out_id = n.output;
        res_id = 0;
        if (!only_consumer(n.output) || ci + 1 >= nodes.size())
            return 1;
        const NodeDesc& e = nodes[ci + 1];
        if (e.op == Op::kLeakyRelu && e.inputs[0] == n.output) {
            epi = kEpiLeaky;
            alpha = e.alpha;
            out_id = e.output;
            return 2;
        }
        if (e.op == Op::kAdd && (e.inputs[0] == n.output || e.inputs[1] == n.output)) {
            const uint32_t r = e.inputs[0] == n.output ? e.inputs[1] : e.inputs[0];
            if (r != n.output && values_[r].nhwc && values_[r].shape == oshape && values_[e.output].shape == oshape) {
                epi = kEpiResidual;
                res_id = r;
                out_id = e.output;
                return 2;
            }
        }
        return 1;
    };

    // Channel concats read in place by the 1x1 conv right after them: a Concat
    // of two NHWC tensors (channels multiples of 64) whose only consumer is the
    // next node, a plain 1x1 conv with tensor-core output channels, is not
    // materialised; the conv streams its K panels from both tensors
    // (ConvTcParams::a_split).
    // An operand that is a channel slice of a wider NHWC tensor, consumed only
    // by the concat, is read in place as well: its A map starts at the slice's
    // first channel and steps by the wider tensor's row (the slice is not
    // materialised either).
    struct ConcatSrc {
        uint32_t a, b;  // tensors the two K ranges are read from
        int c1;         // channels of the first operand
        int a_off, a_row, b_off, b_row;  // first channel and row width (channels) within a / b
    };
    std::map<uint32_t, ConcatSrc> concat_src;  // concat output -> its two sources
    auto channel_view = [&](uint32_t id, uint32_t& base, int& off, int& row, size_t& slice_node) -> bool {
        if (!only_consumer(id))
            return false;
        for (size_t q = 0; q < nodes.size(); ++q) {
            const NodeDesc& sl = nodes[q];
            if (sl.output != id)
                continue;
            if (sl.op != Op::kSlice || absorbed[q])
                return false;
            const uint32_t src = sl.inputs[0];
            const Value& sv = values_[src];
            if (!sv.nhwc || sv.dtype != DType::kFp16 || sv.kind == Value::kWeight || sv.shape.size() != 4 ||
                sv.shape[1] % 8)
                return false;
            const auto starts = int64s(sl.inputs[1]);
            if (starts.size() != 1 || starts[0] < 0 || starts[0] % 8 ||
                !is_channel_slice(sl, src, starts[0], starts[0] + values_[id].shape[1]))
                return false;
            base = src;
            off = static_cast<int>(starts[0]);
            row = static_cast<int>(sv.shape[1]);
            slice_node = q;
            return true;
        }
        return false;
    };
    for (size_t j = 0; j + 1 < nodes.size(); ++j) {
        const NodeDesc& c = nodes[j];
        const NodeDesc& v = nodes[j + 1];
        if (c.op != Op::kConcat || absorbed[j] || c.inputs.size() != 2 || v.op != Op::kConv ||
            v.inputs[0] != c.output || !only_consumer(c.output))
            continue;
        const Value &o = values_[c.output], &va = values_[c.inputs[0]], &vb = values_[c.inputs[1]];
        if (!o.nhwc || !va.nhwc || !vb.nhwc || o.shape.size() != 4 || o.shape[0] != 1 || va.shape.size() != 4 ||
            vb.shape.size() != 4 || (c.axis != 1 && c.axis != -3))
            continue;
        const int c1 = static_cast<int>(va.shape[1]), c2 = static_cast<int>(vb.shape[1]);
        const Value& wv = values_[v.inputs[1]];
        if (c1 % 64 || c2 % 64 || c1 + c2 > 1024 || v.groups != 1 || v.strides[0] != 1 || v.strides[1] != 1 ||
            v.pads[0] != 0 || v.pads[1] != 0 || wv.kind != Value::kWeight || wv.dtype != DType::kFp16 ||
            wv.shape.size() != 4 || wv.shape[1] != c1 + c2 || wv.shape[2] != 1 || wv.shape[3] != 1 || wv.shape[0] % 8)
            continue;
        ConcatSrc cs{c.inputs[0], c.inputs[1], c1, 0, c1, 0, c2};
        uint32_t base = 0;
        int off = 0, row = 0;
        size_t qa = 0, qb = 0;
        const bool view_a = channel_view(c.inputs[0], base, off, row, qa);
        if (view_a) {
            cs.a = base;
            cs.a_off = off;
            cs.a_row = row;
        }
        const bool view_b = channel_view(c.inputs[1], base, off, row, qb);
        if (view_b) {
            cs.b = base;
            cs.b_off = off;
            cs.b_row = row;
        }
        concat_src[c.output] = cs;
        absorbed[j] = true;
        if (view_a)
            absorbed[qa] = true;
        if (view_b)
            absorbed[qb] = true;
    }

    for (size_t i = 0; i < nodes.size();) {
        const NodeDesc& n = nodes[i];
        if (absorbed[i]) {
            ++i;
            continue;
        }
        if (n.op == Op::kConv) {
            const uint32_t x_id = n.inputs[0], w_id = n.inputs[1];
            const uint32_t b_id = n.inputs.size() > 2 ? n.inputs[2] : 0;
            const Value &xv = values_[x_id], &wv = values_[w_id];
            if (wv.kind != Value::kWeight || wv.dtype != DType::kFp16 || xv.shape.size() != 4 || !xv.nhwc)
                throw std::runtime_error("mlvc-b200: Conv expects an NHWC FP16 activation and FP16 weights");
            if (b_id && values_[b_id].kind != Value::kWeight)
                throw std::runtime_error("mlvc-b200: Conv bias must be an initializer");
            const int N = static_cast<int>(xv.shape[0]), IC = static_cast<int>(xv.shape[1]);
            const int IH = static_cast<int>(xv.shape[2]), IW = static_cast<int>(xv.shape[3]);
            const int OC = static_cast<int>(wv.shape[0]), ICG = static_cast<int>(wv.shape[1]);
            const int KH = static_cast<int>(wv.shape[2]), KW = static_cast<int>(wv.shape[3]);
            const int SH = n.strides[0], SW = n.strides[1], PH = n.pads[0], PW = n.pads[1], G = n.groups;
            const auto& oshape = values_[n.output].shape;
            const int OH = static_cast<int>(oshape[2]), OW = static_cast<int>(oshape[3]);

            // ---- fusion detection
            int epi = kEpiBias;
            float alpha = 0.0f, lo = 0.0f, hi = 0.0f;
            uint32_t out_id = n.output, res_id = 0;
            size_t consumed = conv_epilogue(i, epi, alpha, out_id, res_id);
            const bool is1x1 = G == 1 && KH == 1 && KW == 1 && SH == 1 && SW == 1 && PH == 0 && PW == 0;
            bool reglu = false;
            if (epi == kEpiBias && is1x1 && match_reglu_tail(i + 1, n.output, lo, hi)) {
                reglu = true;
                epi = kEpiReglu;
                out_id = nodes[i + 4].output;
                consumed = 5;
            }
            const uint16_t* w = wdata(w_id);
            const uint16_t* bias = b_id ? wdata(b_id) : nullptr;
            std::vector<uint16_t> bias_full(OC, 0);
            if (bias)
                std::copy(bias, bias + OC, bias_full.begin());

            const auto split_it = concat_src.find(x_id);
            const bool split_a = split_it != concat_src.end();  // x is a concat read in place (1x1 path only)
            Step s;
            s.reads = split_a ? std::vector<uint32_t>{split_it->second.a, split_it->second.b} : std::vector<uint32_t>{x_id};
            if (res_id)
                s.reads.push_back(res_id);
            s.writes = {out_id};
            {
                std::ostringstream os;
                os << i;
                if (consumed > 1)
                    os << "-" << (i + consumed - 1);
                s.info.nodes = os.str();
            }
            s.info.flops = 2.0 * N * OH * OW * static_cast<double>(OC) * ICG * KH * KW;
            const double out_elems = static_cast<double>(element_count(values_[out_id].shape));
            // algorithmic bytes: one read of each distinct tensor, one write of the output
            s.info.bytes = 2.0 * (element_count(xv.shape) + element_count(wv.shape) + (bias ? OC : 0) + out_elems +
                                  (res_id && res_id != x_id ? out_elems : 0));

            const bool tc_shape = G == 1 && N == 1 && IC % 8 == 0 && OC % 8 == 0 && (!reglu || OC % 64 == 0);
            const int header = kTcHeaderBytes;
            const int smem_cap = max_smem_optin_ - 1024;  // slack for the in-kernel 1024-byte alignment
            if (reglu && tc_shape && is1x1 && ffn_fusion_ && !split_a && i + 5 < nodes.size() && IC % 64 == 0 && IC <= 256 &&
                (OC / 2) % kFfnChunk == 0 && OC / 2 <= kFfnMaxHidden) {
                // ---- fused feed-forward block: this ReGLU conv and the 1x1 conv that
                // consumes its output, with the hidden tensor kept on chip
                const NodeDesc& n2 = nodes[i + 5];
                const int H = OC / 2;
                const uint32_t hid_id = out_id;
                bool ok = n2.op == Op::kConv && n2.inputs[0] == hid_id && only_consumer(hid_id) && n2.groups == 1 &&
                          n2.strides[0] == 1 && n2.strides[1] == 1 && n2.pads[0] == 0 && n2.pads[1] == 0;
                const uint32_t w2_id = ok ? n2.inputs[1] : 0;
                const uint32_t b2_id = ok && n2.inputs.size() > 2 ? n2.inputs[2] : 0;
                int OC2 = 0;
                if (ok) {
                    const Value& w2v = values_[w2_id];
                    ok = w2v.kind == Value::kWeight && w2v.dtype == DType::kFp16 && w2v.shape.size() == 4 &&
                         w2v.shape[1] == H && w2v.shape[2] == 1 && w2v.shape[3] == 1 &&
                         (!b2_id || values_[b2_id].kind == Value::kWeight);
                    OC2 = ok ? static_cast<int>(w2v.shape[0]) : 0;
                    // output tile staged in the two hidden panels: at most 128 columns
                    ok = ok && OC2 % 64 == 0 && OC2 <= 128;
                }
                const int kpan = IC / 64, M = IH * IW;
                const int slot = std::max(16384, OC2 * 128);
                const int m_tiles = (M + 127) / 128;
                const int grid = std::min(m_tiles, sm_count_);
                const int per_cta = (m_tiles + grid - 1) / grid;
                // Fixed part: alignment slack, header, two hidden panels (which are
                // also the output staging buffers).
                const int fixed = 1024 + kFfnHeaderBytes + 2 * 16384;
                auto ws_for = [&](int xs) { return (max_smem_optin_ - fixed - xs * kpan * 16384) / slot; };
                int xs = per_cta > 1 && ws_for(2) >= 6 ? 2 : 1;
                const int ws = std::min(kFfnMaxWStages, ws_for(xs));
                // One CTA per SM (above half of the SM's shared memory): its 512 TMEM
                // columns never wait for another CTA's.
                const int ffn_smem = fixed + xs * kpan * 16384 + ws * slot;
                int epi2 = kEpiBias;
                float alpha2 = 0.0f;
                uint32_t out2 = 0, res2 = 0;
                const size_t consumed2 = ok ? conv_epilogue(i + 5, epi2, alpha2, out2, res2) : 0;
                // The residual is read from the X tile in shared memory: only the
                // FFN input itself can be the residual.
                ok = ok && (res2 == 0 || res2 == x_id);
                if (ok && ws >= 2 && ffn_smem > 233472 / 2) {
                    // W1 rows in chunk order: per 64 hidden channels, 64 gate rows then 64 linear rows.
                    std::vector<uint16_t> w1p(static_cast<size_t>(OC) * IC), b1p(OC);
                    for (int r = 0; r < OC; ++r) {
                        const int j = r / 128, k = r % 128;
                        const int src = k < 64 ? j * 64 + k : H + j * 64 + (k - 64);
                        std::memcpy(&w1p[static_cast<size_t>(r) * IC], w + static_cast<size_t>(src) * IC, IC * 2);
                        b1p[r] = bias_full[src];
                    }
                    std::vector<uint16_t> b2p(OC2, 0);
                    if (b2_id)
                        std::copy(wdata(b2_id), wdata(b2_id) + OC2, b2p.begin());
                    const size_t w1_off = prep(w1p.data(), w1p.size() * 2);
                    const size_t b1_off = prep(b1p.data(), b1p.size() * 2);
                    const size_t w2_off = prep(wdata(w2_id), static_cast<size_t>(OC2) * H * 2);
                    const size_t b2_off = prep(b2p.data(), b2p.size() * 2);
                    Step f;
                    f.reads = {x_id};
                    if (res2)
                        f.reads.push_back(res2);
                    f.writes = {out2};
                    {
                        std::ostringstream os;
                        os << i << "-" << (i + 5 + consumed2 - 1);
                        f.info.nodes = os.str();
                    }
                    f.info.flops = 2.0 * M * (static_cast<double>(OC) * IC + static_cast<double>(OC2) * H);
                    f.info.bytes = 2.0 * (static_cast<double>(M) * IC + static_cast<double>(OC) * IC + OC +
                                          static_cast<double>(OC2) * H + OC2 +
                                          static_cast<double>(M) * OC2 * (res2 && res2 != x_id ? 2 : 1));
                    f.kernel = "mlvc_ffn_tc";
                    f.info.kernel = f.kernel;
                    f.smem = static_cast<unsigned>(ffn_smem);
                    f.block = 320;
                    f.grid = static_cast<unsigned>(grid);
                    const float clip_lo = lo, clip_hi = hi;
                    f.build = [=, this](Step& st) {
                        FfnTcParams fp{};
                        ConvTcParams& p = fp.c;
                        const cuuint32_t elem1[2] = {1, 1};
                        auto encode = [&](CUtensorMap* map, CUdeviceptr addr, cuuint64_t cols, cuuint64_t rows,
                                          cuuint32_t box_cols, cuuint32_t box_rows, CUtensorMapSwizzle swz,
                                          const char* what) {
                            const cuuint64_t dims[2] = {cols, rows};
                            const cuuint64_t strides[1] = {cols * 2};
                            const cuuint32_t box[2] = {box_cols, box_rows};
                            check(cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                                         reinterpret_cast<void*>(addr), dims, strides, box, elem1,
                                                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  what);
                        };
                        encode(&p.map_a0, values_[x_id].addr, IC, M, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B,
                               "cuTensorMapEncodeTiled(ffn X)");
                        encode(&p.map_b, prepped_dev_.get() + w1_off, IC, OC, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B,
                               "cuTensorMapEncodeTiled(ffn W1)");
                        encode(&fp.map_w2, prepped_dev_.get() + w2_off, H, OC2, 64, static_cast<cuuint32_t>(OC2),
                               CU_TENSOR_MAP_SWIZZLE_128B, "cuTensorMapEncodeTiled(ffn W2)");
                        encode_tile_map(&p.map_out, values_[out2].addr, OC2, M, 0, 0, "cuTensorMapEncodeTiled(ffn out)");
                        p.map_res = p.map_out;  // unused: the residual comes from the X tile
                        p.map_a1 = p.map_a0;
                        p.bias = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b2_off);
                        p.out = reinterpret_cast<mlvc_half*>(values_[out2].addr);
                        p.M = M;
                        p.N = OC2;
                        p.n_valid = OC2;
                        p.K = IC;
                        p.BN = OC2;
                        p.n_tiles = 1;
                        p.m_tiles = m_tiles;
                        p.epilogue = epi2;
                        p.alpha = alpha2;
                        p.clip_lo = clip_lo;
                        p.clip_hi = clip_hi;
                        p.a_stages = xs;
                        p.b_stages = ws;
                        fp.bias1 = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b1_off);
                        fp.hidden = H;
                        fp.w_slot_bytes = slot;
                        st.set(fp);
                    };
                    steps_.push_back(std::move(f));
                    i += 5 + consumed2;
                    continue;
                }
            }
            if (tc_shape && is1x1 && !reglu && mb_fusion_ && !split_a && (epi == kEpiBias || epi == kEpiLeaky) && IC % 64 == 0 &&
                IC <= 128 && OC % 64 == 0 && OC <= kMbMaxExpand && i + consumed + 1 < nodes.size()) {
                // ---- fused inverted-residual block: this expand conv, the depthwise
                // 3x3 that consumes it and the 1x1 projection of the depthwise
                // result, with both intermediates kept on chip
                const uint32_t e_id = out_id;
                const NodeDesc& nd = nodes[i + consumed];
                bool ok = nd.op == Op::kConv && nd.inputs[0] == e_id && only_consumer(e_id) && nd.groups == OC &&
                          nd.strides[0] == 1 && nd.strides[1] == 1 && nd.pads[0] == 1 && nd.pads[1] == 1;
                const uint32_t wd_id = ok ? nd.inputs[1] : 0;
                const uint32_t bd_id = ok && nd.inputs.size() > 2 ? nd.inputs[2] : 0;
                if (ok) {
                    const Value& wdv = values_[wd_id];
                    ok = wdv.kind == Value::kWeight && wdv.dtype == DType::kFp16 &&
                         wdv.shape == std::vector<int64_t>{OC, 1, 3, 3} && (!bd_id || values_[bd_id].kind == Value::kWeight) &&
                         values_[nd.output].shape == values_[e_id].shape && only_consumer(nd.output);
                }
                const size_t pj = i + consumed + 1;
                const NodeDesc& np = nodes[pj];
                ok = ok && np.op == Op::kConv && np.inputs[0] == nd.output && np.groups == 1 && np.strides[0] == 1 &&
                     np.strides[1] == 1 && np.pads[0] == 0 && np.pads[1] == 0;
                const uint32_t w2_id = ok ? np.inputs[1] : 0;
                const uint32_t b2_id = ok && np.inputs.size() > 2 ? np.inputs[2] : 0;
                int OC2 = 0;
                if (ok) {
                    const Value& w2v = values_[w2_id];
                    ok = w2v.kind == Value::kWeight && w2v.dtype == DType::kFp16 && w2v.shape.size() == 4 &&
                         w2v.shape[1] == OC && w2v.shape[2] == 1 && w2v.shape[3] == 1 &&
                         (!b2_id || values_[b2_id].kind == Value::kWeight);
                    OC2 = ok ? static_cast<int>(w2v.shape[0]) : 0;
                    // one W2 K slice per ring slot, output staged in its own panels
                    ok = ok && OC2 % 64 == 0 && OC2 <= 128;
                }
                const int kpx = IC / 64, panels2 = OC2 / 64;
                // header, x halo slices, two e chunk buffers (180 rows x 128 bytes),
                // two A panels, weight ring, output staging, depthwise taps + bias
                const int mb_smem = 1024 + kMbHeaderBytes + kpx * kMbSliceBytes + 2 * 180 * 128 + 2 * 16384 +
                                    kMbWStages * kMbWSlotBytes + panels2 * kTcStagePanelBytes + 10 * OC * 2;
                if (ok && mb_smem <= max_smem_optin_) {
                    int epi2 = kEpiBias;
                    float alpha2 = 0.0f;
                    uint32_t out2 = 0, res2 = 0;
                    const size_t consumed2 = conv_epilogue(pj, epi2, alpha2, out2, res2);
                    const uint16_t* wd = wdata(wd_id);
                    std::vector<uint16_t> dwp(static_cast<size_t>(10) * OC, 0);  // taps, then the bias row
                    for (int c = 0; c < OC; ++c)
                        for (int k = 0; k < 9; ++k)
                            dwp[static_cast<size_t>(k) * OC + c] = wd[static_cast<size_t>(c) * 9 + k];
                    if (bd_id)
                        std::copy(wdata(bd_id), wdata(bd_id) + OC, dwp.begin() + static_cast<size_t>(9) * OC);
                    std::vector<uint16_t> b2p(OC2, 0);
                    if (b2_id)
                        std::copy(wdata(b2_id), wdata(b2_id) + OC2, b2p.begin());
                    const size_t w1_off = prep(w, static_cast<size_t>(OC) * IC * 2);
                    const size_t b1_off = prep(bias_full.data(), bias_full.size() * 2);
                    const size_t dww_off = prep(dwp.data(), dwp.size() * 2);
                    const size_t w2_off = prep(wdata(w2_id), static_cast<size_t>(OC2) * OC * 2);
                    const size_t b2_off = prep(b2p.data(), b2p.size() * 2);
                    const int M = IH * IW;
                    const int tiles_x = (IW + kDwTileW - 1) / kDwTileW, tiles_y = (IH + kDwTileH - 1) / kDwTileH;
                    const int m_tiles = tiles_x * tiles_y;
                    Step f;
                    f.reads = {x_id};
                    if (res2)
                        f.reads.push_back(res2);
                    f.writes = {out2};
                    f.info.nodes = std::to_string(i) + "-" + std::to_string(pj + consumed2 - 1);
                    f.info.flops = 2.0 * M * static_cast<double>(IC) * OC + 18.0 * M * OC + 2.0 * M * static_cast<double>(OC) * OC2;
                    f.info.bytes = 2.0 * (static_cast<double>(M) * IC + static_cast<double>(OC) * IC + OC + 10.0 * OC +
                                          static_cast<double>(OC2) * OC + OC2 +
                                          static_cast<double>(M) * OC2 * (res2 && res2 != x_id ? 2 : 1));
                    f.kernel = "mlvc_mbconv_tc";
                    f.info.kernel = f.kernel;
                    f.smem = static_cast<unsigned>(mb_smem);
                    f.block = kMbBlockThreads;
                    f.grid = static_cast<unsigned>(std::min(m_tiles, sm_count_));
                    const int E = OC, C = IC;
                    const int epi1 = epi;
                    const float alpha1 = alpha;
                    f.build = [=, this](Step& st) {
                        MbConvTcParams mp{};
                        ConvTcParams& p = mp.c;
                        const cuuint32_t elem1[2] = {1, 1};
                        auto encode2 = [&](CUtensorMap* map, CUdeviceptr addr, cuuint64_t cols, cuuint64_t rows,
                                           cuuint32_t box_cols, cuuint32_t box_rows, CUtensorMapSwizzle swz,
                                           const char* what) {
                            const cuuint64_t dims[2] = {cols, rows};
                            const cuuint64_t strides[1] = {cols * 2};
                            const cuuint32_t box[2] = {box_cols, box_rows};
                            check(cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                                         reinterpret_cast<void*>(addr), dims, strides, box, elem1,
                                                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  what);
                        };
                        {
                            const cuuint32_t elem3[3] = {1, 1, 1};
                            const cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(IW),
                                                        static_cast<cuuint64_t>(IH)};
                            const cuuint64_t strides[2] = {static_cast<cuuint64_t>(C) * 2,
                                                           static_cast<cuuint64_t>(IW) * C * 2};
                            const cuuint32_t box[3] = {64, kDwTileW + 2, kDwTileH + 2};
                            check(cuTensorMapEncodeTiled(&mp.map_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                                                         reinterpret_cast<void*>(values_[x_id].addr), dims, strides, box,
                                                         elem3, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(mbconv x halo)");
                        }
                        encode2(&mp.map_w1, prepped_dev_.get() + w1_off, C, E, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B,
                                "cuTensorMapEncodeTiled(mbconv W1)");
                        encode2(&p.map_b, prepped_dev_.get() + w2_off, E, OC2, 64, static_cast<cuuint32_t>(OC2),
                                CU_TENSOR_MAP_SWIZZLE_128B, "cuTensorMapEncodeTiled(mbconv W2)");
                        encode2(&mp.map_dw, prepped_dev_.get() + dww_off, E, 10, static_cast<cuuint32_t>(E), 10,
                                CU_TENSOR_MAP_SWIZZLE_NONE, "cuTensorMapEncodeTiled(mbconv taps)");
                        encode_tile_map(&p.map_out, values_[out2].addr, OC2, 0, IW, IH,
                                        "cuTensorMapEncodeTiled(mbconv out)", kDwTileW, kDwTileH);
                        if (res2)
                            encode_tile_map(&p.map_res, values_[res2].addr, OC2, 0, IW, IH,
                                            "cuTensorMapEncodeTiled(mbconv residual)", kDwTileW, kDwTileH);
                        else
                            p.map_res = p.map_out;
                        p.map_a0 = p.map_a1 = mp.map_x;
                        p.bias = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b2_off);
                        p.out = reinterpret_cast<mlvc_half*>(values_[out2].addr);
                        p.M = M;
                        p.N = OC2;
                        p.n_valid = OC2;
                        p.K = E;
                        p.BN = OC2;
                        p.n_tiles = 1;
                        p.m_tiles = m_tiles;
                        p.epilogue = epi2;
                        p.alpha = alpha2;
                        p.a_stages = 2;
                        p.b_stages = kMbWStages;
                        mp.bias1 = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b1_off);
                        mp.alpha1 = alpha1;
                        mp.epi1 = epi1;
                        mp.c_in = C;
                        mp.expand = E;
                        mp.width = IW;
                        mp.height = IH;
                        mp.tiles_x = tiles_x;
                        st.set(mp);
                    };
                    steps_.push_back(std::move(f));
                    i = pj + consumed2;
                    continue;
                }
            }
            if (tc_shape && is1x1) {
                // ---- tcgen05 GEMM
                // Weight rows padded to a multiple of 64: the epilogue stages and
                // stores 64-column panels (ReGLU: 64 output columns = 128 weight rows).
                const int K = IC, NN = (OC + 63) / 64 * 64;
                const int k_panels = (K + 63) / 64;
                // A 2x pixel shuffle (CRD) that is the only consumer of the conv's
                // output (after a bias or LeakyReLU epilogue) is folded into the
                // store: weight rows ordered [sub-pixel][channel], row-aligned
                // tiles, each 64-column panel stored through a 5-D view of the
                // shuffled output, so the 4C-channel tensor is never written.
                uint32_t d2s_out = 0;
                if (!reglu && epi != kEpiResidual && OC % 256 == 0 && i + consumed < nodes.size() && d2s_fusion_) {
                    const size_t di = i + consumed;
                    const NodeDesc& dn = nodes[di];
                    if (dn.op == Op::kDepthToSpace && dn.block == 2 && dn.inputs[0] == out_id && !absorbed[di] &&
                        only_consumer(out_id) && !values_[out_id].graph_output && values_[dn.output].nhwc)
                        d2s_out = dn.output;
                }
                const int row_tiles = (IW + 127) / 128;
                const int m_tiles = d2s_out ? IH * row_tiles : (IH * IW + 127) / 128;
                // Candidate N tiles divide NN and keep the CTA's weight slice resident.
                // Every N tile re-reads the activations from L2, and L2 -> SM traffic
                // paces these GEMMs once four A panels are in flight (a deeper ring
                // measured no faster), so the widest N tile that keeps four A stages
                // at one CTA per SM comes first (at 136 x 240: expand 256 -> 512
                // 17.3 -> 14.9 us, 256 -> 192 8.5 -> 6.7 us against 64-column tiles
                // at two CTAs per SM), as long as its tiles still occupy 80 % of the
                // SMs (on smaller planes the fill matters more: at 640 x 368 the
                // wide tiles cost 3-6 % of the frame).  Otherwise
                // (MLVC_B200_CONV1X1_POLICY=pair, or no such tile) a footprint that
                // lets two CTAs share an SM (<= 113 KB of smem, 2 x BN TMEM columns
                // <= 512), the largest BN that still gives one tile per SM, else
                // one CTA per SM.
                constexpr int kTwoCtaSmem = 233472 / 2 - 1024;
                auto stage_for = [&](int bn) { return (reglu ? bn / 2 : bn) / 64 * kTcStagePanelBytes; };
                std::vector<int> cands;
                for (int bn = std::min(256, NN); bn >= 64; bn -= 64)
                    if (NN % bn == 0 && (!reglu || bn % 128 == 0) &&
                        header + k_panels * bn * 128 + 2 * 16384 + stage_for(bn) <= smem_cap)
                        cands.push_back(bn);
                auto stages_for = [&](int bn, int cap) {
                    return (cap - header - 1024 - stage_for(bn) - k_panels * bn * 128) / 16384;
                };
                int best = 0, ctas_per_sm = 1;
                if (const char* e_pol = std::getenv("MLVC_B200_CONV1X1_POLICY"); !(e_pol && std::string(e_pol) == "pair"))
                    for (int bn : cands)  // largest N tile that keeps four A stages at one CTA per SM
                        if (!best && stages_for(bn, smem_cap + 1024) >= 4 && 5 * m_tiles * (NN / bn) >= 4 * sm_count_)
                            best = bn;
                for (int bn : cands)
                    if (!best && bn <= 128 && stages_for(bn, kTwoCtaSmem) >= 2 && m_tiles * (NN / bn) >= sm_count_) {
                        best = bn;
                        ctas_per_sm = 2;
                        break;
                    }
                if (!best)
                    for (int bn : cands)
                        if (bn <= 128 && stages_for(bn, kTwoCtaSmem) >= 2) {
                            best = bn;
                            ctas_per_sm = 2;
                            break;
                        }
                if (!best)
                    for (int bn : cands)
                        if (m_tiles * (NN / bn) >= sm_count_) {
                            best = bn;
                            break;
                        }
                if (!best && !cands.empty())
                    best = cands.back() >= 64 ? cands.back() : cands.front();
                {
                    // tuning override (sweeps): MLVC_B200_CONV1X1_BN = N tile when it is a
                    // candidate, MLVC_B200_CONV1X1_CTAS = CTAs per SM (1 or 2)
                    const char* e_bn = std::getenv("MLVC_B200_CONV1X1_BN");
                    const char* e_ct = std::getenv("MLVC_B200_CONV1X1_CTAS");
                    if (e_bn && std::find(cands.begin(), cands.end(), std::atoi(e_bn)) != cands.end()) {
                        best = std::atoi(e_bn);
                        ctas_per_sm = 1;
                    }
                    if (e_ct && (std::atoi(e_ct) == 1 ||
                                 (std::atoi(e_ct) == 2 && best <= 128 && stages_for(best, kTwoCtaSmem) >= 2)))
                        ctas_per_sm = std::atoi(e_ct);
                }
                if (best) {
                    const int BN = best, n_tiles = NN / BN;
                    if (d2s_out) {  // the step now also covers the pixel shuffle
                        out_id = d2s_out;
                        consumed += 1;
                        s.symbol = "mlvc_conv1x1_d2s_tc";
                        s.writes = {out_id};
                        s.info.nodes = std::to_string(i) + "-" + std::to_string(i + consumed - 1);
                    }
                    std::vector<uint16_t> wp(static_cast<size_t>(NN) * K, 0), bp(NN, 0);
                    for (int r = 0; r < OC; ++r) {
                        int src = r;
                        if (reglu) {  // interleave gate/linear halves per N tile
                            const int t = r / BN, j = r % BN, half = BN / 2, c = OC / 2;
                            src = j < half ? t * half + j : c + t * half + (j - half);
                        }
                        if (d2s_out) {  // row sub * C + c <- conv channel c * 4 + sub (CRD order)
                            const int C = OC / 4;
                            src = (r % C) * 4 + r / C;
                        }
                        std::memcpy(&wp[static_cast<size_t>(r) * K], w + static_cast<size_t>(src) * K, K * 2);
                        bp[r] = bias_full[src];
                    }
                    const size_t w_off = prep(wp.data(), wp.size() * 2);
                    const size_t b_off = prep(bp.data(), bp.size() * 2);
                    int a_stages =
                        std::min(8, ctas_per_sm == 2 ? stages_for(BN, kTwoCtaSmem) : stages_for(BN, smem_cap + 1024));
                    // Two output staging buffers when at least four A stages remain: a
                    // tile's rows are then written while the previous tile's TMA store
                    // still reads the other buffer (MLVC_B200_STAGE_BUFS=1: one buffer).
                    int stage_bufs = 1;
                    {
                        const int cap = ctas_per_sm == 2 ? kTwoCtaSmem : smem_cap + 1024;
                        const int with2 = (cap - header - 1024 - 2 * stage_for(BN) - k_panels * BN * 128) / 16384;
                        const char* e = std::getenv("MLVC_B200_STAGE_BUFS");
                        if (!(e && e[0] == '1') && with2 >= 4) {
                            stage_bufs = 2;
                            a_stages = std::min(8, with2);
                        }
                    }
                    {
                        // tuning override (sweeps): MLVC_B200_CONV1X1_STAGES caps the A ring depth
                        const char* e_st = std::getenv("MLVC_B200_CONV1X1_STAGES");
                        if (e_st && std::atoi(e_st) >= 2)
                            a_stages = std::min(a_stages, std::atoi(e_st));
                    }
                    if (a_stages < 2)  // the A ring needs two slots (load one while the MMA reads the other)
                        throw std::runtime_error("mlvc-b200: conv1x1 plan leaves fewer than two A stages");
                    const int slots = sm_count_ * ctas_per_sm;
                    const int grid = n_tiles * std::max(1, std::min(m_tiles, slots / n_tiles));
                    s.kernel = "mlvc_conv1x1_tc";
                    s.info.kernel = s.kernel;
                    s.smem = static_cast<unsigned>(header + k_panels * BN * 128 + a_stages * 16384 +
                                                   stage_bufs * stage_for(BN) + 1024);
                    s.block = 320;
                    s.grid = static_cast<unsigned>(grid);
                    const int M = IH * IW;
                    // A sources: x itself, or the two tensors of a concat read in place
                    const uint32_t a0_id = split_a ? split_it->second.a : x_id;
                    const uint32_t a1_id = split_a ? split_it->second.b : 0;
                    const int c0 = split_a ? split_it->second.c1 : K;
                    const int a0_off = split_a ? split_it->second.a_off : 0, a0_row = split_a ? split_it->second.a_row : K;
                    const int a1_off = split_a ? split_it->second.b_off : 0, a1_row = split_a ? split_it->second.b_row : 0;
                    s.build = [=, this](Step& st) {
                        ConvTcParams p{};
                        const CUdeviceptr wdev = prepped_dev_.get() + w_off;
                        const cuuint32_t elem1[2] = {1, 1};
                        // channels [off, off + channels) of a tensor whose rows hold `row` channels
                        auto encode_a = [&](CUtensorMap* map, uint32_t id, int channels, int off, int row,
                                            const char* what) {
                            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(channels), static_cast<cuuint64_t>(M)};
                            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row) * 2};
                            const cuuint32_t box[2] = {64, 128};
                            check(cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                                         reinterpret_cast<void*>(values_[id].addr + off * 2), dims,
                                                         strides, box,
                                                         elem1, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  what);
                        };
                        encode_a(&p.map_a0, a0_id, c0, a0_off, a0_row, "cuTensorMapEncodeTiled(conv1x1 A)");
                        {
                            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(NN)};
                            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
                            const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(BN)};
                            check(cuTensorMapEncodeTiled(&p.map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                                         reinterpret_cast<void*>(wdev), dims, strides, box, elem1,
                                                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(conv1x1 B)");
                        }
                        if (a1_id) {
                            encode_a(&p.map_a1, a1_id, K - c0, a1_off, a1_row,
                                     "cuTensorMapEncodeTiled(conv1x1 A, second concat operand)");
                            p.a_split = c0 / 64;
                        } else {
                            p.map_a1 = p.map_a0;
                        }
                        if (d2s_out) {
                            // {C, dx, x, dy, y}: the packed [2 IH][2 IW][C] output seen from the input pixels
                            const cuuint64_t C = static_cast<cuuint64_t>(OC / 4);
                            const cuuint64_t dims[5] = {C, 2, static_cast<cuuint64_t>(IW), 2, static_cast<cuuint64_t>(IH)};
                            const cuuint64_t strides[4] = {C * 2, 2 * C * 2, 2 * static_cast<cuuint64_t>(IW) * C * 2,
                                                           4 * static_cast<cuuint64_t>(IW) * C * 2};
                            const cuuint32_t box[5] = {64, 1, 128, 1, 1};
                            const cuuint32_t elem5[5] = {1, 1, 1, 1, 1};
                            check(cuTensorMapEncodeTiled(&p.map_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                                                         reinterpret_cast<void*>(values_[out_id].addr), dims, strides,
                                                         box, elem5, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(conv1x1 out, pixel shuffle)");
                            p.d2s_c = OC / 4;
                            p.row_tiles = row_tiles;
                            p.in_w = IW;
                            p.in_h = IH;
                        } else {
                            encode_tile_map(&p.map_out, values_[out_id].addr, reglu ? OC / 2 : OC, M, 0, 0,
                                            "cuTensorMapEncodeTiled(conv1x1 out)");
                        }
                        if (res_id)
                            encode_tile_map(&p.map_res, values_[res_id].addr, OC, M, 0, 0,
                                            "cuTensorMapEncodeTiled(conv1x1 residual)");
                        else
                            p.map_res = p.map_out;
                        p.bias = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b_off);
                        p.out = reinterpret_cast<mlvc_half*>(values_[out_id].addr);
                        p.M = M;
                        p.N = NN;
                        p.n_valid = OC;
                        p.K = K;
                        p.BN = BN;
                        p.n_tiles = n_tiles;
                        p.m_tiles = m_tiles;
                        p.epilogue = epi;
                        p.alpha = alpha;
                        p.clip_lo = lo;
                        p.clip_hi = hi;
                        p.a_stages = a_stages;
                        p.stage_bufs = stage_bufs;
                        st.set(p);
                    };
                    steps_.push_back(std::move(s));
                    i += consumed;
                    continue;
                }
            }
            if (tc_shape && IC % 64 == 0 && !is1x1 && !reglu && (SH == 1 || SH == 2) && SH == SW &&
                KH <= 8 && KW <= 8 &&
                PH == PW && PW < KW && OW >= 1) {
                // ---- tcgen05 implicit GEMM with halo tiles
                const int stride = SH, pad = PW, taps = KH * KW, k_panels = IC / 64;
                int px_min, halo_px;
                if (stride == 1) {
                    px_min = -pad;
                    halo_px = 128 + KW - 1;
                } else {
                    px_min = -((pad + 1) / 2);
                    const int max_pair = (KW - 1 - pad) >= 0 ? (KW - 1 - pad) / 2 : -((pad - KW + 2) / 2);
                    halo_px = 128 + max_pair - px_min;
                }
                const int parities = stride;
                const int chunk_bytes = static_cast<int>(align_up(static_cast<size_t>(KH) * halo_px * 16, 128));
                const int halo_bytes = parities * 8 * chunk_bytes;
                const int halo_stride = static_cast<int>(align_up(halo_bytes, 1024));
                const bool halo_ok = halo_px <= 256 && (stride == 1 || IW >= 2);
                // Weight rows padded to a multiple of 64 (64-column output panels).
                const int NN = (OC + 63) / 64 * 64;
                int BN = 0, a_st = 0, b_st = 0, resident = 0;
                for (int bn = std::min(256, NN); halo_ok && bn >= 64 && !BN; bn -= 64) {
                    if (NN % bn)
                        continue;
                    const int bpanel = bn * 128;
                    const int res_bytes = taps * k_panels * bpanel;
                    const int fixed = header + bn / 64 * kTcStagePanelBytes;
                    if (fixed + res_bytes + 2 * halo_stride <= smem_cap) {
                        BN = bn;
                        resident = 1;
                        a_st = std::min(4, (smem_cap - fixed - res_bytes) / halo_stride);
                        b_st = 1;
                    } else {
                        for (int as = 2; as >= 1 && !BN; --as)
                            for (int bs = 4; bs >= 2 && !BN; --bs)
                                if (fixed + bs * bpanel + as * halo_stride <= smem_cap) {
                                    BN = bn;
                                    a_st = as;
                                    b_st = bs;
                                }
                    }
                }
                if (BN) {
                    // weights OIHW -> [NN][KH][KW][IC] (rows past OC stay zero)
                    std::vector<uint16_t> wp(static_cast<size_t>(NN) * taps * IC, 0);
                    std::vector<uint16_t> bp(NN, 0);
                    std::copy(bias_full.begin(), bias_full.end(), bp.begin());
                    for (int o = 0; o < OC; ++o)
                        for (int ky = 0; ky < KH; ++ky)
                            for (int kx = 0; kx < KW; ++kx)
                                for (int c = 0; c < IC; ++c)
                                    wp[((static_cast<size_t>(o) * KH + ky) * KW + kx) * IC + c] =
                                        w[((static_cast<size_t>(o) * IC + c) * KH + ky) * KW + kx];
                    const size_t w_off = prep(wp.data(), wp.size() * 2);
                    const size_t b_off = prep(bp.data(), bp.size() * 2);
                    const int n_tiles = NN / BN, tiles_per_row = (OW + 127) / 128, m_tiles = OH * tiles_per_row;
                    const int grid = n_tiles * std::max(1, std::min(m_tiles, sm_count_ / n_tiles));
                    const int b_slots = resident ? taps * k_panels : b_st;
                    s.kernel = "mlvc_convkxk_tc";
                    s.info.kernel = s.kernel;
                    s.smem =
                        static_cast<unsigned>(header + b_slots * BN * 128 + a_st * halo_stride +
                                              BN / 64 * kTcStagePanelBytes + 1024);
                    s.block = 320;
                    s.grid = static_cast<unsigned>(grid);
                    s.build = [=, this](Step& st) {
                        ConvTcParams p{};
                        const cuuint32_t elem1[3] = {1, 1, 1};
                        for (int q = 0; q < parities; ++q) {
                            const cuuint64_t wq = stride == 1 ? IW : (IW - q + 1) / 2;
                            const cuuint64_t dims[3] = {static_cast<cuuint64_t>(IC), wq, static_cast<cuuint64_t>(IH)};
                            const cuuint64_t strides[2] = {static_cast<cuuint64_t>(IC) * 2 * stride,
                                                           static_cast<cuuint64_t>(IW) * IC * 2};
                            const cuuint32_t box[3] = {8, static_cast<cuuint32_t>(halo_px),
                                                       static_cast<cuuint32_t>(KH)};
                            void* base = reinterpret_cast<void*>(values_[x_id].addr + static_cast<size_t>(q) * IC * 2);
                            check(cuTensorMapEncodeTiled(q ? &p.map_a1 : &p.map_a0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                                                         base, dims, strides, box, elem1, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(convkxk halo)");
                        }
                        if (parities == 1)
                            p.map_a1 = p.map_a0;
                        encode_tile_map(&p.map_out, values_[out_id].addr, OC, 0, OW, OH,
                                        "cuTensorMapEncodeTiled(convkxk out)");
                        if (res_id)
                            encode_tile_map(&p.map_res, values_[res_id].addr, OC, 0, OW, OH,
                                            "cuTensorMapEncodeTiled(convkxk residual)");
                        else
                            p.map_res = p.map_out;
                        {
                            const cuuint64_t Kt = static_cast<cuuint64_t>(taps) * IC;
                            const cuuint64_t dims[2] = {Kt, static_cast<cuuint64_t>(NN)};
                            const cuuint64_t strides[1] = {Kt * 2};
                            const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(BN)};
                            check(cuTensorMapEncodeTiled(&p.map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                                         reinterpret_cast<void*>(prepped_dev_.get() + w_off), dims,
                                                         strides, box, elem1, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(convkxk B)");
                        }
                        p.bias = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b_off);
                        p.out = reinterpret_cast<mlvc_half*>(values_[out_id].addr);
                        p.M = OH * OW;
                        p.N = NN;
                        p.n_valid = OC;
                        p.K = taps * IC;
                        p.BN = BN;
                        p.n_tiles = n_tiles;
                        p.m_tiles = m_tiles;
                        p.epilogue = epi;
                        p.alpha = alpha;
                        p.a_stages = a_st;
                        p.b_resident = resident;
                        p.b_stages = b_st;
                        p.in_h = IH;
                        p.in_w = IW;
                        p.in_c = IC;
                        p.out_h = OH;
                        p.out_w = OW;
                        p.kh = KH;
                        p.kw = KW;
                        p.stride = stride;
                        p.pad = pad;
                        p.halo_px = halo_px;
                        p.px_min = px_min;
                        st.set(p);
                    };
                    steps_.push_back(std::move(s));
                    i += consumed;
                    continue;
                }
            }
            if (reglu) {  // no tensor-core path: run the conv alone, the ReGLU tail separately
                epi = kEpiBias;
                out_id = n.output;
                consumed = 1;
                s.writes = {out_id};
                s.info.nodes = std::to_string(i);
            }
            const bool depthwise = G == IC && OC == IC && ICG == 1 && IC % 8 == 0 && epi == kEpiBias;
            if (depthwise && dw_fusion_ && N == 1 && KH == 3 && KW == 3 && SH == 1 && SW == 1 && PH == 1 && PW == 1 &&
                IC % 64 == 0 && IC <= 512 && i + 1 < nodes.size()) {
                // ---- fused depthwise 3x3 + the 1x1 conv that consumes it: the
                // depthwise result is the GEMM's A operand in shared memory
                const NodeDesc& n2 = nodes[i + 1];
                bool ok = n2.op == Op::kConv && n2.inputs[0] == n.output && only_consumer(n.output) && n2.groups == 1 &&
                          n2.strides[0] == 1 && n2.strides[1] == 1 && n2.pads[0] == 0 && n2.pads[1] == 0;
                const uint32_t w2_id = ok ? n2.inputs[1] : 0;
                const uint32_t b2_id = ok && n2.inputs.size() > 2 ? n2.inputs[2] : 0;
                int OC2 = 0;
                if (ok) {
                    const Value& w2v = values_[w2_id];
                    ok = w2v.kind == Value::kWeight && w2v.dtype == DType::kFp16 && w2v.shape.size() == 4 &&
                         w2v.shape[1] == IC && w2v.shape[2] == 1 && w2v.shape[3] == 1 &&
                         (!b2_id || values_[b2_id].kind == Value::kWeight);
                    OC2 = ok ? static_cast<int>(w2v.shape[0]) : 0;
                    ok = ok && OC2 % 64 == 0 && OC2 <= 256;
                }
                const int M = OH * OW, halo_stride = kDwHaloBytes;
                const int tiles_x = (OW + kDwTileW - 1) / kDwTileW, tiles_y = (OH + kDwTileH - 1) / kDwTileH;
                // + the depthwise taps and bias ([10][C] FP16, one TMA box: C <= 256)
                const int fixed = 1024 + kDwHeaderBytes + 2 * 16384 + 2 * OC2 * 128 + OC2 / 64 * kTcStagePanelBytes +
                                  static_cast<int>(align_up(static_cast<size_t>(10) * IC * 2, 1024));
                int h_stages = 0;
                if (ok)
                    h_stages = fixed + 2 * halo_stride <= max_smem_optin_ ? 2 : (fixed + halo_stride <= max_smem_optin_ ? 1 : 0);
                if (h_stages) {
                    int epi2 = kEpiBias;
                    float alpha2 = 0.0f;
                    uint32_t out2 = 0, res2 = 0;
                    const size_t consumed2 = conv_epilogue(i + 1, epi2, alpha2, out2, res2);
                    std::vector<uint16_t> dwp(static_cast<size_t>(10) * IC, 0);  // taps, then the bias row
                    for (int c = 0; c < IC; ++c)
                        for (int k = 0; k < 9; ++k)
                            dwp[static_cast<size_t>(k) * IC + c] = w[static_cast<size_t>(c) * 9 + k];
                    if (bias)
                        std::copy(bias, bias + IC, dwp.begin() + static_cast<size_t>(9) * IC);
                    std::vector<uint16_t> b2p(OC2, 0);
                    if (b2_id)
                        std::copy(wdata(b2_id), wdata(b2_id) + OC2, b2p.begin());
                    const size_t dww_off = prep(dwp.data(), dwp.size() * 2);
                    const size_t w2_off = prep(wdata(w2_id), static_cast<size_t>(OC2) * IC * 2);
                    const size_t b2_off = prep(b2p.data(), b2p.size() * 2);
                    const int m_tiles = tiles_x * tiles_y;
                    Step f;
                    f.reads = {x_id};
                    if (res2)
                        f.reads.push_back(res2);
                    f.writes = {out2};
                    f.info.nodes = std::to_string(i) + "-" + std::to_string(i + consumed2);
                    f.info.flops = 2.0 * M * IC * 9 + 2.0 * M * static_cast<double>(IC) * OC2;
                    f.info.bytes = 2.0 * (static_cast<double>(M) * IC + 9.0 * IC + IC + static_cast<double>(OC2) * IC +
                                          OC2 + static_cast<double>(M) * OC2 * (res2 && res2 != x_id ? 2 : 1));
                    f.kernel = "mlvc_dwconv_tc";
                    f.info.kernel = f.kernel;
                    f.smem = static_cast<unsigned>(fixed + h_stages * halo_stride);
                    f.block = kDwThreads;
                    f.grid = static_cast<unsigned>(std::min(m_tiles, sm_count_));
                    f.build = [=, this](Step& st) {
                        DwConvTcParams dwp_{};
                        ConvTcParams& p = dwp_.c;
                        const cuuint32_t elem1[2] = {1, 1};
                        {
                            const cuuint32_t elem3[3] = {1, 1, 1};
                            const cuuint64_t dims[3] = {static_cast<cuuint64_t>(IC), static_cast<cuuint64_t>(OW),
                                                        static_cast<cuuint64_t>(OH)};
                            const cuuint64_t strides[2] = {static_cast<cuuint64_t>(IC) * 2,
                                                           static_cast<cuuint64_t>(OW) * IC * 2};
                            const cuuint32_t box[3] = {64, kDwTileW + 2, kDwTileH + 2};
                            check(cuTensorMapEncodeTiled(&dwp_.map_halo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                                                         reinterpret_cast<void*>(values_[x_id].addr), dims, strides, box,
                                                         elem3, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(dwconv halo)");
                        }
                        {
                            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(IC), static_cast<cuuint64_t>(OC2)};
                            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(IC) * 2};
                            const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(OC2)};
                            check(cuTensorMapEncodeTiled(&p.map_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                                         reinterpret_cast<void*>(prepped_dev_.get() + w2_off), dims,
                                                         strides, box, elem1, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(dwconv W)");
                        }
                        encode_tile_map(&p.map_out, values_[out2].addr, OC2, 0, OW, OH, "cuTensorMapEncodeTiled(dwconv out)",
                                        kDwTileW, kDwTileH);
                        if (res2)
                            encode_tile_map(&p.map_res, values_[res2].addr, OC2, 0, OW, OH,
                                            "cuTensorMapEncodeTiled(dwconv residual)", kDwTileW, kDwTileH);
                        else
                            p.map_res = p.map_out;
                        {
                            // [10][C], loaded as dw_tap_group(C)-channel boxes that tile C exactly
                            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(IC), 10};
                            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(IC) * 2};
                            const cuuint32_t box[2] = {static_cast<cuuint32_t>(dw_tap_group(IC)), 10};
                            check(cuTensorMapEncodeTiled(&dwp_.map_dw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                                         reinterpret_cast<void*>(prepped_dev_.get() + dww_off), dims,
                                                         strides, box, elem1, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
                                  "cuTensorMapEncodeTiled(dwconv taps)");
                        }
                        p.map_a0 = p.map_a1 = dwp_.map_halo;
                        p.bias = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b2_off);
                        p.out = reinterpret_cast<mlvc_half*>(values_[out2].addr);
                        p.M = M;
                        p.N = OC2;
                        p.n_valid = OC2;
                        p.K = IC;
                        p.BN = OC2;
                        p.n_tiles = 1;
                        p.m_tiles = m_tiles;
                        p.epilogue = epi2;
                        p.alpha = alpha2;
                        p.a_stages = 2;
                        p.b_stages = 2;
                        dwp_.width = OW;
                        dwp_.height = OH;
                        dwp_.tiles_x = tiles_x;
                        dwp_.h_stages = h_stages;
                        st.set(dwp_);
                    };
                    steps_.push_back(std::move(f));
                    i += 1 + consumed2;
                    continue;
                }
            }
            if (split_a)  // the pre-pass only defers concats for convs with a tensor-core 1x1 plan
                throw std::runtime_error("mlvc-b200: internal: concat read in place by a conv without a 1x1 plan");
            DirectConvParams dp{};
            dp.n = N;
            dp.ih = IH;
            dp.iw = IW;
            dp.ic = IC;
            dp.oh = OH;
            dp.ow = OW;
            dp.oc = OC;
            dp.kh = KH;
            dp.kw = KW;
            dp.sh = SH;
            dp.sw = SW;
            dp.ph = PH;
            dp.pw = PW;
            dp.groups = G;
            dp.epilogue = epi;
            dp.alpha = alpha;
            size_t w_off;
            long long work;
            if (depthwise) {
                std::vector<uint16_t> wp(static_cast<size_t>(KH) * KW * OC);
                for (int c = 0; c < OC; ++c)
                    for (int k = 0; k < KH * KW; ++k)
                        wp[static_cast<size_t>(k) * OC + c] = w[static_cast<size_t>(c) * KH * KW + k];
                w_off = prep(wp.data(), wp.size() * 2);
                const bool dw3 = KH == 3 && KW == 3 && SH == SW && (SH == 1 || SH == 2) && PH == PW && PH <= 1;
                if (dw3 && OC / 8 <= 256) {
                    s.kernel = "mlvc_depthwise3x3_f16";
                    work = 0;
                    const int per_block = 256 / (OC / 8);
                    s.grid = static_cast<unsigned>((OW + per_block - 1) / per_block);
                    s.grid_y = static_cast<unsigned>((OH + 3) / 4);  // four output rows per thread
                    s.grid_z = static_cast<unsigned>(N);
                } else {
                    s.kernel = "mlvc_depthwise_v8_f16";
                    work = static_cast<long long>(N) * OH * OW * (OC / 8);
                }
            } else {
                std::vector<uint16_t> wp(static_cast<size_t>(OC) * KH * KW * ICG);
                for (int o = 0; o < OC; ++o)
                    for (int ky = 0; ky < KH; ++ky)
                        for (int kx = 0; kx < KW; ++kx)
                            for (int c = 0; c < ICG; ++c)
                                wp[((static_cast<size_t>(o) * KH + ky) * KW + kx) * ICG + c] =
                                    w[((static_cast<size_t>(o) * ICG + c) * KH + ky) * KW + kx];
                w_off = prep(wp.data(), wp.size() * 2);
                s.kernel = "mlvc_conv_direct_f16";
                work = static_cast<long long>(N) * OH * OW * OC;
            }
            const size_t b_off = prep(bias_full.data(), bias_full.size() * 2);
            s.info.kernel = s.kernel;
            if (work)
                s.grid = blocks_for(work, 256, sm_count_);
            s.build = [=, this](Step& st) {
                DirectConvParams p = dp;
                p.x = reinterpret_cast<const mlvc_half*>(values_[x_id].addr);
                p.w = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + w_off);
                p.bias = reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + b_off);
                p.residual = res_id ? reinterpret_cast<const mlvc_half*>(values_[res_id].addr) : nullptr;
                p.y = reinterpret_cast<mlvc_half*>(values_[out_id].addr);
                st.set(p);
            };
            steps_.push_back(std::move(s));
            i += consumed;
            continue;
        }

        // ---- latent quantisation tails (reference matchers:
        // fusion_registry.cpp:14-225 for y0, :226-404 for y1; the CPU twins
        // backends/cpu/src/fusion_matcher.cpp:543-850).  As there, the operands
        // of the Adds and Muls may come in either order, the Clip's upper bound
        // may be absent or >= 65504 (the reference's exporter writes 65504), and
        // in the y0 tail an optional Mul of the reciprocal by an FP16 scalar 1
        // may follow the Reciprocal.
        if (tail_fusion_ && (n.op == Op::kSlice || n.op == Op::kSub)) {
            const bool y0 = n.op == Op::kSlice;
            static constexpr Op kY0[19] = {Op::kSlice, Op::kSlice, Op::kClip,   Op::kReciprocal, Op::kMul,
                                           Op::kSub,   Op::kMul,   Op::kSlice,  Op::kSlice,      Op::kAdd,
                                           Op::kRound, Op::kSlice, Op::kSlice,  Op::kAdd,        Op::kMul,
                                           Op::kAdd,   Op::kMul,   Op::kConcat, Op::kConcat};
            static constexpr Op kY1[15] = {Op::kSub, Op::kMul,   Op::kSlice, Op::kSlice, Op::kAdd,
                                           Op::kRound, Op::kSlice, Op::kSlice, Op::kAdd,   Op::kMul,
                                           Op::kAdd, Op::kMul,   Op::kConcat, Op::kAdd,  Op::kMul};
            auto is_one = [&](uint32_t id) {
                if (id == 0 || values_[id].kind != Value::kWeight || values_[id].dtype != DType::kFp16 ||
                    element_count(values_[id].shape) != 1)
                    return false;
                return std::fabs(half_bits_to_float(wdata(id)[0]) - 1.0f) <= 1e-4f;
            };
            // y0 with the Mul-by-one: chain nodes 4.. sit one index later
            size_t extra = 0;
            if (y0 && i + 20 <= nodes.size() && nodes[i + 3].op == Op::kReciprocal && nodes[i + 4].op == Op::kMul &&
                nodes[i + 5].op == Op::kMul && nodes[i + 4].inputs.size() == 2 && !absorbed[i + 4]) {
                const auto& m = nodes[i + 4].inputs;
                const uint32_t r = nodes[i + 3].output;
                if ((m[0] == r && is_one(m[1])) || (m[1] == r && is_one(m[0])))
                    extra = 1;
            }
            auto at = [&](size_t k) { return i + k + (k >= 4 ? extra : 0); };
            const Op* pat = y0 ? kY0 : kY1;
            const size_t chain = y0 ? 19 : 15;
            const size_t len = chain + extra;
            bool ok = i + len <= nodes.size();
            for (size_t k = 0; ok && k < chain; ++k)
                ok = nodes[at(k)].op == pat[k] && !absorbed[at(k)];
            auto out = [&](size_t k) { return nodes[at(k)].output; };
            auto in = [&](size_t k) -> const std::vector<uint32_t>& { return nodes[at(k)].inputs; };
            auto vec = [](std::initializer_list<uint32_t> l) { return std::vector<uint32_t>(l); };
            auto pair = [&](size_t k, uint32_t a, uint32_t b) {  // inputs are {a, b} in either order
                const auto& v = in(k);
                return v.size() == 2 && ((v[0] == a && v[1] == b) || (v[0] == b && v[1] == a));
            };
            auto other = [&](size_t k, uint32_t a) -> uint32_t {  // the operand beside `a`, or 0
                const auto& v = in(k);
                if (v.size() != 2)
                    return 0;
                return v[0] == a ? v[1] : v[1] == a ? v[0] : 0;
            };
            auto rt = [&](uint32_t id) {  // runtime NHWC FP16 rank-4 value
                const Value& v = values_[id];
                return id != 0 && v.present && v.nhwc && v.dtype == DType::kFp16 && v.shape.size() == 4;
            };
            auto cons = [&](uint32_t id, int c) { return values_[id].consumers == c && !values_[id].graph_output; };
            // chain offsets of: scaled, y_raw, prior slices, updates (y0 numbering minus 5 for y1)
            const size_t d = y0 ? 0 : 5;
            uint32_t prior_id = 0, latent_id = 0, norm_id = 0, qs_id = 0, us0_id = 0, us1_id = 0, c2_id = 0, cl_id = 0;
            int Q = 0;
            if (ok) {
                const uint32_t scaled = out(6 - d), y_raw = out(10 - d);
                qs_id = other(6 - d, out(5 - d));
                us0_id = other(14 - d, out(13 - d));
                us1_id = other(16 - d, out(15 - d));
                ok = rt(y_raw) && pair(9 - d, out(7 - d), out(8 - d)) && in(10 - d) == vec({out(9 - d)}) &&
                     pair(13 - d, y_raw, out(11 - d)) && pair(15 - d, y_raw, out(12 - d)) &&
                     in(17 - d) == vec({out(14 - d), out(16 - d)}) && rt(qs_id) && rt(us0_id) && rt(us1_id);
                if (ok) {
                    Q = static_cast<int>(values_[y_raw].shape[1]);
                    ok = Q % 8 == 0 && is_channel_slice(nodes[at(7 - d)], scaled, 0, Q) &&
                         is_channel_slice(nodes[at(8 - d)], scaled, Q, 2 * Q) && cons(out(5 - d), 1) &&
                         cons(scaled, 2) && cons(out(7 - d), 1) && cons(out(8 - d), 1) && cons(out(9 - d), 1) &&
                         values_[y_raw].consumers >= 2 && cons(out(11 - d), 1) && cons(out(12 - d), 1) &&
                         cons(out(13 - d), 1) && cons(out(14 - d), 1) && cons(out(15 - d), 1) &&
                         cons(out(16 - d), 1) && (nodes[at(17 - d)].axis == 1 || nodes[at(17 - d)].axis == -3);
                }
            }
            if (ok && y0) {
                prior_id = n.inputs[0];
                const uint32_t inv = extra ? nodes[i + 4].output : out(3);
                latent_id = other(4, inv);
                ok = in(1)[0] == prior_id && rt(prior_id) && values_[prior_id].shape[1] == 4 * Q &&
                     is_channel_slice(nodes[i], prior_id, 0, 2 * Q) && is_channel_slice(nodes[i + 1], prior_id, 2 * Q, 4 * Q) &&
                     in(2).size() >= 2 && in(2)[0] == out(0) &&
                     (in(2).size() < 3 || in(2)[2] == 0 || scalar(in(2)[2], INFINITY) >= 65504.0f) &&
                     in(3) == vec({out(2)}) && rt(latent_id) && in(5) == vec({out(4), out(1)}) &&
                     is_channel_slice(nodes[at(11)], out(1), 0, Q) && is_channel_slice(nodes[at(12)], out(1), Q, 2 * Q) &&
                     in(18) == vec({out(17), prior_id}) && (nodes[at(18)].axis == 1 || nodes[at(18)].axis == -3) &&
                     cons(out(0), 1) && cons(out(1), 3) && cons(out(3), 1) && (!extra || cons(inv, 1)) &&
                     values_[prior_id].consumers >= 3 && rt(out(18));
            } else if (ok) {
                norm_id = n.inputs[0];
                prior_id = n.inputs.size() == 2 ? n.inputs[1] : 0;
                c2_id = other(13, out(12));
                cl_id = other(14, out(13));
                ok = rt(norm_id) && rt(prior_id) && rt(c2_id) && rt(cl_id) && is_channel_slice(nodes[at(6)], prior_id, 0, Q) &&
                     is_channel_slice(nodes[at(7)], prior_id, Q, 2 * Q) && values_[prior_id].consumers >= 3 &&
                     cons(out(12), 1) && cons(out(13), 1) && rt(out(14));
            }
            if (ok) {
                const std::vector<int64_t> raw = values_[out(10 - d)].shape;
                const std::vector<int64_t> two{raw[0], 2 * raw[1], raw[2], raw[3]};
                ok = values_[qs_id].shape == two && values_[us0_id].shape == raw && values_[us1_id].shape == raw;
                if (y0)
                    ok = ok && values_[latent_id].shape == two && values_[prior_id].shape ==
                                   std::vector<int64_t>{raw[0], 4 * raw[1], raw[2], raw[3]};
                else
                    ok = ok && values_[norm_id].shape == two && values_[prior_id].shape == two &&
                         values_[c2_id].shape == two && values_[cl_id].shape == two;
            }
            if (ok) {
                const uint32_t y_raw = out(10 - d);
                const long long pixels = element_count(values_[y_raw].shape) / Q;
                float clip_lo = 0.0f;
                uint32_t norm_out = 0, clip_out = 0, c2_out = 0, c3_out = 0, result = 0;
                if (y0) {
                    clip_lo = scalar(in(2)[1], -INFINITY);
                    norm_out = values_[out(4)].consumers > 1 || values_[out(4)].graph_output ? out(4) : 0;
                    clip_out = values_[out(2)].consumers > 1 || values_[out(2)].graph_output ? out(2) : 0;
                    c2_out = values_[out(17)].consumers > 1 || values_[out(17)].graph_output ? out(17) : 0;
                    c3_out = out(18);
                } else {
                    result = out(14);
                }
                Step s;
                s.kernel = y0 ? "mlvc_y0_tail_f16" : "mlvc_y1_tail_f16";
                s.info.kernel = s.kernel;
                s.info.nodes = std::to_string(i) + "-" + std::to_string(i + len - 1);
                s.reads = y0 ? std::vector<uint32_t>{prior_id, latent_id, qs_id, us0_id, us1_id}
                             : std::vector<uint32_t>{norm_id, prior_id, qs_id, us0_id, us1_id, c2_id, cl_id};
                s.writes = {y_raw};
                for (uint32_t w : {norm_out, clip_out, c2_out, c3_out, result})
                    if (w)
                        s.writes.push_back(w);
                s.info.bytes = 2.0 * pixels * Q * (y0 ? 4 + 2 + 2 + 2 + 1 + 6 : 2 + 2 + 2 + 2 + 2 + 2 + 1 + 2);
                s.grid = blocks_for(pixels * (Q / 8), 256, sm_count_);
                s.block = 256;
                const bool is_y0 = y0;
                s.build = [=, this](Step& st) {
                    auto ptr = [&](uint32_t id) { return id ? reinterpret_cast<mlvc_half*>(values_[id].addr) : nullptr; };
                    QuantTailParams p{};
                    p.latent = ptr(latent_id);
                    p.normalized = ptr(norm_id);
                    p.prior = ptr(prior_id);
                    p.qscale = ptr(qs_id);
                    p.uscale0 = ptr(us0_id);
                    p.uscale1 = ptr(us1_id);
                    p.concat2_in = ptr(c2_id);
                    p.clipped_in = ptr(cl_id);
                    p.normalized_out = ptr(norm_out);
                    p.clipped_out = ptr(clip_out);
                    p.y_raw = ptr(y_raw);
                    p.concat2_out = ptr(c2_out);
                    p.concat3 = ptr(c3_out);
                    p.result = ptr(result);
                    p.pixels = pixels;
                    p.q = Q;
                    p.clip_lo = is_y0 ? clip_lo : 0.0f;
                    st.set(p);
                };
                steps_.push_back(std::move(s));
                i += len;
                continue;
            }
        }

        // ---- recurrent-feature update: Slice x3, Sigmoid x2, Mul, Sub, Mul, Add,
        // Mul, Mul (+ a later Concat of the last Mul and the Add on channels),
        // the reference's fusion patterns of fusion_registry.cpp:405-709
        if (n.op == Op::kSlice && tail_fusion_ && i + 10 < nodes.size()) {
            static constexpr Op kPattern[11] = {Op::kSlice, Op::kSlice, Op::kSlice, Op::kSigmoid, Op::kSigmoid,
                                                Op::kMul,   Op::kSub,   Op::kMul,   Op::kAdd,     Op::kMul,
                                                Op::kMul};
            bool ok = true;
            for (int k = 0; ok && k < 11; ++k)
                ok = nodes[i + k].op == kPattern[k] && !absorbed[i + k];
            const uint32_t src_id = n.inputs[0];
            auto out = [&](int k) { return nodes[i + k].output; };
            auto in = [&](int k) -> const std::vector<uint32_t>& { return nodes[i + k].inputs; };
            const Value& sv = values_[src_id];
            int C = 0;
            if (ok && sv.nhwc && sv.dtype == DType::kFp16 && sv.shape.size() == 4 && sv.shape[1] % 3 == 0) {
                C = static_cast<int>(sv.shape[1] / 3);
                ok = C % 8 == 0 && in(1)[0] == src_id && in(2)[0] == src_id && is_channel_slice(nodes[i], src_id, 0, C) &&
                     is_channel_slice(nodes[i + 1], src_id, C, 2 * C) &&
                     is_channel_slice(nodes[i + 2], src_id, 2 * C, 3 * C);
            } else {
                ok = false;
            }
            uint32_t hist_id = 0, one_id = 0, scale_id = 0;
            if (ok) {
                ok = in(3) == std::vector<uint32_t>{out(1)} && in(4) == std::vector<uint32_t>{out(2)} &&
                     in(5).size() == 2 && in(5)[0] == out(3) && in(6).size() == 2 && in(6)[1] == out(3) &&
                     in(7) == std::vector<uint32_t>{out(6), out(0)} && in(8) == std::vector<uint32_t>{out(5), out(7)} &&
                     in(9) == std::vector<uint32_t>{out(4), out(8)} && in(10).size() == 2 && in(10)[0] == out(9);
            }
            if (ok) {
                hist_id = in(5)[1];
                one_id = in(6)[0];
                scale_id = in(10)[1];
                const auto& fs = values_[out(0)].shape;
                const Value &hv = values_[hist_id], &ov = values_[one_id], &scv = values_[scale_id];
                ok = hv.nhwc && hv.dtype == DType::kFp16 && hv.shape == fs && ov.kind == Value::kWeight &&
                     ov.dtype == DType::kFp16 && element_count(ov.shape) == 1 && scv.kind == Value::kWeight &&
                     scv.dtype == DType::kFp16 && scv.shape == std::vector<int64_t>{1, C, 1, 1};
                for (int k = 3; ok && k <= 10; ++k)
                    ok = values_[out(k)].nhwc && values_[out(k)].shape == fs && values_[out(k)].dtype == DType::kFp16;
                // chain-internal values: read only inside the chain
                const int internal[] = {0, 1, 2, 4, 5, 6, 7, 9};
                for (int k : internal)
                    ok = ok && only_consumer(out(k));
                ok = ok && values_[out(3)].consumers == 2 && !values_[out(3)].graph_output;
            }
            if (ok) {
                const uint32_t scaled_id = out(10), blended_id = out(8);
                // a later Concat(scaled, blended) on channels is produced here too
                size_t concat_j = 0;
                for (size_t j = i + 11; j < nodes.size() && !concat_j; ++j)
                    if (nodes[j].op == Op::kConcat && !absorbed[j] &&
                        nodes[j].inputs == std::vector<uint32_t>{scaled_id, blended_id} &&
                        (nodes[j].axis == 1 || nodes[j].axis == -3) && values_[nodes[j].output].nhwc)
                        concat_j = j;
                const uint32_t concat_id = concat_j ? nodes[concat_j].output : 0;
                // scaled / blended on their own when anything but the concat (and, for
                // blended, the gated Mul of the chain) reads them
                const int in_chain_blended = 1 + (concat_j ? 1 : 0);
                const bool keep_scaled = !concat_j || values_[scaled_id].consumers > 1 || values_[scaled_id].graph_output;
                const bool keep_blended =
                    values_[blended_id].consumers > in_chain_blended || values_[blended_id].graph_output;
                if (concat_j)
                    absorbed[concat_j] = true;
                const float one_value = half_bits_to_float(wdata(one_id)[0]);
                const long long pixels = element_count(values_[out(0)].shape) / C;
                Step s;
                s.kernel = "mlvc_feature_update_f16";
                s.info.kernel = s.kernel;
                s.info.nodes = std::to_string(i) + "-" + std::to_string(i + 10) +
                               (concat_j ? "+" + std::to_string(concat_j) : std::string());
                s.reads = {src_id, hist_id};
                if (concat_id)
                    s.writes.push_back(concat_id);
                if (keep_scaled)
                    s.writes.push_back(scaled_id);
                if (keep_blended)
                    s.writes.push_back(blended_id);
                s.info.bytes = 2.0 * pixels * C * (3 + 1 + (concat_id ? 2 : 0) + (keep_scaled ? 1 : 0) + (keep_blended ? 1 : 0));
                s.grid = blocks_for(pixels * (C / 8), 256, sm_count_);
                s.block = 256;
                s.build = [=, this](Step& st) {
                    FeatureUpdateParams p{};
                    p.src = reinterpret_cast<const mlvc_half*>(values_[src_id].addr);
                    p.history = reinterpret_cast<const mlvc_half*>(values_[hist_id].addr);
                    p.scale = reinterpret_cast<const mlvc_half*>(values_[scale_id].addr);
                    p.concat = concat_id ? reinterpret_cast<mlvc_half*>(values_[concat_id].addr) : nullptr;
                    p.scaled = keep_scaled ? reinterpret_cast<mlvc_half*>(values_[scaled_id].addr) : nullptr;
                    p.blended = keep_blended ? reinterpret_cast<mlvc_half*>(values_[blended_id].addr) : nullptr;
                    p.pixels = pixels;
                    p.c = C;
                    p.one = one_value;
                    st.set(p);
                };
                steps_.push_back(std::move(s));
                i += 11;
                continue;
            }
        }

        // ---- stand-alone ReGLU: Slice, Slice, Clip, Mul on one tensor
        if (n.op == Op::kSlice) {
            float lo, hi;
            const uint32_t t_id = n.inputs[0];
            if (values_[t_id].nhwc && match_reglu_tail(i, t_id, lo, hi)) {
                const uint32_t out_id = nodes[i + 3].output;
                Step s;
                s.kernel = "mlvc_reglu_f16";
                s.info.kernel = s.kernel;
                s.info.nodes = std::to_string(i) + "-" + std::to_string(i + 3);
                s.reads = {t_id};
                s.writes = {out_id};
                const auto& sh = values_[t_id].shape;
                const long long pixels = sh[0] * sh[2] * sh[3];
                const int c = static_cast<int>(sh[1] / 2);
                s.info.bytes = 2.0 * pixels * c * 3;
                s.grid = blocks_for(pixels * c, 256, sm_count_);
                s.build = [=, this](Step& st) {
                    RegluParams p{};
                    p.src = reinterpret_cast<const mlvc_half*>(values_[t_id].addr);
                    p.dst = reinterpret_cast<mlvc_half*>(values_[out_id].addr);
                    p.pixels = pixels;
                    p.c = c;
                    p.lo = lo;
                    p.hi = hi;
                    st.set(p);
                };
                steps_.push_back(std::move(s));
                i += 4;
                continue;
            }
        }

        // ---- single operators
        Step s;
        s.info.nodes = std::to_string(i);
        const uint32_t out_id = n.output;
        s.writes = {out_id};
        const Value& ov = values_[out_id];
        const long long out_count = element_count(ov.shape);
        s.info.bytes = 2.0 * out_count;
        switch (n.op) {
        case Op::kAdd:
        case Op::kSub:
        case Op::kMul: {
            const uint32_t a = n.inputs[0], b = n.inputs[1];
            s.reads = {a, b};
            const int op = n.op == Op::kAdd ? 0 : n.op == Op::kMul ? 1 : 2;
            const Value &av = values_[a], &bv = values_[b];
            s.info.bytes += 2.0 * (element_count(av.shape) + element_count(bv.shape));
            const bool same = av.shape == ov.shape && bv.shape == ov.shape && av.nhwc == ov.nhwc &&
                              bv.nhwc == ov.nhwc;
            s.kernel = same ? "mlvc_binary_same_f16" : "mlvc_binary_bcast_f16";
            s.grid = blocks_for(same ? out_count / 8 + 1 : out_count, 256, sm_count_);
            s.build = [=, this](Step& st) {
                ElementwiseParams p{};
                const Value &A = values_[a], &B = values_[b], &O = values_[out_id];
                p.a = reinterpret_cast<const mlvc_half*>(A.addr);
                p.b = reinterpret_cast<const mlvc_half*>(B.addr);
                p.out = reinterpret_cast<mlvc_half*>(O.addr);
                p.count = out_count;
                p.op = op;
                const auto od = dims4(O.shape), ad = dims4(A.shape), bd = dims4(B.shape);
                const auto as = A.strides(), bs = B.strides();
                // physical iteration order of the output
                const int order_nhwc[4] = {0, 2, 3, 1}, order_nchw[4] = {0, 1, 2, 3};
                const int* ord = O.nhwc ? order_nhwc : order_nchw;
                for (int k = 0; k < 4; ++k) {
                    const int l = ord[k];
                    p.dims[k] = static_cast<int>(od[l]);
                    p.sa[k] = ad[l] == 1 ? 0 : as[l];
                    p.sb[k] = bd[l] == 1 ? 0 : bs[l];
                }
                st.set(p);
            };
            break;
        }
        case Op::kLeakyRelu:
        case Op::kClip:
        case Op::kSigmoid:
        case Op::kReciprocal:
        case Op::kRound: {
            const uint32_t a = n.inputs[0];
            s.reads = {a};
            if (values_[a].nhwc != ov.nhwc || values_[a].kind == Value::kWeight)
                throw std::runtime_error("mlvc-b200: unary operator on an initializer is not supported");
            s.info.bytes += 2.0 * out_count;
            const int op = n.op == Op::kLeakyRelu ? 0 : n.op == Op::kClip ? 1 : n.op == Op::kSigmoid ? 2
                         : n.op == Op::kReciprocal ? 3 : 4;
            const float lo = n.op == Op::kClip && n.inputs.size() > 1 ? scalar(n.inputs[1], -INFINITY) : -INFINITY;
            const float hi = n.op == Op::kClip && n.inputs.size() > 2 ? scalar(n.inputs[2], INFINITY) : INFINITY;
            const float alpha = n.alpha;
            s.kernel = "mlvc_unary_f16";
            s.grid = blocks_for(out_count / 8 + 1, 256, sm_count_);
            s.build = [=, this](Step& st) {
                ElementwiseParams p{};
                p.a = reinterpret_cast<const mlvc_half*>(values_[a].addr);
                p.out = reinterpret_cast<mlvc_half*>(values_[out_id].addr);
                p.count = out_count;
                p.op = op;
                p.alpha = alpha;
                p.lo = lo;
                p.hi = hi;
                st.set(p);
            };
            break;
        }
        case Op::kSlice: {
            const uint32_t a = n.inputs[0];
            s.reads = {a};
            const Value& av = values_[a];
            const auto starts = int64s(n.inputs[1]);
            const auto axes = n.inputs.size() > 3 && n.inputs[3] ? int64s(n.inputs[3]) : std::vector<int64_t>{};
            const auto stepv = n.inputs.size() > 4 && n.inputs[4] ? int64s(n.inputs[4]) : std::vector<int64_t>{};
            const int rank = static_cast<int>(av.shape.size());
            std::array<long long, 4> start4{0, 0, 0, 0}, step4{1, 1, 1, 1};
            const auto id4 = dims4(av.shape);
            for (size_t k = 0; k < starts.size(); ++k) {
                int axis = axes.empty() ? static_cast<int>(k) : static_cast<int>(axes[k]);
                if (axis < 0)
                    axis += rank;
                axis += 4 - rank;
                long long st0 = starts[k];
                if (st0 < 0)
                    st0 += id4[axis];
                // clamped to [0, dim] like the reference CPU plan
                // (backends/cpu/src/execution_plan.cpp:596-599)
                start4[axis] = std::clamp<long long>(st0, 0, id4[axis]);
                if (!stepv.empty())
                    step4[axis] = stepv[k];
            }
            {
                // Contiguous result (every dimension inside the sliced one whole,
                // every one outside it of extent 1, unit steps, same layout): a
                // view into the source at a 256-byte aligned offset, no copy.
                const auto od4 = dims4(ov.shape);
                const Value& src = av.alias_of ? values_[av.alias_of] : av;
                const bool producible = src.kind == Value::kNone || src.kind == Value::kArena;
                bool contiguous = ov.nhwc == av.nhwc && ov.dtype == av.dtype && producible && !src.graph_output &&
                                  !ov.graph_output && step4 == std::array<long long, 4>{1, 1, 1, 1};
                const int order_nhwc[4] = {0, 2, 3, 1}, order_nchw[4] = {0, 1, 2, 3};
                const int* ord = av.nhwc ? order_nhwc : order_nchw;
                int k = 3;  // innermost physical dimension that is not taken whole
                while (k >= 0 && od4[ord[k]] == id4[ord[k]])
                    --k;
                for (int q = 0; contiguous && q < k; ++q)
                    contiguous = od4[ord[q]] == 1;
                const auto as = av.strides();
                long long off = 0;
                for (int l = 0; l < 4; ++l)
                    off += start4[l] * as[l];
                const size_t bytes_off = static_cast<size_t>(off) * 2 + (av.alias_of ? av.alias_off : 0);
                if (contiguous && bytes_off % 256 == 0) {
                    Value& o = values_[out_id];
                    o.alias_of = av.alias_of ? av.alias_of : a;
                    o.alias_off = bytes_off;
                    ++i;
                    continue;
                }
            }
            s.info.bytes += 2.0 * out_count;
            const bool nhwc = ov.nhwc;
            s.kernel = "mlvc_strided_copy_f16";
            s.grid = blocks_for(out_count, 256, sm_count_);
            // vector path: channels innermost and contiguous with 8-aligned offsets
            const auto od4 = dims4(ov.shape);
            if (nhwc && av.nhwc && step4[1] == 1 && od4[1] % 8 == 0 && start4[1] % 8 == 0 && id4[1] % 8 == 0) {
                s.kernel = "mlvc_strided_copy_v8_f16";
                s.grid = blocks_for(out_count / 8, 256, sm_count_);
            }
            s.build = [=, this](Step& st) {
                CopyParams p{};
                const Value &A = values_[a], &O = values_[out_id];
                const auto as = A.strides(), os = O.strides();
                long long base = 0;
                for (int l = 0; l < 4; ++l)
                    base += start4[l] * as[l];
                p.src = reinterpret_cast<const mlvc_half*>(A.addr) + base;
                p.dst = reinterpret_cast<mlvc_half*>(O.addr);
                const int order_nhwc[4] = {0, 2, 3, 1}, order_nchw[4] = {0, 1, 2, 3};
                const int* ord = O.nhwc ? order_nhwc : order_nchw;
                for (int k = 0; k < 4; ++k) {
                    const int l = ord[k];
                    p.dims[k] = static_cast<int>(od4[l]);
                    p.ss[k] = as[l] * step4[l];
                    p.ds[k] = os[l];
                }
                p.count = out_count;
                st.set(p);
            };
            break;
        }
        case Op::kConcat: {
            // One copy step per operand; the operator's own step is the last one.
            int axis = n.axis;
            const int rank = static_cast<int>(ov.shape.size());
            if (axis < 0)
                axis += rank;
            axis += 4 - rank;
            long long offset = 0;
            const auto od4 = dims4(ov.shape);
            for (size_t k = 0; k < n.inputs.size(); ++k) {
                const uint32_t a = n.inputs[k];
                const auto ad4 = dims4(values_[a].shape);
                Step c;
                c.info.nodes = std::to_string(i);
                c.reads = {a};
                c.writes = {out_id};
                const long long cnt = element_count(values_[a].shape);
                c.info.bytes = 4.0 * cnt;
                const bool vec = ov.nhwc && values_[a].nhwc && axis == 1 && ad4[1] % 8 == 0 && offset % 8 == 0 &&
                                 od4[1] % 8 == 0;
                c.kernel = vec ? "mlvc_strided_copy_v8_f16" : "mlvc_strided_copy_f16";
                c.info.kernel = c.kernel;
                c.grid = blocks_for(vec ? cnt / 8 : cnt, 256, sm_count_);
                const long long off = offset;
                c.build = [=, this](Step& st) {
                    CopyParams p{};
                    const Value &A = values_[a], &O = values_[out_id];
                    const auto as = A.strides(), os = O.strides();
                    p.src = reinterpret_cast<const mlvc_half*>(A.addr);
                    p.dst = reinterpret_cast<mlvc_half*>(O.addr) + off * os[axis];
                    const int order_nhwc[4] = {0, 2, 3, 1}, order_nchw[4] = {0, 1, 2, 3};
                    const int* ord = O.nhwc ? order_nhwc : order_nchw;
                    for (int q = 0; q < 4; ++q) {
                        const int l = ord[q];
                        p.dims[q] = static_cast<int>(ad4[l]);
                        p.ss[q] = as[l];
                        p.ds[q] = os[l];
                    }
                    p.count = cnt;
                    st.set(p);
                };
                offset += ad4[axis];
                if (k + 1 < n.inputs.size()) {
                    c.writes = {out_id};
                    steps_.push_back(std::move(c));
                } else {
                    s = std::move(c);
                }
            }
            break;
        }
        case Op::kGather: {
            const uint32_t data = n.inputs[0], idx = n.inputs[1];
            s.reads = {data, idx};
            const Value& dv = values_[data];
            if (n.axis != 0 || values_[idx].dtype != DType::kInt32)
                throw std::runtime_error("mlvc-b200: only Gather on axis 0 with an INT32 index is supported");
            const int rows = static_cast<int>(dv.shape[0]);
            const long long row_elems = element_count(dv.shape) / rows;
            size_t table_off = 0;
            bool prepped = false;
            if (dv.kind == Value::kWeight) {
                // Store the table in the output's physical layout once.
                const auto od4 = dims4(ov.shape);
                std::vector<uint16_t> tab(static_cast<size_t>(element_count(dv.shape)));
                const uint16_t* src = wdata(data);
                if (ov.nhwc) {
                    const long long C = od4[1], HW = od4[2] * od4[3];
                    for (int r = 0; r < rows; ++r)
                        for (long long c = 0; c < C; ++c)
                            for (long long p = 0; p < HW; ++p)
                                tab[r * row_elems + p * C + c] = src[r * row_elems + c * HW + p];
                } else {
                    std::copy(src, src + tab.size(), tab.begin());
                }
                table_off = prep(tab.data(), tab.size() * 2);
                prepped = true;
            } else if (dv.nhwc != ov.nhwc) {
                throw std::runtime_error("mlvc-b200: Gather on a runtime tensor must keep its layout");
            }
            s.kernel = "mlvc_gather_rows_f16";
            s.grid = blocks_for(row_elems, 256, sm_count_);
            s.build = [=, this](Step& st) {
                GatherParams p{};
                p.src = prepped ? reinterpret_cast<const mlvc_half*>(prepped_dev_.get() + table_off)
                                : reinterpret_cast<const mlvc_half*>(values_[data].addr);
                p.index = reinterpret_cast<const int32_t*>(values_[idx].addr);
                p.dst = reinterpret_cast<mlvc_half*>(values_[out_id].addr);
                p.row_elems = row_elems;
                p.rows = rows;
                st.set(p);
            };
            break;
        }
        case Op::kDepthToSpace:
        case Op::kSpaceToDepth: {
            const uint32_t a = n.inputs[0];
            s.reads = {a};
            if (!values_[a].nhwc || !ov.nhwc)
                throw std::runtime_error("mlvc-b200: pixel (un)shuffle expects rank-4 activations");
            s.info.bytes += 2.0 * out_count;
            const auto& sh = values_[a].shape;
            const int r = n.block;
            const bool d2s = n.op == Op::kDepthToSpace;
            // r = 2 with 8-channel output (d2s) / input (s2d) blocks: 16-byte vectors;
            // one item = one pixel x 8 channels on the narrow side = 32 output elements
            const bool v8 = r == 2 && (d2s ? sh[1] % 32 == 0 : sh[1] % 8 == 0);
            const long long items = v8 ? out_count / 32 : out_count;
            s.kernel = v8 ? (d2s ? "mlvc_depth_to_space_r2_v8_f16" : "mlvc_space_to_depth_r2_v8_f16")
                          : (d2s ? "mlvc_depth_to_space_f16" : "mlvc_space_to_depth_f16");
            s.grid = blocks_for(items, 256, sm_count_);
            s.build = [=, this](Step& st) {
                PixelShuffleParams p{};
                p.src = reinterpret_cast<const mlvc_half*>(values_[a].addr);
                p.dst = reinterpret_cast<mlvc_half*>(values_[out_id].addr);
                p.n = static_cast<int>(sh[0]);
                p.c = static_cast<int>(sh[1]);
                p.h = static_cast<int>(sh[2]);
                p.w = static_cast<int>(sh[3]);
                p.r = r;
                p.count = items;
                st.set(p);
            };
            break;
        }
        default:
            throw std::runtime_error("mlvc-b200: unsupported operator " + std::to_string(static_cast<int>(n.op)));
        }
        s.info.kernel = s.kernel;
        steps_.push_back(std::move(s));
        ++i;
    }

    // ---- output boundary
    for (size_t k = 0; k < ext_outputs_.size(); ++k) {
        const uint32_t id = graph_.outputs[ext_outputs_[k]];
        if (!needs_conversion(values_[id]) && output_source[k].second == 1)
            continue;
        steps_.push_back(boundary_step(id, output_source[k].first, output_source[k].second, true, k));
    }
    state_alias_.assign(bindings_.size(), false);
    for (const auto& b : bindings_) {
        const uint32_t out_id = graph_.outputs[b.output_index];
        const uint32_t in_id = graph_.inputs[b.input_index];
        const size_t bi = static_cast<size_t>(&b - bindings_.data());
        // The output aliases the state buffer (the reference's contract: state
        // aliases the final node's output) when every step that reads the state
        // input runs before the first step that writes the output; otherwise it
        // is copied into the state buffer after the frame.
        long long last_read = -1, first_write = -1;
        for (size_t k = 0; k < steps_.size(); ++k) {
            for (uint32_t r : steps_[k].reads)
                if (r == in_id)
                    last_read = static_cast<long long>(k);
            for (uint32_t w : steps_[k].writes)
                if (w == out_id && first_write < 0)
                    first_write = static_cast<long long>(k);
        }
        if (first_write >= 0 && last_read < first_write && values_[out_id].bytes == values_[in_id].bytes &&
            values_[out_id].nhwc == values_[in_id].nhwc && values_[out_id].kind != Value::kWeight &&
            values_[out_id].kind != Value::kInput && values_[out_id].kind != Value::kState) {
            state_alias_[bi] = true;
            continue;
        }
        Step s;
        s.type = Step::kCopy;
        s.kernel = "state-copy";
        s.info.kernel = s.kernel;
        s.info.nodes = "state:" + graph_.tensors[out_id].name;
        s.reads = {out_id};
        s.build = [this, out_id, bi](Step& st) {
            st.src = values_[out_id].addr;
            st.dst = state_dev_.at(bi).get();
            st.bytes = values_[out_id].bytes;
        };
        s.info.bytes = 2.0 * values_[out_id].bytes;
        steps_.push_back(std::move(s));
    }
}

// ------------------------------------------------ allocation & parameters
void Backend::build_schedule()
{
    // Liveness of arena values over the step list.
    const long total = static_cast<long>(steps_.size());
    for (long si = 0; si < total; ++si) {
        for (auto id : steps_[si].writes) {
            Value& v = values_[id];
            if (v.kind == Value::kNone)
                v.kind = Value::kArena;
            if (v.kind == Value::kArena && v.first < 0)
                v.first = si;
            v.last = std::max(v.last, si);
        }
        for (auto id : steps_[si].reads) {
            Value& v = values_[values_[id].alias_of ? values_[id].alias_of : id];
            if (v.kind == Value::kArena || v.kind == Value::kNone)
                v.last = std::max(v.last, si);
        }
    }
    for (auto id : graph_.outputs) {
        Value& v = values_[id];
        if (std::find(absorbed_outputs_.begin(), absorbed_outputs_.end(), id) != absorbed_outputs_.end())
            continue;  // produced directly into its host staging buffer
        if (v.kind == Value::kNone)
            throw std::runtime_error("mlvc-b200: graph output is never produced");
        if (v.kind == Value::kArena)
            v.last = total;
    }
    if (keep_all_values_)
        for (auto& v : values_)
            if (v.kind == Value::kArena)
                v.last = total;
    // Greedy first-fit arena over [first, last] intervals (256-byte slots).
    std::vector<uint32_t> order;
    for (size_t id = 1; id < values_.size(); ++id)
        if (values_[id].kind == Value::kArena)
            order.push_back(static_cast<uint32_t>(id));
    std::sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        return values_[a].first != values_[b].first ? values_[a].first < values_[b].first : a < b;
    });
    std::vector<uint32_t> placed;
    size_t arena_bytes = 256;
    for (auto id : order) {
        Value& v = values_[id];
        const size_t size = align_up(std::max<size_t>(v.bytes, 1), 256);
        std::vector<std::pair<size_t, size_t>> busy;
        for (auto o : placed) {
            const Value& u = values_[o];
            if (!(u.last < v.first || v.last < u.first))
                busy.emplace_back(u.arena_off, u.arena_off + align_up(std::max<size_t>(u.bytes, 1), 256));
        }
        std::sort(busy.begin(), busy.end());
        size_t off = 0;
        for (const auto& [lo, hi] : busy) {
            if (lo >= off + size)
                break;
            off = std::max(off, hi);
        }
        v.arena_off = off;
        arena_bytes = std::max(arena_bytes, off + size);
        placed.push_back(id);
    }

    // Device memory.
    weights_dev_ = DeviceBuffer(std::max<size_t>(weights_host_.size(), 256));
    if (!weights_host_.empty())
        check(cuMemcpyHtoD(weights_dev_.get(), weights_host_.data(), weights_host_.size()), "cuMemcpyHtoD(weights)");
    prepped_dev_ = DeviceBuffer(std::max<size_t>(prepped_host_.size(), 256));
    if (!prepped_host_.empty())
        check(cuMemcpyHtoD(prepped_dev_.get(), prepped_host_.data(), prepped_host_.size()), "cuMemcpyHtoD(prepared)");
    arena_dev_ = DeviceBuffer(arena_bytes);
    check(cuMemsetD8(arena_dev_.get(), 0, arena_bytes), "cuMemsetD8(arena)");
    input_dev_.clear();
    input_stage_dev_.clear();
    output_stage_dev_.clear();
    state_dev_.clear();
    for (size_t k = 0; k < ext_inputs_.size(); ++k) {
        const uint32_t id = graph_.inputs[ext_inputs_[k]];
        Value& v = values_[id];
        input_dev_.emplace_back(align_up(v.bytes, 256));
        v.addr = input_dev_.back().get();
        const auto d = dims4(v.shape);
        const bool convert = v.nhwc && d[1] > 1 && d[2] * d[3] > 1;
        input_stage_dev_.emplace_back(convert ? align_up(v.bytes, 256) : 0);
    }
    for (const auto& b : bindings_) {
        const uint32_t id = graph_.inputs[b.input_index];
        Value& v = values_[id];
        state_dev_.emplace_back(align_up(v.bytes, 256));
        check(cuMemsetD8(state_dev_.back().get(), 0, state_dev_.back().bytes()), "cuMemsetD8(state)");
        v.addr = state_dev_.back().get();
    }
    for (size_t k = 0; k < ext_outputs_.size(); ++k) {
        const uint32_t id = graph_.outputs[ext_outputs_[k]];
        const Value& v = values_[id];
        const auto d = dims4(v.shape);
        const bool convert = (v.nhwc && d[1] > 1 && d[2] * d[3] > 1) ||
                             std::find(absorbed_outputs_.begin(), absorbed_outputs_.end(), id) != absorbed_outputs_.end();
        output_stage_dev_.emplace_back(convert ? align_up(v.bytes, 256) : 0);
    }
    for (size_t id = 1; id < values_.size(); ++id) {
        Value& v = values_[id];
        if (v.kind == Value::kArena)
            v.addr = arena_dev_.get() + v.arena_off;
        else if (v.kind == Value::kWeight)
            v.addr = weights_dev_.get() + v.weight_off;
    }
    for (size_t bi = 0; bi < bindings_.size(); ++bi)
        if (bi < state_alias_.size() && state_alias_[bi])
            values_[graph_.outputs[bindings_[bi].output_index]].addr = state_dev_.at(bi).get();
    for (auto& v : values_)
        if (v.alias_of)
            v.addr = values_[v.alias_of].addr + v.alias_off;
    for (auto id : graph_.outputs)
        if (!values_[id].addr &&
            std::find(absorbed_outputs_.begin(), absorbed_outputs_.end(), id) == absorbed_outputs_.end())
            throw std::runtime_error("mlvc-b200: unresolved graph output address");

    // The dynamic shared-memory limit is a property of the function, shared by
    // every step that launches it: set it once to the largest request.
    std::map<std::string, unsigned> smem_max;
    for (const auto& st : steps_)
        if (st.type == Step::kKernel) {
            const std::string& sym = st.symbol.empty() ? st.kernel : st.symbol;
            smem_max[sym] = std::max(smem_max[sym], st.smem);
        }
    for (const auto& [name, bytes] : smem_max)
        if (bytes > 48 * 1024)
            check(cuFuncSetAttribute(fn(name.c_str()), CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                     static_cast<int>(bytes)),
                  "cuFuncSetAttribute(smem)");
    step_info_.clear();
    for (auto& st : steps_) {
        if (st.type == Step::kKernel)
            st.f = fn((st.symbol.empty() ? st.kernel : st.symbol).c_str());
        if (st.build)
            st.build(st);
        st.info.kernel = st.kernel;
        st.info.grid = st.grid * st.grid_y * st.grid_z;
        st.info.block = st.block * st.block_y;
        st.info.smem = st.smem;
        step_info_.push_back(st.info);
    }
}

void Backend::launch_steps(CUstream s, size_t skip)
{
    // Kernels are launched with programmatic stream serialisation: each one
    // may start its prologue (barriers, TMEM, weight loads) while its
    // predecessor drains, and waits in-kernel (griddepcontrol.wait) before it
    // touches activations.  MLVC_B200_PDL=0 turns this off.
    const char* env = std::getenv("MLVC_B200_PDL");
    const bool pdl = !(env && env[0] == '0');
    for (size_t i = 0; i < steps_.size(); ++i) {
        if (i == skip)
            continue;
        auto& st = steps_[i];
        if (st.type == Step::kCopy) {
            check(cuMemcpyDtoDAsync(st.dst, st.src, st.bytes, s), "cuMemcpyDtoDAsync");
            continue;
        }
        void* args[] = {st.params.data()};
        if (!pdl) {
            check(cuLaunchKernel(st.f, st.grid, st.grid_y, st.grid_z, st.block, st.block_y, 1, st.smem, s, args,
                                 nullptr),
                  st.kernel.c_str());
            continue;
        }
        CUlaunchAttribute attr{};
        attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        attr.value.programmaticStreamSerializationAllowed = 1;
        CUlaunchConfig cfg{};
        cfg.gridDimX = st.grid;
        cfg.gridDimY = st.grid_y;
        cfg.gridDimZ = st.grid_z;
        cfg.blockDimX = st.block;
        cfg.blockDimY = st.block_y;
        cfg.blockDimZ = 1;
        cfg.sharedMemBytes = st.smem;
        cfg.hStream = s;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        check(cuLaunchKernelEx(&cfg, st.f, args, nullptr), st.kernel.c_str());
    }
}

void Backend::capture()
{
    check(cuStreamBeginCapture(stream_, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL), "cuStreamBeginCapture");
    try {
        launch_steps(stream_);
    } catch (...) {
        CUgraph g = nullptr;
        cuStreamEndCapture(stream_, &g);
        if (g)
            cuGraphDestroy(g);
        throw;
    }
    check(cuStreamEndCapture(stream_, &graph_handle_), "cuStreamEndCapture");
    check(cuGraphInstantiateWithFlags(&graph_exec_, graph_handle_, 0), "cuGraphInstantiate");
}

// In-graph kernel spans.  Consecutive kernels of a replayed frame overlap
// (programmatic dependent launch), so events between them would separate
// them only by removing the overlap.  Instead the schedule is captured once
// more with the phase trace of every tensor-core step enabled and replayed
// exactly like a frame; each such step's span is its last CTA's exit stamp
// minus its first CTA's entry stamp (%globaltimer, written by the kernel),
// averaged over the replays.  Steps without a trace report 0.
std::vector<float> Backend::trace_spans(int iterations, size_t flush_bytes)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (!loaded_)
        throw std::runtime_error("mlvc-b200: load() must be called before trace_spans()");
    if (iterations < 1)
        throw std::runtime_error("mlvc-b200: trace_spans needs at least one iteration");
    ContextGuard guard(ctx_);
    auto traced = [](const Step& st) {
        return st.type == Step::kKernel &&
               (st.kernel == "mlvc_conv1x1_tc" || st.kernel == "mlvc_convkxk_tc" || st.kernel == "mlvc_ffn_tc" ||
                st.kernel == "mlvc_dwconv_tc" || st.kernel == "mlvc_mbconv_tc");
    };
    std::vector<size_t> offs(steps_.size(), 0);
    size_t total = 0;
    for (size_t k = 0; k < steps_.size(); ++k)
        if (traced(steps_[k])) {
            offs[k] = total;
            total += static_cast<size_t>(steps_[k].grid) * kTracePoints;
        }
    std::vector<float> out(steps_.size(), 0.0f);
    if (total == 0)
        return out;
    DeviceBuffer buf(total * sizeof(uint64_t));
    if (flush_bytes && flush_dev_.bytes() < flush_bytes)
        flush_dev_ = DeviceBuffer(flush_bytes);
    // patch the trace pointers in, capture, restore the normal parameters
    std::vector<std::vector<uint8_t>> saved(steps_.size());
    for (size_t k = 0; k < steps_.size(); ++k)
        if (traced(steps_[k])) {
            saved[k] = steps_[k].params;
            unsigned long long* ptr = reinterpret_cast<unsigned long long*>(buf.get() + offs[k] * sizeof(uint64_t));
            std::memcpy(steps_[k].params.data() + offsetof(ConvTcParams, trace), &ptr, sizeof(ptr));
        }
    CUgraph g = nullptr;
    CUgraphExec ge = nullptr;
    CUresult rc = cuStreamBeginCapture(stream_, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL);
    if (rc == CUDA_SUCCESS) {
        try {
            launch_steps(stream_);
        } catch (...) {
            rc = CUDA_ERROR_UNKNOWN;
        }
        const CUresult end = cuStreamEndCapture(stream_, &g);
        if (rc == CUDA_SUCCESS)
            rc = end;
        if (rc == CUDA_SUCCESS)
            rc = cuGraphInstantiateWithFlags(&ge, g, 0);
    }
    for (size_t k = 0; k < steps_.size(); ++k)
        if (!saved[k].empty())
            steps_[k].params = std::move(saved[k]);
    if (rc != CUDA_SUCCESS) {
        if (g)
            cuGraphDestroy(g);
        check(rc, "capture (trace_spans)");
    }
    std::vector<uint64_t> host(total);
    std::vector<double> acc(steps_.size(), 0.0);
    try {
        for (int it = 0; it < iterations; ++it) {
            if (flush_bytes)
                check(cuMemsetD8Async(flush_dev_.get(), static_cast<unsigned char>(it), flush_bytes, stream_),
                      "cuMemsetD8Async(flush)");
            check(cuMemsetD8Async(buf.get(), 0, buf.bytes(), stream_), "cuMemsetD8Async(trace)");
            check(cuGraphLaunch(ge, stream_), "cuGraphLaunch(trace_spans)");
            check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
            check(cuMemcpyDtoH(host.data(), buf.get(), buf.bytes()), "cuMemcpyDtoH(trace)");
            for (size_t k = 0; k < steps_.size(); ++k) {
                if (!traced(steps_[k]))
                    continue;
                // from the first CTA whose producer passed griddepcontrol.wait
                // (the previous kernel's outputs visible; the prologue before it
                // overlaps the previous kernel) to the last CTA's exit
                uint64_t first = UINT64_MAX, last = 0;
                for (unsigned c = 0; c < steps_[k].grid; ++c) {
                    const uint64_t* s = host.data() + offs[k] + static_cast<size_t>(c) * kTracePoints;
                    const uint64_t start = s[kTrDepReady] ? s[kTrDepReady] : s[kTrEntry];
                    if (start)
                        first = std::min<uint64_t>(first, start);
                    last = std::max<uint64_t>(last, s[kTrExit]);
                }
                if (first != UINT64_MAX && last > first)
                    acc[k] += static_cast<double>(last - first) * 1e-6;  // ns -> ms
            }
        }
    } catch (...) {
        cuGraphExecDestroy(ge);
        cuGraphDestroy(g);
        throw;
    }
    cuGraphExecDestroy(ge);
    cuGraphDestroy(g);
    check_status();
    for (size_t k = 0; k < steps_.size(); ++k)
        out[k] = static_cast<float>(acc[k] / iterations);
    return out;
}

int Backend::kernel_launches_per_run() const
{
    int n = 0;
    for (const auto& st : steps_)
        n += st.type == Step::kKernel ? 1 : 0;
    return n;
}

size_t Backend::device_bytes() const
{
    size_t t = weights_dev_.bytes() + prepped_dev_.bytes() + arena_dev_.bytes();
    for (const auto* v : {&input_dev_, &input_stage_dev_, &output_stage_dev_, &state_dev_})
        for (const auto& b : *v)
            t += b.bytes();
    return t;
}

std::vector<uint64_t> Backend::trace_step(size_t index)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    Step& st = steps_.at(index);
    if (st.kernel != "mlvc_conv1x1_tc" && st.kernel != "mlvc_convkxk_tc" && st.kernel != "mlvc_ffn_tc" &&
        st.kernel != "mlvc_dwconv_tc" && st.kernel != "mlvc_mbconv_tc")
        throw std::runtime_error("mlvc-b200: only tensor-core conv steps carry a phase trace");
    ContextGuard guard(ctx_);
    const size_t n = static_cast<size_t>(st.grid) * kTracePoints;
    DeviceBuffer buf(n * sizeof(uint64_t));
    check(cuMemsetD8(buf.get(), 0, buf.bytes()), "cuMemsetD8(trace)");
    std::vector<uint8_t> params = st.params;
    unsigned long long* ptr = reinterpret_cast<unsigned long long*>(buf.get());
    std::memcpy(params.data() + offsetof(ConvTcParams, trace), &ptr, sizeof(ptr));
    void* args[] = {params.data()};
    check(cuLaunchKernel(st.f, st.grid, st.grid_y, st.grid_z, st.block, st.block_y, 1, st.smem, stream_, args, nullptr),
          "cuLaunchKernel(trace)");
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
    std::vector<uint64_t> out(n);
    check(cuMemcpyDtoH(out.data(), buf.get(), buf.bytes()), "cuMemcpyDtoH(trace)");
    check_status();
    return out;
}

uint32_t Backend::test_wait_expiry(size_t index, uint64_t limit_ns)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (!loaded_)
        throw std::runtime_error("mlvc-b200: load() must be called before test_wait_expiry()");
    Step& st = steps_.at(index);
    if (st.kernel != "mlvc_conv1x1_tc")
        throw std::runtime_error("mlvc-b200: the wait-expiry test relaunches a mlvc_conv1x1_tc step");
    constexpr uint64_t kDefaultLimit = 2000000000ull;  // the kernels' kWaitLimitNs
    if (limit_ns == 0 || limit_ns > kDefaultLimit)
        throw std::runtime_error("mlvc-b200: wait limit must be in (0, 2 s]");
    ContextGuard guard(ctx_);
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
    check_status();
    CUdeviceptr limit_ptr = 0;
    size_t limit_size = 0;
    check(cuModuleGetGlobal(&limit_ptr, &limit_size, module_, "mlvc_b200_wait_limit_ns"),
          "cuModuleGetGlobal(mlvc_b200_wait_limit_ns)");
    const unsigned long long shortened = limit_ns, restored = kDefaultLimit;
    check(cuMemcpyHtoD(limit_ptr, &shortened, sizeof(shortened)), "cuMemcpyHtoD(wait limit)");
    std::vector<uint8_t> params = st.params;
    const int withhold = 1;
    std::memcpy(params.data() + offsetof(ConvTcParams, withhold_a), &withhold, sizeof(withhold));
    void* args[] = {params.data()};
    CUresult launched = cuLaunchKernel(st.f, st.grid, st.grid_y, st.grid_z, st.block, st.block_y, 1, st.smem, stream_,
                                       args, nullptr);
    const CUresult finished = launched == CUDA_SUCCESS ? cuStreamSynchronize(stream_) : launched;
    const CUresult reset = cuMemcpyHtoD(limit_ptr, &restored, sizeof(restored));
    check(launched, "cuLaunchKernel(wait expiry)");
    check(finished, "cuStreamSynchronize(wait expiry)");
    check(reset, "cuMemcpyHtoD(wait limit)");
    unsigned int status = 0;
    check(cuMemcpyDtoH(&status, status_ptr_, sizeof(status)), "cuMemcpyDtoH(status)");
    const unsigned int zero = 0;
    check(cuMemcpyHtoD(status_ptr_, &zero, sizeof(zero)), "cuMemcpyHtoD(status)");
    return status;
}

void Backend::set_keep_all_values(bool keep)
{
    if (loaded_)
        throw std::runtime_error("mlvc-b200: debug tensor mode must be set before load()");
    keep_all_values_ = keep;
}

bool Backend::read_value(const std::string& name, void* dst, size_t bytes)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (!keep_all_values_)
        throw std::runtime_error("mlvc-b200: tensor read-back needs debug tensor mode (set before load)");
    for (size_t id = 1; id < values_.size(); ++id) {
        const Value& v = values_[id];
        if (!v.present || graph_.tensors[id].name != name)
            continue;
        if (!v.addr || v.kind == Value::kNone)
            return false;
        if (bytes < v.bytes)
            throw std::runtime_error("mlvc-b200: read_value buffer too small");
        ContextGuard guard(ctx_);
        check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
        std::vector<uint8_t> tmp(v.bytes);
        check(cuMemcpyDtoH(tmp.data(), v.addr, v.bytes), "cuMemcpyDtoH(read_value)");
        const auto d = dims4(v.shape);
        if (v.nhwc && d[1] > 1 && d[2] * d[3] > 1) {  // NHWC -> NCHW
            const auto* src = reinterpret_cast<const uint16_t*>(tmp.data());
            auto* out = static_cast<uint16_t*>(dst);
            const long long C = d[1], HW = d[2] * d[3];
            for (long long n = 0; n < d[0]; ++n)
                for (long long p = 0; p < HW; ++p)
                    for (long long c = 0; c < C; ++c)
                        out[(n * C + c) * HW + p] = src[(n * HW + p) * C + c];
        } else {
            std::memcpy(dst, tmp.data(), v.bytes);
        }
        return true;
    }
    throw std::runtime_error("mlvc-b200: no tensor named " + name);
}

void Backend::check_status()
{
    unsigned int status = 0;
    check(cuMemcpyDtoH(&status, status_ptr_, sizeof(status)), "cuMemcpyDtoH(status)");
    if (status) {
        const unsigned int zero = 0;
        cuMemcpyHtoD(status_ptr_, &zero, sizeof(zero));
        std::ostringstream os;
        os << "mlvc-b200:";
        if (status & 0xffu)  // wait-timeout / alignment bits of the tensor-core kernels
            os << " a device-side wait timed out or a TMA destination was misaligned;";
        if (status & 0x100u)  // mlvc_gather_rows_f16 (reference: "cpu: GATHER index out of range")
            os << " GATHER index out of range;";
        os << " status 0x" << std::hex << status;
        throw std::runtime_error(os.str());
    }
}

// -------------------------------------------------------------- execution
void Backend::run(const HostTensorRef* inputs, size_t n_in, HostTensorRef* outputs, size_t n_out)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (!loaded_)
        throw std::runtime_error("mlvc-b200: load() must be called before run()");
    if (!state_ready_)
        throw std::runtime_error("mlvc-b200: reset_state() must be called before run()");
    if (n_in != ext_inputs_.size() || n_out != ext_outputs_.size())
        throw std::runtime_error("mlvc-b200: graph input/output count mismatch");
    ContextGuard guard(ctx_);
    for (size_t k = 0; k < n_in; ++k) {
        const TensorDesc& d = input_desc(k);
        const HostTensorRef& h = inputs[k];
        const int want = d.dtype == DType::kInt32 ? 1 : 0;
        bool ok = h.dtype == want && h.rank == static_cast<int>(d.shape.size()) && h.data &&
                  h.bytes == static_cast<size_t>(element_count(d.shape)) * dtype_size(d.dtype);
        for (int r = 0; ok && r < h.rank; ++r)
            ok = h.shape[r] == d.shape[r];
        if (!ok)
            throw std::runtime_error("mlvc-b200: graph input shape, dtype, or byte size mismatch (" + d.name + ")");
        const CUdeviceptr dst = input_stage_dev_[k] ? input_stage_dev_[k].get() : input_dev_[k].get();
        check(cuMemcpyHtoDAsync(dst, h.data, h.bytes, stream_), "cuMemcpyHtoDAsync(input)");
    }
    check(cuGraphLaunch(graph_exec_, stream_), "cuGraphLaunch");
    for (size_t k = 0; k < n_out; ++k) {
        const TensorDesc& d = output_desc(k);
        HostTensorRef& h = outputs[k];
        const size_t bytes = static_cast<size_t>(element_count(d.shape)) * dtype_size(d.dtype);
        if (!h.data || h.bytes < bytes)
            throw std::runtime_error("mlvc-b200: output buffer too small (" + d.name + ")");
        const uint32_t id = graph_.outputs[ext_outputs_[k]];
        const CUdeviceptr src = output_stage_dev_[k] ? output_stage_dev_[k].get() : values_[id].addr;
        check(cuMemcpyDtoHAsync(h.data, src, bytes, stream_), "cuMemcpyDtoHAsync(output)");
        h.dtype = d.dtype == DType::kInt32 ? 1 : 0;
        h.rank = static_cast<int>(d.shape.size());
        for (int r = 0; r < h.rank; ++r)
            h.shape[r] = d.shape[r];
        h.bytes = bytes;
    }
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
    check_status();
}

void Backend::reset_state()
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (!loaded_)
        throw std::runtime_error("mlvc-b200: load() must be called before reset_state()");
    ContextGuard guard(ctx_);
    for (auto& b : state_dev_)
        check(cuMemsetD8Async(b.get(), 0, b.bytes(), stream_), "cuMemsetD8Async(state)");
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
    state_ready_ = true;
}

// ------------------------------------------------- entropy-coder inputs
void Backend::scale_plane(const ScaleConfig& c, int* z_height, int* z_width, int* y_height, int* y_width)
{
    if (c.hyperprior_channels <= 0 || c.model_width <= 0 || c.model_height <= 0 || c.latent_channels <= 0 ||
        c.downsample_latent <= 0 || c.downsample_hyperprior <= 0 || c.y_scale_repeat <= 0 || c.scale_max_index < 0)
        throw std::runtime_error("mlvc-b200: scale configuration values must be positive");
    auto ceil_div = [](long long a, long long b) { return static_cast<int>((a + b - 1) / b); };
    const long long zf = static_cast<long long>(c.downsample_latent) * c.downsample_hyperprior;
    *z_height = ceil_div(c.model_height, zf);
    *z_width = ceil_div(c.model_width, zf);
    *y_height = ceil_div(c.model_height, c.downsample_latent);
    *y_width = ceil_div(c.model_width, c.downsample_latent);
    const int half = c.latent_channels / 2, base = c.latent_channels / c.y_scale_repeat;
    if (base > c.hyperprior_channels)
        throw std::runtime_error("scale decoder channel mapping is invalid");
    // The reference indexes its base table with (channel + half) / repeat
    // without a bound; reject the configurations where that leaves the table.
    if (half == 0 || (2 * half - 1) / c.y_scale_repeat >= base)
        throw std::runtime_error("scale decoder channel mapping is invalid");
}

void Backend::extract_scales_device(CUdeviceptr z, const ScaleConfig& cfg, CUdeviceptr scales_0, CUdeviceptr scales_1)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    int zh = 0, zw = 0, yh = 0, yw = 0;
    scale_plane(cfg, &zh, &zw, &yh, &yw);
    const size_t out_count = static_cast<size_t>(cfg.latent_channels / 2) * yh * yw;
    ContextGuard guard(ctx_);
    ScaleParams sp{};
    sp.z = reinterpret_cast<const mlvc_half*>(z);
    sp.scales_0 = reinterpret_cast<int32_t*>(scales_0);
    sp.scales_1 = reinterpret_cast<int32_t*>(scales_1);
    sp.z_height = zh;
    sp.z_width = zw;
    sp.latent = cfg.latent_channels;
    sp.repeat = cfg.y_scale_repeat;
    sp.y_height = yh;
    sp.y_width = yw;
    sp.spatial = cfg.downsample_hyperprior;
    sp.max_index = cfg.scale_max_index;
    sp.vec4 = yw % 4 == 0 && scales_0 % 16 == 0 && scales_1 % 16 == 0;
    void* args[] = {&sp};
    const unsigned grid = blocks_for(static_cast<long long>(sp.vec4 ? out_count / 4 : out_count), 256, sm_count_);
    check(cuLaunchKernel(fn("mlvc_extract_scales"), grid, 1, 1, 256, 1, 1, 0, stream_, args, nullptr),
          "mlvc_extract_scales");
}

void Backend::integer_values_device(CUdeviceptr values, size_t count, CUdeviceptr symbols, CUdeviceptr out_of_range)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (count == 0)
        return;
    ContextGuard guard(ctx_);
    IntegerValuesParams ip{};
    ip.src = reinterpret_cast<const mlvc_half*>(values);
    ip.dst = reinterpret_cast<int32_t*>(symbols);
    ip.count = static_cast<long long>(count);
    ip.out_of_range = reinterpret_cast<unsigned int*>(out_of_range);
    ip.vec8 = values % 16 == 0 && symbols % 16 == 0;
    void* args[] = {&ip};
    const unsigned grid = blocks_for(static_cast<long long>(ip.vec8 ? (count + 7) / 8 : count), 256, sm_count_);
    check(cuLaunchKernel(fn("mlvc_integer_values_f16"), grid, 1, 1, 256, 1, 1, 0, stream_, args, nullptr),
          "mlvc_integer_values_f16");
}

CUdeviceptr Backend::entropy_scratch(size_t bytes)
{
    if (entropy_scratch_.bytes() < bytes) {
        check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
        entropy_scratch_ = DeviceBuffer(bytes);
    }
    return entropy_scratch_.get();
}

void Backend::extract_scales(const uint16_t* z, const ScaleConfig& cfg, int32_t* scales_0, int32_t* scales_1)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    int zh = 0, zw = 0, yh = 0, yw = 0;
    scale_plane(cfg, &zh, &zw, &yh, &yw);
    const size_t z_bytes = (static_cast<size_t>(cfg.hyperprior_channels) * zh * zw * 2 + 255) & ~size_t{255};
    const size_t out_bytes = static_cast<size_t>(cfg.latent_channels / 2) * yh * yw * sizeof(int32_t);
    ContextGuard guard(ctx_);
    const CUdeviceptr buf = entropy_scratch(z_bytes + 2 * out_bytes);
    const CUdeviceptr s0 = buf + z_bytes, s1 = s0 + out_bytes;
    check(cuMemcpyHtoDAsync(buf, z, static_cast<size_t>(cfg.hyperprior_channels) * zh * zw * 2, stream_),
          "cuMemcpyHtoDAsync(z)");
    extract_scales_device(buf, cfg, s0, s1);
    check(cuMemcpyDtoHAsync(scales_0, s0, out_bytes, stream_), "cuMemcpyDtoHAsync(scales_0)");
    check(cuMemcpyDtoHAsync(scales_1, s1, out_bytes, stream_), "cuMemcpyDtoHAsync(scales_1)");
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
}

void Backend::integer_values(const uint16_t* values, size_t count, int32_t* symbols)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (count == 0)
        return;
    ContextGuard guard(ctx_);
    const size_t src_bytes = (count * 2 + 255) & ~size_t{255};
    const CUdeviceptr src = entropy_scratch(src_bytes + count * sizeof(int32_t) + 16);
    const CUdeviceptr dst = src + src_bytes, flag = dst + count * sizeof(int32_t);
    check(cuMemsetD8Async(flag, 0, sizeof(uint32_t), stream_), "cuMemsetD8Async(flag)");
    check(cuMemcpyHtoDAsync(src, values, count * 2, stream_), "cuMemcpyHtoDAsync(values)");
    integer_values_device(src, count, dst, flag);
    uint32_t bad = 0;
    check(cuMemcpyDtoHAsync(&bad, flag, sizeof(bad), stream_), "cuMemcpyDtoHAsync(flag)");
    check(cuMemcpyDtoHAsync(symbols, dst, count * sizeof(int32_t), stream_), "cuMemcpyDtoHAsync(symbols)");
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
    if (bad)
        throw std::runtime_error("entropy symbol is outside signed 16-bit range");
}

void Backend::configure_slots(size_t count)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (!loaded_)
        throw std::runtime_error("mlvc-b200: load() must be called before configure_slots()");
    if (count == 0 || count > 16)
        throw std::runtime_error("mlvc-b200: slot count must be in [1, 16]");
    ContextGuard guard(ctx_);
    for (auto& s : slots_)
        if (s.pending)
            check(cuEventSynchronize(s.done.get()), "cuEventSynchronize");
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
    slots_.clear();
    if (!copy_in_)
        check(cuStreamCreate(&copy_in_, CU_STREAM_NON_BLOCKING), "cuStreamCreate(copy in)");
    if (!copy_out_)
        check(cuStreamCreate(&copy_out_, CU_STREAM_NON_BLOCKING), "cuStreamCreate(copy out)");
    slots_ = std::vector<Slot>(count);
    const size_t yuv_bytes = static_cast<size_t>(codec_.width) * codec_.height * 3 / 2;
    auto yuv_launch = [&](const char* kernel, YuvParams yp, long long work) {
        void* args[] = {&yp};
        const unsigned grid = blocks_for(work, 256, sm_count_);
        check(cuLaunchKernel(fn(kernel), grid, 1, 1, 256, 1, 1, 0, stream_, args, nullptr), kernel);
    };
    auto yuv_params = [&]() {
        YuvParams yp{};
        yp.width = codec_.width;
        yp.height = codec_.height;
        yp.model_width = codec_.model_width;
        yp.model_height = codec_.model_height;
        yp.pad_left = codec_.pad_left;
        yp.pad_top = codec_.pad_top;
        yp.rotated = codec_.rotated ? 1 : 0;
        yp.pixel_range = codec_.pixel_range;
        return yp;
    };
    // The decoded frame straight from the NHWC tensor that the x8 output
    // boundary would convert (mlvc_nhwc8_to_yuv420): the boundary step is left
    // out of the slot graphs when the frame is not rotated and sits on the
    // canvas at multiples of 8 (MLVC_B200_YUV_FUSION=0: boundary + conversion).
    size_t& fused_yuv_step = fused_yuv_step_;
    fused_yuv_step = static_cast<size_t>(-1);
    CUdeviceptr fused_yuv_src = 0;
    {
        const char* env = std::getenv("MLVC_B200_YUV_FUSION");
        const bool allowed = !(env && env[0] == '0');
        if (allowed && codec_.output != kNoCodecTensor && !codec_.rotated && codec_.width % 8 == 0 &&
            codec_.height % 8 == 0 && codec_.pad_left % 8 == 0 && codec_.pad_top % 8 == 0 &&
            codec_.pad_left + codec_.width <= codec_.model_width && codec_.pad_top + codec_.height <= codec_.model_height &&
            output_stage_dev_.at(codec_.output)) {
            const CUdeviceptr stage = output_stage_dev_[codec_.output].get();
            for (size_t i = 0; i < steps_.size(); ++i) {
                const Step& st = steps_[i];
                if (st.type != Step::kKernel || st.kernel != "mlvc_boundary_f16" ||
                    st.params.size() != sizeof(BoundaryParams))
                    continue;
                BoundaryParams bp;
                std::memcpy(&bp, st.params.data(), sizeof(bp));
                if (bp.to_host && bp.r == 8 && bp.c == 192 && bp.n == 1 &&
                    reinterpret_cast<CUdeviceptr>(bp.dst) == stage && bp.w * 8 == codec_.model_width &&
                    bp.h * 8 == codec_.model_height && reinterpret_cast<uintptr_t>(bp.src) % 16 == 0) {
                    fused_yuv_step = i;
                    fused_yuv_src = reinterpret_cast<CUdeviceptr>(bp.src);
                }
            }
        }
    }
    for (auto& s : slots_) {
        for (size_t k = 0; k < ext_inputs_.size(); ++k) {
            const auto& d = input_desc(k);
            const size_t bytes = k == codec_.input ? yuv_bytes
                                                   : static_cast<size_t>(element_count(d.shape)) * dtype_size(d.dtype);
            s.in.emplace_back(bytes);
            s.din.emplace_back(align_up(bytes, 256));
        }
        for (size_t k = 0; k < ext_outputs_.size(); ++k) {
            const auto& d = output_desc(k);
            const size_t bytes = k == codec_.output ? yuv_bytes
                                                    : static_cast<size_t>(element_count(d.shape)) * dtype_size(d.dtype);
            s.out.emplace_back(bytes);
            s.dout.emplace_back(align_up(bytes, 256));
        }
        // graph: staged inputs -> schedule inputs (a YUV frame through the
        // YUV -> tensor kernel), schedule, outputs -> staging (the decoded
        // frame through the tensor -> YUV kernel)
        check(cuStreamBeginCapture(stream_, CU_STREAM_CAPTURE_MODE_THREAD_LOCAL), "cuStreamBeginCapture(slot)");
        try {
            for (size_t k = 0; k < ext_inputs_.size(); ++k) {
                const CUdeviceptr dst = input_stage_dev_[k] ? input_stage_dev_[k].get() : input_dev_[k].get();
                if (k == codec_.input) {
                    YuvParams yp = yuv_params();
                    yp.yuv_in = reinterpret_cast<const uint8_t*>(s.din[k].get());
                    yp.t_out = reinterpret_cast<mlvc_half*>(dst);
                    yuv_launch("mlvc_yuv420_to_tensor_f16", yp,
                               3LL * codec_.model_width * static_cast<long long>(codec_.model_height));
                } else {
                    check(cuMemcpyDtoDAsync(dst, s.din[k].get(), s.in[k].bytes(), stream_), "cuMemcpyDtoDAsync(slot in)");
                }
            }
            launch_steps(stream_, fused_yuv_step);
            for (size_t k = 0; k < ext_outputs_.size(); ++k) {
                const uint32_t id = graph_.outputs[ext_outputs_[k]];
                const CUdeviceptr src = output_stage_dev_[k] ? output_stage_dev_[k].get() : values_[id].addr;
                if (k == codec_.output && fused_yuv_src) {
                    YuvParams yp = yuv_params();
                    yp.t_in = reinterpret_cast<const mlvc_half*>(fused_yuv_src);
                    yp.yuv_out = reinterpret_cast<uint8_t*>(s.dout[k].get());
                    yuv_launch("mlvc_nhwc8_to_yuv420", yp, static_cast<long long>(codec_.width) * codec_.height / 8);
                } else if (k == codec_.output) {
                    YuvParams yp = yuv_params();
                    yp.t_in = reinterpret_cast<const mlvc_half*>(src);
                    yp.yuv_out = reinterpret_cast<uint8_t*>(s.dout[k].get());
                    yuv_launch("mlvc_tensor_to_yuv420", yp, static_cast<long long>(codec_.width) * codec_.height);
                } else {
                    check(cuMemcpyDtoDAsync(s.dout[k].get(), src, s.out[k].bytes(), stream_), "cuMemcpyDtoDAsync(slot out)");
                }
            }
        } catch (...) {
            CUgraph g = nullptr;
            cuStreamEndCapture(stream_, &g);
            if (g)
                cuGraphDestroy(g);
            throw;
        }
        check(cuStreamEndCapture(stream_, &s.graph), "cuStreamEndCapture(slot)");
        check(cuGraphInstantiateWithFlags(&s.exec, s.graph, 0), "cuGraphInstantiate(slot)");
    }
}

size_t Backend::slot_count() const { return slots_.size(); }

void* Backend::slot_input(size_t slot, size_t i) { return slots_.at(slot).in.at(i).get(); }
const void* Backend::slot_output(size_t slot, size_t i) const { return slots_.at(slot).out.at(i).get(); }

// Reference: BufferedCodecBackend::configure_codec_io with CodecIoConfig
// (runtime/include/mlvc/runtime/backend.hpp:69-83) and the frame placement of
// frame_padding (core/src/yuv.cpp:324-337).
void Backend::configure_codec_io(int width, int height, int model_width, int model_height, float pixel_range,
                                 size_t slots, size_t input_index, size_t output_index)
{
    if (!loaded_)
        throw std::runtime_error("mlvc-b200: load() must be called before configure_codec_io()");
    auto even = [](int w, int h) { return w > 0 && h > 0 && w % 2 == 0 && h % 2 == 0; };
    if (!even(width, height) || !even(model_width, model_height))
        throw std::runtime_error("mlvc-b200: YUV420 dimensions must be positive and even");
    if (!std::isfinite(pixel_range) || pixel_range <= 0.0f)
        throw std::runtime_error("mlvc-b200: pixel range must be finite and positive");
    const bool native = width <= model_width && height <= model_height;
    const bool rotated = height <= model_width && width <= model_height;
    if (!native && !rotated)
        throw std::runtime_error("mlvc-b200: input frame is larger than the model dimensions");
    auto check_tensor = [&](const TensorDesc& d, const char* what) {
        const std::vector<int64_t> want{1, 3, model_height, model_width};
        if (d.dtype != DType::kFp16 || d.shape != want)
            throw std::runtime_error(std::string("mlvc-b200: codec ") + what + " must be FP16 [1, 3, model_height, model_width]");
    };
    if (input_index != kNoCodecTensor) {
        if (input_index >= ext_inputs_.size())
            throw std::runtime_error("mlvc-b200: codec input index out of range");
        check_tensor(input_desc(input_index), "input");
    }
    if (output_index != kNoCodecTensor) {
        if (output_index >= ext_outputs_.size())
            throw std::runtime_error("mlvc-b200: codec output index out of range");
        check_tensor(output_desc(output_index), "output");
    }
    CodecIo c;
    c.width = width;
    c.height = height;
    c.model_width = model_width;
    c.model_height = model_height;
    c.pixel_range = pixel_range;
    c.rotated = !native;
    c.pad_left = 0;
    c.pad_top = 0;
    c.input = input_index;
    c.output = output_index;
    codec_ = c;
    configure_slots(slots);
}

void Backend::slot_input_yuv(size_t slot, uint8_t** y, uint8_t** u, uint8_t** v)
{
    if (codec_.input == kNoCodecTensor)
        throw std::runtime_error("mlvc-b200: no codec input configured");
    auto* base = static_cast<uint8_t*>(slot_input(slot, codec_.input));
    const size_t ys = static_cast<size_t>(codec_.width) * codec_.height;
    *y = base;
    *u = base + ys;
    *v = base + ys + ys / 4;
}

void Backend::slot_output_yuv(size_t slot, const uint8_t** y, const uint8_t** u, const uint8_t** v) const
{
    if (codec_.output == kNoCodecTensor)
        throw std::runtime_error("mlvc-b200: no codec output configured");
    const auto* base = static_cast<const uint8_t*>(slot_output(slot, codec_.output));
    const size_t ys = static_cast<size_t>(codec_.width) * codec_.height;
    *y = base;
    *u = base + ys;
    *v = base + ys + ys / 4;
}

void Backend::submit(size_t slot)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    if (!state_ready_)
        throw std::runtime_error("mlvc-b200: reset_state() must be called before submit()");
    ContextGuard guard(ctx_);
    Slot& s = slots_.at(slot);
    if (s.pending)
        throw std::runtime_error("mlvc-b200: slot resubmitted before wait_slot()");
    // host -> device on the input copy stream, once the slot's previous graph
    // has read its device staging
    check(cuStreamWaitEvent(copy_in_, s.computed.get(), 0), "cuStreamWaitEvent(copy in)");
    for (size_t k = 0; k < ext_inputs_.size(); ++k)
        check(cuMemcpyHtoDAsync(s.din[k].get(), s.in[k].get(), s.in[k].bytes(), copy_in_), "cuMemcpyHtoDAsync(slot)");
    check(cuEventRecord(s.in_done.get(), copy_in_), "cuEventRecord(in)");
    // the schedule, in submission order on the compute stream (recurrent state
    // passes from frame to frame there)
    check(cuStreamWaitEvent(stream_, s.in_done.get(), 0), "cuStreamWaitEvent(compute)");
    check(cuGraphLaunch(s.exec, stream_), "cuGraphLaunch(slot)");
    check(cuEventRecord(s.computed.get(), stream_), "cuEventRecord(computed)");
    // device -> host on the output copy stream
    check(cuStreamWaitEvent(copy_out_, s.computed.get(), 0), "cuStreamWaitEvent(copy out)");
    for (size_t k = 0; k < ext_outputs_.size(); ++k)
        check(cuMemcpyDtoHAsync(s.out[k].get(), s.dout[k].get(), s.out[k].bytes(), copy_out_), "cuMemcpyDtoHAsync(slot)");
    check(cuEventRecord(s.done.get(), copy_out_), "cuEventRecord(done)");
    s.pending = true;
}

void Backend::submit_q(size_t slot, int shifted_q)
{
    size_t index = ext_inputs_.size();
    for (size_t k = 0; k < ext_inputs_.size(); ++k)
        if (input_desc(k).name == "q_index_shifted")
            index = k;
    if (index == ext_inputs_.size())
        throw std::runtime_error("mlvc-b200: graph has no q_index_shifted input");
    const auto& d = input_desc(index);
    if (d.dtype != DType::kInt32 || d.shape != std::vector<int64_t>{1} || index == codec_.input)
        throw std::runtime_error("mlvc-b200: invalid q_index_shifted input");
    if (slots_.at(slot).pending)
        throw std::runtime_error("mlvc-b200: slot resubmitted before wait_slot()");
    std::memcpy(slot_input(slot, index), &shifted_q, sizeof(shifted_q));
    submit(slot);
}

void Backend::wait_slot(size_t slot)
{
    ContextGuard guard(ctx_);
    Slot& s = slots_.at(slot);
    if (s.pending) {
        check(cuEventSynchronize(s.done.get()), "cuEventSynchronize");
        s.pending = false;
    }
    check_status();
}

void Backend::enqueue()
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    ContextGuard guard(ctx_);
    check(cuGraphLaunch(graph_exec_, stream_), "cuGraphLaunch");
}

void Backend::synchronize()
{
    ContextGuard guard(ctx_);
    check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
    check_status();
}

std::vector<float> Backend::time_steps(int iterations, size_t flush_bytes)
{
    if (offline_)
        throw std::runtime_error("mlvc-b200: planning-only backend cannot execute");
    ContextGuard guard(ctx_);
    // With flush_bytes > 0 every step runs after a memset of a buffer larger
    // than L2, i.e. from a cold cache, and only the step itself is timed.
    if (flush_bytes && flush_dev_.bytes() < flush_bytes)
        flush_dev_ = DeviceBuffer(flush_bytes);
    std::vector<Event> ev(2 * steps_.size());
    std::vector<double> acc(steps_.size(), 0.0);
    for (int it = 0; it < iterations; ++it) {
        for (size_t k = 0; k < steps_.size(); ++k) {
            auto& st = steps_[k];
            if (flush_bytes)
                check(cuMemsetD8Async(flush_dev_.get(), static_cast<unsigned char>(it + k), flush_bytes, stream_),
                      "cuMemsetD8Async(flush)");
            check(cuEventRecord(ev[2 * k].get(), stream_), "cuEventRecord");
            if (st.type == Step::kCopy) {
                check(cuMemcpyDtoDAsync(st.dst, st.src, st.bytes, stream_), "cuMemcpyDtoDAsync");
            } else {
                void* args[] = {st.params.data()};
                check(cuLaunchKernel(st.f, st.grid, st.grid_y, st.grid_z, st.block, st.block_y, 1, st.smem, stream_,
                                     args, nullptr),
                      st.kernel.c_str());
            }
            check(cuEventRecord(ev[2 * k + 1].get(), stream_), "cuEventRecord");
        }
        check(cuStreamSynchronize(stream_), "cuStreamSynchronize");
        for (size_t k = 0; k < steps_.size(); ++k) {
            float ms = 0.0f;
            check(cuEventElapsedTime(&ms, ev[2 * k].get(), ev[2 * k + 1].get()), "cuEventElapsedTime");
            acc[k] += ms;
        }
    }
    check_status();
    std::vector<float> out(steps_.size());
    for (size_t k = 0; k < steps_.size(); ++k)
        out[k] = static_cast<float>(acc[k] / std::max(1, iterations));
    return out;
}

}  // namespace mlvc_b200
