// Test infrastructure only (oracle side). Never linked into the product.
//
// A small extern "C" surface over the reference's own CPU backend
// (backends/cpu/src/cpu_backend.cpp:16-127, compiled unchanged) so that the
// Python tests and bench.py's reference arm can drive the reference
// InferenceBackend contract (runtime/include/mlvc/runtime/backend.hpp:48-63)
// through ctypes: create -> load(model, state bindings) -> reset_state ->
// run(inputs) -> outputs.  Errors are reported as a non-zero return plus a
// message, the same convention as the reference C ABI (codec/src/c_api.cpp:60-88).
#include "mlvc/core/assets.hpp"
#include "mlvc/core/yuv.hpp"
#include "mlvc/runtime/backend.hpp"

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace mlvc::cpu_backend {
void register_cpu_backend(bool make_default);
}

namespace {

struct RefHandle {
    std::unique_ptr<mlvc::InferenceBackend> backend;
    std::vector<mlvc::Tensor> outputs;
};

void set_error(char* err, std::size_t len, const char* what)
{
    if (err && len) {
        std::strncpy(err, what, len - 1);
        err[len - 1] = '\0';
    }
}

}  // namespace

extern "C" {

void* mlvc_ref_create(const char* model_dir, int num_threads, char* err, std::size_t err_len)
{
    try {
        static const bool registered = [] {
            mlvc::cpu_backend::register_cpu_backend(true);
            return true;
        }();
        (void)registered;
        mlvc::BackendOptions options;
        options.model_dir = model_dir;
        options.num_threads = num_threads;
        options.backend_name = "cpu";
        auto handle = std::make_unique<RefHandle>();
        handle->backend = mlvc::create_backend(options);
        return handle.release();
    } catch (const std::exception& e) {
        set_error(err, err_len, e.what());
        return nullptr;
    }
}

int mlvc_ref_load(void* h, const char* model_name, int n_state, const std::uint64_t* state_inputs,
                  const std::uint64_t* state_outputs, const std::int64_t* state_shapes4,
                  char* err, std::size_t err_len)
{
    try {
        auto* handle = static_cast<RefHandle*>(h);
        mlvc::ModelExecutionConfig config;
        for (int i = 0; i < n_state; ++i) {
            mlvc::StateTensorBinding b;
            b.input_index = state_inputs[i];
            b.output_index = state_outputs[i];
            b.data_type = mlvc::TensorDataType::kFloat16;
            b.shape.assign(state_shapes4 + 4 * i, state_shapes4 + 4 * i + 4);
            config.state_bindings.push_back(b);
        }
        handle->backend->load(model_name, config);
        return 0;
    } catch (const std::exception& e) {
        set_error(err, err_len, e.what());
        return -1;
    }
}

int mlvc_ref_reset_state(void* h, char* err, std::size_t err_len)
{
    try {
        static_cast<RefHandle*>(h)->backend->reset_state();
        return 0;
    } catch (const std::exception& e) {
        set_error(err, err_len, e.what());
        return -1;
    }
}

// Inputs: n tensors; dtype 0 = fp16 (uint16 bits), 1 = int32; shapes are
// rank-prefixed in `shapes` (ranks[i] entries each).
int mlvc_ref_run(void* h, int n, const void* const* data, const int* dtypes, const int* ranks,
                 const std::int64_t* shapes, char* err, std::size_t err_len)
{
    try {
        auto* handle = static_cast<RefHandle*>(h);
        std::vector<mlvc::Tensor> inputs(n);
        std::size_t cursor = 0;
        for (int i = 0; i < n; ++i) {
            auto& t = inputs[i];
            t.shape.assign(shapes + cursor, shapes + cursor + ranks[i]);
            cursor += ranks[i];
            std::size_t count = 1;
            for (auto d : t.shape)
                count *= static_cast<std::size_t>(d);
            if (dtypes[i] == 0) {
                std::vector<mlvc::Float16Storage> v(count);
                std::memcpy(v.data(), data[i], count * 2);
                t.data = std::move(v);
            } else {
                std::vector<std::int32_t> v(count);
                std::memcpy(v.data(), data[i], count * 4);
                t.data = std::move(v);
            }
        }
        handle->outputs = handle->backend->run(inputs);
        return 0;
    } catch (const std::exception& e) {
        set_error(err, err_len, e.what());
        return -1;
    }
}

int mlvc_ref_output_count(void* h)
{
    return static_cast<int>(static_cast<RefHandle*>(h)->outputs.size());
}

// Writes dtype (0 fp16, 1 int32), rank and up to 4 dims; returns byte size.
std::int64_t mlvc_ref_output_info(void* h, int i, int* dtype, int* rank, std::int64_t* shape4)
{
    const auto& t = static_cast<RefHandle*>(h)->outputs.at(i);
    *dtype = t.data_type() == mlvc::TensorDataType::kFloat16 ? 0 : 1;
    *rank = static_cast<int>(t.shape.size());
    for (std::size_t d = 0; d < t.shape.size() && d < 4; ++d)
        shape4[d] = t.shape[d];
    return static_cast<std::int64_t>(t.byte_size());
}

int mlvc_ref_output_copy(void* h, int i, void* dst, std::size_t capacity)
{
    const auto& t = static_cast<RefHandle*>(h)->outputs.at(i);
    if (capacity < t.byte_size())
        return -1;
    std::memcpy(dst, t.raw_data(), t.byte_size());
    return 0;
}

void mlvc_ref_destroy(void* h)
{
    delete static_cast<RefHandle*>(h);
}

// The reference's codec I/O conversions (core/src/yuv.cpp, compiled
// unchanged): prepare_model_input (frame -> [1, 3, mh, mw] FP16 tensor,
// placement from frame_padding) and prepare_model_output_into (tensor ->
// frame).  Planes are Y (w x h) then U, V (w/2 x h/2).
int mlvc_ref_yuv_to_tensor(const std::uint8_t* yuv, int w, int h, int mw, int mh, float pixel_range,
                           std::uint16_t* out, int* rotated, char* err, std::size_t err_len)
{
    try {
        const std::size_t ys = static_cast<std::size_t>(w) * h;
        mlvc::Yuv420FrameView frame(w, h, {yuv, ys}, {yuv + ys, ys / 4}, {yuv + ys + ys / 4, ys / 4});
        mlvc::FramePadding padding;
        const mlvc::Tensor t = mlvc::prepare_model_input(frame, mw, mh, pixel_range, padding);
        std::memcpy(out, t.raw_data(), t.byte_size());
        *rotated = padding.rotated ? 1 : 0;
        return 0;
    } catch (const std::exception& e) {
        set_error(err, err_len, e.what());
        return -1;
    }
}

int mlvc_ref_tensor_to_yuv(const std::uint16_t* tensor, int mw, int mh, int w, int h, float pixel_range,
                           std::uint8_t* yuv, char* err, std::size_t err_len)
{
    try {
        const std::size_t ys = static_cast<std::size_t>(w) * h;
        mlvc::Tensor t{"x_hat", {1, 3, mh, mw},
                       std::vector<mlvc::Float16Storage>(tensor, tensor + static_cast<std::size_t>(3) * mw * mh)};
        const mlvc::FramePadding padding = mlvc::frame_padding(w, h, mw, mh);
        mlvc::MutableYuv420FrameView frame(w, h, {yuv, ys}, {yuv + ys, ys / 4}, {yuv + ys + ys / 4, ys / 4});
        mlvc::prepare_model_output_into(t, frame, pixel_range, padding);
        return 0;
    } catch (const std::exception& e) {
        set_error(err, err_len, e.what());
        return -1;
    }
}

}  // extern "C"
