// extern "C" layer over mlvc_b200::Backend (declarations and the reference
// interface each entry replaces: include/mlvc_b200.h).  Exceptions never
// cross the boundary: they become -1 plus a thread-local message.
#include "../../../include/mlvc_b200.h"

#include "backend.hpp"

#include <exception>
#include <memory>
#include <string>
#include <vector>

struct mlvc_b200_backend {
    std::unique_ptr<mlvc_b200::Backend> impl;
};

namespace mlvc_b200 {
// csrc/noalloc/integer_values_noalloc.cu
void integer_values_noalloc(const uint16_t* values, size_t count, int32_t* symbols);
}  // namespace mlvc_b200

namespace {

thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f)
{
    try {
        f();
        g_last_error.clear();
        return 0;
    } catch (const std::exception& e) {
        g_last_error = e.what();
    } catch (...) {
        g_last_error = "mlvc-b200: unknown error";
    }
    return -1;
}

std::vector<mlvc_b200::StateBinding> to_bindings(const mlvc_b200_state_binding* b, size_t n)
{
    std::vector<mlvc_b200::StateBinding> out;
    for (size_t i = 0; i < n; ++i)
        out.push_back({b[i].input_index, b[i].output_index});
    return out;
}

void describe(const mlvc_b200::TensorDesc& d, mlvc_b200_tensor* info)
{
    info->dtype = d.dtype == mlvc_b200::DType::kInt32 ? 1 : 0;
    info->rank = static_cast<int32_t>(d.shape.size());
    for (int i = 0; i < 4; ++i)
        info->shape[i] = i < info->rank ? d.shape[i] : 1;
    info->data = nullptr;
    info->bytes = static_cast<size_t>(mlvc_b200::element_count(d.shape)) * mlvc_b200::dtype_size(d.dtype);
}

mlvc_b200::Backend& require(const mlvc_b200_backend* b)
{
    if (!b || !b->impl)
        throw std::runtime_error("mlvc-b200: null backend handle");
    return *b->impl;
}

}  // namespace

extern "C" {

int mlvc_b200_abi_version(void) { return MLVC_B200_ABI_VERSION; }

const char* mlvc_b200_last_error(void) { return g_last_error.c_str(); }

int mlvc_b200_create(int device_id, mlvc_b200_backend** out)
{
    return guarded([&] {
        if (!out)
            throw std::runtime_error("mlvc-b200: null output handle");
        auto h = std::make_unique<mlvc_b200_backend>();
        h->impl = std::make_unique<mlvc_b200::Backend>(device_id);
        *out = h.release();
    });
}

int mlvc_b200_create_offline(int sm_count, int smem_optin_bytes, mlvc_b200_backend** out)
{
    return guarded([&] {
        if (!out || sm_count <= 0 || smem_optin_bytes <= 0)
            throw std::runtime_error("mlvc-b200: invalid planning target");
        auto h = std::make_unique<mlvc_b200_backend>();
        h->impl = std::make_unique<mlvc_b200::Backend>(sm_count, smem_optin_bytes, true);
        *out = h.release();
    });
}

void mlvc_b200_destroy(mlvc_b200_backend* backend) { delete backend; }

const char* mlvc_b200_name(const mlvc_b200_backend*) { return "b200"; }

int mlvc_b200_load(mlvc_b200_backend* backend, const char* model_dir, const char* model_name,
                   const mlvc_b200_state_binding* bindings, size_t binding_count)
{
    return guarded([&] {
        if (!model_dir || !model_name)
            throw std::runtime_error("mlvc-b200: null model path");
        require(backend).load(model_dir, model_name, to_bindings(bindings, binding_count));
    });
}

int mlvc_b200_load_memory(mlvc_b200_backend* backend, const void* graph_pb, size_t graph_bytes, const void* weights,
                          size_t weights_bytes, const mlvc_b200_state_binding* bindings, size_t binding_count)
{
    return guarded([&] {
        require(backend).load_bytes(static_cast<const uint8_t*>(graph_pb), graph_bytes,
                                    static_cast<const uint8_t*>(weights), weights_bytes,
                                    to_bindings(bindings, binding_count));
    });
}

size_t mlvc_b200_input_count(const mlvc_b200_backend* backend)
{
    return backend && backend->impl ? backend->impl->input_count() : 0;
}

size_t mlvc_b200_output_count(const mlvc_b200_backend* backend)
{
    return backend && backend->impl ? backend->impl->output_count() : 0;
}

int mlvc_b200_input_info(const mlvc_b200_backend* backend, size_t index, mlvc_b200_tensor* info, const char** name)
{
    return guarded([&] {
        const auto& d = require(backend).input_desc(index);
        if (info)
            describe(d, info);
        if (name)
            *name = d.name.c_str();
    });
}

int mlvc_b200_output_info(const mlvc_b200_backend* backend, size_t index, mlvc_b200_tensor* info, const char** name)
{
    return guarded([&] {
        const auto& d = require(backend).output_desc(index);
        if (info)
            describe(d, info);
        if (name)
            *name = d.name.c_str();
    });
}

int mlvc_b200_run(mlvc_b200_backend* backend, const mlvc_b200_tensor* inputs, size_t input_count,
                  mlvc_b200_tensor* outputs, size_t output_count)
{
    return guarded([&] {
        std::vector<mlvc_b200::HostTensorRef> in(input_count), out(output_count);
        for (size_t i = 0; i < input_count; ++i) {
            const auto& t = inputs[i];
            in[i] = {t.dtype, t.rank, {t.shape[0], t.shape[1], t.shape[2], t.shape[3]}, t.data, t.bytes};
        }
        for (size_t i = 0; i < output_count; ++i) {
            const auto& t = outputs[i];
            out[i] = {t.dtype, t.rank, {t.shape[0], t.shape[1], t.shape[2], t.shape[3]}, t.data, t.bytes};
        }
        require(backend).run(in.data(), in.size(), out.data(), out.size());
        for (size_t i = 0; i < output_count; ++i) {
            auto& t = outputs[i];
            t.dtype = out[i].dtype;
            t.rank = out[i].rank;
            for (int r = 0; r < 4; ++r)
                t.shape[r] = r < t.rank ? out[i].shape[r] : 1;
            t.bytes = out[i].bytes;
        }
    });
}

int mlvc_b200_reset_state(mlvc_b200_backend* backend)
{
    return guarded([&] { require(backend).reset_state(); });
}

namespace {
mlvc_b200::ScaleConfig scale_config(const mlvc_b200_scale_config* c)
{
    if (!c)
        throw std::runtime_error("mlvc-b200: null scale configuration");
    return {c->hyperprior_channels, c->model_width,     c->model_height,          c->latent_channels,
            c->downsample_latent,   c->downsample_hyperprior, c->y_scale_repeat, c->scale_max_index};
}
}  // namespace

int mlvc_b200_scale_shape(const mlvc_b200_scale_config* config, size_t* z_count, size_t* scale_count)
{
    return guarded([&] {
        const mlvc_b200::ScaleConfig c = scale_config(config);
        int zh = 0, zw = 0, yh = 0, yw = 0;
        mlvc_b200::Backend::scale_plane(c, &zh, &zw, &yh, &yw);
        if (z_count)
            *z_count = static_cast<size_t>(c.hyperprior_channels) * zh * zw;
        if (scale_count)
            *scale_count = static_cast<size_t>(c.latent_channels / 2) * yh * yw;
    });
}

int mlvc_b200_extract_scales(mlvc_b200_backend* backend, const uint16_t* z_raw, size_t z_count,
                             const mlvc_b200_scale_config* config, int32_t* scales_0, int32_t* scales_1,
                             size_t scale_count)
{
    return guarded([&] {
        const mlvc_b200::ScaleConfig c = scale_config(config);
        int zh = 0, zw = 0, yh = 0, yw = 0;
        mlvc_b200::Backend::scale_plane(c, &zh, &zw, &yh, &yw);
        if (z_count != static_cast<size_t>(c.hyperprior_channels) * zh * zw)
            throw std::runtime_error("z_raw shape or dtype does not match model metadata");
        if (scale_count < static_cast<size_t>(c.latent_channels / 2) * yh * yw)
            throw std::runtime_error("mlvc-b200: scale buffers are too small");
        if (!z_raw || !scales_0 || !scales_1)
            throw std::runtime_error("mlvc-b200: null scale buffer");
        require(backend).extract_scales(z_raw, c, scales_0, scales_1);
    });
}

int mlvc_b200_extract_scales_device(mlvc_b200_backend* backend, uint64_t z_raw, const mlvc_b200_scale_config* config,
                                    uint64_t scales_0, uint64_t scales_1)
{
    return guarded([&] {
        const mlvc_b200::ScaleConfig c = scale_config(config);
        if (!z_raw || !scales_0 || !scales_1 || (z_raw & 1) || (scales_0 & 3) || (scales_1 & 3))
            throw std::runtime_error("mlvc-b200: null or misaligned device pointer");
        require(backend).extract_scales_device(z_raw, c, scales_0, scales_1);
    });
}

int mlvc_b200_integer_values_device(mlvc_b200_backend* backend, uint64_t values, size_t count, uint64_t symbols,
                                    uint64_t out_of_range)
{
    return guarded([&] {
        if (count && (!values || !symbols || !out_of_range || (values & 1) || (symbols & 3) || (out_of_range & 3)))
            throw std::runtime_error("mlvc-b200: null or misaligned device pointer");
        require(backend).integer_values_device(values, count, symbols, out_of_range);
    });
}

int mlvc_b200_integer_values(mlvc_b200_backend* backend, const uint16_t* values, size_t count, int32_t* symbols)
{
    return guarded([&] {
        if (count && (!values || !symbols))
            throw std::runtime_error("mlvc-b200: null value buffer");
        require(backend).integer_values(values, count, symbols);
    });
}

int mlvc_b200_integer_values_noalloc(const uint16_t* values, size_t count, int32_t* symbols)
{
    return guarded([&] { mlvc_b200::integer_values_noalloc(values, count, symbols); });
}

int mlvc_b200_configure_slots(mlvc_b200_backend* backend, size_t slot_count)
{
    return guarded([&] { require(backend).configure_slots(slot_count); });
}

size_t mlvc_b200_slot_count(const mlvc_b200_backend* backend)
{
    return backend && backend->impl ? backend->impl->slot_count() : 0;
}

void* mlvc_b200_slot_input(mlvc_b200_backend* backend, size_t slot, size_t input_index)
{
    void* p = nullptr;
    guarded([&] { p = require(backend).slot_input(slot, input_index); });
    return p;
}

const void* mlvc_b200_slot_output(const mlvc_b200_backend* backend, size_t slot, size_t output_index)
{
    const void* p = nullptr;
    guarded([&] { p = require(backend).slot_output(slot, output_index); });
    return p;
}

int mlvc_b200_configure_codec_io(mlvc_b200_backend* backend, int width, int height, int model_width,
                                 int model_height, float pixel_range, size_t slots, size_t input_index,
                                 size_t output_index)
{
    return guarded([&] {
        require(backend).configure_codec_io(width, height, model_width, model_height, pixel_range, slots, input_index,
                                            output_index);
    });
}

int mlvc_b200_codec_output_fused(const mlvc_b200_backend* backend, int* fused)
{
    return guarded([&] {
        if (!fused)
            throw std::invalid_argument("mlvc-b200: null output pointer");
        *fused = require(backend).codec_output_fused() ? 1 : 0;
    });
}

int mlvc_b200_slot_input_yuv(mlvc_b200_backend* backend, size_t slot, uint8_t** y, uint8_t** u, uint8_t** v)
{
    return guarded([&] {
        if (!y || !u || !v)
            throw std::runtime_error("mlvc-b200: null plane pointer");
        require(backend).slot_input_yuv(slot, y, u, v);
    });
}

int mlvc_b200_slot_output_yuv(const mlvc_b200_backend* backend, size_t slot, const uint8_t** y, const uint8_t** u,
                              const uint8_t** v)
{
    return guarded([&] {
        if (!y || !u || !v)
            throw std::runtime_error("mlvc-b200: null plane pointer");
        require(backend).slot_output_yuv(slot, y, u, v);
    });
}

int mlvc_b200_submit(mlvc_b200_backend* backend, size_t slot)
{
    return guarded([&] { require(backend).submit(slot); });
}

int mlvc_b200_test_wait_expiry(mlvc_b200_backend* backend, size_t step_index, uint64_t limit_ns,
                               uint32_t* status)
{
    return guarded([&] {
        if (!status)
            throw std::runtime_error("mlvc-b200: status pointer is null");
        *status = require(backend).test_wait_expiry(step_index, limit_ns);
    });
}

int mlvc_b200_submit_q(mlvc_b200_backend* backend, size_t slot, int32_t shifted_q)
{
    return guarded([&] { require(backend).submit_q(slot, shifted_q); });
}

int mlvc_b200_wait_slot(mlvc_b200_backend* backend, size_t slot)
{
    return guarded([&] { require(backend).wait_slot(slot); });
}

int mlvc_b200_enqueue(mlvc_b200_backend* backend)
{
    return guarded([&] { require(backend).enqueue(); });
}

int mlvc_b200_synchronize(mlvc_b200_backend* backend)
{
    return guarded([&] { require(backend).synchronize(); });
}

void* mlvc_b200_stream(const mlvc_b200_backend* backend)
{
    return backend && backend->impl ? static_cast<void*>(backend->impl->stream()) : nullptr;
}

size_t mlvc_b200_step_count(const mlvc_b200_backend* backend)
{
    return backend && backend->impl ? backend->impl->steps().size() : 0;
}

int mlvc_b200_step_info(const mlvc_b200_backend* backend, size_t index, const char** kernel, const char** nodes,
                        double* flops, double* bytes, uint32_t* grid, uint32_t* block, uint32_t* smem)
{
    return guarded([&] {
        const auto& s = require(backend).steps().at(index);
        if (kernel)
            *kernel = s.kernel.c_str();
        if (nodes)
            *nodes = s.nodes.c_str();
        if (flops)
            *flops = s.flops;
        if (bytes)
            *bytes = s.bytes;
        if (grid)
            *grid = s.grid;
        if (block)
            *block = s.block;
        if (smem)
            *smem = s.smem;
    });
}

int mlvc_b200_time_steps(mlvc_b200_backend* backend, int iterations, size_t flush_bytes, float* ms_per_step)
{
    return guarded([&] {
        const auto t = require(backend).time_steps(iterations, flush_bytes);
        for (size_t i = 0; i < t.size(); ++i)
            ms_per_step[i] = t[i];
    });
}

int mlvc_b200_trace_spans(mlvc_b200_backend* backend, int iterations, size_t flush_bytes, float* ms_per_step)
{
    return guarded([&] {
        const auto t = require(backend).trace_spans(iterations, flush_bytes);
        for (size_t i = 0; i < t.size(); ++i)
            ms_per_step[i] = t[i];
    });
}

int mlvc_b200_kernel_launches(const mlvc_b200_backend* backend)
{
    return backend && backend->impl ? backend->impl->kernel_launches_per_run() : -1;
}

int mlvc_b200_trace_step(mlvc_b200_backend* backend, size_t index, uint64_t* stamps, size_t capacity,
                         size_t* count)
{
    return guarded([&] {
        const auto t = require(backend).trace_step(index);
        if (count)
            *count = t.size();
        if (stamps)
            for (size_t i = 0; i < t.size() && i < capacity; ++i)
                stamps[i] = t[i];
    });
}

int mlvc_b200_set_debug_tensors(mlvc_b200_backend* backend, int enable)
{
    return guarded([&] { require(backend).set_keep_all_values(enable != 0); });
}

int mlvc_b200_read_tensor(mlvc_b200_backend* backend, const char* name, void* dst, size_t bytes, int* found)
{
    return guarded([&] {
        if (!name || !dst)
            throw std::runtime_error("mlvc-b200: null argument");
        const bool ok = require(backend).read_value(name, dst, bytes);
        if (found)
            *found = ok ? 1 : 0;
    });
}

size_t mlvc_b200_device_bytes(const mlvc_b200_backend* backend)
{
    return backend && backend->impl ? backend->impl->device_bytes() : 0;
}

}  // extern "C"
