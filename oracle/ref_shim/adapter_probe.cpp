// Test infrastructure only (oracle side). Never linked into the product.
//
// Drives include/mlvc_b200_adapter.hpp the way the reference codec drives a
// backend: the adapter is registered in the reference's own backend registry
// (runtime/src/backend_registry.cpp, compiled unchanged into
// libmlvc_ref_cpu.so), created through mlvc::create_backend by name, loaded
// through the ModelAssetReader the registry resolves, recognised as a
// BufferedCodecBackend by the same dynamic_cast the codec makes
// (codec/src/pipeline.cpp:825-826), and run through the decoder slot calls
// of decode_buffered (configure_codec_io with make_codec_io_config's
// placement, decoder_inputs, submit_decoder(slot, shifted_q),
// wait_codec_slot, decoder_output_yuv).  The extern "C" surface is for the
// Python tests (ctypes); errors are a non-zero return plus a message.
#include "mlvc_b200_adapter.hpp"

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>

namespace {

struct Probe {
    std::unique_ptr<mlvc::InferenceBackend> backend;
    mlvc::BufferedCodecBackend* buffered = nullptr;
};

void set_error(char* err, std::size_t len, const char* what)
{
    if (err && len) {
        std::strncpy(err, what, len - 1);
        err[len - 1] = '\0';
    }
}

template <typename F>
int guarded(char* err, std::size_t len, F&& f)
{
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        set_error(err, len, e.what());
        return -1;
    }
}

}  // namespace

extern "C" {

// create_backend({model_dir, device_id, backend_name = "b200"}); *buffered
// tells whether the codec's dynamic_cast to BufferedCodecBackend succeeds.
void* probe_create(const char* model_dir, int device_id, int* buffered, char* err, std::size_t len)
{
    auto probe = std::make_unique<Probe>();
    const int rc = guarded(err, len, [&] {
        static const bool registered = [] {
            mlvc::b200_backend::register_b200_backend(false);
            return true;
        }();
        (void)registered;
        mlvc::BackendOptions options;
        options.model_dir = model_dir;
        options.device_id = device_id;
        options.backend_name = "b200";
        probe->backend = mlvc::create_backend(options);
        probe->buffered = dynamic_cast<mlvc::BufferedCodecBackend*>(probe->backend.get());
        *buffered = probe->buffered != nullptr;
    });
    return rc == 0 ? probe.release() : nullptr;
}

void probe_destroy(void* h) { delete static_cast<Probe*>(h); }

int probe_name(void* h, char* out, std::size_t len)
{
    const auto name = static_cast<Probe*>(h)->backend->name();
    set_error(out, len, std::string(name).c_str());
    return 0;
}

// load(model, {state binding input_index <- output_index, FP16 [1, c, h, w]})
int probe_load(void* h, const char* model, int n_state, const std::uint64_t* state_in, const std::uint64_t* state_out,
               char* err, std::size_t len)
{
    return guarded(err, len, [&] {
        mlvc::ModelExecutionConfig config;
        for (int i = 0; i < n_state; ++i) {
            mlvc::StateTensorBinding b;
            b.input_index = state_in[i];
            b.output_index = state_out[i];
            config.state_bindings.push_back(b);
        }
        static_cast<Probe*>(h)->backend->load(model, config);
    });
}

int probe_reset_state(void* h, char* err, std::size_t len)
{
    return guarded(err, len, [&] { static_cast<Probe*>(h)->backend->reset_state(); });
}

// configure_codec_io with the codec's placement (frame_padding).
int probe_configure(void* h, int width, int height, int model_width, int model_height, int slots, char* err,
                    std::size_t len)
{
    return guarded(err, len, [&] {
        mlvc::CodecIoConfig config;
        config.width = width;
        config.height = height;
        config.model_width = model_width;
        config.model_height = model_height;
        config.pixel_range = 1.0F;
        config.padding = mlvc::frame_padding(width, height, model_width, model_height);
        config.slots = static_cast<std::size_t>(slots);
        static_cast<Probe*>(h)->buffered->configure_codec_io(config);
    });
}

// decoder_inputs(slot)[index]: its name, byte size and host pointer.
int probe_decoder_input(void* h, std::size_t slot, std::size_t index, char* name, std::size_t name_len, void** data,
                        std::size_t* bytes, char* err, std::size_t len)
{
    return guarded(err, len, [&] {
        auto inputs = static_cast<Probe*>(h)->buffered->decoder_inputs(slot);
        if (index >= inputs.size())
            throw std::runtime_error("decoder input index out of range");
        set_error(name, name_len, std::string(inputs[index].name()).c_str());
        *data = inputs[index].raw_data();
        *bytes = inputs[index].byte_size();
    });
}

int probe_decoder_input_count(void* h, std::size_t slot, std::size_t* count, char* err, std::size_t len)
{
    return guarded(err, len, [&] { *count = static_cast<Probe*>(h)->buffered->decoder_inputs(slot).size(); });
}

int probe_submit_decoder(void* h, std::size_t slot, int shifted_q, char* err, std::size_t len)
{
    return guarded(err, len, [&] { static_cast<Probe*>(h)->buffered->submit_decoder(slot, shifted_q); });
}

int probe_wait(void* h, std::size_t slot, char* err, std::size_t len)
{
    return guarded(err, len, [&] { static_cast<Probe*>(h)->buffered->wait_codec_slot(slot); });
}

// decoder_output_yuv(slot) copied into `yuv` (Y, then U, then V).
int probe_decoder_output(void* h, std::size_t slot, std::uint8_t* yuv, std::size_t capacity, char* err,
                         std::size_t len)
{
    return guarded(err, len, [&] {
        const mlvc::Yuv420FrameView f = static_cast<Probe*>(h)->buffered->decoder_output_yuv(slot);
        const std::size_t total = f.y().size() + f.u().size() + f.v().size();
        if (capacity < total)
            throw std::runtime_error("output buffer too small");
        std::memcpy(yuv, f.y().data(), f.y().size());
        std::memcpy(yuv + f.y().size(), f.u().data(), f.u().size());
        std::memcpy(yuv + f.y().size() + f.u().size(), f.v().data(), f.v().size());
    });
}

}  // extern "C"
