// mlvc_b200_adapter.hpp - reference-side binding of the B200 backend.
//
// Header-only C++ adapter that a maintainer of the reference codec compiles
// inside its tree (include paths: the reference's core/include and
// runtime/include, plus this directory; link: libmlvc_b200.so).  It
// implements both reference backend interfaces over the C ABI of
// mlvc_b200.h:
//   * mlvc::InferenceBackend (runtime/include/mlvc/runtime/backend.hpp:48-63):
//     name, load (assets through the ModelAssetReader the codec resolved),
//     run, reset_state;
//   * mlvc::BufferedCodecBackend (backend.hpp:69-96): configure_codec_io,
//     codec_slot_count, encoder_input_yuv / submit_encoder / encoder_outputs,
//     decoder_inputs / submit_decoder / decoder_output_yuv, wait_codec_slot.
// Because the class derives from BufferedCodecBackend, the codec's check
// dynamic_cast<BufferedCodecBackend*> (codec/src/pipeline.cpp:825-826 for
// encoding, the same test before decode_buffered) succeeds and the codec
// takes its buffered slot path.  register_b200_backend() registers the class
// as "b200" the way the driver-cubin backend registers itself
// (backends/driver_cubin/src/backend.cpp:129-137, called from
// backends/selected_backends.cpp:18-30).
//
// As in the reference's fixed-shape backend (cuda_graph_executor.cpp:243-373):
// the encoder is the graph with an FP16 [1, 3, H, W] input named "x", the
// decoder the graph with an output named "x_hat"; the int32 [1] input
// "q_index_shifted" is set by submit_encoder / submit_decoder and is not one
// of decoder_inputs(); state-bound tensors are never host-visible.  Views
// returned by the slot accessors point into the backend's pinned slot
// buffers and are valid until the slot is submitted again; read them after
// wait_codec_slot().
#pragma once

#include "mlvc/runtime/backend.hpp"
#include "mlvc_b200.h"

#include <cstddef>
#include <cstdint>
#include <filesystem>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace mlvc::b200_backend {

inline void check(int rc)
{
    if (rc != 0)
        throw std::runtime_error(mlvc_b200_last_error());
}

class B200Backend final : public InferenceBackend, public BufferedCodecBackend {
public:
    explicit B200Backend(BackendOptions options) : options_(std::move(options))
    {
        check(mlvc_b200_create(options_.device_id, &handle_));
    }
    ~B200Backend() override { mlvc_b200_destroy(handle_); }
    B200Backend(const B200Backend&) = delete;
    B200Backend& operator=(const B200Backend&) = delete;

    // ---------------------------------------------------- InferenceBackend
    std::string_view name() const noexcept override { return "b200"; }

    void load(const std::string& model_name, const ModelExecutionConfig& config) override
    {
        const auto reader = resolve_model_asset_reader(options_.model_dir, options_.asset_reader);
        const std::filesystem::path part = std::filesystem::path("aot") / model_name;
        const std::vector<std::byte> graph = reader->read_binary(part / "graph.pb");
        const std::vector<std::byte> weights = reader->read_binary(part / "weights.bin");
        std::vector<mlvc_b200_state_binding> bindings;
        for (const StateTensorBinding& b : config.state_bindings)
            bindings.push_back({b.input_index, b.output_index});
        check(mlvc_b200_load_memory(handle_, graph.data(), graph.size(), weights.data(), weights.size(),
                                    bindings.data(), bindings.size()));
        inputs_ = describe(true);
        outputs_ = describe(false);
        codec_input_ = codec_output_ = MLVC_B200_NO_CODEC_TENSOR;
    }

    std::vector<Tensor> run(const std::vector<Tensor>& inputs) override
    {
        std::vector<mlvc_b200_tensor> in(inputs.size());
        for (std::size_t i = 0; i < inputs.size(); ++i) {
            const Tensor& t = inputs[i];
            if (t.shape.size() > 4)
                throw std::runtime_error("b200: tensor rank above 4");
            in[i].dtype = t.data_type() == TensorDataType::kFloat16 ? 0 : 1;
            in[i].rank = static_cast<int32_t>(t.shape.size());
            for (std::size_t d = 0; d < t.shape.size(); ++d)
                in[i].shape[d] = t.shape[d];
            in[i].data = const_cast<void*>(t.raw_data());
            in[i].bytes = t.byte_size();
        }
        std::vector<Tensor> result(outputs_.size());
        std::vector<mlvc_b200_tensor> out(outputs_.size());
        for (std::size_t i = 0; i < outputs_.size(); ++i) {
            const Info& o = outputs_[i];
            result[i].name = o.name;
            result[i].shape = o.shape;
            if (o.type == TensorDataType::kFloat16)
                result[i].data = std::vector<Float16Storage>(o.bytes / sizeof(Float16Storage));
            else
                result[i].data = std::vector<std::int32_t>(o.bytes / sizeof(std::int32_t));
            out[i].data = const_cast<void*>(result[i].raw_data());
            out[i].bytes = o.bytes;
        }
        check(mlvc_b200_run(handle_, in.data(), in.size(), out.data(), out.size()));
        return result;
    }

    void reset_state() override { check(mlvc_b200_reset_state(handle_)); }

    // ------------------------------------------------ BufferedCodecBackend
    void configure_codec_io(const CodecIoConfig& config) override
    {
        // The backend places the frame as frame_padding does (core/src/yuv.cpp:
        // 324-337); a codec that asks for another placement is rejected.
        const FramePadding want = frame_padding(config.width, config.height, config.model_width, config.model_height);
        const FramePadding& got = config.padding;
        if (got.left != want.left || got.top != want.top || got.right != want.right || got.bottom != want.bottom ||
            got.rotated != want.rotated)
            throw std::runtime_error("b200: codec frame padding differs from frame_padding()");
        std::size_t in = MLVC_B200_NO_CODEC_TENSOR, out = MLVC_B200_NO_CODEC_TENSOR;
        for (std::size_t i = 0; i < inputs_.size(); ++i)
            if (inputs_[i].name == "x")
                in = i;
        for (std::size_t i = 0; i < outputs_.size(); ++i)
            if (outputs_[i].name == "x_hat")
                out = i;
        if (in == MLVC_B200_NO_CODEC_TENSOR && out == MLVC_B200_NO_CODEC_TENSOR)
            throw std::runtime_error("b200: codec I/O needs an encoder input \"x\" or a decoder output \"x_hat\"");
        check(mlvc_b200_configure_codec_io(handle_, config.width, config.height, config.model_width,
                                           config.model_height, config.pixel_range, config.slots, in, out));
        codec_input_ = in;
        codec_output_ = out;
        width_ = config.width;
        height_ = config.height;
    }

    std::size_t codec_slot_count() const noexcept override { return mlvc_b200_slot_count(handle_); }

    MutableYuv420FrameView encoder_input_yuv(std::size_t slot) override
    {
        require(codec_input_ != MLVC_B200_NO_CODEC_TENSOR, "encoder");
        std::uint8_t *y = nullptr, *u = nullptr, *v = nullptr;
        check(mlvc_b200_slot_input_yuv(handle_, slot, &y, &u, &v));
        const std::size_t ys = static_cast<std::size_t>(width_) * height_;
        return MutableYuv420FrameView(width_, height_, {y, ys}, {u, ys / 4}, {v, ys / 4});
    }

    void submit_encoder(std::size_t slot, int shifted_q) override
    {
        require(codec_input_ != MLVC_B200_NO_CODEC_TENSOR, "encoder");
        check(mlvc_b200_submit_q(handle_, slot, shifted_q));
    }

    std::vector<TensorView> encoder_outputs(std::size_t slot) const override
    {
        require(codec_input_ != MLVC_B200_NO_CODEC_TENSOR, "encoder");
        std::vector<TensorView> views;
        for (std::size_t i = 0; i < outputs_.size(); ++i) {
            const void* data = mlvc_b200_slot_output(handle_, slot, i);
            if (!data)
                check(-1);
            const Info& o = outputs_[i];
            views.push_back(TensorView::from_raw(o.name, o.shape, o.type, data, o.bytes));
        }
        return views;
    }

    std::vector<MutableTensorView> decoder_inputs(std::size_t slot) override
    {
        require(codec_output_ != MLVC_B200_NO_CODEC_TENSOR, "decoder");
        std::vector<MutableTensorView> views;
        for (std::size_t i = 0; i < inputs_.size(); ++i) {
            const Info& d = inputs_[i];
            if (d.name == "q_index_shifted")
                continue;
            void* data = mlvc_b200_slot_input(handle_, slot, i);
            if (!data)
                check(-1);
            views.push_back(MutableTensorView::from_raw(d.name, d.shape, d.type, data, d.bytes));
        }
        return views;
    }

    void submit_decoder(std::size_t slot, int shifted_q) override
    {
        require(codec_output_ != MLVC_B200_NO_CODEC_TENSOR, "decoder");
        check(mlvc_b200_submit_q(handle_, slot, shifted_q));
    }

    Yuv420FrameView decoder_output_yuv(std::size_t slot) const override
    {
        require(codec_output_ != MLVC_B200_NO_CODEC_TENSOR, "decoder");
        const std::uint8_t *y = nullptr, *u = nullptr, *v = nullptr;
        check(mlvc_b200_slot_output_yuv(handle_, slot, &y, &u, &v));
        const std::size_t ys = static_cast<std::size_t>(width_) * height_;
        return Yuv420FrameView(width_, height_, {y, ys}, {u, ys / 4}, {v, ys / 4});
    }

    void wait_codec_slot(std::size_t slot) override { check(mlvc_b200_wait_slot(handle_, slot)); }

private:
    struct Info {
        std::string name;
        TensorDataType type = TensorDataType::kFloat16;
        std::vector<std::int64_t> shape;
        std::size_t bytes = 0;
    };

    std::vector<Info> describe(bool inputs) const
    {
        std::vector<Info> out(inputs ? mlvc_b200_input_count(handle_) : mlvc_b200_output_count(handle_));
        for (std::size_t i = 0; i < out.size(); ++i) {
            mlvc_b200_tensor t{};
            const char* name = nullptr;
            check(inputs ? mlvc_b200_input_info(handle_, i, &t, &name) : mlvc_b200_output_info(handle_, i, &t, &name));
            out[i].name = name;
            out[i].type = t.dtype == 0 ? TensorDataType::kFloat16 : TensorDataType::kInt32;
            out[i].shape.assign(t.shape, t.shape + t.rank);
            out[i].bytes = t.bytes;
        }
        return out;
    }

    static void require(bool ok, const char* side)
    {
        if (!ok)
            throw std::runtime_error(std::string("b200: ") + side + " codec I/O is unavailable");
    }

    BackendOptions options_;
    mlvc_b200_backend* handle_ = nullptr;
    std::vector<Info> inputs_, outputs_;
    std::size_t codec_input_ = MLVC_B200_NO_CODEC_TENSOR, codec_output_ = MLVC_B200_NO_CODEC_TENSOR;
    int width_ = 0, height_ = 0;
};

// Registers the backend as "b200" (register_backend, runtime/src/backend_registry.cpp).
inline void register_b200_backend(bool make_default)
{
    register_backend(
        "b200", [](const BackendOptions& options) { return std::make_unique<B200Backend>(options); }, make_default);
}

}  // namespace mlvc::b200_backend
