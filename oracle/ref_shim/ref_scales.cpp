// Test infrastructure only (the checker, never the product): extern "C"
// access to the reference's own scale extraction (core/src/scales.cpp:25-105,
// compiled unchanged from the reference tree) for the GPU scale-extraction
// parity tests.
//
// scales.cpp reads the latent and hyper-latent plane sizes from
// mlvc::ModelConfig, whose methods live in core/src/model.cpp next to the
// protobuf metadata loader (which needs the absent protobuf runtime).  The
// few plane-size methods are defined here with the reference's rule
// (core/src/model.cpp:94-126): ceil(model size / downsample factor), the
// hyper-latent plane using downsample_latent * downsample_hyperprior.
#include "mlvc/core/model.hpp"
#include "mlvc/core/scales.hpp"
#include "mlvc/core/tensor.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <span>
#include <vector>

namespace mlvc {
namespace {
int ceil_div(std::int64_t a, std::int64_t b) { return static_cast<int>((a + b - 1) / b); }
}  // namespace

int ModelConfig::feature_height() const { return ceil_div(model_height, downsample_feature); }
int ModelConfig::feature_width() const { return ceil_div(model_width, downsample_feature); }
int ModelConfig::latent_height() const { return ceil_div(model_height, downsample_latent); }
int ModelConfig::latent_width() const { return ceil_div(model_width, downsample_latent); }
int ModelConfig::hyperprior_height() const
{
    return ceil_div(model_height, static_cast<std::int64_t>(downsample_latent) * downsample_hyperprior);
}
int ModelConfig::hyperprior_width() const
{
    return ceil_div(model_width, static_cast<std::int64_t>(downsample_latent) * downsample_hyperprior);
}

}  // namespace mlvc

extern "C" int mlvc_ref_extract_scales(const std::uint16_t* z_raw, int hyperprior_channels, int model_width,
                                       int model_height, int latent_channels, int downsample_latent,
                                       int downsample_hyperprior, int y_scale_repeat, int scale_max_index,
                                       std::int32_t* scales_0, std::int32_t* scales_1, char* err, std::size_t err_len)
{
    try {
        mlvc::ModelConfig c;
        c.model_width = model_width;
        c.model_height = model_height;
        c.hyperprior_channels = hyperprior_channels;
        c.latent_channels = latent_channels;
        c.downsample_latent = downsample_latent;
        c.downsample_hyperprior = downsample_hyperprior;
        c.y_scale_repeat = y_scale_repeat;
        const std::int64_t shape[4] = {1, hyperprior_channels, c.hyperprior_height(), c.hyperprior_width()};
        const std::size_t n = static_cast<std::size_t>(hyperprior_channels) * shape[2] * shape[3];
        const mlvc::TensorView z("z_raw", std::span<const std::int64_t>(shape, 4),
                                 std::span<const std::uint16_t>(z_raw, n));
        std::vector<std::int32_t> s0, s1;
        mlvc::extract_scales(z, c, scale_max_index, s0, s1);
        std::memcpy(scales_0, s0.data(), s0.size() * sizeof(std::int32_t));
        std::memcpy(scales_1, s1.data(), s1.size() * sizeof(std::int32_t));
        return 0;
    } catch (const std::exception& e) {
        if (err && err_len) {
            std::strncpy(err, e.what(), err_len - 1);
            err[err_len - 1] = 0;
        }
        return -1;
    }
}
