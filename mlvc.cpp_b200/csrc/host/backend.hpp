// The B200 inference backend: one loaded graph part on one device.
//
// Host-side mirror of the reference contracts it replaces:
//   * InferenceBackend::load / run / reset_state
//     (runtime/include/mlvc/runtime/backend.hpp:48-63)
//   * the fixed-shape buffered slot path of BufferedCodecBackend
//     (runtime/include/mlvc/runtime/backend.hpp:79-96), here with tensor slots
//     (pinned host inputs/outputs per slot, submit / wait)
//   * AotGraph's load -> plan -> capture -> replay life cycle
//     (backends/driver_cubin/src/model_loader.cpp:11-63,
//      cuda_graph_executor.cpp:31-412).
#pragma once

#include "driver.hpp"
#include "graph.hpp"

#include <cuda.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

namespace mlvc_b200 {

struct HostTensorRef {
    int dtype;  // 0 = FP16 (uint16 bits), 1 = INT32
    int rank;
    int64_t shape[4];
    void* data;
    size_t bytes;
};

struct StateBinding {
    size_t input_index;
    size_t output_index;
};

// Entropy-coder scale extraction parameters: the mlvc::ModelConfig fields
// extract_scales reads (core/src/scales.cpp:25-105) plus the scale table's
// last index (GaussianPmf::scale_levels - 1).
struct ScaleConfig {
    int hyperprior_channels;
    int model_width, model_height;
    int latent_channels;
    int downsample_latent, downsample_hyperprior;
    int y_scale_repeat;
    int scale_max_index;
};

struct StepInfo {
    std::string kernel;
    std::string nodes;   // graph node indices covered by the step
    uint32_t grid = 0, block = 0, smem = 0;
    double flops = 0.0;  // algorithmic work
    double bytes = 0.0;  // algorithmic HBM bytes (one read of each input, one write of each output)
};

class Backend {
public:
    explicit Backend(int device_id);
    // Planning-only instance: no device is touched; load_bytes() decodes,
    // validates and plans the graph (kernel choice, fusion, weight preparation)
    // for a machine with `sm_count` SMs and `smem_optin` bytes of shared memory
    // per block, so the host logic can be tested without a GPU.
    Backend(int sm_count, int smem_optin, bool /*offline*/);
    ~Backend();
    Backend(const Backend&) = delete;
    Backend& operator=(const Backend&) = delete;

    void load(const std::string& model_dir, const std::string& part, const std::vector<StateBinding>& bindings);
    void load_bytes(const uint8_t* graph, size_t graph_size, const uint8_t* weights, size_t weights_size,
                    const std::vector<StateBinding>& bindings);

    size_t input_count() const { return ext_inputs_.size(); }
    size_t output_count() const { return ext_outputs_.size(); }
    const TensorDesc& input_desc(size_t i) const;
    const TensorDesc& output_desc(size_t i) const;

    void run(const HostTensorRef* inputs, size_t n_in, HostTensorRef* outputs, size_t n_out);
    void reset_state();

    // Entropy-coder inputs computed on the GPU; they need no loaded graph.
    // extract_scales: z [1][hyper][zh][zw] FP16 bits -> scales_0 / scales_1
    // int32 [latent / 2][yh][yw] (zh = ceil(model_height / (downsample_latent
    // * downsample_hyperprior)), yh = ceil(model_height / downsample_latent)).
    // integer_values: FP16 bits -> int32 by truncation; throws the reference's
    // error when a value is not finite or outside [-32768, 32767].
    static void scale_plane(const ScaleConfig& cfg, int* z_height, int* z_width, int* y_height, int* y_width);
    void extract_scales(const uint16_t* z, const ScaleConfig& cfg, int32_t* scales_0, int32_t* scales_1);
    void integer_values(const uint16_t* values, size_t count, int32_t* symbols);
    // Device-memory forms: launch on stream() without copies or a sync.  The
    // caller zeroes *out_of_range (a device uint32) and reads it afterwards.
    void extract_scales_device(CUdeviceptr z, const ScaleConfig& cfg, CUdeviceptr scales_0, CUdeviceptr scales_1);
    void integer_values_device(CUdeviceptr values, size_t count, CUdeviceptr symbols, CUdeviceptr out_of_range);

    // Slot path: pinned host staging per slot, asynchronous submit, wait.
    void configure_slots(size_t count);
    size_t slot_count() const;
    bool codec_output_fused() const { return fused_yuv_step_ != static_cast<size_t>(-1); }
    void* slot_input(size_t slot, size_t i);
    const void* slot_output(size_t slot, size_t i) const;
    void submit(size_t slot);
    // submit_encoder / submit_decoder(slot, shifted_q): writes shifted_q into
    // the slot's buffer of the int32 [1] graph input "q_index_shifted", then
    // submits (set_q_index, backends/driver_cubin/src/cuda_graph_executor.cpp:66-82).
    void submit_q(size_t slot, int shifted_q);
    void wait_slot(size_t slot);

    // Codec I/O on the slot path: the graph input `input_index` takes a YUV420
    // frame (converted on the GPU) and the output `output_index` returns one
    // (kNoCodecTensor: that side stays a tensor).  Calls configure_slots(slots).
    static constexpr size_t kNoCodecTensor = static_cast<size_t>(-1);
    void configure_codec_io(int width, int height, int model_width, int model_height, float pixel_range,
                            size_t slots, size_t input_index, size_t output_index);
    void slot_input_yuv(size_t slot, uint8_t** y, uint8_t** u, uint8_t** v);
    void slot_output_yuv(size_t slot, const uint8_t** y, const uint8_t** u, const uint8_t** v) const;

    // Device-resident replay of the whole schedule (no host copies) for
    // timing; optional per-step event timing.
    void enqueue();
    void synchronize();
    std::vector<float> time_steps(int iterations, size_t flush_bytes);
    // Per-step device span inside a replayed frame for the tensor-core steps
    // (%globaltimer stamps of the kernels; 0 for other steps).
    std::vector<float> trace_spans(int iterations, size_t flush_bytes);
    const std::vector<StepInfo>& steps() const { return step_info_; }
    int kernel_launches_per_run() const;
    CUstream stream() const { return stream_; }
    CUcontext context() const { return ctx_; }
    size_t device_bytes() const;
    // Copies a tensor the last run materialised on the device (graph inputs,
    // outputs and every intermediate a step wrote; chain-internal values of a
    // fused step are never materialised) to host memory in NCHW order.
    // Returns false when the tensor does not exist on the device.
    bool read_value(const std::string& name, void* dst, size_t bytes);
    // Launches tensor-core conv step `index` once more with its phase trace
    // enabled and returns kTracePoints %globaltimer stamps per CTA (0 = not
    // reached).  Uses the device state of the last run.
    std::vector<uint64_t> trace_step(size_t index);
    // Failure-detection test: relaunches 1x1 tensor-core conv step `index`
    // once with every bounded wait of this backend's module limited to
    // `limit_ns` and CTA 0's producer withholding its first activation panel
    // (nothing is loaded or armed for it), waits for the launch, restores the
    // 2 s limit and returns the module status word it left (then cleared):
    // the wait bit of the role whose wait ran out first.  Uses the device
    // state of the last run; the step's output is left incomplete.
    uint32_t test_wait_expiry(size_t index, uint64_t limit_ns);
    // Before load(): give every materialised tensor its own arena slot so
    // read_value() sees all of them after a run (costs memory; debug only).
    void set_keep_all_values(bool keep);

private:
    struct Value;
    struct Step;
    struct Slot;

    void plan();
    void build_schedule();
    void capture();
    void check_status();
    // Launches every step in order on `s` (skip: index of a step left out, e.g. the
    // output boundary that the slot path's fused YUV conversion replaces).
    void launch_steps(CUstream s, size_t skip = static_cast<size_t>(-1));
    CUfunction fn(const char* name);
    CUdeviceptr entropy_scratch(size_t bytes);  // grow-only staging of the host-buffer entropy calls

    int device_ = 0;
    CUdevice dev_ = 0;
    CUcontext ctx_ = nullptr;
    CUstream stream_ = nullptr;                             // compute: every schedule launch
    CUstream copy_in_ = nullptr, copy_out_ = nullptr;       // slot pipeline copies
    CUmodule module_ = nullptr;
    CUdeviceptr status_ptr_ = 0;
    int sm_count_ = 148;
    int max_smem_optin_ = 227 * 1024;

    GraphDesc graph_;
    std::vector<uint8_t> weights_host_;
    std::vector<StateBinding> bindings_;
    // per binding: the bound output is written straight into the state buffer
    // (every read of the state input precedes the first write of the output)
    std::vector<bool> state_alias_;
    std::vector<size_t> ext_inputs_;   // indices into graph_.inputs
    std::vector<size_t> ext_outputs_;  // indices into graph_.outputs
    std::vector<uint32_t> absorbed_outputs_;  // outputs written straight into host staging

    std::vector<Value> values_;
    std::vector<Step> steps_;
    std::vector<StepInfo> step_info_;
    std::vector<Slot> slots_;
    struct CodecIo {
        int width = 0, height = 0, model_width = 0, model_height = 0;
        float pixel_range = 1.0f;
        int pad_left = 0, pad_top = 0;
        bool rotated = false;
        size_t input = kNoCodecTensor, output = kNoCodecTensor;
    } codec_;
    size_t fused_yuv_step_ = static_cast<size_t>(-1);  // output boundary replaced in the slot graphs

    DeviceBuffer weights_dev_, prepped_dev_, arena_dev_, flush_dev_, entropy_scratch_;
    std::vector<DeviceBuffer> input_dev_, input_stage_dev_, output_stage_dev_, state_dev_;
    std::vector<uint8_t> prepped_host_;

    CUgraph graph_handle_ = nullptr;
    CUgraphExec graph_exec_ = nullptr;
    bool state_ready_ = false;
    bool loaded_ = false;
    bool offline_ = false;
    // FFN fusion (ReGLU conv + following 1x1 conv in one kernel); MLVC_B200_FFN_FUSION=0 plans
    // the two convs as separate steps (same results, for comparison).
    bool ffn_fusion_ = true;
    // Depthwise 3x3 + following 1x1 conv in one kernel; MLVC_B200_DW_FUSION=0
    // plans them as separate steps (same results, for comparison).
    bool dw_fusion_ = true;
    // 1x1 expand conv (+ LeakyReLU) + depthwise 3x3 + 1x1 projection in one kernel;
    // MLVC_B200_MB_FUSION=0 plans them as the depthwise + 1x1 pair after a 1x1
    // conv (same results, for comparison).
    bool mb_fusion_ = true;
    // Recurrent-feature update chain in one kernel; MLVC_B200_TAIL_FUSION=0
    // runs its operators one by one (same results, for comparison).
    bool tail_fusion_ = true;
    // A 2x pixel shuffle after a 1x1 conv folded into the conv's store;
    // MLVC_B200_D2S_FUSION=0 plans it as its own step (same results).
    bool d2s_fusion_ = true;
    bool keep_all_values_ = false;
};

}  // namespace mlvc_b200
