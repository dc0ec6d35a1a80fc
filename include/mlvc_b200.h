/*
 * mlvc_b200.h - C ABI of the B200 (sm_100a) inference backend for mlvc's
 * FP16 convolution stack.
 *
 * The backend executes the reference's AOT graph parts (graph schema 3:
 * aot/<part>/graph.pb + weights.bin, proto/mlvc_model.proto:30-83) on one
 * GPU.  Each entry point replaces one member of the reference backend
 * contract in runtime/include/mlvc/runtime/backend.hpp; the mapping is given
 * beside every declaration.  All functions return 0 on success and -1 on
 * failure; mlvc_b200_last_error() then returns the message of the exception
 * the C++ layer raised (the reference C ABI's convention,
 * codec/src/c_api.cpp:60-88).  Calls on one backend must come from one host
 * thread at a time (backend.hpp: one instance per session, one stream).
 *
 * Host tensors are NCHW, FP16 as raw IEEE binary16 bits (dtype 0) or INT32
 * (dtype 1), exactly as mlvc::Tensor (core/include/mlvc/core/tensor.hpp).
 */
#ifndef MLVC_B200_H
#define MLVC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLVC_B200_ABI_VERSION 1

typedef struct mlvc_b200_backend mlvc_b200_backend;

typedef struct mlvc_b200_tensor {
    int32_t dtype;     /* 0 = FP16, 1 = INT32 */
    int32_t rank;      /* 0..4 */
    int64_t shape[4];  /* NCHW */
    void* data;        /* host memory */
    size_t bytes;      /* capacity (outputs) / size (inputs) */
} mlvc_b200_tensor;

/* mlvc::StateTensorBinding (backend.hpp:34-40): graph output `output_index`
 * feeds graph input `input_index` of the next run and stays on the device. */
typedef struct mlvc_b200_state_binding {
    size_t input_index;
    size_t output_index;
} mlvc_b200_state_binding;

int mlvc_b200_abi_version(void);

/* Thread-local message of the last failing call ("" if none). */
const char* mlvc_b200_last_error(void);

/* Backend factory: replaces the "driver-cubin" factory registered through
 * register_backend() (backends/driver_cubin/src/backend.cpp:129-137) with
 * BackendOptions::device_id (backend.hpp:24-32). */
int mlvc_b200_create(int device_id, mlvc_b200_backend** out);
void mlvc_b200_destroy(mlvc_b200_backend* backend);

/* Planning-only instance (no reference counterpart): no GPU is touched;
 * load / load_memory decode, validate and plan the graph for a device with
 * `sm_count` SMs and `smem_optin_bytes` of shared memory per block, and the
 * step_* queries report the chosen kernels.  Execution calls fail. */
int mlvc_b200_create_offline(int sm_count, int smem_optin_bytes, mlvc_b200_backend** out);

/* InferenceBackend::name() (backend.hpp:52). Returns "b200". */
const char* mlvc_b200_name(const mlvc_b200_backend* backend);

/* InferenceBackend::load(model_name, ModelExecutionConfig) (backend.hpp:55-56),
 * reading <model_dir>/aot/<model_name>/{graph.pb,weights.bin} like
 * load_aot_graph (runtime/src/aot_graph.cpp:291-317). */
int mlvc_b200_load(mlvc_b200_backend* backend, const char* model_dir, const char* model_name,
                   const mlvc_b200_state_binding* bindings, size_t binding_count);

/* Same as mlvc_b200_load with the two assets in memory (the reference's
 * ModelAssetReader indirection, core/include/mlvc/core/assets.hpp:16-24). */
int mlvc_b200_load_memory(mlvc_b200_backend* backend, const void* graph_pb, size_t graph_bytes,
                          const void* weights, size_t weights_bytes, const mlvc_b200_state_binding* bindings,
                          size_t binding_count);

/* Host-visible graph inputs / outputs (state-bound tensors removed, graph
 * order kept; backend.hpp:58-60).  `info->data` is left NULL; `name` points to
 * storage owned by the backend. */
size_t mlvc_b200_input_count(const mlvc_b200_backend* backend);
size_t mlvc_b200_output_count(const mlvc_b200_backend* backend);
int mlvc_b200_input_info(const mlvc_b200_backend* backend, size_t index, mlvc_b200_tensor* info, const char** name);
int mlvc_b200_output_info(const mlvc_b200_backend* backend, size_t index, mlvc_b200_tensor* info,
                          const char** name);

/* InferenceBackend::run(inputs) -> outputs (backend.hpp:58-60): synchronous.
 * `outputs[i].data` must hold output_info(i).bytes. */
int mlvc_b200_run(mlvc_b200_backend* backend, const mlvc_b200_tensor* inputs, size_t input_count,
                  mlvc_b200_tensor* outputs, size_t output_count);

/* InferenceBackend::reset_state() (backend.hpp:62): zero every bound state. */
int mlvc_b200_reset_state(mlvc_b200_backend* backend);

/* BufferedCodecBackend slot path (backend.hpp:79-96), tensor form:
 * configure_codec_io(slots) / codec_slot_count / decoder_inputs(slot) /
 * submit_decoder(slot) / wait_codec_slot(slot).  Slot buffers are pinned host
 * memory owned by the backend, valid until the slot is resubmitted; a slot
 * must be waited before its buffers are reused (cuda_graph_executor.cpp:243-290). */
int mlvc_b200_configure_slots(mlvc_b200_backend* backend, size_t slot_count);
size_t mlvc_b200_slot_count(const mlvc_b200_backend* backend);
void* mlvc_b200_slot_input(mlvc_b200_backend* backend, size_t slot, size_t input_index);
const void* mlvc_b200_slot_output(const mlvc_b200_backend* backend, size_t slot, size_t output_index);
int mlvc_b200_submit(mlvc_b200_backend* backend, size_t slot);
/* submit_encoder(slot, shifted_q) / submit_decoder(slot, shifted_q)
 * (backend.hpp:87, 92): stores shifted_q in the slot's buffer of the int32 [1]
 * graph input named "q_index_shifted" and submits the slot, like the
 * reference's set_q_index (backends/driver_cubin/src/cuda_graph_executor.cpp:
 * 66-82, 286, 353).  Fails when the graph has no such input. */
int mlvc_b200_submit_q(mlvc_b200_backend* backend, size_t slot, int32_t shifted_q);
int mlvc_b200_wait_slot(mlvc_b200_backend* backend, size_t slot);

/* BufferedCodecBackend codec I/O (backend.hpp:69-93): CodecIoConfig {width,
 * height, model_width, model_height, pixel_range, slots} with the frame
 * placement of frame_padding (core/src/yuv.cpp:324-337: top-left, transposed
 * when it only fits rotated).  Graph input `input_index` then takes a YUV420
 * frame per slot, converted on the GPU like prepare_model_input
 * (yuv.cpp:339-400), and output `output_index` returns one, converted like
 * prepare_model_output_into (yuv.cpp:410-525); pass MLVC_B200_NO_CODEC_TENSOR
 * to keep either side a tensor.  Configures `slots` slots. */
#define MLVC_B200_NO_CODEC_TENSOR ((size_t)-1)
int mlvc_b200_configure_codec_io(mlvc_b200_backend* backend, int width, int height, int model_width,
                                 int model_height, float pixel_range, size_t slots, size_t input_index,
                                 size_t output_index);
/* encoder_input_yuv(slot) / decoder_output_yuv(slot) (backend.hpp:86, 93):
 * the slot's pinned Y, U, V planes (width x height, then two quarter planes). */
int mlvc_b200_slot_input_yuv(mlvc_b200_backend* backend, size_t slot, uint8_t** y, uint8_t** u, uint8_t** v);
int mlvc_b200_slot_output_yuv(const mlvc_b200_backend* backend, size_t slot, const uint8_t** y, const uint8_t** u,
                              const uint8_t** v);
/* Diagnostic (no reference counterpart): *fused = 1 when the slot graphs
 * convert the decoded frame to YUV420 straight from the NHWC tensor of the x8
 * output pixel shuffle (the output boundary step is left out of them), else 0. */
int mlvc_b200_codec_output_fused(const mlvc_b200_backend* backend, int* fused);

/* Entropy-coder inputs on the GPU.  These need a backend from
 * mlvc_b200_create but no loaded graph.
 *
 * mlvc_b200_scale_config carries the mlvc::ModelConfig fields that
 * extract_scales reads (core/include/mlvc/core/model.hpp; plane sizes of
 * core/src/model.cpp:94-126: ceil(model size / downsample_latent) for the
 * latent plane, ceil(model size / (downsample_latent * downsample_hyperprior))
 * for the hyper-latent plane) and the scale table's last index
 * (GaussianPmf::scale_levels - 1, core/src/entropy.cpp:389-391). */
typedef struct mlvc_b200_scale_config {
    int32_t hyperprior_channels;
    int32_t model_width;
    int32_t model_height;
    int32_t latent_channels;
    int32_t downsample_latent;
    int32_t downsample_hyperprior;
    int32_t y_scale_repeat;
    int32_t scale_max_index;
} mlvc_b200_scale_config;

/* Element counts of z_raw [1][hyper][zh][zw] and of each scale plane
 * [latent / 2][yh][yw] for `config`; validates it like extract_scales. */
int mlvc_b200_scale_shape(const mlvc_b200_scale_config* config, size_t* z_count, size_t* scale_count);

/* extract_scales(z_raw, config, scale_max_index, scales_0, scales_1)
 * (core/include/mlvc/core/scales.hpp:15-19, core/src/scales.cpp:25-105):
 * z_raw as FP16 bits (z_count elements, which must match the model's plane),
 * scales_0 / scales_1 with room for scale_count int32 each.  Errors carry the
 * reference's messages. */
int mlvc_b200_extract_scales(mlvc_b200_backend* backend, const uint16_t* z_raw, size_t z_count,
                             const mlvc_b200_scale_config* config, int32_t* scales_0, int32_t* scales_1,
                             size_t scale_count);

/* integer_values(tensor, result) (core/src/entropy.cpp:201-226): FP16 bits ->
 * int32 by truncation; fails with "entropy symbol is outside signed 16-bit
 * range" when a value is not finite or outside [-32768, 32767]. */
int mlvc_b200_integer_values(mlvc_b200_backend* backend, const uint16_t* values, size_t count, int32_t* symbols);

/* Device-memory forms of the two calls above (no reference counterpart: the
 * reference runs them on host tensors).  Pointers are device addresses
 * (CUdeviceptr) on the backend's device, from any allocator; the kernels are
 * enqueued on mlvc_b200_stream() and the calls return without waiting.  The
 * caller zeroes the device uint32 *out_of_range before the call; it is
 * non-zero afterwards when a value was not finite or outside [-32768, 32767]
 * (that element's symbol is then left unwritten). */
int mlvc_b200_extract_scales_device(mlvc_b200_backend* backend, uint64_t z_raw, const mlvc_b200_scale_config* config,
                                    uint64_t scales_0, uint64_t scales_1);
int mlvc_b200_integer_values_device(mlvc_b200_backend* backend, uint64_t values, size_t count, uint64_t symbols,
                                    uint64_t out_of_range);

/* integer_values without any device allocation (no counterpart in the
 * reference).  For callers that cannot allocate device memory: a device
 * allocation synchronises the whole GPU, which a real-time encoder thread
 * with a per-frame latency budget cannot afford, and a process whose device
 * memory is owned by another framework's pool must not allocate behind its
 * back.  Same arguments, results and errors as mlvc_b200_integer_values, but
 * the staging of values and symbols and the out-of-range word live in a fixed
 * array inside the library (about 12 MiB, held by every GPU that loads the
 * library until the process exits), so needs no backend handle.  Limits:
 * at most 2,097,152 values per call (larger calls fail with an error); runs
 * on the calling thread's current device (cudaSetDevice, device 0 by
 * default) and returns when the work is done; every call on a device shares
 * the one array, so calls from several host threads at once race; the first
 * call on a device looks the array's address up, so make it before any
 * stream capture on that device, and do not call it after a
 * cudaDeviceReset of that device (or anything else that destroys its primary
 * context) in the same process: it keeps the address it looked up. */
int mlvc_b200_integer_values_noalloc(const uint16_t* values, size_t count, int32_t* symbols);

/* Measurement hooks (no reference counterpart; the reference times whole
 * runs with steady_clock, codec/src/pipeline.cpp:341-415).  enqueue replays
 * the captured schedule on the backend's stream with the device-resident
 * inputs of the previous run; time_steps launches every step separately
 * between CUDA events and returns the mean milliseconds per step (with
 * flush_bytes > 0, each step is preceded by an untimed memset of that many
 * bytes so it starts from a cold L2). */
int mlvc_b200_enqueue(mlvc_b200_backend* backend);
int mlvc_b200_synchronize(mlvc_b200_backend* backend);
void* mlvc_b200_stream(const mlvc_b200_backend* backend);
size_t mlvc_b200_step_count(const mlvc_b200_backend* backend);
int mlvc_b200_step_info(const mlvc_b200_backend* backend, size_t index, const char** kernel, const char** nodes,
                        double* flops, double* bytes, uint32_t* grid, uint32_t* block, uint32_t* smem);
int mlvc_b200_time_steps(mlvc_b200_backend* backend, int iterations, size_t flush_bytes, float* ms_per_step);
/* In-frame kernel spans (no reference counterpart): consecutive kernels of a
 * replayed frame overlap (programmatic dependent launch), so CUDA events
 * between them cannot separate them without removing the overlap.  The
 * schedule is captured once more with the phase trace of every tensor-core
 * step enabled and replayed `iterations` times like a frame (flush_bytes > 0:
 * an L2 flush before each); for those steps ms_per_step[i] = the last CTA's
 * exit minus the first CTA's passing of griddepcontrol.wait (%globaltimer,
 * written by the kernel), averaged; 0 for other steps. */
int mlvc_b200_trace_spans(mlvc_b200_backend* backend, int iterations, size_t flush_bytes, float* ms_per_step);
int mlvc_b200_kernel_launches(const mlvc_b200_backend* backend);

/* Phase trace of one tensor-core conv or fused FFN step: relaunches it once
 * with %globaltimer stamps enabled; writes 64 stamps per CTA (CTA start,
 * setup done, weights issued, weights landed, first activation panel, last
 * MMA commit, first accumulator seen by the epilogue, epilogue done, exit,
 * then fused-FFN, fused-depthwise and fused-block chunk events; 0 = not
 * reached) and the total count to
 * *count.  Debug facility: no counterpart in the reference. */
int mlvc_b200_trace_step(mlvc_b200_backend* backend, size_t index, uint64_t* stamps, size_t capacity,
                         size_t* count);
size_t mlvc_b200_device_bytes(const mlvc_b200_backend* backend);

/* Failure-detection test hook (no reference counterpart; the reference's
 * kernels have no bounded waits).  Relaunches step `step_index`, which must
 * be a mlvc_conv1x1_tc step of the loaded schedule, once with every bounded
 * device wait of this backend limited to `limit_ns` (at most 2 s) and CTA 0's
 * TMA producer withholding its first activation panel: no copy is issued or
 * armed for it, so the tensor-core issuer stalls on it (and behind it the
 * epilogue and the producer); the first of those bounded waits to run out
 * sets the CTA's abort flag, every role winds down (producer drains the
 * copies it armed, epilogue drains its residual load) and the kernel
 * returns.  Then waits, restores the 2 s limit and stores the module status
 * word in *status (wait bits: 0x1 producer, 0x2 tensor-core issuer, 0x4
 * epilogue), clearing it.  The step's output is left
 * incomplete; the next run recomputes it.  Uses the device state of the last
 * run. */
int mlvc_b200_test_wait_expiry(mlvc_b200_backend* backend, size_t step_index, uint64_t limit_ns, uint32_t* status);

/* Debug dump of one named tensor of the last run, NCHW on the host: the
 * reference's --debug-dir tensor dumps (codec/src/pipeline.cpp:225-266).
 * Requires mlvc_b200_set_debug_tensors(backend, 1) before load, which keeps
 * every materialised tensor in its own arena slot.  *found is 0 for tensors
 * that exist only inside a fused step. */
int mlvc_b200_set_debug_tensors(mlvc_b200_backend* backend, int enable);
int mlvc_b200_read_tensor(mlvc_b200_backend* backend, const char* name, void* dst, size_t bytes, int* found);

#ifdef __cplusplus
}
#endif
#endif /* MLVC_B200_H */
