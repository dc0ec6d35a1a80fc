// FP16 -> int32 entropy symbols with no device allocation at all.
//
// mlvc_b200_integer_values (host buffers) stages the values, the symbols and
// the kernel's out-of-range word in device memory that the backend allocates
// on first use and grows with cuMemAlloc.  Some callers cannot allow that: a
// device allocation synchronises the whole GPU (a real-time encoder thread
// with a per-frame latency budget cannot afford the stall), and processes
// whose device memory is owned by another framework's pool must not allocate
// behind its back.  This file gives them one entry point whose staging and
// out-of-range word live in a fixed file-scope __device__ array instead.
//
// Limits and sharing:
//   * at most kNoAllocMaxValues values per call; larger calls are rejected;
//   * the array (kNoAllocScratchBytes, about 12 MiB) is part of the library
//     image: every GPU that loads the library holds it until the process exits;
//   * every call on a device uses the same array.  A call waits for its own
//     work before it returns, so calls from one host thread never overlap;
//     calls from several host threads at once race on the array;
//   * the work runs on the calling thread's current device (cudaSetDevice;
//     device 0 by default) and its per-thread default stream;
//   * the first call on a device looks the array's device address up; make
//     that first call before any stream capture on that device;
//   * that address belongs to the device's primary context: do not call this
//     entry point after a cudaDeviceReset (or anything else that destroys the
//     primary context) in the same process, since it would still use the old
//     address.
//
// The arithmetic is the one of mlvc_integer_values_f16 (reference
// integer_values, core/src/entropy.cpp:201-226): truncation towards zero, and
// an error when a value is not finite or lies outside [-32768, 32767].
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>

namespace mlvc_b200 {

constexpr size_t kNoAllocMaxValues = size_t{1} << 21;  // 2,097,152 values per call
constexpr size_t kNoAllocFlagBytes = 256;              // out-of-range word, padded to keep the staging aligned
constexpr size_t kNoAllocScratchBytes = kNoAllocFlagBytes + kNoAllocMaxValues * (2 + 4);

}  // namespace mlvc_b200

// Layout: [0, 256) out-of-range word; then the FP16 values; then the int32 symbols.
static __device__ __align__(256) unsigned char mlvc_noalloc_scratch[mlvc_b200::kNoAllocScratchBytes];

namespace mlvc_b200 {
namespace {

__device__ __forceinline__ bool noalloc_symbol(float v, int32_t& out)
{
    if (!(v >= -32768.0f && v <= 32767.0f))  // also true for NaN
        return false;
    out = __float2int_rz(v);
    return true;
}

// Grid-stride: 8 values per thread (16-byte load, two 16-byte stores; the
// staging areas are 256-byte aligned), then the scalar tail.
__global__ void __launch_bounds__(256)
    integer_values_noalloc_kernel(const __half* src, long long count, int32_t* dst, unsigned int* out_of_range)
{
    bool bad = false;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
    const long long nvec = count / 8;
    for (long long i = tid; i < nvec; i += stride) {
        const uint4 raw = reinterpret_cast<const uint4*>(src)[i];
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        int32_t o[8];
        bool all = true;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
            all = noalloc_symbol(f.x, o[2 * k]) && all;
            all = noalloc_symbol(f.y, o[2 * k + 1]) && all;
        }
        if (all) {
            reinterpret_cast<int4*>(dst)[2 * i] = make_int4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<int4*>(dst)[2 * i + 1] = make_int4(o[4], o[5], o[6], o[7]);
        } else {
            bad = true;
        }
    }
    for (long long i = nvec * 8 + tid; i < count; i += stride) {
        int32_t o;
        if (noalloc_symbol(__half2float(src[i]), o))
            dst[i] = o;
        else
            bad = true;
    }
    if (bad)
        atomicOr(out_of_range, 1u);
}

void check_rt(cudaError_t e, const char* what)
{
    if (e != cudaSuccess)
        throw std::runtime_error(std::string("mlvc-b200: ") + what + ": " + cudaGetErrorString(e));
}

// Per-device set-up, done once with that device current: the array's device
// address (host code only sees a host-side stand-in under its name) and the
// SM count for the grid size.
constexpr int kMaxDevices = 64;
struct DeviceScratch {
    std::once_flag once;
    cudaError_t status = cudaSuccess;
    unsigned char* base = nullptr;
    int sm_count = 0;
};
DeviceScratch g_scratch[kMaxDevices];

const DeviceScratch& scratch_for_current_device()
{
    int dev = 0;
    check_rt(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        throw std::runtime_error("mlvc-b200: device index out of range for the no-allocation scratch");
    DeviceScratch& s = g_scratch[dev];
    std::call_once(s.once, [&] {
        void* ptr = nullptr;
        s.status = cudaGetSymbolAddress(&ptr, mlvc_noalloc_scratch);
        if (s.status == cudaSuccess)
            s.status = cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev);
        s.base = static_cast<unsigned char*>(ptr);
    });
    check_rt(s.status, "cudaGetSymbolAddress(no-allocation scratch)");
    return s;
}

}  // namespace

void integer_values_noalloc(const uint16_t* values, size_t count, int32_t* symbols)
{
    if (count > kNoAllocMaxValues)
        throw std::runtime_error("mlvc-b200: mlvc_b200_integer_values_noalloc takes at most " +
                                 std::to_string(kNoAllocMaxValues) + " values per call (got " +
                                 std::to_string(count) + ")");
    if (count == 0)
        return;
    if (!values || !symbols)
        throw std::runtime_error("mlvc-b200: null value buffer");
    const DeviceScratch& s = scratch_for_current_device();
    unsigned int* flag = reinterpret_cast<unsigned int*>(s.base);
    __half* src = reinterpret_cast<__half*>(s.base + kNoAllocFlagBytes);
    int32_t* dst = reinterpret_cast<int32_t*>(s.base + kNoAllocFlagBytes + kNoAllocMaxValues * 2);
    const cudaStream_t st = cudaStreamPerThread;
    // the array keeps the previous call's contents: the out-of-range word must start at zero
    check_rt(cudaMemsetAsync(flag, 0, sizeof(unsigned int), st), "cudaMemsetAsync(out-of-range word)");
    check_rt(cudaMemcpyAsync(src, values, count * 2, cudaMemcpyHostToDevice, st), "cudaMemcpyAsync(values)");
    const long long work = static_cast<long long>((count + 7) / 8);
    const long long cap = static_cast<long long>(s.sm_count > 0 ? s.sm_count : 1) * 16;
    const unsigned grid = static_cast<unsigned>(std::max(1LL, std::min((work + 255) / 256, cap)));
    integer_values_noalloc_kernel<<<grid, 256, 0, st>>>(src, static_cast<long long>(count), dst, flag);
    check_rt(cudaGetLastError(), "integer_values_noalloc_kernel");
    unsigned int bad = 0;
    check_rt(cudaMemcpyAsync(&bad, flag, sizeof(bad), cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync(out-of-range word)");
    check_rt(cudaMemcpyAsync(symbols, dst, count * sizeof(int32_t), cudaMemcpyDeviceToHost, st),
             "cudaMemcpyAsync(symbols)");
    check_rt(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (bad)
        throw std::runtime_error("entropy symbol is outside signed 16-bit range");
}

}  // namespace mlvc_b200
