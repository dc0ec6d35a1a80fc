// Lazy binding of the CUDA Driver API.
//
// The library does not link against libcuda: each Driver API entry point the
// backend uses is defined here (hidden visibility) as a trampoline that
// resolves the real function from libcuda.so.1 with dlopen/dlsym on first use.
// The shared object therefore loads on machines without a GPU driver (its C
// ABI can be inspected and tested there); any backend call made without a
// driver fails with CUDA_ERROR_NOT_INITIALIZED, which the caller reports.
// The reference's backend loads the driver the same way
// (backends/driver_cubin/src/driver.cpp:12-50).
//
// cuda.h maps several names to versioned symbols (cuMemAlloc ->
// cuMemAlloc_v2, ...); the two-level stringification below resolves the same
// versioned symbol the header declares.
#include <cuda.h>
#include <dlfcn.h>

#include <mutex>

namespace {

void* driver_handle()
{
    static void* h = [] {
        void* p = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
        if (!p)
            p = dlopen("libcuda.so", RTLD_NOW | RTLD_LOCAL);
        return p;
    }();
    return h;
}

void* resolve(const char* name)
{
    void* h = driver_handle();
    return h ? dlsym(h, name) : nullptr;
}

}  // namespace

#define MLVC_STR2(x) #x
#define MLVC_STR(x) MLVC_STR2(x)
#define MLVC_FWD(name, params, args)                                                      \
    extern "C" __attribute__((visibility("hidden"))) CUresult CUDAAPI name params          \
    {                                                                                     \
        using Fn = CUresult(CUDAAPI*) params;                                             \
        static Fn fn = reinterpret_cast<Fn>(resolve(MLVC_STR(name)));                     \
        return fn ? fn args : CUDA_ERROR_NOT_INITIALIZED;                                 \
    }

MLVC_FWD(cuInit, (unsigned int flags), (flags))
MLVC_FWD(cuDeviceGetCount, (int* count), (count))
MLVC_FWD(cuDeviceGet, (CUdevice * device, int ordinal), (device, ordinal))
MLVC_FWD(cuDeviceGetAttribute, (int* pi, CUdevice_attribute attrib, CUdevice dev), (pi, attrib, dev))
MLVC_FWD(cuDevicePrimaryCtxRetain, (CUcontext * pctx, CUdevice dev), (pctx, dev))
MLVC_FWD(cuDevicePrimaryCtxRelease, (CUdevice dev), (dev))
MLVC_FWD(cuCtxGetCurrent, (CUcontext * pctx), (pctx))
MLVC_FWD(cuCtxSetCurrent, (CUcontext ctx), (ctx))
MLVC_FWD(cuStreamCreate, (CUstream * phStream, unsigned int Flags), (phStream, Flags))
MLVC_FWD(cuStreamDestroy, (CUstream hStream), (hStream))
MLVC_FWD(cuStreamSynchronize, (CUstream hStream), (hStream))
MLVC_FWD(cuModuleLoadData, (CUmodule * module, const void* image), (module, image))
MLVC_FWD(cuModuleUnload, (CUmodule hmod), (hmod))
MLVC_FWD(cuModuleGetGlobal, (CUdeviceptr * dptr, size_t* bytes, CUmodule hmod, const char* name),
         (dptr, bytes, hmod, name))
MLVC_FWD(cuModuleGetFunction, (CUfunction * hfunc, CUmodule hmod, const char* name), (hfunc, hmod, name))
MLVC_FWD(cuFuncSetAttribute, (CUfunction hfunc, CUfunction_attribute attrib, int value), (hfunc, attrib, value))
MLVC_FWD(cuMemAlloc, (CUdeviceptr * dptr, size_t bytesize), (dptr, bytesize))
MLVC_FWD(cuMemFree, (CUdeviceptr dptr), (dptr))
MLVC_FWD(cuMemHostAlloc, (void** pp, size_t bytesize, unsigned int Flags), (pp, bytesize, Flags))
MLVC_FWD(cuMemFreeHost, (void* p), (p))
MLVC_FWD(cuMemcpyHtoD, (CUdeviceptr dstDevice, const void* srcHost, size_t ByteCount), (dstDevice, srcHost, ByteCount))
MLVC_FWD(cuMemcpyDtoH, (void* dstHost, CUdeviceptr srcDevice, size_t ByteCount), (dstHost, srcDevice, ByteCount))
MLVC_FWD(cuMemcpyHtoDAsync, (CUdeviceptr dstDevice, const void* srcHost, size_t ByteCount, CUstream hStream),
         (dstDevice, srcHost, ByteCount, hStream))
MLVC_FWD(cuMemcpyDtoHAsync, (void* dstHost, CUdeviceptr srcDevice, size_t ByteCount, CUstream hStream),
         (dstHost, srcDevice, ByteCount, hStream))
MLVC_FWD(cuMemcpyDtoDAsync, (CUdeviceptr dstDevice, CUdeviceptr srcDevice, size_t ByteCount, CUstream hStream),
         (dstDevice, srcDevice, ByteCount, hStream))
MLVC_FWD(cuMemsetD8, (CUdeviceptr dstDevice, unsigned char uc, size_t N), (dstDevice, uc, N))
MLVC_FWD(cuMemsetD8Async, (CUdeviceptr dstDevice, unsigned char uc, size_t N, CUstream hStream),
         (dstDevice, uc, N, hStream))
MLVC_FWD(cuEventCreate, (CUevent * phEvent, unsigned int Flags), (phEvent, Flags))
MLVC_FWD(cuEventDestroy, (CUevent hEvent), (hEvent))
MLVC_FWD(cuEventRecord, (CUevent hEvent, CUstream hStream), (hEvent, hStream))
MLVC_FWD(cuEventSynchronize, (CUevent hEvent), (hEvent))
MLVC_FWD(cuStreamWaitEvent, (CUstream hStream, CUevent hEvent, unsigned int Flags), (hStream, hEvent, Flags))
MLVC_FWD(cuEventElapsedTime, (float* pMilliseconds, CUevent hStart, CUevent hEnd), (pMilliseconds, hStart, hEnd))
MLVC_FWD(cuLaunchKernel,
         (CUfunction f, unsigned int gridDimX, unsigned int gridDimY, unsigned int gridDimZ, unsigned int blockDimX,
          unsigned int blockDimY, unsigned int blockDimZ, unsigned int sharedMemBytes, CUstream hStream,
          void** kernelParams, void** extra),
         (f, gridDimX, gridDimY, gridDimZ, blockDimX, blockDimY, blockDimZ, sharedMemBytes, hStream, kernelParams,
          extra))
MLVC_FWD(cuLaunchKernelEx, (const CUlaunchConfig* config, CUfunction f, void** kernelParams, void** extra),
         (config, f, kernelParams, extra))
MLVC_FWD(cuStreamBeginCapture, (CUstream hStream, CUstreamCaptureMode mode), (hStream, mode))
MLVC_FWD(cuStreamEndCapture, (CUstream hStream, CUgraph* phGraph), (hStream, phGraph))
MLVC_FWD(cuGraphInstantiateWithFlags, (CUgraphExec * phGraphExec, CUgraph hGraph, unsigned long long flags),
         (phGraphExec, hGraph, flags))
MLVC_FWD(cuGraphLaunch, (CUgraphExec hGraphExec, CUstream hStream), (hGraphExec, hStream))
MLVC_FWD(cuGraphExecDestroy, (CUgraphExec hGraphExec), (hGraphExec))
MLVC_FWD(cuGraphDestroy, (CUgraph hGraph), (hGraph))
MLVC_FWD(cuTensorMapEncodeTiled,
         (CUtensorMap * tensorMap, CUtensorMapDataType tensorDataType, cuuint32_t tensorRank, void* globalAddress,
          const cuuint64_t* globalDim, const cuuint64_t* globalStrides, const cuuint32_t* boxDim,
          const cuuint32_t* elementStrides, CUtensorMapInterleave interleave, CUtensorMapSwizzle swizzle,
          CUtensorMapL2promotion l2Promotion, CUtensorMapFloatOOBfill oobFill),
         (tensorMap, tensorDataType, tensorRank, globalAddress, globalDim, globalStrides, boxDim, elementStrides,
          interleave, swizzle, l2Promotion, oobFill))

extern "C" __attribute__((visibility("hidden"))) CUresult CUDAAPI cuGetErrorName(CUresult error, const char** pStr)
{
    using Fn = CUresult(CUDAAPI*)(CUresult, const char**);
    static Fn fn = reinterpret_cast<Fn>(resolve("cuGetErrorName"));
    if (fn)
        return fn(error, pStr);
    *pStr = error == CUDA_ERROR_NOT_INITIALIZED ? "CUDA_ERROR_NOT_INITIALIZED (libcuda.so.1 not found)" : "unknown";
    return CUDA_SUCCESS;
}

extern "C" __attribute__((visibility("hidden"))) CUresult CUDAAPI cuGetErrorString(CUresult error, const char** pStr)
{
    using Fn = CUresult(CUDAAPI*)(CUresult, const char**);
    static Fn fn = reinterpret_cast<Fn>(resolve("cuGetErrorString"));
    if (fn)
        return fn(error, pStr);
    *pStr = "the CUDA driver library could not be loaded";
    return CUDA_SUCCESS;
}
