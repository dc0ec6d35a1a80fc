// Thin RAII layer over the CUDA Driver API: the backend's only device
// dependency.  Every failing call throws std::runtime_error naming the call
// and the CUresult (the reference formats driver errors the same way:
// backends/driver_cubin/src/driver.cpp:63-81).
#pragma once

#include <cuda.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

namespace mlvc_b200 {

[[noreturn]] inline void throw_driver(CUresult r, const char* what)
{
    const char* name = nullptr;
    const char* desc = nullptr;
    cuGetErrorName(r, &name);
    cuGetErrorString(r, &desc);
    throw std::runtime_error(std::string("mlvc-b200: ") + what + " failed: " + (name ? name : "?") + " (" +
                             (desc ? desc : "") + ")");
}

inline void check(CUresult r, const char* what)
{
    if (r != CUDA_SUCCESS)
        throw_driver(r, what);
}

// Makes the device's primary context current on the calling thread for the
// lifetime of the guard (restores the previous one afterwards).
class ContextGuard {
public:
    explicit ContextGuard(CUcontext ctx)
    {
        check(cuCtxGetCurrent(&previous_), "cuCtxGetCurrent");
        if (previous_ != ctx)
            check(cuCtxSetCurrent(ctx), "cuCtxSetCurrent");
        restore_ = previous_ != ctx;
    }
    ~ContextGuard()
    {
        if (restore_)
            cuCtxSetCurrent(previous_);
    }
    ContextGuard(const ContextGuard&) = delete;
    ContextGuard& operator=(const ContextGuard&) = delete;

private:
    CUcontext previous_ = nullptr;
    bool restore_ = false;
};

class DeviceBuffer {
public:
    DeviceBuffer() = default;
    explicit DeviceBuffer(size_t bytes) : bytes_(bytes)
    {
        if (bytes)
            check(cuMemAlloc(&ptr_, bytes), "cuMemAlloc");
    }
    ~DeviceBuffer() { reset(); }
    DeviceBuffer(DeviceBuffer&& o) noexcept : ptr_(std::exchange(o.ptr_, 0)), bytes_(std::exchange(o.bytes_, 0)) {}
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept
    {
        if (this != &o) {
            reset();
            ptr_ = std::exchange(o.ptr_, 0);
            bytes_ = std::exchange(o.bytes_, 0);
        }
        return *this;
    }
    void reset()
    {
        if (ptr_)
            cuMemFree(ptr_);
        ptr_ = 0;
        bytes_ = 0;
    }
    CUdeviceptr get() const { return ptr_; }
    size_t bytes() const { return bytes_; }
    explicit operator bool() const { return ptr_ != 0; }

private:
    CUdeviceptr ptr_ = 0;
    size_t bytes_ = 0;
};

class PinnedBuffer {
public:
    PinnedBuffer() = default;
    explicit PinnedBuffer(size_t bytes) : bytes_(bytes)
    {
        if (bytes)
            check(cuMemHostAlloc(&ptr_, bytes, CU_MEMHOSTALLOC_PORTABLE), "cuMemHostAlloc");
    }
    ~PinnedBuffer() { reset(); }
    PinnedBuffer(PinnedBuffer&& o) noexcept : ptr_(std::exchange(o.ptr_, nullptr)), bytes_(std::exchange(o.bytes_, 0))
    {
    }
    PinnedBuffer& operator=(PinnedBuffer&& o) noexcept
    {
        if (this != &o) {
            reset();
            ptr_ = std::exchange(o.ptr_, nullptr);
            bytes_ = std::exchange(o.bytes_, 0);
        }
        return *this;
    }
    void reset()
    {
        if (ptr_)
            cuMemFreeHost(ptr_);
        ptr_ = nullptr;
        bytes_ = 0;
    }
    void* get() const { return ptr_; }
    size_t bytes() const { return bytes_; }

private:
    void* ptr_ = nullptr;
    size_t bytes_ = 0;
};

class Event {
public:
    explicit Event(unsigned int flags = CU_EVENT_DEFAULT) { check(cuEventCreate(&ev_, flags), "cuEventCreate"); }
    ~Event()
    {
        if (ev_)
            cuEventDestroy(ev_);
    }
    Event(Event&& o) noexcept : ev_(std::exchange(o.ev_, nullptr)) {}
    Event& operator=(Event&& o) noexcept
    {
        if (this != &o) {
            if (ev_)
                cuEventDestroy(ev_);
            ev_ = std::exchange(o.ev_, nullptr);
        }
        return *this;
    }
    CUevent get() const { return ev_; }

private:
    CUevent ev_ = nullptr;
};

}  // namespace mlvc_b200
