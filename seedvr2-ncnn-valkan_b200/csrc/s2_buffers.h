// Host-side RAII helpers for the layer objects: growable device buffers and a
// current-device guard.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

namespace s2 {

// Failure injection for tests (s2_debug_fail_allocations): true while the
// counter of allocations to fail is positive (it is decremented).
bool alloc_fault();

struct DeviceBuffer {
    void *ptr = nullptr;
    size_t bytes = 0;
    bool ensure(size_t want)
    {
        if (want <= bytes) return true;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
        if (alloc_fault()) return false;
        if (cudaMalloc(&ptr, want) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        bytes = want;
        return true;
    }
    void release()
    {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev)
    {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard()
    {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace s2
