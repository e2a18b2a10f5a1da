// Per-device one-time kernel set-up for the CUDA sources.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "s2_internal.h"

namespace s2 {

// Function attributes such as a kernel's dynamic shared-memory limit belong to
// each device's context, so they are set once per device, not once per
// process. `done` (one per kernel) records the devices (ids 0..63) on which
// `setup()` has returned S2_OK; later devices run it on first use. Two threads
// may both run `setup` for a new device: it only sets attributes, so that is
// harmless.
template <class F>
inline s2_status once_per_device(std::atomic<uint64_t> &done, F &&setup)
{
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(S2_INFERENCE_FAILED, "cudaGetDevice: %s", cudaGetErrorString(e));
    const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return S2_OK;
    const s2_status s = setup();
    if (s == S2_OK && bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
    return s;
}

}  // namespace s2
