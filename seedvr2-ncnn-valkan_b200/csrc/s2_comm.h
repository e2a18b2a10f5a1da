// Internal collectives of the sharded DiT step (s2_comm.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "s2_b200.h"

namespace s2 {

// In-place fp32 sum over all ranks (no-op for a single rank or a null comm).
s2_status comm_allreduce_f32(s2_comm *c, float *buf, size_t n, cudaStream_t st);

// Every rank sends send[send_off[p] .. + send_bytes[p]) to rank p and receives
// recv_bytes[p] bytes from rank p at recv + recv_off[p]; the rank's own
// segment is a device copy. All ranks call it with matching sizes.
s2_status comm_exchange(s2_comm *c, const void *send, const size_t *send_off, const size_t *send_bytes, void *recv,
                        const size_t *recv_off, const size_t *recv_bytes, cudaStream_t st);

}  // namespace s2
