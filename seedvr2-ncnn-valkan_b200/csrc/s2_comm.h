// Internal collectives of the sharded DiT step (s2_comm.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "s2_b200.h"

namespace s2 {

// In-place fp32 sum over all ranks (no-op for a single rank or a null comm).
s2_status comm_allreduce_f32(s2_comm *c, float *buf, size_t n, cudaStream_t st);

// Gathers `bytes` of host data from every rank: all = rank 0's, rank 1's, ...
// (comm size x bytes). Host-synchronising, bounded by the communicator's
// timeout (a rank that never joins aborts the communicator); not for stream
// capture. Every rank must call it at the same point.
s2_status comm_allgather_host(s2_comm *c, const void *local, size_t bytes, void *all, cudaStream_t st);

// Maps every rank's `local` allocation (a cudaMalloc base pointer; all ranks
// pass their buffer of the same role) into this process through CUDA IPC
// handles all-gathered over NCCL: peers[p] = rank p's allocation, peers[rank] =
// local (peers has comm size entries). Host-synchronising set-up call, not for
// stream capture; ranks must be processes on GPUs with peer access.
// comm_unshare closes the peers' mappings (before those allocations change).
s2_status comm_share(s2_comm *c, void *local, void **peers, cudaStream_t st);
void comm_unshare(s2_comm *c, void **peers);

}  // namespace s2
