// s2_comm: the multi-GPU communicator of the sharded DiT step -- one rank per
// GPU, NCCL over NVLink / NVSwitch. NCCL is loaded on first use with dlopen
// ("libnccl.so.2"): a process that already holds an NCCL (PyTorch's) reuses
// that copy, any other loads the system one, and a process that never creates
// a communicator never loads NCCL at all.
//
// The step needs (no counterpart in the reference, which runs on one device):
//   * an fp32 sum all-reduce of each block's per-rank text attention mean
//     [58][2560] (and of the disjoint per-rank parts of the output latent);
//   * every rank's buffers of the row exchange between the window ownerships
//     of consecutive blocks mapped into every other rank (comm_share: CUDA IPC
//     handles all-gathered over NCCL); the exchange itself is the epilogue of
//     the DiT block's last GEMM, which stores rows into peer memory.
//
// Failures: the ranks meet through a non-blocking communicator
// (ncclConfig_t.blocking = 0) whose creation is polled with
// ncclCommGetAsyncError against a deadline (s2_comm_init_timeout), so a rank
// that never joins cannot block the host: at the deadline it is aborted and
// S2_INFERENCE_FAILED returned. The collectives then run on a blocking
// communicator split from it (the same enqueue semantics as before, which CUDA
// graph capture of the sharded step relies on); every call's result and the
// communicator's asynchronous state are checked, and s2_comm_wait waits for a
// stream holding collectives under a watchdog that aborts the communicator on
// an asynchronous error (a peer gone) or at the deadline. An aborted
// communicator refuses further work.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "s2_buffers.h"
#include "s2_comm.h"
#include "s2_internal.h"

namespace {

struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    decltype(&ncclCommInitRankConfig) comm_init_rank_config = nullptr;
    decltype(&ncclCommGetAsyncError) comm_async_error = nullptr;
    decltype(&ncclCommAbort) comm_abort = nullptr;
    decltype(&ncclCommSplit) comm_split = nullptr;
    bool ok = false;
};

const Nccl &nccl()
{
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
#define S2_SYM(field, name) n.field = reinterpret_cast<decltype(n.field)>(dlsym(h, name))
        S2_SYM(get_unique_id, "ncclGetUniqueId");
        S2_SYM(comm_init_rank, "ncclCommInitRank");
        S2_SYM(comm_destroy, "ncclCommDestroy");
        S2_SYM(all_reduce, "ncclAllReduce");
        S2_SYM(all_gather, "ncclAllGather");
        S2_SYM(error_string, "ncclGetErrorString");
        S2_SYM(comm_init_rank_config, "ncclCommInitRankConfig");
        S2_SYM(comm_async_error, "ncclCommGetAsyncError");
        S2_SYM(comm_abort, "ncclCommAbort");
        S2_SYM(comm_split, "ncclCommSplit");
#undef S2_SYM
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce && n.all_gather &&
               n.error_string && n.comm_init_rank_config && n.comm_async_error && n.comm_abort && n.comm_split;
    });
    return n;
}

}  // namespace

struct s2_comm {
    int device = 0, nranks = 1, rank = 0;
    ncclComm_t comm = nullptr;   // blocking: the collectives
    ncclComm_t meet = nullptr;   // non-blocking: the deadline-guarded rendezvous it was split from
    long long timeout_ms = 300000;
    bool aborted = false;
};

namespace {

using Clock = std::chrono::steady_clock;

// Default deadline of communicator creation and of every NCCL call:
// $S2_COMM_TIMEOUT_MS, else 300 s.
long long default_timeout_ms()
{
    const char *e = std::getenv("S2_COMM_TIMEOUT_MS");
    const long long v = e ? std::atoll(e) : 0;
    return v > 0 ? v : 300000;
}

// Aborts the communicator (its in-flight NCCL kernels stop, its bootstrap and
// proxy threads end) and records why.
s2_status abort_comm(s2_comm *c, const char *what, const char *why)
{
    if (!c->aborted) {
        if (c->comm) nccl().comm_abort(c->comm);
        if (c->meet) nccl().comm_abort(c->meet);
        c->comm = c->meet = nullptr;
    }
    c->aborted = true;
    return s2::set_error(S2_INFERENCE_FAILED, "%s: %s; communicator aborted (rank %d of %d)", what, why, c->rank,
                         c->nranks);
}

// Polls communicator `nc`'s asynchronous state until its last call completed
// (ncclSuccess), failed, or the deadline passed.
s2_status settle_on(s2_comm *c, ncclComm_t nc, ncclResult_t r, const char *what)
{
    const Nccl &n = nccl();
    if (r != ncclSuccess && r != ncclInProgress) return abort_comm(c, what, n.error_string(r));
    const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t q = n.comm_async_error(nc, &st);
        if (q != ncclSuccess) return abort_comm(c, what, n.error_string(q));
        if (st == ncclSuccess) return S2_OK;
        if (st != ncclInProgress) return abort_comm(c, what, n.error_string(st));
        if (Clock::now() > deadline) return abort_comm(c, what, "timed out");
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

s2_status settle(s2_comm *c, ncclResult_t r, const char *what) { return settle_on(c, c->comm, r, what); }

}  // namespace

static_assert(sizeof(ncclUniqueId) == S2_COMM_ID_BYTES, "NCCL unique id size");

extern "C" s2_status s2_comm_unique_id(char *id)
{
    s2::clear_error();
    if (!id) return s2::set_error(S2_INVALID_ARGUMENT, "s2_comm_unique_id: id is NULL");
    const Nccl &n = nccl();
    if (!n.ok) return s2::set_error(S2_UNSUPPORTED, "s2_comm_unique_id: libnccl.so.2 not available");
    ncclUniqueId u;
    const ncclResult_t r = n.get_unique_id(&u);
    if (r != ncclSuccess) return s2::set_error(S2_INFERENCE_FAILED, "ncclGetUniqueId: %s", n.error_string(r));
    std::memcpy(id, &u, sizeof(u));
    return S2_OK;
}

extern "C" s2_status s2_comm_init_timeout(int device, int nranks, int rank, const char *id, long long timeout_ms,
                                          s2_comm **out)
{
    s2::clear_error();
    if (!out || !id || nranks <= 0 || rank < 0 || rank >= nranks || timeout_ms <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_comm_init: invalid arguments");
    *out = nullptr;
    const Nccl &n = nccl();
    if (!n.ok) return s2::set_error(S2_UNSUPPORTED, "s2_comm_init: libnccl.so.2 not available");
    s2::DeviceGuard guard(device);
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    auto *c = new s2_comm();
    c->device = device;
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_ms = timeout_ms;
    // non-blocking: the call returns at once and the ranks' rendezvous is polled
    // against the deadline, so a peer that never joins cannot block the host
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = n.comm_init_rank_config(&c->meet, nranks, u, rank, &cfg);
    if (!c->meet) {
        delete c;
        return s2::set_error(S2_INFERENCE_FAILED, "ncclCommInitRankConfig: %s", n.error_string(r));
    }
    s2_status s = settle_on(c, c->meet, r, "s2_comm_init (waiting for every rank to join)");
    if (s == S2_OK) {
        // every rank is there: split the blocking communicator of the collectives
        ncclConfig_t bcfg = NCCL_CONFIG_INITIALIZER;
        bcfg.blocking = 1;
        const ncclResult_t rs = n.comm_split(c->meet, 0, rank, &c->comm, &bcfg);
        s = settle_on(c, c->meet, rs, "s2_comm_init (split)");
        if (s == S2_OK && !c->comm) s = abort_comm(c, "s2_comm_init (split)", "no communicator returned");
        if (s == S2_OK) s = settle(c, ncclSuccess, "s2_comm_init (split)");
    }
    if (s != S2_OK) {
        delete c;  // abort_comm released both communicators
        return s;
    }
    *out = c;
    return S2_OK;
}

extern "C" s2_status s2_comm_init(int device, int nranks, int rank, const char *id, s2_comm **out)
{
    return s2_comm_init_timeout(device, nranks, rank, id, default_timeout_ms(), out);
}

extern "C" s2_status s2_comm_set_timeout(s2_comm *c, long long timeout_ms)
{
    if (!c || timeout_ms <= 0) return s2::set_error(S2_INVALID_ARGUMENT, "s2_comm_set_timeout: invalid arguments");
    c->timeout_ms = timeout_ms;
    return S2_OK;
}

extern "C" s2_status s2_comm_wait(s2_comm *c, void *stream)
{
    s2::clear_error();
    if (!c) return s2::set_error(S2_INVALID_ARGUMENT, "s2_comm_wait: communicator is NULL");
    if (c->aborted) return s2::set_error(S2_INFERENCE_FAILED, "s2_comm_wait: communicator was aborted");
    s2::DeviceGuard guard(c->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const Nccl &n = nccl();
    const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return S2_OK;
        if (q != cudaErrorNotReady)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_comm_wait: stream failed: %s", cudaGetErrorString(q));
        if (c->comm && c->nranks > 1) {
            ncclResult_t as = ncclSuccess;
            if (n.comm_async_error(c->comm, &as) != ncclSuccess || (as != ncclSuccess && as != ncclInProgress))
                return abort_comm(c, "s2_comm_wait", n.error_string(as));
        }
        if (Clock::now() > deadline) return abort_comm(c, "s2_comm_wait", "stream did not finish in time");
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

extern "C" s2_status s2_comm_destroy(s2_comm *c)
{
    if (!c) return S2_OK;
    s2::DeviceGuard guard(c->device);
    if (c->comm) nccl().comm_destroy(c->comm);
    if (c->meet) nccl().comm_abort(c->meet);  // idle since the split; no collective to finish
    delete c;
    return S2_OK;
}

extern "C" int s2_comm_size(const s2_comm *c) { return c ? c->nranks : 1; }
extern "C" int s2_comm_rank(const s2_comm *c) { return c ? c->rank : 0; }

namespace s2 {

s2_status comm_allreduce_f32(s2_comm *c, float *buf, size_t n, cudaStream_t st)
{
    if (!c || c->nranks == 1 || n == 0) return S2_OK;
    if (c->aborted) return set_error(S2_INFERENCE_FAILED, "ncclAllReduce: communicator was aborted");
    const Nccl &nc = nccl();
    return settle(c, nc.all_reduce(buf, buf, n, ncclFloat, ncclSum, c->comm, st), "ncclAllReduce");
}

s2_status comm_allgather_host(s2_comm *c, const void *local, size_t bytes, void *all, cudaStream_t st)
{
    const int n = c ? c->nranks : 1, me = c ? c->rank : 0;
    if (n == 1) {
        std::memcpy(all, local, bytes);
        return S2_OK;
    }
    if (c->aborted) return set_error(S2_INFERENCE_FAILED, "all-gather: communicator was aborted");
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
        return set_error(S2_UNSUPPORTED, "all-gather: not during stream capture");
    struct Tmp {  // the device buffer of the all-gather, released on every path
        DeviceBuffer b;
        ~Tmp() { b.release(); }
    } dev;
    if (!dev.b.ensure(n * bytes)) return set_error(S2_OUT_OF_MEMORY, "all-gather: device buffer");
    char *d = static_cast<char *>(dev.b.ptr);
    if (cudaMemcpy(d + me * bytes, local, bytes, cudaMemcpyHostToDevice) != cudaSuccess)
        return set_error(S2_INFERENCE_FAILED, "all-gather: upload failed");
    s2_status s = settle(c, nccl().all_gather(d + me * bytes, d, bytes, ncclChar, c->comm, st), "ncclAllGather");
    if (s != S2_OK) return s;
    if (cudaMemcpyAsync(all, d, n * bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return set_error(S2_INFERENCE_FAILED, "all-gather: download failed");
    // bounded: a rank that never joins ends in an aborted communicator, not a blocked host
    return s2_comm_wait(c, st);
}

s2_status comm_share(s2_comm *c, void *local, void **peers, cudaStream_t st)
{
    const int n = c ? c->nranks : 1, me = c ? c->rank : 0;
    for (int p = 0; p < n; ++p) peers[p] = p == me ? local : nullptr;
    if (n == 1) return S2_OK;
    if (c->aborted) return set_error(S2_INFERENCE_FAILED, "share: communicator was aborted");
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, local) != cudaSuccess)
        return set_error(S2_INFERENCE_FAILED, "share: cudaIpcGetMemHandle failed (not a cudaMalloc base pointer?)");
    std::vector<cudaIpcMemHandle_t> all(n);
    const s2_status s = comm_allgather_host(c, &h, sizeof(h), all.data(), st);
    if (s != S2_OK) return s;
    for (int p = 0; p < n; ++p) {
        if (p == me) continue;
        if (cudaIpcOpenMemHandle(&peers[p], all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            for (int q = 0; q < p; ++q)
                if (q != me && peers[q]) cudaIpcCloseMemHandle(peers[q]);
            for (int q = 0; q < n; ++q) peers[q] = q == me ? local : nullptr;
            return set_error(S2_INFERENCE_FAILED,
                             "share: cudaIpcOpenMemHandle of rank %d failed (ranks must be processes with peer access)", p);
        }
    }
    return S2_OK;
}

void comm_unshare(s2_comm *c, void **peers)
{
    const int n = c ? c->nranks : 1, me = c ? c->rank : 0;
    for (int p = 0; p < n; ++p) {
        if (p != me && peers[p]) cudaIpcCloseMemHandle(peers[p]);
        peers[p] = nullptr;
    }
}

}  // namespace s2
