// s2_comm: the multi-GPU communicator of the sharded DiT step -- one rank per
// GPU, NCCL over NVLink / NVSwitch. NCCL is loaded on first use with dlopen
// ("libnccl.so.2"): a process that already holds an NCCL (PyTorch's) reuses
// that copy, any other loads the system one, and a process that never creates
// a communicator never loads NCCL at all.
//
// The step needs two collectives (no counterpart in the reference, which runs
// on one device):
//   * an fp32 sum all-reduce of each block's per-rank text attention mean
//     [58][2560] (and of the disjoint per-rank parts of the output latent);
//   * a row exchange between the window ownerships of consecutive blocks
//     (plain <-> shifted windows): one grouped ncclSend / ncclRecv per peer,
//     the rank's own rows copied on the device.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "s2_buffers.h"
#include "s2_comm.h"
#include "s2_internal.h"

namespace {

struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
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
        S2_SYM(send, "ncclSend");
        S2_SYM(recv, "ncclRecv");
        S2_SYM(group_start, "ncclGroupStart");
        S2_SYM(group_end, "ncclGroupEnd");
        S2_SYM(error_string, "ncclGetErrorString");
#undef S2_SYM
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_reduce && n.send && n.recv &&
               n.group_start && n.group_end && n.error_string;
    });
    return n;
}

}  // namespace

struct s2_comm {
    int device = 0, nranks = 1, rank = 0;
    ncclComm_t comm = nullptr;
};

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

extern "C" s2_status s2_comm_init(int device, int nranks, int rank, const char *id, s2_comm **out)
{
    s2::clear_error();
    if (!out || !id || nranks <= 0 || rank < 0 || rank >= nranks)
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
    const ncclResult_t r = n.comm_init_rank(&c->comm, nranks, u, rank);
    if (r != ncclSuccess) {
        delete c;
        return s2::set_error(S2_INFERENCE_FAILED, "ncclCommInitRank: %s", n.error_string(r));
    }
    *out = c;
    return S2_OK;
}

extern "C" s2_status s2_comm_destroy(s2_comm *c)
{
    if (!c) return S2_OK;
    s2::DeviceGuard guard(c->device);
    if (c->comm) nccl().comm_destroy(c->comm);
    delete c;
    return S2_OK;
}

extern "C" int s2_comm_size(const s2_comm *c) { return c ? c->nranks : 1; }
extern "C" int s2_comm_rank(const s2_comm *c) { return c ? c->rank : 0; }

namespace s2 {

s2_status comm_allreduce_f32(s2_comm *c, float *buf, size_t n, cudaStream_t st)
{
    if (!c || c->nranks == 1 || n == 0) return S2_OK;
    const Nccl &nc = nccl();
    const ncclResult_t r = nc.all_reduce(buf, buf, n, ncclFloat, ncclSum, c->comm, st);
    return r == ncclSuccess ? S2_OK : set_error(S2_INFERENCE_FAILED, "ncclAllReduce: %s", nc.error_string(r));
}

s2_status comm_exchange(s2_comm *c, const void *send, const size_t *send_off, const size_t *send_bytes, void *recv,
                        const size_t *recv_off, const size_t *recv_bytes, cudaStream_t st)
{
    const int me = c ? c->rank : 0;
    // own part: a device copy
    if (send_bytes[me] != recv_bytes[me])
        return set_error(S2_INVALID_ARGUMENT, "exchange: own segment %zu != %zu bytes", send_bytes[me], recv_bytes[me]);
    if (send_bytes[me] &&
        cudaMemcpyAsync(static_cast<char *>(recv) + recv_off[me], static_cast<const char *>(send) + send_off[me],
                        send_bytes[me], cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return set_error(S2_INFERENCE_FAILED, "exchange: own copy failed");
    if (!c || c->nranks == 1) return S2_OK;
    const Nccl &nc = nccl();
    ncclResult_t r = nc.group_start();
    for (int p = 0; p < c->nranks && r == ncclSuccess; ++p) {
        if (p == me) continue;
        if (send_bytes[p])
            r = nc.send(static_cast<const char *>(send) + send_off[p], send_bytes[p], ncclChar, p, c->comm, st);
        if (r == ncclSuccess && recv_bytes[p])
            r = nc.recv(static_cast<char *>(recv) + recv_off[p], recv_bytes[p], ncclChar, p, c->comm, st);
    }
    const ncclResult_t e = nc.group_end();
    if (r == ncclSuccess) r = e;
    return r == ncclSuccess ? S2_OK : set_error(S2_INFERENCE_FAILED, "exchange: %s", nc.error_string(r));
}

}  // namespace s2
