// Thin inline-PTX wrappers for the sm_100a features the attention core uses:
// mbarriers (with bounded waits), TMA tiled loads (no multicast), and the
// 5th-generation tensor core (tcgen05: TMEM alloc, MMA, commit, TMEM ld/st).
// Encodings follow the PTX ISA (tcgen05 instruction / shared-memory matrix
// descriptors) as also used by CUTLASS's cute/arch/mma_sm100_desc.hpp.
#pragma once

#include <cstdint>

namespace s2dev {

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the phase of `bar` with parity `parity` to complete. Bounded: gives
// up after `timeout_ns` (or as soon as another role raised *abort), sets
// *abort and the global error word to `code`, and returns false, so a broken
// pipeline ends the kernel with an error instead of hanging the GPU.
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s; a healthy wait is < 100 us

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort, int *err, int code,
                                          uint64_t timeout_ns = kWaitTimeoutNs)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort) return false;
            if (global_timer_ns() - t0 > timeout_ns) {
                *abort = 1;
                if (err) atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

// ---- TMA -------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 3-D tiled bulk tensor load global -> shared, completion on an mbarrier.
// No multicast: every CTA fetches its own tiles.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void *tmap, uint32_t bar, int c0, int c1, int c2)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// 4-D tiled bulk tensor load global -> shared (c0 = innermost coordinate, which
// must be 16-byte aligned; the outer coordinates may be negative or past the
// extent, those elements are zero-filled). No multicast.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void *tmap, uint32_t bar, int c0, int c1, int c2,
                                            int c3)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// 2-D tiled bulk tensor load global -> shared (c0 = innermost coordinate).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, uint32_t bar, int c0, int c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// 2-D tiled bulk tensor store shared -> global (bulk async group). Elements
// outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const void *tmap, uint32_t src, int c0, int c1)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(src), "r"(c0), "r"(c1)
                 : "memory");
}
// Untiled bulk copy shared -> global of `bytes` (a multiple of 16; both addresses
// 16-byte aligned), tracked in this thread's bulk async group.
__device__ __forceinline__ void bulk_store(void *gdst, uint32_t ssrc, uint32_t bytes)
{
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(gdst)),
                 "r"(ssrc), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N bulk groups of this thread still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until all bulk groups of this thread have completed.
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---- tcgen05 ---------------------------------------------------------------

// Allocate `ncols` TMEM columns (power of two >= 32); the warp must be converged.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- CTA pairs (cluster of 2, tcgen05 cta_group::2) --------------------------
// The pair's MMAs are issued by CTA rank 0 and cover both CTAs' shared-memory
// operands and TMEM accumulators. No load here uses cluster multicast.

__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// arrive on an mbarrier of another CTA of the cluster
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// Relaxed arrive on another CTA's mbarrier, for hand-offs of TMEM data that the
// arriving thread has already completed (tcgen05.wait::st) and fenced
// (tcgen05.fence::before_thread_sync): the release form orders this thread's
// memory operations at cluster scope and costs ~1,000 cycles per arrive.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_bar)
{
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted on
// an mbarrier of the pair (the leader's)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void *tmap, uint32_t cluster_bar, int c0, int c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(cluster_bar), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// commit of the pair's MMAs to one mbarrier (any CTA of the pair, cluster address)
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
                 : "memory");
}

// One K=64 slice of a pair tile D[256][N] (+)= A[256][64] B[N][64]^T: four K=16
// MMAs; A rows 0-127 / 128-255 and B rows 0-N/2-1 / N/2-N-1 live at the same
// shared-memory offsets of CTA rank 0 / 1.
__device__ __forceinline__ void mma_chunk_pair_k64(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                   uint32_t acc_first)
{
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b64 a, b;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t"
        "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, t;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc_first)
        : "memory");
}

// A 128-key P V tile of a pair: D[256][N] (+)= P[256][128] V[128][N] with P in
// each CTA's TMEM (8 packed columns per K=16 step) and each CTA holding N/2
// columns of V, MN-major (16 keys = 2 KB per step; 64-column blocks LBO apart).
__device__ __forceinline__ void mma_tile_ts_pair_k128(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                      uint32_t idesc, uint32_t acc_first)
{
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b32 a;\n\t.reg .b64 b;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t"
        "add.u32 a, %1, 8;\n\tadd.s64 b, %2, 128;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 16;\n\tadd.s64 b, %2, 256;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 24;\n\tadd.s64 b, %2, 384;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 32;\n\tadd.s64 b, %2, 512;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 40;\n\tadd.s64 b, %2, 640;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 48;\n\tadd.s64 b, %2, 768;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 56;\n\tadd.s64 b, %2, 896;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [a], b, %3, t;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc_first)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Make generic-proxy shared-memory writes visible to the async proxy (MMA operand reads).
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/f16 in, f32 accumulate).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16. A (M x K, K-major) lives in
// TMEM: lane m = row m, each 32-bit column holds two consecutive K elements.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One 128x128x128 tile as 8 back-to-back K=16 MMAs in a single asm block,
// both operands 128B-swizzled K-major in shared memory: the descriptor start
// address advances +2 (32 B) per step and +1024 (16 KB, the second 64-element
// box) after four steps. Straight-line issue keeps the tensor core fed (a
// loop or branch between MMAs of the same accumulator leaves it idle).
// acc_first = 0 overwrites D with the first product.
__device__ __forceinline__ void mma_tile_ss_k128(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t acc_first)
{
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b64 a, b;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
        "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 1024;\n\tadd.s64 b, %2, 1024;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 1026;\n\tadd.s64 b, %2, 1026;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 1028;\n\tadd.s64 b, %2, 1028;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 1030;\n\tadd.s64 b, %2, 1030;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc_first)
        : "memory");
}

// One K=64 slice (a single 128B-swizzled 64-element box of each operand, both
// K-major) as 4 straight-line K=16 MMAs: descriptor start +2 (32 B) per step.
// The N extent comes from idesc, so the same helper serves N = 128 and 256.
__device__ __forceinline__ void mma_chunk_ss_k64(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t acc_first)
{
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b64 a, b;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
        "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
        "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc_first)
        : "memory");
}

// One 128x128x128 tile O (+)= P V as 8 K=16 MMAs in a single asm block: A = P
// in TMEM (8 columns per step), B = V 128B-swizzled MN-major in shared memory
// (16 key rows = 2 KB = +128 per step).
__device__ __forceinline__ void mma_tile_ts_k128(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t acc_first)
{
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t.reg .b32 a;\n\t.reg .b64 b;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.eq.u32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
        "add.u32 a, %1, 8;\n\tadd.s64 b, %2, 128;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 16;\n\tadd.s64 b, %2, 256;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 24;\n\tadd.s64 b, %2, 384;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 32;\n\tadd.s64 b, %2, 512;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 40;\n\tadd.s64 b, %2, 640;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 48;\n\tadd.s64 b, %2, 768;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
        "add.u32 a, %1, 56;\n\tadd.s64 b, %2, 896;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc_first)
        : "memory");
}

// Arrive on `bar` once all previously issued tcgen05 async ops of this thread complete.
__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// Instruction descriptor, kind::f16: D f32, A/B bf16 (fmt 1) or f16 (fmt 0),
// M = 128, N = n; b_mn_major selects an MN-major B operand.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t fmt, uint32_t n, uint32_t b_mn_major, uint32_t m = 128u)
{
    return (1u << 4)                 // D format f32
           | (fmt << 7) | (fmt << 10) // A, B formats
           | (b_mn_major << 16)       // B major
           | ((n >> 3) << 17)         // N >> 3
           | ((m >> 4) << 24);        // M >> 4 (128, or 256 for a CTA pair)
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version field.
// K-major tiles: lbo = 16 (unused), sbo = 1024 (8 rows x 128 B).
// MN-major tiles: lbo = byte stride between 64-element MN blocks,
//                 sbo = byte stride between 8-row K groups (1024).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// TMEM -> registers: 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r)
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Warpgroup register reallocation (all 4 warps of a warpgroup execute it).
template <uint32_t N>
__device__ __forceinline__ void regs_dec()
{
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_inc()
{
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ float ex2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

}  // namespace s2dev
