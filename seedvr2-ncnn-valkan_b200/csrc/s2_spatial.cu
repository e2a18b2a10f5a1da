// Single-head spatial attention for the VAE mid block on sm_100a:
// O = softmax(Q K^T * scale) V per frame over all H*W tokens of the frame
// (DynamicFramewiseSpatialAttention::forward,
// dynamic_framewise_spatial_attention.cpp:149-180), head dim d = channels
// padded to 128, 256 or 512 (zero channels change neither Q K^T nor the
// real output columns).
//
// TMEM holds 512 columns = 128 rows x (two S tiles + a 256-wide O): O for a
// 128-query tile over all 512 output columns would take all of TMEM, so a
// work item is (frame, 128-query tile, output half) with dout = min(d, 256)
// output columns; for d = 512 the two halves of a query tile recompute the
// same S = Q K^T (K = 512) in two CTAs.
//
// Per item the CTA keeps Q (128 x d fp16, up to 128 KB) resident and streams
// K slices (128 keys x 64 dims) and V slices (128 keys x 64 output columns)
// through one 6-slot ring of 16 KB slots in consumption order
// K0, K1, V0, K2, V1, K3, ... . The tensor core runs S(j+1) = Q K(j+1)^T into
// the second S buffer while the softmax warpgroup works on S(j), then
// O += P(j) V(j) with P in TMEM (written over S(j)'s columns). The running
// max is rescaled lazily (only when it grows by more than 2^8, exact because
// O and the row sum share the stale max); a rescale first waits for the
// previous P V to retire. The epilogue divides by the row sum and stores fp16
// rows into out[token][d] (columns of this half).
//
// CTA pairs (head dim 256 and 512): a cluster of two CTAs takes two
// consecutive query tiles of a frame (an M = 256 item) and runs tcgen05
// cta_group::2 MMAs issued by rank 0: each CTA keeps its own Q tile and loads
// only half of every K tile (64 keys, B split by N for Q K^T) and half of the
// item's V columns (128 of 256, B split by N for P V), while S, P and O stay
// per CTA (split by M). Every query tile re-reads its frame's whole K/V
// stream from L2, ~22 MB per item at d = 512; the pair halves those bytes per
// FLOP, which bound the single-CTA kernel near the L2-to-SM bandwidth
// (~7.7 TB/s of a measured ~9.4). Both CTAs' loads complete on rank 0's
// barriers; rank 0's commits arrive in both CTAs; rank 1's softmax warps
// announce P on rank 0's barrier. No load uses cluster multicast.
//
// Roles (192 threads): warps 0-3 softmax + epilogue (thread r <-> query row r
// <-> TMEM lane r), warp 4 TMA producer, warp 5 TMEM allocator + MMA issuer.
// Every wait is bounded (s2dev::mbar_wait); on timeout the CTA records an
// error code, drains its copies and MMAs, frees TMEM and exits.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <atomic>
#include <cstdint>

#include "s2_gemm.h"
#include "s2_internal.h"
#include "s2_launch.h"
#include "s2_sm100.cuh"

using namespace s2dev;

namespace {

constexpr int kBM = 128, kBN = 128;
constexpr int kSlots = 6;                                   // ring depth (even: V slice pairs never wrap)
constexpr uint32_t kBox = 128 * 64 * 2;                     // one 128-row x 64-element slice, 16 KB
constexpr uint32_t kOffQ = 0;                               // up to 8 slices (d = 512)
constexpr uint32_t kOffRing = 8 * kBox;
constexpr uint32_t kOffBar = kOffRing + kSlots * kBox;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");
constexpr int kThreads = 192;
constexpr int kProducerWarp = 4, kMmaWarp = 5;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColP = 32;                              // P inside its S buffer
constexpr uint32_t kColO = 256;

enum Bar {
    B_QFULL = 0,
    B_QEMPTY,                       // last Q K^T of an item retired
    B_FULL,                         // [kSlots]
    B_EMPTY = B_FULL + kSlots,      // [kSlots]
    B_SFULL = B_EMPTY + kSlots,     // [2] S buffer b holds the next S tile
    B_PFULL = B_SFULL + 2,          // P(j) in TMEM (128 thread arrivals; pairs: 8 warp arrivals on rank 0)
    B_ORDY,                         // one phase per retired P V
    B_ODONE,                        // last P V of an item retired
    B_DRAIN,
    B_COUNT
};
static_assert(8 * B_COUNT + 8 <= 256, "barrier area");

enum : int { E_Q = 32, E_SLOT = 33, E_EMPTY = 34, E_S = 35, E_P = 36, E_O = 37, E_DRAIN = 38 };

struct SpArgs {
    __half *out;
    int32_t *err;
    int tokens;      // per frame
    int cpad;        // head dim (128, 256 or 512)
    int dout;        // output columns per item
    int n_half;      // cpad / dout
    int n_qt;        // query units per frame: 128-row tiles, or tile pairs in pair mode
    int n_kv;        // key tiles per frame
    int n_items;
    float scale_log2;
};

struct Item {
    int frame, qt, half;  // qt: query unit (a tile, or a pair of tiles)
};

__device__ __forceinline__ Item decode(const SpArgs &a, int t)
{
    Item it;
    it.half = t % a.n_half;
    it.qt = (t / a.n_half) % a.n_qt;
    it.frame = t / (a.n_half * a.n_qt);
    return it;
}

__device__ __forceinline__ float max3f(float a, float b, float c)
{
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ bool wait_drain(uint32_t bar, uint32_t parity, int *err)
{
    int dummy = 0;
    return mbar_wait(bar, parity, &dummy, err, E_DRAIN);
}

template <bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    spatial_attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const SpArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    const uint32_t sQ = base + kOffQ, sRing = base + kOffRing;
    const uint32_t bar0 = base + kOffBar;
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + kOffBar + 8 * B_COUNT);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kOffBar + 8 * B_COUNT + 4);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = kPair ? cluster_rank() : 0u;
    const int unit = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int n_units = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
    const int kc = a.cpad / 64;                         // Q slices
    const int ks = kPair ? kc / 2 : kc;                 // ring slots per K tile (pairs: 64 keys x 128 dims)
    const int vc = kPair ? a.dout / 128 : a.dout / 64;  // ring slots per V tile (this CTA's columns; even)
    // this CTA's 128-row query tile within the item's query unit
    auto cta_tile = [&](int qt) { return kPair ? 2 * qt + static_cast<int>(rank) : qt; };
    // a pair's loads complete on rank 0's barriers
    auto lead_bar = [&](uint32_t bar) { return kPair ? cluster_map(bar, 0) : bar; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < B_COUNT; ++i) mbar_init(BAR(i), i == B_PFULL ? (kPair ? 8u : 128u) : 1u);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        if constexpr (kPair) {
            tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            uint32_t p = 0, nq = 0;
            bool ok = true;
            auto load = [&](uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1) {
                if constexpr (kPair)
                    tma_load_2d_pair(dst, map, lead_bar(bar), c0, c1);
                else
                    tma_load_2d(dst, map, bar, c0, c1);
            };
            // one ring slot: a 16 KB box (a V slice, or a single-CTA K slice) or, for a
            // pair's K, 64 keys x 128 dims as two 8 KB boxes
            auto slot = [&](const CUtensorMap *map, int c0, int c1, bool two) {
                const uint32_t s = p % kSlots, u = p / kSlots;
                if (!(ok = mbar_wait(BAR(B_EMPTY + s), (u & 1u) ^ 1u, abort, a.err, E_EMPTY))) return;
                if (!kPair || rank == 0) mbar_arrive_expect_tx(BAR(B_FULL + s), kPair ? 2 * kBox : kBox);
                load(sRing + s * kBox, map, BAR(B_FULL + s), c0, c1);
                if (two) load(sRing + s * kBox + kBox / 2, map, BAR(B_FULL + s), c0 + 64, c1);
                ++p;
            };
            for (int t = unit; ok && t < a.n_items; t += n_units) {
                const Item it = decode(a, t);
                const int row0 = it.frame * a.tokens;
                if (!(ok = mbar_wait(BAR(B_QEMPTY), (nq & 1u) ^ 1u, abort, a.err, E_Q))) break;
                if (!kPair || rank == 0) mbar_arrive_expect_tx(BAR(B_QFULL), (kPair ? 2 : 1) * kBox * kc);
                for (int c = 0; c < kc; ++c)
                    load(sQ + c * kBox, &tmQ, BAR(B_QFULL), c * 64, row0 + cta_tile(it.qt) * kBM);
                ++nq;
                auto load_k = [&](int j) {
                    if constexpr (kPair) {
                        for (int c = 0; ok && c < ks; ++c)
                            slot(&tmK, c * 128, row0 + j * kBN + static_cast<int>(rank) * (kBN / 2), true);
                    } else {
                        for (int c = 0; ok && c < ks; ++c) slot(&tmK, c * 64, row0 + j * kBN, false);
                    }
                };
                auto load_v = [&](int j) {
                    const int col0 = it.half * a.dout + (kPair ? static_cast<int>(rank) * (a.dout / 2) : 0);
                    for (int c = 0; ok && c < vc; ++c) slot(&tmV, col0 + c * 64, row0 + j * kBN, false);
                };
                load_k(0);
                if (a.n_kv > 1) load_k(1);
                for (int j = 0; ok && j < a.n_kv; ++j) {
                    load_v(j);
                    if (j + 2 < a.n_kv) load_k(j + 2);
                }
            }
            // No load may still be landing when the CTA exits. A pair's loads complete on rank
            // 0's barriers, which rank 0 drains; rank 1 waits until rank 0's MMAs released the
            // buffers its last loads filled (each release follows the loads it consumed).
            if (!kPair || rank == 0) {
                if (nq) wait_drain(BAR(B_QFULL), (nq - 1) & 1u, a.err);
                for (uint32_t s = 0; s < kSlots; ++s)
                    if (p > s) wait_drain(BAR(B_FULL + s), ((p - 1 - s) / kSlots) & 1u, a.err);
            } else {
                if (nq) wait_drain(BAR(B_QEMPTY), (nq - 1) & 1u, a.err);
                for (uint32_t s = 0; s < kSlots; ++s)
                    if (p > s) wait_drain(BAR(B_EMPTY + s), ((p - 1 - s) / kSlots) & 1u, a.err);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0 && rank == 0) {
            const uint32_t id_qk = idesc_f16(0u, kBN, 0, kPair ? 256u : 128u);
            const uint32_t id_pv = kPair ? idesc_f16(0u, static_cast<uint32_t>(a.dout), 1, 256u) : idesc_f16(0u, 128, 1);
            const uint64_t dq0 = smem_desc_sw128(sQ, 16, 1024);
            const uint64_t dk0 = smem_desc_sw128(sRing, 16, 1024);
            const uint64_t dv0 = smem_desc_sw128(sRing, kBox, 1024);  // MN-major: 64-column blocks one slot apart
            uint32_t p = 0, nq = 0, np = 0, g = 0;
            bool ok = true;
            // a pair's commits arrive in both CTAs
            auto commit = [&](uint32_t bar) {
                if constexpr (kPair) {
                    mma_commit_pair(cluster_map(bar, 0));
                    mma_commit_pair(cluster_map(bar, 1));
                } else {
                    mma_commit(bar);
                }
            };
            auto wait_slot = [&](uint32_t q) {
                ok = mbar_wait(BAR(B_FULL + q % kSlots), (q / kSlots) & 1u, abort, a.err, E_SLOT);
                return ok;
            };
            // S(b) = Q K(tile)^T, K streamed as ks ring slots
            auto qk = [&](uint32_t b) {
                for (int c = 0; c < ks; ++c, ++p) {
                    if (!wait_slot(p)) return;
                    tc_fence_after();
                    const uint32_t s = p % kSlots;
                    const uint64_t dk = dk0 + static_cast<uint64_t>((s * kBox) >> 4);
                    if constexpr (kPair) {
                        // 128 dims: Q slices 2c, 2c+1 against the slot's two 8 KB boxes
                        mma_chunk_pair_k64(tmem + b * 128u, dq0 + static_cast<uint64_t>((2 * c * kBox) >> 4), dk, id_qk,
                                           c > 0 ? 1u : 0u);
                        mma_chunk_pair_k64(tmem + b * 128u, dq0 + static_cast<uint64_t>(((2 * c + 1) * kBox) >> 4),
                                           dk + static_cast<uint64_t>((kBox / 2) >> 4), id_qk, 1u);
                    } else {
                        mma_chunk_ss_k64(tmem + b * 128u, dq0 + static_cast<uint64_t>((c * kBox) >> 4), dk, id_qk,
                                         c > 0 ? 1u : 0u);
                    }
                    commit(BAR(B_EMPTY + s));
                }
                commit(BAR(B_SFULL + b));
            };
            for (int t = unit; ok && t < a.n_items; t += n_units) {
                if (!(ok = mbar_wait(BAR(B_QFULL), nq & 1u, abort, a.err, E_Q))) break;
                ++nq;
                tc_fence_after();
                qk(g & 1u);
                if (ok && a.n_kv > 1) qk((g + 1) & 1u);
                if (!ok) break;
                if (a.n_kv <= 2) commit(BAR(B_QEMPTY));
                for (int j = 0; ok && j < a.n_kv; ++j) {
                    const uint32_t b = (g + j) & 1u;
                    if (!(ok = mbar_wait(BAR(B_PFULL), np & 1u, abort, a.err, E_P))) break;
                    ++np;
                    tc_fence_after();
                    for (int gr = 0; gr < vc / 2; ++gr, p += 2) {
                        if (!wait_slot(p) || !wait_slot(p + 1)) break;
                        tc_fence_after();
                        const uint32_t s = p % kSlots;
                        const uint64_t dv = dv0 + static_cast<uint64_t>((s * kBox) >> 4);
                        if constexpr (kPair)
                            mma_tile_ts_pair_k128(tmem + kColO, tmem + b * 128u + kColP, dv, id_pv, j > 0 ? 1u : 0u);
                        else
                            mma_tile_ts_k128(tmem + kColO + gr * 128u, tmem + b * 128u + kColP, dv, id_pv,
                                             j > 0 ? 1u : 0u);
                        commit(BAR(B_EMPTY + s));
                        commit(BAR(B_EMPTY + s + 1));
                    }
                    if (!ok) break;
                    commit(BAR(B_ORDY));
                    if (j + 2 < a.n_kv) {
                        qk(b);  // S buffer b is free once P(j) V(j) has read it: in-order issue
                        if (ok && j + 3 == a.n_kv) commit(BAR(B_QEMPTY));
                    }
                }
                if (!ok) break;
                commit(BAR(B_ODONE));
                g += a.n_kv;
            }
            if constexpr (kPair)
                mma_commit_pair(cluster_map(BAR(B_DRAIN), 0));
            else
                mma_commit(BAR(B_DRAIN));
            wait_drain(BAR(B_DRAIN), 0, a.err);
        }
    } else {
        // ---- softmax warpgroup: thread r <-> query row r of the tile <-> TMEM lane r ----
        const int r = threadIdx.x;
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const float c = a.scale_log2;
        uint32_t g = 0, no = 0;
        bool ok = true;
        for (int t = unit; ok && t < a.n_items; t += n_units) {
            const Item it = decode(a, t);
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < a.n_kv; ++j) {
                const uint32_t gg = g + j, b = gg & 1u;
                const uint32_t scol = tmem + lane_off + b * 128u;
                ok = mbar_wait(BAR(B_SFULL + b), (gg >> 1) & 1u, abort, a.err, E_S);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc_fence_after();
                uint32_t x[4][32];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) tmem_ld32(scol + cc * 32, x[cc]);
                tmem_wait_ld();
                const int valid = min(a.tokens - j * kBN, kBN);
                if (valid < kBN) {
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (cc * 32 + i >= valid) x[cc][i] = __float_as_uint(-INFINITY);
                }
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                    for (int i = 0; i < 32; i += 2)
                        mx4[(i >> 1) & 3] = max3f(mx4[(i >> 1) & 3], __uint_as_float(x[cc][i]), __uint_as_float(x[cc][i + 1]));
                const float cand = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * c;
                float m_use = m, alpha = 1.f;
                bool rescale = false;
                if (j == 0) {
                    m_use = cand;
                } else if (cand > m + 8.f) {
                    m_use = cand;
                    alpha = ex2_approx(m - cand);
                    rescale = true;
                }
                if (__any_sync(0xffffffffu, rescale)) {
                    // P(j-1) V(j-1) may still run: wait for its phase (PV(j-2) retired before S(j) was announced)
                    ok = mbar_wait(BAR(B_ORDY), (gg - 1) & 1u, abort, a.err, E_O);
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) break;
                    tc_fence_after();
                    for (int cc = 0; cc < a.dout / 32; ++cc) {
                        uint32_t o[32];
                        tmem_ld32(tmem + lane_off + kColO + cc * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(tmem + lane_off + kColO + cc * 32, o);
                    }
                }
                float2 rs2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 a2 = __ffma2_rn(make_float2(__uint_as_float(x[cc][2 * i]), __uint_as_float(x[cc][2 * i + 1])), c2, nm2);
                        float2 p2;
                        p2.x = ex2_approx(a2.x);
                        p2.y = ex2_approx(a2.y);
                        rs2[i & 3] = __fadd2_rn(rs2[i & 3], p2);
                        pk[i] = pack_h2(p2.x, p2.y);
                    }
                    tmem_st16(scol + kColP + cc * 16, pk);
                }
                tmem_wait_st();
                l = l * alpha + (((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y)) + ((rs2[2].x + rs2[2].y) + (rs2[3].x + rs2[3].y)));
                m = m_use;
                tc_fence_before();
                if constexpr (kPair) {
                    // one arrival per warp on rank 0's barrier (8 = 4 warps x 2 CTAs)
                    __syncwarp();
                    if (lane == 0) {
                        if (rank == 0)
                            mbar_arrive(BAR(B_PFULL));
                        else
                            mbar_arrive_remote_relaxed(cluster_map(BAR(B_PFULL), 0));
                    }
                } else {
                    mbar_arrive(BAR(B_PFULL));
                }
            }
            if (!ok) break;
            g += a.n_kv;
            ok = mbar_wait(BAR(B_ODONE), no & 1u, abort, a.err, E_O);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            ++no;
            tc_fence_after();
            // O is read before this group's next P_FULL lets the next item's first P V overwrite it
            const int q = cta_tile(it.qt) * kBM + r;
            __half *dst = q < a.tokens
                              ? a.out + (static_cast<size_t>(it.frame) * a.tokens + q) * a.cpad + it.half * a.dout
                              : nullptr;
            const float inv = 1.f / l;
            for (int cc = 0; cc < a.dout / 32; ++cc) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_off + kColO + cc * 32, o);
                tmem_wait_ld();
                if (dst) {
                    uint4 *d4 = reinterpret_cast<uint4 *>(dst + cc * 32);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const uint32_t *w = o + v * 8;
                        d4[v] = make_uint4(pack_h2(__uint_as_float(w[0]) * inv, __uint_as_float(w[1]) * inv),
                                           pack_h2(__uint_as_float(w[2]) * inv, __uint_as_float(w[3]) * inv),
                                           pack_h2(__uint_as_float(w[4]) * inv, __uint_as_float(w[5]) * inv),
                                           pack_h2(__uint_as_float(w[6]) * inv, __uint_as_float(w[7]) * inv));
                    }
                }
            }
            tc_fence_before();
        }
    }

    tc_fence_before();
    __syncthreads();
    // the pair's MMAs write both CTAs' TMEM and rank 1 signals rank 0: neither CTA
    // releases TMEM or exits before the other is done
    if constexpr (kPair) cluster_sync();
    if (warp == kMmaWarp) {
        tc_fence_after();
        if constexpr (kPair)
            tmem_dealloc_pair(tmem, kTmemCols);
        else
            tmem_dealloc(tmem, kTmemCols);
    }
#undef BAR
}

}  // namespace

extern "C" s2_status s2_spatial_attention(void *stream, const void *q, const void *k, const void *v, int channels,
                                          int head_dim, int frames, int tokens, void *out, int32_t *err)
{
    if (!q || !k || !v || !out || !err || channels <= 0 || frames <= 0 || tokens <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_spatial_attention: invalid arguments");
    if (head_dim != 128 && head_dim != 256 && head_dim != 512)
        return s2::set_error(S2_UNSUPPORTED, "s2_spatial_attention: head_dim %d (padded channels must be 128, 256 or 512)",
                             head_dim);
    if (channels > head_dim)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_spatial_attention: channels %d > head_dim %d", channels, head_dim);
    if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
          reinterpret_cast<uintptr_t>(out)) & 15u) != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_spatial_attention: buffers must be 16-byte aligned");
    const long long rows = 1LL * frames * tokens;
    if (rows > 0x7fffffffLL) return s2::set_error(S2_INVALID_ARGUMENT, "s2_spatial_attention: too many tokens");
    SpArgs a;
    a.out = static_cast<__half *>(out);
    a.err = err;
    a.tokens = tokens;
    a.cpad = head_dim;
    a.dout = head_dim < 256 ? head_dim : 256;
    a.n_half = head_dim / a.dout;
    const int n_tiles = (tokens + kBM - 1) / kBM;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // CTA pairs for 256-wide output halves (head dim 256 or 512) once a frame has at
    // least two query tiles; an odd tile count leaves the last pair's second tile past
    // the frame (rows whose outputs are not stored)
    const bool pair = a.dout == 256 && n_tiles >= 2 && sms >= 2;
    a.n_qt = pair ? (n_tiles + 1) / 2 : n_tiles;
    a.n_kv = (tokens + kBN - 1) / kBN;
    const long long items = 1LL * frames * a.n_qt * a.n_half;
    if (items > 0x7fffffffLL) return s2::set_error(S2_INVALID_ARGUMENT, "s2_spatial_attention: too many items");
    a.n_items = static_cast<int>(items);
    a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(channels)));
    CUtensorMap mq, mk, mv;
    const uint64_t pitch = static_cast<uint64_t>(head_dim) * 2;
    // a pair's CTA loads 64 keys of each K tile
    if (!s2::make_map_2d(&mq, q, head_dim, rows, pitch, 64, kBM) ||
        !s2::make_map_2d(&mk, k, head_dim, rows, pitch, 64, pair ? kBN / 2 : kBN) ||
        !s2::make_map_2d(&mv, v, head_dim, rows, pitch, 64, kBN))
        return s2::set_error(S2_INFERENCE_FAILED, "s2_spatial_attention: cuTensorMapEncodeTiled failed");
    static std::atomic<uint64_t> configured[2] = {};
    const s2_status cs = s2::once_per_device(configured[pair ? 1 : 0], [pair] {
        const cudaError_t e = cudaFuncSetAttribute(pair ? spatial_attention_kernel<true> : spatial_attention_kernel<false>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_spatial_attention: smem attribute: %s", cudaGetErrorString(e));
        return S2_OK;
    });
    if (cs != S2_OK) return cs;
    if (pair) {
        const long long pairs = items < sms / 2 ? items : sms / 2;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = kSmemBytes;
        cfg.stream = static_cast<cudaStream_t>(stream);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t le = cudaLaunchKernelEx(&cfg, spatial_attention_kernel<true>, mq, mk, mv, a);
        if (le != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_spatial_attention: pair launch failed: %s",
                                 cudaGetErrorString(le));
    } else {
        const int grid = static_cast<int>(items < sms ? items : sms);
        spatial_attention_kernel<false><<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(mq, mk, mv, a);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_spatial_attention: launch failed: %s", cudaGetErrorString(e));
    return S2_OK;
}
