// Dense GEMM D = A B^T for sm_100a (tcgen05 MMA into TMEM, TMA-fed 4-stage
// shared-memory ring), used for the 1x1 projections around the VAE mid-block
// attention (DynamicFramewiseSpatialAttention's linear(),
// dynamic_framewise_spatial_attention.cpp:79-103: Q/K/V and the output
// projection with its residual, :145-147 and :185-194).
//
// Tiles are 128 rows x 256 columns with K streamed in 64-element slices
// (A slice 16 KB + B slice 32 KB per stage); each slice is 4 K=16 MMAs of
// M128 N256. The CTA is persistent over tiles (row-block major, column block
// minor, so the 128-row A block is re-read from L2, not HBM, for every column
// block) and keeps two accumulators in TMEM (2 x 256 columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer, warps 2-5 epilogue (thread <-> accumulator row == TMEM lane).
// Every wait is bounded (s2dev::mbar_wait): on timeout the CTA records an
// error code in args.err, drains its in-flight copies and MMAs and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "s2_gemm.h"
#include "s2_internal.h"
#include "s2_launch.h"
#include "s2_sm100.cuh"

using namespace s2dev;

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr uint32_t kABytes = kBM * kBK * 2;   // 16 KB
constexpr uint32_t kStageChunk = 32 * 32 * 4;  // epilogue staging chunk, sized for fp32 (fp16 uses the first half)
constexpr int kThreads = 192;

// Tile shape: 128 x BN per CTA with BN = 256 (the default) or 128 (twice the
// tiles, for GEMMs too small to fill the grid with 256-wide tiles); with kPair a
// cluster of two CTAs computes a 256 x 256 tile with tcgen05 cta_group::2 MMAs
// (each CTA holds its 128 rows of A, half of the tile's B rows, and its 128 rows
// of the accumulator), halving the B bytes each CTA loads and reads per FLOP.
template <int BN, bool kPair = false>
struct Tile {
    static constexpr int kBN = BN;
    static constexpr int kBRows = kPair ? BN / 2 : BN;  // B rows this CTA loads per slice
    static constexpr int kTileRows = kPair ? 2 * kBM : kBM;
    static constexpr uint32_t kBBytes = kBRows * kBK * 2;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = kStageBytes > 32768 ? 4 : 6;
    static constexpr uint32_t kOffStage = kStages * kStageBytes;  // epilogue staging: 4 warps x 2 chunks
    static constexpr uint32_t kOffBar = kOffStage + 4 * 2 * kStageChunk;
    static constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers/flags + alignment slack
    static constexpr uint32_t kTmemCols = 2 * BN;                 // two accumulators
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

constexpr int kMaxStages = 6;
enum Bar {
    B_FULL = 0,                     // [kStages] A and B slices landed
    B_EMPTY = B_FULL + kMaxStages,  // [kStages] MMAs reading the stage retired
    B_ACCF = B_EMPTY + kMaxStages,  // [2] accumulator complete
    B_ACCE = B_ACCF + 2,            // [2] epilogue finished reading it (128 arrivals)
    B_DRAIN = B_ACCE + 2,
    B_COUNT
};
static_assert(8 * B_COUNT + 8 <= 256, "barrier area");

// device error codes of this kernel
enum : int { E_FULL = 16, E_EMPTY = 17, E_ACCF = 18, E_ACCE = 19, E_DRAIN = 20 };

__device__ __forceinline__ bool wait_drain(uint32_t bar, uint32_t parity, int *err)
{
    int dummy = 0;
    return mbar_wait(bar, parity, &dummy, err, E_DRAIN);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Round two values to bf16 (RNE), then store those values as fp16 (exact in
// fp16's normal range): the attention core's operand format.
__device__ __forceinline__ uint32_t pack_bf16_h2(float a, float b)
{
    const __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
    const uint32_t u = *reinterpret_cast<const uint32_t *>(&r);
    return pack_h2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

template <int BN, bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmO0, const __grid_constant__ CUtensorMap tmO1,
                const __grid_constant__ CUtensorMap tmO2, const s2::GemmArgs a)
{
    using T = Tile<BN, kPair>;
    constexpr int kBN = T::kBN, kStages = T::kStages, kTileRows = T::kTileRows;
    constexpr uint32_t kStageBytes = T::kStageBytes, kOffStage = T::kOffStage, kOffBar = T::kOffBar;
    constexpr uint32_t kTmemCols = T::kTmemCols;
    // CTA pair: rank 0 issues the MMAs; tiles are distributed over clusters
    const uint32_t rank = kPair ? cluster_rank() : 0u;
    const int unit = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int n_units = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    const uint32_t bar0 = base + kOffBar;
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + kOffBar + 8 * B_COUNT);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kOffBar + 8 * B_COUNT + 4);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_blocks = (a.N + kBN - 1) / kBN;
    const int n_tiles = ((a.M + kTileRows - 1) / kTileRows) * n_blocks;
    const int n_k = a.K / kBK;
    // split-K: work unit t = (tile t / ks, K range t % ks), the K slices [kc_lo, kc_hi)
    const int ks = kPair ? 1 : (a.ksplit > 1 ? a.ksplit : 1);
    const int n_work = n_tiles * ks;
    auto kc_lo = [&](int t) { return static_cast<int>((1LL * (t % ks) * n_k) / ks); };
    auto kc_hi = [&](int t) { return static_cast<int>((1LL * (t % ks + 1) * n_k) / ks); };

    if (threadIdx.x == 0) {
        // a pair's accumulator-empty barrier (rank 0's) counts both CTAs' epilogue threads
        for (int i = 0; i < B_COUNT; ++i)
            mbar_init(BAR(i), (i >= B_ACCE && i < B_ACCE + 2) ? (kPair ? 256u : 128u) : 1u);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
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

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            uint32_t p = 0;  // stage uses issued
            bool ok = true;
            for (int t = unit; ok && t < n_work; t += n_units) {
                const int tile = t / ks;
                const int m0 = (tile / n_blocks) * kTileRows + static_cast<int>(rank) * kBM;
                const int n0 = (tile % n_blocks) * kBN + static_cast<int>(rank) * T::kBRows;
                // convolution: the tile's 128 rows are 4 runs of 32 output columns, each in
                // one output row (owp is a multiple of 32); their input origins
                int seg_w[4] = {0, 0, 0, 0}, seg_h[4] = {0, 0, 0, 0}, seg_d[4] = {0, 0, 0, 0};
                if (!kPair && a.conv) {
                    const s2::ConvGeom &g = a.geom;
                    for (int sg = 0; sg < 4; ++sg) {
                        const int pos = m0 + sg * 32, plane = g.oh * g.owp;
                        const int z = pos / plane, rem = pos - z * plane, i = rem / g.owp, j0 = rem - i * g.owp;
                        seg_w[sg] = j0 * g.sw - g.pl;
                        seg_h[sg] = i * g.sh - g.pt;
                        seg_d[sg] = z * g.sd - g.pf;
                    }
                }
                for (int kc = kc_lo(t); kc < kc_hi(t); ++kc, ++p) {
                    const uint32_t s = p % kStages, u = p / kStages;
                    if (!(ok = mbar_wait(BAR(B_EMPTY + s), (u & 1u) ^ 1u, abort, a.err, E_EMPTY))) break;
                    const uint32_t sa = base + s * kStageBytes;
                    if (!kPair && a.conv) {
                        // tap (td, th, tw) and channel slice cs of this K slice
                        const s2::ConvGeom &g = a.geom;
                        const int tap = kc / g.cslices, cs = kc - tap * g.cslices;
                        const int td = tap / (g.kh * g.kw), th = (tap / g.kw) % g.kh, tw = tap % g.kw;
                        mbar_arrive_expect_tx(BAR(B_FULL + s), kStageBytes);
#pragma unroll
                        for (int sg = 0; sg < 4; ++sg)
                            tma_load_4d(sa + sg * (kABytes / 4), &tmA, BAR(B_FULL + s), cs * kBK,
                                        seg_w[sg] + tw * g.dw, seg_h[sg] + th * g.dh, seg_d[sg] + td * g.dd);
                        tma_load_2d(sa + kABytes, &tmB, BAR(B_FULL + s), kc * kBK, n0);
                    } else if constexpr (kPair) {
                        // both CTAs' slices are counted on rank 0's full barrier
                        if (rank == 0) mbar_arrive_expect_tx(BAR(B_FULL + s), 2 * kStageBytes);
                        const uint32_t fb = cluster_map(BAR(B_FULL + s), 0);
                        tma_load_2d_pair(sa, &tmA, fb, kc * kBK, m0);
                        tma_load_2d_pair(sa + kABytes, &tmB, fb, kc * kBK, n0);
                    } else {
                        mbar_arrive_expect_tx(BAR(B_FULL + s), kStageBytes);
                        tma_load_2d(sa, &tmA, BAR(B_FULL + s), kc * kBK, m0);
                        tma_load_2d(sa + kABytes, &tmB, BAR(B_FULL + s), kc * kBK, n0);
                    }
                }
            }
            // No copy may still be landing when the CTA exits. A pair's loads complete on
            // rank 0's barriers, which rank 0 drains; rank 1 waits for its last stages to be
            // released by rank 0's MMAs (each release follows the loads that filled it).
            for (uint32_t s = 0; s < kStages; ++s)
                if (p > s) {
                    if (!kPair || rank == 0)
                        wait_drain(BAR(B_FULL + s), ((p - 1 - s) / kStages) & 1u, a.err);
                    else
                        wait_drain(BAR(B_EMPTY + s), ((p - 1 - s) / kStages) & 1u, a.err);
                }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = idesc_f16(0u, kBN, 0, kPair ? 256u : 128u);
            const uint64_t d0 = smem_desc_sw128(base, 16, 1024);
            // a pair's commits arrive on the barrier in each CTA
            auto commit = [&](uint32_t bar) {
                if constexpr (kPair) {
                    mma_commit_pair(cluster_map(bar, 0));
                    mma_commit_pair(cluster_map(bar, 1));
                } else {
                    mma_commit(bar);
                }
            };
            uint32_t p = 0, lt = 0;
            bool ok = true;
            for (int t = unit; ok && t < n_work; t += n_units, ++lt) {
                const uint32_t b = lt & 1u;
                if (!(ok = mbar_wait(BAR(B_ACCE + b), ((lt >> 1) & 1u) ^ 1u, abort, a.err, E_ACCE))) break;
                tc_fence_after();
                const int k0 = kc_lo(t);
                for (int kc = k0; kc < kc_hi(t); ++kc, ++p) {
                    const uint32_t s = p % kStages, u = p / kStages;
                    if (!(ok = mbar_wait(BAR(B_FULL + s), u & 1u, abort, a.err, E_FULL))) break;
                    tc_fence_after();
                    const uint64_t da = d0 + static_cast<uint64_t>((s * kStageBytes) >> 4);
                    const uint64_t db = da + static_cast<uint64_t>(kABytes >> 4);
                    if constexpr (kPair)
                        mma_chunk_pair_k64(tmem + b * kBN, da, db, idesc, kc > k0 ? 1u : 0u);
                    else
                        mma_chunk_ss_k64(tmem + b * kBN, da, db, idesc, kc > k0 ? 1u : 0u);
                    commit(BAR(B_EMPTY + s));
                }
                if (!ok) break;
                commit(BAR(B_ACCF + b));
            }
            if constexpr (kPair)
                mma_commit_pair(cluster_map(BAR(B_DRAIN), 0));
            else
                mma_commit(BAR(B_DRAIN));
            wait_drain(BAR(B_DRAIN), 0, a.err);
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (accumulator rows)
        const int quad = warp & 3;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
        // fp16 outputs leave through shared memory as TMA bulk stores of 32 rows x 32 columns
        const uint32_t stg0 = base + kOffStage + static_cast<uint32_t>(warp - 2) * 2 * kStageChunk;
        uint8_t *stg0_g = gbase + kOffStage + static_cast<uint32_t>(warp - 2) * 2 * kStageChunk;
        uint32_t sb = 0;
        auto store_chunk = [&](const CUtensorMap *map, const uint4 (&v)[4], int col, int row) {
            if (lane == 0) bulk_wait_group_read<1>();  // the store that last used this buffer has read it
            __syncwarp();
            uint4 *dst = reinterpret_cast<uint4 *>(stg0_g + sb * kStageChunk + lane * 64);
#pragma unroll
            for (int k = 0; k < 4; ++k) dst[k] = v[k];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(map, stg0 + sb * kStageChunk, col, row);
                bulk_commit_group();
            }
            sb ^= 1u;
        };
        // fp32: 32 rows x 128 B per chunk, 128B-swizzled (16-byte chunk k of row r at k ^ (r % 8)),
        // which the output map's swizzle mode undoes; conflict-free shared stores
        auto store_chunk32 = [&](const CUtensorMap *map, const float4 (&v)[8], int col, int row) {
            if (lane == 0) bulk_wait_group_read<1>();
            __syncwarp();
            float4 *dst = reinterpret_cast<float4 *>(stg0_g + sb * kStageChunk + lane * 128);
#pragma unroll
            for (int k = 0; k < 8; ++k) dst[k ^ (lane & 7)] = v[k];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(map, stg0 + sb * kStageChunk, col, row);
                bulk_commit_group();
            }
            sb ^= 1u;
        };
        uint32_t lt = 0;
        bool ok = true;
        for (int t = unit; ok && t < n_work; t += n_units, ++lt) {
            const int tile = t / ks;
            const int m0 = (tile / n_blocks) * kTileRows + static_cast<int>(rank) * kBM, n0 = (tile % n_blocks) * kBN;
            const uint32_t b = lt & 1u;
            ok = mbar_wait(BAR(B_ACCF + b), (lt >> 1) & 1u, abort, a.err, E_ACCF);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            const int row = m0 + quad * 32 + lane;
            const bool row_ok = row < a.M;
            const bool split_k = ks > 1;
            for (int c = 0; c < kBN / 32 && (split_k || (a.epilogue != s2::GEMM_EPI_SWIGLU_F16 &&
                                                          a.epilogue != s2::GEMM_EPI_QKV_PACK)); ++c) {
                const int n = n0 + c * 32;
                if (n >= a.N) break;
                uint32_t r[32];
                tmem_ld32(tmem + lane_off + b * kBN + c * 32, r);
                tmem_wait_ld();
                if (split_k) {
                    // raw fp32 partial sums of this K range; the finish kernel applies the epilogue
                    if (row_ok) {
                        float4 *dst = reinterpret_cast<float4 *>(
                            a.partial + (static_cast<size_t>(t % ks) * a.M + row) * a.N + n);
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                 __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                    }
                } else if (a.epilogue == s2::GEMM_EPI_SPLIT_F16) {
                    const int which = n / a.split, col = n - which * a.split;
                    uint4 v4[4];
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            f[e] = __uint_as_float(r[v * 8 + e]) + (a.bias ? __ldg(a.bias + n + v * 8 + e) : 0.f);
                        v4[v] = make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]),
                                           pack_h2(f[6], f[7]));
                    }
                    store_chunk(which == 0 ? &tmO0 : (which == 1 ? &tmO1 : &tmO2), v4, col, m0 + quad * 32);
                } else if (a.epilogue == s2::GEMM_EPI_RESID_T_F32) {
                    // channel-major store: for a fixed column the warp's 32 rows are 128 contiguous bytes.
                    // All 32 residual loads of the chunk are issued before its stores (y and resid are
                    // distinct buffers; interleaving them would serialise every load behind a store).
                    float res[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        res[e] = (a.resid && row_ok && n + e < a.n_valid)
                                     ? __ldg(a.resid + static_cast<size_t>(n + e) * a.ldt + row)
                                     : 0.f;
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const int col = n + e;
                        if (row_ok && col < a.n_valid)
                            a.y[static_cast<size_t>(col) * a.ldt + row] =
                                __uint_as_float(r[e]) + (a.bias ? __ldg(a.bias + col) : 0.f) + res[e];
                    }
                } else if (a.epilogue == s2::GEMM_EPI_SHUFFLE_F32) {
                    // columns in (oy, ot, c, ox) order, ox innermost: the chunk holds the (ox = 0, 1)
                    // pairs of 16 channels with one (oy, ot), so each thread writes 16 float2 and a
                    // warp's 32 tokens fill 256 contiguous bytes of each output row
                    const int pair0 = n >> 1;
                    const int q = pair0 / a.sh_cin, c0 = pair0 - q * a.sh_cin;
                    const int oy = q / a.sh_tr, ot = q - oy * a.sh_tr;
                    const int hw = a.sh_h * a.sh_w;
                    const int f = row / hw, yx = row - f * hw, yy = yx / a.sh_w, xx = yx - yy * a.sh_w;
                    const int rawf = f * a.sh_tr + ot;
                    const bool keep = row_ok && !(a.sh_tr > 1 && rawf == 1);
                    const int of = (a.sh_tr > 1 && rawf > 1) ? rawf - 1 : rawf;
                    const size_t pos = (static_cast<size_t>(of) * 2 * a.sh_h + 2 * yy + oy) * (2 * a.sh_w) + 2 * xx;
                    if (keep) {
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            float2 v;
                            v.x = __uint_as_float(r[2 * k]) + (a.bias ? __ldg(a.bias + n + 2 * k) : 0.f);
                            v.y = __uint_as_float(r[2 * k + 1]) + (a.bias ? __ldg(a.bias + n + 2 * k + 1) : 0.f);
                            *reinterpret_cast<float2 *>(a.y + static_cast<size_t>(c0 + k) * a.ldt + pos) = v;
                        }
                    }
                } else if (a.epilogue == s2::GEMM_EPI_CONV_F32) {
                    // output position of this row on the grid padded to owp columns
                    const s2::ConvGeom &g = a.geom;
                    const int plane = g.oh * g.owp;
                    const int z = row / plane, rem = row - z * plane, i = rem / g.owp, j = rem - i * g.owp;
                    if (row_ok && j < g.ow) {
                        const size_t pos = (static_cast<size_t>(z) * g.oh + i) * g.ow + j;
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (n + e < a.n_valid)
                                a.y[static_cast<size_t>(n + e) * a.ldt + pos] =
                                    __uint_as_float(r[e]) + (a.bias ? __ldg(a.bias + n + e) : 0.f);
                    }
                } else if (a.epilogue == s2::GEMM_EPI_GATED_RESID_F32) {
                    // rows below the split (or all rows) leave by TMA store through the y map, which
                    // clips at that row count; rows past the split go to y2 with per-thread stores
                    const bool second = a.split_row > 0 && row >= a.split_row;
                    const int rr = second ? row - a.split_row : row;
                    const float *rbase = second ? a.resid2 : a.resid;
                    float4 outv[8];
                    if (row_ok) {
                        const float4 *rs = reinterpret_cast<const float4 *>(rbase + static_cast<size_t>(rr) * a.N + n);
                        float4 res[8];
#pragma unroll
                        for (int v = 0; v < 8; ++v) res[v] = rbase ? __ldg(rs + v) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int v = 0; v < 8; ++v) {
                            float o[4];
                            const float rv[4] = {res[v].x, res[v].y, res[v].z, res[v].w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int col = n + v * 4 + e;
                                float t = __uint_as_float(r[v * 4 + e]);
                                if (a.bias) t = __fadd_rn(t, __ldg(a.bias + col));
                                if (a.gmul) t = __fmul_rn(t, __ldg(a.gmul + col));
                                o[e] = __fmul_rn(__fadd_rn(t, rv[e]), a.out_scale);
                            }
                            outv[v] = make_float4(o[0], o[1], o[2], o[3]);
                        }
                        if (second) {
                            float4 *yd = reinterpret_cast<float4 *>(a.y2 + static_cast<size_t>(rr) * a.N + n);
#pragma unroll
                            for (int v = 0; v < 8; ++v) yd[v] = outv[v];
                        }
                    }
                    const int y_rows = a.split_row > 0 ? a.split_row : a.M;
                    if (a.row_dest) {
                        // every row to its own destination: the warp stages its 32 rows' 128-byte
                        // segments (16-byte chunk k of row r at k ^ (r % 8)) and stores them four
                        // rows per instruction
                        float *my_dst = nullptr;
                        if (row_ok && row < y_rows) {
                            const int2 dd = __ldg(a.row_dest + row);
                            float *bp = a.dest_base[0];
#pragma unroll
                            for (int q = 1; q < 8; ++q)
                                if (dd.x == q) bp = a.dest_base[q];
                            my_dst = bp + static_cast<size_t>(dd.y) * a.N + n;
                        }
                        float4 *stg = reinterpret_cast<float4 *>(stg0_g);
                        __syncwarp();
#pragma unroll
                        for (int k = 0; k < 8; ++k) stg[lane * 8 + (k ^ (lane & 7))] = outv[k];
                        __syncwarp();
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int rr = 4 * k + (lane >> 3), cc = lane & 7;
                            const unsigned long long pa =
                                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(my_dst), rr);
                            const float4 v = stg[rr * 8 + (cc ^ (rr & 7))];
                            if (pa) reinterpret_cast<float4 *>(pa)[cc] = v;
                        }
                    } else if (m0 + quad * 32 < y_rows) {
                        store_chunk32(&tmO0, outv, n, m0 + quad * 32);
                    }
                }
            }
            if (kBN == 256 && a.epilogue == s2::GEMM_EPI_SWIGLU_F16 && !split_k && ok) {
                // pairs (gate chunk c, in chunk c + 4) of the 256-column tile
                for (int c = 0; c < 4; ++c) {
                    uint32_t gr[32], ur[32];
                    tmem_ld32(tmem + lane_off + b * kBN + c * 32, gr);
                    tmem_ld32(tmem + lane_off + b * kBN + 128 + c * 32, ur);
                    tmem_wait_ld();
                    uint4 v4[4];
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const float g = __uint_as_float(gr[v * 8 + e]);
                            f[e] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), __uint_as_float(ur[v * 8 + e]));
                        }
                        v4[v] = make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]),
                                           pack_h2(f[6], f[7]));
                    }
                    store_chunk(&tmO0, v4, n0 / 2 + c * 32, m0 + quad * 32);
                }
            }
            if (a.epilogue == s2::GEMM_EPI_QKV_PACK && !split_k && ok) {
                // Per 128-column head block: Q/K rows are RMS-normalised over the head (two
                // passes over TMEM: the fp64 square sum, then the scaled values), V rows only
                // rounded. The warp stages its 32 rows x 256 B (16-byte chunk k of row r at
                // k ^ (r % 8): conflict-free) and stores them as whole 256-byte packed rows.
                const s2::PackArgs &pk = a.pk;
                // map entries: packed row >= 0 (video), -1 - l (text row l), -0x7fffffff (a video
                // row the layer's window subset does not hold: nothing stored)
                const int4 mp = row_ok ? __ldg(pk.map + row) : make_int4(-0x7fffffff, 0, 0, 0);
                const bool text = row_ok && mp.x < 0 && mp.x != -0x7fffffff;
                const float *gam = pk.gammas + (text ? 2 : 0) * 128;
                uint4 *stage = reinterpret_cast<uint4 *>(stg0_g);
                for (int hc = 0; hc < kBN / 128; ++hc) {
                    const int col0 = n0 + hc * 128;
                    if (col0 >= a.N) break;
                    const int sec = col0 / pk.dim, head = (col0 - sec * pk.dim) >> 7;
                    const uint32_t tcol = tmem + lane_off + b * kBN + hc * 128;
                    float inv = 1.f;
                    if (sec < 2) {
                        // Square sum in fp32 over four interleaved chains. The reference sums in
                        // fp64; here the fp32 sum is within ~2e-6 (relative) of it, below the
                        // ~1e-6-level difference between this accumulator and the reference's
                        // CPU projection it normalises, and the fp64 pipe of this part made the
                        // fp64 sum cost +20 % of the whole GEMM (760 vs 633 us per 720p block).
                        float sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
                        for (int c = 0; c < 4; ++c) {
                            uint32_t r[32];
                            tmem_ld32(tcol + c * 32, r);
                            tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 32; ++e) {
                                const float x = __uint_as_float(r[e]);
                                sq[e & 3] = __fmaf_rn(x, x, sq[e & 3]);
                            }
                        }
                        const float ss = __fadd_rn(__fadd_rn(sq[0], sq[1]), __fadd_rn(sq[2], sq[3]));
                        inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.f / 128.f), pk.eps)));
                    }
                    __syncwarp();  // the previous head block's stores have read the staging rows
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t r[32];
                        tmem_ld32(tcol + c * 32, r);
                        tmem_wait_ld();
                        float x[32];
#pragma unroll
                        for (int e = 0; e < 32; ++e) x[e] = __uint_as_float(r[e]);
                        if (sec < 2) {
                            const float *gm = gam + sec * 128 + c * 32;
#pragma unroll
                            for (int e = 0; e < 32; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], inv), __ldg(gm + e));
                            // pairs (2 gp, 2 gp + 1), gp = axis * 21 + pair over dims 0..125
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const int gp = c * 16 + i;
                                if (gp < 63) {
                                    const int axis = gp / 21, pr = gp - axis * 21;
                                    const int pos = axis == 0 ? mp.y : (axis == 1 ? mp.z : mp.w);
                                    const float2 cs = __ldg(pk.rope + pr * pk.max_pos + pos);
                                    const float f0 = x[2 * i], f1 = x[2 * i + 1];
                                    x[2 * i] = __fsub_rn(__fmul_rn(f0, cs.x), __fmul_rn(f1, cs.y));
                                    x[2 * i + 1] = __fadd_rn(__fmul_rn(f1, cs.x), __fmul_rn(f0, cs.y));
                                }
                            }
                        }
#pragma unroll
                        for (int v = 0; v < 4; ++v)
                            stage[lane * 16 + ((4 * c + v) ^ (lane & 7))] =
                                make_uint4(pack_bf16_h2(x[8 * v], x[8 * v + 1]), pack_bf16_h2(x[8 * v + 2], x[8 * v + 3]),
                                           pack_bf16_h2(x[8 * v + 4], x[8 * v + 5]),
                                           pack_bf16_h2(x[8 * v + 6], x[8 * v + 7]));
                    }
                    __syncwarp();
                    uint4 *outb = static_cast<uint4 *>(sec == 0 ? pk.q : (sec == 1 ? pk.k : pk.v)) +
                                  static_cast<size_t>(head) * pk.n_rows * 16;
                    const int dst_me = mp.x;
                    // video rows: two whole rows per store instruction
#pragma unroll 4
                    for (int k2 = 0; k2 < 16; ++k2) {
                        const int rr = 2 * k2 + (lane >> 4), chunk = lane & 15;
                        const int d = __shfl_sync(0xffffffffu, dst_me, rr);
                        const uint4 v4 = stage[rr * 16 + (chunk ^ (rr & 7))];
                        if (d >= 0) outb[static_cast<size_t>(d) * 16 + chunk] = v4;
                    }
                    // text rows: the same values into every window's copy of the row
                    uint32_t tmask = __ballot_sync(0xffffffffu, text);
                    while (tmask) {
                        const int rr = __ffs(tmask) - 1;
                        tmask &= tmask - 1;
                        const int l = -1 - __shfl_sync(0xffffffffu, dst_me, rr);
                        const uint4 v4 = stage[rr * 16 + ((lane & 15) ^ (rr & 7))];
                        for (int w = lane >> 4; w < pk.n_windows; w += 2)
                            outb[static_cast<size_t>(__ldg(pk.text_dst + w) + l) * 16 + (lane & 15)] = v4;
                    }
                }
            }
            if (a.row_dest) __threadfence_system();  // row stores into peers' memory, before the kernel ends
            tc_fence_before();
            if constexpr (kPair) {
                if (rank == 0)
                    mbar_arrive(BAR(B_ACCE + b));
                else
                    mbar_arrive_remote(cluster_map(BAR(B_ACCE + b), 0));  // rank 0's barrier counts both CTAs
            } else {
                mbar_arrive(BAR(B_ACCE + b));
            }
        }
        if (lane == 0) bulk_wait_group_all();  // every bulk store of this warp has landed
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    // the pair's MMAs write both CTAs' TMEM and its epilogue signals rank 0: neither CTA
    // releases TMEM or exits before the other is done
    if constexpr (kPair) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (kPair)
            tmem_dealloc_pair(tmem, kTmemCols);
        else
            tmem_dealloc(tmem, kTmemCols);
    }
#undef BAR
}

// Split-K finish of GEMM_EPI_QKV_PACK (the text rows' projection): one warp per
// (row, 128-column head block), each lane four consecutive dims; the splits are
// added in order, then the same prologue as the fused epilogue (fp32 square sum,
// here reduced across the warp; inv-RMS x gamma; RoPE pairs; bf16 rounding) and
// the packed stores (text rows into every window).
__global__ void __launch_bounds__(256) splitk_pack_kernel(const s2::GemmArgs a, int ks)
{
    const int gw = static_cast<int>((blockIdx.x * 256LL + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    const int nhb = a.N / 128;
    if (gw >= a.M * nhb) return;
    const int row = gw / nhb, col0 = (gw - row * nhb) * 128;
    const s2::PackArgs &pk = a.pk;
    const int4 mp = __ldg(pk.map + row);
    if (mp.x == -0x7fffffff) return;  // a row without a packed row
    const bool text = mp.x < 0;
    const int sec = col0 / pk.dim, head = (col0 - sec * pk.dim) >> 7;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < ks; ++sp) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(a.partial + (static_cast<size_t>(sp) * a.M + row) * a.N +
                                                                col0) + lane);
        x[0] = __fadd_rn(x[0], v.x);
        x[1] = __fadd_rn(x[1], v.y);
        x[2] = __fadd_rn(x[2], v.z);
        x[3] = __fadd_rn(x[3], v.w);
    }
    if (sec < 2) {
        float ss = __fmaf_rn(x[3], x[3], __fmaf_rn(x[2], x[2], __fmaf_rn(x[1], x[1], __fmul_rn(x[0], x[0]))));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.f / 128.f), pk.eps)));
        const float *gm = pk.gammas + (text ? 2 : 0) * 128 + sec * 128 + 4 * lane;
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = __fmul_rn(__fmul_rn(x[e], inv), __ldg(gm + e));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int gp = 2 * lane + i;
            if (gp < 63) {
                const int axis = gp / 21, pr = gp - axis * 21;
                const int pos = axis == 0 ? mp.y : (axis == 1 ? mp.z : mp.w);
                const float2 cs = __ldg(pk.rope + pr * pk.max_pos + pos);
                const float f0 = x[2 * i], f1 = x[2 * i + 1];
                x[2 * i] = __fsub_rn(__fmul_rn(f0, cs.x), __fmul_rn(f1, cs.y));
                x[2 * i + 1] = __fadd_rn(__fmul_rn(f1, cs.x), __fmul_rn(f0, cs.y));
            }
        }
    }
    const uint2 v2 = make_uint2(pack_bf16_h2(x[0], x[1]), pack_bf16_h2(x[2], x[3]));
    uint2 *outb = static_cast<uint2 *>(sec == 0 ? pk.q : (sec == 1 ? pk.k : pk.v)) +
                  static_cast<size_t>(head) * pk.n_rows * 32;
    if (!text) {
        outb[static_cast<size_t>(mp.x) * 32 + lane] = v2;
    } else {
        const int l = -1 - mp.x;
        for (int w = 0; w < pk.n_windows; ++w) outb[static_cast<size_t>(__ldg(pk.text_dst + w) + l) * 32 + lane] = v2;
    }
}

// Split-K finish: out = epilogue(sum over splits of partial[split][row][n]), the
// splits added in order (deterministic), then the same per-element arithmetic as
// gemm_kernel's epilogues. One thread per output element (per hidden element
// for SwiGLU).
__global__ void __launch_bounds__(256) splitk_finish_kernel(const s2::GemmArgs a, int ks)
{
    const bool swiglu = a.epilogue == s2::GEMM_EPI_SWIGLU_F16;
    const int n_out = swiglu ? a.N / 2 : a.N;
    const long long total = 1LL * a.M * n_out;
    const size_t slab = static_cast<size_t>(a.M) * a.N;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
        const int row = static_cast<int>(i / n_out), j = static_cast<int>(i - 1LL * row * n_out);
        auto sum = [&](int n) {
            const float *p = a.partial + static_cast<size_t>(row) * a.N + n;
            float acc = p[0];
            for (int s = 1; s < ks; ++s) acc = __fadd_rn(acc, p[s * slab]);
            return acc;
        };
        if (swiglu) {
            // hidden column j: gate at tile column (j / 128) * 256 + j % 128, "in" 128 columns on
            const int n = (j / 128) * 256 + (j % 128);
            const float g = sum(n), u = sum(n + 128);
            const float f = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
            static_cast<__half *>(a.out[0])[static_cast<size_t>(row) * n_out + j] = __float2half_rn(f);
        } else if (a.epilogue == s2::GEMM_EPI_SPLIT_F16) {
            const float f = sum(j) + (a.bias ? __ldg(a.bias + j) : 0.f);
            const int which = j / a.split, col = j - which * a.split;
            static_cast<__half *>(a.out[which])[static_cast<size_t>(row) * a.split + col] = __float2half_rn(f);
        } else {  // GEMM_EPI_GATED_RESID_F32
            const bool second = a.split_row > 0 && row >= a.split_row;
            const int rr = second ? row - a.split_row : row;
            const float *rbase = second ? a.resid2 : a.resid;
            float t = sum(j);
            if (a.bias) t = __fadd_rn(t, __ldg(a.bias + j));
            if (a.gmul) t = __fmul_rn(t, __ldg(a.gmul + j));
            const float rv = rbase ? __ldg(rbase + static_cast<size_t>(rr) * a.N + j) : 0.f;
            (second ? a.y2 : a.y)[static_cast<size_t>(rr) * a.N + j] = __fmul_rn(__fadd_rn(t, rv), a.out_scale);
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

namespace s2 {

bool make_map_2d(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_rows)
{
    auto encode = get_encode();
    if (!encode) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The convolution input [D][H][W][cp] fp16 as a 4-D map (cp innermost): box
// = 64 channels x (32 * sw) columns with element stride sw along W (32 output
// columns' inputs), one row, one frame; 128B swizzle so that four boxes fill a
// 128-row A stage exactly like one 2-D box. Out-of-range elements read zero.
bool make_map_conv(CUtensorMap *map, const void *ptr, int cp, int W, int H, int D, int sw)
{
    auto encode = get_encode();
    if (!encode) return false;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(cp), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                          static_cast<cuuint64_t>(D)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(cp) * 2, static_cast<cuuint64_t>(cp) * 2 * W,
                             static_cast<cuuint64_t>(cp) * 2 * W * H};
    cuuint32_t box[4] = {64, static_cast<cuuint32_t>(32 * sw), 1, 1};
    cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(sw), 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_2d_plain(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                       uint32_t box_inner, uint32_t box_rows)
{
    auto encode = get_encode();
    if (!encode) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_2d_plain_f32(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                           uint32_t box_inner, uint32_t box_rows)
{
    auto encode = get_encode();
    if (!encode) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

s2_status gemm_f16(cudaStream_t st, const void *A, const void *B, const GemmArgs &args)
{
    if (!A || !B || args.M <= 0 || args.N <= 0 || args.K <= 0 || args.K % kBK != 0 || !args.err)
        return set_error(S2_INVALID_ARGUMENT, "gemm: invalid arguments (M %d N %d K %d)", args.M, args.N, args.K);
    if (((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15u) != 0)
        return set_error(S2_INVALID_ARGUMENT, "gemm: operands must be 16-byte aligned");
    if (args.epilogue == GEMM_EPI_SPLIT_F16) {
        if (args.split <= 0 || args.split % 32 != 0 || args.N % 32 != 0 || (args.N + args.split - 1) / args.split > 3)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad output split %d for N %d", args.split, args.N);
        for (int i = 0; i < (args.N + args.split - 1) / args.split; ++i)
            if (!args.out[i] || (reinterpret_cast<uintptr_t>(args.out[i]) & 15u) != 0)
                return set_error(S2_INVALID_ARGUMENT, "gemm: output %d missing or not 16-byte aligned", i);
    } else if (args.epilogue == GEMM_EPI_RESID_T_F32) {
        if (!args.y || args.ldt < args.M || args.n_valid > args.N)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad channel-major output");
    } else if (args.epilogue == GEMM_EPI_SHUFFLE_F32) {
        if (!args.y || args.sh_cin <= 0 || args.sh_cin % 16 != 0 || args.sh_tr <= 0 || args.sh_h <= 0 ||
            args.sh_w <= 0 || args.N != 4 * args.sh_tr * args.sh_cin || args.M % (args.sh_h * args.sh_w) != 0 ||
            args.ldt % 2 != 0 || (reinterpret_cast<uintptr_t>(args.y) & 7u) != 0)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad space-time shuffle output");
    } else if (args.epilogue == GEMM_EPI_CONV_F32) {
        const ConvGeom &g = args.geom;
        if (!args.y || !args.conv || g.ow <= 0 || g.owp % 32 != 0 || g.owp < g.ow ||
            args.M != g.od * g.oh * g.owp || args.n_valid > args.N ||
            args.ldt < 1LL * g.od * g.oh * g.ow)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad convolution output");
    } else if (args.epilogue == GEMM_EPI_GATED_RESID_F32) {
        if ((!args.y && !args.row_dest) || args.N % 32 != 0 ||
            (args.split_row > 0 && (!args.y2 || (args.resid && !args.resid2))) ||
            ((reinterpret_cast<uintptr_t>(args.y) | reinterpret_cast<uintptr_t>(args.resid)) & 15u) != 0)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad gated-residual output");
    } else if (args.epilogue == GEMM_EPI_SWIGLU_F16) {
        if (!args.out[0] || args.N % 256 != 0 || (reinterpret_cast<uintptr_t>(args.out[0]) & 15u) != 0)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad SwiGLU output (N %d must be a multiple of 256)", args.N);
    } else if (args.epilogue == GEMM_EPI_QKV_PACK) {
        const PackArgs &pk = args.pk;
        if (pk.dim <= 0 || pk.dim % 128 != 0 || args.N != 3 * pk.dim || !pk.map || !pk.q || !pk.k || !pk.v ||
            !pk.gammas || !pk.rope || pk.n_rows <= 0 || (pk.n_windows > 0 && !pk.text_dst) ||
            ((reinterpret_cast<uintptr_t>(pk.q) | reinterpret_cast<uintptr_t>(pk.k) | reinterpret_cast<uintptr_t>(pk.v)) &
             15u) != 0)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad packed Q/K/V output");
    } else {
        return set_error(S2_UNSUPPORTED, "gemm: unknown epilogue %d", args.epilogue);
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // Tile width: 256 unless 128-wide tiles fill the persistent grid's waves
    // much better. A 128 x 128 tile runs at ~0.76-0.81 of a 128 x 256 tile's
    // rate (its QK-style MMA reads 128 B of shared memory per clock, the
    // limit), so in practice this picks 128 only for a few dozen rows (the
    // text rows of a block), where twice the CTAs cut the latency by ~15 %.
    const long long mt = (args.M + kBM - 1) / kBM;
    auto fill = [&](int bn) {
        const long long t = mt * ((args.N + bn - 1) / bn);
        const long long waves = (t + sms - 1) / sms;
        return static_cast<double>(t) / static_cast<double>(waves * sms);
    };
    int bn = args.bn;
    if (bn == 0) bn = (args.epilogue != GEMM_EPI_SWIGLU_F16 && args.N % 128 == 0 && fill(128) * 0.75 > fill(256)) ? 128 : 256;
    if ((bn != 128 && bn != 256) || (bn == 128 && args.epilogue == GEMM_EPI_SWIGLU_F16))
        return set_error(S2_INVALID_ARGUMENT, "gemm: tile width %d not available for this epilogue", bn);
    // CTA pairs (256 x 256 tiles over two SMs, a third fewer operand bytes per
    // FLOP) for 256-wide tiles: measured 2-8 % faster on the DiT block GEMMs at
    // 10-20 k rows (SwiGLU +7.6 %), but slower for short K (the VAE projections,
    // K = 512: -6 %) and a few thousand rows (-6 % on a 2.7 k-row QKV), so only
    // for M >= 4096 and K >= 1024. Needs N a multiple of 256.
    bool pair = !args.conv && (args.pair > 0 || (args.pair < 0 && bn == 256 && args.M >= 4096 && args.K >= 1024 &&
                                                  args.N % 256 == 0 && sms >= 2));
    // Split-K for a few dozen rows (the text rows of a block): the tiles alone would
    // occupy a small part of the grid while each streams its whole weight slab; with
    // the K range split, up to 8 CTAs per tile stream it together (each split keeps
    // at least 4 K slices). Not for the channel-major epilogue (the VAE, many rows).
    int ks = 1;
    const long long tiles_k = mt * ((args.N + bn - 1) / bn);
    if (args.partial && !pair && args.M <= kBM && !args.conv && !args.row_dest &&
        (args.epilogue == GEMM_EPI_SPLIT_F16 || args.epilogue == GEMM_EPI_GATED_RESID_F32 ||
         args.epilogue == GEMM_EPI_SWIGLU_F16 || args.epilogue == GEMM_EPI_QKV_PACK) &&
        tiles_k * 2 <= sms) {
        ks = static_cast<int>(std::min<long long>({8LL, sms / tiles_k, (args.K / kBK) / 4}));
        while (ks > 1 && static_cast<size_t>(ks) * args.M * args.N > args.partial_floats) --ks;
        if (ks < 2) ks = 1;
    }
    if (pair && (bn != 256 || args.N % 256 != 0 || sms < 2))
        return set_error(S2_INVALID_ARGUMENT, "gemm: CTA pairs need 256-wide tiles and N %% 256 == 0 (N %d)", args.N);
    CUtensorMap ma, mb, mo[3];
    if (args.conv) {
        // A: the convolution input [D][H][W][Cp] as a 4-D map, boxes of 64 channels x
        // 32 output columns (element stride sw along W), 128B-swizzled like the 2-D A map
        const ConvGeom &g = args.geom;
        if (g.cslices <= 0 || args.K != g.cslices * kBK * g.kd * g.kh * g.kw || g.sw <= 0 || g.sw > 4 ||
            ((reinterpret_cast<uintptr_t>(A)) & 15u) != 0)
            return set_error(S2_INVALID_ARGUMENT, "gemm: bad convolution geometry");
        if (!make_map_conv(&ma, A, g.cslices * kBK, g.in_w, g.in_h, g.in_d, g.sw))
            return set_error(S2_INFERENCE_FAILED, "gemm: convolution input tensor map failed");
    } else if (!make_map_2d(&ma, A, args.K, args.M, static_cast<uint64_t>(args.K) * 2, kBK, kBM)) {
        return set_error(S2_INFERENCE_FAILED, "gemm: cuTensorMapEncodeTiled failed");
    }
    if (
        !make_map_2d(&mb, B, args.K, args.N, static_cast<uint64_t>(args.K) * 2, kBK,
                     static_cast<uint32_t>(pair ? bn / 2 : bn)))
        return set_error(S2_INFERENCE_FAILED, "gemm: cuTensorMapEncodeTiled failed");
    // fp16 outputs: 32 x 32 store boxes, no swizzle (the unused maps repeat the first valid one)
    std::memset(mo, 0, sizeof(mo));
    if (args.epilogue == GEMM_EPI_SPLIT_F16 || args.epilogue == GEMM_EPI_SWIGLU_F16) {
        const int n_out = args.epilogue == GEMM_EPI_SWIGLU_F16 ? 1 : (args.N + args.split - 1) / args.split;
        const uint64_t cols = args.epilogue == GEMM_EPI_SWIGLU_F16 ? static_cast<uint64_t>(args.N / 2)
                                                                   : static_cast<uint64_t>(args.split);
        for (int i = 0; i < 3; ++i) {
            const void *ptr = args.out[i < n_out ? i : 0];
            if (!make_map_2d_plain(&mo[i], ptr, cols, args.M, cols * 2, 32, 32))
                return set_error(S2_INFERENCE_FAILED, "gemm: output tensor map failed");
        }
    } else if (args.epilogue == GEMM_EPI_GATED_RESID_F32 && !args.row_dest) {
        const uint64_t rows = args.split_row > 0 ? static_cast<uint64_t>(args.split_row) : static_cast<uint64_t>(args.M);
        if (!make_map_2d_plain_f32(&mo[0], args.y, args.N, rows, static_cast<uint64_t>(args.N) * 4, 32, 32))
            return set_error(S2_INFERENCE_FAILED, "gemm: output tensor map failed");
        mo[1] = mo[2] = mo[0];
    } else {
        mo[0] = mo[1] = mo[2] = ma;  // not used by the channel-major epilogue
    }
    static std::atomic<uint64_t> configured[3] = {};
    const int ci = pair ? 2 : (bn == 256 ? 0 : 1);
    const s2_status cs = once_per_device(configured[ci], [ci] {
        const cudaError_t e =
            ci == 2   ? cudaFuncSetAttribute(gemm_kernel<256, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Tile<256, true>::kSmemBytes)
            : ci == 0 ? cudaFuncSetAttribute(gemm_kernel<256, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Tile<256>::kSmemBytes)
                      : cudaFuncSetAttribute(gemm_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Tile<128>::kSmemBytes);
        if (e != cudaSuccess) return set_error(S2_INFERENCE_FAILED, "gemm: smem attribute: %s", cudaGetErrorString(e));
        return S2_OK;
    });
    if (cs != S2_OK) return cs;
    if (pair) {
        const long long tiles = ((args.M + 255) / 256) * (args.N / 256);
        const long long pairs = tiles < sms / 2 ? tiles : sms / 2;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = Tile<256, true>::kSmemBytes;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t le = cudaLaunchKernelEx(&cfg, gemm_kernel<256, true>, ma, mb, mo[0], mo[1], mo[2], args);
        if (le != cudaSuccess)
            return set_error(S2_INFERENCE_FAILED, "gemm: pair launch failed: %s", cudaGetErrorString(le));
    } else {
        GemmArgs ka = args;
        ka.ksplit = ks;
        const long long units = mt * ((args.N + bn - 1) / bn) * ks;
        const int grid = static_cast<int>(units < sms ? units : sms);
        if (bn == 256)
            gemm_kernel<256, false><<<grid, kThreads, Tile<256>::kSmemBytes, st>>>(ma, mb, mo[0], mo[1], mo[2], ka);
        else
            gemm_kernel<128, false><<<grid, kThreads, Tile<128>::kSmemBytes, st>>>(ma, mb, mo[0], mo[1], mo[2], ka);
        if (ks > 1 && args.epilogue == GEMM_EPI_QKV_PACK) {
            const long long warps = 1LL * args.M * (args.N / 128);
            splitk_pack_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(ka, ks);
            if (args.extra_launches) ++*args.extra_launches;
        } else if (ks > 1) {
            const long long outs = 1LL * args.M * (args.epilogue == GEMM_EPI_SWIGLU_F16 ? args.N / 2 : args.N);
            const int fgrid = static_cast<int>(std::min<long long>((outs + 255) / 256, 4LL * sms));
            splitk_finish_kernel<<<fgrid, 256, 0, st>>>(ka, ks);
            if (args.extra_launches) ++*args.extra_launches;
        }
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(S2_INFERENCE_FAILED, "gemm: launch failed: %s", cudaGetErrorString(e));
    return S2_OK;
}

}  // namespace s2

extern "C" s2_status s2_gemm(void *stream, const s2_gemm_desc *d, int *extra_launches)
{
    s2::clear_error();
    if (!d || !d->a || !d->b || !d->err || d->M <= 0 || d->N <= 0 || d->K <= 0 || d->K % 64 != 0)
        return s2::set_error(S2_INVALID_ARGUMENT,
                             "s2_gemm: NULL operand or error word, or bad shape (K must be a multiple of 64)");
    if (d->epilogue != S2_GEMM_SPLIT_F16 && d->epilogue != S2_GEMM_GATED_RESID_F32 && d->epilogue != S2_GEMM_SWIGLU_F16)
        return s2::set_error(S2_UNSUPPORTED, "s2_gemm: unknown epilogue %d", d->epilogue);
    if (d->epilogue == S2_GEMM_SPLIT_F16 && (d->split <= 0 || d->split % 32 != 0 || !d->out0 ||
                                             (d->N > d->split && !d->out1) || (d->N > 2 * d->split && !d->out2) ||
                                             d->N > 3 * d->split))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_gemm: split output needs split %% 32 == 0 and one buffer per part");
    s2::GemmArgs g;
    g.M = d->M;
    g.N = d->N;
    g.K = d->K;
    g.bias = d->bias;
    g.epilogue = d->epilogue;
    g.out[0] = d->out0;
    g.out[1] = d->out1;
    g.out[2] = d->out2;
    g.split = d->split;
    g.gmul = d->gmul;
    g.resid = d->resid;
    g.y = d->y;
    g.split_row = d->split_row;
    g.resid2 = d->resid2;
    g.y2 = d->y2;
    g.out_scale = d->out_scale;
    g.partial = d->workspace;
    g.partial_floats = d->workspace ? d->workspace_floats : 0;
    g.err = d->err;
    if (d->row_dest) {
        if (d->epilogue != S2_GEMM_GATED_RESID_F32 || !d->y)
            return s2::set_error(S2_INVALID_ARGUMENT, "s2_gemm: row_dest needs the gated-residual epilogue and y");
        g.row_dest = reinterpret_cast<const int2 *>(d->row_dest);
        g.dest_base[0] = d->y;
        g.y = nullptr;
    }
    int extra = 0;
    g.extra_launches = &extra;
    const s2_status s = s2::gemm_f16(static_cast<cudaStream_t>(stream), d->a, d->b, g);
    if (extra_launches) *extra_launches = extra;
    return s;
}

