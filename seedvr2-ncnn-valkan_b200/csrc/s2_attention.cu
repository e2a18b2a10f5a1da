// Varlen window attention core for sm_100a.
//
// Operands are fp16 (Q/K/V hold the reference's bf16-rounded values exactly;
// P in fp16 keeps 11 mantissa bits), accumulation is fp32 in TMEM; kF16
// selects the output type: bf16 RNE (the reference CPU rounding) or fp16.
//
// One CTA computes two 128-query tiles (256 query rows) of one (window, head):
// the window's packed sequence is its video tokens followed by the shared
// text tokens, and every query attends to all S_w = L_w + Lt keys of its own
// window (seedvr2_dit_block.cpp:1045-1079; non-causal).
//
// Roles (384 threads, one CTA per SM):
//   warps 0-3, 4-7  softmax + epilogue of Q tile 0 / Q tile 1; thread r of a
//                   warpgroup owns query row r == TMEM lane r (224 registers).
//   warp 8          TMA producer: both Q tiles once, then K and V tiles of 128
//                   keys into separate 2-stage rings (no multicast).
//   warp 9          TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 10-11     idle (they complete the control warpgroup's register
//                   hand-back; 56 registers each).
// TMEM (512 columns): S_i at 128*i (P_i is written over it, columns 32..95 of
// S_i, as the A operand of the PV MMA), O_i at 256 + 128*i.
// The tensor core ping-pongs between the two Q tiles: per key tile j it runs
// P_0(j-1) V(j-1), S_0(j) = Q_0 K(j)^T, then the same for tile 1, so one
// warpgroup's softmax overlaps the other tile's GEMMs. Because tcgen05.mma
// operations of one thread execute in issue order, the commit that announces
// S_i(j) also guarantees P_i(j-1) V(j-1) has retired: the softmax warps may
// then overwrite P_i and rescale O_i without a further wait. O is rescaled only
// when the running max grew by more than 2^8 (log2 domain); the stale max is
// otherwise kept, which is exact because O and the row sum share it.
// The epilogue divides by the row sum, rounds to the output type and scatters
// video rows to their global token row and text rows to the window's
// text-partial slab (no atomics: every output row has one writer).
//
// Every wait is bounded (s2dev::mbar_wait): on timeout the CTA raises an abort
// flag, records an error code in the caller's error word, drains its own
// in-flight MMAs and TMA loads (bounded), frees TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "s2_internal.h"
#include "s2_launch.h"
#include "s2_sm100.cuh"

using namespace s2dev;

namespace {

constexpr int kBM = s2::kTileM;                      // rows per Q tile
constexpr int kQT = s2::kQTiles;                     // Q tiles per CTA
constexpr int kBN = s2::kTileN;                      // keys per K/V tile
constexpr int kHD = S2_HEAD_DIM;
constexpr int kStages = 2;
constexpr uint32_t kBoxBytes = 128 * 64 * 2;         // one TMA box: 128 rows x 128 B (64 elements)
constexpr uint32_t kTileBytes = 2 * kBoxBytes;       // 128 rows x 128 head dims
constexpr uint32_t kOffQ = 0;                        // kQT tiles
constexpr uint32_t kOffK = kOffQ + kQT * kTileBytes; // kStages tiles
constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
constexpr uint32_t kStageBytes = 16 * 256;            // epilogue staging per softmax warp: 16 rows x 256 B
constexpr uint32_t kOffStage = kOffV + kStages * kTileBytes;
constexpr uint32_t kOffBar = kOffStage + 4 * kQT * kStageBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers/flags + 1 KB alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");

enum Bar {
    B_QFULL = 0,                   // [kQT] Q_i landed
    B_QEMPTY = B_QFULL + kQT,      // [kQT] last Q_i K^T of an item retired
    B_KFULL = B_QEMPTY + kQT,      // [kStages]
    B_KEMPTY = B_KFULL + kStages,
    B_VFULL = B_KEMPTY + kStages,
    B_VEMPTY = B_VFULL + kStages,
    B_SFULL = B_VEMPTY + kStages,  // [kQT] S_i(j) ready (and P_i(j-1) V retired)
    B_PFULL = B_SFULL + kQT,       // [kQT] P_i(j) in TMEM, O_i rescaled (128 arrivals)
    B_ODONE = B_PFULL + kQT,       // [kQT] last P_i V of an item retired
    B_OFREE = B_ODONE + kQT,       // [kQT] epilogue finished reading O_i (128 arrivals)
    B_DRAIN = B_OFREE + kQT,
    B_COUNT
};
static_assert(8 * B_COUNT + 8 <= 256, "barrier area");

// Three warpgroups: kQT softmax groups, then one control group (producer warp,
// MMA warp, two idle warps). The control group gives registers back with
// setmaxnreg so the softmax groups can hold a full 128-column S row:
// launch 384 x 168 = 64,512 = 128 x (2 x 224 + 56). The host launcher checks
// the compiled launch register count against this split before launching.
constexpr int kThreads = 128 * (kQT + 1);
constexpr int kProducerWarp = 4 * kQT;
constexpr int kMmaWarp = kProducerWarp + 1;
constexpr uint32_t kRegsSoftmax = 224, kRegsControl = 56;
static_assert(128 * (kQT * kRegsSoftmax + kRegsControl) <= 65536, "register split exceeds the register file");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColP = 32;                       // P_i offset inside S_i
constexpr uint32_t kColO = 256;

// device error codes (first failure wins)
enum : int { E_WAIT_Q = 1, E_WAIT_K = 2, E_WAIT_V = 3, E_WAIT_P = 4, E_WAIT_S = 5, E_WAIT_O = 6, E_DRAIN = 7,
             E_WAIT_OFREE = 8 };

struct AttnArgs {
    const s2_row *rows;
    const int32_t *cu;
    const int32_t *work;
    void *vid_out;
    void *txt_partial;
    int32_t *err;
    int heads;
    int text_len;
    int n_items;      // n_work * heads
    float scale_log2;
    unsigned long long wait_ns;  // limit of every bounded wait
    int skip_k;        // failure injection (tests): CTA 0's producer skips this K tile (-1: none)
};

// One (window, q-block, head) work item.
struct Item {
    int head, win, seq0, S, Lw, q0, n_q, n_kv;
};

// Item decode in two steps, so that every role issues the loads of its next
// item while it works on the current one: the work word two items ahead and
// the window bounds one item ahead (two dependent global loads per item would
// otherwise stall each role at every item boundary).
struct ItemPrefetch {
    int t, w, c0, c1;
};

__device__ __forceinline__ int load_work(const AttnArgs &a, int t)
{
    return t < a.n_items ? __ldg(a.work + t / a.heads) : 0;
}

__device__ __forceinline__ ItemPrefetch prefetch_item(const AttnArgs &a, int t, int w)
{
    ItemPrefetch p{t, w, 0, 0};
    if (t < a.n_items) {
        p.c0 = __ldg(a.cu + (w >> 16));
        p.c1 = __ldg(a.cu + (w >> 16) + 1);
    }
    return p;
}

__device__ __forceinline__ Item finish_item(const AttnArgs &a, const ItemPrefetch &p)
{
    Item it;
    it.head = p.t % a.heads;
    it.win = p.w >> 16;
    const int qb = p.w & 0xFFFF;
    it.seq0 = p.c0;
    it.S = p.c1 - p.c0;
    it.Lw = it.S - a.text_len;
    it.q0 = qb * (kQT * kBM);
    it.n_q = min(kQT, (it.S - it.q0 + kBM - 1) / kBM);
    it.n_kv = (it.S + kBN - 1) / kBN;
    return it;
}

// 3-input max (one ALU instruction for two new values)
__device__ __forceinline__ float max3f(float a, float b, float c)
{
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ uint32_t pack_p(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Output element pair in the mode's type: kOut = S2_MODE_BF16_REF (bf16 RNE),
// S2_MODE_F16 (fp16 RNE) or S2_MODE_BF16_F16 (bf16 RNE, then stored as fp16:
// exact in fp16's normal range).
template <int kOut>
__device__ __forceinline__ uint32_t pack_out(float a, float b)
{
    if constexpr (kOut == S2_MODE_F16) {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    } else if constexpr (kOut == S2_MODE_BF16_F16) {
        const __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
        const __half2 h = __floats2half2_rn(__low2float(r), __high2float(r));
        return *reinterpret_cast<const uint32_t *>(&h);
    } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    }
}

// Wait that ignores the abort flag (used only to drain in-flight async work).
__device__ __forceinline__ bool wait_drain(uint32_t bar, uint32_t parity, int *err, uint64_t timeout_ns)
{
    int dummy = 0;
    return mbar_wait(bar, parity, &dummy, err, E_DRAIN, timeout_ns);
}

// Persistent: CTA b processes items b, b + gridDim.x, ... of the cost-ordered
// list; every barrier's phase counter runs on across items.
template <int kOut>
__global__ void __launch_bounds__(kThreads, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    const uint32_t sQ = base + kOffQ, sK = base + kOffK, sV = base + kOffV;
    const uint32_t bar0 = base + kOffBar;
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + kOffBar + 8 * B_COUNT);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kOffBar + 8 * B_COUNT + 4);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < B_COUNT; ++i) {
            const bool wg_arrive = (i >= B_PFULL && i < B_PFULL + kQT) || (i >= B_OFREE && i < B_OFREE + kQT);
            mbar_init(BAR(i), wg_arrive ? 128u : 1u);
        }
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= kProducerWarp) {
      regs_dec<kRegsControl>();
      if (warp == kProducerWarp) {
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            uint32_t nq[kQT] = {0, 0};   // Q_i loads issued
            uint32_t kv = 0;             // K/V tiles issued (ring position)
            uint32_t k_skipped = 0xffffffffu;  // ring position of a K load left out (failure injection)
            bool ok = true;
            ItemPrefetch pf_next = prefetch_item(a, blockIdx.x, load_work(a, blockIdx.x));
            int w_next = load_work(a, blockIdx.x + gridDim.x);
            for (int t = blockIdx.x; ok && t < a.n_items; t += gridDim.x) {
                const Item it = finish_item(a, pf_next);
                pf_next = prefetch_item(a, t + gridDim.x, w_next);
                w_next = load_work(a, t + 2 * gridDim.x);
                for (int i = 0; i < it.n_q; ++i) {
                    if (!(ok = mbar_wait(BAR(B_QEMPTY + i), (nq[i] & 1u) ^ 1u, abort, a.err, E_WAIT_Q, a.wait_ns))) break;
                    const int row_q = it.seq0 + it.q0 + i * kBM;
                    mbar_arrive_expect_tx(BAR(B_QFULL + i), kTileBytes);
                    tma_load_3d(sQ + i * kTileBytes, &tmQ, BAR(B_QFULL + i), 0, row_q, it.head);
                    tma_load_3d(sQ + i * kTileBytes + kBoxBytes, &tmQ, BAR(B_QFULL + i), 64, row_q, it.head);
                    nq[i]++;
                }
                for (int j = 0; ok && j < it.n_kv; ++j, ++kv) {
                    const uint32_t s = kv & 1u, u = kv >> 1;
                    const int row_kv = it.seq0 + j * kBN;
                    if (!(ok = mbar_wait(BAR(B_KEMPTY + s), (u & 1u) ^ 1u, abort, a.err, E_WAIT_K, a.wait_ns))) break;
                    if (blockIdx.x == 0 && static_cast<int>(kv) == a.skip_k) {
                        k_skipped = kv;  // injected failure: this K tile never arrives
                    } else {
                        mbar_arrive_expect_tx(BAR(B_KFULL + s), kTileBytes);
                        tma_load_3d(sK + s * kTileBytes, &tmK, BAR(B_KFULL + s), 0, row_kv, it.head);
                        tma_load_3d(sK + s * kTileBytes + kBoxBytes, &tmK, BAR(B_KFULL + s), 64, row_kv, it.head);
                    }
                    if (!(ok = mbar_wait(BAR(B_VEMPTY + s), (u & 1u) ^ 1u, abort, a.err, E_WAIT_V, a.wait_ns))) {
                        ++kv;  // the K half of this tile is in flight
                        break;
                    }
                    mbar_arrive_expect_tx(BAR(B_VFULL + s), kTileBytes);
                    tma_load_3d(sV + s * kTileBytes, &tmV, BAR(B_VFULL + s), 0, row_kv, it.head);
                    tma_load_3d(sV + s * kTileBytes + kBoxBytes, &tmV, BAR(B_VFULL + s), 64, row_kv, it.head);
                }
            }
            // No load may still be landing in shared memory when the CTA exits:
            // wait for the last load issued into every buffer.
            for (int i = 0; i < kQT; ++i)
                if (nq[i]) wait_drain(BAR(B_QFULL + i), (nq[i] - 1) & 1u, a.err, a.wait_ns);
            for (uint32_t s = 0; s < kStages; ++s) {
                if (kv > s) {
                    const uint32_t last = (kv - 1 - s) / kStages;  // use count - 1 of stage s
                    if (s + last * kStages != k_skipped) wait_drain(BAR(B_KFULL + s), last & 1u, a.err, a.wait_ns);
                    wait_drain(BAR(B_VFULL + s), last & 1u, a.err, a.wait_ns);
                }
            }
        }
      } else if (warp == kMmaWarp) {
        if (lane == 0) {
            const uint32_t id_qk = idesc_f16(0u, kBN, 0);  // f16 x f16 -> f32, K-major A and B
            const uint32_t id_pv = idesc_f16(0u, kHD, 1);  // A = P from TMEM, B = V MN-major
            // Each 128x128x128 tile is 8 straight-line K=16 MMAs (s2_sm100.cuh):
            // any per-MMA loop or branch overhead in this thread shows up
            // directly as tensor-core idle time.
            const uint64_t dq0 = smem_desc_sw128(sQ, 16, 1024), dk0 = smem_desc_sw128(sK, 16, 1024);
            const uint64_t dv0 = smem_desc_sw128(sV, kBoxBytes, 1024);
            // S_i = Q_i K^T (K tile in ring stage s) into S_i's columns
            auto qk = [&](int i, uint32_t s) {
                mma_tile_ss_k128(tmem + static_cast<uint32_t>(i) * 128u,
                                 dq0 + static_cast<uint64_t>(i) * (kTileBytes >> 4),
                                 dk0 + static_cast<uint64_t>(s) * (kTileBytes >> 4), id_qk, 0u);
            };
            // O_i (+)= P_i V (V tile in ring stage s), P_i read from TMEM
            auto pv = [&](int i, uint32_t s, uint32_t acc) {
                mma_tile_ts_k128(tmem + kColO + static_cast<uint32_t>(i) * 128u,
                                 tmem + static_cast<uint32_t>(i) * 128u + kColP,
                                 dv0 + static_cast<uint64_t>(s) * (kTileBytes >> 4), id_pv, acc);
            };
            uint32_t nq[kQT] = {0, 0};   // items seen per Q tile (Q_FULL / Q_EMPTY / O phases)
            uint32_t np[kQT] = {0, 0};   // P_i tiles consumed (P_FULL phases)
            uint32_t kv = 0;             // K/V tiles consumed
            bool ok = true;
            ItemPrefetch pf_next = prefetch_item(a, blockIdx.x, load_work(a, blockIdx.x));
            int w_next = load_work(a, blockIdx.x + gridDim.x);
            for (int t = blockIdx.x; ok && t < a.n_items; t += gridDim.x) {
                const Item it = finish_item(a, pf_next);
                pf_next = prefetch_item(a, t + gridDim.x, w_next);
                w_next = load_work(a, t + 2 * gridDim.x);
                // S_i(0)
                const uint32_t s0 = kv & 1u;
                ok = mbar_wait(BAR(B_KFULL + s0), (kv >> 1) & 1u, abort, a.err, E_WAIT_K, a.wait_ns);
                for (int i = 0; ok && i < it.n_q; ++i) {
                    if (!(ok = mbar_wait(BAR(B_QFULL + i), nq[i] & 1u, abort, a.err, E_WAIT_Q, a.wait_ns))) break;
                    tc_fence_after();
                    qk(i, s0);
                    mma_commit(BAR(B_SFULL + i));
                    if (it.n_kv == 1) mma_commit(BAR(B_QEMPTY + i));
                }
                if (!ok) break;
                mma_commit(BAR(B_KEMPTY + s0));
                for (int j = 0; ok && j < it.n_kv; ++j) {
                    const uint32_t s = (kv + j) & 1u, sn = (kv + j + 1) & 1u;
                    const bool more = j + 1 < it.n_kv;
                    ok = mbar_wait(BAR(B_VFULL + s), ((kv + j) >> 1) & 1u, abort, a.err, E_WAIT_V, a.wait_ns);
                    bool k_next = false;
                    for (int i = 0; ok && i < it.n_q; ++i) {
                        if (!(ok = mbar_wait(BAR(B_PFULL + i), np[i] & 1u, abort, a.err, E_WAIT_P, a.wait_ns))) break;
                        np[i]++;
                        // the previous item's epilogue must have read O_i before it is overwritten
                        if (j == 0 && !(ok = mbar_wait(BAR(B_OFREE + i), (nq[i] & 1u) ^ 1u, abort, a.err,
                                                       E_WAIT_OFREE, a.wait_ns)))
                            break;
                        tc_fence_after();
                        pv(i, s, j > 0 ? 1u : 0u);
                        if (more) {
                            if (!k_next) {
                                if (!(ok = mbar_wait(BAR(B_KFULL + sn), ((kv + j + 1) >> 1) & 1u, abort, a.err,
                                                     E_WAIT_K, a.wait_ns)))
                                    break;
                                tc_fence_after();
                                k_next = true;
                            }
                            qk(i, sn);  // overwrites S_i/P_i after P_i V: in-order tcgen05 issue
                            mma_commit(BAR(B_SFULL + i));
                            if (j + 2 == it.n_kv) mma_commit(BAR(B_QEMPTY + i));
                        } else {
                            mma_commit(BAR(B_ODONE + i));
                        }
                    }
                    if (!ok) break;
                    mma_commit(BAR(B_VEMPTY + s));
                    if (more) mma_commit(BAR(B_KEMPTY + sn));
                }
                for (int i = 0; i < it.n_q; ++i) nq[i]++;
                kv += it.n_kv;
            }
            // All issued MMAs must retire before TMEM is released.
            mma_commit(BAR(B_DRAIN));
            wait_drain(BAR(B_DRAIN), 0, a.err, a.wait_ns);
        }
      }
    } else {
        regs_inc<kRegsSoftmax>();
        // ---- softmax warpgroups: thread r of group g <-> query row q0 + g*128 + r <-> TMEM lane r ----
        const int g = warp >> 2;
        const int r = threadIdx.x & 127;
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t scol = tmem + lane_off + static_cast<uint32_t>(g) * 128u;
        const uint32_t pcol = scol + kColP;
        const uint32_t ocol = tmem + lane_off + kColO + static_cast<uint32_t>(g) * 128u;
        const float c = a.scale_log2;
        const int dim = a.heads * kHD;
        uint32_t ns = 0, no = 0;  // S_FULL phases consumed, items finished
        bool ok = true;
        ItemPrefetch pf_next = prefetch_item(a, blockIdx.x, load_work(a, blockIdx.x));
        int w_next = load_work(a, blockIdx.x + gridDim.x);
        for (int t = blockIdx.x; ok && t < a.n_items; t += gridDim.x) {
            const Item it = finish_item(a, pf_next);
            pf_next = prefetch_item(a, t + gridDim.x, w_next);
            w_next = load_work(a, t + 2 * gridDim.x);
            if (g >= it.n_q) continue;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < it.n_kv; ++j) {
                ok = mbar_wait(BAR(B_SFULL + g), ns & 1u, abort, a.err, E_WAIT_S, a.wait_ns);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                ns++;
                tc_fence_after();
                uint32_t x[4][32];
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) tmem_ld32(scol + cc * 32, x[cc]);
                tmem_wait_ld();
                const int valid = min(it.S - j * kBN, kBN);
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
                // O_i is stable here: P_i V(j-1) retired before S_i(j) was announced.
                if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t o[32];
                        tmem_ld32(ocol + cc * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(ocol + cc * 32, o);
                    }
                }
                // packed fp32x2 FMA/add halve the instruction count of the exp loop
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
                        pk[i] = pack_p(p2.x, p2.y);
                    }
                    tmem_st16(pcol + cc * 16, pk);
                }
                tmem_wait_st();
                l = l * alpha + (((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y)) + ((rs2[2].x + rs2[2].y) + (rs2[3].x + rs2[3].y)));
                m = m_use;
                tc_fence_before();
                mbar_arrive(BAR(B_PFULL + g));
            }
            if (!ok) break;
            ok = mbar_wait(BAR(B_ODONE + g), no & 1u, abort, a.err, E_WAIT_O, a.wait_ns);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            no++;
            tc_fence_after();
            uint32_t o[4][32];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) tmem_ld32(ocol + cc * 32, o[cc]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(BAR(B_OFREE + g));  // O_i may be overwritten by the next item
            const int qrow = it.q0 + g * kBM + r;
            uint16_t *dst_row = nullptr;
            if (qrow < it.S) {
                if (qrow < it.Lw)
                    dst_row = static_cast<uint16_t *>(a.vid_out) +
                              static_cast<size_t>(a.rows[it.seq0 + qrow].src) * dim + it.head * kHD;
                else
                    dst_row = static_cast<uint16_t *>(a.txt_partial) +
                              (static_cast<size_t>(it.win) * a.text_len + (qrow - it.Lw)) * dim + it.head * kHD;
            }
            const float inv = 1.f / l;
            const float2 inv2 = make_float2(inv, inv);
            uint4 packed[16];
#pragma unroll
            for (int c16 = 0; c16 < 16; ++c16) {
                const int cc = c16 >> 2, i0 = (c16 & 3) * 8;
                uint32_t w4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 v = __fmul2_rn(
                        make_float2(__uint_as_float(o[cc][i0 + 2 * e]), __uint_as_float(o[cc][i0 + 2 * e + 1])), inv2);
                    w4[e] = pack_out<kOut>(v.x, v.y);
                }
                packed[c16] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
            // Output rows go out through a per-warp shared staging buffer, 16 rows at a
            // time, so that each warp store instruction writes two whole 256-byte rows
            // instead of 32 scattered 16-byte pieces. (Per-row bulk copies from the same
            // buffer were measured 5 % slower: hundreds of thousands of 256-byte bulk
            // operations per launch compete with the Q/K/V tile loads for the TMA unit.)
            uint4 *stage = reinterpret_cast<uint4 *>(gbase + kOffStage + static_cast<uint32_t>(warp) * kStageBytes);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int srow = lane - 16 * half;  // this lane's row inside the staged half
                if (srow >= 0 && srow < 16) {
#pragma unroll
                    for (int c16 = 0; c16 < 16; ++c16) stage[srow * 16 + (c16 ^ (srow & 7))] = packed[c16];
                }
                __syncwarp();
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int row = 2 * k + (lane >> 4), chunk = lane & 15;
                    const unsigned long long pa =
                        __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst_row), 16 * half + row);
                    const uint4 v4 = stage[row * 16 + (chunk ^ (row & 7))];
                    if (pa) reinterpret_cast<uint4 *>(pa)[chunk] = v4;
                }
                __syncwarp();
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
#undef BAR
}

// ---- host side ---------------------------------------------------------------

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

// [heads][n_rows][128] 16-bit tensor; box = 64 dims x 128 rows x 1 head, 128B swizzle.
bool make_map(CUtensorMap *map, const void *ptr, int heads, int n_rows)
{
    auto encode = get_encode();
    if (!encode) return false;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHD), static_cast<cuuint64_t>(n_rows),
                          static_cast<cuuint64_t>(heads)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHD) * 2, static_cast<cuuint64_t>(n_rows) * kHD * 2};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kBN), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r =
        encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
               const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int kOut>
s2_status launch(cudaStream_t st, const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                 const AttnArgs &args, int grid)
{
    static std::atomic<uint64_t> configured{0};
    const s2_status cs = s2::once_per_device(configured, [] {
        const cudaError_t e = cudaFuncSetAttribute(window_attention_kernel<kOut>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_window_attention: smem attribute: %s", cudaGetErrorString(e));
        // setmaxnreg.inc waits until the block's launch registers can cover the
        // softmax groups' request: refuse to launch a build whose register
        // count at launch is smaller than the split assumes.
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, window_attention_kernel<kOut>) != cudaSuccess ||
            static_cast<long long>(fa.numRegs) * kThreads < 128LL * (kQT * kRegsSoftmax + kRegsControl))
            return s2::set_error(S2_INFERENCE_FAILED,
                                 "s2_window_attention: kernel built with %d registers/thread, register split needs %d",
                                 fa.numRegs, (128 * (kQT * kRegsSoftmax + kRegsControl) + kThreads - 1) / kThreads);
        return S2_OK;
    });
    if (cs != S2_OK) return cs;
    window_attention_kernel<kOut><<<grid, kThreads, kSmemBytes, st>>>(mq, mk, mv, args);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_window_attention: launch failed: %s", cudaGetErrorString(e));
    return S2_OK;
}

}  // namespace

extern "C" s2_status s2_window_attention(void *stream, s2_mode mode, const void *q, const void *k, const void *v,
                                         int heads, int n_rows, const int32_t *cu_seqlens, int n_windows,
                                         int text_len, const s2_row *rows, const int32_t *work, int n_work,
                                         void *vid_out, void *txt_partial, int32_t *err)
{
    if (!q || !k || !v || heads <= 0 || n_rows <= 0 || !cu_seqlens || n_windows <= 0 || text_len < 0 || !rows ||
        !work || n_work <= 0 || !vid_out || (text_len > 0 && !txt_partial) || !err)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_window_attention: invalid arguments");
    if (mode != S2_MODE_BF16_REF && mode != S2_MODE_F16 && mode != S2_MODE_BF16_F16)
        return s2::set_error(S2_UNSUPPORTED, "s2_window_attention: unknown mode %d", (int)mode);
    if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
          reinterpret_cast<uintptr_t>(vid_out) | reinterpret_cast<uintptr_t>(txt_partial)) & 15u) != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_window_attention: buffers must be 16-byte aligned");
    const long long n_items = 1LL * n_work * heads;
    if (n_items > 0x7fffffffLL) return s2::set_error(S2_INVALID_ARGUMENT, "s2_window_attention: too many work items");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long grid = n_items < sms ? n_items : sms;  // persistent: one CTA per SM
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, q, heads, n_rows) || !make_map(&mk, k, heads, n_rows) || !make_map(&mv, v, heads, n_rows))
        return s2::set_error(S2_INFERENCE_FAILED, "s2_window_attention: cuTensorMapEncodeTiled failed");
    AttnArgs args;
    args.rows = rows;
    args.cu = cu_seqlens;
    args.work = work;
    args.vid_out = vid_out;
    args.txt_partial = txt_partial;
    args.err = err;
    args.heads = heads;
    args.text_len = text_len;
    args.n_items = static_cast<int>(n_items);
    args.scale_log2 = static_cast<float>(1.4426950408889634 / 11.313708498984761);  // log2(e) / sqrt(128)
    s2::take_attention_fault(&args.skip_k, &args.wait_ns);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (mode) {
    case S2_MODE_F16: return launch<S2_MODE_F16>(st, mq, mk, mv, args, static_cast<int>(grid));
    case S2_MODE_BF16_F16: return launch<S2_MODE_BF16_F16>(st, mq, mk, mv, args, static_cast<int>(grid));
    default: return launch<S2_MODE_BF16_REF>(st, mq, mk, mv, args, static_cast<int>(grid));
    }
}
