// Varlen window attention core for sm_100a.
//
// Operands are fp16 (Q/K/V hold the reference's bf16-rounded values exactly;
// P in fp16 keeps 11 mantissa bits), accumulation is fp32 in TMEM; kF16
// selects the output type: bf16 RNE (the reference CPU rounding) or fp16.
//
// One CTA computes one 128-query tile of one (window, head): the window's
// packed sequence is its video tokens followed by the shared text tokens, and
// every query attends to all S_w = L_w + Lt keys of its own window
// (seedvr2_dit_block.cpp:1045-1079; non-causal).
//
// Roles (192 threads, one CTA per SM):
//   warps 0-3  softmax + epilogue. Thread r owns query row r == TMEM lane r.
//   warp 4     TMA producer: Q once, then K/V tiles of 128 keys into a
//              2-stage ring (separate K and V stages so a K stage frees as
//              soon as its QK^T MMA retires).
//   warp 5     TMEM allocator + single-thread tcgen05.mma issuer.
// TMEM (512 columns): S double buffer at 0 and 128, O accumulator at 256.
// Per key tile j: S_j = Q K_j^T (M=N=K=128, 8 MMAs of K=16) -> softmax warps
// read S_j with tcgen05.ld, update the running max (log2 domain), write
// P_j = exp2(S_j*c - m) as fp16 into a 128B-swizzled shared tile and
// rescale O in TMEM only when the max grew by more than 2^8 (the stale max is
// otherwise kept, which is exact because O and the row sum share it); then
// O += P_j V_j (V as an MN-major operand). S_{j+2} is issued right after
// P_j V_j so the tensor core works on the next tile while the softmax warps
// finish this one. The epilogue divides by the row sum, rounds to the output
// type and scatters video rows to their global token row and text rows to the
// window's text-partial slab (no atomics: every output row has one writer).
//
// Every wait is bounded (s2dev::mbar_wait): on timeout the CTA raises an abort
// flag, records an error code in the caller's error word, drains its own
// in-flight MMAs and TMA loads (bounded), frees TMEM and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "s2_internal.h"
#include "s2_sm100.cuh"

using namespace s2dev;

namespace {

constexpr int kBM = s2::kTileM;
constexpr int kBN = s2::kTileN;
constexpr int kHD = S2_HEAD_DIM;
constexpr int kStages = 2;
constexpr uint32_t kBoxBytes = 128 * 64 * 2;     // one TMA box: 128 rows x 128 B (64 elements)
constexpr uint32_t kTileBytes = 2 * kBoxBytes;   // 128 rows x 128 head dims
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kTileBytes;
constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
constexpr uint32_t kOffP = kOffV + kStages * kTileBytes;
constexpr uint32_t kOffBar = kOffP + kTileBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers/flags + 1 KB alignment slack

enum Bar { B_Q = 0, B_KFULL = 1, B_KEMPTY = 3, B_VFULL = 5, B_VEMPTY = 7, B_SFULL = 9, B_PFULL = 11, B_ODONE = 12,
           B_DRAIN = 13, B_COUNT = 14 };

constexpr int kThreads = 192;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;

// device error codes (first failure wins)
enum : int { E_WAIT_Q = 1, E_WAIT_K = 2, E_WAIT_V = 3, E_WAIT_P = 4, E_WAIT_S = 5, E_WAIT_O = 6, E_DRAIN = 7 };

struct AttnArgs {
    const s2_row *rows;
    const int32_t *cu;
    const int32_t *work;
    void *vid_out;
    void *txt_partial;
    int32_t *err;
    int heads;
    int text_len;
    float scale_log2;
};

__device__ __forceinline__ uint32_t pack_p(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

template <bool kF16>
__device__ __forceinline__ uint32_t pack_out(float a, float b)
{
    if constexpr (kF16) {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    }
}

__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int *abort, int *err, int code)
{
    return mbar_wait(bar, parity, abort, err, code);
}

// Wait that ignores the abort flag (used only to drain in-flight async work).
__device__ __forceinline__ bool wait_drain(uint32_t bar, uint32_t parity, int *err)
{
    int dummy = 0;
    return mbar_wait(bar, parity, &dummy, err, E_DRAIN);
}

template <bool kF16>
__global__ void __launch_bounds__(kThreads, 1)
    window_attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (base - raw);
    const uint32_t sQ = base + kOffQ, sK = base + kOffK, sV = base + kOffV, sP = base + kOffP;
    const uint32_t bar0 = base + kOffBar;
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + kOffBar + 8 * B_COUNT);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kOffBar + 8 * B_COUNT + 4);
#define BAR(i) (bar0 + 8u * static_cast<uint32_t>(i))

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x % a.heads;
    const int item = a.work[blockIdx.x / a.heads];
    const int win = item >> 16, qt = item & 0xFFFF;
    const int seq0 = a.cu[win];
    const int S = a.cu[win + 1] - seq0;
    const int Lw = S - a.text_len;
    const int q0 = qt * kBM;
    const int n_kv = (S + kBN - 1) / kBN;

    if (threadIdx.x == 0) {
        for (int i = 0; i < B_COUNT; ++i) mbar_init(BAR(i), i == B_PFULL ? 128u : 1u);
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

    if (warp == kProducerWarp) {
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            int issued_k[kStages] = {0, 0}, issued_v[kStages] = {0, 0};
            const int row_q = seq0 + q0;
            mbar_arrive_expect_tx(BAR(B_Q), kTileBytes);
            tma_load_3d(sQ, &tmQ, BAR(B_Q), 0, row_q, head);
            tma_load_3d(sQ + kBoxBytes, &tmQ, BAR(B_Q), 64, row_q, head);
            for (int j = 0; j < n_kv; ++j) {
                const int s = j & 1;
                const uint32_t u = static_cast<uint32_t>(j >> 1);
                const int row_kv = seq0 + j * kBN;
                if (!wait_or_abort(BAR(B_KEMPTY + s), (u & 1u) ^ 1u, abort, a.err, E_WAIT_K)) break;
                mbar_arrive_expect_tx(BAR(B_KFULL + s), kTileBytes);
                tma_load_3d(sK + s * kTileBytes, &tmK, BAR(B_KFULL + s), 0, row_kv, head);
                tma_load_3d(sK + s * kTileBytes + kBoxBytes, &tmK, BAR(B_KFULL + s), 64, row_kv, head);
                issued_k[s]++;
                if (!wait_or_abort(BAR(B_VEMPTY + s), (u & 1u) ^ 1u, abort, a.err, E_WAIT_V)) break;
                mbar_arrive_expect_tx(BAR(B_VFULL + s), kTileBytes);
                tma_load_3d(sV + s * kTileBytes, &tmV, BAR(B_VFULL + s), 0, row_kv, head);
                tma_load_3d(sV + s * kTileBytes + kBoxBytes, &tmV, BAR(B_VFULL + s), 64, row_kv, head);
                issued_v[s]++;
            }
            // No load may still be landing in shared memory when the CTA exits.
            wait_drain(BAR(B_Q), 0, a.err);
            for (int s = 0; s < kStages; ++s) {
                if (issued_k[s]) wait_drain(BAR(B_KFULL + s), static_cast<uint32_t>(issued_k[s] - 1) & 1u, a.err);
                if (issued_v[s]) wait_drain(BAR(B_VFULL + s), static_cast<uint32_t>(issued_v[s] - 1) & 1u, a.err);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            const uint32_t id_qk = idesc_f16(0u, kBN, 0);  // f16 x f16 -> f32
            const uint32_t id_pv = idesc_f16(0u, kHD, 1);
            bool ok = wait_or_abort(BAR(B_Q), 0, abort, a.err, E_WAIT_Q);
            if (ok) tc_fence_after();
            auto issue_qk = [&](int j) -> bool {
                const int s = j & 1;
                if (!wait_or_abort(BAR(B_KFULL + s), static_cast<uint32_t>(j >> 1) & 1u, abort, a.err, E_WAIT_K))
                    return false;
                tc_fence_after();
                const uint32_t kb = sK + s * kTileBytes;
                const uint32_t d = tmem + static_cast<uint32_t>(s) * kBN;
#pragma unroll
                for (int ks = 0; ks < kHD / 16; ++ks) {
                    const uint32_t off = static_cast<uint32_t>(ks >> 2) * kBoxBytes + static_cast<uint32_t>(ks & 3) * 32u;
                    mma_f16_ss(d, smem_desc_sw128(sQ + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), id_qk,
                               ks > 0 ? 1u : 0u);
                }
                mma_commit(BAR(B_SFULL + s));
                mma_commit(BAR(B_KEMPTY + s));
                return true;
            };
            if (ok) ok = issue_qk(0);
            if (ok && n_kv > 1) ok = issue_qk(1);
            for (int j = 0; ok && j < n_kv; ++j) {
                const int s = j & 1;
                if (!wait_or_abort(BAR(B_PFULL), static_cast<uint32_t>(j) & 1u, abort, a.err, E_WAIT_P)) break;
                if (!wait_or_abort(BAR(B_VFULL + s), static_cast<uint32_t>(j >> 1) & 1u, abort, a.err, E_WAIT_V))
                    break;
                tc_fence_after();
                const uint32_t vb = sV + s * kTileBytes;
#pragma unroll
                for (int ks = 0; ks < kBN / 16; ++ks) {
                    const uint32_t a_off = static_cast<uint32_t>(ks >> 2) * kBoxBytes + static_cast<uint32_t>(ks & 3) * 32u;
                    mma_f16_ss(tmem + kColO, smem_desc_sw128(sP + a_off, 16, 1024),
                               smem_desc_sw128(vb + static_cast<uint32_t>(ks) * 2048u, kBoxBytes, 1024), id_pv,
                               (j > 0 || ks > 0) ? 1u : 0u);
                }
                mma_commit(BAR(B_ODONE));
                mma_commit(BAR(B_VEMPTY + s));
                if (j + 2 < n_kv) ok = issue_qk(j + 2);
            }
            // All issued MMAs must retire before TMEM is released.
            mma_commit(BAR(B_DRAIN));
            wait_drain(BAR(B_DRAIN), 0, a.err);
        }
    } else {
        // ---- softmax warps: thread r <-> query row r <-> TMEM lane r ----
        const int r = threadIdx.x;
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        const float c = a.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kv; ++j) {
            const int s = j & 1;
            ok = wait_or_abort(BAR(B_SFULL + s), static_cast<uint32_t>(j >> 1) & 1u, abort, a.err, E_WAIT_S);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            uint32_t x[4][32];
            const uint32_t scol = tmem + lane_off + static_cast<uint32_t>(s) * kBN;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) tmem_ld32(scol + cc * 32, x[cc]);
            tmem_wait_ld();
            const int valid = min(S - j * kBN, kBN);
            float mx = -INFINITY;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float sv = (cc * 32 + i) < valid ? __uint_as_float(x[cc][i]) : -INFINITY;
                    x[cc][i] = __float_as_uint(sv);
                    mx = fmaxf(mx, sv);
                }
            const float cand = mx * c;
            float m_use = m, alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m_use = cand;
            } else if (cand > m + 8.f) {
                m_use = cand;
                alpha = ex2_approx(m - cand);
                rescale = true;
            }
            float rs = 0.f;
            uint32_t pk[4][16];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = ex2_approx(fmaf(__uint_as_float(x[cc][2 * i]), c, -m_use));
                    const float p1 = ex2_approx(fmaf(__uint_as_float(x[cc][2 * i + 1]), c, -m_use));
                    rs += p0 + p1;
                    pk[cc][i] = pack_p(p0, p1);
                }
            if (j > 0) {
                ok = wait_or_abort(BAR(B_ODONE), static_cast<uint32_t>(j - 1) & 1u, abort, a.err, E_WAIT_O);
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                tc_fence_after();
            }
            if (__any_sync(0xffffffffu, rescale)) {
                const uint32_t ocol = tmem + lane_off + kColO;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t o[32];
                    tmem_ld32(ocol + cc * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(ocol + cc * 32, o);
                }
                tmem_wait_st();
            }
            l = l * alpha + rs;
            m = m_use;
            // P row r -> 128B-swizzled K-major tile (two 64-key blocks).
#pragma unroll
            for (int c16 = 0; c16 < 16; ++c16) {
                const uint32_t blk = static_cast<uint32_t>(c16 >> 3), chunk = static_cast<uint32_t>(c16 & 7);
                const uint32_t addr = sP + blk * kBoxBytes + static_cast<uint32_t>(r) * 128u +
                                      ((chunk ^ static_cast<uint32_t>(r & 7)) << 4);
                const int cc = c16 >> 2, i0 = (c16 & 3) * 4;
                st_shared_v4(addr, pk[cc][i0], pk[cc][i0 + 1], pk[cc][i0 + 2], pk[cc][i0 + 3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(BAR(B_PFULL));
        }
        if (ok) {
            ok = wait_or_abort(BAR(B_ODONE), static_cast<uint32_t>(n_kv - 1) & 1u, abort, a.err, E_WAIT_O);
            ok = __all_sync(0xffffffffu, ok);
        }
        if (ok) {
            tc_fence_after();
            uint32_t o[4][32];
            const uint32_t ocol = tmem + lane_off + kColO;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) tmem_ld32(ocol + cc * 32, o[cc]);
            tmem_wait_ld();
            const int qrow = q0 + r;
            if (qrow < S) {
                const float inv = 1.f / l;
                const int dim = a.heads * kHD;
                uint4 *dst;
                if (qrow < Lw) {
                    const int g = a.rows[seq0 + qrow].src;
                    dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.vid_out) + static_cast<size_t>(g) * dim +
                                                    head * kHD);
                } else {
                    dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.txt_partial) +
                                                    (static_cast<size_t>(win) * a.text_len + (qrow - Lw)) * dim +
                                                    head * kHD);
                }
#pragma unroll
                for (int c16 = 0; c16 < 16; ++c16) {
                    const int cc = c16 >> 2, i0 = (c16 & 3) * 8;
                    uint4 w;
                    w.x = pack_out<kF16>(__uint_as_float(o[cc][i0 + 0]) * inv, __uint_as_float(o[cc][i0 + 1]) * inv);
                    w.y = pack_out<kF16>(__uint_as_float(o[cc][i0 + 2]) * inv, __uint_as_float(o[cc][i0 + 3]) * inv);
                    w.z = pack_out<kF16>(__uint_as_float(o[cc][i0 + 4]) * inv, __uint_as_float(o[cc][i0 + 5]) * inv);
                    w.w = pack_out<kF16>(__uint_as_float(o[cc][i0 + 6]) * inv, __uint_as_float(o[cc][i0 + 7]) * inv);
                    dst[c16] = w;
                }
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

template <bool kF16>
s2_status launch(cudaStream_t st, const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                 const AttnArgs &args, int grid)
{
    static bool configured = false;
    if (!configured) {
        const cudaError_t e = cudaFuncSetAttribute(window_attention_kernel<kF16>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_window_attention: smem attribute: %s", cudaGetErrorString(e));
        configured = true;
    }
    window_attention_kernel<kF16><<<grid, kThreads, kSmemBytes, st>>>(mq, mk, mv, args);
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
    if (mode != S2_MODE_BF16_REF && mode != S2_MODE_F16)
        return s2::set_error(S2_UNSUPPORTED, "s2_window_attention: unknown mode %d", (int)mode);
    if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
          reinterpret_cast<uintptr_t>(vid_out) | reinterpret_cast<uintptr_t>(txt_partial)) & 15u) != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_window_attention: buffers must be 16-byte aligned");
    const long long grid = 1LL * n_work * heads;
    if (grid > 0x7fffffffLL) return s2::set_error(S2_INVALID_ARGUMENT, "s2_window_attention: grid too large");
    const bool f16 = mode == S2_MODE_F16;
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
    args.scale_log2 = static_cast<float>(1.4426950408889634 / 11.313708498984761);  // log2(e) / sqrt(128)
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return f16 ? launch<true>(st, mq, mk, mv, args, static_cast<int>(grid))
               : launch<false>(st, mq, mk, mv, args, static_cast<int>(grid));
}
