// Allocation-free variant of the attention stage.
//
// Some callers cannot allocate device memory at the point where they run the
// attention: code executing inside another framework's memory pool or
// allocator hooks (a cudaMalloc there would bypass the owner's accounting or
// deadlock on its lock), hosts that pre-reserve all HBM for themselves, or
// embedded runtimes that forbid allocation after start-up. For them this file
// provides s2_dit_window_attention_noalloc: the same prologue -> attention ->
// text-mean sequence as s2_attention_layer_forward, but every scratch buffer
// (packed Q/K/V, per-window text slabs, plan tables, RoPE table, error word)
// lives in one file-scope __device__ array of fixed size. The caller passes
// only inputs and outputs; nothing here calls cudaMalloc, cudaFree or any
// allocating library routine.
//
// The array (kScratchBytes, about 29 MiB) is part of this library's device
// image: a GPU holds it from the moment the module is loaded on that device
// (on first use under CUDA's default lazy module loading) until the process
// exits. All calls on a device share it and it keeps the last call's
// contents, so two calls whose GPU work overlaps (different streams, or
// different host threads, without ordering between them) race on it.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "s2_internal.h"

namespace {

// Limits of the fixed scratch (stated in include/s2_b200.h).
constexpr long long kMaxRowHeads = S2_NOALLOC_MAX_ROW_HEADS;  // packed rows x heads
constexpr long long kMaxTextElems = S2_NOALLOC_MAX_TEXT_ELEMS;  // windows x text_len x dim
constexpr int kMaxWindows = S2_NOALLOC_MAX_WINDOWS;
constexpr int kMaxPos = S2_NOALLOC_MAX_ROPE_POS;
constexpr int kMaxWork = static_cast<int>(kMaxRowHeads / s2::kTileM) + kMaxWindows;  // upper bound on q-tiles

// Region offsets inside the scratch array, each 256-byte aligned.
constexpr size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
constexpr size_t kQKVBytes = static_cast<size_t>(kMaxRowHeads) * S2_HEAD_DIM * 2;
constexpr size_t kOffQ = 0;
constexpr size_t kOffK = kOffQ + align256(kQKVBytes);
constexpr size_t kOffV = kOffK + align256(kQKVBytes);
constexpr size_t kOffText = kOffV + align256(kQKVBytes);
constexpr size_t kOffRows = kOffText + align256(static_cast<size_t>(kMaxTextElems) * 2);
constexpr size_t kOffCu = kOffRows + align256(static_cast<size_t>(kMaxRowHeads) * sizeof(s2_row));
constexpr size_t kOffWin = kOffCu + align256((kMaxWindows + 1) * sizeof(int32_t));
constexpr size_t kOffWork = kOffWin + align256(kMaxWindows * sizeof(s2_window));
constexpr size_t kOffRope = kOffWork + align256(kMaxWork * sizeof(int32_t));
constexpr size_t kOffErr = kOffRope + align256(static_cast<size_t>(kMaxPos) * S2_ROPE_PAIRS * 8);
constexpr size_t kScratchBytes = kOffErr + 256;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Device address of g_scratch per device, resolved once per device with that
// device current. In host code `g_scratch` only names a host-side shadow, so
// kernels must be given this address, never the symbol itself.
std::mutex g_mu;
void *g_addr[128] = {};

s2_status scratch_address(void **out)
{
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 128)
        return s2::set_error(S2_UNSUPPORTED, "noalloc: no current CUDA device (%s)", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess || !p)
            return s2::set_error(S2_INFERENCE_FAILED, "noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                                 cudaGetErrorString(e));
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return S2_OK;
}

// The whole plan of one call, passed BY VALUE as a kernel parameter (about
// 17 KB, under the 32,764-byte parameter limit of sm_70+ with CUDA 12.1+), so
// the launch carries its own copy and no host pointer outlives the call.
struct NoallocPlan {
    s2_window wins[kMaxWindows];
    int32_t cu[kMaxWindows + 1];
    int32_t work[kMaxWork];
    int32_t n_windows, n_work;
};
static_assert(sizeof(NoallocPlan) <= 32000, "plan must fit the kernel parameter space");

// Writes the plan tables into the scratch array, clears the error word and
// builds the packed row table (the device-side counterpart of s2_build_varlen,
// so no host-side row array is needed).
__global__ void plan_rows_kernel(const NoallocPlan p, int n_rows, int height, int width, int text_len,
                                 s2_window *__restrict__ d_win, int32_t *__restrict__ d_cu,
                                 int32_t *__restrict__ d_work, int32_t *__restrict__ d_err,
                                 s2_row *__restrict__ rows)
{
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nthr = gridDim.x * blockDim.x;
    for (int i = tid; i < p.n_windows; i += nthr) d_win[i] = p.wins[i];
    for (int i = tid; i <= p.n_windows; i += nthr) d_cu[i] = p.cu[i];
    for (int i = tid; i < p.n_work; i += nthr) d_work[i] = p.work[i];
    if (tid == 0) *d_err = 0;
    const int n_windows = p.n_windows;
    for (int r = tid; r < n_rows; r += nthr) {
        int lo = 0, hi = n_windows - 1;  // last window with cu[w] <= r
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (p.cu[mid] <= r) lo = mid; else hi = mid - 1;
        }
        const s2_window b = p.wins[lo];
        const int i = r - p.cu[lo];
        const int lh = b.h1 - b.h0, lw = b.w1 - b.w0;
        const int lvid = (b.t1 - b.t0) * lh * lw;
        s2_row o;
        if (i < lvid) {
            const int tl = i / (lh * lw), yx = i - tl * lh * lw, yl = yx / lw, xl = yx - yl * lw;
            o.src = ((b.t0 + tl) * height + (b.h0 + yl)) * width + (b.w0 + xl);
            o.pt = text_len + tl;
            o.ph = yl;
            o.pw = xl;
        } else {
            const int l = i - lvid;
            o.src = -(l + 1);
            o.pt = o.ph = o.pw = l;
        }
        rows[r] = o;
    }
}

}  // namespace

extern "C" s2_status s2_dit_window_attention_noalloc(void *stream, s2_mode mode, const void *vid_qkv,
                                                     const void *txt_qkv, s2_dtype in_dtype, int frames, int height,
                                                     int width, int text_len, int heads, float eps, int shifted,
                                                     int wt, int wh, int ww, const float *gammas,
                                                     const float *freqs21, void *vid_out, float *txt_out,
                                                     int32_t *err)
{
    // ---- host-side validation and planning (host memory only) ----
    if (!vid_qkv || !gammas || !freqs21 || !vid_out || text_len < 0 || (text_len > 0 && (!txt_qkv || !txt_out)) ||
        heads <= 0 || heads > 64)
        return s2::set_error(S2_INVALID_ARGUMENT, "noalloc: NULL buffer or invalid heads/text_len");
    if (mode != S2_MODE_BF16_REF && mode != S2_MODE_F16 && mode != S2_MODE_BF16_F16)
        return s2::set_error(S2_UNSUPPORTED, "noalloc: unknown mode");
    // The plan lives in one struct that the launch below copies as its
    // parameter (static: ~17 KB is too large for some callers' thread stacks;
    // the mutex serialises host threads that plan at the same time).
    static std::mutex plan_mu;
    std::lock_guard<std::mutex> plan_lock(plan_mu);
    static NoallocPlan plan;
    s2_window *wins = plan.wins;
    int32_t *cu = plan.cu;
    int32_t *work = plan.work;
    int n = 0;
    s2_status rc = s2_make_windows(frames, height, width, shifted, wt, wh, ww, wins, kMaxWindows, &n);
    if (rc != S2_OK) return rc;
    if (n > kMaxWindows)
        return s2::set_error(S2_INVALID_ARGUMENT, "noalloc: %d windows exceed the fixed scratch limit of %d", n,
                             kMaxWindows);
    long long rows = 0;
    int max_pos = std::max(text_len, 1);
    for (int w = 0; w < n; w++) {
        cu[w] = static_cast<int32_t>(rows);
        const s2_window &b = wins[w];
        rows += 1LL * (b.t1 - b.t0) * (b.h1 - b.h0) * (b.w1 - b.w0) + text_len;
        max_pos = std::max({max_pos, text_len + (b.t1 - b.t0), b.h1 - b.h0, b.w1 - b.w0});
    }
    cu[n] = static_cast<int32_t>(std::min(rows, 1LL << 30));
    const int dim = heads * S2_HEAD_DIM;
    if (rows * heads > kMaxRowHeads)
        return s2::set_error(S2_INVALID_ARGUMENT,
                             "noalloc: %lld packed rows x %d heads exceed the fixed scratch limit of %lld row-heads",
                             rows, heads, kMaxRowHeads);
    if (1LL * n * text_len * dim > kMaxTextElems)
        return s2::set_error(S2_INVALID_ARGUMENT, "noalloc: %d windows x %d text tokens x %d exceed the limit of %lld",
                             n, text_len, dim, kMaxTextElems);
    if (max_pos > kMaxPos)
        return s2::set_error(S2_INVALID_ARGUMENT, "noalloc: RoPE position %d exceeds the limit of %d", max_pos - 1,
                             kMaxPos - 1);
    int n_work = 0;
    rc = s2_plan_work(cu, n, work, kMaxWork, &n_work);
    if (rc != S2_OK) return rc;
    if (n_work > kMaxWork) return s2::set_error(S2_INVALID_ARGUMENT, "noalloc: work list exceeds its limit");

    // ---- device side: fixed scratch only ----
    void *base = nullptr;
    rc = scratch_address(&base);
    if (rc != S2_OK) return rc;
    auto *sc = static_cast<unsigned char *>(base);
    auto *d_rows = reinterpret_cast<s2_row *>(sc + kOffRows);
    auto *d_cu = reinterpret_cast<int32_t *>(sc + kOffCu);
    auto *d_win = reinterpret_cast<s2_window *>(sc + kOffWin);
    auto *d_work = reinterpret_cast<int32_t *>(sc + kOffWork);
    auto *d_err = err ? err : reinterpret_cast<int32_t *>(sc + kOffErr);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    plan.n_windows = n;
    plan.n_work = n_work;
    const int n_rows = static_cast<int>(rows);
    plan_rows_kernel<<<std::max(1, std::min((n_rows + 255) / 256, 1184)), 256, 0, st>>>(
        plan, n_rows, height, width, text_len, d_win, d_cu, d_work, d_err, d_rows);
    if (cudaGetLastError() != cudaSuccess) return s2::set_error(S2_INFERENCE_FAILED, "noalloc: plan launch failed");
    void *rope = sc + kOffRope;
    rc = s2_rope_table(stream, freqs21, max_pos, rope);
    if (rc != S2_OK) return rc;
    void *q = sc + kOffQ, *k = sc + kOffK, *v = sc + kOffV, *tp = sc + kOffText;
    rc = s2_qk_norm_rope(stream, vid_qkv, txt_qkv, in_dtype, heads, eps, gammas, rope, d_rows, n_rows, mode, q, k, v);
    if (rc != S2_OK) return rc;
    rc = s2_window_attention(stream, mode, q, k, v, heads, n_rows, d_cu, n, text_len, d_rows, d_work, n_work, vid_out,
                             tp, d_err);
    if (rc != S2_OK) return rc;
    if (text_len > 0)
        rc = s2_text_window_sum(stream, mode, tp, n, text_len, dim, 1.f / static_cast<float>(n), 0, txt_out);
    return rc;
}
