// Host-side planning for the windowed MM-attention path: window boxes,
// varlen packing, CTA work list, error state.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <vector>

#include "s2_internal.h"

namespace s2 {

namespace {
thread_local std::string g_last_error;
}

s2_status set_error(s2_status st, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

void clear_error() { g_last_error.clear(); }

const char *last_error() { return g_last_error.c_str(); }

}  // namespace s2

using s2::ceil_div;

extern "C" const char *s2_last_error(void) { return s2::last_error(); }

extern "C" int s2_version(void) { return 1; }

// Window boxes. The reference rule (seedvr2_dit_block.cpp:827-868): the grid
// is rescaled to a ~3600-token footprint (ties-to-even rounding), cut in
// thirds spatially and in quarters of min(T, 30) temporally; a shifted layer
// offsets the grid by half a window on every axis that has more than one
// window, truncating the border windows. Iteration order is w, h, t with t
// innermost, and empty boxes are dropped. The same grid arithmetic (double
// offsets truncated toward zero) is used so the boxes are bit-identical.
extern "C" s2_status s2_make_windows(int frames, int height, int width, int shifted,
                                     int wt, int wh, int ww,
                                     s2_window *out, int cap, int *count)
{
    if (frames <= 0 || height <= 0 || width <= 0 || !count)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_make_windows: invalid grid %dx%dx%d", frames, height, width);
    if ((wt > 0 || wh > 0 || ww > 0) && !(wt > 0 && wh > 0 && ww > 0))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_make_windows: window override needs all of wt, wh, ww > 0");
    int size_t_ = wt, size_h = wh, size_w = ww;
    if (wt <= 0) {
        const double scale = std::sqrt(3600.0 / static_cast<double>(height * width));
        const int rh = static_cast<int>(std::nearbyint(height * scale));
        const int rw = static_cast<int>(std::nearbyint(width * scale));
        size_h = ceil_div(rh, 3);
        size_w = ceil_div(rw, 3);
        size_t_ = ceil_div(std::min(frames, 30), 4);
    }
    if (size_t_ <= 0 || size_h <= 0 || size_w <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_make_windows: degenerate window size");
    const double off_t = shifted && size_t_ < frames ? 0.5 : 0.0;
    const double off_h = shifted && size_h < height ? 0.5 : 0.0;
    const double off_w = shifted && size_w < width ? 0.5 : 0.0;
    auto count_axis = [&](int extent, int size, double off) {
        if (!shifted) return ceil_div(extent, size);
        return off > 0.0 ? static_cast<int>(std::ceil((extent - off) / size)) + 1 : 1;
    };
    const int nt = count_axis(frames, size_t_, off_t);
    const int nh = count_axis(height, size_h, off_h);
    const int nw = count_axis(width, size_w, off_w);
    int n = 0;
    for (int iw = 0; iw < nw; iw++)
        for (int ih = 0; ih < nh; ih++)
            for (int it = 0; it < nt; it++) {
                s2_window b;
                b.t0 = std::max(static_cast<int>((it - off_t) * size_t_), 0);
                b.t1 = std::min(static_cast<int>((it - off_t + 1.0) * size_t_), frames);
                b.h0 = std::max(static_cast<int>((ih - off_h) * size_h), 0);
                b.h1 = std::min(static_cast<int>((ih - off_h + 1.0) * size_h), height);
                b.w0 = std::max(static_cast<int>((iw - off_w) * size_w), 0);
                b.w1 = std::min(static_cast<int>((iw - off_w + 1.0) * size_w), width);
                if (b.t1 > b.t0 && b.h1 > b.h0 && b.w1 > b.w0) {
                    if (out && n < cap) out[n] = b;
                    n++;
                }
            }
    *count = n;
    return S2_OK;
}

extern "C" s2_status s2_build_varlen(int frames, int height, int width,
                                     const s2_window *windows, int n, int text_len,
                                     int32_t *cu_seqlens, s2_row *rows, int *total_rows)
{
    if (!windows || n <= 0 || text_len < 0 || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_build_varlen: invalid arguments");
    long long total = 0;
    for (int w = 0; w < n; w++) {
        const s2_window &b = windows[w];
        if (b.t0 < 0 || b.t1 > frames || b.t0 >= b.t1 || b.h0 < 0 || b.h1 > height || b.h0 >= b.h1 ||
            b.w0 < 0 || b.w1 > width || b.w0 >= b.w1)
            return s2::set_error(S2_INVALID_ARGUMENT, "s2_build_varlen: window %d outside the %dx%dx%d grid", w,
                                 frames, height, width);
        if (cu_seqlens) cu_seqlens[w] = static_cast<int32_t>(total);
        const long long lw = 1LL * (b.t1 - b.t0) * (b.h1 - b.h0) * (b.w1 - b.w0);
        if (rows) {
            s2_row *r = rows + total;
            for (int t = b.t0; t < b.t1; t++)
                for (int y = b.h0; y < b.h1; y++)
                    for (int x = b.w0; x < b.w1; x++, r++) {
                        r->src = (t * height + y) * width + x;
                        r->pt = text_len + (t - b.t0);
                        r->ph = y - b.h0;
                        r->pw = x - b.w0;
                    }
            for (int l = 0; l < text_len; l++, r++) {
                r->src = -(l + 1);
                r->pt = r->ph = r->pw = l;
            }
        }
        total += lw + text_len;
        if (total > (1LL << 30))
            return s2::set_error(S2_INVALID_ARGUMENT, "s2_build_varlen: packed sequence too long");
    }
    if (cu_seqlens) cu_seqlens[n] = static_cast<int32_t>(total);
    if (total_rows) *total_rows = static_cast<int>(total);
    return S2_OK;
}

// Work items (window << 16 | q_block), one per kCtaRows (256) query rows,
// costliest first: every q-block of a window costs ceil(S_w / kTileN) key
// tiles, so sorting windows by S_w descending is a longest-processing-time
// order for the hardware block scheduler.
extern "C" s2_status s2_plan_work(const int32_t *cu_seqlens, int n_windows, int32_t *work, int cap, int *n_work)
{
    if (!cu_seqlens || n_windows <= 0 || !n_work)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_plan_work: invalid arguments");
    if (n_windows > 65535)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_plan_work: too many windows (%d)", n_windows);
    std::vector<int> order(n_windows);
    for (int w = 0; w < n_windows; w++) order[w] = w;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
        return cu_seqlens[a + 1] - cu_seqlens[a] > cu_seqlens[b + 1] - cu_seqlens[b];
    });
    int n = 0;
    for (int w : order) {
        const int s = cu_seqlens[w + 1] - cu_seqlens[w];
        const int tiles = ceil_div(s, s2::kCtaRows);
        if (tiles > 65535) return s2::set_error(S2_INVALID_ARGUMENT, "s2_plan_work: window %d too long", w);
        for (int qt = 0; qt < tiles; qt++) {
            if (work && n < cap) work[n] = (w << 16) | qt;
            n++;
        }
    }
    *n_work = n;
    return S2_OK;
}

// Longest-processing-time assignment of a layer's windows to ranks: windows in
// descending cost S_w^2 (S_w = L_w + text_len; ties keep window order), each to
// the least-loaded rank (ties to the lowest rank). Deterministic, so every rank
// derives the same ownership without communicating.
extern "C" s2_status s2_shard_windows(const s2_window *windows, int n, int text_len, int n_ranks, int32_t *owner)
{
    if (!windows || !owner || n <= 0 || n_ranks <= 0 || text_len < 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_shard_windows: invalid arguments");
    std::vector<double> cost(n);
    for (int i = 0; i < n; ++i) {
        const s2_window &w = windows[i];
        const double s = static_cast<double>(w.t1 - w.t0) * (w.h1 - w.h0) * (w.w1 - w.w0) + text_len;
        cost[i] = s * s;
    }
    std::vector<int> order(n);
    for (int i = 0; i < n; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
    std::vector<double> load(n_ranks, 0.0);
    for (int i : order) {
        int r = 0;
        for (int k = 1; k < n_ranks; ++k)
            if (load[k] < load[r]) r = k;
        owner[i] = r;
        load[r] += cost[i];
    }
    return S2_OK;
}

// ---- failure injection (tests) ------------------------------------------------

namespace {
std::atomic<int> g_fail_allocs{0};
std::atomic<int> g_fault_skip_k{-1};
std::atomic<unsigned long long> g_fault_wait_ns{0};
}  // namespace

namespace s2 {
bool alloc_fault()
{
    int n = g_fail_allocs.load();
    while (n > 0)
        if (g_fail_allocs.compare_exchange_weak(n, n - 1)) return true;
    return false;
}

void take_attention_fault(int *skip_k, unsigned long long *wait_ns)
{
    *skip_k = g_fault_skip_k.exchange(-1);
    const unsigned long long w = g_fault_wait_ns.exchange(0);
    *wait_ns = w ? w : 1000000000ull;  // the default limit: 1 s
}
}  // namespace s2

extern "C" s2_status s2_debug_fail_allocations(int n)
{
    g_fail_allocs.store(n > 0 ? n : 0);
    return S2_OK;
}

extern "C" s2_status s2_debug_attention_fault(int skip_k_tile, unsigned long long wait_ns)
{
    g_fault_skip_k.store(skip_k_tile >= 0 ? skip_k_tile : -1);
    g_fault_wait_ns.store(wait_ns);
    return S2_OK;
}

