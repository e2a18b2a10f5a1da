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

// ---- joint ownership and row-exchange maps of the sharded step ---------------

namespace {

s2_status windows_of(int T, int H, int W, int kind, int wt, int wh, int ww, std::vector<s2_window> &w)
{
    int n = 0;
    s2_status s = s2_make_windows(T, H, W, kind, wt, wh, ww, nullptr, 0, &n);
    if (s != S2_OK) return s;
    w.resize(n);
    return s2_make_windows(T, H, W, kind, wt, wh, ww, w.data(), n, &n);
}

// A window's share of a sharded DiT block's time, in units of one video row's
// per-row work (the projections, MLP and norms: ~128 ns per row per block at
// 720p) plus its attention (~11 ps per S_w^2 with S_w = video rows + text rows):
// the projections dominate, so ownership balances rows first.
constexpr double kAttnPerRow = 1e-4;
double window_cost(const s2_window &w, int text_len)
{
    const double l = static_cast<double>(w.t1 - w.t0) * (w.h1 - w.h0) * (w.w1 - w.w0);
    const double s = l + text_len;
    return l + kAttnPerRow * s * s;
}

}  // namespace

extern "C" s2_status s2_shard_windows_joint(int frames, int height, int width, int wt, int wh, int ww, int text_len,
                                            int n_ranks, int32_t *owner_plain, int32_t *owner_shifted)
{
    s2::clear_error();
    if (!owner_plain || !owner_shifted || n_ranks <= 0 || text_len < 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_shard_windows_joint: invalid arguments");
    std::vector<s2_window> w0, w1;
    s2_status s = windows_of(frames, height, width, 0, wt, wh, ww, w0);
    if (s == S2_OK) s = windows_of(frames, height, width, 1, wt, wh, ww, w1);
    if (s != S2_OK) return s;
    // plain windows: contiguous runs of the window order (width-major, then height, then
    // time: neighbouring windows share a column band), the runs chosen to minimise the
    // largest run cost (bisection on that cap; greedy packing decides feasibility)
    std::vector<double> c0(w0.size());
    double total = 0.0, biggest = 0.0;
    for (size_t i = 0; i < w0.size(); ++i) {
        c0[i] = window_cost(w0[i], text_len);
        total += c0[i];
        biggest = std::max(biggest, c0[i]);
    }
    auto runs = [&](double cap, int32_t *own) {
        int r = 0;
        double acc = 0.0;
        for (size_t i = 0; i < c0.size(); ++i) {
            if (acc > 0.0 && acc + c0[i] > cap) {
                ++r;
                acc = 0.0;
            }
            acc += c0[i];
            if (own) own[i] = std::min(r, n_ranks - 1);
        }
        return r + 1;
    };
    double lo = std::max(biggest, total / n_ranks), hi = total;
    for (int it = 0; it < 64 && hi - lo > 1e-9 * total; ++it) {
        const double mid = 0.5 * (lo + hi);
        (runs(mid, nullptr) <= n_ranks ? hi : lo) = mid;
    }
    runs(hi, owner_plain);
    // the owner of every token under the plain ownership
    const long long L = 1LL * frames * height * width;
    std::vector<int32_t> tok_owner(static_cast<size_t>(L), 0);
    for (size_t i = 0; i < w0.size(); ++i)
        for (int t = w0[i].t0; t < w0[i].t1; ++t)
            for (int y = w0[i].h0; y < w0[i].h1; ++y)
                for (int x = w0[i].w0; x < w0[i].w1; ++x)
                    tok_owner[(static_cast<size_t>(t) * height + y) * width + x] = owner_plain[i];
    // shifted windows, costliest first: to the rank holding most of its rows whose load
    // stays within 2 % of the mean; otherwise to the least loaded rank
    double total1 = 0.0;
    for (const s2_window &w : w1) total1 += window_cost(w, text_len);
    const double cap = 1.02 * total1 / n_ranks;
    std::vector<int> order(w1.size());
    for (size_t i = 0; i < w1.size(); ++i) order[i] = static_cast<int>(i);
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return window_cost(w1[a], text_len) > window_cost(w1[b], text_len); });
    std::vector<double> load(n_ranks, 0.0);
    std::vector<long long> overlap(n_ranks);
    for (int i : order) {
        std::fill(overlap.begin(), overlap.end(), 0);
        for (int t = w1[i].t0; t < w1[i].t1; ++t)
            for (int y = w1[i].h0; y < w1[i].h1; ++y)
                for (int x = w1[i].w0; x < w1[i].w1; ++x) ++overlap[tok_owner[(static_cast<size_t>(t) * height + y) * width + x]];
        const double c = window_cost(w1[i], text_len);
        int best = -1;
        for (int r = 0; r < n_ranks; ++r)
            if (load[r] + c <= cap && (best < 0 || overlap[r] > overlap[best])) best = r;
        if (best < 0) {
            best = 0;
            for (int r = 1; r < n_ranks; ++r)
                if (load[r] < load[best]) best = r;
        }
        owner_shifted[i] = best;
        load[best] += c;
    }
    // Per-kind LPT (s2_shard_windows) is kept instead when it happens to move fewer rows
    // at no worse balance (small grids whose two tilings split along the same frames).
    std::vector<int32_t> lpt0(w0.size()), lpt1(w1.size());
    if (s2_shard_windows(w0.data(), static_cast<int>(w0.size()), text_len, n_ranks, lpt0.data()) == S2_OK &&
        s2_shard_windows(w1.data(), static_cast<int>(w1.size()), text_len, n_ranks, lpt1.data()) == S2_OK) {
        auto score = [&](const int32_t *o0, const int32_t *o1, long long &moved, double &worst) {
            std::vector<int32_t> own(static_cast<size_t>(L));
            for (size_t i = 0; i < w0.size(); ++i)
                for (int t = w0[i].t0; t < w0[i].t1; ++t)
                    for (int y = w0[i].h0; y < w0[i].h1; ++y)
                        for (int x = w0[i].w0; x < w0[i].w1; ++x)
                            own[(static_cast<size_t>(t) * height + y) * width + x] = o0[i];
            moved = 0;
            for (size_t i = 0; i < w1.size(); ++i)
                for (int t = w1[i].t0; t < w1[i].t1; ++t)
                    for (int y = w1[i].h0; y < w1[i].h1; ++y)
                        for (int x = w1[i].w0; x < w1[i].w1; ++x)
                            moved += own[(static_cast<size_t>(t) * height + y) * width + x] != o1[i];
            worst = 0.0;
            for (int k = 0; k < 2; ++k) {
                const std::vector<s2_window> &w = k ? w1 : w0;
                const int32_t *o = k ? o1 : o0;
                std::vector<double> ld(n_ranks, 0.0);
                double sum = 0.0;
                for (size_t i = 0; i < w.size(); ++i) {
                    ld[o[i]] += window_cost(w[i], text_len);
                    sum += window_cost(w[i], text_len);
                }
                worst = std::max(worst, *std::max_element(ld.begin(), ld.end()) / (sum / n_ranks));
            }
        };
        long long mj = 0, ml = 0;
        double bj = 0.0, bl = 0.0;
        score(owner_plain, owner_shifted, mj, bj);
        score(lpt0.data(), lpt1.data(), ml, bl);
        if (ml < mj && bl <= bj) {
            std::copy(lpt0.begin(), lpt0.end(), owner_plain);
            std::copy(lpt1.begin(), lpt1.end(), owner_shifted);
        }
    }
    return S2_OK;
}

namespace s2 {

s2_status shard_exchange_maps(int T, int H, int W, int wt, int wh, int ww, int text_len, int n_ranks, int rank,
                              ShardMaps &m)
{
    std::vector<s2_window> w[2];
    for (int k = 0; k < 2; ++k) {
        const s2_status s = windows_of(T, H, W, k, wt, wh, ww, w[k]);
        if (s != S2_OK) return s;
    }
    std::vector<int32_t> owner[2] = {std::vector<int32_t>(w[0].size()), std::vector<int32_t>(w[1].size())};
    s2_status s = s2_shard_windows_joint(T, H, W, wt, wh, ww, text_len, n_ranks, owner[0].data(), owner[1].data());
    if (s != S2_OK) return s;
    const long long L = 1LL * T * H * W;
    std::vector<std::vector<std::vector<int32_t>>> tok(2, std::vector<std::vector<int32_t>>(n_ranks));
    std::vector<std::vector<int32_t>> own_rank(2, std::vector<int32_t>(L, -1)), own_idx(2, std::vector<int32_t>(L, -1));
    for (int k = 0; k < 2; ++k) {
        m.ids[k].clear();
        for (size_t i = 0; i < w[k].size(); ++i) {
            const int o = owner[k][i];
            if (o == rank) m.ids[k].push_back(static_cast<int32_t>(i));
            auto &list = tok[k][o];
            for (int t = w[k][i].t0; t < w[k][i].t1; ++t)
                for (int y = w[k][i].h0; y < w[k][i].h1; ++y)
                    for (int x = w[k][i].w0; x < w[k][i].w1; ++x) {
                        const int p = (t * H + y) * W + x;
                        own_rank[k][p] = o;
                        own_idx[k][p] = static_cast<int32_t>(list.size());
                        list.push_back(p);
                    }
        }
        for (long long p = 0; p < L; ++p)
            if (own_rank[k][p] < 0) return set_error(S2_INFERENCE_FAILED, "shard: token %lld has no window", p);
        m.tok[k] = tok[k][rank];
    }
    m.moved_rows[0] = m.moved_rows[1] = 0;
    for (int k = 0; k < 2; ++k) {
        const int k2 = 1 - k;
        m.src[k].clear();
        m.dst[k].clear();
        m.send_count[k].assign(n_ranks, 0);
        m.recv_count[k].assign(n_ranks, 0);
        for (int p2 = 0; p2 < n_ranks; ++p2) {  // rows I send to p2, in p2's local order of kind k2
            for (int p : tok[k2][p2])
                if (own_rank[k][p] == rank) {
                    m.src[k].push_back(own_idx[k][p]);
                    ++m.send_count[k][p2];
                }
        }
        for (int p1 = 0; p1 < n_ranks; ++p1)  // rows I receive from p1, in my local order of kind k2
            for (size_t i = 0; i < tok[k2][rank].size(); ++i)
                if (own_rank[k][tok[k2][rank][i]] == p1) {
                    m.dst[k].push_back(static_cast<int32_t>(i));
                    ++m.recv_count[k][p1];
                }
        for (long long p = 0; p < L; ++p)
            if (own_rank[k][p] != own_rank[k2][p]) ++m.moved_rows[k];
        m.dest_rank[k].resize(m.tok[k].size());
        m.dest_row[k].resize(m.tok[k].size());
        for (size_t i = 0; i < m.tok[k].size(); ++i) {
            const int p = m.tok[k][i];
            m.dest_rank[k][i] = own_rank[k2][p];
            m.dest_row[k][i] = own_idx[k2][p];
        }
    }
    return S2_OK;
}

}  // namespace s2

extern "C" s2_status s2_shard_exchange(int frames, int height, int width, int wt, int wh, int ww, int text_len,
                                       int n_ranks, int rank, int kind, int32_t *window_ids, int *n_windows,
                                       int32_t *local_tokens, int *n_local, int32_t *send_counts, int32_t *send_rows,
                                       int32_t *recv_counts, int32_t *recv_rows, long long *moved_rows)
{
    s2::clear_error();
    if (n_ranks <= 0 || rank < 0 || rank >= n_ranks || (kind != 0 && kind != 1) || !n_windows || !n_local)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_shard_exchange: invalid arguments");
    s2::ShardMaps m;
    const s2_status s = s2::shard_exchange_maps(frames, height, width, wt, wh, ww, text_len, n_ranks, rank, m);
    if (s != S2_OK) return s;
    *n_windows = static_cast<int>(m.ids[kind].size());
    *n_local = static_cast<int>(m.tok[kind].size());
    if (window_ids) std::copy(m.ids[kind].begin(), m.ids[kind].end(), window_ids);
    if (local_tokens) std::copy(m.tok[kind].begin(), m.tok[kind].end(), local_tokens);
    if (send_counts) std::copy(m.send_count[kind].begin(), m.send_count[kind].end(), send_counts);
    if (recv_counts) std::copy(m.recv_count[kind].begin(), m.recv_count[kind].end(), recv_counts);
    if (send_rows) std::copy(m.src[kind].begin(), m.src[kind].end(), send_rows);
    if (recv_rows) std::copy(m.dst[kind].begin(), m.dst[kind].end(), recv_rows);
    if (moved_rows) *moved_rows = m.moved_rows[kind];
    return S2_OK;
}

extern "C" s2_status s2_shard_row_destinations(int frames, int height, int width, int wt, int wh, int ww,
                                              int text_len, int n_ranks, int rank, int kind, int32_t *dest_rank,
                                              int32_t *dest_row, int *n_local)
{
    s2::clear_error();
    if (n_ranks <= 0 || rank < 0 || rank >= n_ranks || (kind != 0 && kind != 1) || !n_local)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_shard_row_destinations: invalid arguments");
    s2::ShardMaps m;
    const s2_status s = s2::shard_exchange_maps(frames, height, width, wt, wh, ww, text_len, n_ranks, rank, m);
    if (s != S2_OK) return s;
    *n_local = static_cast<int>(m.tok[kind].size());
    if (dest_rank) std::copy(m.dest_rank[kind].begin(), m.dest_rank[kind].end(), dest_rank);
    if (dest_row) std::copy(m.dest_row[kind].begin(), m.dest_row[kind].end(), dest_row);
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

