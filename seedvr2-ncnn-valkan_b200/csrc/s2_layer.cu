// s2_attention_layer: the attention stage of SeedVR2DiTBlock as a CUDA
// object (load_param / load_model / set_runtime_shape / forward,
// seedvr2_dit_block.cpp:643-688, 870-1091; seedvr2_dit_block.h:38-58).
//
// Per runtime shape it caches a plan -- windows, varlen offsets, packed row
// table, CTA work list, RoPE cos/sin table -- in device memory, so a forward
// is three stream-ordered launches (prologue, attention, text mean) with no
// host synchronisation. Workspaces (packed Q/K/V, per-window text slabs) grow
// on demand and are reused across calls.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <vector>

#include "s2_buffers.h"
#include "s2_gemm.h"
#include "s2_internal.h"
#include "s2_ops.h"

namespace s2 {
s2_status to_f32(cudaStream_t st, s2_mode mode, const void *src, long long n, float *dst);
s2_status qk_norm_rope_range(void *stream, const void *vid_qkv, const void *txt_qkv, s2_dtype in_dtype, int heads,
                             float eps, const float *gammas, const void *rope_table, const s2_row *rows, int n_rows,
                             s2_mode mode, int src_lo, int src_hi, int do_text, void *q, void *k, void *v);
}

using s2::DeviceBuffer;
using s2::DeviceGuard;

// Packed Q/K/V and per-window text outputs: the layer's large activation
// buffers, shareable between layers that run one after another.
struct AttnScratch {
    int device = 0;
    DeviceBuffer q, k, v, txt_partial;
    ~AttnScratch()
    {
        DeviceGuard g(device);
        for (DeviceBuffer *b : {&q, &k, &v, &txt_partial}) b->release();
    }
};

struct s2_attention_layer {
    int device = 0;
    int heads = 20;
    float eps = 1e-5f;
    int shifted = 0;
    int wt = 0, wh = 0, ww = 0;
    s2_mode mode = S2_MODE_BF16_REF;
    bool loaded = false;
    int T = 0, H = 0, W = 0;
    bool shape_valid = false;
    std::vector<int32_t> subset;
    bool local_rows = false;  // video rows are the subset's tokens, compacted in packed order
    int n_video = 0;          // video rows the plan reads and writes

    // plan
    bool plan_valid = false;
    int plan_T = 0, plan_H = 0, plan_W = 0, plan_Lt = -1;
    int n_total_windows = 0, n_local = 0, n_rows = 0, n_work = 0, max_pos = 0;
    std::vector<int32_t> h_cu;
    DeviceBuffer d_cu, d_rows, d_work, d_rope;
    // fused-prologue targets: per video row (then per text row) its packed row and
    // RoPE positions, and per window the packed row of its first text row
    DeviceBuffer d_pack_map, d_text_dst, d_rope_pairs;

    DeviceBuffer d_weights;  // gammas [4][128] + freqs [21]
    std::shared_ptr<AttnScratch> sc = std::make_shared<AttnScratch>();
    DeviceBuffer d_err;
    DeviceBuffer d_in_vid, d_in_txt, d_out_vid, d_out_vid32, d_out_txt;  // host-forward staging
    cudaStream_t last_stream = nullptr;
    int last_launches = 0;

    // Host-buffer forward pipeline: the windows grouped by their frame range
    // (the t-slabs of the tiling), each with its own work list, so that the
    // upload of slab s+1, the compute of slab s and the download of slab s-1
    // overlap. Built with the plan (whole window set only).
    // A slab is uploaded, computed and downloaded in parts: rows [h0, h1) of
    // each of its frames, holding the windows of one height range (they span
    // the full width); one part of all rows when the height ranges do not tile.
    struct Part {
        int h0 = 0, h1 = 0;
        int work_off = 0, n_work = 0;
    };
    struct Slab {
        int t0 = 0, t1 = 0;      // frames [t0, t1)
        std::vector<Part> parts;
    };
    std::vector<Slab> slabs;
    bool slabs_valid = false;
    DeviceBuffer d_slab_work;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    std::vector<cudaEvent_t> ev_in, ev_cmp;
    cudaEvent_t ev_start = nullptr, ev_out = nullptr;

    ~s2_attention_layer()
    {
        DeviceGuard g(device);
        for (DeviceBuffer *b : {&d_cu, &d_rows, &d_work, &d_rope, &d_pack_map, &d_text_dst, &d_rope_pairs, &d_weights, &d_err, &d_in_vid, &d_in_txt, &d_out_vid, &d_out_vid32, &d_out_txt, &d_slab_work})
            b->release();
        for (cudaEvent_t e : ev_in) cudaEventDestroy(e);
        for (cudaEvent_t e : ev_cmp) cudaEventDestroy(e);
        if (ev_start) cudaEventDestroy(ev_start);
        if (ev_out) cudaEventDestroy(ev_out);
        if (s_in) cudaStreamDestroy(s_in);
        if (s_out) cudaStreamDestroy(s_out);
    }

    // Slab work lists (window index << 16 | q-block, costliest window first
    // within a part, as s2_plan_work) for the current plan; false when the
    // windows do not split into full-frame slabs (then the forward is serial).
    // Each slab is split into parts by the windows' height ranges, so that every
    // part's download overlaps the next part's upload and only the last part's
    // compute and download remain after the last upload.
    bool build_slabs()
    {
        if (slabs_valid) return !slabs.empty();
        slabs.clear();
        slabs_valid = true;
        if (!subset.empty() || local_rows) return false;
        int count = 0;
        if (s2_make_windows(T, H, W, shifted, wt, wh, ww, nullptr, 0, &count) != S2_OK || count != n_local) return false;
        std::vector<s2_window> all(count);
        s2_make_windows(T, H, W, shifted, wt, wh, ww, all.data(), count, &count);
        std::vector<std::pair<int, int>> ranges;
        for (const s2_window &w : all)
            if (std::find(ranges.begin(), ranges.end(), std::make_pair(w.t0, w.t1)) == ranges.end())
                ranges.emplace_back(w.t0, w.t1);
        std::sort(ranges.begin(), ranges.end());
        // the ranges must tile [0, T) and every slab's windows cover its frames entirely
        for (size_t i = 0; i < ranges.size(); ++i)
            if (ranges[i].first != (i == 0 ? 0 : ranges[i - 1].second)) return false;
        if (ranges.empty() || ranges.back().second != T) return false;
        std::vector<int32_t> h_work;
        for (const auto &rg : ranges) {
            std::vector<int> ids;
            long long cover = 0;
            for (int i = 0; i < count; ++i)
                if (all[i].t0 == rg.first && all[i].t1 == rg.second) {
                    ids.push_back(i);
                    cover += 1LL * (all[i].h1 - all[i].h0) * (all[i].w1 - all[i].w0) * (all[i].t1 - all[i].t0);
                }
            if (cover != 1LL * (rg.second - rg.first) * H * W) return false;
            std::stable_sort(ids.begin(), ids.end(), [&](int a, int b) {
                return h_cu[a + 1] - h_cu[a] > h_cu[b + 1] - h_cu[b];
            });
            // height ranges of the slab's windows; each must cover full rows of the slab
            std::vector<std::pair<int, int>> hr;
            {
                for (int i : ids)
                    if (std::find(hr.begin(), hr.end(), std::make_pair(all[i].h0, all[i].h1)) == hr.end())
                        hr.emplace_back(all[i].h0, all[i].h1);
                std::sort(hr.begin(), hr.end());
                bool tiles = !hr.empty() && hr.front().first == 0 && hr.back().second == H;
                for (size_t k = 1; tiles && k < hr.size(); ++k) tiles = hr[k].first == hr[k - 1].second;
                for (size_t k = 0; tiles && k < hr.size(); ++k) {
                    long long area = 0;
                    for (int i : ids)
                        if (all[i].h0 == hr[k].first && all[i].h1 == hr[k].second)
                            area += 1LL * (all[i].h1 - all[i].h0) * (all[i].w1 - all[i].w0);
                    tiles = area == 1LL * (hr[k].second - hr[k].first) * W;
                }
                if (!tiles) hr.clear();
            }
            if (hr.empty()) hr.emplace_back(0, H);
            Slab sl;
            sl.t0 = rg.first;
            sl.t1 = rg.second;
            for (const auto &h : hr) {
                Part pt;
                pt.h0 = h.first;
                pt.h1 = h.second;
                pt.work_off = static_cast<int>(h_work.size());
                for (int w : ids) {
                    if (hr.size() > 1 && (all[w].h0 != h.first || all[w].h1 != h.second)) continue;
                    const int seq = h_cu[w + 1] - h_cu[w];
                    for (int qb = 0; qb * s2::kCtaRows < seq; ++qb) h_work.push_back((w << 16) | qb);
                }
                pt.n_work = static_cast<int>(h_work.size()) - pt.work_off;
                sl.parts.push_back(pt);
            }
            slabs.push_back(sl);
        }
        if (!d_slab_work.ensure(h_work.size() * sizeof(int32_t)) ||
            cudaMemcpy(d_slab_work.ptr, h_work.data(), h_work.size() * sizeof(int32_t), cudaMemcpyHostToDevice) !=
                cudaSuccess) {
            slabs.clear();
            return false;
        }
        return true;
    }

    size_t n_parts() const
    {
        size_t n = 0;
        for (const Slab &sl : slabs) n += sl.parts.size();
        return n;
    }

    // n: the number of parts (one upload event per slab, one compute event per part)
    bool ensure_pipeline_objects(size_t n)
    {
        if (!s_in && cudaStreamCreateWithFlags(&s_in, cudaStreamNonBlocking) != cudaSuccess) return false;
        if (!s_out && cudaStreamCreateWithFlags(&s_out, cudaStreamNonBlocking) != cudaSuccess) return false;
        if (!ev_start && cudaEventCreateWithFlags(&ev_start, cudaEventDisableTiming) != cudaSuccess) return false;
        if (!ev_out && cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming) != cudaSuccess) return false;
        while (ev_in.size() < n) {
            cudaEvent_t a = nullptr, b = nullptr;
            if (cudaEventCreateWithFlags(&a, cudaEventDisableTiming) != cudaSuccess) return false;
            if (cudaEventCreateWithFlags(&b, cudaEventDisableTiming) != cudaSuccess) {
                cudaEventDestroy(a);
                return false;
            }
            ev_in.push_back(a);
            ev_cmp.push_back(b);
        }
        return true;
    }

    const float *gammas() const { return static_cast<const float *>(d_weights.ptr); }
    const float *freqs() const { return static_cast<const float *>(d_weights.ptr) + 4 * S2_HEAD_DIM; }

    s2_status build_plan(int Lt, cudaStream_t st)
    {
        if (plan_valid && plan_T == T && plan_H == H && plan_W == W && plan_Lt == Lt) return S2_OK;
        // The tables below are overwritten by synchronous copies, which are not
        // ordered after kernels still queued on a non-blocking stream: wait for
        // the forwards that read the old plan (on whatever stream) first.
        if (plan_valid) cudaDeviceSynchronize();
        plan_valid = false;
        slabs_valid = false;
        int count = 0;
        s2_status rc = s2_make_windows(T, H, W, shifted, wt, wh, ww, nullptr, 0, &count);
        if (rc != S2_OK) return rc;
        std::vector<s2_window> all(count);
        s2_make_windows(T, H, W, shifted, wt, wh, ww, all.data(), count, &count);
        std::vector<s2_window> local;
        if (subset.empty()) {
            local = all;
        } else {
            for (int32_t id : subset) {
                if (id < 0 || id >= count)
                    return s2::set_error(S2_INVALID_ARGUMENT, "window subset id %d out of range [0,%d)", id, count);
                local.push_back(all[id]);
            }
        }
        n_total_windows = count;
        n_local = static_cast<int>(local.size());
        int rows = 0;
        rc = s2_build_varlen(T, H, W, local.data(), n_local, Lt, nullptr, nullptr, &rows);
        if (rc != S2_OK) return rc;
        h_cu.assign(n_local + 1, 0);
        std::vector<s2_row> h_rows(rows);
        rc = s2_build_varlen(T, H, W, local.data(), n_local, Lt, h_cu.data(), h_rows.data(), &rows);
        if (rc != S2_OK) return rc;
        int nw = 0;
        rc = s2_plan_work(h_cu.data(), n_local, nullptr, 0, &nw);
        if (rc != S2_OK) return rc;
        std::vector<int32_t> h_work(nw);
        s2_plan_work(h_cu.data(), n_local, h_work.data(), nw, &nw);
        int mp = 1;
        for (const s2_row &r : h_rows) mp = std::max(mp, std::max(r.pt, std::max(r.ph, r.pw)) + 1);
        n_video = T * H * W;
        if (local_rows) {
            // the i-th video row of the packed sequence is local row i
            int next = 0;
            for (s2_row &r : h_rows)
                if (r.src >= 0) r.src = next++;
            n_video = next;
        }
        n_rows = rows;
        n_work = nw;
        max_pos = mp;
        // inverse of the packed row table for the fused prologue: video row -> its packed
        // row and positions; text row l -> {-1 - l, l, l, l} (the same in every window)
        std::vector<int4> h_map(static_cast<size_t>(n_video) + std::max(Lt, 0), make_int4(-0x7fffffff, 0, 0, 0));
        for (int p = 0; p < rows; ++p)
            if (h_rows[p].src >= 0 && h_rows[p].src < n_video)
                h_map[h_rows[p].src] = make_int4(p, h_rows[p].pt, h_rows[p].ph, h_rows[p].pw);
        for (int t = 0; t < Lt; ++t) h_map[static_cast<size_t>(n_video) + t] = make_int4(-1 - t, t, t, t);
        std::vector<int32_t> h_tdst(std::max(n_local, 1), 0);
        for (int w = 0; w < n_local; ++w) h_tdst[w] = h_cu[w + 1] - Lt;
        if (!d_cu.ensure(h_cu.size() * sizeof(int32_t)) || !d_rows.ensure(h_rows.size() * sizeof(s2_row)) ||
            !d_work.ensure(h_work.size() * sizeof(int32_t)) || !d_rope.ensure(s2_rope_table_bytes(max_pos)) ||
            !d_pack_map.ensure(h_map.size() * sizeof(int4)) || !d_text_dst.ensure(h_tdst.size() * sizeof(int32_t)) ||
            !d_rope_pairs.ensure(s2_rope_table_bytes(max_pos)))
            return s2::set_error(S2_OUT_OF_MEMORY, "attention plan: device allocation failed");
        if (cudaMemcpy(d_pack_map.ptr, h_map.data(), h_map.size() * sizeof(int4), cudaMemcpyHostToDevice) !=
                cudaSuccess ||
            cudaMemcpy(d_text_dst.ptr, h_tdst.data(), h_tdst.size() * sizeof(int32_t), cudaMemcpyHostToDevice) !=
                cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "attention plan: upload failed");
        // Stream-ordered uploads from host vectors need the host side to stay
        // alive until the copy completes: copy synchronously (plans change
        // rarely -- once per runtime shape).
        if (cudaMemcpy(d_cu.ptr, h_cu.data(), h_cu.size() * sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d_rows.ptr, h_rows.data(), h_rows.size() * sizeof(s2_row), cudaMemcpyHostToDevice) !=
                cudaSuccess ||
            cudaMemcpy(d_work.ptr, h_work.data(), h_work.size() * sizeof(int32_t), cudaMemcpyHostToDevice) !=
                cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "attention plan: upload failed");
        rc = s2_rope_table(st, freqs(), max_pos, d_rope.ptr);
        if (rc != S2_OK) return rc;
        rc = s2::rope_table_pairs(st, freqs(), max_pos, d_rope_pairs.ptr);
        if (rc != S2_OK) return rc;
        plan_T = T;
        plan_H = H;
        plan_W = W;
        plan_Lt = Lt;
        plan_valid = true;
        return S2_OK;
    }
};

extern "C" s2_status s2_device_check(int device)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return s2::set_error(S2_UNSUPPORTED, "no CUDA device available");
    }
    if (device < 0 || device >= n) return s2::set_error(S2_INVALID_ARGUMENT, "device %d out of range", device);
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0)
        return s2::set_error(S2_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a (B200)", device, major,
                             minor);
    return S2_OK;
}

extern "C" s2_status s2_attention_layer_create(int device, int heads, int head_dim, float eps, int shifted, int wt,
                                               int wh, int ww, s2_mode mode, s2_attention_layer **out)
{
    if (!out) return s2::set_error(S2_INVALID_ARGUMENT, "s2_attention_layer_create: out is NULL");
    *out = nullptr;
    if (head_dim != S2_HEAD_DIM)
        return s2::set_error(S2_INVALID_ARGUMENT, "head_dim must be %d (got %d)", S2_HEAD_DIM, head_dim);
    if (heads <= 0 || heads > 64) return s2::set_error(S2_INVALID_ARGUMENT, "heads must be in [1, 64]");
    if (mode != S2_MODE_BF16_REF && mode != S2_MODE_F16 && mode != S2_MODE_BF16_F16)
        return s2::set_error(S2_UNSUPPORTED, "unknown mode");
    if ((wt > 0 || wh > 0 || ww > 0) && !(wt > 0 && wh > 0 && ww > 0))
        return s2::set_error(S2_INVALID_ARGUMENT, "window override needs wt, wh, ww > 0");
    const s2_status dc = s2_device_check(device);
    if (dc != S2_OK) return dc;
    auto *l = new s2_attention_layer;
    l->device = device;
    l->sc->device = device;
    l->heads = heads;
    l->eps = eps;
    l->shifted = shifted ? 1 : 0;
    l->wt = wt > 0 ? wt : 0;
    l->wh = wh > 0 ? wh : 0;
    l->ww = ww > 0 ? ww : 0;
    l->mode = mode;
    *out = l;
    return S2_OK;
}

extern "C" s2_status s2_attention_layer_destroy(s2_attention_layer *layer)
{
    delete layer;
    return S2_OK;
}

extern "C" s2_status s2_attention_layer_load(s2_attention_layer *l, const float *nq_vid, const float *nk_vid,
                                             const float *nq_txt, const float *nk_txt, const float *freqs21)
{
    if (!l || !nq_vid || !nk_vid || !nq_txt || !nk_txt || !freqs21)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_attention_layer_load: NULL argument");
    DeviceGuard g(l->device);
    std::vector<float> host(4 * S2_HEAD_DIM + S2_ROPE_PAIRS);
    std::memcpy(host.data() + 0 * S2_HEAD_DIM, nq_vid, S2_HEAD_DIM * sizeof(float));
    std::memcpy(host.data() + 1 * S2_HEAD_DIM, nk_vid, S2_HEAD_DIM * sizeof(float));
    std::memcpy(host.data() + 2 * S2_HEAD_DIM, nq_txt, S2_HEAD_DIM * sizeof(float));
    std::memcpy(host.data() + 3 * S2_HEAD_DIM, nk_txt, S2_HEAD_DIM * sizeof(float));
    std::memcpy(host.data() + 4 * S2_HEAD_DIM, freqs21, S2_ROPE_PAIRS * sizeof(float));
    if (!l->d_weights.ensure(host.size() * sizeof(float)))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_attention_layer_load: allocation failed");
    if (cudaMemcpy(l->d_weights.ptr, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_attention_layer_load: upload failed");
    l->loaded = true;
    l->plan_valid = false;  // the RoPE table depends on freqs
    return S2_OK;
}

extern "C" s2_status s2_attention_layer_set_runtime_shape(s2_attention_layer *l, int frames, int height, int width)
{
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "layer is NULL");
    l->T = frames;
    l->H = height;
    l->W = width;
    l->shape_valid = frames > 0 && height > 0 && width > 0;
    return l->shape_valid ? S2_OK : s2::set_error(S2_INVALID_ARGUMENT, "invalid runtime shape");
}

extern "C" s2_status s2_attention_layer_set_window_subset(s2_attention_layer *l, const int32_t *ids, int n)
{
    if (!l || n < 0 || (n > 0 && !ids)) return s2::set_error(S2_INVALID_ARGUMENT, "invalid window subset");
    l->subset.assign(ids, ids + n);
    l->plan_valid = false;
    return S2_OK;
}

extern "C" s2_status s2_attention_layer_set_local_rows(s2_attention_layer *l, int enable)
{
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "layer is NULL");
    l->local_rows = enable != 0;
    l->plan_valid = false;
    return S2_OK;
}

extern "C" s2_status s2_attention_layer_local_rows(s2_attention_layer *l, int Lt, int *n_video)
{
    if (!l || !n_video) return s2::set_error(S2_INVALID_ARGUMENT, "layer is NULL");
    if (!l->loaded || !l->shape_valid)
        return s2::set_error(S2_NOT_LOADED, "attention layer: weights or runtime shape not set");
    s2::DeviceGuard g(l->device);
    const s2_status rc = l->build_plan(Lt, nullptr);
    if (rc != S2_OK) return rc;
    *n_video = l->n_video;
    return S2_OK;
}

extern "C" int s2_attention_layer_last_launches(const s2_attention_layer *l) { return l ? l->last_launches : 0; }

// Packed Q/K/V and text-slab workspace for the current plan, and the error word.
static s2_status ensure_workspace(s2_attention_layer *l, int Lt)
{
    const int dim = l->heads * S2_HEAD_DIM;
    const size_t qkv_bytes = static_cast<size_t>(l->n_rows) * dim * 2;
    const size_t txt_bytes = static_cast<size_t>(std::max(l->n_local, 1)) * std::max(Lt, 1) * dim * 2;
    AttnScratch &sc = *l->sc;
    if (!sc.q.ensure(qkv_bytes) || !sc.k.ensure(qkv_bytes) || !sc.v.ensure(qkv_bytes) || !sc.txt_partial.ensure(txt_bytes))
        return s2::set_error(S2_OUT_OF_MEMORY, "attention layer: workspace allocation failed");
    if (!l->d_err.ptr && (!l->d_err.ensure(sizeof(int32_t)) || cudaMemset(l->d_err.ptr, 0, sizeof(int32_t)) != cudaSuccess))
        return s2::set_error(S2_OUT_OF_MEMORY, "attention layer: error word allocation failed");
    return S2_OK;
}

// The attention core over the packed operands of the current plan, then the text
// mean of the per-window text outputs; sets last_launches.
static s2_status attention_and_text(s2_attention_layer *l, cudaStream_t st, int Lt, void *vid_out, float *txt_out)
{
    const int dim = l->heads * S2_HEAD_DIM;
    AttnScratch &sc = *l->sc;
    s2_status rc = s2_window_attention(st, l->mode, sc.q.ptr, sc.k.ptr, sc.v.ptr, l->heads, l->n_rows,
                                       static_cast<const int32_t *>(l->d_cu.ptr), l->n_local, Lt,
                                       static_cast<const s2_row *>(l->d_rows.ptr),
                                       static_cast<const int32_t *>(l->d_work.ptr), l->n_work, vid_out,
                                       sc.txt_partial.ptr, static_cast<int32_t *>(l->d_err.ptr));
    if (rc != S2_OK) return rc;
    l->last_launches = 1;
    if (Lt > 0) {
        rc = s2_text_window_sum(st, l->mode, sc.txt_partial.ptr, l->n_local, Lt, dim,
                                1.f / static_cast<float>(l->n_total_windows), 0, txt_out);
        if (rc != S2_OK) return rc;
        l->last_launches = 2;
    }
    return S2_OK;
}

extern "C" s2_status s2_attention_layer_forward(s2_attention_layer *l, void *stream, const void *vid_qkv,
                                                s2_dtype in_dtype, int L, const void *txt_qkv, int Lt,
                                                void *vid_out, float *txt_out)
{
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "layer is NULL");
    l->last_launches = 0;
    if (!l->loaded) return s2::set_error(S2_NOT_LOADED, "attention layer: weights not loaded");
    if (!l->shape_valid) return s2::set_error(S2_NOT_LOADED, "attention layer: runtime shape not set");
    if (Lt < 0 || (Lt > 0 && !txt_qkv) || !vid_qkv || !vid_out || (Lt > 0 && !txt_out))
        return s2::set_error(S2_INVALID_ARGUMENT, "attention layer: NULL buffer");
    DeviceGuard g(l->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    l->last_stream = st;
    s2_status rc = l->build_plan(Lt, st);
    if (rc == S2_OK && L != l->n_video)
        return s2::set_error(S2_INVALID_ARGUMENT, "attention layer: vid rows %d != %d (%s)", L, l->n_video,
                             l->local_rows ? "the subset's video tokens" : "T*H*W");
    if (rc != S2_OK) return rc;
    if ((rc = ensure_workspace(l, Lt)) != S2_OK) return rc;
    AttnScratch &sc = *l->sc;
    rc = s2_qk_norm_rope(stream, vid_qkv, txt_qkv, in_dtype, l->heads, l->eps, l->gammas(), l->d_rope.ptr,
                         static_cast<const s2_row *>(l->d_rows.ptr), l->n_rows, l->mode, sc.q.ptr, sc.k.ptr,
                         sc.v.ptr);
    if (rc != S2_OK) return rc;
    rc = attention_and_text(l, st, Lt, vid_out, txt_out);
    if (rc == S2_OK) ++l->last_launches;
    return rc;
}

s2_status s2::attention_pack_target(s2_attention_layer *l, cudaStream_t st, int L, int Lt, s2::GemmArgs *g)
{
    if (!l || !g) return s2::set_error(S2_INVALID_ARGUMENT, "attention pack target: NULL argument");
    if (!l->loaded) return s2::set_error(S2_NOT_LOADED, "attention layer: weights not loaded");
    if (!l->shape_valid) return s2::set_error(S2_NOT_LOADED, "attention layer: runtime shape not set");
    if (Lt < 0) return s2::set_error(S2_INVALID_ARGUMENT, "attention layer: negative text length");
    DeviceGuard dg(l->device);
    l->last_stream = st;
    s2_status rc = l->build_plan(Lt, st);
    if (rc != S2_OK) return rc;
    if (L != l->n_video)
        return s2::set_error(S2_INVALID_ARGUMENT, "attention layer: vid rows %d != %d (%s)", L, l->n_video,
                             l->local_rows ? "the subset's video tokens" : "T*H*W");
    if ((rc = ensure_workspace(l, Lt)) != S2_OK) return rc;
    AttnScratch &sc = *l->sc;
    s2::PackArgs &pk = g->pk;
    pk.map = static_cast<const int4 *>(l->d_pack_map.ptr);
    pk.text_dst = static_cast<const int32_t *>(l->d_text_dst.ptr);
    pk.n_windows = Lt > 0 ? l->n_local : 0;
    pk.q = sc.q.ptr;
    pk.k = sc.k.ptr;
    pk.v = sc.v.ptr;
    pk.n_rows = l->n_rows;
    pk.dim = l->heads * S2_HEAD_DIM;
    pk.gammas = l->gammas();
    pk.rope = static_cast<const float2 *>(l->d_rope_pairs.ptr);
    pk.max_pos = l->max_pos;
    pk.eps = l->eps;
    return S2_OK;
}

s2_status s2::attention_forward_packed(s2_attention_layer *l, cudaStream_t st, int L, int Lt, void *vid_out,
                                       float *txt_out)
{
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "layer is NULL");
    l->last_launches = 0;
    if (!l->plan_valid || l->plan_Lt != Lt || L != l->n_video || !l->sc->q.ptr)
        return s2::set_error(S2_INVALID_ARGUMENT, "attention layer: packed forward without a matching pack target");
    if (!vid_out || (Lt > 0 && !txt_out)) return s2::set_error(S2_INVALID_ARGUMENT, "attention layer: NULL buffer");
    DeviceGuard dg(l->device);
    l->last_stream = st;
    return attention_and_text(l, st, Lt, vid_out, txt_out);
}

// The host-buffer forward as a three-stream pipeline over the frame slabs:
// upload (text rows, then slab by slab) on s_in; per slab, once its rows have
// landed, the prologue for the slab's video rows (text rows with the first
// slab) and the attention of the slab's windows on the caller's stream; the
// download of the slab's output rows (a contiguous block of frames) on s_out.
// The text mean follows the last slab. Same kernels, same arithmetic and the
// same results as the serial path; only the copies overlap the compute.
static s2_status forward_host_pipelined(s2_attention_layer *l, cudaStream_t st, const void *vid_qkv,
                                        const void *txt_qkv, s2_dtype io_dtype, int L, int Lt, void *vid_out,
                                        float *txt_out)
{
    const int dim = l->heads * S2_HEAD_DIM;
    const size_t esz = io_dtype == S2_F32 ? 4 : 2;
    const size_t row_in = static_cast<size_t>(3) * dim * esz;
    const size_t row_out = static_cast<size_t>(dim) * (io_dtype == S2_F32 ? 4 : 2);
    const int hw = l->H * l->W;
    AttnScratch &sc = *l->sc;
    const size_t qkv_bytes = static_cast<size_t>(l->n_rows) * dim * 2;
    const size_t txt_bytes = static_cast<size_t>(std::max(l->n_local, 1)) * std::max(Lt, 1) * dim * 2;
    if (!sc.q.ensure(qkv_bytes) || !sc.k.ensure(qkv_bytes) || !sc.v.ensure(qkv_bytes) || !sc.txt_partial.ensure(txt_bytes))
        return s2::set_error(S2_OUT_OF_MEMORY, "forward_host: workspace allocation failed");
    if (!l->d_err.ptr && (!l->d_err.ensure(sizeof(int32_t)) || cudaMemset(l->d_err.ptr, 0, sizeof(int32_t)) != cudaSuccess))
        return s2::set_error(S2_OUT_OF_MEMORY, "forward_host: error word allocation failed");
    l->last_stream = st;
    l->last_launches = 0;
    auto *in = static_cast<char *>(l->d_in_vid.ptr);
    const auto *hin = static_cast<const char *>(vid_qkv);
    auto *hout = static_cast<char *>(vid_out);
    const void *dout = io_dtype == S2_F32 ? l->d_out_vid32.ptr : l->d_out_vid.ptr;
    bool ok = cudaEventRecord(l->ev_start, st) == cudaSuccess && cudaStreamWaitEvent(l->s_in, l->ev_start, 0) == cudaSuccess &&
              cudaStreamWaitEvent(l->s_out, l->ev_start, 0) == cudaSuccess;
    if (ok && Lt > 0)
        ok = cudaMemcpyAsync(l->d_in_txt.ptr, txt_qkv, static_cast<size_t>(Lt) * row_in, cudaMemcpyHostToDevice,
                             l->s_in) == cudaSuccess;
    // A part's rows: one range per frame, or the whole slab at once when the part is the slab.
    auto n_pieces = [&](const s2_attention_layer::Slab &sl, const s2_attention_layer::Part &pt) {
        return pt.h0 == 0 && pt.h1 == l->H ? 1 : sl.t1 - sl.t0;
    };
    auto piece = [&](const s2_attention_layer::Slab &sl, const s2_attention_layer::Part &pt, int k, size_t &a,
                     size_t &n) {
        if (pt.h0 == 0 && pt.h1 == l->H) {
            a = static_cast<size_t>(sl.t0) * hw, n = static_cast<size_t>(sl.t1 - sl.t0) * hw;
        } else {
            a = static_cast<size_t>(sl.t0 + k) * hw + static_cast<size_t>(pt.h0) * l->W;
            n = static_cast<size_t>(pt.h1 - pt.h0) * l->W;
        }
    };
    {
        size_t pi = 0;
        for (size_t i = 0; ok && i < l->slabs.size(); ++i)
            for (const auto &pt : l->slabs[i].parts) {
                for (int k = 0; ok && k < n_pieces(l->slabs[i], pt); ++k) {
                    size_t a = 0, n = 0;
                    piece(l->slabs[i], pt, k, a, n);
                    ok = cudaMemcpyAsync(in + a * row_in, hin + a * row_in, n * row_in, cudaMemcpyHostToDevice,
                                         l->s_in) == cudaSuccess;
                }
                ok = ok && cudaEventRecord(l->ev_in[pi++], l->s_in) == cudaSuccess;
            }
    }
    if (!ok) return s2::set_error(S2_INFERENCE_FAILED, "forward_host: upload failed");
    size_t part_idx = 0;
    bool text_done = false;
    for (size_t i = 0; i < l->slabs.size(); ++i) {
        const auto &sl = l->slabs[i];
        for (const auto &pt : sl.parts) {
            if (cudaStreamWaitEvent(st, l->ev_in[part_idx], 0) != cudaSuccess)
                return s2::set_error(S2_INFERENCE_FAILED, "forward_host: stream wait failed");
            s2_status rc = S2_OK;
            for (int k = 0; k < n_pieces(sl, pt); ++k) {
                size_t a = 0, n = 0;
                piece(sl, pt, k, a, n);
                rc = s2::qk_norm_rope_range(st, in, l->d_in_txt.ptr, io_dtype, l->heads, l->eps, l->gammas(),
                                            l->d_rope.ptr, static_cast<const s2_row *>(l->d_rows.ptr), l->n_rows,
                                            l->mode, static_cast<int>(a), static_cast<int>(a + n), text_done ? 0 : 1,
                                            sc.q.ptr, sc.k.ptr, sc.v.ptr);
                if (rc != S2_OK) return rc;
                text_done = true;
                l->last_launches++;
            }
            rc = s2_window_attention(st, l->mode, sc.q.ptr, sc.k.ptr, sc.v.ptr, l->heads, l->n_rows,
                                     static_cast<const int32_t *>(l->d_cu.ptr), l->n_local, Lt,
                                     static_cast<const s2_row *>(l->d_rows.ptr),
                                     static_cast<const int32_t *>(l->d_slab_work.ptr) + pt.work_off, pt.n_work,
                                     l->d_out_vid.ptr, sc.txt_partial.ptr, static_cast<int32_t *>(l->d_err.ptr));
            if (rc != S2_OK) return rc;
            l->last_launches++;
            if (io_dtype == S2_F32) {
                for (int k = 0; k < n_pieces(sl, pt); ++k) {
                    size_t a = 0, n = 0;
                    piece(sl, pt, k, a, n);
                    rc = s2::to_f32(st, l->mode, static_cast<const char *>(l->d_out_vid.ptr) + a * dim * 2,
                                    static_cast<long long>(n) * dim, static_cast<float *>(l->d_out_vid32.ptr) + a * dim);
                    if (rc != S2_OK) return rc;
                    l->last_launches++;
                }
            }
            bool ok2 = cudaEventRecord(l->ev_cmp[part_idx], st) == cudaSuccess &&
                       cudaStreamWaitEvent(l->s_out, l->ev_cmp[part_idx], 0) == cudaSuccess;
            ++part_idx;
            for (int k = 0; ok2 && k < n_pieces(sl, pt); ++k) {
                size_t a = 0, n = 0;
                piece(sl, pt, k, a, n);
                ok2 = cudaMemcpyAsync(hout + a * row_out, static_cast<const char *>(dout) + a * row_out, n * row_out,
                                      cudaMemcpyDeviceToHost, l->s_out) == cudaSuccess;
            }
            if (!ok2) return s2::set_error(S2_INFERENCE_FAILED, "forward_host: download failed");
        }
    }
    if (Lt > 0) {
        const s2_status rc = s2_text_window_sum(st, l->mode, sc.txt_partial.ptr, l->n_local, Lt, dim,
                                                1.f / static_cast<float>(l->n_total_windows), 0,
                                                static_cast<float *>(l->d_out_txt.ptr));
        if (rc != S2_OK) return rc;
        l->last_launches++;
        if (cudaMemcpyAsync(txt_out, l->d_out_txt.ptr, static_cast<size_t>(Lt) * dim * 4, cudaMemcpyDeviceToHost, st) !=
            cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "forward_host: text download failed");
    }
    if (cudaEventRecord(l->ev_out, l->s_out) != cudaSuccess || cudaStreamWaitEvent(st, l->ev_out, 0) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "forward_host: stream join failed");
    const cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "forward_host: stream failed: %s", cudaGetErrorString(e));
    (void)L;
    int code = 0;
    return s2_attention_layer_device_error(l, &code);
}

static s2_status forward_host_serial(s2_attention_layer *l, cudaStream_t st, const void *vid_qkv, const void *txt_qkv,
                                     s2_dtype io_dtype, int L, int Lt, void *vid_out, float *txt_out);

extern "C" s2_status s2_attention_layer_forward_host(s2_attention_layer *l, void *stream, const void *vid_qkv,
                                                     const void *txt_qkv, s2_dtype io_dtype, int L, int Lt,
                                                     const int32_t *vid_shape, void *vid_out, float *txt_out)
{
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "layer is NULL");
    if (!vid_shape || !vid_qkv || !vid_out || (Lt > 0 && (!txt_qkv || !txt_out)) || L <= 0 || Lt < 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "forward_host: NULL buffer or bad size");
    const s2_dtype mode_dtype = l->mode == S2_MODE_BF16_REF ? S2_BF16 : S2_F16;
    if (io_dtype != S2_F32 && io_dtype != mode_dtype)
        return s2::set_error(S2_UNSUPPORTED, "forward_host: io dtype must be f32 or the mode's 16-bit type");
    // The shape blob is authoritative on this path (the CPU forward reads vid_shape).
    s2_status rc = s2_attention_layer_set_runtime_shape(l, vid_shape[0], vid_shape[1], vid_shape[2]);
    if (rc != S2_OK) return rc;
    if (L != l->T * l->H * l->W)
        return s2::set_error(S2_INVALID_ARGUMENT, "forward_host: vid rows %d != T*H*W", L);
    DeviceGuard g(l->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int dim = l->heads * S2_HEAD_DIM;
    const size_t esz = io_dtype == S2_F32 ? 4 : 2;
    const size_t in_vid = static_cast<size_t>(L) * 3 * dim * esz, in_txt = static_cast<size_t>(Lt) * 3 * dim * esz;
    const size_t out_vid16 = static_cast<size_t>(L) * dim * 2;
    if (!l->d_in_vid.ensure(in_vid) || !l->d_in_txt.ensure(std::max<size_t>(in_txt, 16)) ||
        !l->d_out_vid.ensure(out_vid16) || !l->d_out_txt.ensure(std::max<size_t>(static_cast<size_t>(Lt) * dim * 4, 16)) ||
        (io_dtype == S2_F32 && !l->d_out_vid32.ensure(static_cast<size_t>(L) * dim * 4)))
        return s2::set_error(S2_OUT_OF_MEMORY, "forward_host: staging allocation failed");
    if (!l->loaded || !l->shape_valid)
        return s2::set_error(S2_NOT_LOADED, "attention layer: weights or runtime shape not set");
    rc = l->build_plan(Lt, st);
    if (rc != S2_OK) return rc;
    // Once a copy touching the caller's host buffers is queued, an error return
    // first waits for the copies in flight, so the caller may free its buffers
    // as soon as the call returns.
    auto drain = [&](s2_status s) {
        if (s != S2_OK) {
            if (l->s_in) cudaStreamSynchronize(l->s_in);
            if (l->s_out) cudaStreamSynchronize(l->s_out);
            cudaStreamSynchronize(st);
        }
        return s;
    };
    if (l->build_slabs() && l->ensure_pipeline_objects(l->n_parts()))
        return drain(forward_host_pipelined(l, st, vid_qkv, txt_qkv, io_dtype, L, Lt, vid_out, txt_out));
    return drain(forward_host_serial(l, st, vid_qkv, txt_qkv, io_dtype, L, Lt, vid_out, txt_out));
}

// The host-buffer forward without the pipeline (window subsets): copies in,
// the device forward, copies out, one stream.
static s2_status forward_host_serial(s2_attention_layer *l, cudaStream_t st, const void *vid_qkv, const void *txt_qkv,
                                     s2_dtype io_dtype, int L, int Lt, void *vid_out, float *txt_out)
{
    const int dim = l->heads * S2_HEAD_DIM;
    const size_t esz = io_dtype == S2_F32 ? 4 : 2;
    const size_t in_vid = static_cast<size_t>(L) * 3 * dim * esz, in_txt = static_cast<size_t>(Lt) * 3 * dim * esz;
    const size_t out_vid16 = static_cast<size_t>(L) * dim * 2;
    void *stream = st;
    s2_status rc = S2_OK;
    if (cudaMemcpyAsync(l->d_in_vid.ptr, vid_qkv, in_vid, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        (Lt > 0 && cudaMemcpyAsync(l->d_in_txt.ptr, txt_qkv, in_txt, cudaMemcpyHostToDevice, st) != cudaSuccess))
        return s2::set_error(S2_INFERENCE_FAILED, "forward_host: H2D copy failed");
    // Rows of windows outside a subset are not written by the kernel: keep them zero.
    if (!l->subset.empty() && cudaMemsetAsync(l->d_out_vid.ptr, 0, out_vid16, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "forward_host: memset failed");
    rc = s2_attention_layer_forward(l, stream, l->d_in_vid.ptr, io_dtype, L, l->d_in_txt.ptr, Lt, l->d_out_vid.ptr,
                                    static_cast<float *>(l->d_out_txt.ptr));
    if (rc != S2_OK) return rc;
    const void *vsrc = l->d_out_vid.ptr;
    size_t vbytes = out_vid16;
    if (io_dtype == S2_F32) {
        rc = s2::to_f32(st, l->mode, l->d_out_vid.ptr, static_cast<long long>(L) * dim,
                        static_cast<float *>(l->d_out_vid32.ptr));
        if (rc != S2_OK) return rc;
        l->last_launches++;
        vsrc = l->d_out_vid32.ptr;
        vbytes = static_cast<size_t>(L) * dim * 4;
    }
    if (cudaMemcpyAsync(vid_out, vsrc, vbytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        (Lt > 0 && cudaMemcpyAsync(txt_out, l->d_out_txt.ptr, static_cast<size_t>(Lt) * dim * 4,
                                   cudaMemcpyDeviceToHost, st) != cudaSuccess))
        return s2::set_error(S2_INFERENCE_FAILED, "forward_host: D2H copy failed");
    const cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "forward_host: stream failed: %s", cudaGetErrorString(e));
    int code = 0;
    return s2_attention_layer_device_error(l, &code);
}

extern "C" s2_status s2_attention_layer_device_error(s2_attention_layer *l, int *code)
{
    if (!l || !code) return s2::set_error(S2_INVALID_ARGUMENT, "NULL argument");
    *code = 0;
    if (!l->d_err.ptr) return S2_OK;
    DeviceGuard g(l->device);
    cudaError_t e = cudaStreamSynchronize(l->last_stream);
    int32_t h = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&h, l->d_err.ptr, sizeof h, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "device error query failed: %s", cudaGetErrorString(e));
    *code = h;
    if (h != 0) {
        cudaMemset(l->d_err.ptr, 0, sizeof(int32_t));
        return s2::set_error(S2_INFERENCE_FAILED, "attention kernel reported device error %d (bounded wait timed out)",
                             h);
    }
    return S2_OK;
}

// ---- debug capture (the block's set_debug_tensors) -----------------------------

namespace {

__device__ __forceinline__ float load_f(const void *p, size_t i, int dtype)
{
    if (dtype == S2_F32) return static_cast<const float *>(p)[i];
    if (dtype == S2_F16) return __half2float(static_cast<const __half *>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
}

// packed [heads][n_rows][128] fp16 -> [n_rows][heads * 128] fp32
__global__ void packed_rows_kernel(const __half *__restrict__ p, int heads, int n_rows, float *__restrict__ out)
{
    const long long n = 1LL * n_rows * heads * S2_HEAD_DIM;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x) {
        const int row = static_cast<int>(i / (heads * S2_HEAD_DIM)), c = static_cast<int>(i % (heads * S2_HEAD_DIM));
        const int h = c / S2_HEAD_DIM, d = c % S2_HEAD_DIM;
        out[i] = __half2float(p[(static_cast<size_t>(h) * n_rows + row) * S2_HEAD_DIM + d]);
    }
}

// the per-window output of every packed row: video rows from vid_out, text rows
// from their window's text slab (the values the text mean sums)
__global__ void window_outputs_kernel(const s2_row *__restrict__ rows, const int32_t *__restrict__ cu, int n_windows,
                                      int n_rows, int text_len, int dim, const void *vid_out, const void *txt_partial,
                                      int dtype, float *__restrict__ out)
{
    const long long n = 1LL * n_rows * dim;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x) {
        const int r = static_cast<int>(i / dim), c = static_cast<int>(i % dim);
        const int src = rows[r].src;
        if (src >= 0) {
            out[i] = load_f(vid_out, static_cast<size_t>(src) * dim + c, dtype);
        } else {
            int lo = 0, hi = n_windows - 1;  // last window with cu[w] <= r
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (cu[mid] <= r) lo = mid; else hi = mid - 1;
            }
            out[i] = load_f(txt_partial, (static_cast<size_t>(lo) * text_len + (-src - 1)) * dim + c, dtype);
        }
    }
}

// x * (1 / sqrt(mean(x^2) + eps)) * gamma per (row, head) of the q and k parts of
// [n][3 dim] rows, before RoPE and rounding (the reference's normalized values,
// seedvr2_dit_block.cpp:942-952: double sum, float scale, no contraction)
__global__ void norm_capture_kernel(const void *qkv, int dtype, int n, int heads, float eps, const float *__restrict__ gq,
                                    const float *__restrict__ gk, float *__restrict__ out_q, float *__restrict__ out_k)
{
    const int dim = heads * S2_HEAD_DIM;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < 2 * n * heads; t += gridDim.x * blockDim.x) {
        const int part = t / (n * heads), rh = t % (n * heads), row = rh / heads, h = rh % heads;
        float *out = part == 0 ? out_q : out_k;
        if (!out) continue;
        const float *g = part == 0 ? gq : gk;
        const size_t base = static_cast<size_t>(row) * 3 * dim + static_cast<size_t>(part) * dim + h * S2_HEAD_DIM;
        double ss = 0.0;
        for (int d = 0; d < S2_HEAD_DIM; ++d) {
            const float x = load_f(qkv, base + d, dtype);
            ss += static_cast<double>(x) * x;
        }
        const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(static_cast<float>(ss / S2_HEAD_DIM), eps)));
        for (int d = 0; d < S2_HEAD_DIM; ++d)
            out[static_cast<size_t>(row) * dim + h * S2_HEAD_DIM + d] =
                __fmul_rn(__fmul_rn(load_f(qkv, base + d, dtype), inv), g[d]);
    }
}

int grid_for_n(long long n) { return static_cast<int>(std::min<long long>((n + 255) / 256, 4096)); }

}  // namespace

namespace s2 {

int attention_debug_rows(const s2_attention_layer *l) { return l && l->plan_valid ? l->n_rows : 0; }

s2_status attention_debug_capture(s2_attention_layer *l, cudaStream_t st, const void *vid_qkv, s2_dtype in_dtype,
                                  int L, const void *txt_qkv, int Lt, const void *vid_out, float *att_q, float *att_k,
                                  float *att_v, float *att_o, float *nq_vid, float *nk_vid, float *nq_txt,
                                  float *nk_txt)
{
    if (!l || !l->plan_valid) return set_error(S2_NOT_LOADED, "debug capture: the layer has not run");
    DeviceGuard g(l->device);
    const int dim = l->heads * S2_HEAD_DIM;
    const long long n = 1LL * l->n_rows * dim;
    const AttnScratch &sc = *l->sc;
    const __half *packed[3] = {static_cast<const __half *>(sc.q.ptr), static_cast<const __half *>(sc.k.ptr),
                               static_cast<const __half *>(sc.v.ptr)};
    float *outs[3] = {att_q, att_k, att_v};
    for (int i = 0; i < 3; ++i)
        if (outs[i]) packed_rows_kernel<<<grid_for_n(n), 256, 0, st>>>(packed[i], l->heads, l->n_rows, outs[i]);
    const int out_dtype = l->mode == S2_MODE_BF16_REF ? S2_BF16 : S2_F16;
    if (att_o)
        window_outputs_kernel<<<grid_for_n(n), 256, 0, st>>>(static_cast<const s2_row *>(l->d_rows.ptr),
                                                              static_cast<const int32_t *>(l->d_cu.ptr), l->n_local,
                                                              l->n_rows, Lt, dim, vid_out, sc.txt_partial.ptr,
                                                              out_dtype, att_o);
    const float *gm = l->gammas();  // [4][128]: q_vid, k_vid, q_txt, k_txt
    if (nq_vid || nk_vid)
        norm_capture_kernel<<<grid_for_n(2LL * L * l->heads), 256, 0, st>>>(vid_qkv, in_dtype, L, l->heads, l->eps, gm,
                                                                          gm + 128, nq_vid, nk_vid);
    if (Lt > 0 && (nq_txt || nk_txt))
        norm_capture_kernel<<<grid_for_n(2LL * Lt * l->heads), 256, 0, st>>>(txt_qkv, in_dtype, Lt, l->heads, l->eps,
                                                                           gm + 256, gm + 384, nq_txt, nk_txt);
    return cudaGetLastError() == cudaSuccess ? S2_OK : set_error(S2_INFERENCE_FAILED, "debug capture: launch failed");
}

void share_attention_scratch(s2_attention_layer *dst, const s2_attention_layer *src)
{
    if (dst && src && dst != src) dst->sc = src->sc;
}
}  // namespace s2
