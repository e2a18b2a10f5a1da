// TEST INFRASTRUCTURE: numerical runner for the C++ layer mirror
// (seedvr2-ncnn-valkan_b200/host/s2_layers.hpp), shaped like the reference's own
// layer runners (tests/dit_block_vulkan_runner.cpp, tests/attention_vulkan_runner.cpp):
// each case builds one layer through load_param / load_model / set_runtime_shape,
// runs forward on the B200 (host blobs), runs the reference's CPU code on the same
// inputs (the reference's layer sources built into oracle/_ref/libs2ref.so, loaded
// with dlopen) and prints max|diff| with PASS / FAIL. Exit status 0 when every case
// and every error-path check passes.
//
// Inputs and weights are the runners' deterministic patterns (restated, as in
// tests/refcases.py): block cases dit_block_vulkan_runner.cpp:213-218 with fill()
// :43-53 and the weight stream :80-119; VAE cases attention_vulkan_runner.cpp:155-160
// with make_input() :83-95 and weights :50-68 in load_model order.
//
// Thresholds are the reference runners' own: max|diff| < 1e-3 for the block, < 1e-4
// for the VAE attention layer. Two more cases compare the 14 debug capture points
// (set_debug_tensors) with the reference's own captures of the same forward.
//
// usage: layer_runner <path to libs2ref.so>
#include <dlfcn.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "s2_layers.hpp"

namespace
{

using RefBlock = int (*)(int, int, int, int, int, int, int, int, float, const float *, size_t, const float *, int,
                         const float *, int, const float *, int, int, int, int, float *, float *);
using RefVae = int (*)(int, int, int, int, const float *, size_t, const float *, int, float *);
using RefBlockDebug = int (*)(int, int, int, int, int, int, int, int, float, const float *, size_t, const float *, int,
                              const float *, int, const float *, int, int, int, int, float *, float *, float **, int *);

struct BlockCase {
    int dim, heads, head_dim, mlp, T, H, W, text_len;
    bool shared, last, shifted;
    const char *name;
};

struct VaeCase {
    int C, T, H, W;
    const char *name;
};

// fill(): ((index + offset) % 11 - 5) * 0.1 over a row-major [rows][cols] blob
void fill_rows(std::vector<float> &v, int cols, int rows, int off)
{
    v.resize(static_cast<size_t>(cols) * rows);
    for (size_t i = 0; i < v.size(); ++i) v[i] = static_cast<float>(static_cast<int>((i + off) % 11) - 5) * 0.1f;
}

void push_vec(std::vector<float> &s, int n, int seed)
{
    for (int i = 0; i < n; ++i) s.push_back(0.01f * static_cast<float>((i + seed) % 9 - 4));
}

void push_ip(std::vector<float> &s, int n_in, int n_out, bool bias, int seed)
{
    const long long n = 1LL * n_in * n_out;
    for (long long i = 0; i < n; ++i) s.push_back(0.005f * static_cast<float>(static_cast<int>((i + seed) % 7) - 3));
    if (bias)
        for (int j = 0; j < n_out; ++j) s.push_back(0.01f * static_cast<float>((j + seed) % 5 - 2));
}

void push_branch(std::vector<float> &s, const BlockCase &tc, int base)
{
    for (int k = 0; k < 6; ++k) push_vec(s, tc.dim, base + k);       // attn / mlp shift, scale, gate
    push_ip(s, tc.dim, 3 * tc.dim, false, base + 6);               // qkv
    push_ip(s, tc.dim, tc.dim, true, base + 7);                    // proj + bias
    push_vec(s, tc.head_dim, base + 8);                            // norm_q
    push_vec(s, tc.head_dim, base + 9);                            // norm_k
    push_ip(s, tc.dim, tc.mlp, false, base + 10);                  // gate
    push_ip(s, tc.dim, tc.mlp, false, base + 11);                  // in
    push_ip(s, tc.mlp, tc.dim, false, base + 12);                  // out
}

double max_abs(const float *a, const float *b, size_t n)
{
    double worst = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double d = std::fabs(static_cast<double>(a[i]) - static_cast<double>(b[i]));
        if (!(d <= worst)) worst = d;  // NaN counts as worst
    }
    return worst;
}

// With `refd` set, both sides capture the reference's 14 debug tensors
// (set_debug_tensors, seedvr2_dit_block.h:20-36) and *debug_worst receives the
// largest per-capture max|diff| relative to its allowance: 2e-3 of the
// capture's scale (this build keeps the QKV projections in fp16), or one bf16
// ulp of it for the bf16-rounded attention captures; <= 1 passes.
int run_block(const BlockCase &tc, RefBlock ref, double &diff, RefBlockDebug refd = nullptr,
              double *debug_worst = nullptr)
{
    std::vector<float> weights;
    push_branch(weights, tc, 0);
    if (!tc.shared) push_branch(weights, tc, 50);
    push_vec(weights, 21, 100);  // RoPE frequencies
    const int L = tc.T * tc.H * tc.W;
    std::vector<float> vid, txt, emb;
    fill_rows(vid, tc.dim, L, 0);
    fill_rows(txt, tc.dim, tc.text_len, 100);
    fill_rows(emb, tc.dim * 6, 1, 200);

    std::vector<float> rv(vid.size()), rt(txt.size());
    s2b200::SeedVR2DiTBlockDebugTensors mine;
    std::vector<std::vector<float>> theirs(14);
    if (refd) {
        // capture sizes: packed rows = sum over windows of (L_w + text_len)
        int n_win = 0, rows = 0;
        s2_make_windows(tc.T, tc.H, tc.W, tc.shifted ? 1 : 0, 0, 0, 0, nullptr, 0, &n_win);
        std::vector<s2_window> wins(n_win);
        s2_make_windows(tc.T, tc.H, tc.W, tc.shifted ? 1 : 0, 0, 0, 0, wins.data(), n_win, &n_win);
        for (const s2_window &w : wins) rows += (w.t1 - w.t0) * (w.h1 - w.h0) * (w.w1 - w.w0) + tc.text_len;
        const int h[14] = {L, tc.text_len, L, tc.text_len, L, tc.text_len, rows, rows, rows, rows,
                           L, tc.text_len, L, tc.text_len};
        float *ptrs[14];
        for (int k = 0; k < 14; ++k) {
            theirs[k].assign(static_cast<size_t>(h[k]) * (k < 2 ? 3 * tc.dim : tc.dim), 0.f);
            ptrs[k] = theirs[k].data();
        }
        int got_rows = 0;
        if (refd(0, tc.shared, tc.last, tc.shifted, tc.dim, tc.heads, tc.head_dim, tc.mlp, 1e-5f, weights.data(),
                 weights.size(), vid.data(), L, txt.data(), tc.text_len, emb.data(), tc.T, tc.H, tc.W, 4, rv.data(),
                 rt.data(), ptrs, &got_rows) != 0 || got_rows != rows)
            return -2;
    } else if (ref(0, tc.shared, tc.last, tc.shifted, tc.dim, tc.heads, tc.head_dim, tc.mlp, 1e-5f, weights.data(),
                   weights.size(), vid.data(), L, txt.data(), tc.text_len, emb.data(), tc.T, tc.H, tc.W, 4, rv.data(),
                   rt.data()) != 0) {
        return -2;
    }

    s2b200::SeedVR2DiTBlock layer;
    s2b200::ParamDict pd;
    pd.set(0, 0);
    pd.set(1, tc.shared ? 1 : 0);
    pd.set(2, tc.last ? 1 : 0);
    pd.set(3, tc.shifted ? 1 : 0);
    pd.set(4, tc.dim);
    pd.set(5, tc.heads);
    pd.set(6, tc.head_dim);
    pd.set(7, tc.mlp);
    pd.set(8, 1e-5f);
    s2b200::ModelBinFromFloats mb(weights.data(), weights.size());
    if (layer.load_param(pd) != 0 || layer.load_model(mb) != 0 || mb.consumed() != weights.size()) {
        std::fprintf(stderr, "load failed: %s\n", layer.last_error().c_str());
        return -1;
    }
    layer.set_runtime_shape(tc.T, tc.H, tc.W);
    if (refd) layer.set_debug_tensors(&mine);
    std::vector<s2b200::Mat> bottom(4), top(2);
    bottom[0].create(tc.dim, L);
    bottom[1].create(tc.dim, tc.text_len);
    bottom[2].create(tc.dim * 6);
    bottom[3].create(3);
    std::memcpy(bottom[0].data, vid.data(), vid.size() * 4);
    std::memcpy(bottom[1].data, txt.data(), txt.size() * 4);
    std::memcpy(bottom[2].data, emb.data(), emb.size() * 4);
    int *shape = bottom[3];
    shape[0] = tc.T, shape[1] = tc.H, shape[2] = tc.W;
    s2b200::Option opt;
    if (layer.forward(bottom, top, opt) != 0) {
        std::fprintf(stderr, "forward failed: %s\n", layer.last_error().c_str());
        return -1;
    }
    diff = std::fmax(max_abs(top[0], rv.data(), rv.size()), max_abs(top[1], rt.data(), rt.size()));
    if (refd && debug_worst) {
        const s2b200::Mat *m[14] = {&mine.qkv_vid, &mine.qkv_txt, &mine.norm_q_vid, &mine.norm_q_txt, &mine.norm_k_vid,
                                    &mine.norm_k_txt, &mine.attention_q, &mine.attention_k, &mine.attention_v,
                                    &mine.attention_output, &mine.projected_vid, &mine.projected_txt,
                                    &mine.output_vid, &mine.output_txt};
        *debug_worst = 0.0;
        for (int k = 0; k < 14; ++k) {
            const std::vector<float> &r = theirs[k];
            if (r.empty()) continue;
            if (m[k]->empty() || static_cast<size_t>(m[k]->w) * m[k]->h != r.size()) {
                *debug_worst = 1e9;
                continue;
            }
            double amax = 0.0;
            for (float v : r) amax = std::fmax(amax, std::fabs(v));
            const double allow = (k >= 6 && k <= 9) ? std::fmax(2e-3 * std::fmax(1.0, amax), amax / 128.0)
                                                    : 2e-3 * std::fmax(1.0, amax);
            *debug_worst = std::fmax(*debug_worst, max_abs(*m[k], r.data(), r.size()) / allow);
        }
    }
    return 0;
}

int run_vae(const VaeCase &tc, RefVae ref, double &diff)
{
    const int C = tc.C, m = C * C;
    auto pattern = [](std::vector<float> &s, int n, float base, float step) {
        for (int i = 0; i < n; ++i) s.push_back(base + step * static_cast<float>(i % 7 - 3));
    };
    // load_model order: norm_bias, norm_weight, k_b, k_W, out_b, out_W, q_b, q_W, v_b, v_W
    std::vector<float> w;
    pattern(w, C, 0.f, 0.02f);
    pattern(w, C, 1.f, 0.02f);
    pattern(w, C, 0.f, 0.01f);
    pattern(w, m, 0.f, 0.005f);
    pattern(w, C, 0.f, 0.01f);
    pattern(w, m, 0.f, 0.005f);
    pattern(w, C, 0.f, 0.01f);
    pattern(w, m, 0.f, 0.005f);
    pattern(w, C, 0.f, 0.01f);
    pattern(w, m, 0.f, 0.005f);
    const size_t plane = static_cast<size_t>(tc.T) * tc.H * tc.W;
    std::vector<float> x(plane * C), ry(plane * C);
    for (size_t i = 0; i < x.size(); ++i) x[i] = static_cast<float>(static_cast<int>(i % 11) - 5) * 0.1f;
    if (ref(C, tc.T, tc.H, tc.W, w.data(), w.size(), x.data(), 4, ry.data()) != 0) return -2;

    s2b200::DynamicFramewiseSpatialAttention layer;
    s2b200::ParamDict pd;
    s2b200::Mat chan(1);
    static_cast<int *>(chan)[0] = C;
    pd.set(10, chan);
    s2b200::ModelBinFromFloats mb(w.data(), w.size());
    if (layer.load_param(pd) != 0 || layer.load_model(mb) != 0) {
        std::fprintf(stderr, "load failed: %s\n", layer.last_error().c_str());
        return -1;
    }
    s2b200::Mat in(tc.W, tc.H, tc.T, C), out;
    for (int c = 0; c < C; ++c) std::memcpy(in.channel(c), x.data() + plane * c, plane * 4);
    s2b200::Option opt;
    if (layer.forward(in, out, opt) != 0) {
        std::fprintf(stderr, "forward failed: %s\n", layer.last_error().c_str());
        return -1;
    }
    diff = 0.0;
    for (int c = 0; c < C; ++c) diff = std::fmax(diff, max_abs(out.channel(c), ry.data() + plane * c, plane));
    return 0;
}

// The reference's error behaviour: -1 for a bad head split and for wrong blob counts / shapes.
bool error_paths()
{
    bool ok = true;
    s2b200::SeedVR2DiTBlock block;
    s2b200::ParamDict pd;
    pd.set(4, 128);
    pd.set(5, 2);
    pd.set(6, 128);  // 2 x 128 != 128
    ok &= block.load_param(pd) == -1;
    pd.set(5, 1);
    pd.set(7, 128);
    ok &= block.load_param(pd) == 0;
    std::vector<s2b200::Mat> three(3), top(2);
    s2b200::Option opt;
    ok &= block.forward(three, top, opt) == -1;
    std::vector<s2b200::Mat> bad(4);
    bad[0].create(64, 8);  // width != dim
    bad[1].create(128, 2);
    bad[2].create(768);
    bad[3].create(3);
    ok &= block.forward(bad, top, opt) == -1;
    s2b200::DynamicFramewiseSpatialAttention vae;
    s2b200::ParamDict vp;
    s2b200::Mat chan(1);
    static_cast<int *>(chan)[0] = 48;  // not a multiple of 32
    vp.set(10, chan);
    ok &= vae.load_param(vp) == -1;
    ok &= vae.load_param(s2b200::ParamDict()) == -1;
    return ok;
}

}  // namespace

int main(int argc, char **argv)
{
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <libs2ref.so>\n", argv[0]);
        return 2;
    }
    void *lib = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
        std::fprintf(stderr, "dlopen: %s\n", dlerror());
        return 2;
    }
    auto ref_block = reinterpret_cast<RefBlock>(dlsym(lib, "ref_block_forward"));
    auto ref_vae = reinterpret_cast<RefVae>(dlsym(lib, "ref_vae_attention"));
    auto ref_block_debug = reinterpret_cast<RefBlockDebug>(dlsym(lib, "ref_block_forward_debug"));
    if (!ref_block || !ref_vae || !ref_block_debug) {
        std::fprintf(stderr, "reference symbols missing\n");
        return 2;
    }
    if (s2_device_check(0) != S2_OK) {
        std::fprintf(stderr, "no usable sm_100 device: %s\n", s2_last_error());
        return 2;
    }
    const BlockCase blocks[] = {
        {128, 1, 128, 128, 2, 2, 2, 3, false, false, false, "dim=128 heads=1 T=2 plain"},
        {128, 1, 128, 128, 2, 2, 2, 3, false, false, true, "shifted (video summed across windows)"},
        {128, 1, 128, 128, 1, 1, 1, 2, true, true, false, "last layer + shared weights, one patch"},
        {256, 2, 128, 128, 3, 2, 2, 4, false, false, false, "dim=256 heads=2 T=3"},
    };
    const VaeCase vaes[] = {
        {32, 2, 4, 4, "C=32 T=2 4x4"},
        {64, 3, 5, 5, "C=64 T=3 5x5"},
        {32, 1, 8, 8, "C=32 T=1 8x8"},
        {64, 2, 3, 5, "C=64 T=2 3x5"},
    };
    int pass = 0, fail = 0;
    int i = 0;
    for (const BlockCase &tc : blocks) {
        double diff = 0.0;
        const int r = run_block(tc, ref_block, diff);
        const bool ok = r == 0 && diff < 1e-3;
        std::printf("[block %d] %s : max|diff| = %.6g %s\n", i++, tc.name, r == 0 ? diff : -1.0, ok ? "PASS" : "FAIL");
        ok ? ++pass : ++fail;
    }
    for (int c : {1, 3}) {  // set_debug_tensors on a shifted and an unshifted case
        double diff = 0.0, worst = 0.0;
        const int r = run_block(blocks[c], ref_block, diff, ref_block_debug, &worst);
        const bool ok = r == 0 && diff < 1e-3 && worst <= 1.0;
        std::printf("[debug %d] 14 capture points vs the reference's : worst diff / allowance = %.4g %s\n", c,
                    r == 0 ? worst : -1.0, ok ? "PASS" : "FAIL");
        ok ? ++pass : ++fail;
    }
    i = 0;
    for (const VaeCase &tc : vaes) {
        double diff = 0.0;
        const int r = run_vae(tc, ref_vae, diff);
        const bool ok = r == 0 && diff < 1e-4;
        std::printf("[vae %d] %s : max|diff| = %.6g %s\n", i++, tc.name, r == 0 ? diff : -1.0, ok ? "PASS" : "FAIL");
        ok ? ++pass : ++fail;
    }
    const bool errs = error_paths();
    std::printf("[errors] reference return codes : %s\n", errs ? "PASS" : "FAIL");
    errs ? ++pass : ++fail;
    std::printf("======== result: %d pass, %d fail ========\n", pass, fail);
    dlclose(lib);
    return fail == 0 ? 0 : 1;
}
