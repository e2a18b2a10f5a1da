// TEST INFRASTRUCTURE ONLY -- builds oracle/_ref/libs2ref.so, the reference's
// OWN CPU code for the hot path, used by tests and by bench.py's cpu_baseline /
// --impl reference arm as the checker and timed baseline. Never shipped.
//
// This translation unit #includes, unmodified and from where they lie under the
// reference tree, the two reference layer sources:
//   src/layers/seedvr2_dit_block.cpp                 (SeedVR2DiTBlock, CPU path)
//   src/layers/dynamic_framewise_spatial_attention.cpp (VAE mid-block attention)
// compiled with NCNN_VULKAN=0 against the ncnn-API shim in oracle/ncnn_shim/.
// `private` is widened to `public` for the reference headers only, so the
// harness can call SeedVR2DiTBlock::make_windows / ::attention directly and set
// the QK-norm gammas and RoPE frequencies without synthesising a full model bin.
// Standard headers are included first so the access override cannot reach them.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <memory>
#include <string>
#include <vector>

#include "layer.h"
#include "mat.h"

#define private public
#define protected public
#include "layers/seedvr2_dit_block.cpp"
#include "layers/dynamic_framewise_spatial_attention.cpp"
#undef private
#undef protected

namespace {

ncnn::Mat mat_from(const float* src, int w, int h)
{
    ncnn::Mat m(w, h);
    std::memcpy(m.data, src, sizeof(float) * (size_t)w * h);
    return m;
}

ncnn::Mat vec_from(const float* src, int w)
{
    ncnn::Mat m(w);
    std::memcpy(m.data, src, sizeof(float) * (size_t)w);
    return m;
}

void copy_out(const ncnn::Mat& m, float* dst)
{
    if (dst && !m.empty()) std::memcpy(dst, m.data, sizeof(float) * (size_t)m.w * m.h);
}

} // namespace

extern "C" {

// SeedVR2DiTBlock::make_windows (seedvr2_dit_block.cpp:827-868).
// Writes {t0,t1,h0,h1,w0,w1} per window into `out` (capacity `cap` windows);
// returns the window count (may exceed cap; nothing past cap is written).
int ref_make_windows(int frames, int height, int width, int shifted, int* out, int cap)
{
    SeedVR2DiTBlock layer;
    layer.shifted_window = shifted != 0;
    const std::vector<SeedVR2DiTBlock::Window> windows = layer.make_windows(frames, height, width);
    for (size_t i = 0; i < windows.size() && (int)i < cap; i++)
    {
        const SeedVR2DiTBlock::Window& w = windows[i];
        int* o = out + 6 * i;
        o[0] = w.t0; o[1] = w.t1; o[2] = w.h0; o[3] = w.h1; o[4] = w.w0; o[5] = w.w1;
    }
    return (int)windows.size();
}

// SeedVR2DiTBlock::attention (seedvr2_dit_block.cpp:870-1091): QK-RMSNorm,
// MM-RoPE, bf16 rounding, joint video+text window attention, text mean.
//   vid_qkv [L, 3*heads*head_dim], txt_qkv [Lt, 3*heads*head_dim] fp32.
//   head_count <= heads restricts the computed heads to 0..head_count-1 (the
//   CPU-baseline sample); the other output columns stay zero.
//   dbg_* (optional, may be null) receive the reference's debug captures
//   [sum_w (L_w+Lt), heads*head_dim]: rounded q/k/v and the rounded output.
// Returns the reference's status (0 ok, -1 bad shape, -100 alloc).
int ref_attention(const float* vid_qkv, int L, const float* txt_qkv, int Lt,
                  int frames, int height, int width, int heads, int head_dim, int shifted, float eps,
                  const float* norm_q_vid, const float* norm_k_vid,
                  const float* norm_q_txt, const float* norm_k_txt, const float* freqs21,
                  int num_threads, int head_count,
                  float* vid_out, float* txt_out,
                  float* dbg_q, float* dbg_k, float* dbg_v, float* dbg_o, int* dbg_rows)
{
    SeedVR2DiTBlock layer;
    layer.dim = heads * head_dim;
    layer.heads = head_count > 0 && head_count < heads ? head_count : heads;
    layer.head_dim = head_dim;
    layer.shifted_window = shifted != 0;
    layer.norm_eps = eps;
    layer.rope_freqs = vec_from(freqs21, 21);
    layer.vid_weights.norm_q = vec_from(norm_q_vid, head_dim);
    layer.vid_weights.norm_k = vec_from(norm_k_vid, head_dim);
    layer.txt_weights.norm_q = vec_from(norm_q_txt, head_dim);
    layer.txt_weights.norm_k = vec_from(norm_k_txt, head_dim);

    const int dim3 = 3 * heads * head_dim;
    ncnn::Mat vq = mat_from(vid_qkv, dim3, L);
    ncnn::Mat tq = mat_from(txt_qkv, dim3, Lt);
    ncnn::Mat shape(3);
    ((int*)shape.data)[0] = frames;
    ((int*)shape.data)[1] = height;
    ((int*)shape.data)[2] = width;

    SeedVR2DiTBlockDebugTensors dbg;
    const bool want_dbg = dbg_q || dbg_k || dbg_v || dbg_o || dbg_rows;
    if (want_dbg) layer.set_debug_tensors(&dbg);

    ncnn::Option opt;
    opt.num_threads = num_threads > 0 ? num_threads : 1;
    ncnn::Mat vo, to;
    const int ret = layer.attention(vq, tq, shape, layer.vid_weights, layer.txt_weights, vo, to, opt);
    if (ret != 0) return ret;
    copy_out(vo, vid_out);
    copy_out(to, txt_out);
    if (want_dbg)
    {
        if (dbg_rows) *dbg_rows = dbg.attention_q.h;
        copy_out(dbg.attention_q, dbg_q);
        copy_out(dbg.attention_k, dbg_k);
        copy_out(dbg.attention_v, dbg_v);
        copy_out(dbg.attention_output, dbg_o);
    }
    return 0;
}

// SeedVR2DiTBlock::load_param / load_model / forward (seedvr2_dit_block.cpp:
// 643-688, 1114-1267): the whole block through the public layer API.
// `weights` is the ModelBin stream in load_model order (all fp32).
int ref_block_forward_debug(int block_index, int shared, int last, int shifted,
                            int dim, int heads, int head_dim, int mlp_hidden, float eps,
                            const float* weights, size_t n_weights,
                            const float* vid, int L, const float* txt, int Lt, const float* emb,
                            int frames, int height, int width, int num_threads,
                            float* vid_out, float* txt_out, float** captures, int* capture_rows);

int ref_block_forward(int block_index, int shared, int last, int shifted,
                      int dim, int heads, int head_dim, int mlp_hidden, float eps,
                      const float* weights, size_t n_weights,
                      const float* vid, int L, const float* txt, int Lt, const float* emb,
                      int frames, int height, int width, int num_threads,
                      float* vid_out, float* txt_out)
{
    return ref_block_forward_debug(block_index, shared, last, shifted, dim, heads, head_dim, mlp_hidden, eps,
                                   weights, n_weights, vid, L, txt, Lt, emb, frames, height, width, num_threads,
                                   vid_out, txt_out, nullptr, nullptr);
}

// The same with the layer's debug capture (set_debug_tensors,
// seedvr2_dit_block.h:20-36, 58): captures[0..13] receive, when non-NULL,
// qkv_vid, qkv_txt, norm_q_vid, norm_q_txt, norm_k_vid, norm_k_txt,
// attention_q, attention_k, attention_v, attention_output, projected_vid,
// projected_txt, output_vid, output_txt ([rows][channels] each, the
// SeedVR2DiTBlockDebugTensors order); *capture_rows = packed attention rows.
int ref_block_forward_debug(int block_index, int shared, int last, int shifted,
                            int dim, int heads, int head_dim, int mlp_hidden, float eps,
                            const float* weights, size_t n_weights,
                            const float* vid, int L, const float* txt, int Lt, const float* emb,
                            int frames, int height, int width, int num_threads,
                            float* vid_out, float* txt_out, float** captures, int* capture_rows)
{
    SeedVR2DiTBlock layer;
    ncnn::ParamDict pd;
    pd.set(0, block_index);
    pd.set(1, shared);
    pd.set(2, last);
    pd.set(3, shifted);
    pd.set(4, dim);
    pd.set(5, heads);
    pd.set(6, head_dim);
    pd.set(7, mlp_hidden);
    pd.set(8, eps);
    if (layer.load_param(pd) != 0) return -1;
    ncnn::ModelBinFromFloats mb(weights, n_weights);
    if (layer.load_model(mb) != 0) return -100;
    if (mb.consumed() != n_weights) return -1;
    ncnn::Option opt;
    opt.num_threads = num_threads > 0 ? num_threads : 1;
    if (layer.create_pipeline(opt) != 0) return -100;

    std::vector<ncnn::Mat> bottom(4), top(2);
    bottom[0] = mat_from(vid, dim, L);
    bottom[1] = mat_from(txt, dim, Lt);
    bottom[2] = vec_from(emb, dim * 6);
    ncnn::Mat shape(3);
    ((int*)shape.data)[0] = frames;
    ((int*)shape.data)[1] = height;
    ((int*)shape.data)[2] = width;
    bottom[3] = shape;
    layer.set_runtime_shape(frames, height, width);
    SeedVR2DiTBlockDebugTensors dbg;
    if (captures) layer.set_debug_tensors(&dbg);
    const int ret = layer.forward(bottom, top, opt);
    layer.destroy_pipeline(opt);
    if (ret != 0) return ret;
    copy_out(top[0], vid_out);
    copy_out(top[1], txt_out);
    if (captures) {
        const ncnn::Mat* m[14] = {&dbg.qkv_vid, &dbg.qkv_txt, &dbg.norm_q_vid, &dbg.norm_q_txt, &dbg.norm_k_vid,
                                  &dbg.norm_k_txt, &dbg.attention_q, &dbg.attention_k, &dbg.attention_v,
                                  &dbg.attention_output, &dbg.projected_vid, &dbg.projected_txt, &dbg.output_vid,
                                  &dbg.output_txt};
        for (int i = 0; i < 14; i++) copy_out(*m[i], captures[i]);
        if (capture_rows) *capture_rows = dbg.attention_q.h;
    }
    return 0;
}

// DynamicFramewiseSpatialAttention (dynamic_framewise_spatial_attention.cpp:
// 50-210). x / y are dense [C][T][H][W] fp32; weights in load_model order
// (norm_bias, norm_weight, k_b, k_W, out_b, out_W, q_b, q_W, v_b, v_W).
int ref_vae_attention(int channels, int frames, int height, int width,
                      const float* weights, size_t n_weights, const float* x, int num_threads, float* y)
{
    DynamicFramewiseSpatialAttention layer;
    ncnn::ParamDict pd;
    ncnn::Mat shape(1);
    ((int*)shape.data)[0] = channels;
    pd.set(10, shape);
    if (layer.load_param(pd) != 0) return -1;
    ncnn::ModelBinFromFloats mb(weights, n_weights);
    if (layer.load_model(mb) != 0) return -100;
    if (mb.consumed() != n_weights) return -1;

    ncnn::Mat in(width, height, frames, channels, 4u, 1);
    const size_t plane = (size_t)width * height * frames;
    for (int c = 0; c < channels; c++)
        std::memcpy((float*)in.channel(c), x + plane * c, plane * sizeof(float));
    ncnn::Option opt;
    opt.num_threads = num_threads > 0 ? num_threads : 1;
    ncnn::Mat out;
    const int ret = layer.forward(in, out, opt);
    if (ret != 0) return ret;
    for (int c = 0; c < channels; c++)
        std::memcpy(y + plane * c, (const float*)out.channel(c), plane * sizeof(float));
    return 0;
}

} // extern "C"
