// TEST INFRASTRUCTURE ONLY -- part of oracle/_ref/libs2ref.so (see
// ref_harness.cpp). This translation unit #includes, unmodified and from where
// it lies under the reference tree, src/layers/seedvr2_dit_output.cpp
// (SeedVR2DiTOutput, CPU path; NCNN_VULKAN=0), and drives it through its
// public layer API (a separate translation unit for the same reason as
// ref_input.cpp).
#include <cmath>
#include <cstddef>
#include <cstring>
#include <vector>

#include "layer.h"
#include "mat.h"

#include "layers/seedvr2_dit_output.cpp"

extern "C" {

// SeedVR2DiTOutput load_param / load_model / forward
// (seedvr2_dit_output.cpp:256-270, 349-431). video [frames*H*W][dim] on the
// patched grid, emb [6 dim]; out [frames*2H*2W][oc] (token-major).
int ref_dit_output(int dim, int oc, float eps, const float *weights, size_t n_weights, const float *video,
                   int frames, int height, int width, const float *emb, int num_threads, float *out)
{
    SeedVR2DiTOutput layer;
    ncnn::ParamDict pd;
    pd.set(0, dim);
    pd.set(1, oc);
    pd.set(2, eps);
    if (layer.load_param(pd) != 0) return -1;
    ncnn::ModelBinFromFloats mb(weights, n_weights);
    if (layer.load_model(mb) != 0) return -100;
    if (mb.consumed() != n_weights) return -1;
    ncnn::Option opt;
    opt.num_threads = num_threads > 0 ? num_threads : 1;
    if (layer.create_pipeline(opt) != 0) return -100;
    const int L = frames * height * width;
    std::vector<ncnn::Mat> bottom(3), top(2);
    bottom[0] = ncnn::Mat(dim, L);
    std::memcpy(bottom[0].data, video, sizeof(float) * (size_t)dim * L);
    bottom[1] = ncnn::Mat(dim * 6);
    std::memcpy(bottom[1].data, emb, sizeof(float) * (size_t)dim * 6);
    bottom[2] = ncnn::Mat(3);
    ((int *)bottom[2].data)[0] = frames;
    ((int *)bottom[2].data)[1] = height;
    ((int *)bottom[2].data)[2] = width;
    const int ret = layer.forward(bottom, top, opt);
    layer.destroy_pipeline(opt);
    if (ret != 0) return ret;
    std::memcpy(out, top[0].data, sizeof(float) * (size_t)top[0].w * top[0].h);
    return 0;
}

}  // extern "C"
