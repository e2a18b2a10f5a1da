// TEST INFRASTRUCTURE ONLY -- part of oracle/_ref/libs2ref.so (see
// ref_harness.cpp). This translation unit #includes, unmodified and from where
// it lies under the reference tree, src/layers/seedvr2_dit_input.cpp
// (SeedVR2DiTInput, CPU path; NCNN_VULKAN=0), and drives it through its
// public layer API. It is a separate translation unit because the reference's
// layer sources each define the same file-local helpers.
#include <cmath>
#include <cstddef>
#include <cstring>
#include <vector>

#include "layer.h"
#include "mat.h"

#include "layers/seedvr2_dit_input.cpp"

extern "C" {

// SeedVR2DiTInput load_param / load_model / forward
// (seedvr2_dit_input.cpp:207-224, 311-405). video: flat [frames*H*W][vc]
// (the flatten_latent layout), text [Lt][tc]; outputs vid_out
// [frames*(H/2)*(W/2)][dim], txt_out [Lt][dim], emb [ed].
int ref_dit_input(int dim, int vc, int tc, int sd, int ed, const float *weights, size_t n_weights,
                  const float *video, int frames, int height, int width, const float *text, int Lt, float timestep,
                  int num_threads, float *vid_out, float *txt_out, float *emb)
{
    SeedVR2DiTInput layer;
    ncnn::ParamDict pd;
    pd.set(0, dim);
    pd.set(1, vc);
    pd.set(2, tc);
    pd.set(3, sd);
    pd.set(4, ed);
    if (layer.load_param(pd) != 0) return -1;
    ncnn::ModelBinFromFloats mb(weights, n_weights);
    if (layer.load_model(mb) != 0) return -100;
    if (mb.consumed() != n_weights) return -1;
    ncnn::Option opt;
    opt.num_threads = num_threads > 0 ? num_threads : 1;
    if (layer.create_pipeline(opt) != 0) return -100;
    const int L = frames * height * width;
    std::vector<ncnn::Mat> bottom(4), top(4);
    bottom[0] = ncnn::Mat(vc, L);
    std::memcpy(bottom[0].data, video, sizeof(float) * (size_t)vc * L);
    bottom[1] = ncnn::Mat(tc, Lt);
    std::memcpy(bottom[1].data, text, sizeof(float) * (size_t)tc * Lt);
    bottom[2] = ncnn::Mat(1);
    ((float *)bottom[2].data)[0] = timestep;
    bottom[3] = ncnn::Mat(3);
    ((int *)bottom[3].data)[0] = frames;
    ((int *)bottom[3].data)[1] = height;
    ((int *)bottom[3].data)[2] = width;
    const int ret = layer.forward(bottom, top, opt);
    layer.destroy_pipeline(opt);
    if (ret != 0) return ret;
    std::memcpy(vid_out, top[0].data, sizeof(float) * (size_t)top[0].w * top[0].h);
    std::memcpy(txt_out, top[1].data, sizeof(float) * (size_t)top[1].w * top[1].h);
    std::memcpy(emb, top[2].data, sizeof(float) * top[2].total());
    return 0;
}

}  // extern "C"
