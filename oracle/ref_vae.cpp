// TEST INFRASTRUCTURE ONLY -- part of oracle/_ref/libs2ref.so (see
// ref_harness.cpp). This translation unit #includes, unmodified and from where
// they lie under the reference tree, the VAE layers
//   src/layers/dynamic_framewise_group_norm.cpp   (DynamicFramewiseGroupNorm)
//   src/layers/dynamic_space_time_shuffle.cpp     (DynamicSpaceTimeShuffle)
// (CPU paths, NCNN_VULKAN=0) and drives them through their public layer API:
// load_param with the exporter's shape arrays, load_model from a float stream,
// forward on a 4-D [C][T][H][W] blob.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <vector>

#include "layer.h"
#include "mat.h"

#include "layers/dynamic_framewise_group_norm.cpp"
#include "layers/dynamic_space_time_shuffle.cpp"

namespace {

ncnn::Mat blob_from(const float* x, int channels, int frames, int height, int width)
{
    ncnn::Mat in(width, height, frames, channels, 4u, 1);
    const size_t plane = (size_t)width * height * frames;
    for (int c = 0; c < channels; c++)
        std::memcpy((float*)in.channel(c), x + plane * c, plane * sizeof(float));
    return in;
}

void blob_to(const ncnn::Mat& out, float* y)
{
    const size_t plane = (size_t)out.w * out.h * out.d;
    for (int c = 0; c < out.c; c++)
        std::memcpy(y + plane * c, (const float*)out.channel(c), plane * sizeof(float));
}

} // namespace

extern "C" {

// DynamicFramewiseGroupNorm: load_param key 10 = bias shape [C]
// (dynamic_framewise_group_norm.cpp:43-53), load_model bias then weight
// (:55-61), forward (:63-121). x, y: [C][T][H][W].
int ref_group_norm(int channels, int frames, int height, int width, const float* bias, const float* weight,
                   const float* x, int num_threads, float* y)
{
    DynamicFramewiseGroupNorm layer;
    ncnn::ParamDict pd;
    ncnn::Mat shape(1);
    ((int*)shape.data)[0] = channels;
    pd.set(10, shape);
    if (layer.load_param(pd) != 0) return -1;
    std::vector<float> w(bias, bias + channels);
    w.insert(w.end(), weight, weight + channels);
    ncnn::ModelBinFromFloats mb(w.data(), w.size());
    if (layer.load_model(mb) != 0) return -100;
    ncnn::Option opt;
    opt.num_threads = num_threads > 0 ? num_threads : 1;
    ncnn::Mat out;
    const int ret = layer.forward(blob_from(x, channels, frames, height, width), out, opt);
    if (ret != 0) return ret;
    blob_to(out, y);
    return 0;
}

// DynamicSpaceTimeShuffle: load_param key 10 = bias shape [P], key 11 = weight
// shape [P, Cin] (dynamic_space_time_shuffle.cpp:41-55), load_model bias then
// weight (:57-63), forward (:65-130). x: [Cin][T][H][W]; y: [Cin][T'][2H][2W]
// with T' = T * tr - 1 when the temporal ratio tr > 1, else T; *out_frames = T'.
int ref_space_time_shuffle(int in_channels, int projected_channels, int frames, int height, int width,
                           const float* bias, const float* weight, const float* x, int num_threads, float* y,
                           int* out_frames)
{
    DynamicSpaceTimeShuffle layer;
    ncnn::ParamDict pd;
    ncnn::Mat bshape(1), wshape(2);
    ((int*)bshape.data)[0] = projected_channels;
    ((int*)wshape.data)[0] = projected_channels;
    ((int*)wshape.data)[1] = in_channels;
    pd.set(10, bshape);
    pd.set(11, wshape);
    if (layer.load_param(pd) != 0) return -1;
    std::vector<float> w(bias, bias + projected_channels);
    w.insert(w.end(), weight, weight + (size_t)projected_channels * in_channels);
    ncnn::ModelBinFromFloats mb(w.data(), w.size());
    if (layer.load_model(mb) != 0) return -100;
    ncnn::Option opt;
    opt.num_threads = num_threads > 0 ? num_threads : 1;
    ncnn::Mat out;
    const int ret = layer.forward(blob_from(x, in_channels, frames, height, width), out, opt);
    if (ret != 0) return ret;
    if (out_frames) *out_frames = out.d;
    if (y) blob_to(out, y);
    return 0;
}

} // extern "C"
