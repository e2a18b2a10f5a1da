// TEST INFRASTRUCTURE ONLY -- part of oracle/_ref/libs2ref.so (see
// ref_harness.cpp). This translation unit #includes, unmodified and from where
// it lies under the reference tree, src/model/sampler.cpp (EulerSampler, CPU
// path; NCNN_VULKAN=0) and drives its public methods on dense fp32 4D Mats
// [C][T][H][W] (a separate translation unit, like ref_input.cpp, so that its
// anonymous-namespace helpers do not meet the layer sources').
#include <cstddef>
#include <cstring>
#include <string>

#include "mat.h"

#include "model/sampler.cpp"

namespace {

ncnn::Mat mat4(const float *src, int C, int T, int H, int W)
{
    ncnn::Mat m(W, H, T, C, 4u, 1);
    for (int c = 0; c < C; ++c)
        for (int t = 0; t < T; ++t)
            for (int y = 0; y < H; ++y)
                std::memcpy(m.channel(c).depth(t).row(y), src + (((size_t)c * T + t) * H + y) * W, sizeof(float) * W);
    return m;
}

void unmat4(const ncnn::Mat &m, float *dst)
{
    for (int c = 0; c < m.c; ++c)
        for (int t = 0; t < m.d; ++t)
            for (int y = 0; y < m.h; ++y)
                std::memcpy(dst + (((size_t)c * m.d + t) * m.h + y) * m.w, m.channel(c).depth(t).row(y),
                            sizeof(float) * m.w);
}

}  // namespace

extern "C" {

// EulerSampler(steps).timesteps() (sampler.cpp:181-187)
int ref_sampler_timesteps(int steps, float *out)
{
    seedvr2::EulerSampler s(steps);
    const std::vector<float> &t = s.timesteps();
    std::memcpy(out, t.data(), sizeof(float) * t.size());
    return static_cast<int>(t.size());
}

// EulerSampler::apply_cfg (sampler.cpp:200-238)
int ref_apply_cfg(const float *pos, const float *neg, int C, int T, int H, int W, float scale, float rescale,
                  float *out)
{
    seedvr2::EulerSampler s(1);
    ncnn::Mat o;
    std::string err;
    const int rc = s.apply_cfg(mat4(pos, C, T, H, W), mat4(neg, C, T, H, W), scale, rescale, o, err);
    if (rc == 0) unmat4(o, out);
    return rc;
}

// EulerSampler::step_to (sampler.cpp:240-265)
int ref_step_to(const float *pred, const float *cur, int C, int T, int H, int W, float t, float t_next, float *out)
{
    seedvr2::EulerSampler s(1);
    ncnn::Mat o;
    std::string err;
    const int rc = s.step_to(mat4(pred, C, T, H, W), mat4(cur, C, T, H, W), t, t_next, o, err);
    if (rc == 0) unmat4(o, out);
    return rc;
}

// EulerSampler::endpoint (sampler.cpp:267-286)
int ref_endpoint(const float *pred, const float *cur, int C, int T, int H, int W, float t, float *out)
{
    seedvr2::EulerSampler s(1);
    ncnn::Mat o;
    std::string err;
    const int rc = s.endpoint(mat4(pred, C, T, H, W), mat4(cur, C, T, H, W), t, o, err);
    if (rc == 0) unmat4(o, out);
    return rc;
}

}  // extern "C"
