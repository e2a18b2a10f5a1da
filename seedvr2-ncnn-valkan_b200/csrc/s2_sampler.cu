// Euler sampler and classifier-free guidance on the device (the CPU EulerSampler
// of src/model/sampler.cpp and the condition / DiT-input builders of
// src/core/engine.cpp), so that a multi-step, guided sampling loop runs without
// leaving the GPU.
//
// Every update is elementwise over the fp32 latent [C][T][H][W]; the float
// operations are written with explicitly rounded intrinsics in the reference's
// order, so no multiply/add pair is contracted into an FMA. The guidance
// rescale needs two standard deviations (fp64 sum and sum of squares over the
// whole tensor, sampler.cpp:41-62): per-block fp64 partial sums, then one block
// adds the partials in block order and writes the scale factor, which the
// update kernels read from device memory (no host round trip).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "s2_internal.h"
#include "s2_ops.h"

namespace {

constexpr int kStatBlocks = 512;   // partial-sum blocks of the guidance statistics
constexpr int kThreads = 256;

unsigned grid_for(long long n) { return static_cast<unsigned>(std::min<long long>((n + kThreads - 1) / kThreads, 4096)); }

__device__ __forceinline__ float guided(float pos, float neg, float scale)
{
    // neg + scale * (pos - neg)  (sampler.cpp:217-218)
    return __fadd_rn(neg, __fmul_rn(scale, __fsub_rn(pos, neg)));
}

// Per-block fp64 sums of the guided prediction and of the positive one:
// part[b] = {sum g, sum g^2, sum p, sum p^2}.
__global__ void __launch_bounds__(kThreads) cfg_partials_kernel(const float *__restrict__ pos,
                                                                const float *__restrict__ neg, long long n, float scale,
                                                                double4 *__restrict__ part)
{
    double sg = 0.0, qg = 0.0, sp = 0.0, qp = 0.0;
    for (long long i = blockIdx.x * 1LL * kThreads + threadIdx.x; i < n; i += 1LL * gridDim.x * kThreads) {
        const float p = pos[i];
        const float g = guided(p, neg[i], scale);
        sg += g;
        qg += static_cast<double>(g) * g;
        sp += p;
        qp += static_cast<double>(p) * p;
    }
    __shared__ double red[4][kThreads];
    red[0][threadIdx.x] = sg;
    red[1][threadIdx.x] = qg;
    red[2][threadIdx.x] = sp;
    red[3][threadIdx.x] = qp;
    __syncthreads();
    for (int o = kThreads / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o)
#pragma unroll
            for (int k = 0; k < 4; ++k) red[k][threadIdx.x] += red[k][threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) part[blockIdx.x] = make_double4(red[0][0], red[1][0], red[2][0], red[3][0]);
}

__device__ __forceinline__ double std_from_sums(double sum, double square_sum, long long count)
{
    // sampler.cpp:58-61: sample standard deviation, variance clamped at 0
    if (count <= 1) return 0.0;
    const double c = static_cast<double>(count);
    const double variance = fmax(0.0, (square_sum - sum * sum / c) / (c - 1.0));
    return sqrt(variance);
}

// factor = rescale * std(pos) / std(guided) + (1 - rescale), or 1 when std(guided) == 0
// (sampler.cpp:219-226).
__global__ void __launch_bounds__(kThreads) cfg_factor_kernel(const double4 *__restrict__ part, int n_part,
                                                              long long count, float rescale, float *__restrict__ factor)
{
    __shared__ double red[4][kThreads];
    double a[4] = {0.0, 0.0, 0.0, 0.0};
    for (int b = threadIdx.x; b < n_part; b += kThreads) {
        const double4 v = part[b];
        a[0] += v.x;
        a[1] += v.y;
        a[2] += v.z;
        a[3] += v.w;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) red[k][threadIdx.x] = a[k];
    __syncthreads();
    for (int o = kThreads / 2; o > 0; o >>= 1) {
        if (threadIdx.x < o)
#pragma unroll
            for (int k = 0; k < 4; ++k) red[k][threadIdx.x] += red[k][threadIdx.x + o];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const double cfg_std = std_from_sums(red[0][0], red[1][0], count);
        float f = 1.f;
        if (cfg_std > 0.0)
            f = static_cast<float>(static_cast<double>(rescale) * std_from_sums(red[2][0], red[3][0], count) / cfg_std +
                                   static_cast<double>(1.0f - rescale));
        *factor = f;
    }
}

// out = guided(pos, neg) [* factor]
__global__ void cfg_apply_kernel(const float *__restrict__ pos, const float *__restrict__ neg, long long n, float scale,
                                 const float *__restrict__ factor, float *__restrict__ out)
{
    const float f = factor ? *factor : 1.f;
    for (long long i = blockIdx.x * 1LL * kThreads + threadIdx.x; i < n; i += 1LL * gridDim.x * kThreads) {
        const float g = guided(pos[i], neg[i], scale);
        out[i] = factor ? __fmul_rn(g, f) : g;
    }
}

// One sampler update of the latent x (in place allowed): the prediction is the
// positive one, or guided by the negative one (neg != null) and optionally
// rescaled (factor != null); then step_to (final = 0, sampler.cpp:255-264) or
// endpoint (final = 1, :283-284).
__global__ void sampler_update_kernel(const float *__restrict__ x, const float *__restrict__ pos,
                                      const float *__restrict__ neg, float scale, const float *__restrict__ factor,
                                      long long n, float bt, float at, float bs, float as, int final_step,
                                      float *__restrict__ out)
{
    const float f = factor ? *factor : 1.f;
    for (long long i = blockIdx.x * 1LL * kThreads + threadIdx.x; i < n; i += 1LL * gridDim.x * kThreads) {
        float pred = pos[i];
        if (neg) {
            pred = guided(pred, neg[i], scale);
            if (factor) pred = __fmul_rn(pred, f);
        }
        const float xv = x[i];
        const float x0 = __fsub_rn(xv, __fmul_rn(bt, pred));
        if (final_step) {
            out[i] = x0;
        } else {
            const float xT = __fadd_rn(xv, __fmul_rn(at, pred));
            out[i] = __fadd_rn(__fmul_rn(as, x0), __fmul_rn(bs, xT));
        }
    }
}

// condition = (1 - ratio) * encoded + ratio * noise (engine.cpp:106-121)
__global__ void make_condition_kernel(const float *__restrict__ enc, const float *__restrict__ noise, long long n,
                                      float ratio, float *__restrict__ out)
{
    const float keep = 1.0f - ratio;
    for (long long i = blockIdx.x * 1LL * kThreads + threadIdx.x; i < n; i += 1LL * gridDim.x * kThreads)
        out[i] = __fadd_rn(__fmul_rn(keep, enc[i]), __fmul_rn(ratio, noise[i]));
}

bool aligned4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace

namespace s2 {

void sampler_coefficients(float timestep, float next_timestep, int final_step, float *bt, float *at, float *bs,
                          float *as)
{
    // sampler.cpp:255-258 (step_to) and :283 (endpoint), in float
    *bt = timestep / 1000.0f;
    *at = 1.0f - *bt;
    *bs = final_step ? 0.f : std::clamp(next_timestep / 1000.0f, 0.0f, 1.0f);
    *as = 1.0f - *bs;
}

size_t cfg_workspace_bytes() { return sizeof(double4) * kStatBlocks + 256; }

s2_status cfg_factor(cudaStream_t st, const float *pos, const float *neg, long long n, float scale, float rescale,
                     void *workspace, float **factor)
{
    auto *part = static_cast<double4 *>(workspace);
    float *f = reinterpret_cast<float *>(static_cast<char *>(workspace) + sizeof(double4) * kStatBlocks);
    const int blocks = static_cast<int>(std::min<long long>(kStatBlocks, std::max<long long>(1, (n + kThreads - 1) / kThreads)));
    cfg_partials_kernel<<<blocks, kThreads, 0, st>>>(pos, neg, n, scale, part);
    cfg_factor_kernel<<<1, kThreads, 0, st>>>(part, blocks, n, rescale, f);
    if (cudaGetLastError() != cudaSuccess) return set_error(S2_INFERENCE_FAILED, "guidance statistics: launch failed");
    *factor = f;
    return S2_OK;
}

s2_status sampler_update(cudaStream_t st, const float *x, const float *pos, const float *neg, float scale,
                         const float *factor, long long n, float timestep, float next_timestep, int final_step,
                         float *out)
{
    float bt, at, bs, as;
    sampler_coefficients(timestep, next_timestep, final_step, &bt, &at, &bs, &as);
    sampler_update_kernel<<<grid_for(n), kThreads, 0, st>>>(x, pos, neg, scale, factor, n, bt, at, bs, as,
                                                            final_step, out);
    if (cudaGetLastError() != cudaSuccess) return set_error(S2_INFERENCE_FAILED, "sampler update: launch failed");
    return S2_OK;
}

}  // namespace s2

extern "C" s2_status s2_sampler_timesteps(int steps, float *timesteps)
{
    s2::clear_error();
    if (steps <= 0 || !timesteps) return s2::set_error(S2_INVALID_ARGUMENT, "s2_sampler_timesteps: invalid arguments");
    // EulerSampler::EulerSampler (sampler.cpp:181-187)
    for (int i = 0; i < steps; ++i) timesteps[i] = 1000.0f * (1.0f - static_cast<float>(i) / steps);
    return S2_OK;
}

extern "C" float s2_condition_ratio(float noise_scale, int latent_frames, int latent_height, int latent_width)
{
    // transformed_condition_timestep (engine.cpp:79-92) / 1000: the pixel-space
    // frames, height and width of the latent's video
    const float timestep = noise_scale * 1000.0f;
    if (timestep == 0.0f) return 0.0f;
    const float frames = static_cast<float>((latent_frames - 1) * 4 + 1);
    const float height = static_cast<float>(latent_height * 8);
    const float width = static_cast<float>(latent_width * 8);
    const float x1 = 256.0f * 256.0f * 37.0f;
    const float x2 = 1280.0f * 720.0f * 145.0f;
    const float shift = 1.0f + (height * width * frames - x1) * (5.0f - 1.0f) / (x2 - x1);
    const float normalized = timestep / 1000.0f;
    return 1000.0f * shift * normalized / (1.0f + (shift - 1.0f) * normalized) / 1000.0f;
}

extern "C" s2_status s2_make_condition(void *stream, const float *encoded, const float *noise, int C, int T, int H,
                                       int W, float noise_scale, float *condition)
{
    s2::clear_error();
    if (!encoded || !noise || !condition || C <= 0 || T <= 0 || H <= 0 || W <= 0 || !aligned4(encoded) ||
        !aligned4(noise) || !aligned4(condition))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_make_condition: invalid arguments");
    const long long n = 1LL * C * T * H * W;
    const float ratio = s2_condition_ratio(noise_scale, T, H, W);
    make_condition_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(encoded, noise, n, ratio,
                                                                                          condition);
    if (cudaGetLastError() != cudaSuccess) return s2::set_error(S2_INFERENCE_FAILED, "s2_make_condition: launch failed");
    return S2_OK;
}

extern "C" size_t s2_apply_cfg_workspace_bytes(void) { return s2::cfg_workspace_bytes(); }

extern "C" s2_status s2_apply_cfg(void *stream, const float *positive, const float *negative, long long n,
                                  float scale, float rescale, void *workspace, float *output)
{
    s2::clear_error();
    if (!positive || !negative || !output || n <= 0 || (rescale != 0.0f && !workspace))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_apply_cfg: invalid arguments");
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_apply_cfg: workspace must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float *factor = nullptr;
    if (rescale != 0.0f) {
        const s2_status s = s2::cfg_factor(st, positive, negative, n, scale, rescale, workspace, &factor);
        if (s != S2_OK) return s;
    }
    cfg_apply_kernel<<<grid_for(n), kThreads, 0, st>>>(positive, negative, n, scale, factor, output);
    if (cudaGetLastError() != cudaSuccess) return s2::set_error(S2_INFERENCE_FAILED, "s2_apply_cfg: launch failed");
    return S2_OK;
}

extern "C" s2_status s2_euler_step_to(void *stream, const float *prediction, const float *current, long long n,
                                      float timestep, float next_timestep, float *output)
{
    s2::clear_error();
    if (!prediction || !current || !output || n <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_euler_step_to: invalid arguments");
    return s2::sampler_update(static_cast<cudaStream_t>(stream), current, prediction, nullptr, 1.f, nullptr, n,
                              timestep, next_timestep, 0, output);
}

extern "C" s2_status s2_euler_endpoint(void *stream, const float *prediction, const float *current, long long n,
                                       float timestep, float *output)
{
    s2::clear_error();
    if (!prediction || !current || !output || n <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_euler_endpoint: invalid arguments");
    return s2::sampler_update(static_cast<cudaStream_t>(stream), current, prediction, nullptr, 1.f, nullptr, n,
                              timestep, 0.f, 1, output);
}
