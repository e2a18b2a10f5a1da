// s2_vae_attention: DynamicFramewiseSpatialAttention (the VAE mid-block
// attention, src/layers/dynamic_framewise_spatial_attention.cpp) as a CUDA
// layer object: load_param (channels) / load_model (weights in the
// reference's order) / forward on an ncnn 4-D blob [C][cstep] whose channel
// plane holds frames x H x W fp32 values.
//
// A forward is five stream-ordered launches:
//   1. per (frame, channel) double sums of x and x^2 (the GroupNorm
//      statistics, :121-134, accumulated in double like the reference);
//   2. GroupNorm(32, eps 1e-6, affine) applied and transposed to token-major
//      fp16 rows [frame * H*W + token][Cp] (Cp = channels padded to 128, 256
//      or 512, zero-filled), :135-144;
//   3. the fused Q|K|V 1x1 projection on the tensor cores (+ bias), :145-147;
//   4. single-head attention per frame (s2_spatial_attention), :149-180;
//   5. the output 1x1 projection (+ bias) added to the residual x and written
//      back channel-major into y, :182-194.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "s2_buffers.h"
#include "s2_gemm.h"
#include "s2_internal.h"

extern "C" s2_status s2_spatial_attention(void *stream, const void *q, const void *k, const void *v, int channels,
                                          int head_dim, int frames, int tokens, void *out, int32_t *err);

namespace {

constexpr int kGroups = 32;

// Block sum of (s, q) over 256 threads, result in thread 0.
__device__ __forceinline__ void block_sum2(double &s, double &q)
{
    __shared__ double ss[8], sq[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_down_sync(0xffffffffu, s, o);
        q += __shfl_down_sync(0xffffffffu, q, o);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        ss[w] = s;
        sq[w] = q;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < 8; ++i) {
            s += ss[i];
            q += sq[i];
        }
    }
}

// part[frame][channel] = (sum x, sum x^2) over the frame's H*W values, in double.
__global__ void __launch_bounds__(256) gn_partial_kernel(const float *__restrict__ x, long long cstep, int tokens,
                                                         int C, double2 *__restrict__ part)
{
    const int c = blockIdx.x, f = blockIdx.y;
    const float *p = x + static_cast<size_t>(c) * cstep + static_cast<size_t>(f) * tokens;
    double s = 0.0, q = 0.0;
    for (int i = threadIdx.x; i < tokens; i += 256) {
        const double v = p[i];
        s += v;
        q += v * v;
    }
    block_sum2(s, q);
    if (threadIdx.x == 0) part[static_cast<size_t>(f) * C + c] = make_double2(s, q);
}

// xn[(f*tokens + t)][c] = fp16(x[c][f*tokens + t] * scale_c + offset_c), zero for
// padded channels; tile = 64 tokens x 64 channels through shared memory.
__global__ void __launch_bounds__(256) gn_apply_kernel(const float *__restrict__ x, long long cstep, int tokens, int C,
                                                       int cpad, const double2 *__restrict__ part,
                                                       const float *__restrict__ gamma,
                                                       const float *__restrict__ beta, __half *__restrict__ xn)
{
    __shared__ float tile[64][65];
    __shared__ float sc[64], off[64];
    const int t0 = blockIdx.x * 64, c0 = blockIdx.y * 64, f = blockIdx.z;
    if (threadIdx.x < 64) {
        const int c = c0 + threadIdx.x;
        float s_ = 0.f, o_ = 0.f;
        if (c < C) {
            // group statistics exactly as the reference forms them (:131-134)
            const int cpg = C / kGroups, g = c / cpg;
            double s = 0.0, q = 0.0;
            for (int lc = 0; lc < cpg; ++lc) {
                const double2 pr = part[static_cast<size_t>(f) * C + g * cpg + lc];
                s += pr.x;
                q += pr.y;
            }
            const double count = static_cast<double>(cpg) * tokens;
            const float mean = static_cast<float>(s / count);
            const float var = static_cast<float>(q / count - static_cast<double>(mean) * mean);
            const float inv_std = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.f), 1e-6f)));
            s_ = __fmul_rn(gamma[c], inv_std);
            o_ = __fsub_rn(beta[c], __fmul_rn(mean, s_));
        }
        sc[threadIdx.x] = s_;
        off[threadIdx.x] = o_;
    }
    __syncthreads();
    // 16 independent loads per thread in flight (a warp reads 128 contiguous bytes per channel row)
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int i = threadIdx.x + 256 * k, cc = i >> 6, tt = i & 63;
        const int c = c0 + cc, t = t0 + tt;
        v[k] = (c < C && t < tokens) ? __ldg(x + static_cast<size_t>(c) * cstep + static_cast<size_t>(f) * tokens + t)
                                     : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int i = threadIdx.x + 256 * k, cc = i >> 6, tt = i & 63;
        tile[cc][tt] = c0 + cc < C ? __fadd_rn(__fmul_rn(v[k], sc[cc]), off[cc]) : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 32; i += 256) {
        const int tt = i >> 5, cp = (i & 31) * 2;
        const int t = t0 + tt;
        if (t < tokens) {
            const __half2 h = __floats2half2_rn(tile[cp][tt], tile[cp + 1][tt]);
            *reinterpret_cast<__half2 *>(xn + (static_cast<size_t>(f) * tokens + t) * cpad + c0 + cp) = h;
        }
    }
}

int pad_channels(int C) { return C <= 128 ? 128 : (C <= 256 ? 256 : 512); }

}  // namespace

struct s2_vae_attention {
    int device = 0;
    int C = 0, cpad = 0;
    bool loaded = false;
    s2::DeviceBuffer w_qkv, b_qkv, w_o, b_o, gn;   // gn = gamma [C] + beta [C]
    s2::DeviceBuffer part, xn, q, k, v, att, err;
    int last_launches = 0;
    cudaStream_t last_stream = nullptr;
    s2::DeviceBuffer hx, hy;  // device staging for forward_host
    // forward_host's frame pipeline: upload and download streams, one upload and
    // one compute event per frame
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t ev_start = nullptr, ev_out = nullptr;
    std::vector<cudaEvent_t> ev_in, ev_cmp;

    bool ensure_pipeline(int frames)
    {
        if (!s_in && cudaStreamCreateWithFlags(&s_in, cudaStreamNonBlocking) != cudaSuccess) return false;
        if (!s_out && cudaStreamCreateWithFlags(&s_out, cudaStreamNonBlocking) != cudaSuccess) return false;
        if (!ev_start && cudaEventCreateWithFlags(&ev_start, cudaEventDisableTiming) != cudaSuccess) return false;
        if (!ev_out && cudaEventCreateWithFlags(&ev_out, cudaEventDisableTiming) != cudaSuccess) return false;
        while (static_cast<int>(ev_in.size()) < frames) {
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
};

extern "C" s2_status s2_vae_attention_create(int device, int channels, s2_vae_attention **out)
{
    s2::clear_error();
    if (!out) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_create: out is NULL");
    *out = nullptr;
    if (channels <= 0 || channels % kGroups != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_create: channels %d must be a positive multiple of 32",
                             channels);
    if (channels > 512)
        return s2::set_error(S2_UNSUPPORTED, "s2_vae_attention_create: channels %d > 512", channels);
    const s2_status st = s2_device_check(device);
    if (st != S2_OK) return st;
    auto *l = new s2_vae_attention();
    l->device = device;
    l->C = channels;
    l->cpad = pad_channels(channels);
    *out = l;
    return S2_OK;
}

extern "C" s2_status s2_vae_attention_destroy(s2_vae_attention *l)
{
    if (!l) return S2_OK;
    s2::DeviceGuard guard(l->device);
    for (s2::DeviceBuffer *b : {&l->w_qkv, &l->b_qkv, &l->w_o, &l->b_o, &l->gn, &l->part, &l->xn, &l->q, &l->k, &l->v,
                                &l->att, &l->err, &l->hx, &l->hy})
        b->release();
    for (cudaEvent_t e : l->ev_in) cudaEventDestroy(e);
    for (cudaEvent_t e : l->ev_cmp) cudaEventDestroy(e);
    if (l->ev_start) cudaEventDestroy(l->ev_start);
    if (l->ev_out) cudaEventDestroy(l->ev_out);
    if (l->s_in) cudaStreamDestroy(l->s_in);
    if (l->s_out) cudaStreamDestroy(l->s_out);
    delete l;
    return S2_OK;
}

extern "C" s2_status s2_vae_attention_load(s2_vae_attention *l, const float *norm_bias, const float *norm_weight,
                                           const float *k_bias, const float *k_weight, const float *out_bias,
                                           const float *out_weight, const float *q_bias, const float *q_weight,
                                           const float *v_bias, const float *v_weight)
{
    s2::clear_error();
    if (!l || !norm_bias || !norm_weight || !k_bias || !k_weight || !out_bias || !out_weight || !q_bias || !q_weight ||
        !v_bias || !v_weight)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_load: null argument");
    s2::DeviceGuard guard(l->device);
    const int C = l->C, P = l->cpad;
    // weights [out][in] -> fp16, zero-padded to [P][P]; Q|K|V stacked
    std::vector<__half> wqkv(static_cast<size_t>(3) * P * P, __float2half(0.f)), wo(static_cast<size_t>(P) * P,
                                                                                      __float2half(0.f));
    std::vector<float> bqkv(3 * P, 0.f), bo(P, 0.f), gn(2 * C);
    const float *ws[3] = {q_weight, k_weight, v_weight}, *bs[3] = {q_bias, k_bias, v_bias};
    for (int m = 0; m < 3; ++m)
        for (int o = 0; o < C; ++o) {
            for (int i = 0; i < C; ++i)
                wqkv[(static_cast<size_t>(m) * P + o) * P + i] = __float2half(ws[m][static_cast<size_t>(o) * C + i]);
            bqkv[m * P + o] = bs[m][o];
        }
    for (int o = 0; o < C; ++o) {
        for (int i = 0; i < C; ++i) wo[static_cast<size_t>(o) * P + i] = __float2half(out_weight[static_cast<size_t>(o) * C + i]);
        bo[o] = out_bias[o];
    }
    std::memcpy(gn.data(), norm_weight, sizeof(float) * C);
    std::memcpy(gn.data() + C, norm_bias, sizeof(float) * C);
    if (!l->w_qkv.ensure(wqkv.size() * 2) || !l->b_qkv.ensure(bqkv.size() * 4) || !l->w_o.ensure(wo.size() * 2) ||
        !l->b_o.ensure(bo.size() * 4) || !l->gn.ensure(gn.size() * 4))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_attention_load: cudaMalloc failed");
    if (cudaMemcpy(l->w_qkv.ptr, wqkv.data(), wqkv.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->b_qkv.ptr, bqkv.data(), bqkv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->w_o.ptr, wo.data(), wo.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->b_o.ptr, bo.data(), bo.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(l->gn.ptr, gn.data(), gn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_load: upload failed: %s",
                             cudaGetErrorString(cudaGetLastError()));
    l->loaded = true;
    return S2_OK;
}

// Workspaces of a forward over `frames` frames of `rows` tokens in total.
static bool ensure_workspace(s2_vae_attention *l, int frames, long long rows)
{
    const size_t act = static_cast<size_t>(rows) * l->cpad * 2;
    return l->part.ensure(sizeof(double2) * frames * l->C) && l->xn.ensure(act) && l->q.ensure(act) &&
           l->k.ensure(act) && l->v.ensure(act) && l->att.ensure(act) && l->err.ensure(4);
}

extern "C" s2_status s2_vae_attention_forward(s2_vae_attention *l, void *stream, const float *x, int frames,
                                              int height, int width, long long cstep, float *y)
{
    s2::clear_error();
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_forward: layer is NULL");
    if (!l->loaded) return s2::set_error(S2_NOT_LOADED, "s2_vae_attention_forward: weights not loaded");
    if (!x || !y || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_forward: invalid arguments");
    const long long tokens = 1LL * height * width, rows = tokens * frames;
    if (cstep < rows || rows > 0x7fffffffLL)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_forward: cstep %lld < frames*H*W %lld", cstep, rows);
    if (x == y) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_forward: in-place forward is not supported");
    s2::DeviceGuard guard(l->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int C = l->C, P = l->cpad;
    bool fresh_err = l->err.ptr == nullptr;
    if (!ensure_workspace(l, frames, rows))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_attention_forward: workspace allocation failed");
    if (fresh_err && cudaMemsetAsync(l->err.ptr, 0, 4, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_forward: memset failed");
    int32_t *err = static_cast<int32_t *>(l->err.ptr);
    const float *gamma = static_cast<const float *>(l->gn.ptr), *beta = gamma + C;
    l->last_launches = 0;
    l->last_stream = st;

    gn_partial_kernel<<<dim3(C, frames), 256, 0, st>>>(x, cstep, static_cast<int>(tokens), C,
                                                       static_cast<double2 *>(l->part.ptr));
    gn_apply_kernel<<<dim3(static_cast<unsigned>((tokens + 63) / 64), P / 64, frames), 256, 0, st>>>(
        x, cstep, static_cast<int>(tokens), C, P, static_cast<const double2 *>(l->part.ptr), gamma, beta,
        static_cast<__half *>(l->xn.ptr));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_forward: group norm launch: %s", cudaGetErrorString(e));
    l->last_launches = 2;

    s2::GemmArgs g;
    g.M = static_cast<int>(rows);
    g.N = 3 * P;
    g.K = P;
    g.bias = static_cast<const float *>(l->b_qkv.ptr);
    g.epilogue = s2::GEMM_EPI_SPLIT_F16;
    g.out[0] = l->q.ptr;
    g.out[1] = l->k.ptr;
    g.out[2] = l->v.ptr;
    g.split = P;
    g.err = err;
    s2_status s = s2::gemm_f16(st, l->xn.ptr, l->w_qkv.ptr, g);
    if (s != S2_OK) return s;
    ++l->last_launches;

    s = s2_spatial_attention(st, l->q.ptr, l->k.ptr, l->v.ptr, C, P, frames, static_cast<int>(tokens), l->att.ptr, err);
    if (s != S2_OK) return s;
    ++l->last_launches;

    s2::GemmArgs o;
    o.M = static_cast<int>(rows);
    o.N = P;
    o.K = P;
    o.bias = static_cast<const float *>(l->b_o.ptr);
    o.epilogue = s2::GEMM_EPI_RESID_T_F32;
    o.resid = x;
    o.y = y;
    o.ldt = cstep;
    o.n_valid = C;
    o.err = err;
    s = s2::gemm_f16(st, l->att.ptr, l->w_o.ptr, o);
    if (s != S2_OK) return s;
    ++l->last_launches;
    return S2_OK;
}

extern "C" s2_status s2_vae_attention_forward_host(s2_vae_attention *l, void *stream, const float *x, int frames,
                                                   int height, int width, long long cstep, float *y)
{
    s2::clear_error();
    if (!l || !x || !y || frames <= 0 || height <= 0 || width <= 0 || cstep < 1LL * frames * height * width)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_forward_host: invalid arguments");
    if (!l->loaded) return s2::set_error(S2_NOT_LOADED, "s2_vae_attention_forward_host: weights not loaded");
    s2::DeviceGuard guard(l->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t bytes = static_cast<size_t>(cstep) * l->C * sizeof(float);
    const long long tokens = 1LL * height * width;
    // Every part of the layer works frame by frame (GroupNorm statistics, the
    // attention, and the row-wise projections), so the frames are pipelined: the
    // upload of frame f + 1, the forward of frame f and the download of frame f - 1
    // run on three streams. A frame is one strided copy of the [C][cstep] blob
    // (C rows of H*W floats, cstep apart). Each frame's forward is the same
    // arithmetic as the whole blob's, so the result is the same bit for bit.
    const bool fresh_err = l->err.ptr == nullptr;
    if (!l->hx.ensure(bytes) || !l->hy.ensure(bytes) || !ensure_workspace(l, 1, tokens) || !l->ensure_pipeline(frames))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_attention_forward_host: staging allocation failed");
    if (fresh_err && cudaMemsetAsync(l->err.ptr, 0, 4, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_forward_host: memset failed");
    auto *dx = static_cast<float *>(l->hx.ptr), *dy = static_cast<float *>(l->hy.ptr);
    const size_t pitch = static_cast<size_t>(cstep) * sizeof(float), width_b = static_cast<size_t>(tokens) * sizeof(float);
    // After the first copy is queued, every error return first waits for the
    // copies in flight on the caller's host buffers, so the caller may free
    // them as soon as the call returns.
    auto drain = [&](s2_status s) {
        cudaStreamSynchronize(l->s_in);
        cudaStreamSynchronize(l->s_out);
        cudaStreamSynchronize(st);
        return s;
    };
    bool ok = cudaEventRecord(l->ev_start, st) == cudaSuccess && cudaStreamWaitEvent(l->s_in, l->ev_start, 0) == cudaSuccess &&
              cudaStreamWaitEvent(l->s_out, l->ev_start, 0) == cudaSuccess;
    for (int f = 0; ok && f < frames; ++f)
        ok = cudaMemcpy2DAsync(dx + f * tokens, pitch, x + f * tokens, pitch, width_b, l->C, cudaMemcpyHostToDevice,
                               l->s_in) == cudaSuccess &&
             cudaEventRecord(l->ev_in[f], l->s_in) == cudaSuccess;
    if (!ok) return drain(s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_forward_host: upload failed"));
    int launches = 0;
    for (int f = 0; f < frames; ++f) {
        if (cudaStreamWaitEvent(st, l->ev_in[f], 0) != cudaSuccess)
            return drain(s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_forward_host: stream wait failed"));
        const s2_status s = s2_vae_attention_forward(l, stream, dx + f * tokens, 1, height, width, cstep, dy + f * tokens);
        if (s != S2_OK) return drain(s);
        launches += l->last_launches;
        if (cudaEventRecord(l->ev_cmp[f], st) != cudaSuccess || cudaStreamWaitEvent(l->s_out, l->ev_cmp[f], 0) != cudaSuccess ||
            cudaMemcpy2DAsync(y + f * tokens, pitch, dy + f * tokens, pitch, width_b, l->C, cudaMemcpyDeviceToHost,
                              l->s_out) != cudaSuccess)
            return drain(s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_forward_host: download failed"));
    }
    l->last_launches = launches;
    if (cudaEventRecord(l->ev_out, l->s_out) != cudaSuccess || cudaStreamWaitEvent(st, l->ev_out, 0) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention_forward_host: %s",
                             cudaGetErrorString(cudaGetLastError()));
    int code = 0;
    return s2_vae_attention_device_error(l, &code);
}

extern "C" int s2_vae_attention_last_launches(const s2_vae_attention *l) { return l ? l->last_launches : 0; }

extern "C" s2_status s2_vae_attention_device_error(s2_vae_attention *l, int *code)
{
    if (code) *code = 0;
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_attention_device_error: layer is NULL");
    if (!l->err.ptr) return S2_OK;
    s2::DeviceGuard guard(l->device);
    int32_t h = 0;
    if (cudaStreamSynchronize(l->last_stream) != cudaSuccess ||
        cudaMemcpy(&h, l->err.ptr, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention: device failure: %s",
                             cudaGetErrorString(cudaGetLastError()));
    if (code) *code = h;
    if (h != 0) return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_attention: device wait timed out (code %d)", h);
    return S2_OK;
}
