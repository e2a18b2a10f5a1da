// The SeedVR2 VAE's other custom layers and its 3-D convolution on sm_100a,
// as layer objects on ncnn 4-D blobs [C][cstep] (channel plane = frames x H x W
// fp32, the layout the reference's layers read and write):
//
//  * s2_vae_group_norm  -- DynamicFramewiseGroupNorm
//    (src/layers/dynamic_framewise_group_norm.cpp:43-121): per frame and group
//    of C/32 channels, double sums of x and x^2, mean and variance rounded to
//    float as there, y = x * scale + offset. Two HBM-bound launches: the
//    per-(frame, channel) sums, then the normalisation (which re-reads x).
//  * s2_vae_space_time_shuffle -- DynamicSpaceTimeShuffle
//    (src/layers/dynamic_space_time_shuffle.cpp:41-130): the 1x1x1 projection
//    on the tensor cores with an epilogue that writes every projected channel
//    straight to its (frame, row, column) offset of the upsampled output,
//    dropping the duplicated raw frame 1 when the temporal ratio is 2.
//  * s2_vae_conv3d -- ncnn's Convolution3D as the reference patches it
//    (patches/0001-feat-Convolution3D-Vulkan-pack1.patch: the stated formula
//    :17-25, SAME padding :240-265): an implicit GEMM whose A operand is read
//    through a 4-D tensor map over a token-major fp16 copy of the input (boxes
//    of 64 channels x 32 output columns, out-of-range taps zero-filled by the
//    TMA unit), K = taps x channels, fp32 accumulation in TMEM, the output
//    written channel-major with its bias.
//
// The projections and the convolution take fp16 operands with fp32
// accumulation (the reference accumulates the projection in double and the
// convolution in fp32 from fp32 operands).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "s2_buffers.h"
#include "s2_gemm.h"
#include "s2_internal.h"

namespace {

constexpr int kGroups = 32;

int round_up(int x, int m) { return (x + m - 1) / m * m; }

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

// part[f][c] = (sum x, sum x^2) in double over the frame's hw values of channel c.
__global__ void __launch_bounds__(256) gn_stats_kernel(const float *__restrict__ x, long long cstep, int hw, int C,
                                                       int vec4, double2 *__restrict__ part)
{
    const int c = blockIdx.x, f = blockIdx.y;
    const float *p = x + static_cast<size_t>(c) * cstep + static_cast<size_t>(f) * hw;
    double s = 0.0, q = 0.0;
    if (vec4) {
        const float4 *p4 = reinterpret_cast<const float4 *>(p);
        for (int i = threadIdx.x; i < hw / 4; i += 256) {
            const float4 v = __ldg(p4 + i);
            s += static_cast<double>(v.x) + static_cast<double>(v.y) + static_cast<double>(v.z) + static_cast<double>(v.w);
            q += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
                 static_cast<double>(v.w) * v.w;
        }
    } else {
        for (int i = threadIdx.x; i < hw; i += 256) {
            const double v = p[i];
            s += v;
            q += v * v;
        }
    }
    block_sum2(s, q);
    if (threadIdx.x == 0) part[static_cast<size_t>(f) * C + c] = make_double2(s, q);
}

// y[c][f*hw + i] = x * scale + offset, the group statistics formed as the
// reference does (:99-111): mean = float(sum / count), var = float(sq / count -
// mean^2), inv_std = 1 / sqrt(max(var, 0) + eps), scale = w * inv_std, offset =
// b - mean * scale; explicitly rounded operations (no contraction).
__global__ void __launch_bounds__(256) gn_norm_kernel(const float *__restrict__ x, long long cstep, int hw, int C,
                                                      const double2 *__restrict__ part, const float *__restrict__ bias,
                                                      const float *__restrict__ weight, float eps, int vec4,
                                                      int per_block, float *__restrict__ y, long long ycstep)
{
    __shared__ float sc_off[2];
    const int c = blockIdx.y, f = blockIdx.z;
    if (threadIdx.x == 0) {
        const int cpg = C / kGroups, g = c / cpg;
        double s = 0.0, q = 0.0;
        for (int lc = 0; lc < cpg; ++lc) {
            const double2 pr = part[static_cast<size_t>(f) * C + g * cpg + lc];
            s += pr.x;
            q += pr.y;
        }
        const double count = static_cast<double>(cpg) * hw;
        const float mean = static_cast<float>(s / count);
        const float var = static_cast<float>(q / count - static_cast<double>(mean) * mean);
        const float inv_std = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(fmaxf(var, 0.f), eps)));
        const float scale = __fmul_rn(weight[c], inv_std);
        sc_off[0] = scale;
        sc_off[1] = __fsub_rn(bias[c], __fmul_rn(mean, scale));
    }
    __syncthreads();
    const float scale = sc_off[0], offset = sc_off[1];
    const int i0 = blockIdx.x * per_block, i1 = min(hw, i0 + per_block);
    const float *src = x + static_cast<size_t>(c) * cstep + static_cast<size_t>(f) * hw;
    float *dst = y + static_cast<size_t>(c) * ycstep + static_cast<size_t>(f) * hw;
    if (vec4) {
        for (int i = i0 + 4 * threadIdx.x; i < i1; i += 1024) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(src + i));
            float4 o;
            o.x = __fadd_rn(__fmul_rn(v.x, scale), offset);
            o.y = __fadd_rn(__fmul_rn(v.y, scale), offset);
            o.z = __fadd_rn(__fmul_rn(v.z, scale), offset);
            o.w = __fadd_rn(__fmul_rn(v.w, scale), offset);
            *reinterpret_cast<float4 *>(dst + i) = o;
        }
    } else {
        for (int i = i0 + threadIdx.x; i < i1; i += 256) dst[i] = __fadd_rn(__fmul_rn(src[i], scale), offset);
    }
}

// Token-major fp16 copy of a channel-major blob: out[t][c] = fp16(x[c][t]) for
// t < tokens, c < C; zero for C <= c < cpad. Tile = 64 tokens x 64 channels.
__global__ void __launch_bounds__(256) to_tokens_f16_kernel(const float *__restrict__ x, long long cstep, long long tokens,
                                                            int C, int cpad, __half *__restrict__ out)
{
    __shared__ float tile[64][65];
    const long long t0 = static_cast<long long>(blockIdx.x) * 64;
    const int c0 = blockIdx.y * 64;
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int i = threadIdx.x + 256 * k, cc = i >> 6, tt = i & 63;
        const int c = c0 + cc;
        const long long t = t0 + tt;
        v[k] = (c < C && t < tokens) ? __ldg(x + static_cast<size_t>(c) * cstep + static_cast<size_t>(t)) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int i = threadIdx.x + 256 * k;
        tile[i >> 6][i & 63] = v[k];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 32; i += 256) {
        const int tt = i >> 5, cp = (i & 31) * 2;
        const long long t = t0 + tt;
        if (t < tokens)
            *reinterpret_cast<__half2 *>(out + static_cast<size_t>(t) * cpad + c0 + cp) =
                __floats2half2_rn(tile[cp][tt], tile[cp + 1][tt]);
    }
}

s2_status to_tokens(cudaStream_t st, const float *x, long long cstep, long long tokens, int C, int cpad, __half *out)
{
    const dim3 grid(static_cast<unsigned>((tokens + 63) / 64), static_cast<unsigned>(cpad / 64));
    to_tokens_f16_kernel<<<grid, 256, 0, st>>>(x, cstep, tokens, C, cpad, out);
    return cudaGetLastError() == cudaSuccess ? S2_OK
                                             : s2::set_error(S2_INFERENCE_FAILED, "vae layer: transpose launch failed");
}

// Host fp32 -> device fp16 weights, [rows][src_cols] -> [rows][dst_cols] with
// column map col(j) (dst index of source column j), zeros elsewhere.
template <typename ColMap>
bool upload_f16(s2::DeviceBuffer &dst, const float *src, int rows, int src_cols, int dst_cols, ColMap col)
{
    std::vector<__half> h(static_cast<size_t>(rows) * dst_cols, __float2half(0.f));
    for (int r = 0; r < rows; ++r)
        for (int j = 0; j < src_cols; ++j)
            h[static_cast<size_t>(r) * dst_cols + col(j)] = __float2half_rn(src[static_cast<size_t>(r) * src_cols + j]);
    return dst.ensure(h.size() * sizeof(__half)) &&
           cudaMemcpy(dst.ptr, h.data(), h.size() * sizeof(__half), cudaMemcpyHostToDevice) == cudaSuccess;
}

bool upload_f32(s2::DeviceBuffer &dst, const float *src, size_t n)
{
    return dst.ensure(n * sizeof(float)) && cudaMemcpy(dst.ptr, src, n * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess;
}

// Host-buffer forward shared by the layers: copy x in, run, copy y out.
template <typename Fwd>
s2_status forward_host(int device, void *stream, s2::DeviceBuffer &dx, s2::DeviceBuffer &dy, const float *x,
                       size_t x_floats, float *y, size_t y_floats, Fwd fwd)
{
    s2::DeviceGuard guard(device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!dx.ensure(x_floats * 4) || !dy.ensure(y_floats * 4))
        return s2::set_error(S2_OUT_OF_MEMORY, "vae layer forward_host: staging allocation failed");
    if (cudaMemcpyAsync(dx.ptr, x, x_floats * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) {
        cudaStreamSynchronize(st);
        return s2::set_error(S2_INFERENCE_FAILED, "vae layer forward_host: upload failed");
    }
    s2_status s = fwd(static_cast<const float *>(dx.ptr), static_cast<float *>(dy.ptr));
    if (s == S2_OK && cudaMemcpyAsync(y, dy.ptr, y_floats * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        s = s2::set_error(S2_INFERENCE_FAILED, "vae layer forward_host: download failed");
    // the copies read and write the caller's buffers: finish them before returning, on every path
    const cudaError_t e = cudaStreamSynchronize(st);
    if (s == S2_OK && e != cudaSuccess)
        s = s2::set_error(S2_INFERENCE_FAILED, "vae layer forward_host: %s", cudaGetErrorString(e));
    return s;
}

s2_status check_err(int device, cudaStream_t st, s2::DeviceBuffer &err, const char *what)
{
    if (!err.ptr) return S2_OK;
    s2::DeviceGuard guard(device);
    int32_t h = 0;
    if (cudaStreamSynchronize(st) != cudaSuccess || cudaMemcpy(&h, err.ptr, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "%s: device failure: %s", what, cudaGetErrorString(cudaGetLastError()));
    if (h != 0) {
        cudaMemset(err.ptr, 0, 4);
        return s2::set_error(S2_INFERENCE_FAILED, "%s: device wait timed out (code %d)", what, h);
    }
    return S2_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// DynamicFramewiseGroupNorm
// ---------------------------------------------------------------------------

struct s2_vae_group_norm {
    int device = 0, C = 0;
    float eps = 1e-6f;
    bool loaded = false;
    s2::DeviceBuffer bias, weight, part, hx, hy;
    int last_launches = 0;
};

extern "C" s2_status s2_vae_group_norm_create(int device, int channels, s2_vae_group_norm **out)
{
    s2::clear_error();
    if (!out) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_group_norm_create: out is NULL");
    *out = nullptr;
    // load_param (:43-53): channels from the bias shape, a multiple of the 32 groups
    if (channels <= 0 || channels % kGroups != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_group_norm_create: channels %d must be a positive multiple of 32",
                             channels);
    const s2_status st = s2_device_check(device);
    if (st != S2_OK) return st;
    auto *l = new s2_vae_group_norm();
    l->device = device;
    l->C = channels;
    *out = l;
    return S2_OK;
}

extern "C" s2_status s2_vae_group_norm_destroy(s2_vae_group_norm *l)
{
    if (!l) return S2_OK;
    s2::DeviceGuard guard(l->device);
    for (s2::DeviceBuffer *b : {&l->bias, &l->weight, &l->part, &l->hx, &l->hy}) b->release();
    delete l;
    return S2_OK;
}

extern "C" s2_status s2_vae_group_norm_load(s2_vae_group_norm *l, const float *bias, const float *weight)
{
    s2::clear_error();
    if (!l || !bias || !weight) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_group_norm_load: NULL argument");
    s2::DeviceGuard guard(l->device);
    if (!upload_f32(l->bias, bias, l->C) || !upload_f32(l->weight, weight, l->C))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_group_norm_load: upload failed");
    l->loaded = true;
    return S2_OK;
}

extern "C" s2_status s2_vae_group_norm_forward(s2_vae_group_norm *l, void *stream, const float *x, int frames,
                                               int height, int width, long long cstep, float *y, long long y_cstep)
{
    s2::clear_error();
    if (!l || !x || !y || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_group_norm_forward: invalid arguments");
    const long long plane = 1LL * frames * height * width;
    if (cstep < plane || y_cstep < plane || plane > (1LL << 31))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_group_norm_forward: cstep smaller than the channel plane");
    if (!l->loaded) return s2::set_error(S2_NOT_LOADED, "s2_vae_group_norm_forward: weights not loaded");
    s2::DeviceGuard guard(l->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int hw = height * width;
    if (!l->part.ensure(static_cast<size_t>(frames) * l->C * sizeof(double2)))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_group_norm_forward: workspace allocation failed");
    const bool v4 = hw % 4 == 0 && cstep % 4 == 0 && y_cstep % 4 == 0 &&
                    ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u) == 0;
    auto *part = static_cast<double2 *>(l->part.ptr);
    gn_stats_kernel<<<dim3(l->C, frames), 256, 0, st>>>(x, cstep, hw, l->C, v4 ? 1 : 0, part);
    constexpr int kPerBlock = 8192;
    gn_norm_kernel<<<dim3((hw + kPerBlock - 1) / kPerBlock, l->C, frames), 256, 0, st>>>(
        x, cstep, hw, l->C, part, static_cast<const float *>(l->bias.ptr), static_cast<const float *>(l->weight.ptr),
        l->eps, v4 ? 1 : 0, kPerBlock, y, y_cstep);
    if (cudaGetLastError() != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_group_norm_forward: launch failed");
    l->last_launches = 2;
    return S2_OK;
}

extern "C" s2_status s2_vae_group_norm_forward_host(s2_vae_group_norm *l, void *stream, const float *x, int frames,
                                                    int height, int width, float *y)
{
    s2::clear_error();
    if (!l || !x || !y || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_group_norm_forward_host: invalid arguments");
    const long long plane = 1LL * frames * height * width;
    const size_t n = static_cast<size_t>(plane) * l->C;
    return forward_host(l->device, stream, l->hx, l->hy, x, n, y, n, [&](const float *dx, float *dy) {
        return s2_vae_group_norm_forward(l, stream, dx, frames, height, width, plane, dy, plane);
    });
}

extern "C" int s2_vae_group_norm_last_launches(const s2_vae_group_norm *l) { return l ? l->last_launches : 0; }

// ---------------------------------------------------------------------------
// DynamicSpaceTimeShuffle
// ---------------------------------------------------------------------------

struct s2_vae_space_time_shuffle {
    int device = 0, cin = 0, proj = 0, tr = 1, cpad = 64;
    bool loaded = false;
    s2::DeviceBuffer w16, bias, a16, err, hx, hy;
    int last_launches = 0;
    cudaStream_t last_stream = nullptr;
};

extern "C" s2_status s2_vae_space_time_shuffle_create(int device, int in_channels, int projected_channels,
                                                      s2_vae_space_time_shuffle **out)
{
    s2::clear_error();
    if (!out) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_space_time_shuffle_create: out is NULL");
    *out = nullptr;
    // load_param (:41-55): the projected channels must split into 2 x 2 spatial
    // offsets x a temporal ratio
    if (in_channels <= 0 || projected_channels <= 0 || projected_channels % (4 * in_channels) != 0)
        return s2::set_error(S2_INVALID_ARGUMENT,
                             "s2_vae_space_time_shuffle_create: projected channels %d != in channels %d x 4 x ratio",
                             projected_channels, in_channels);
    if (in_channels % 32 != 0)
        return s2::set_error(S2_UNSUPPORTED, "s2_vae_space_time_shuffle_create: in channels %d must be a multiple of 32",
                             in_channels);
    const s2_status st = s2_device_check(device);
    if (st != S2_OK) return st;
    auto *l = new s2_vae_space_time_shuffle();
    l->device = device;
    l->cin = in_channels;
    l->proj = projected_channels;
    l->tr = projected_channels / in_channels / 4;
    l->cpad = round_up(in_channels, 64);
    *out = l;
    return S2_OK;
}

extern "C" s2_status s2_vae_space_time_shuffle_destroy(s2_vae_space_time_shuffle *l)
{
    if (!l) return S2_OK;
    s2::DeviceGuard guard(l->device);
    for (s2::DeviceBuffer *b : {&l->w16, &l->bias, &l->a16, &l->err, &l->hx, &l->hy}) b->release();
    delete l;
    return S2_OK;
}

extern "C" s2_status s2_vae_space_time_shuffle_load(s2_vae_space_time_shuffle *l, const float *bias,
                                                    const float *weight)
{
    s2::clear_error();
    if (!l || !bias || !weight) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_space_time_shuffle_load: NULL argument");
    s2::DeviceGuard guard(l->device);
    // load_model (:57-63): bias [P], then weight [P][Cin]. The projected channel
    // p = ((oy * 2 + ox) * tr + ot) * Cin + c becomes GEMM column
    // ((oy * tr + ot) * Cin + c) * 2 + ox, so that the epilogue writes (ox = 0, 1) pairs.
    const int cin = l->cin, tr = l->tr, P = l->proj;
    std::vector<float> wp(static_cast<size_t>(P) * cin), bp(P);
    for (int p = 0; p < P; ++p) {
        const int c = p % cin, t = p / cin, ot = t % tr, oxy = t / tr, ox = oxy & 1, oy = oxy >> 1;
        const int n = ((oy * tr + ot) * cin + c) * 2 + ox;
        bp[n] = bias[p];
        std::copy(weight + static_cast<size_t>(p) * cin, weight + static_cast<size_t>(p + 1) * cin,
                  wp.begin() + static_cast<size_t>(n) * cin);
    }
    if (!upload_f32(l->bias, bp.data(), P) || !upload_f16(l->w16, wp.data(), P, cin, l->cpad, [](int j) { return j; }))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_space_time_shuffle_load: upload failed");
    l->loaded = true;
    return S2_OK;
}

extern "C" s2_status s2_vae_space_time_shuffle_output_shape(const s2_vae_space_time_shuffle *l, int frames,
                                                            int height, int width, int *out_frames, int *out_height,
                                                            int *out_width)
{
    if (!l || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_space_time_shuffle_output_shape: invalid arguments");
    if (out_frames) *out_frames = l->tr > 1 ? frames * l->tr - 1 : frames;
    if (out_height) *out_height = 2 * height;
    if (out_width) *out_width = 2 * width;
    return S2_OK;
}

extern "C" s2_status s2_vae_space_time_shuffle_forward(s2_vae_space_time_shuffle *l, void *stream, const float *x,
                                                       int frames, int height, int width, long long cstep, float *y,
                                                       long long y_cstep)
{
    s2::clear_error();
    if (!l || !x || !y || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_space_time_shuffle_forward: invalid arguments");
    const long long tokens = 1LL * frames * height * width;
    const int of = l->tr > 1 ? frames * l->tr - 1 : frames;
    if (cstep < tokens || y_cstep < 4LL * of * height * width || tokens > (1LL << 30) || y_cstep % 2 != 0 ||
        (reinterpret_cast<uintptr_t>(y) & 7u) != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_space_time_shuffle_forward: bad cstep or unaligned y");
    if (!l->loaded) return s2::set_error(S2_NOT_LOADED, "s2_vae_space_time_shuffle_forward: weights not loaded");
    s2::DeviceGuard guard(l->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool fresh = !l->err.ptr;
    if (!l->a16.ensure(static_cast<size_t>(tokens) * l->cpad * 2) || !l->err.ensure(4))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_space_time_shuffle_forward: workspace allocation failed");
    if (fresh && cudaMemsetAsync(l->err.ptr, 0, 4, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_space_time_shuffle_forward: memset failed");
    l->last_stream = st;
    s2_status s = to_tokens(st, x, cstep, tokens, l->cin, l->cpad, static_cast<__half *>(l->a16.ptr));
    if (s != S2_OK) return s;
    s2::GemmArgs g;
    g.M = static_cast<int>(tokens);
    g.N = l->proj;
    g.K = l->cpad;
    g.bias = static_cast<const float *>(l->bias.ptr);
    g.epilogue = s2::GEMM_EPI_SHUFFLE_F32;
    g.y = y;
    g.ldt = y_cstep;
    g.n_valid = l->proj;
    g.sh_cin = l->cin;
    g.sh_tr = l->tr;
    g.sh_h = height;
    g.sh_w = width;
    // K is short (the channels) and N long (4 x ratio x channels): with one CTA per 128 x 256
    // tile every tile re-reads its 256 weight rows from L2; CTA pairs halve that traffic
    g.pair = (tokens >= 4096 && l->proj % 256 == 0) ? 1 : 0;
    g.err = static_cast<int32_t *>(l->err.ptr);
    s = s2::gemm_f16(st, l->a16.ptr, l->w16.ptr, g);
    if (s != S2_OK) return s;
    l->last_launches = 2;
    return S2_OK;
}

extern "C" s2_status s2_vae_space_time_shuffle_forward_host(s2_vae_space_time_shuffle *l, void *stream,
                                                            const float *x, int frames, int height, int width,
                                                            float *y)
{
    s2::clear_error();
    if (!l || !x || !y || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_space_time_shuffle_forward_host: invalid arguments");
    const long long tokens = 1LL * frames * height * width;
    const int of = l->tr > 1 ? frames * l->tr - 1 : frames;
    const long long out_plane = 4LL * of * height * width;
    s2_status s = forward_host(l->device, stream, l->hx, l->hy, x, static_cast<size_t>(tokens) * l->cin, y,
                               static_cast<size_t>(out_plane) * l->cin, [&](const float *dx, float *dy) {
                                   return s2_vae_space_time_shuffle_forward(l, stream, dx, frames, height, width,
                                                                            tokens, dy, out_plane);
                               });
    if (s != S2_OK) return s;
    return check_err(l->device, static_cast<cudaStream_t>(stream), l->err, "s2_vae_space_time_shuffle");
}

extern "C" int s2_vae_space_time_shuffle_last_launches(const s2_vae_space_time_shuffle *l)
{
    return l ? l->last_launches : 0;
}

extern "C" s2_status s2_vae_space_time_shuffle_device_error(s2_vae_space_time_shuffle *l, int *code)
{
    if (code) *code = 0;
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_space_time_shuffle_device_error: layer is NULL");
    return check_err(l->device, l->last_stream, l->err, "s2_vae_space_time_shuffle");
}

// ---------------------------------------------------------------------------
// Convolution3D
// ---------------------------------------------------------------------------

struct s2_vae_conv3d {
    int device = 0;
    int cin = 0, cout = 0, cpad = 64;
    int kd = 1, kh = 1, kw = 1, dd = 1, dh = 1, dw = 1, sd = 1, sh = 1, sw = 1;
    int pf = 0, pt = 0, pl = 0, pb = 0, pbt = 0, pr = 0;  // front, top, left, behind, bottom, right (or -233/-234)
    int bias_term = 0;
    bool loaded = false;
    s2::DeviceBuffer w16, bias, x16, err, hx, hy;
    int last_launches = 0;
    cudaStream_t last_stream = nullptr;

    // effective pads for an input of d x h x w (SAME modes resolved as the patch does, :240-265)
    void pads(int d, int h, int w, int &f, int &t, int &l, int &b, int &bo, int &r) const
    {
        f = pf, t = pt, l = pl, b = pb, bo = pbt, r = pr;
        const int ew = dw * (kw - 1) + 1, eh = dh * (kh - 1) + 1, ed = dd * (kd - 1) + 1;
        const bool upper = pf == -233 && pt == -233 && pl == -233 && pb == -233 && pbt == -233 && pr == -233;
        const bool lower = pf == -234 && pt == -234 && pl == -234 && pb == -234 && pbt == -234 && pr == -234;
        if (upper || lower) {
            const int wpad = ew + (w - 1) / sw * sw - w, hpad = eh + (h - 1) / sh * sh - h, dpad = ed + (d - 1) / sd * sd - d;
            if (upper) {
                l = wpad / 2, r = wpad - wpad / 2, t = hpad / 2, bo = hpad - hpad / 2, f = dpad / 2, b = dpad - dpad / 2;
            } else {
                l = wpad - wpad / 2, r = wpad / 2, t = hpad - hpad / 2, bo = hpad / 2, f = dpad - dpad / 2, b = dpad / 2;
            }
        }
    }
    bool out_shape(int d, int h, int w, int &od, int &oh, int &ow) const
    {
        int f, t, l, b, bo, r;
        pads(d, h, w, f, t, l, b, bo, r);
        if (f < 0 || t < 0 || l < 0 || b < 0 || bo < 0 || r < 0) return false;
        od = (d + f + b - (dd * (kd - 1) + 1)) / sd + 1;
        oh = (h + t + bo - (dh * (kh - 1) + 1)) / sh + 1;
        ow = (w + l + r - (dw * (kw - 1) + 1)) / sw + 1;
        return od > 0 && oh > 0 && ow > 0;
    }
};

extern "C" s2_status s2_vae_conv3d_create(int device, int in_channels, int out_channels, int kernel_d, int kernel_h,
                                          int kernel_w, int dilation_d, int dilation_h, int dilation_w, int stride_d,
                                          int stride_h, int stride_w, int pad_front, int pad_top, int pad_left,
                                          int pad_behind, int pad_bottom, int pad_right, float pad_value,
                                          int bias_term, s2_vae_conv3d **out)
{
    s2::clear_error();
    if (!out) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_create: out is NULL");
    *out = nullptr;
    if (in_channels <= 0 || out_channels <= 0 || kernel_d <= 0 || kernel_h <= 0 || kernel_w <= 0 || dilation_d <= 0 ||
        dilation_h <= 0 || dilation_w <= 0 || stride_d <= 0 || stride_h <= 0 || stride_w <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_create: non-positive channel count, kernel, dilation or stride");
    const int pads[6] = {pad_front, pad_top, pad_left, pad_behind, pad_bottom, pad_right};
    const bool same = std::all_of(pads, pads + 6, [&](int p) { return p == pads[0]; }) && (pads[0] == -233 || pads[0] == -234);
    if (!same && std::any_of(pads, pads + 6, [](int p) { return p < 0; }))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_create: pads must be >= 0 or all -233 / all -234");
    if (pad_value != 0.f)
        return s2::set_error(S2_UNSUPPORTED, "s2_vae_conv3d_create: pad_value %g (this build zero-pads)", pad_value);
    if (stride_w > 4) return s2::set_error(S2_UNSUPPORTED, "s2_vae_conv3d_create: stride_w %d > 4", stride_w);
    const s2_status st = s2_device_check(device);
    if (st != S2_OK) return st;
    auto *l = new s2_vae_conv3d();
    l->device = device;
    l->cin = in_channels;
    l->cout = out_channels;
    l->cpad = round_up(in_channels, 64);
    l->kd = kernel_d, l->kh = kernel_h, l->kw = kernel_w;
    l->dd = dilation_d, l->dh = dilation_h, l->dw = dilation_w;
    l->sd = stride_d, l->sh = stride_h, l->sw = stride_w;
    l->pf = pad_front, l->pt = pad_top, l->pl = pad_left, l->pb = pad_behind, l->pbt = pad_bottom, l->pr = pad_right;
    l->bias_term = bias_term ? 1 : 0;
    *out = l;
    return S2_OK;
}

extern "C" s2_status s2_vae_conv3d_destroy(s2_vae_conv3d *l)
{
    if (!l) return S2_OK;
    s2::DeviceGuard guard(l->device);
    for (s2::DeviceBuffer *b : {&l->w16, &l->bias, &l->x16, &l->err, &l->hx, &l->hy}) b->release();
    delete l;
    return S2_OK;
}

extern "C" s2_status s2_vae_conv3d_load(s2_vae_conv3d *l, const float *weight, const float *bias)
{
    s2::clear_error();
    if (!l || !weight || (l->bias_term && !bias))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_load: NULL argument");
    s2::DeviceGuard guard(l->device);
    // weight [out][in][taps] -> fp16 [out][taps][cpad] (tap-major K, zero channels past in)
    const int taps = l->kd * l->kh * l->kw, cin = l->cin, cpad = l->cpad;
    if (!upload_f16(l->w16, weight, l->cout, cin * taps, taps * cpad,
                    [=](int j) { return (j % taps) * cpad + j / taps; }))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_conv3d_load: upload failed");
    std::vector<float> b(l->cout, 0.f);
    if (l->bias_term) std::copy(bias, bias + l->cout, b.begin());
    if (!upload_f32(l->bias, b.data(), l->cout)) return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_conv3d_load: upload failed");
    l->loaded = true;
    return S2_OK;
}

extern "C" s2_status s2_vae_conv3d_output_shape(const s2_vae_conv3d *l, int frames, int height, int width,
                                                int *out_frames, int *out_height, int *out_width)
{
    int od = 0, oh = 0, ow = 0;
    if (!l || frames <= 0 || height <= 0 || width <= 0 || !l->out_shape(frames, height, width, od, oh, ow))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_output_shape: input smaller than the kernel");
    if (out_frames) *out_frames = od;
    if (out_height) *out_height = oh;
    if (out_width) *out_width = ow;
    return S2_OK;
}

extern "C" s2_status s2_vae_conv3d_forward(s2_vae_conv3d *l, void *stream, const float *x, int frames, int height,
                                           int width, long long cstep, float *y, long long y_cstep)
{
    s2::clear_error();
    if (!l || !x || !y || frames <= 0 || height <= 0 || width <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_forward: invalid arguments");
    int od = 0, oh = 0, ow = 0;
    if (!l->out_shape(frames, height, width, od, oh, ow))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_forward: input smaller than the kernel");
    const long long tokens = 1LL * frames * height * width;
    const int owp = round_up(ow, 32);
    const long long rows = 1LL * od * oh * owp;
    if (cstep < tokens || y_cstep < 1LL * od * oh * ow || rows > (1LL << 31) - 256 || tokens > (1LL << 31))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_forward: bad cstep or too large");
    if (!l->loaded) return s2::set_error(S2_NOT_LOADED, "s2_vae_conv3d_forward: weights not loaded");
    s2::DeviceGuard guard(l->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool fresh = !l->err.ptr;
    if (!l->x16.ensure(static_cast<size_t>(tokens) * l->cpad * 2) || !l->err.ensure(4))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_vae_conv3d_forward: workspace allocation failed");
    if (fresh && cudaMemsetAsync(l->err.ptr, 0, 4, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_vae_conv3d_forward: memset failed");
    l->last_stream = st;
    s2_status s = to_tokens(st, x, cstep, tokens, l->cin, l->cpad, static_cast<__half *>(l->x16.ptr));
    if (s != S2_OK) return s;
    int f, t, lft, b, bo, r;
    l->pads(frames, height, width, f, t, lft, b, bo, r);
    s2::GemmArgs g;
    g.M = static_cast<int>(rows);
    g.N = l->cout;
    g.K = l->kd * l->kh * l->kw * l->cpad;
    g.bias = static_cast<const float *>(l->bias.ptr);
    g.epilogue = s2::GEMM_EPI_CONV_F32;
    g.y = y;
    g.ldt = y_cstep;
    g.n_valid = l->cout;
    g.conv = 1;
    g.err = static_cast<int32_t *>(l->err.ptr);
    s2::ConvGeom &cg = g.geom;
    cg.od = od, cg.oh = oh, cg.ow = ow, cg.owp = owp;
    cg.kd = l->kd, cg.kh = l->kh, cg.kw = l->kw;
    cg.sd = l->sd, cg.sh = l->sh, cg.sw = l->sw;
    cg.dd = l->dd, cg.dh = l->dh, cg.dw = l->dw;
    cg.pf = f, cg.pt = t, cg.pl = lft;
    cg.cslices = l->cpad / 64;
    cg.in_d = frames, cg.in_h = height, cg.in_w = width;
    s = s2::gemm_f16(st, l->x16.ptr, l->w16.ptr, g);
    if (s != S2_OK) return s;
    l->last_launches = 2;
    return S2_OK;
}

extern "C" s2_status s2_vae_conv3d_forward_host(s2_vae_conv3d *l, void *stream, const float *x, int frames,
                                                int height, int width, float *y)
{
    s2::clear_error();
    int od = 0, oh = 0, ow = 0;
    if (!l || !x || !y || frames <= 0 || height <= 0 || width <= 0 || !l->out_shape(frames, height, width, od, oh, ow))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_forward_host: invalid arguments");
    const long long tokens = 1LL * frames * height * width, out_plane = 1LL * od * oh * ow;
    s2_status s = forward_host(l->device, stream, l->hx, l->hy, x, static_cast<size_t>(tokens) * l->cin, y,
                               static_cast<size_t>(out_plane) * l->cout, [&](const float *dx, float *dy) {
                                   return s2_vae_conv3d_forward(l, stream, dx, frames, height, width, tokens, dy,
                                                                out_plane);
                               });
    if (s != S2_OK) return s;
    return check_err(l->device, static_cast<cudaStream_t>(stream), l->err, "s2_vae_conv3d");
}

extern "C" int s2_vae_conv3d_last_launches(const s2_vae_conv3d *l) { return l ? l->last_launches : 0; }

extern "C" s2_status s2_vae_conv3d_device_error(s2_vae_conv3d *l, int *code)
{
    if (code) *code = 0;
    if (!l) return s2::set_error(S2_INVALID_ARGUMENT, "s2_vae_conv3d_device_error: layer is NULL");
    return check_err(l->device, l->last_stream, l->err, "s2_vae_conv3d");
}
