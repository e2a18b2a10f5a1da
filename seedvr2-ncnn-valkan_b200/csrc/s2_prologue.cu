// Fused attention prologue and the text-mean epilogue.
//
// s2_qk_norm_rope: one pass over the QKV projection rows that produces the
// window-packed, head-major Q/K/V operands of the attention core (fp16 holding
// the reference's bf16-rounded values). Per (packed row, head): RMSNorm over
// the 128 head dims (sum of squares in fp32; the reference's accumulator is a
// double), times the branch gamma, 3-axis MM-RoPE on
// dims 0..125, bf16 round-to-nearest-even; V is only rounded
// (seedvr2_dit_block.cpp:942-1028). Every multiply/add of the normalisation
// and rotation uses explicitly rounded intrinsics so nothing is contracted
// into an FMA, matching the reference's float arithmetic step by step.
// Work split: 8 lanes per (row, head), each owning two 8-element chunks of the
// 128 head dims (so a warp covers 4 heads of a row and every per-(row, head)
// fixed cost -- the sum reduction, the IEEE sqrt and divide -- is paid
// once per 16 elements per lane); every 8-lane group moves full 128-byte lines
// with 128-bit loads and stores.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "s2_internal.h"

namespace {

constexpr int kHD = S2_HEAD_DIM;
constexpr int kPairs = S2_ROPE_PAIRS;

// cos/sin of pos * freqs[p] for every integer position used by a plan.
__global__ void rope_table_kernel(const float *__restrict__ freqs, int max_pos, float2 *__restrict__ table)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= max_pos * kPairs) return;
    const int pos = i / kPairs, pair = i - pos * kPairs;
    const float angle = __fmul_rn(static_cast<float>(pos), freqs[pair]);
    float s, c;
    sincosf(angle, &s, &c);
    table[i] = make_float2(c, s);
}

// The same values pair-major: table[pair * max_pos + pos] (a warp whose rows have
// different positions reads one pair's entries from one or two cache lines).
__global__ void rope_table_pairs_kernel(const float *__restrict__ freqs, int max_pos, float2 *__restrict__ table)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= max_pos * kPairs) return;
    const int pair = i / max_pos, pos = i - pair * max_pos;
    const float angle = __fmul_rn(static_cast<float>(pos), freqs[pair]);
    float s, c;
    sincosf(angle, &s, &c);
    table[i] = make_float2(c, s);
}

template <typename T>
struct Load8;

template <>
struct Load8<float> {
    __device__ __forceinline__ static void run(const float *p, float (&x)[8])
    {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
        const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
};

template <>
struct Load8<__half> {
    __device__ __forceinline__ static void run(const __half *p, float (&x)[8])
    {
        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    }
};

template <>
struct Load8<__nv_bfloat16> {
    __device__ __forceinline__ static void run(const __nv_bfloat16 *p, float (&x)[8])
    {
        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    }
};

// Round to bf16 (RNE) as the reference does, then store that value as fp16.
// The conversion is exact for bf16 values in fp16's normal range
// (6.1e-5 <= |x| < 65504); smaller magnitudes keep an absolute error below
// 3e-8. Both attention GEMMs then run as f16 x f16 on the tensor cores.
__device__ __forceinline__ uint32_t pack2(float a, float b)
{
    // one packed bf16x2 conversion (RNE) for both values, then one f16x2 pack
    const __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
    const uint32_t u = *reinterpret_cast<const uint32_t *>(&r);
    const __half2 h = __floats2half2_rn(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    return *reinterpret_cast<const uint32_t *>(&h);
}

template <typename TIn, bool kRange>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const TIn *__restrict__ vid_qkv,
                                                           const TIn *__restrict__ txt_qkv, int heads, float eps,
                                                           const float *__restrict__ gammas,
                                                           const float2 *__restrict__ table,
                                                           const s2_row *__restrict__ rows, int n_rows,
                                                           int src_lo, int src_hi, int do_text,
                                                           uint4 *__restrict__ q, uint4 *__restrict__ k,
                                                           uint4 *__restrict__ v)
{
    // kRange: only video rows whose source token is in [src_lo, src_hi) (and the
    // text rows when do_text) are processed; the others neither load nor store
    // (a host-buffer forward runs one pass per frame slab as its rows arrive).
    // Without kRange the loads stay unconditional, as the fastest schedule.
    // 8 lanes per (row, head); lane `sub` owns dims [64c + 8 sub, 64c + 8 sub + 8) for c = 0, 1.
    const int dim = heads * kHD;
    const int sub = threadIdx.x & 7;
    const long long n_pairs = 1LL * n_rows * heads;
    const long long per_block = blockDim.x >> 3;
    const long long stride = 1LL * gridDim.x * per_block;
    const long long lane_grp = (threadIdx.x >> 3) & 3;  // pair slot inside the warp
    for (long long pr = 1LL * blockIdx.x * per_block + (threadIdx.x >> 3); pr - lane_grp < n_pairs; pr += stride) {
        const bool active = pr < n_pairs;
        const long long prc = active ? pr : n_pairs - 1;
        const int row = static_cast<int>(prc / heads);
        const int head = static_cast<int>(prc - 1LL * row * heads);
        const s2_row rd = rows[row];
        const bool text = rd.src < 0;
        const bool use = !kRange || (active && (text ? do_text != 0 : (rd.src >= src_lo && rd.src < src_hi)));
        const TIn *src = text ? txt_qkv + static_cast<size_t>(-rd.src - 1) * 3 * dim
                              : vid_qkv + static_cast<size_t>(rd.src) * 3 * dim;
        src += head * kHD + sub * 8;
        const float *gq = gammas + (text ? 2 : 0) * kHD + sub * 8;
        const float *gk = gq + kHD;

        float xq[2][8], xk[2][8], xv[2][8];
#pragma unroll
        for (int c = 0; c < 2; c++) {
            if (!kRange || use) {
                Load8<TIn>::run(src + 64 * c, xq[c]);
                Load8<TIn>::run(src + dim + 64 * c, xk[c]);
                Load8<TIn>::run(src + 2 * dim + 64 * c, xv[c]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) xq[c][i] = xk[c][i] = xv[c][i] = 1.f;
            }
        }
        // Square sums in fp32, two chains per lane, then across the 8 lanes. The
        // reference sums in fp64; the fp32 sum of 128 squares is within ~1e-6
        // (relative) of it, which moves a bf16-rounded output by one unit only
        // where it sits that close to a rounding boundary. The fp64 form was
        // measured 4-6 % slower on this part.
        float sq2[2] = {0.f, 0.f}, sk2[2] = {0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                sq2[i & 1] = __fmaf_rn(xq[c][i], xq[c][i], sq2[i & 1]);
                sk2[i & 1] = __fmaf_rn(xk[c][i], xk[c][i], sk2[i & 1]);
            }
        float sq = __fadd_rn(sq2[0], sq2[1]), sk = __fadd_rn(sk2[0], sk2[1]);
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) {
            sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o, 8));
            sk = __fadd_rn(sk, __shfl_xor_sync(0xffffffffu, sk, o, 8));
        }
        const float inv_q = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(sq, 1.f / kHD), eps)));
        const float inv_k = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(sk, 1.f / kHD), eps)));
#pragma unroll
        for (int c = 0; c < 2; c++) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                xq[c][i] = __fmul_rn(__fmul_rn(xq[c][i], inv_q), __ldg(gq + 64 * c + i));
                xk[c][i] = __fmul_rn(__fmul_rn(xk[c][i], inv_k), __ldg(gk + 64 * c + i));
            }
            // pairs (d, d+1), d = 2 * gp; gp = axis * 21 + p covers gp < 63 (dims 0..125)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int gp = 32 * c + sub * 4 + i;
                if (gp < 3 * kPairs) {
                    const int axis = gp / kPairs, pair = gp - axis * kPairs;
                    const int pos = axis == 0 ? rd.pt : (axis == 1 ? rd.ph : rd.pw);
                    const float2 cs = __ldg(table + pos * kPairs + pair);
                    const float a0 = xq[c][2 * i], b0 = xq[c][2 * i + 1];
                    xq[c][2 * i] = __fsub_rn(__fmul_rn(a0, cs.x), __fmul_rn(b0, cs.y));
                    xq[c][2 * i + 1] = __fadd_rn(__fmul_rn(b0, cs.x), __fmul_rn(a0, cs.y));
                    const float c0 = xk[c][2 * i], d0 = xk[c][2 * i + 1];
                    xk[c][2 * i] = __fsub_rn(__fmul_rn(c0, cs.x), __fmul_rn(d0, cs.y));
                    xk[c][2 * i + 1] = __fadd_rn(__fmul_rn(d0, cs.x), __fmul_rn(c0, cs.y));
                }
            }
        }
        if (!active || !use) continue;
        const size_t o = (static_cast<size_t>(head) * n_rows + row) * (kHD / 8) + sub;
#pragma unroll
        for (int c = 0; c < 2; c++) {
            q[o + 8 * c] = make_uint4(pack2(xq[c][0], xq[c][1]), pack2(xq[c][2], xq[c][3]), pack2(xq[c][4], xq[c][5]),
                                      pack2(xq[c][6], xq[c][7]));
            k[o + 8 * c] = make_uint4(pack2(xk[c][0], xk[c][1]), pack2(xk[c][2], xk[c][3]), pack2(xk[c][4], xk[c][5]),
                                      pack2(xk[c][6], xk[c][7]));
            v[o + 8 * c] = make_uint4(pack2(xv[c][0], xv[c][1]), pack2(xv[c][2], xv[c][3]), pack2(xv[c][4], xv[c][5]),
                                      pack2(xv[c][6], xv[c][7]));
        }
    }
}

// txt_out[i] = (sum_w partial[w][i]) * scale: windows added in order in fp32,
// the reference's summation order (seedvr2_dit_block.cpp:1075, :1081-1088).
// One element per thread (the most loads in flight for a latency-bound
// in-order chain); the window loop is unrolled 16 deep so the loads of many
// windows are issued ahead of the in-order adds.
template <typename T>
__global__ void text_window_sum_kernel(const T *__restrict__ partial, int n_windows, long long n, float scale,
                                       int accumulate, float *__restrict__ out)
{
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x) {
        float acc = 0.f;
#pragma unroll 16
        for (int w = 0; w < n_windows; w++) acc = __fadd_rn(acc, static_cast<float>(partial[w * n + i]));
        acc = __fmul_rn(acc, scale);
        out[i] = accumulate ? __fadd_rn(out[i], acc) : acc;
    }
}

template <typename T>
__global__ void to_f32_kernel(const T *__restrict__ src, long long n, float *__restrict__ dst)
{
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x)
        dst[i] = static_cast<float>(src[i]);
}

int sm_count()
{
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" size_t s2_rope_table_bytes(int max_pos)
{
    return static_cast<size_t>(max_pos > 0 ? max_pos : 0) * kPairs * sizeof(float2);
}

extern "C" s2_status s2_rope_table(void *stream, const float *freqs21, int max_pos, void *rope_table)
{
    if (!freqs21 || max_pos <= 0 || !rope_table)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_rope_table: invalid arguments");
    const int tcount = max_pos * kPairs;
    rope_table_kernel<<<(tcount + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        freqs21, max_pos, static_cast<float2 *>(rope_table));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_rope_table: launch failed: %s", cudaGetErrorString(e));
    return S2_OK;
}

namespace s2 {

s2_status qk_norm_rope_range(void *stream, const void *vid_qkv, const void *txt_qkv, s2_dtype in_dtype, int heads,
                             float eps, const float *gammas, const void *rope_table, const s2_row *rows, int n_rows,
                             s2_mode mode, int src_lo, int src_hi, int do_text, void *q, void *k, void *v);

}  // namespace s2

extern "C" s2_status s2_qk_norm_rope(void *stream, const void *vid_qkv, const void *txt_qkv, s2_dtype in_dtype,
                                     int heads, float eps, const float *gammas, const void *rope_table,
                                     const s2_row *rows, int n_rows, s2_mode mode, void *q, void *k, void *v)
{
    return s2::qk_norm_rope_range(stream, vid_qkv, txt_qkv, in_dtype, heads, eps, gammas, rope_table, rows, n_rows,
                                  mode, 0, 0x7fffffff, 1, q, k, v);
}

s2_status s2::qk_norm_rope_range(void *stream, const void *vid_qkv, const void *txt_qkv, s2_dtype in_dtype,
                                 int heads, float eps, const float *gammas, const void *rope_table,
                                 const s2_row *rows, int n_rows, s2_mode mode, int src_lo, int src_hi, int do_text,
                                 void *q, void *k, void *v)
{
    if (heads <= 0 || heads > 64 || n_rows <= 0 || !vid_qkv || !gammas || !rows || !rope_table || !q || !k || !v)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_qk_norm_rope: invalid arguments");
    if (!aligned16(vid_qkv) || (txt_qkv && !aligned16(txt_qkv)) || !aligned16(q) || !aligned16(k) || !aligned16(v))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_qk_norm_rope: buffers must be 16-byte aligned");
    if (mode != S2_MODE_BF16_REF && mode != S2_MODE_F16 && mode != S2_MODE_BF16_F16)
        return s2::set_error(S2_UNSUPPORTED, "s2_qk_norm_rope: unknown mode %d", (int)mode);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool ranged = !(src_lo <= 0 && src_hi == 0x7fffffff && do_text);
    const long long pairs = 1LL * n_rows * heads;
    const long long want = (pairs + 31) / 32;
    // exactly the resident blocks: every block grid-strides to the end, so no
    // partial last wave of blocks runs at a fraction of the occupancy
    static int resident_per_sm[3] = {0, 0, 0};  // per input dtype, queried once
    const int di = in_dtype == S2_F32 ? 0 : in_dtype == S2_F16 ? 1 : 2;
    int per_sm = resident_per_sm[di];
    if (per_sm <= 0) {
        switch (in_dtype) {
        case S2_F32: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_norm_rope_kernel<float, false>, 256, 0); break;
        case S2_F16: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_norm_rope_kernel<__half, false>, 256, 0); break;
        default: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qk_norm_rope_kernel<__nv_bfloat16, false>, 256, 0); break;
        }
        if (per_sm <= 0) per_sm = 1;
        resident_per_sm[di] = per_sm;
    }
    const long long resident = 1LL * per_sm * sm_count();
    const int grid = static_cast<int>(want < resident ? want : resident);
    auto *Q = static_cast<uint4 *>(q);
    auto *K = static_cast<uint4 *>(k);
    auto *V = static_cast<uint4 *>(v);
    const auto *T = static_cast<const float2 *>(rope_table);
#define S2_LAUNCH(TIN)                                                                                              \
    if (ranged)                                                                                                     \
        qk_norm_rope_kernel<TIN, true><<<grid, 256, 0, st>>>(static_cast<const TIN *>(vid_qkv),                     \
                                                             static_cast<const TIN *>(txt_qkv), heads, eps, gammas, \
                                                             T, rows, n_rows, src_lo, src_hi, do_text, Q, K, V);    \
    else                                                                                                            \
        qk_norm_rope_kernel<TIN, false><<<grid, 256, 0, st>>>(static_cast<const TIN *>(vid_qkv),                    \
                                                              static_cast<const TIN *>(txt_qkv), heads, eps,        \
                                                              gammas, T, rows, n_rows, 0, 0, 1, Q, K, V)
    switch (in_dtype) {
    case S2_F32: S2_LAUNCH(float); break;
    case S2_F16: S2_LAUNCH(__half); break;
    case S2_BF16: S2_LAUNCH(__nv_bfloat16); break;
    default: return s2::set_error(S2_UNSUPPORTED, "s2_qk_norm_rope: unknown input dtype %d", (int)in_dtype);
    }
#undef S2_LAUNCH
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_qk_norm_rope: launch failed: %s", cudaGetErrorString(e));
    return S2_OK;
}

extern "C" s2_status s2_text_window_sum(void *stream, s2_mode mode, const void *txt_partial, int n_windows,
                                        int text_len, int dim, float scale, int accumulate, float *txt_out)
{
    if (text_len == 0) return S2_OK;
    if (!txt_partial || !txt_out || n_windows <= 0 || text_len < 0 || dim <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_text_window_sum: invalid arguments");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const long long n = 1LL * text_len * dim;
    const int grid = static_cast<int>((n + 255) / 256 < 8LL * sm_count() ? (n + 255) / 256 : 8LL * sm_count());
    if (mode == S2_MODE_F16 || mode == S2_MODE_BF16_F16)
        text_window_sum_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half *>(txt_partial), n_windows, n,
                                                             scale, accumulate, txt_out);
    else
        text_window_sum_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
            static_cast<const __nv_bfloat16 *>(txt_partial), n_windows, n, scale, accumulate, txt_out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_text_window_sum: launch failed: %s", cudaGetErrorString(e));
    return S2_OK;
}

namespace s2 {
s2_status rope_table_pairs(cudaStream_t st, const float *freqs21, int max_pos, void *table)
{
    if (!freqs21 || max_pos <= 0 || !table) return set_error(S2_INVALID_ARGUMENT, "rope table: invalid arguments");
    const int n = max_pos * kPairs;
    rope_table_pairs_kernel<<<(n + 255) / 256, 256, 0, st>>>(freqs21, max_pos, static_cast<float2 *>(table));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? S2_OK : set_error(S2_INFERENCE_FAILED, "rope table: launch failed: %s", cudaGetErrorString(e));
}

// 16-bit (mode dtype) -> fp32, used by the host-buffer forward.
s2_status to_f32(cudaStream_t st, s2_mode mode, const void *src, long long n, float *dst)
{
    if (n <= 0) return S2_OK;
    const int grid = static_cast<int>((n + 255) / 256 < 8LL * sm_count() ? (n + 255) / 256 : 8LL * sm_count());
    if (mode == S2_MODE_F16 || mode == S2_MODE_BF16_F16)
        to_f32_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half *>(src), n, dst);
    else
        to_f32_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(src), n, dst);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? S2_OK : set_error(S2_INFERENCE_FAILED, "to_f32: %s", cudaGetErrorString(e));
}
}  // namespace s2
