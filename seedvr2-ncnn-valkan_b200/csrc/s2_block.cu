// s2_dit_block: one SeedVR2DiTBlock (src/layers/seedvr2_dit_block.cpp:1114-1267)
// on sm_100a -- the block around the windowed attention:
//
//   a_x   = RMSNorm(x) (no gamma, eps) then adaLN shift/scale (slot 0)     :770-805, :1144-1150
//   qkv_x = a_x W_qkv^T                      (tcgen05 GEMM, fp16 out)     :1152-1154
//   attn  = s2_attention_layer (prologue + window attention + text mean)  :1168-1171
//   h_x   = (attn W_proj^T + b) * (emb[6c+2] + attn_gate) + x  (epilogue) :1180-1204
//   m_x   = RMSNorm(h_x) then shift/scale (slot 3)                        :1206-1208
//   hid   = silu(m W_gate^T) * (m W_in^T)    (one GEMM, SwiGLU epilogue)   :1093-1112
//   out_x = (hid W_out^T) * (emb[6c+5] + mlp_gate) + h_x   (epilogue)     :1216
//
// for x = video and text (text uses the text branch's weights unless the
// block shares them). The last block's text skips the adaLN input
// modulation and gate and returns 2 * (proj + txt) (:1146-1150, :1190-1200,
// :1220-1240). Activations entering a GEMM are fp16 (RNE); accumulation and
// residual streams stay fp32. Weights are uploaded once as fp16; the SwiGLU
// gate and "in" weights are interleaved in 128-row groups so one 256-column
// GEMM tile holds matching gate and in columns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <vector>

#include "s2_buffers.h"
#include "s2_gemm.h"
#include "s2_internal.h"
#include "s2_ops.h"

namespace {

// y = fp16( ada( x * inv_rms(x) [* gamma] ) ), one warp per row.
//   inv_rms = 1 / sqrt(float(sum x^2 (double) / dim) + eps)           (:770-782)
//   ada: (v * mul[c] + add0[c]) + add1[c] with mul = emb[6c + s + 1] + scale[c],
//        add0 = emb[6c + s], add1 = shift[c] precomputed (:784-805)
// mul == nullptr skips the modulation (the last block's text input); gamma is
// the output head's RMSNorm weight (seedvr2_dit_output.cpp:383).
// A run of rows with its own input, modulation vectors and output: one launch
// normalises the video rows and the text rows of a block (each with its branch's
// vectors), where the text rows alone would be a launch of a few dozen warps.
struct RmsSeg {
    const float *x = nullptr;
    const float *gamma = nullptr, *mul = nullptr, *add0 = nullptr, *add1 = nullptr;
    __half *y = nullptr;
    int rows = 0;
};

__global__ void __launch_bounds__(256) rms_ada_kernel(const RmsSeg s0, const RmsSeg s1, int dim, float eps)
{
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= s0.rows + s1.rows) return;
    const bool second = w >= s0.rows;
    const int warp = second ? w - s0.rows : w;
    const float *x = second ? s1.x : s0.x;
    const float *gamma = second ? s1.gamma : s0.gamma, *mul = second ? s1.mul : s0.mul;
    const float *add0 = second ? s1.add0 : s0.add0, *add1 = second ? s1.add1 : s0.add1;
    __half *y = second ? s1.y : s0.y;
    const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<size_t>(warp) * dim);
    double ss = 0.0;
    for (int i = lane; i < dim / 4; i += 32) {
        const float4 v = __ldg(xr + i);
        ss += static_cast<double>(v.x) * v.x;
        ss += static_cast<double>(v.y) * v.y;
        ss += static_cast<double>(v.z) * v.z;
        ss += static_cast<double>(v.w) * v.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(static_cast<float>(ss / dim), eps)));
    __half2 *yr = reinterpret_cast<__half2 *>(y + static_cast<size_t>(warp) * dim);
    for (int i = lane; i < dim / 4; i += 32) {
        const float4 v = __ldg(xr + i);
        float f[4] = {__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv), __fmul_rn(v.w, inv)};
        if (gamma) {
            const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma) + i);
            f[0] = __fmul_rn(f[0], g.x);
            f[1] = __fmul_rn(f[1], g.y);
            f[2] = __fmul_rn(f[2], g.z);
            f[3] = __fmul_rn(f[3], g.w);
        }
        if (mul) {
            const float4 m = __ldg(reinterpret_cast<const float4 *>(mul) + i);
            const float4 a = __ldg(reinterpret_cast<const float4 *>(add0) + i);
            const float4 b = __ldg(reinterpret_cast<const float4 *>(add1) + i);
            f[0] = __fadd_rn(__fadd_rn(__fmul_rn(f[0], m.x), a.x), b.x);
            f[1] = __fadd_rn(__fadd_rn(__fmul_rn(f[1], m.y), a.y), b.y);
            f[2] = __fadd_rn(__fadd_rn(__fmul_rn(f[2], m.z), a.z), b.z);
            f[3] = __fadd_rn(__fadd_rn(__fmul_rn(f[3], m.w), a.w), b.w);
        }
        yr[2 * i] = __floats2half2_rn(f[0], f[1]);
        yr[2 * i + 1] = __floats2half2_rn(f[2], f[3]);
    }
}

// Per-forward modulation vectors of a branch from the block input emb and the
// branch's [6][dim] adaLN parameters (attn shift, scale, gate, mlp shift,
// scale, gate): out [8][dim] = attn {mul, add0, add1}, mlp {mul, add0, add1},
// attn gate, mlp gate, with mul = emb[6c + s + 1] + scale, add0 = emb[6c + s],
// add1 = shift, gate = emb[6c + s + 2] + gate (s = 0 attention, 3 MLP).
__global__ void modulation_kernel(const float *__restrict__ emb, const float *__restrict__ mod6, int dim,
                                  float *__restrict__ out)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= dim) return;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int s = 3 * k;
        out[(3 * k + 0) * dim + c] = __fadd_rn(emb[6 * c + s + 1], mod6[(s + 1) * dim + c]);
        out[(3 * k + 1) * dim + c] = emb[6 * c + s];
        out[(3 * k + 2) * dim + c] = mod6[s * dim + c];
        out[(6 + k) * dim + c] = __fadd_rn(emb[6 * c + s + 2], mod6[(s + 2) * dim + c]);
    }
}

__global__ void f32_to_f16_kernel(const float *__restrict__ x, long long n, __half *__restrict__ y)
{
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += 256LL * gridDim.x) y[i] = __float2half_rn(x[i]);
}

struct Branch {
    s2::DeviceBuffer mod;    // fp32 [6][dim]: attn_shift, attn_scale, attn_gate, mlp_shift, mlp_scale, mlp_gate
    s2::DeviceBuffer qkv;    // fp16 [3 dim][dim]
    s2::DeviceBuffer proj;   // fp16 [dim][dim]
    s2::DeviceBuffer proj_b; // fp32 [dim]
    s2::DeviceBuffer gu;     // fp16 [2 hidden][dim], gate/in interleaved by 128 rows
    s2::DeviceBuffer out;    // fp16 [dim][hidden]
    std::vector<float> norm_q, norm_k;
    void release()
    {
        for (s2::DeviceBuffer *b : {&mod, &qkv, &proj, &proj_b, &gu, &out}) b->release();
    }
    const float *m(int k, int dim) const { return static_cast<const float *>(mod.ptr) + static_cast<size_t>(k) * dim; }
};

bool upload(s2::DeviceBuffer &b, const void *src, size_t bytes)
{
    return b.ensure(bytes) && cudaMemcpy(b.ptr, src, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
}

__global__ void f32_to_f16_kernel(const float *__restrict__ x, long long n, __half *__restrict__ y);

// fp32 host weights -> fp16 device weights, converted on the device
bool upload_f16(s2::DeviceBuffer &b, const float *src, size_t n)
{
    if (!b.ensure(n * 2)) return false;
    void *tmp = nullptr;
    if (cudaMalloc(&tmp, n * 4) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    bool ok = cudaMemcpy(tmp, src, n * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    if (ok) {
        f32_to_f16_kernel<<<static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 4096)), 256>>>(
            static_cast<const float *>(tmp), static_cast<long long>(n), static_cast<__half *>(b.ptr));
        ok = cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaFree(tmp);
    return ok;
}

}  // namespace

// Activation workspaces of a block forward, shareable between blocks that run
// one after another.
struct BlockScratch {
    int device = 0;
    s2::DeviceBuffer a_vid, a_txt, qkv_vid, qkv_txt, att_vid, att_txt32, att_txt16, h_vid, h_txt, hid_vid, hid_txt;
    // split-K partial sums of the projections of a few dozen rows (the text rows):
    // gemm_f16 splits only GEMMs of at most 128 rows and keeps splits x tiles <=
    // the SM count, each split holding at most 128 rows x 256 columns, so
    // 128 x 256 x SMs floats bound every split GEMM of the device.
    s2::DeviceBuffer splitk;
    static size_t splitk_floats(int device)
    {
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        return static_cast<size_t>(128) * 256 * static_cast<size_t>(std::max(sms, 1));
    }
    ~BlockScratch()
    {
        s2::DeviceGuard guard(device);
        for (s2::DeviceBuffer *x : {&a_vid, &a_txt, &qkv_vid, &qkv_txt, &att_vid, &att_txt32, &att_txt16, &h_vid, &h_txt,
                                    &hid_vid, &hid_txt, &splitk})
            x->release();
    }
};

struct s2_dit_block {
    int device = 0;
    int block_index = 0, shared = 0, last = 0, shifted = 0;
    int dim = 2560, heads = 20, head_dim = 128, hidden = 6912;
    float eps = 1e-5f;
    bool loaded = false;
    Branch vid, txt;
    s2_attention_layer *attn = nullptr;
    std::shared_ptr<BlockScratch> sc = std::make_shared<BlockScratch>();
    s2::DeviceBuffer mods;  // fp32 [2 branches][8][dim] modulation vectors of the current forward
    s2::DeviceBuffer err;
    s2::DeviceBuffer hv, ht, he, hov, hot;  // forward_host staging
    int last_launches = 0;
    cudaStream_t last_stream = nullptr;
    bool debug_on = false;  // set_debug_tensors (device buffers)
    s2_block_debug debug{};
    bool debug_host_on = false;  // set_debug_tensors_host (host buffers, forward_host)
    static_assert(sizeof(s2_block_debug) == 14 * sizeof(float *), "s2_block_debug is 14 pointers");
    s2_block_debug debug_host{};
    s2::DeviceBuffer debug_stage;
    const Branch &tb() const { return shared ? vid : txt; }
};

extern "C" s2_status s2_dit_block_create(int device, int block_index, int shared, int last, int shifted, int dim,
                                         int heads, int head_dim, int mlp_hidden, float eps, int wt, int wh, int ww,
                                         s2_dit_block **out)
{
    s2::clear_error();
    if (!out) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_create: out is NULL");
    *out = nullptr;
    if (dim != heads * head_dim || heads <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_create: dim %d != heads %d * head_dim %d", dim, heads,
                             head_dim);
    if (head_dim != S2_HEAD_DIM)
        return s2::set_error(S2_UNSUPPORTED, "s2_dit_block_create: head_dim %d (only 128)", head_dim);
    if (mlp_hidden <= 0 || mlp_hidden % 128 != 0)
        return s2::set_error(S2_UNSUPPORTED, "s2_dit_block_create: mlp_hidden %d must be a multiple of 128", mlp_hidden);
    auto *b = new s2_dit_block();
    b->device = device;
    b->sc->device = device;
    b->block_index = block_index;
    b->shared = shared != 0;
    b->last = last != 0;
    b->shifted = shifted != 0;
    b->dim = dim;
    b->heads = heads;
    b->head_dim = head_dim;
    b->hidden = mlp_hidden;
    b->eps = eps;
    const s2_status st =
        s2_attention_layer_create(device, heads, head_dim, eps, shifted, wt, wh, ww, S2_MODE_BF16_F16, &b->attn);
    if (st != S2_OK) {
        delete b;
        return st;
    }
    *out = b;
    return S2_OK;
}

extern "C" s2_status s2_dit_block_destroy(s2_dit_block *b)
{
    if (!b) return S2_OK;
    {
        s2::DeviceGuard guard(b->device);
        b->vid.release();
        b->txt.release();
        for (s2::DeviceBuffer *x : {&b->mods, &b->err, &b->hv, &b->ht, &b->he, &b->hov, &b->hot, &b->debug_stage})
            x->release();
    }
    s2_attention_layer_destroy(b->attn);
    delete b;
    return S2_OK;
}

// Number of floats of one branch in the weight stream (load_branch, :657-680).
static size_t branch_floats(const s2_dit_block *b)
{
    const size_t d = b->dim, h = b->hidden, hd = b->head_dim;
    return 6 * d + 3 * d * d + d * d + d + 2 * hd + 2 * h * d + d * h;
}

extern "C" size_t s2_dit_block_weight_count(const s2_dit_block *b)
{
    return b ? branch_floats(b) * (b->shared ? 1 : 2) + S2_ROPE_PAIRS : 0;
}

extern "C" s2_status s2_dit_block_load(s2_dit_block *b, const float *w, size_t n_floats)
{
    s2::clear_error();
    if (!b || !w) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_load: null argument");
    if (n_floats != s2_dit_block_weight_count(b))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_load: %zu floats, the layer reads %zu", n_floats,
                             s2_dit_block_weight_count(b));
    s2::DeviceGuard guard(b->device);
    const size_t d = b->dim, h = b->hidden, hd = b->head_dim;
    auto load_branch = [&](const float *p, Branch &br) -> bool {
        bool ok = upload(br.mod, p, 6 * d * 4);
        p += 6 * d;
        ok = ok && upload_f16(br.qkv, p, 3 * d * d);
        p += 3 * d * d;
        ok = ok && upload_f16(br.proj, p, d * d);
        p += d * d;
        ok = ok && upload(br.proj_b, p, d * 4);
        p += d;
        br.norm_q.assign(p, p + hd);
        p += hd;
        br.norm_k.assign(p, p + hd);
        p += hd;
        // interleave gate / in rows by groups of 128 -> [2h][d]
        std::vector<float> gu(2 * h * d);
        const float *gate = p, *in = p + h * d;
        for (size_t g = 0; g < h / 128; ++g) {
            std::memcpy(&gu[(2 * g) * 128 * d], gate + g * 128 * d, 128 * d * 4);
            std::memcpy(&gu[(2 * g + 1) * 128 * d], in + g * 128 * d, 128 * d * 4);
        }
        p += 2 * h * d;
        ok = ok && upload_f16(br.gu, gu.data(), gu.size());
        ok = ok && upload_f16(br.out, p, d * h);
        return ok;
    };
    if (!load_branch(w, b->vid))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_block_load: weight upload failed");
    const float *freqs = w + branch_floats(b);
    if (!b->shared) {
        if (!load_branch(w + branch_floats(b), b->txt))
            return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_block_load: weight upload failed");
        freqs += branch_floats(b);
    }
    const Branch &t = b->tb();
    const s2_status st =
        s2_attention_layer_load(b->attn, b->vid.norm_q.data(), b->vid.norm_k.data(), t.norm_q.data(), t.norm_k.data(), freqs);
    if (st != S2_OK) return st;
    b->loaded = true;
    return S2_OK;
}

extern "C" s2_status s2_dit_block_set_runtime_shape(s2_dit_block *b, int frames, int height, int width)
{
    if (!b) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_set_runtime_shape: block is NULL");
    return s2_attention_layer_set_runtime_shape(b->attn, frames, height, width);
}

extern "C" s2_status s2_dit_block_set_window_subset(s2_dit_block *b, const int32_t *ids, int n)
{
    if (!b) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_set_window_subset: block is NULL");
    return s2_attention_layer_set_window_subset(b->attn, ids, n);
}

namespace {

RmsSeg seg3(const float *x, int rows, int dim, const float *mod3, __half *y)
{
    RmsSeg g;
    g.x = x;
    g.rows = rows;
    g.mul = mod3;
    g.add0 = mod3 ? mod3 + dim : nullptr;
    g.add1 = mod3 ? mod3 + 2 * dim : nullptr;
    g.y = y;
    return g;
}

s2_status rms_launch(cudaStream_t st, const RmsSeg &a, const RmsSeg &b, int dim, float eps)
{
    const int rows = a.rows + b.rows;
    if (rows <= 0) return S2_OK;
    if (dim % 4 != 0) return s2::set_error(S2_INVALID_ARGUMENT, "rms_ada: dim %d not a multiple of 4", dim);
    rms_ada_kernel<<<(rows + 7) / 8, 256, 0, st>>>(a, b, dim, eps);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? S2_OK : s2::set_error(S2_INFERENCE_FAILED, "rms_ada launch: %s", cudaGetErrorString(e));
}

// RMSNorm + adaLN (slot given by mod3) of `rows` rows, and of a second run of rows
// with its own vectors in the same launch
s2_status rms_ada3(cudaStream_t st, const float *x, int rows, int dim, float eps, const float *mod3, __half *y,
                   const float *x2 = nullptr, int rows2 = 0, const float *mod3_2 = nullptr, __half *y2 = nullptr)
{
    return rms_launch(st, seg3(x, rows, dim, mod3, y), seg3(x2, rows2, dim, mod3_2, y2), dim, eps);
}

}  // namespace

namespace s2 {

s2_status rms_ada(cudaStream_t st, const float *x, int rows, int dim, float eps, const float *gamma, const float *mul,
                  const float *add0, const float *add1, void *y)
{
    RmsSeg a;
    a.x = x;
    a.rows = rows;
    a.gamma = gamma;
    a.mul = mul;
    a.add0 = add0;
    a.add1 = add1;
    a.y = static_cast<__half *>(y);
    return rms_launch(st, a, RmsSeg{}, dim, eps);
}

s2_status modulation_vectors(cudaStream_t st, const float *emb, const float *mod6, int dim, float *out)
{
    modulation_kernel<<<(dim + 255) / 256, 256, 0, st>>>(emb, mod6, dim, out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? S2_OK : set_error(S2_INFERENCE_FAILED, "modulation launch: %s", cudaGetErrorString(e));
}

s2_status f32_to_f16(cudaStream_t st, const float *x, long long n, void *y)
{
    if (n <= 0) return S2_OK;
    f32_to_f16_kernel<<<static_cast<unsigned>(std::min<long long>((n + 255) / 256, 1024)), 256, 0, st>>>(
        x, n, static_cast<__half *>(y));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? S2_OK : set_error(S2_INFERENCE_FAILED, "f32_to_f16 launch: %s", cudaGetErrorString(e));
}

void share_block_scratch(s2_dit_block *dst, const s2_dit_block *src)
{
    if (!dst || !src || dst == src) return;
    dst->sc = src->sc;
    share_attention_scratch(dst->attn, src->attn);
}

}  // namespace s2

extern "C" s2_status s2_dit_block_forward(s2_dit_block *b, void *stream, const float *vid, int L, const float *txt,
                                          int Lt, const float *emb, float *vid_out, float *txt_out)
{
    return s2::dit_block_forward_ex(b, stream, vid, L, txt, Lt, emb, vid_out, txt_out, nullptr);
}

s2_attention_layer *s2::dit_block_attention(s2_dit_block *b) { return b ? b->attn : nullptr; }

extern "C" s2_status s2_dit_block_set_local_rows(s2_dit_block *b, int enable)
{
    if (!b) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_set_local_rows: block is NULL");
    return s2_attention_layer_set_local_rows(b->attn, enable);
}

s2_status s2::dit_block_forward_ex(s2_dit_block *b, void *stream, const float *vid, int L, const float *txt, int Lt,
                                   const float *emb, float *vid_out, float *txt_out, const TextReduce *reduce,
                                   const RowScatter *scatter)
{
    s2::clear_error();
    if (!b) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_forward: block is NULL");
    if (!b->loaded) return s2::set_error(S2_NOT_LOADED, "s2_dit_block_forward: weights not loaded");
    if (!vid || !emb || !vid_out || L <= 0 || Lt < 0 || (Lt > 0 && (!txt || !txt_out)))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_forward: invalid arguments");
    if (vid == vid_out || (Lt > 0 && txt == txt_out))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_forward: in-place forward is not supported");
    if (scatter && (b->debug_on || b->debug_host_on || !scatter->dest))
        return s2::set_error(S2_UNSUPPORTED, "s2_dit_block_forward: row scatter without debug captures only");
    s2::DeviceGuard guard(b->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int d = b->dim, h = b->hidden;
    // With shared weights the text rows ride along as rows L .. L+Lt of the video GEMMs.
    const bool merged = b->shared && Lt > 0;
    const size_t Lz = static_cast<size_t>(L) + static_cast<size_t>(std::max(Lt, 0)), Tz = static_cast<size_t>(std::max(Lt, 1));
    const bool fresh = b->err.ptr == nullptr;
    BlockScratch &sc = *b->sc;
    // gemm_f16 can split K only for GEMMs of at most 128 rows with at least 8
    // K slices of 64 (K >= 512): the text rows of an unshared block or of the
    // last block's projection, or a block of few video rows. Otherwise no
    // workspace is allocated or passed.
    const int gemm_rows_min = Lt > 0 ? std::min(L, Lt) : L;
    const bool need_splitk = gemm_rows_min <= 128 && std::max(d, h) >= 512;
    const size_t splitk_cap = need_splitk ? BlockScratch::splitk_floats(b->device) : 0;
    // The attention prologue (QK-RMSNorm, MM-RoPE, bf16 rounding, window packing) runs in
    // the Q|K|V projection's epilogue on the fp32 accumulator. The projection itself is
    // materialised (fp32, by a second GEMM) only for the debug captures.
    if (!sc.a_vid.ensure(Lz * d * 2) || !sc.a_txt.ensure(Tz * d * 2) ||
        (b->debug_on && (!sc.qkv_vid.ensure(Lz * 3 * d * 4) || !sc.qkv_txt.ensure(Tz * 3 * d * 4))) ||
        !sc.att_vid.ensure(Lz * d * 2) || !sc.att_txt32.ensure(Tz * d * 4) ||
        !sc.att_txt16.ensure(Tz * d * 2) || !sc.h_vid.ensure(Lz * d * 4) || !sc.h_txt.ensure(Tz * d * 4) ||
        !sc.hid_vid.ensure(Lz * h * 2) || !sc.hid_txt.ensure(Tz * h * 2) || !b->err.ensure(4) ||
        (need_splitk && !sc.splitk.ensure(splitk_cap * sizeof(float))) ||
        !b->mods.ensure(static_cast<size_t>(16) * d * 4))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_block_forward: workspace allocation failed");
    if (fresh && cudaMemsetAsync(b->err.ptr, 0, 4, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block_forward: memset failed");
    int32_t *err = static_cast<int32_t *>(b->err.ptr);
    const Branch &V = b->vid, &T = b->tb();
    b->last_stream = st;
    int launches = 0;
    s2_status s;
#define S2_TRY(expr)                 \
    do {                             \
        if ((s = (expr)) != S2_OK) { \
            b->last_launches = launches; \
            return s;                \
        }                            \
        ++launches;                  \
    } while (0)
    const size_t dz = static_cast<size_t>(d);
    __half *a_vid = static_cast<__half *>(sc.a_vid.ptr);
    __half *a_txt = merged ? a_vid + static_cast<size_t>(L) * dz : static_cast<__half *>(sc.a_txt.ptr);
    __half *att_vid = static_cast<__half *>(sc.att_vid.ptr);
    __half *att_txt16 = merged ? att_vid + static_cast<size_t>(L) * dz : static_cast<__half *>(sc.att_txt16.ptr);
    float *h_vid = static_cast<float *>(sc.h_vid.ptr);
    float *h_txt = merged ? h_vid + static_cast<size_t>(L) * dz : static_cast<float *>(sc.h_txt.ptr);

    // modulation vectors: video branch, and the text branch when it has its own weights and uses them
    float *mv = static_cast<float *>(b->mods.ptr), *mt = mv;
    S2_TRY(s2::modulation_vectors(st, emb, V.m(0, d), d, mv));
    if (Lt > 0 && !b->shared && !b->last) {
        mt = mv + 8 * dz;
        S2_TRY(s2::modulation_vectors(st, emb, T.m(0, d), d, mt));
    }
    // attention input: RMSNorm + adaLN (slot 0); the last block's text is only normalised
    S2_TRY(rms_ada3(st, vid, L, d, b->eps, mv, a_vid, txt, Lt, b->last ? nullptr : mt, a_txt));
    // QKV projections (no bias) into the attention core's packed operands; the map
    // covers the L video rows, then the Lt text rows (the merged GEMM's rows L.., or
    // the text GEMM's rows)
    float *splitk = need_splitk ? static_cast<float *>(sc.splitk.ptr) : nullptr;
    int extra = 0;  // split-K finish kernels
    s2::GemmArgs g;
    g.K = d;
    g.N = 3 * d;
    g.err = err;
    g.extra_launches = &extra;
    g.M = merged ? L + Lt : L;
    g.epilogue = s2::GEMM_EPI_QKV_PACK;
    if ((s = s2::attention_pack_target(b->attn, st, L, Lt, &g)) != S2_OK) {  // set-up only, no launch
        b->last_launches = launches;
        return s;
    }
    S2_TRY(s2::gemm_f16(st, a_vid, V.qkv.ptr, g));
    if (Lt > 0 && !merged) {
        g.M = Lt;
        g.pk.map += L;
        g.partial = splitk;  // a few dozen rows: split K, the finish kernel applies the prologue
        g.partial_floats = splitk_cap;
        S2_TRY(s2::gemm_f16(st, a_txt, T.qkv.ptr, g));
    }
    // windowed MM attention (attention core, text mean)
    if ((s = s2::attention_forward_packed(b->attn, st, L, Lt, att_vid, static_cast<float *>(sc.att_txt32.ptr))) !=
        S2_OK) {
        b->last_launches = launches;
        return s;
    }
    launches += s2_attention_layer_last_launches(b->attn);
    if (b->debug_on) {
        // the projection alone in fp32 (the reference's qkv_vid / qkv_txt captures), from
        // which the pre-RoPE normalised q/k captures are taken
        const s2_block_debug &g = b->debug;
        float *q32v = static_cast<float *>(sc.qkv_vid.ptr), *q32t = static_cast<float *>(sc.qkv_txt.ptr);
        s2::GemmArgs q;
        q.K = d;
        q.N = 3 * d;
        q.epilogue = s2::GEMM_EPI_GATED_RESID_F32;
        q.err = err;
        q.M = merged ? L + Lt : L;
        q.y = q32v;
        if (merged) {
            q.split_row = L;
            q.y2 = q32t;
        }
        S2_TRY(s2::gemm_f16(st, a_vid, V.qkv.ptr, q));
        if (Lt > 0 && !merged) {
            q.M = Lt;
            q.y = q32t;
            S2_TRY(s2::gemm_f16(st, a_txt, T.qkv.ptr, q));
        }
        const size_t nq = static_cast<size_t>(L) * 3 * d * 4, nt = static_cast<size_t>(Lt) * 3 * d * 4;
        if ((g.qkv_vid && cudaMemcpyAsync(g.qkv_vid, q32v, nq, cudaMemcpyDeviceToDevice, st) != cudaSuccess) ||
            (g.qkv_txt && Lt > 0 && cudaMemcpyAsync(g.qkv_txt, q32t, nt, cudaMemcpyDeviceToDevice, st) != cudaSuccess)) {
            b->last_launches = launches;
            return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block_forward: debug copy failed");
        }
        if ((s = s2::attention_debug_capture(b->attn, st, q32v, S2_F32, L, q32t, Lt, att_vid, g.attention_q,
                                             g.attention_k, g.attention_v, g.attention_output, g.norm_q_vid,
                                             g.norm_k_vid, g.norm_q_txt, g.norm_k_txt)) != S2_OK) {
            b->last_launches = launches;
            return s;
        }
    }
    if (reduce && reduce->fn && Lt > 0 &&
        (s = reduce->fn(reduce->ctx, static_cast<float *>(sc.att_txt32.ptr), static_cast<size_t>(Lt) * d, st)) != S2_OK) {
        b->last_launches = launches;
        return s;
    }
    if (Lt > 0) {
        const long long n = static_cast<long long>(Lt) * d;
        f32_to_f16_kernel<<<static_cast<unsigned>(std::min<long long>((n + 255) / 256, 1024)), 256, 0, st>>>(
            static_cast<const float *>(sc.att_txt32.ptr), n, att_txt16);
        if (cudaGetLastError() != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block_forward: convert launch failed");
        ++launches;
    }
    // debug capture: the output projection + bias alone (the reference's vid_projected /
    // txt_projected, seedvr2_dit_block.cpp:1176-1191); the forward fuses it with the gate
    if (b->debug_on) {
        const s2_block_debug &g = b->debug;
        s2::GemmArgs q;
        q.K = d;
        q.N = d;
        q.epilogue = s2::GEMM_EPI_GATED_RESID_F32;
        q.err = err;
        if (g.projected_vid) {
            q.M = L;
            q.bias = static_cast<const float *>(V.proj_b.ptr);
            q.y = g.projected_vid;
            S2_TRY(s2::gemm_f16(st, att_vid, V.proj.ptr, q));
        }
        if (g.projected_txt && Lt > 0) {
            q.M = Lt;
            q.bias = static_cast<const float *>(T.proj_b.ptr);
            q.y = g.projected_txt;
            S2_TRY(s2::gemm_f16(st, att_txt16, T.proj.ptr, q));
        }
    }
    // output projection + gated residual
    const bool merged_rest = merged && !b->last;
    s2::GemmArgs p;
    p.K = d;
    p.N = d;
    p.epilogue = s2::GEMM_EPI_GATED_RESID_F32;
    p.err = err;
    p.partial = splitk;
    p.partial_floats = splitk_cap;
    p.extra_launches = &extra;
    p.M = merged_rest ? L + Lt : L;
    p.bias = static_cast<const float *>(V.proj_b.ptr);
    p.gmul = mv + 6 * dz;
    p.resid = vid;
    p.y = h_vid;
    if (merged_rest) {
        p.split_row = L;
        p.resid2 = txt;
        p.y2 = h_txt;
    }
    S2_TRY(s2::gemm_f16(st, att_vid, V.proj.ptr, p));
    if (Lt > 0 && !merged_rest) {
        s2::GemmArgs q;
        q.K = d;
        q.N = d;
        q.epilogue = s2::GEMM_EPI_GATED_RESID_F32;
        q.err = err;
        q.partial = splitk;
        q.partial_floats = splitk_cap;
        q.extra_launches = &extra;
        q.M = Lt;
        q.bias = static_cast<const float *>(T.proj_b.ptr);
        q.resid = txt;
        if (b->last) {
            // vid_only modulation: plain residual, and the text output is 2 * (proj + txt)
            q.out_scale = 2.f;
            q.y = txt_out;
        } else {
            q.gmul = mt + 6 * dz;
            q.y = h_txt;
        }
        S2_TRY(s2::gemm_f16(st, att_txt16, T.proj.ptr, q));
    }
    // MLP: RMSNorm + adaLN (slot 3), SwiGLU GEMM, output GEMM + gated residual
    // a text branch with its own MLP (unshared weights, not the last block) has its MLP input
    // normalised in the video rows' launch
    const bool text_mlp = Lt > 0 && !b->last && !merged_rest;
    auto mlp = [&](const float *mb, const Branch &br, const float *hx, int rows, __half *a16, __half *hid, float *y,
                   int split, float *y2, const s2::RowScatter *sc_rows, bool normed) -> s2_status {
        s2_status r;
        if (!normed) {
            r = text_mlp ? rms_ada3(st, hx, rows, d, b->eps, mb + 3 * dz, a16, h_txt, Lt, mt + 3 * dz,
                                    static_cast<__half *>(sc.a_txt.ptr))
                         : rms_ada3(st, hx, rows, d, b->eps, mb + 3 * dz, a16);
            if (r != S2_OK) return r;
            ++launches;
        }
        s2::GemmArgs u;
        u.M = rows;
        u.N = 2 * h;
        u.K = d;
        u.epilogue = s2::GEMM_EPI_SWIGLU_F16;
        u.out[0] = hid;
        u.err = err;
        u.partial = splitk;
        u.partial_floats = splitk_cap;
        u.extra_launches = &extra;
        if ((r = s2::gemm_f16(st, a16, br.gu.ptr, u)) != S2_OK) return r;
        ++launches;
        s2::GemmArgs o;
        o.M = rows;
        o.N = d;
        o.K = h;
        o.epilogue = s2::GEMM_EPI_GATED_RESID_F32;
        o.gmul = mb + 7 * dz;
        o.partial = splitk;
        o.partial_floats = splitk_cap;
        o.extra_launches = &extra;
        o.resid = hx;
        o.y = y;
        if (sc_rows) {
            o.y = nullptr;
            o.row_dest = sc_rows->dest;
            for (int q = 0; q < 8; ++q) o.dest_base[q] = sc_rows->base[q];
        }
        if (split > 0) {
            o.split_row = split;
            o.resid2 = hx + static_cast<size_t>(split) * dz;
            o.y2 = y2;
        }
        o.err = err;
        if ((r = s2::gemm_f16(st, hid, br.out.ptr, o)) != S2_OK) return r;
        ++launches;
        return S2_OK;
    };
    if ((s = mlp(mv, V, h_vid, merged_rest ? L + Lt : L, a_vid, static_cast<__half *>(sc.hid_vid.ptr), vid_out,
                 merged_rest ? L : 0, txt_out, scatter, false)) != S2_OK) {
        b->last_launches = launches;
        return s;
    }
    if (text_mlp &&
        (s = mlp(mt, T, h_txt, Lt, static_cast<__half *>(sc.a_txt.ptr), static_cast<__half *>(sc.hid_txt.ptr), txt_out,
                 0, nullptr, nullptr, true)) != S2_OK) {
        b->last_launches = launches;
        return s;
    }
    if (b->debug_on) {
        const s2_block_debug &g = b->debug;
        if ((g.output_vid && cudaMemcpyAsync(g.output_vid, vid_out, static_cast<size_t>(L) * dz * 4,
                                             cudaMemcpyDeviceToDevice, st) != cudaSuccess) ||
            (g.output_txt && Lt > 0 &&
             cudaMemcpyAsync(g.output_txt, txt_out, static_cast<size_t>(Lt) * dz * 4, cudaMemcpyDeviceToDevice, st) !=
                 cudaSuccess))
            return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block_forward: debug copy failed");
    }
#undef S2_TRY
    b->last_launches = launches + extra;
    return S2_OK;
}

extern "C" s2_status s2_dit_block_set_debug_tensors(s2_dit_block *b, const s2_block_debug *tensors)
{
    s2::clear_error();
    if (!b) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_set_debug_tensors: block is NULL");
    b->debug_on = tensors != nullptr;
    b->debug = tensors ? *tensors : s2_block_debug{};
    return S2_OK;
}

extern "C" s2_status s2_dit_block_set_debug_tensors_host(s2_dit_block *b, const s2_block_debug *tensors)
{
    s2::clear_error();
    if (!b) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_set_debug_tensors_host: block is NULL");
    b->debug_host_on = tensors != nullptr;
    b->debug_host = tensors ? *tensors : s2_block_debug{};
    return S2_OK;
}

extern "C" s2_status s2_dit_block_debug_rows(s2_dit_block *b, int Lt, int *rows)
{
    s2::clear_error();
    if (!b || !rows || Lt < 0) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_debug_rows: invalid arguments");
    int n_video = 0;
    const s2_status s = s2_attention_layer_local_rows(b->attn, Lt, &n_video);  // builds the plan for Lt
    if (s != S2_OK) return s;
    *rows = s2::attention_debug_rows(b->attn);
    return S2_OK;
}

extern "C" s2_status s2_dit_block_forward_host(s2_dit_block *b, void *stream, const float *vid, int L, const float *txt,
                                               int Lt, const float *emb, const int32_t *vid_shape, float *vid_out,
                                               float *txt_out)
{
    s2::clear_error();
    if (!b || !vid || !emb || !vid_shape || !vid_out || L <= 0 || Lt < 0 || (Lt > 0 && (!txt || !txt_out)))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_forward_host: invalid arguments");
    s2_status s = s2_dit_block_set_runtime_shape(b, vid_shape[0], vid_shape[1], vid_shape[2]);
    if (s != S2_OK) return s;
    if (L != vid_shape[0] * vid_shape[1] * vid_shape[2])
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_forward_host: vid rows %d != T*H*W", L);
    s2::DeviceGuard guard(b->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t d = b->dim, vb = static_cast<size_t>(L) * d * 4, tbytes = static_cast<size_t>(std::max(Lt, 1)) * d * 4;
    if (!b->hv.ensure(vb) || !b->ht.ensure(tbytes) || !b->he.ensure(6 * d * 4) || !b->hov.ensure(vb) ||
        !b->hot.ensure(tbytes))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_block_forward_host: staging allocation failed");
    if (cudaMemcpyAsync(b->hv.ptr, vid, vb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        (Lt > 0 && cudaMemcpyAsync(b->ht.ptr, txt, static_cast<size_t>(Lt) * d * 4, cudaMemcpyHostToDevice, st) !=
                       cudaSuccess) ||
        cudaMemcpyAsync(b->he.ptr, emb, 6 * d * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block_forward_host: upload failed");
    // host debug captures: staged in one device buffer, copied out after the forward
    float *const *hosts = reinterpret_cast<float *const *>(&b->debug_host);
    size_t counts[14] = {};
    const bool host_debug = b->debug_host_on;
    if (host_debug) {
        int rows = 0;
        if ((s = s2_dit_block_debug_rows(b, Lt, &rows)) != S2_OK) return s;
        const size_t Lz = static_cast<size_t>(L), Tz = static_cast<size_t>(Lt), Rz = static_cast<size_t>(rows);
        const size_t n[14] = {Lz * 3 * d, Tz * 3 * d, Lz * d, Tz * d, Lz * d, Tz * d, Rz * d, Rz * d, Rz * d, Rz * d,
                              Lz * d, Tz * d, Lz * d, Tz * d};
        size_t total = 0;
        for (int i = 0; i < 14; ++i) {
            counts[i] = hosts[i] ? n[i] : 0;
            total += (counts[i] + 63) / 64 * 64;
        }
        if (!b->debug_stage.ensure(std::max<size_t>(total, 64) * 4))
            return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_block_forward_host: debug staging allocation failed");
        float **dev = reinterpret_cast<float **>(&b->debug);
        float *at = static_cast<float *>(b->debug_stage.ptr);
        for (int i = 0; i < 14; ++i) {
            dev[i] = counts[i] ? at : nullptr;
            at += (counts[i] + 63) / 64 * 64;
        }
        b->debug_on = true;
    }
    s = s2_dit_block_forward(b, stream, static_cast<const float *>(b->hv.ptr), L, static_cast<const float *>(b->ht.ptr), Lt,
                             static_cast<const float *>(b->he.ptr), static_cast<float *>(b->hov.ptr),
                             static_cast<float *>(b->hot.ptr));
    if (host_debug) {
        b->debug_on = false;
        if (s == S2_OK)
            for (int i = 0; i < 14 && s == S2_OK; ++i)
                if (counts[i] && cudaMemcpyAsync(hosts[i], reinterpret_cast<float **>(&b->debug)[i], counts[i] * 4,
                                                 cudaMemcpyDeviceToHost, st) != cudaSuccess)
                    s = s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block_forward_host: debug download failed");
        b->debug = s2_block_debug{};
    }
    if (s != S2_OK) {
        cudaStreamSynchronize(st);  // no copy may still touch the caller's buffers
        return s;
    }
    if (cudaMemcpyAsync(vid_out, b->hov.ptr, vb, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        (Lt > 0 && cudaMemcpyAsync(txt_out, b->hot.ptr, static_cast<size_t>(Lt) * d * 4, cudaMemcpyDeviceToHost, st) !=
                       cudaSuccess) ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block_forward_host: %s", cudaGetErrorString(cudaGetLastError()));
    int code = 0;
    return s2_dit_block_device_error(b, &code);
}

extern "C" int s2_dit_block_last_launches(const s2_dit_block *b) { return b ? b->last_launches : 0; }

extern "C" s2_status s2_dit_block_device_error(s2_dit_block *b, int *code)
{
    if (code) *code = 0;
    if (!b) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_block_device_error: block is NULL");
    int c = 0;
    s2_status s = s2_attention_layer_device_error(b->attn, &c);
    if (s != S2_OK) {
        if (code) *code = c;
        return s;
    }
    if (!b->err.ptr) return S2_OK;
    s2::DeviceGuard guard(b->device);
    int32_t hcode = 0;
    if (cudaStreamSynchronize(b->last_stream) != cudaSuccess ||
        cudaMemcpy(&hcode, b->err.ptr, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block: device failure: %s", cudaGetErrorString(cudaGetLastError()));
    if (code) *code = hcode;
    if (hcode != 0) return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_block: device wait timed out (code %d)", hcode);
    return S2_OK;
}
