// s2_dit: the SeedVR2 DiT (input head, the block stack, output head) and one
// Euler sampling step on sm_100a -- the device-resident counterpart of
// SeedVR2DiT::forward (src/model/dit.cpp:277-383) with the engine's one-step
// sampling (make_dit_input, src/core/engine.cpp:125-149;
// EulerSampler::endpoint, src/model/sampler.cpp:276-286).
//
//   input head (SeedVR2DiTInput, seedvr2_dit_input.cpp:311-405):
//     patchify 1x2x2 of the vc-channel latent in (dy, dx, c) order -> fp16 rows
//     (K padded to a multiple of 64), video projection and text projection on
//     the tensor cores (+ bias, fp32 out); timestep sinusoid -> Linear + SiLU
//     -> Linear + SiLU -> Linear = the block modulation vector emb [6 dim]
//     (fp32 matrix-vector kernels: one vector, weight-bandwidth bound).
//   blocks: s2_dit_block in order, sharing one set of activation workspaces.
//   output head (SeedVR2DiTOutput, seedvr2_dit_output.cpp:349-431):
//     RMSNorm * weight, adaLN with emb slots 0/1, projection dim -> 4 oc
//     (+ bias), unpatchify -- fused with the Euler endpoint x - (t/1000) pred
//     for a sampling step.
// Every forward is stream-ordered with no host synchronisation. An Euler step
// is about 520 launches; from the second call with the same shapes, buffers
// and timestep it is replayed as one CUDA graph (captured on an internal
// stream, launched on the caller's), so host launch latency stays off the
// GPU's critical path.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "s2_buffers.h"
#include "s2_comm.h"
#include "s2_gemm.h"
#include "s2_internal.h"
#include "s2_ops.h"

namespace {

int round64(int x) { return (x + 63) / 64 * 64; }

// patches[p][col] = latent[c][t][2y + dy][2x + dx], col = (dy * 2 + dx) * vc + c;
// zero for the padding columns col >= 4 vc (seedvr2_dit_input.cpp:335-353).
__global__ void patchify_kernel(const float *__restrict__ latent, int vc, int T, int H, int W, int kp,
                                __half *__restrict__ patches)
{
    const int Hp = H / 2, Wp = W / 2;
    const long long total = 1LL * T * Hp * Wp * kp;
    const long long plane = 1LL * T * H * W;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
        const int col = static_cast<int>(i % kp);
        const long long p = i / kp;
        float v = 0.f;
        if (col < 4 * vc) {
            const int x = static_cast<int>(p % Wp), y = static_cast<int>((p / Wp) % Hp), t = static_cast<int>(p / (1LL * Wp * Hp));
            const int blk = col / vc, c = col - blk * vc, dy = blk >> 1, dx = blk & 1;
            v = latent[c * plane + (1LL * t * H + 2 * y + dy) * W + 2 * x + dx];
        }
        patches[i] = __float2half_rn(v);
    }
}

// latent33 = noise (oc) || condition (oc) || ones (engine.cpp:125-149)
__global__ void make_dit_input_kernel(const float *__restrict__ noise, const float *__restrict__ cond, int oc,
                                      long long plane, float *__restrict__ latent)
{
    const long long total = (2LL * oc + 1) * plane;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
        const long long c = i / plane, o = i - c * plane;
        latent[i] = c < oc ? noise[i] : (c < 2 * oc ? cond[(c - oc) * plane + o] : 1.f);
    }
}

// text rows fp32 [rows][cols] -> fp16 [rows][ld] (zero padding columns)
__global__ void pad_to_f16_kernel(const float *__restrict__ x, int rows, int cols, int ld, __half *__restrict__ y)
{
    const long long total = 1LL * rows * ld;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
        const int c = static_cast<int>(i % ld);
        const long long r = i / ld;
        y[i] = __float2half_rn(c < cols ? x[r * cols + c] : 0.f);
    }
}

// s[i] = sin(t f_i), s[i + half] = cos(t f_i), f_i = exp(-log(10000) i / half)
// (seedvr2_dit_input.cpp:362-372, single-precision like the reference)
__global__ void sinusoid_kernel(float t, int half, float *__restrict__ s)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= half) return;
    const float freq = expf(__fdiv_rn(__fmul_rn(-logf(10000.f), static_cast<float>(i)), static_cast<float>(half)));
    const float v = __fmul_rn(t, freq);
    s[i] = sinf(v);
    s[i + half] = cosf(v);
}

// y[o] = act(b[o] + W[o] . x), one warp per output row, fp32 weights; x staged
// in shared memory. act = SiLU (x / (1 + exp(-x))) when silu != 0.
__global__ void __launch_bounds__(256) gemv_kernel(const float *__restrict__ Wm, const float *__restrict__ b,
                                                   const float *__restrict__ x, int K, int N, int silu,
                                                   float *__restrict__ y)
{
    extern __shared__ float xs[];
    for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const int o = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (o >= N) return;
    const float *w = Wm + static_cast<size_t>(o) * K;
    float acc = 0.f;
    for (int i = lane; i < K; i += 32) acc = fmaf(__ldg(w + i), xs[i], acc);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if (lane == 0) {
        float v = __fadd_rn(acc, b[o]);
        if (silu) v = __fdiv_rn(v, __fadd_rn(1.f, expf(-v)));
        y[o] = v;
    }
}

// out[c][t][Y][X] = proj[p][(dy*2 + dx) * oc + c] with p the patch of (t, Y/2, X/2)
// (seedvr2_dit_output.cpp:402-418); with `noise`, the Euler endpoint
// out = noise - (t/1000) * pred (sampler.cpp:276-286).
__global__ void unpatchify_kernel(const float *__restrict__ proj, int oc, int T, int Hp, int Wp,
                                  const float *__restrict__ noise, float bt, float *__restrict__ out)
{
    const int H = 2 * Hp, W = 2 * Wp;
    const long long plane = 1LL * T * H * W, total = plane * oc;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
        const int c = static_cast<int>(i / plane);
        const long long o = i - c * plane;
        const int X = static_cast<int>(o % W), Y = static_cast<int>((o / W) % H), t = static_cast<int>(o / (1LL * W * H));
        const long long p = (1LL * t * Hp + Y / 2) * Wp + X / 2;
        const float pred = proj[p * 4 * oc + ((Y & 1) * 2 + (X & 1)) * oc + c];
        out[i] = noise ? __fsub_rn(noise[i], __fmul_rn(bt, pred)) : pred;
    }
}

// ---- sharded step (one rank per GPU) ----

// patches for a rank's local rows: local row i is patched-grid token tok[i]
__global__ void patchify_local_kernel(const float *__restrict__ latent, int vc, int T, int H, int W, int kp,
                                      const int32_t *__restrict__ tok, int n, __half *__restrict__ patches)
{
    const int Hp = H / 2, Wp = W / 2;
    const long long total = 1LL * n * kp, plane = 1LL * T * H * W;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
        const int col = static_cast<int>(i % kp);
        const int p = tok[i / kp];
        float v = 0.f;
        if (col < 4 * vc) {
            const int x = p % Wp, y = (p / Wp) % Hp, t = p / (Wp * Hp);
            const int blk = col / vc, c = col - blk * vc, dy = blk >> 1, dx = blk & 1;
            v = latent[c * plane + (1LL * t * H + 2 * y + dy) * W + 2 * x + dx];
        }
        patches[i] = __float2half_rn(v);
    }
}

// the rank's output pixels (zero elsewhere) from its local rows' projections
__global__ void unpatchify_local_kernel(const float *__restrict__ proj, int oc, int T, int Hp, int Wp,
                                        const int32_t *__restrict__ tok, int n, const float *__restrict__ noise,
                                        float bt, float *__restrict__ out)
{
    const int H = 2 * Hp, W = 2 * Wp;
    const long long plane = 1LL * T * H * W, total = 1LL * n * 4 * oc;
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += 256LL * gridDim.x) {
        const int col = static_cast<int>(i % (4 * oc));
        const long long row = i / (4 * oc);
        const int p = tok[row];
        const int x = p % Wp, y = (p / Wp) % Hp, t = p / (Wp * Hp);
        const int blk = col / oc, c = col - blk * oc, dy = blk >> 1, dx = blk & 1;
        const long long o = c * plane + (1LL * t * H + 2 * y + dy) * W + 2 * x + dx;
        const float pred = proj[i];
        out[o] = noise ? __fsub_rn(noise[o], __fmul_rn(bt, pred)) : pred;
    }
}

// ---- row exchange over peer memory (sharded step) -------------------------------
// At a plain <-> shifted boundary the last GEMM of the block before it (the MLP
// output projection with its gated residual) stores every output row straight
// into the next block's input buffer on the rank that owns the row's token
// under the next window kind -- its own buffer, or a peer's mapped through CUDA
// IPC (plain stores over NVLink): the exchange has no pass or collective call
// of its own. Ordering, with the same buffer role (vid_nxt) on every rank:
//   * the destination is free: it is each rank's input of the previous block,
//     last read by that block's output projection; the writer's text
//     all-reduce in the current block, before its MLP, completes only once
//     every rank has reached that all-reduce, i.e. finished the previous block;
//   * the rows have landed before the next block reads them: each epilogue
//     thread fences its stores at system scope; after the GEMM every rank
//     announces epoch e (a device counter all ranks advance in step) to every
//     rank, and waits until every rank announced e.
// The wait is bounded; on expiry the DiT's error word gets a code and the
// kernel returns (a peer that died makes the step fail, not hang).
constexpr int kMaxRanks = 8;
enum : int { XF_DONE = 0, XF_EPOCH = kMaxRanks, XF_WORDS = 16 };
enum : int { E_XFER_DONE = 49 };
constexpr unsigned long long kXferTimeoutNs = 10000000000ull;  // 10 s

struct XferFlags {
    int32_t *flags[kMaxRanks];  // every rank's flag words (this rank's own among them)
};

__device__ __forceinline__ unsigned long long xf_now()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_release_sys(int32_t *p, int v)
{
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int32_t *p)
{
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// this rank's rows of the exchange are stored: announce the next epoch to every rank
__global__ void xfer_done_kernel(XferFlags ff, int32_t *flags, int me, int n)
{
    if (threadIdx.x != 0) return;
    const int e = flags[XF_EPOCH] + 1;
    flags[XF_EPOCH] = e;
    __threadfence_system();
    for (int p = 0; p < n; ++p) st_release_sys(ff.flags[p] + XF_DONE + me, e);
}

// every rank announced this epoch (bounded)
__global__ void xfer_wait_kernel(const int32_t *flags, int n, int32_t *err)
{
    if (threadIdx.x != 0) return;
    const int e = flags[XF_EPOCH];
    const unsigned long long t0 = xf_now();
    for (int p = 0; p < n; ++p)
        while (ld_acquire_sys(flags + XF_DONE + p) < e) {
            if (xf_now() - t0 > kXferTimeoutNs) {
                atomicCAS(err, 0, E_XFER_DONE);
                return;
            }
            __nanosleep(200);
        }
}

unsigned grid_for(long long n) { return static_cast<unsigned>(std::min<long long>((n + 255) / 256, 4096)); }

bool upload(s2::DeviceBuffer &b, const float *src, size_t n)
{
    return b.ensure(n * 4) && cudaMemcpy(b.ptr, src, n * 4, cudaMemcpyHostToDevice) == cudaSuccess;
}

// W [rows][cols] fp32 -> fp16 [rows][ld] (zero padding)
bool upload_f16_pad(s2::DeviceBuffer &b, const float *src, size_t rows, size_t cols, size_t ld)
{
    std::vector<__half> h(rows * ld, __float2half_rn(0.f));
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) h[r * ld + c] = __float2half_rn(src[r * cols + c]);
    return b.ensure(h.size() * 2) && cudaMemcpy(b.ptr, h.data(), h.size() * 2, cudaMemcpyHostToDevice) == cudaSuccess;
}

}  // namespace

struct s2_dit {
    int device = 0;
    int n_blocks = 32, dim = 2560, heads = 20, head_dim = 128, hidden = 6912;
    float eps = 1e-5f;
    int vc = 33, tc = 5120, sd = 256, oc = 16;
    int wt = 0, wh = 0, ww = 0;
    int kp = 192, tcp = 5120;
    bool input_loaded = false, output_loaded = false;
    std::vector<s2_dit_block *> blocks;
    // input head
    s2::DeviceBuffer w_vid, b_vid, w_txt, b_txt, w_t1, b_t1, w_t2, b_t2, w_t3, b_t3;
    // output head
    s2::DeviceBuffer o_norm, o_mod6, w_out, b_out;  // o_mod6 [6][dim] = shift, scale, zeros
    // workspaces
    s2::DeviceBuffer latent, patches, txt16, vid_a, vid_b, txt_a, txt_b, sinus, th1, th2, emb, omods, o16, proj, err;
    s2::DeviceBuffer h_noise, h_cond, h_text, h_x0;  // host-step staging
    s2::DeviceBuffer pred_pos, pred_neg, cfg_ws;     // sampling loop: predictions, guidance statistics
    int last_launches = 0;
    cudaStream_t last_stream = nullptr;
    std::vector<int> shifted;  // per block (the window kind of its attention)
    // sharded step
    s2_comm *comm = nullptr;
    struct Shard {
        bool valid = false;
        int T = 0, Hp = 0, Wp = 0, Lt = -1;
        int n_local[2] = {0, 0};
        std::vector<int32_t> ids[2];
        s2::DeviceBuffer tok[2];   // local row -> patched-grid token, per window kind
        s2::DeviceBuffer dest[2];  // local row of kind k -> (rank, row) under kind 1 - k (int2)
    } sh;
    // peer mappings of the exchange's destination buffers (vid_a, vid_b) and flag words
    struct Xfer {
        int n = 0, me = 0;
        void *mine[3] = {nullptr, nullptr, nullptr};  // the local allocations the mappings were made for
        void *peer[3][kMaxRanks] = {};                // [vid_a, vid_b, flags][rank]
        s2::DeviceBuffer flags;
        void unshare()
        {
            for (int b = 0; b < 3; ++b) {
                for (int p = 0; p < n; ++p)
                    if (p != me && peer[b][p]) cudaIpcCloseMemHandle(peer[b][p]);
                for (int p = 0; p < kMaxRanks; ++p) peer[b][p] = nullptr;
                mine[b] = nullptr;
            }
        }
    } xf;
    // Euler-step graph: the call it was captured for and its launch count
    struct StepKey {
        int T = 0, H = 0, W = 0, Lt = 0;
        const void *noise = nullptr, *cond = nullptr, *text = nullptr, *x0 = nullptr;
        float t = 0.f;
        bool operator==(const StepKey &o) const
        {
            return T == o.T && H == o.H && W == o.W && Lt == o.Lt && noise == o.noise && cond == o.cond &&
                   text == o.text && x0 == o.x0 && t == o.t;
        }
    };
    bool use_graph = true;
    StepKey key;
    bool key_valid = false;
    cudaStream_t cap_stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    int graph_launches = 0;
    void drop_graph()
    {
        if (exec) cudaGraphExecDestroy(exec);
        exec = nullptr;
    }
    // A forward outside the Euler-step graph may grow (reallocate) the buffers
    // the graph's kernels point at, or remake the peer mappings of a sharded
    // step: the next Euler step then runs eagerly and captures again.
    void forget_step_graph()
    {
        drop_graph();
        key_valid = false;
    }
};

extern "C" s2_status s2_dit_create(int device, int n_blocks, int dim, int heads, int head_dim, int mlp_hidden,
                                   float eps, int video_channels, int text_channels, int sinusoidal_dim,
                                   int out_channels, int wt, int wh, int ww, s2_dit **out)
{
    s2::clear_error();
    if (!out) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_create: out is NULL");
    *out = nullptr;
    if (n_blocks <= 0 || dim != heads * head_dim || video_channels <= 0 || text_channels <= 0 || sinusoidal_dim <= 0 ||
        sinusoidal_dim % 2 != 0 || out_channels <= 0 || (4 * out_channels) % 32 != 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_create: invalid configuration");
    const s2_status st = s2_device_check(device);
    if (st != S2_OK) return st;
    auto *d = new s2_dit();
    d->device = device;
    d->n_blocks = n_blocks;
    d->dim = dim;
    d->heads = heads;
    d->head_dim = head_dim;
    d->hidden = mlp_hidden;
    d->eps = eps;
    d->vc = video_channels;
    d->tc = text_channels;
    d->sd = sinusoidal_dim;
    d->oc = out_channels;
    d->wt = wt;
    d->wh = wh;
    d->ww = ww;
    d->kp = round64(4 * video_channels);
    d->tcp = round64(text_channels);
    d->blocks.assign(n_blocks, nullptr);
    d->shifted.assign(n_blocks, 0);
    *out = d;
    return S2_OK;
}

extern "C" s2_status s2_dit_destroy(s2_dit *d)
{
    if (!d) return S2_OK;
    for (s2_dit_block *b : d->blocks) s2_dit_block_destroy(b);
    s2::DeviceGuard guard(d->device);
    d->drop_graph();
    d->xf.unshare();
    if (d->cap_stream) cudaStreamDestroy(d->cap_stream);
    for (s2::DeviceBuffer *b : {&d->w_vid, &d->b_vid, &d->w_txt, &d->b_txt, &d->w_t1, &d->b_t1, &d->w_t2, &d->b_t2,
                                &d->w_t3, &d->b_t3, &d->o_norm, &d->o_mod6, &d->w_out, &d->b_out, &d->omods,
                                &d->latent, &d->patches, &d->txt16, &d->vid_a, &d->vid_b, &d->txt_a, &d->txt_b,
                                &d->sinus, &d->th1, &d->th2, &d->emb, &d->o16, &d->proj, &d->err, &d->h_noise,
                                &d->sh.tok[0], &d->sh.tok[1], &d->sh.dest[0], &d->sh.dest[1], &d->xf.flags,
                                &d->h_cond, &d->h_text, &d->h_x0})
        b->release();
    delete d;
    return S2_OK;
}

extern "C" size_t s2_dit_input_weight_count(const s2_dit *d)
{
    if (!d) return 0;
    const size_t D = d->dim, ed = 6 * D;
    return D * 4 * d->vc + D + D * d->tc + D + D * d->sd + D + D * D + D + ed * D + ed;
}

extern "C" size_t s2_dit_output_weight_count(const s2_dit *d)
{
    return d ? 3 * static_cast<size_t>(d->dim) + 4 * static_cast<size_t>(d->oc) * (d->dim + 1) : 0;
}

extern "C" s2_status s2_dit_load_input(s2_dit *d, const float *w, size_t n)
{
    s2::clear_error();
    if (!d || !w) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_load_input: null argument");
    if (n != s2_dit_input_weight_count(d))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_load_input: %zu floats, the layer reads %zu", n,
                             s2_dit_input_weight_count(d));
    s2::DeviceGuard guard(d->device);
    const size_t D = d->dim, ed = 6 * D;
    // load_model order (seedvr2_dit_input.cpp:217-224): each InnerProduct is W [out][in] then b [out]
    bool ok = upload_f16_pad(d->w_vid, w, D, 4 * d->vc, d->kp) && upload(d->b_vid, w + D * 4 * d->vc, D);
    w += D * 4 * d->vc + D;
    ok = ok && upload_f16_pad(d->w_txt, w, D, d->tc, d->tcp) && upload(d->b_txt, w + D * d->tc, D);
    w += D * d->tc + D;
    ok = ok && upload(d->w_t1, w, D * d->sd) && upload(d->b_t1, w + D * d->sd, D);
    w += D * d->sd + D;
    ok = ok && upload(d->w_t2, w, D * D) && upload(d->b_t2, w + D * D, D);
    w += D * D + D;
    ok = ok && upload(d->w_t3, w, ed * D) && upload(d->b_t3, w + ed * D, ed);
    if (!ok) return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_load_input: weight upload failed");
    d->input_loaded = true;
    return S2_OK;
}

extern "C" s2_status s2_dit_load_output(s2_dit *d, const float *w, size_t n)
{
    s2::clear_error();
    if (!d || !w) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_load_output: null argument");
    if (n != s2_dit_output_weight_count(d))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_load_output: %zu floats, the layer reads %zu", n,
                             s2_dit_output_weight_count(d));
    s2::DeviceGuard guard(d->device);
    const size_t D = d->dim, N = 4 * d->oc;
    // load_model order (seedvr2_dit_output.cpp:264-270): norm weight, shift, scale, projection W then b
    std::vector<float> mod6(6 * D, 0.f);
    std::copy(w + D, w + 3 * D, mod6.begin());  // shift, scale in the adaLN slots 0 and 1
    const bool ok = upload(d->o_norm, w, D) && upload(d->o_mod6, mod6.data(), 6 * D) &&
                    upload_f16_pad(d->w_out, w + 3 * D, N, D, D) && upload(d->b_out, w + 3 * D + N * D, N);
    if (!ok) return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_load_output: weight upload failed");
    d->output_loaded = true;
    return S2_OK;
}

extern "C" s2_status s2_dit_load_block(s2_dit *d, int index, int shared, int last, int shifted, const float *w, size_t n)
{
    s2::clear_error();
    if (!d || !w || index < 0 || index >= d->n_blocks)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_load_block: bad block index %d", index);
    s2_dit_block *b = nullptr;
    s2_status st = s2_dit_block_create(d->device, index, shared, last, shifted, d->dim, d->heads, d->head_dim,
                                       d->hidden, d->eps, d->wt, d->wh, d->ww, &b);
    if (st != S2_OK) return st;
    if ((st = s2_dit_block_load(b, w, n)) != S2_OK) {
        s2_dit_block_destroy(b);
        return st;
    }
    s2_dit_block_destroy(d->blocks[index]);
    d->blocks[index] = b;
    d->shifted[index] = shifted != 0;
    d->drop_graph();
    d->key_valid = false;
    d->sh.valid = false;
    // all blocks run one after another on one stream: one set of activation workspaces
    for (s2_dit_block *o : d->blocks)
        if (o && o != b) {
            s2::share_block_scratch(b, o);
            break;
        }
    return S2_OK;
}

// Window ownership of both window kinds (s2_shard_windows_joint), every rank's
// local row order, and the row-exchange maps between them (s2::shard_exchange_maps,
// the host function the CPU-rank tests check); sets every block's window subset.
static s2_status build_shard(s2_dit *d, int T, int Hp, int Wp, int Lt, cudaStream_t st, bool *rebuilt)
{
    auto &sh = d->sh;
    *rebuilt = false;
    if (sh.valid && sh.T == T && sh.Hp == Hp && sh.Wp == Wp && sh.Lt == Lt) return S2_OK;
    sh.valid = false;
    const int N = s2_comm_size(d->comm), me = s2_comm_rank(d->comm);
    {
        // every rank derives every rank's maps from the grid, so all must run the same one:
        // a rank with other shapes would store rows where no peer expects them
        const int32_t mine[7] = {T, Hp, Wp, Lt, d->wt, d->wh, d->ww};
        std::vector<int32_t> all(7 * static_cast<size_t>(N));
        const s2_status g = s2::comm_allgather_host(d->comm, mine, sizeof(mine), all.data(), st);
        if (g != S2_OK) return g;
        for (int r = 0; r < N; ++r)
            if (!std::equal(mine, mine + 7, all.begin() + 7 * r))
                return s2::set_error(S2_INVALID_ARGUMENT,
                                     "sharded step: rank %d runs a %dx%dx%d token grid with %d text tokens and windows "
                                     "%dx%dx%d, rank %d a %dx%dx%d grid with %d and %dx%dx%d (all ranks must run the "
                                     "same step)",
                                     r, all[7 * r], all[7 * r + 1], all[7 * r + 2], all[7 * r + 3], all[7 * r + 4],
                                     all[7 * r + 5], all[7 * r + 6], me, T, Hp, Wp, Lt, d->wt, d->wh, d->ww);
    }
    s2::ShardMaps m;
    s2_status s = s2::shard_exchange_maps(T, Hp, Wp, d->wt, d->wh, d->ww, Lt, N, me, m);
    if (s != S2_OK) return s;
    for (int k = 0; k < 2; ++k) {
        if (m.tok[k].empty())
            return s2::set_error(S2_UNSUPPORTED,
                                 "sharded step: rank %d owns no %s window of the %dx%dx%d grid (too few windows for %d "
                                 "ranks; use fewer ranks or smaller windows)",
                                 me, k ? "shifted" : "plain", T, Hp, Wp, N);
        sh.ids[k] = m.ids[k];
        sh.n_local[k] = static_cast<int>(m.tok[k].size());
        if (!sh.tok[k].ensure(std::max<size_t>(m.tok[k].size(), 1) * 4) ||
            cudaMemcpy(sh.tok[k].ptr, m.tok[k].data(), m.tok[k].size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return s2::set_error(S2_OUT_OF_MEMORY, "shard: map upload failed");
    }
    const long long rows = 1LL * T * Hp * Wp;  // every rank's hidden-state buffers hold this many rows
    for (int k = 0; k < 2; ++k) {
        std::vector<int2> dest(m.tok[k].size());
        for (size_t i = 0; i < dest.size(); ++i) {
            // the MLP output GEMM stores row i at (rank, row) in peer memory: keep every store
            // inside the destination's buffer whatever the maps say
            if (m.dest_rank[k][i] < 0 || m.dest_rank[k][i] >= N || m.dest_row[k][i] < 0 || m.dest_row[k][i] >= rows)
                return s2::set_error(S2_INFERENCE_FAILED, "shard: row %zu has destination (%d, %d) outside %d ranks x %lld rows",
                                     i, m.dest_rank[k][i], m.dest_row[k][i], N, rows);
            dest[i] = make_int2(m.dest_rank[k][i], m.dest_row[k][i]);
        }
        if (!sh.dest[k].ensure(std::max<size_t>(dest.size(), 1) * sizeof(int2)) ||
            cudaMemcpy(sh.dest[k].ptr, dest.data(), dest.size() * sizeof(int2), cudaMemcpyHostToDevice) != cudaSuccess)
            return s2::set_error(S2_OUT_OF_MEMORY, "shard: map upload failed");
    }
    for (int i = 0; i < d->n_blocks; ++i) {
        const auto &ids = sh.ids[d->shifted[i]];
        s2_status s = s2_dit_block_set_window_subset(d->blocks[i], ids.data(), static_cast<int>(ids.size()));
        if (s == S2_OK) s = s2_dit_block_set_local_rows(d->blocks[i], 1);
        if (s != S2_OK) return s;
    }
    sh.T = T, sh.Hp = Hp, sh.Wp = Wp, sh.Lt = Lt;
    sh.valid = true;
    *rebuilt = true;
    return S2_OK;
}

// Peer mappings of the exchange's destinations (vid_a, vid_b) and flag words,
// made again whenever the shard maps were rebuilt (`rebuilt`: a new grid, which
// every rank meets in the same call, checked by build_shard), so every rank
// makes the same collective calls. The allocations only grow with the grid, so
// they cannot move without a rebuild; if they did, the call fails rather than
// share on one rank alone. Host-synchronising; not during stream capture.
static s2_status xfer_setup(s2_dit *d, cudaStream_t st, bool rebuilt)
{
    auto &x = d->xf;
    const int n = s2_comm_size(d->comm), me = s2_comm_rank(d->comm);
    if (n > kMaxRanks)
        return s2::set_error(S2_UNSUPPORTED, "sharded step: at most %d ranks (got %d)", kMaxRanks, n);
    if (!x.flags.ptr) {
        if (!x.flags.ensure(XF_WORDS * sizeof(int32_t)))
            return s2::set_error(S2_OUT_OF_MEMORY, "sharded step: flag words");
        if (cudaMemset(x.flags.ptr, 0, XF_WORDS * sizeof(int32_t)) != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "sharded step: flag words memset failed");
    }
    void *cur[3] = {d->vid_a.ptr, d->vid_b.ptr, x.flags.ptr};
    const bool same = x.n == n && x.me == me && cur[0] == x.mine[0] && cur[1] == x.mine[1] && cur[2] == x.mine[2];
    if (!rebuilt) {
        if (same) return S2_OK;
        d->sh.valid = false;  // the next call rebuilds the maps and shares again
        return s2::set_error(S2_INFERENCE_FAILED,
                             "sharded step: exchange buffers are not mapped for the current grid (an earlier set-up "
                             "failed or they moved without a new grid)");
    }
    x.unshare();
    x.n = n;
    x.me = me;
    for (int b = 0; b < 3; ++b) {
        const s2_status s = s2::comm_share(d->comm, cur[b], x.peer[b], st);
        if (s != S2_OK) {
            x.unshare();
            d->sh.valid = false;
            return s;
        }
        x.mine[b] = cur[b];
    }
    return S2_OK;
}

static s2_status text_allreduce(void *ctx, float *buf, size_t n, cudaStream_t st)
{
    return s2::comm_allreduce_f32(static_cast<s2_comm *>(ctx), buf, n, st);
}

// The DiT forward; with `noise` the output is the Euler endpoint instead of the prediction.
static s2_status dit_forward_into(s2_dit *d, void *stream, const float *latent, int T, int H, int W,
                                         const float *text, int Lt, float timestep, const float *noise, float *out)
{
    s2::clear_error();
    if (!d) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_forward: model is NULL");
    if (!d->input_loaded || !d->output_loaded)
        return s2::set_error(S2_NOT_LOADED, "s2_dit_forward: input/output heads not loaded");
    for (int i = 0; i < d->n_blocks; ++i)
        if (!d->blocks[i]) return s2::set_error(S2_NOT_LOADED, "s2_dit_forward: block %d not loaded", i);
    if (!latent || !out || T <= 0 || H <= 0 || W <= 0 || H % 2 != 0 || W % 2 != 0 || Lt <= 0 || !text)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_forward: latent needs even H and W, and text tokens");
    s2::DeviceGuard guard(d->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int Hp = H / 2, Wp = W / 2, rows = T * Hp * Wp, D = d->dim, N = 4 * d->oc;
    const size_t Rz = static_cast<size_t>(rows), Tz = static_cast<size_t>(Lt);
    const bool fresh = d->err.ptr == nullptr;
    if (!d->patches.ensure(Rz * d->kp * 2) || !d->txt16.ensure(Tz * d->tcp * 2) || !d->vid_a.ensure(Rz * D * 4) ||
        !d->vid_b.ensure(Rz * D * 4) || !d->txt_a.ensure(Tz * D * 4) || !d->txt_b.ensure(Tz * D * 4) ||
        !d->sinus.ensure(d->sd * 4) || !d->th1.ensure(D * 4) || !d->th2.ensure(D * 4) || !d->emb.ensure(6 * D * 4) ||
        !d->o16.ensure(Rz * D * 2) || !d->proj.ensure(Rz * N * 4) || !d->err.ensure(4) ||
        !d->omods.ensure(static_cast<size_t>(8) * D * 4))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_forward: workspace allocation failed");
    if (fresh && cudaMemsetAsync(d->err.ptr, 0, 4, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_forward: memset failed");
    int32_t *err = static_cast<int32_t *>(d->err.ptr);
    d->last_stream = st;
    int launches = 0;
    s2_status s;
    auto check = [&](const char *what) {
        const cudaError_t e = cudaGetLastError();
        ++launches;
        return e == cudaSuccess ? S2_OK : s2::set_error(S2_INFERENCE_FAILED, "s2_dit_forward: %s: %s", what,
                                                         cudaGetErrorString(e));
    };
#define S2_TRY(expr)                      \
    do {                                  \
        if ((s = (expr)) != S2_OK) {      \
            d->last_launches = launches;  \
            return s;                     \
        }                                 \
    } while (0)

    // sharded: this rank's video rows of each window kind (rows0: the first block's kind)
    const bool sharded = d->comm && s2_comm_size(d->comm) > 1;
    int rows0 = rows;
    if (sharded) {
        bool rebuilt = false;
        S2_TRY(build_shard(d, T, Hp, Wp, Lt, st, &rebuilt));
        S2_TRY(xfer_setup(d, st, rebuilt));
        rows0 = d->sh.n_local[d->shifted[0]];
    } else if (d->sh.valid) {
        for (s2_dit_block *b : d->blocks) {  // back to whole-clip blocks
            S2_TRY(s2_dit_block_set_window_subset(b, nullptr, 0));
            S2_TRY(s2_dit_block_set_local_rows(b, 0));
        }
        d->sh.valid = false;
    }
    s2::TextReduce reduce;
    reduce.fn = text_allreduce;
    reduce.ctx = d->comm;

    // ---- input head ----
    if (sharded)
        patchify_local_kernel<<<grid_for(1LL * rows0 * d->kp), 256, 0, st>>>(
            latent, d->vc, T, H, W, d->kp, static_cast<const int32_t *>(d->sh.tok[d->shifted[0]].ptr), rows0,
            static_cast<__half *>(d->patches.ptr));
    else
        patchify_kernel<<<grid_for(Rz * d->kp), 256, 0, st>>>(latent, d->vc, T, H, W, d->kp,
                                                              static_cast<__half *>(d->patches.ptr));
    S2_TRY(check("patchify"));
    pad_to_f16_kernel<<<grid_for(Tz * d->tcp), 256, 0, st>>>(text, Lt, d->tc, d->tcp, static_cast<__half *>(d->txt16.ptr));
    S2_TRY(check("text convert"));
    s2::GemmArgs g;
    g.epilogue = s2::GEMM_EPI_GATED_RESID_F32;  // no modulation, no residual: acc + bias
    g.N = D;
    g.err = err;
    g.M = rows0;
    g.K = d->kp;
    g.bias = static_cast<const float *>(d->b_vid.ptr);
    g.y = static_cast<float *>(d->vid_a.ptr);
    S2_TRY(s2::gemm_f16(st, d->patches.ptr, d->w_vid.ptr, g));
    ++launches;
    g.M = Lt;
    g.K = d->tcp;
    g.bias = static_cast<const float *>(d->b_txt.ptr);
    g.y = static_cast<float *>(d->txt_a.ptr);
    S2_TRY(s2::gemm_f16(st, d->txt16.ptr, d->w_txt.ptr, g));
    ++launches;
    const int half = d->sd / 2;
    sinusoid_kernel<<<(half + 127) / 128, 128, 0, st>>>(timestep, half, static_cast<float *>(d->sinus.ptr));
    S2_TRY(check("sinusoid"));
    auto gemv = [&](const s2::DeviceBuffer &Wm, const s2::DeviceBuffer &bv, const s2::DeviceBuffer &x, int K, int Nn,
                    int silu, s2::DeviceBuffer &y) {
        gemv_kernel<<<(Nn + 7) / 8, 256, K * 4, st>>>(static_cast<const float *>(Wm.ptr),
                                                      static_cast<const float *>(bv.ptr),
                                                      static_cast<const float *>(x.ptr), K, Nn, silu,
                                                      static_cast<float *>(y.ptr));
        return check("time embedding");
    };
    S2_TRY(gemv(d->w_t1, d->b_t1, d->sinus, d->sd, D, 1, d->th1));
    S2_TRY(gemv(d->w_t2, d->b_t2, d->th1, D, D, 1, d->th2));
    S2_TRY(gemv(d->w_t3, d->b_t3, d->th2, D, 6 * D, 0, d->emb));

    // ---- blocks ----
    float *vid_cur = static_cast<float *>(d->vid_a.ptr), *vid_nxt = static_cast<float *>(d->vid_b.ptr);
    float *txt_cur = static_cast<float *>(d->txt_a.ptr), *txt_nxt = static_cast<float *>(d->txt_b.ptr);
    const float *emb = static_cast<const float *>(d->emb.ptr);
    int kind = d->shifted[0], n_rows = rows0;
    for (int i = 0; i < d->n_blocks; ++i) {
        // a block followed by the other window kind writes its video rows straight into the
        // next block's input (vid_nxt, on this rank and the peers) in the next kind's ownership
        const bool exchange = sharded && i + 1 < d->n_blocks && d->shifted[i + 1] != kind;
        s2::RowScatter rs;
        if (exchange) {
            const auto &x = d->xf;
            const int bi = vid_nxt == static_cast<float *>(d->vid_a.ptr) ? 0 : 1;
            rs.dest = static_cast<const int2 *>(d->sh.dest[kind].ptr);
            for (int p = 0; p < x.n; ++p) rs.base[p] = static_cast<float *>(x.peer[bi][p]);
        }
        S2_TRY(s2_dit_block_set_runtime_shape(d->blocks[i], T, Hp, Wp));
        S2_TRY(s2::dit_block_forward_ex(d->blocks[i], stream, vid_cur, n_rows, txt_cur, Lt, emb, vid_nxt, txt_nxt,
                                        sharded ? &reduce : nullptr, exchange ? &rs : nullptr));
        launches += s2_dit_block_last_launches(d->blocks[i]);
        if (exchange) {
            const auto &x = d->xf;
            XferFlags ff;
            for (int p = 0; p < kMaxRanks; ++p) ff.flags[p] = static_cast<int32_t *>(p < x.n ? x.peer[2][p] : nullptr);
            int32_t *flags = static_cast<int32_t *>(x.flags.ptr);
            xfer_done_kernel<<<1, 32, 0, st>>>(ff, flags, x.me, x.n);
            S2_TRY(check("exchange announce"));
            xfer_wait_kernel<<<1, 32, 0, st>>>(flags, x.n, err);
            S2_TRY(check("exchange wait"));
            kind = d->shifted[i + 1];
            n_rows = d->sh.n_local[kind];
        }
        std::swap(vid_cur, vid_nxt);
        std::swap(txt_cur, txt_nxt);
    }

    // ---- output head ----
    float *om = static_cast<float *>(d->omods.ptr);
    S2_TRY(s2::modulation_vectors(st, emb, static_cast<const float *>(d->o_mod6.ptr), D, om));
    ++launches;
    S2_TRY(s2::rms_ada(st, vid_cur, n_rows, D, d->eps, static_cast<const float *>(d->o_norm.ptr), om, om + D,
                       om + 2 * D, d->o16.ptr));
    ++launches;
    s2::GemmArgs o;
    o.epilogue = s2::GEMM_EPI_GATED_RESID_F32;
    o.M = n_rows;
    o.N = N;
    o.K = D;
    o.bias = static_cast<const float *>(d->b_out.ptr);
    o.y = static_cast<float *>(d->proj.ptr);
    o.err = err;
    S2_TRY(s2::gemm_f16(st, d->o16.ptr, d->w_out.ptr, o));
    ++launches;
    const float bt = timestep / 1000.0f;
    if (sharded) {
        // every rank writes its own pixels of a zeroed output; the sum over ranks is the full output
        const size_t plane_bytes = static_cast<size_t>(T) * H * W * d->oc * 4;
        if (cudaMemsetAsync(out, 0, plane_bytes, st) != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_forward: output memset failed");
        unpatchify_local_kernel<<<grid_for(1LL * n_rows * N), 256, 0, st>>>(
            static_cast<const float *>(d->proj.ptr), d->oc, T, Hp, Wp,
            static_cast<const int32_t *>(d->sh.tok[kind].ptr), n_rows, noise, bt, out);
        S2_TRY(check("unpatchify"));
        S2_TRY(s2::comm_allreduce_f32(d->comm, out, plane_bytes / 4, st));
    } else {
        unpatchify_kernel<<<grid_for(1LL * rows * N), 256, 0, st>>>(static_cast<const float *>(d->proj.ptr), d->oc, T,
                                                                     Hp, Wp, noise, bt, out);
        S2_TRY(check("unpatchify"));
    }
#undef S2_TRY
    d->last_launches = launches;
    return S2_OK;
}

extern "C" s2_status s2_dit_forward(s2_dit *d, void *stream, const float *latent, int T, int H, int W,
                                    const float *text, int Lt, float timestep, float *prediction)
{
    if (d) {
        s2::DeviceGuard guard(d->device);
        d->forget_step_graph();
    }
    return dit_forward_into(d, stream, latent, T, H, W, text, Lt, timestep, nullptr, prediction);
}

static s2_status euler_step_eager(s2_dit *d, cudaStream_t st, const float *noise, const float *condition, int T,
                                  int H, int W, const float *text, int Lt, float timestep, float *x0)
{
    const long long plane = 1LL * T * H * W;
    if (!d->latent.ensure(static_cast<size_t>(plane) * d->vc * 4))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_euler_step: workspace allocation failed");
    make_dit_input_kernel<<<grid_for(plane * d->vc), 256, 0, st>>>(noise, condition, d->oc, plane,
                                                                    static_cast<float *>(d->latent.ptr));
    if (cudaGetLastError() != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step: launch failed");
    const s2_status s = dit_forward_into(d, st, static_cast<const float *>(d->latent.ptr), T, H, W, text, Lt,
                                         timestep, noise, x0);
    if (s == S2_OK) ++d->last_launches;
    return s;
}

extern "C" s2_status s2_dit_euler_step(s2_dit *d, void *stream, const float *noise, const float *condition, int T,
                                       int H, int W, const float *text, int Lt, float timestep, float *x0)
{
    s2::clear_error();
    if (!d || !noise || !condition || !x0 || T <= 0 || H <= 0 || W <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_euler_step: invalid arguments");
    if (d->vc != 2 * d->oc + 1)
        return s2::set_error(S2_UNSUPPORTED, "s2_dit_euler_step: video_channels %d != 2 * out_channels + 1", d->vc);
    s2::DeviceGuard guard(d->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    s2_dit::StepKey k;
    k.T = T, k.H = H, k.W = W, k.Lt = Lt, k.noise = noise, k.cond = condition, k.text = text, k.x0 = x0, k.t = timestep;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (!d->use_graph || cs != cudaStreamCaptureStatusNone)
        return euler_step_eager(d, st, noise, condition, T, H, W, text, Lt, timestep, x0);
    if (d->exec && d->key_valid && d->key == k) {
        if (cudaGraphLaunch(d->exec, st) != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step: graph launch: %s",
                                 cudaGetErrorString(cudaGetLastError()));
        d->last_stream = st;
        d->last_launches = d->graph_launches;
        return S2_OK;
    }
    if (!d->key_valid || !(d->key == k)) {
        // first call for these shapes and buffers: run eagerly (plans, workspaces)
        d->drop_graph();
        const s2_status s = euler_step_eager(d, st, noise, condition, T, H, W, text, Lt, timestep, x0);
        d->key = k;
        d->key_valid = s == S2_OK;
        return s;
    }
    // second call: capture the step once, then replay it
    if (!d->cap_stream && cudaStreamCreateWithFlags(&d->cap_stream, cudaStreamNonBlocking) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step: capture stream");
    if (cudaStreamBeginCapture(d->cap_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step: begin capture: %s",
                             cudaGetErrorString(cudaGetLastError()));
    const s2_status s = euler_step_eager(d, d->cap_stream, noise, condition, T, H, W, text, Lt, timestep, x0);
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(d->cap_stream, &g);
    if (s != S2_OK || ce != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return s != S2_OK ? s
                          : s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step: capture failed: %s",
                                          cudaGetErrorString(ce));
    }
    const cudaError_t ie = cudaGraphInstantiate(&d->exec, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
        d->exec = nullptr;
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step: graph instantiate: %s", cudaGetErrorString(ie));
    }
    d->graph_launches = d->last_launches;
    if (cudaGraphLaunch(d->exec, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step: graph launch: %s",
                             cudaGetErrorString(cudaGetLastError()));
    d->last_stream = st;
    return S2_OK;
}

extern "C" s2_status s2_dit_sample(s2_dit *d, void *stream, const float *noise, const float *condition, int T,
                                   int H, int W, const float *positive_text, const float *negative_text, int Lt,
                                   int steps, float cfg_scale, float cfg_rescale, float *out)
{
    return s2_dit_sample_texts(d, stream, noise, condition, T, H, W, positive_text, Lt, negative_text, Lt, steps,
                               cfg_scale, cfg_rescale, out);
}

extern "C" s2_status s2_dit_sample_texts(s2_dit *d, void *stream, const float *noise, const float *condition, int T,
                                         int H, int W, const float *positive_text, int positive_len,
                                         const float *negative_text, int negative_len, int steps, float cfg_scale,
                                         float cfg_rescale, float *out)
{
    s2::clear_error();
    const bool guide = cfg_scale != 1.0f;  // the engine runs the negative branch only then (engine.cpp:319)
    const int Lt = positive_len;
    if (!d || !noise || !condition || !positive_text || !out || T <= 0 || H <= 0 || W <= 0 || positive_len <= 0 ||
        steps <= 0 || (guide && (!negative_text || negative_len <= 0)))
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_sample: invalid arguments");
    if (d->vc != 2 * d->oc + 1)
        return s2::set_error(S2_UNSUPPORTED, "s2_dit_sample: video_channels %d != 2 * out_channels + 1", d->vc);
    s2::DeviceGuard guard(d->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const long long plane = 1LL * T * H * W, n = plane * d->oc;
    const bool rescale = guide && cfg_rescale != 0.0f;
    d->forget_step_graph();
    if (!d->latent.ensure(static_cast<size_t>(plane) * d->vc * 4) || !d->pred_pos.ensure(static_cast<size_t>(n) * 4) ||
        (guide && !d->pred_neg.ensure(static_cast<size_t>(n) * 4)) ||
        (rescale && !d->cfg_ws.ensure(s2::cfg_workspace_bytes())))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_sample: workspace allocation failed");
    std::vector<float> ts(steps);
    s2_sampler_timesteps(steps, ts.data());
    float *pos = static_cast<float *>(d->pred_pos.ptr), *neg = static_cast<float *>(d->pred_neg.ptr);
    float *lat = static_cast<float *>(d->latent.ptr);
    const float *x = noise;
    int launches = 0;
    for (int i = 0; i < steps; ++i) {
        make_dit_input_kernel<<<grid_for(plane * d->vc), 256, 0, st>>>(x, condition, d->oc, plane, lat);
        if (cudaGetLastError() != cudaSuccess) return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_sample: launch failed");
        s2_status s = dit_forward_into(d, st, lat, T, H, W, positive_text, Lt, ts[i], nullptr, pos);
        if (s != S2_OK) return s;
        launches += d->last_launches + 1;
        float *factor = nullptr;
        if (guide) {
            s = dit_forward_into(d, st, lat, T, H, W, negative_text, negative_len, ts[i], nullptr, neg);
            if (s != S2_OK) return s;
            launches += d->last_launches;
            if (rescale) {
                s = s2::cfg_factor(st, pos, neg, n, cfg_scale, cfg_rescale, d->cfg_ws.ptr, &factor);
                if (s != S2_OK) return s;
                launches += 2;
            }
        }
        const bool final_step = i + 1 == steps;
        s = s2::sampler_update(st, x, pos, guide ? neg : nullptr, cfg_scale, factor, n, ts[i],
                               final_step ? 0.f : ts[i + 1], final_step ? 1 : 0, out);
        if (s != S2_OK) return s;
        ++launches;
        x = out;
    }
    d->last_launches = launches;
    d->last_stream = st;
    return S2_OK;
}

extern "C" s2_status s2_dit_set_comm(s2_dit *d, s2_comm *comm)
{
    if (!d) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_set_comm: model is NULL");
    s2::DeviceGuard guard(d->device);
    d->xf.unshare();
    d->comm = comm;
    d->sh.valid = false;
    d->drop_graph();
    d->key_valid = false;
    if (!comm || s2_comm_size(comm) == 1)
        for (s2_dit_block *b : d->blocks)
            if (b) {
                s2_dit_block_set_window_subset(b, nullptr, 0);
                s2_dit_block_set_local_rows(b, 0);
            }
    return S2_OK;
}

extern "C" s2_status s2_dit_set_graph(s2_dit *d, int enable)
{
    if (!d) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_set_graph: model is NULL");
    s2::DeviceGuard guard(d->device);
    d->use_graph = enable != 0;
    d->drop_graph();
    d->key_valid = false;
    return S2_OK;
}

extern "C" s2_status s2_dit_euler_step_host(s2_dit *d, void *stream, const float *noise, const float *condition,
                                            int T, int H, int W, const float *text, int Lt, float timestep, float *x0)
{
    s2::clear_error();
    if (!d || !noise || !condition || !text || !x0 || T <= 0 || H <= 0 || W <= 0 || Lt <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_euler_step_host: invalid arguments");
    s2::DeviceGuard guard(d->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t lat = static_cast<size_t>(T) * H * W * d->oc * 4, txt = static_cast<size_t>(Lt) * d->tc * 4;
    if (!d->h_noise.ensure(lat) || !d->h_cond.ensure(lat) || !d->h_text.ensure(txt) || !d->h_x0.ensure(lat))
        return s2::set_error(S2_OUT_OF_MEMORY, "s2_dit_euler_step_host: staging allocation failed");
    if (cudaMemcpyAsync(d->h_noise.ptr, noise, lat, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(d->h_cond.ptr, condition, lat, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(d->h_text.ptr, text, txt, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step_host: upload failed");
    s2_status s = s2_dit_euler_step(d, stream, static_cast<const float *>(d->h_noise.ptr),
                                    static_cast<const float *>(d->h_cond.ptr), T, H, W,
                                    static_cast<const float *>(d->h_text.ptr), Lt, timestep,
                                    static_cast<float *>(d->h_x0.ptr));
    if (s != S2_OK) return s;
    if (cudaMemcpyAsync(x0, d->h_x0.ptr, lat, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit_euler_step_host: %s", cudaGetErrorString(cudaGetLastError()));
    int code = 0;
    return s2_dit_device_error(d, &code);
}

extern "C" int s2_dit_last_launches(const s2_dit *d) { return d ? d->last_launches : 0; }

extern "C" s2_status s2_dit_device_error(s2_dit *d, int *code)
{
    if (code) *code = 0;
    if (!d) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_device_error: model is NULL");
    {
        s2::DeviceGuard guard(d->device);
        if (cudaStreamSynchronize(d->last_stream) != cudaSuccess)
            return s2::set_error(S2_INFERENCE_FAILED, "s2_dit: device failure: %s", cudaGetErrorString(cudaGetLastError()));
    }
    for (s2_dit_block *b : d->blocks) {
        if (!b) continue;
        const s2_status s = s2_dit_block_device_error(b, code);
        if (s != S2_OK) return s;
    }
    if (!d->err.ptr) return S2_OK;
    s2::DeviceGuard guard(d->device);
    int32_t h = 0;
    if (cudaStreamSynchronize(d->last_stream) != cudaSuccess || cudaMemcpy(&h, d->err.ptr, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return s2::set_error(S2_INFERENCE_FAILED, "s2_dit: device failure: %s", cudaGetErrorString(cudaGetLastError()));
    if (code) *code = h;
    if (h != 0) return s2::set_error(S2_INFERENCE_FAILED, "s2_dit: device wait timed out (code %d)", h);
    return S2_OK;
}
