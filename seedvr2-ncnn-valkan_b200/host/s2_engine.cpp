// seedvr2::SeedVR2Engine over the B200 C ABI (include/seedvr2/engine.h).
//
// The orchestration of the reference's engine (src/core/engine.cpp:205-374):
// option checks (src/core/vulkan_context.cpp:62-69), the model directory
// layout and optional default text embeddings (engine.cpp:180-199, 211-240),
// the random streams in the engine's order, the condition latent and the
// sampling loop -- here on the GPU through s2_make_condition and
// s2_dit_sample_texts, with the DiT resident in HBM (s2_dit_load_dir).
#include "seedvr2/engine.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <filesystem>
#include <fstream>
#include <limits>
#include <random>
#include <utility>

#include "s2_b200.h"

namespace seedvr2
{
namespace
{
bool element_count(std::initializer_list<int> dims, std::size_t &n)
{
    n = 1;
    for (int d : dims) {
        if (d <= 0) return false;
        if (n > std::numeric_limits<std::size_t>::max() / static_cast<std::size_t>(d)) return false;
        n *= static_cast<std::size_t>(d);
    }
    return true;
}

// default_pos_emb.bin / default_neg_emb.bin: int32 tokens, int32 channels,
// fp32 [tokens][channels] (the reference's tools/export_default_embeddings.py).
bool read_embedding(const std::filesystem::path &path, int channels, TextEmbedding &out)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::int32_t head[2] = {0, 0};
    f.read(reinterpret_cast<char *>(head), sizeof head);
    if (!f || head[0] <= 0 || head[1] != channels) return false;
    TextEmbedding e;
    e.tokens = head[0];
    e.channels = head[1];
    e.data.resize(static_cast<std::size_t>(e.tokens) * e.channels);
    f.read(reinterpret_cast<char *>(e.data.data()), static_cast<std::streamsize>(e.data.size() * sizeof(float)));
    if (!f || !e.valid()) return false;
    out = std::move(e);
    return true;
}

// Device buffer owned by the engine (cudaMalloc'd on the engine's device).
struct DevBuf {
    void *p = nullptr;
    std::size_t bytes = 0;
    bool ensure(std::size_t n)
    {
        if (n <= bytes && p) return true;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        if (cudaMalloc(&p, n) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        bytes = n;
        return true;
    }
    void release()
    {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    float *f() const { return static_cast<float *>(p); }
};
}  // namespace

bool Video::valid() const noexcept
{
    std::size_t n = 0;
    return element_count({frames, height, width, channels}, n) && data.size() == n && std::isfinite(fps) && fps > 0.f;
}

bool TextEmbedding::valid() const noexcept
{
    std::size_t n = 0;
    return element_count({tokens, channels}, n) && data.size() == n;
}

bool Latent::valid() const noexcept
{
    std::size_t n = 0;
    return element_count({channels, frames, height, width}, n) && data.size() == n;
}

class SeedVR2Engine::Impl
{
public:
    ~Impl() { release(); }

    int load(const std::string &model_dir, const RuntimeOptions &requested)
    {
        release();
        if (model_dir.empty()) return fail(Status::InvalidArgument, "model_dir is empty");
        const RuntimeOptions &o = requested;
        if (o.sampling_steps <= 0 || o.cfg_scale < 0.f || o.cfg_rescale < 0.f || o.cfg_rescale > 1.f ||
            o.condition_noise_scale < 0.f || o.condition_noise_scale > 1.f || o.vae_scaling_factor <= 0.f)
            return fail(Status::InvalidArgument, "invalid runtime sampling or scaling option");
        if (o.device != DeviceType::Cuda)
            return fail(Status::UnsupportedBackend,
                        o.device == DeviceType::Vulkan ? "this build has no Vulkan backend (use DeviceType::Cuda)"
                                                       : "this build has no CPU backend (use DeviceType::Cuda)");
        if (s2_device_check(o.cuda_device_index) != S2_OK)
            return fail(Status::UnsupportedBackend, std::string("CUDA device: ") + s2_last_error());
        options = o;
        device = o.cuda_device_index;

        const std::filesystem::path root(model_dir);
        std::error_code ec;
        const std::filesystem::path dit_dir =
            std::filesystem::is_directory(root / "dit_full_fp16", ec) ? root / "dit_full_fp16" : root;
        auto file = [&](const std::string &stem, const char *ext) {
            return (dit_dir / (stem + ".ncnn." + ext)).string();
        };
        for (const char *stem : {"seedvr2_dit_input", "seedvr2_dit_output", "seedvr2_dit_block_00"})
            for (const char *ext : {"param", "bin"})
                if (!std::filesystem::is_regular_file(file(stem, ext), ec))
                    return fail(Status::ModelNotFound, "DiT model file is missing: " + file(stem, ext));
        // architecture from the exported files: heads / head_dim / MLP width from
        // block 00, the head dimensions from the input and output layers
        s2_head_params in{}, out{};
        s2_block_params blk{};
        std::size_t n = 0;
        if (s2_ncnn_read_input(file("seedvr2_dit_input", "param").c_str(), file("seedvr2_dit_input", "bin").c_str(),
                               &in, nullptr, 0, &n) != S2_OK ||
            s2_ncnn_read_output(file("seedvr2_dit_output", "param").c_str(), file("seedvr2_dit_output", "bin").c_str(),
                                &out, nullptr, 0, &n) != S2_OK ||
            s2_ncnn_read_block(file("seedvr2_dit_block_00", "param").c_str(),
                               file("seedvr2_dit_block_00", "bin").c_str(), &blk, nullptr, 0, &n) != S2_OK)
            return fail(Status::ModelLoadFailed, std::string("DiT model files: ") + s2_last_error());
        int n_blocks = 0;
        for (;; ++n_blocks) {
            char stem[64];
            std::snprintf(stem, sizeof stem, "seedvr2_dit_block_%02d", n_blocks);
            if (!std::filesystem::is_regular_file(file(stem, "param"), ec) ||
                !std::filesystem::is_regular_file(file(stem, "bin"), ec))
                break;
        }
        s2_dit *d = nullptr;
        s2_status s = s2_dit_create(device, n_blocks, in.dim, blk.heads, blk.head_dim, blk.mlp_hidden, blk.eps,
                                    in.video_channels, in.text_channels, in.sinusoidal_dim, out.out_channels, 0, 0,
                                    0, &d);
        if (s != S2_OK)
            return fail(s == S2_OUT_OF_MEMORY ? Status::OutOfMemory : Status::ModelLoadFailed,
                        std::string("DiT create: ") + s2_last_error());
        dit = d;
        if ((s = s2_dit_load_dir(dit, dit_dir.string().c_str())) != S2_OK)
            return fail(s == S2_OUT_OF_MEMORY ? Status::OutOfMemory : Status::ModelLoadFailed,
                        std::string("DiT load failed: ") + s2_last_error());
        latent_channels = out.out_channels;
        text_channels = in.text_channels;
        if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess)
            return fail(Status::InferenceFailed, "failed to create the engine's CUDA stream");
        read_embedding(root / "default_pos_emb.bin", text_channels, default_positive);
        read_embedding(root / "default_neg_emb.bin", text_channels, default_negative);
        is_loaded = true;
        error.clear();
        return static_cast<int>(Status::Ok);
    }

    int process(const Video &input, const TextEmbedding &positive, const TextEmbedding &negative, Video &output)
    {
        if (!is_loaded) return fail(Status::NotLoaded, "engine is not loaded");
        const TextEmbedding *pos = nullptr, *neg = nullptr;
        if (const int r = pick_texts(positive, negative, pos, neg)) return r;
        if (!input.valid()) return fail(Status::InvalidArgument, "input video is empty or inconsistent");
        (void)output;
        return fail(Status::UnsupportedBackend,
                    "pixel video needs the VAE encoder/decoder, which this build does not run; pass the VAE "
                    "encoder's moments to process_latent");
    }

    int process_latent(const Latent &moments, const TextEmbedding &positive, const TextEmbedding &negative,
                       Latent &output)
    {
        if (!is_loaded) return fail(Status::NotLoaded, "engine is not loaded");
        const TextEmbedding *pos = nullptr, *neg = nullptr;
        if (const int r = pick_texts(positive, negative, pos, neg)) return r;
        const int C = latent_channels;
        if (!moments.valid() || moments.channels != 2 * C || moments.height % 2 != 0 || moments.width % 2 != 0)
            return fail(Status::InvalidArgument, "moments must be [" + std::to_string(2 * C) +
                                                     "][T][H][W] fp32 with even H and W");
        const int T = moments.frames, H = moments.height, W = moments.width;
        const std::size_t plane = static_cast<std::size_t>(T) * H * W, n = plane * C;

        // Random streams in the engine's order (engine.cpp:280-296, vae.cpp:201-220):
        // one generator seeded once; the posterior draws (only when stochastic),
        // then the initial noise, then the augmentation noise, each phase with a
        // distribution object of its own, element order channel, frame, row, column.
        std::mt19937_64 random(options.seed);
        std::vector<float> encoded(n), noise(n), augment(n);
        {
            std::normal_distribution<float> normal(0.0f, 1.0f);
            const float *mean = moments.data.data(), *logvar = mean + n;
            for (std::size_t i = 0; i < n; ++i) {
                float value = mean[i];
                if (options.stochastic_vae) {
                    const float clamped = std::clamp(logvar[i], -30.0f, 20.0f);
                    value += std::exp(0.5f * clamped) * normal(random);
                }
                encoded[i] = value * options.vae_scaling_factor;
            }
        }
        for (std::vector<float> *v : {&noise, &augment}) {
            std::normal_distribution<float> normal(0.0f, 1.0f);
            for (float &x : *v) x = normal(random);
        }

        if (cudaSetDevice(device) != cudaSuccess) return fail(Status::InferenceFailed, "cudaSetDevice failed");
        const bool guide = options.cfg_scale != 1.0f;
        const std::size_t pos_n = pos->data.size(), neg_n = guide ? neg->data.size() : 0;
        if (!d_enc.ensure(n * 4) || !d_aug.ensure(n * 4) || !d_noise.ensure(n * 4) || !d_cond.ensure(n * 4) ||
            !d_out.ensure(n * 4) || !d_pos.ensure(pos_n * 4) || (guide && !d_neg.ensure(neg_n * 4)))
            return fail(Status::OutOfMemory, "failed to allocate the latent tensors on the GPU");
        if (cudaMemcpyAsync(d_enc.p, encoded.data(), n * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
            cudaMemcpyAsync(d_aug.p, augment.data(), n * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
            cudaMemcpyAsync(d_noise.p, noise.data(), n * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
            cudaMemcpyAsync(d_pos.p, pos->data.data(), pos_n * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess ||
            (guide &&
             cudaMemcpyAsync(d_neg.p, neg->data.data(), neg_n * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess))
            return drain(fail(Status::InferenceFailed, "upload of the latent inputs failed"));
        s2_status s = s2_make_condition(stream, d_enc.f(), d_aug.f(), C, T, H, W, options.condition_noise_scale,
                                        d_cond.f());
        if (s == S2_OK)
            s = s2_dit_sample_texts(dit, stream, d_noise.f(), d_cond.f(), T, H, W, d_pos.f(), pos->tokens,
                                    guide ? d_neg.f() : nullptr, guide ? neg->tokens : 0, options.sampling_steps,
                                    options.cfg_scale, options.cfg_rescale, d_out.f());
        if (s != S2_OK) return drain(fail(to_status(s), std::string("DiT sampling failed: ") + s2_last_error()));
        Latent result;
        result.channels = C;
        result.frames = T;
        result.height = H;
        result.width = W;
        result.data.resize(n);
        if (cudaMemcpyAsync(result.data.data(), d_out.p, n * 4, cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess)
            return drain(fail(Status::InferenceFailed, "download of the sampled latent failed"));
        int code = 0;
        if (s2_dit_device_error(dit, &code) != S2_OK)
            return fail(Status::InferenceFailed, std::string("DiT device error: ") + s2_last_error());
        output = std::move(result);
        error.clear();
        return static_cast<int>(Status::Ok);
    }

    bool is_loaded = false;
    std::string error;

private:
    int fail(Status s, const std::string &msg)
    {
        error = msg;
        return static_cast<int>(s);
    }

    // An error after copies were queued waits for them, so the host vectors they
    // read stay alive until the copies are done.
    int drain(int rc)
    {
        if (stream) cudaStreamSynchronize(stream);
        return rc;
    }

    static Status to_status(s2_status s)
    {
        switch (s) {
        case S2_INVALID_ARGUMENT: return Status::InvalidArgument;
        case S2_NOT_LOADED: return Status::NotLoaded;
        case S2_UNSUPPORTED: return Status::UnsupportedBackend;
        case S2_OUT_OF_MEMORY: return Status::OutOfMemory;
        default: return Status::InferenceFailed;
        }
    }

    // process()'s embedding rules (engine.cpp:247-262): an empty embedding falls
    // back to the model directory's default; the negative one is needed only
    // when guidance is on.
    int pick_texts(const TextEmbedding &positive, const TextEmbedding &negative, const TextEmbedding *&pos,
                   const TextEmbedding *&neg)
    {
        pos = positive.valid() ? &positive : (default_positive.valid() ? &default_positive : &positive);
        neg = negative.valid() ? &negative : (default_negative.valid() ? &default_negative : &negative);
        if (!pos->valid() || pos->channels != text_channels)
            return fail(Status::InvalidArgument, "positive embedding is empty and model dir has no default_pos_emb.bin");
        if (options.cfg_scale != 1.0f && (!neg->valid() || neg->channels != text_channels))
            return fail(Status::InvalidArgument, "negative embedding must be [tokens," +
                                                     std::to_string(text_channels) + "] when CFG is enabled");
        return 0;
    }

    void release()
    {
        if (dit) {
            s2_dit_destroy(dit);
            dit = nullptr;
        }
        if (is_loaded || stream) cudaSetDevice(device);
        for (DevBuf *b : {&d_enc, &d_aug, &d_noise, &d_cond, &d_out, &d_pos, &d_neg}) b->release();
        if (stream) cudaStreamDestroy(stream);
        stream = nullptr;
        is_loaded = false;
        default_positive = TextEmbedding{};
        default_negative = TextEmbedding{};
    }

    RuntimeOptions options;
    int device = 0;
    int latent_channels = 16, text_channels = 5120;
    s2_dit *dit = nullptr;
    cudaStream_t stream = nullptr;
    DevBuf d_enc, d_aug, d_noise, d_cond, d_out, d_pos, d_neg;
    TextEmbedding default_positive, default_negative;
};

SeedVR2Engine::SeedVR2Engine() : impl_(std::make_unique<Impl>()) {}
SeedVR2Engine::~SeedVR2Engine() = default;
SeedVR2Engine::SeedVR2Engine(SeedVR2Engine &&) noexcept = default;
SeedVR2Engine &SeedVR2Engine::operator=(SeedVR2Engine &&) noexcept = default;

int SeedVR2Engine::load(const std::string &model_dir, const RuntimeOptions &options)
{
    if (!impl_) impl_ = std::make_unique<Impl>();
    return impl_->load(model_dir, options);
}

int SeedVR2Engine::process(const Video &input, const TextEmbedding &positive, const TextEmbedding &negative,
                           Video &output)
{
    if (!impl_) impl_ = std::make_unique<Impl>();
    return impl_->process(input, positive, negative, output);
}

int SeedVR2Engine::process_latent(const Latent &moments, const TextEmbedding &positive,
                                  const TextEmbedding &negative, Latent &output)
{
    if (!impl_) impl_ = std::make_unique<Impl>();
    return impl_->process_latent(moments, positive, negative, output);
}

bool SeedVR2Engine::loaded() const noexcept { return impl_ && impl_->is_loaded; }

const std::string &SeedVR2Engine::last_error() const noexcept
{
    static const std::string moved_from = "engine was moved from";
    return impl_ ? impl_->error : moved_from;
}

const char *status_message(Status status) noexcept
{
    switch (status) {
    case Status::Ok: return "ok";
    case Status::InvalidArgument: return "invalid argument";
    case Status::NotLoaded: return "engine is not loaded";
    case Status::ModelNotFound: return "model file not found";
    case Status::ModelLoadFailed: return "model load failed";
    case Status::InferenceFailed: return "inference failed";
    case Status::UnsupportedBackend: return "unsupported backend";
    case Status::OutOfMemory: return "out of memory";
    case Status::IoError: return "io error";
    }
    return "unknown status";
}
}  // namespace seedvr2
