// seedvr2/engine.h -- the SeedVR2 Engine API over the B200 (sm_100a) path.
//
// Drop-in surface of czwdysj/seedvr2-ncnn-valkan's include/seedvr2/engine.h:14-120:
// the same namespace, class, member and enumerator names, the same Status
// values, RuntimeOptions fields and defaults, and Video / TextEmbedding layouts,
// so code written against that header compiles against this one. The engine is
// host C++ that drives the device through the C ABI of include/s2_b200.h.
//
// Additions (no counterpart in the reference):
//  * DeviceType::Cuda (appended; Cpu and Vulkan keep their values) and
//    RuntimeOptions::cuda_device_index. The default device of this build is
//    Cuda: it has no CPU or Vulkan backend, and load() with either returns
//    Status::UnsupportedBackend.
//  * Latent and SeedVR2Engine::process_latent: the part of process() between
//    the VAE encoder and the VAE decoder -- posterior sampling, the diffusion
//    noise, the condition latent and the DiT sampling loop with classifier-
//    free guidance (src/core/engine.cpp:264-347) -- on the GPU. The VAE
//    convolutions are not part of this build, so process() on pixel video
//    returns Status::UnsupportedBackend with a message naming process_latent.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#if defined(__GNUC__)
#define SEEDVR2_API __attribute__((visibility("default")))
#else
#define SEEDVR2_API
#endif

namespace seedvr2
{
enum class DeviceType
{
    Cpu,
    Vulkan,
    Cuda,  // this build's backend (B200, sm_100a)
};

enum class Status
{
    Ok = 0,
    InvalidArgument = -1,
    NotLoaded = -2,
    ModelNotFound = -3,
    ModelLoadFailed = -4,
    InferenceFailed = -5,
    UnsupportedBackend = -6,
    OutOfMemory = -7,
    IoError = -8,
};

struct RuntimeOptions
{
    DeviceType device = DeviceType::Cuda;
    int num_threads = 0;          // host threads; the device path does not use them
    int vulkan_device_index = 0;  // kept for source compatibility
    int sampling_steps = 1;
    float cfg_scale = 1.0f;
    float cfg_rescale = 0.0f;
    float condition_noise_scale = 0.0f;
    float vae_scaling_factor = 0.9152f;
    std::uint64_t seed = 666;
    bool stochastic_vae = true;
    // The device path stores weights and GEMM operands in fp16 and accumulates
    // in fp32 whatever these say; kept for source compatibility.
    bool use_fp16_storage = false;
    bool use_fp16_arithmetic = false;
    // The device path always keeps the 32 blocks' weights resident in HBM
    // (6.7 GB of 180 GB); kept for source compatibility.
    bool dit_resident = false;
    int cuda_device_index = 0;
};

// THWC, RGB, fp32 in [0, 1].
struct SEEDVR2_API Video
{
    int frames = 0;
    int height = 0;
    int width = 0;
    int channels = 3;
    float fps = 24.0f;
    std::vector<float> data;

    bool valid() const noexcept;
};

// [tokens][channels] fp32; channels 5120 for SeedVR2-3B.
struct SEEDVR2_API TextEmbedding
{
    int tokens = 0;
    int channels = 5120;
    std::vector<float> data;

    bool valid() const noexcept;
};

// A latent-space tensor [channels][frames][height][width] fp32 (the VAE's
// 4x temporal / 8x spatial grid). As process_latent's input it holds the VAE
// encoder's moments (mean channels, then log-variance channels); as its output
// the sampled latent the VAE decoder takes.
struct SEEDVR2_API Latent
{
    int channels = 0;
    int frames = 0;
    int height = 0;
    int width = 0;
    std::vector<float> data;

    bool valid() const noexcept;
};

class SEEDVR2_API SeedVR2Engine
{
public:
    SeedVR2Engine();
    ~SeedVR2Engine();

    SeedVR2Engine(SeedVR2Engine&&) noexcept;
    SeedVR2Engine& operator=(SeedVR2Engine&&) noexcept;
    SeedVR2Engine(const SeedVR2Engine&) = delete;
    SeedVR2Engine& operator=(const SeedVR2Engine&) = delete;

    // Loads the DiT from model_dir/dit_full_fp16 (or model_dir itself) -- the
    // exporter's seedvr2_dit_input / _block_NN / _output .ncnn.param + .bin --
    // onto the GPU, and the optional default text embeddings
    // model_dir/default_pos_emb.bin / default_neg_emb.bin (int32 tokens, int32
    // channels, fp32 data). Returns a Status value; last_error() says why.
    int load(const std::string& model_dir, const RuntimeOptions& options = {});

    // Pixel video in and out. Returns Status::UnsupportedBackend in this build
    // (no VAE convolutions); see process_latent.
    int process(const Video& input, const TextEmbedding& positive, const TextEmbedding& negative, Video& output);

    // From VAE-encoder moments [2 C][T][H][W] (H and W even) to the sampled
    // latent [C][T][H][W], with the engine's random streams and order (seed,
    // posterior draws when stochastic_vae, initial noise, augmentation noise).
    // Empty embeddings fall back to the model directory's defaults, as in
    // process().
    int process_latent(const Latent& moments, const TextEmbedding& positive, const TextEmbedding& negative,
                       Latent& output);

    bool loaded() const noexcept;
    const std::string& last_error() const noexcept;

private:
    class Impl;
    std::unique_ptr<Impl> impl_;
};

SEEDVR2_API const char* status_message(Status status) noexcept;
}  // namespace seedvr2
