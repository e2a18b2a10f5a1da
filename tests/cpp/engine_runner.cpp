// TEST INFRASTRUCTURE: runner for seedvr2::SeedVR2Engine (include/seedvr2/engine.h,
// libseedvr2.so over the C ABI), shaped like the reference's install-consumer
// program (tests/install_consumer/main.cpp): a caller that includes only the
// public engine header.
//
//   engine_runner errors
//       Status paths that need no GPU: empty model_dir, invalid sampling
//       options (src/core/vulkan_context.cpp:62-69), the CPU / Vulkan devices
//       this build does not have, process() before load(), status_message().
//   engine_runner run <model_dir> <moments.bin> <out_dir> <2C> <T> <H> <W>
//                     <steps> <cfg> <rescale> <noise_scale> <seed> <stochastic>
//       load() on the CUDA device, process_latent() with empty embeddings (the
//       model directory's defaults), twice on a moved engine (same bytes), plus
//       the error returns of process() and of bad moments. Writes x0.bin (the
//       sampled latent) and the engine's random draws restated here in the
//       reference's order (src/core/engine.cpp:280-296, src/model/vae.cpp:201-220)
//       -- encoded.bin (posterior sample x scaling factor), noise.bin,
//       augment.bin -- for the test to rebuild the expected result with the
//       reference's own sampler code.
//
// Prints one "[name] PASS|FAIL ..." line per check; exit status 0 when all pass.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <utility>
#include <vector>

#include "seedvr2/engine.h"

namespace
{
int failures = 0;

void check(bool ok, const char *name, const std::string &detail = "")
{
    std::printf("[%s] %s%s%s\n", name, ok ? "PASS" : "FAIL", detail.empty() ? "" : " ", detail.c_str());
    if (!ok) ++failures;
}

int code(seedvr2::Status s) { return static_cast<int>(s); }

bool write_file(const std::string &path, const std::vector<float> &v)
{
    FILE *f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    const bool ok = std::fwrite(v.data(), sizeof(float), v.size(), f) == v.size();
    return std::fclose(f) == 0 && ok;
}

int run_errors()
{
    using seedvr2::Status;
    seedvr2::SeedVR2Engine e;
    check(e.load("") == code(Status::InvalidArgument), "empty model_dir");
    seedvr2::RuntimeOptions bad;
    bad.sampling_steps = 0;
    check(e.load("/nonexistent", bad) == code(Status::InvalidArgument), "sampling_steps 0");
    bad = {};
    bad.cfg_rescale = 1.5f;
    check(e.load("/nonexistent", bad) == code(Status::InvalidArgument), "cfg_rescale > 1");
    bad = {};
    bad.condition_noise_scale = -0.1f;
    check(e.load("/nonexistent", bad) == code(Status::InvalidArgument), "condition_noise_scale < 0");
    bad = {};
    bad.vae_scaling_factor = 0.f;
    check(e.load("/nonexistent", bad) == code(Status::InvalidArgument), "vae_scaling_factor 0");
    for (seedvr2::DeviceType d : {seedvr2::DeviceType::Cpu, seedvr2::DeviceType::Vulkan}) {
        seedvr2::RuntimeOptions o;
        o.device = d;
        check(e.load("/nonexistent", o) == code(Status::UnsupportedBackend), "cpu/vulkan device", e.last_error());
    }
    check(!e.loaded(), "not loaded after failures");
    seedvr2::Video in, out;
    seedvr2::TextEmbedding t;
    check(e.process(in, t, t, out) == code(Status::NotLoaded), "process before load");
    seedvr2::Latent m, x;
    check(e.process_latent(m, t, t, x) == code(Status::NotLoaded), "process_latent before load");
    check(std::strcmp(seedvr2::status_message(Status::OutOfMemory), "out of memory") == 0, "status_message");
    seedvr2::Video v;
    v.frames = 1, v.height = 2, v.width = 2;
    v.data.assign(12, 0.5f);
    check(v.valid(), "video valid");
    v.fps = 0.f;
    check(!v.valid(), "video fps 0 invalid");
    return failures == 0 ? 0 : 1;
}

int run_sample(int argc, char **argv)
{
    using seedvr2::Status;
    if (argc != 15) {
        std::fprintf(stderr, "usage: engine_runner run <model_dir> <moments.bin> <out_dir> <2C> <T> <H> <W> <steps> "
                             "<cfg> <rescale> <noise_scale> <seed> <stochastic>\n");
        return 2;
    }
    const std::string model_dir = argv[2], moments_path = argv[3], out_dir = argv[4];
    seedvr2::Latent m;
    m.channels = std::atoi(argv[5]);
    m.frames = std::atoi(argv[6]);
    m.height = std::atoi(argv[7]);
    m.width = std::atoi(argv[8]);
    seedvr2::RuntimeOptions o;
    o.device = seedvr2::DeviceType::Cuda;
    o.sampling_steps = std::atoi(argv[9]);
    o.cfg_scale = static_cast<float>(std::atof(argv[10]));
    o.cfg_rescale = static_cast<float>(std::atof(argv[11]));
    o.condition_noise_scale = static_cast<float>(std::atof(argv[12]));
    o.seed = std::strtoull(argv[13], nullptr, 10);
    o.stochastic_vae = std::atoi(argv[14]) != 0;
    const std::size_t n2 = static_cast<std::size_t>(m.channels) * m.frames * m.height * m.width;
    m.data.resize(n2);
    FILE *f = std::fopen(moments_path.c_str(), "rb");
    if (!f || std::fread(m.data.data(), sizeof(float), n2, f) != n2) {
        std::fprintf(stderr, "cannot read %s\n", moments_path.c_str());
        return 2;
    }
    std::fclose(f);

    seedvr2::SeedVR2Engine engine;
    const int rc = engine.load(model_dir, o);
    check(rc == code(Status::Ok) && engine.loaded(), "load", engine.last_error());
    if (rc != 0) return 1;
    seedvr2::TextEmbedding none;
    seedvr2::Latent x0;
    const int pr = engine.process_latent(m, none, none, x0);
    check(pr == code(Status::Ok), "process_latent", engine.last_error());
    if (pr != 0) return 1;
    check(x0.channels * 2 == m.channels && x0.frames == m.frames && x0.height == m.height && x0.width == m.width,
          "output shape");
    // a moved engine keeps its model and gives the same bytes
    seedvr2::SeedVR2Engine moved(std::move(engine));
    seedvr2::Latent again;
    check(moved.process_latent(m, none, none, again) == code(Status::Ok) && again.data == x0.data,
          "moved engine, same result", moved.last_error());
    // error returns on a loaded engine
    seedvr2::Video v, vout;
    v.frames = 5, v.height = 16, v.width = 16;
    v.data.assign(static_cast<std::size_t>(5) * 16 * 16 * 3, 0.5f);
    check(moved.process(v, none, none, vout) == code(Status::UnsupportedBackend), "process(video)",
          moved.last_error());
    seedvr2::Latent odd = m;
    odd.channels = m.channels / 2;
    odd.data.resize(odd.data.size() / 2);
    seedvr2::Latent dummy;
    check(moved.process_latent(odd, none, none, dummy) == code(Status::InvalidArgument), "moments channel check");
    seedvr2::TextEmbedding wrong;
    wrong.tokens = 3;
    wrong.channels = 7;
    wrong.data.assign(21, 0.f);
    check(moved.process_latent(m, wrong, none, dummy) == code(Status::InvalidArgument), "embedding channels");

    // The engine's random draws, restated in the reference's order.
    const std::size_t n = n2 / 2;
    std::vector<float> encoded(n), noise(n), augment(n);
    std::mt19937_64 random(o.seed);
    {
        std::normal_distribution<float> normal(0.0f, 1.0f);
        for (std::size_t i = 0; i < n; ++i) {
            float value = m.data[i];
            if (o.stochastic_vae)
                value += std::exp(0.5f * std::clamp(m.data[n + i], -30.0f, 20.0f)) * normal(random);
            encoded[i] = value * o.vae_scaling_factor;
        }
    }
    {
        std::normal_distribution<float> normal(0.0f, 1.0f);
        for (float &v2 : noise) v2 = normal(random);
    }
    {
        std::normal_distribution<float> normal(0.0f, 1.0f);
        for (float &v2 : augment) v2 = normal(random);
    }
    const bool wrote = write_file(out_dir + "/x0.bin", x0.data) && write_file(out_dir + "/encoded.bin", encoded) &&
                       write_file(out_dir + "/noise.bin", noise) && write_file(out_dir + "/augment.bin", augment);
    check(wrote, "write outputs");
    return failures == 0 ? 0 : 1;
}
}  // namespace

int main(int argc, char **argv)
{
    if (argc >= 2 && std::strcmp(argv[1], "errors") == 0) return run_errors();
    if (argc >= 2 && std::strcmp(argv[1], "run") == 0) return run_sample(argc, argv);
    std::fprintf(stderr, "usage: engine_runner errors | run ...\n");
    return 2;
}
