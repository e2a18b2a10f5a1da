// Readers for the reference's exported model files (host only): the ncnn
// .param text graph of one custom layer and its .bin weight blobs, decoded
// into the fp32 weight stream the layer's load_model reads -- so a model
// directory written by the reference's exporter (tools/export_seedvr2_dit_ncnn.py)
// loads directly (SeedVR2DiT::load, src/model/dit.cpp:119-214).
//
// .param: "7767517", "<layers> <blobs>", one line per layer:
//   <type> <name> <n_in> <n_out> <in blobs...> <out blobs...> [k=v ...]
// .bin, in load_model order: type-1 blobs are raw little-endian fp32 (biases,
// norms, adaLN vectors); type-0 blobs (InnerProduct weights) start with a
// 4-byte tag: 0x01306B47 = fp16 data padded to 4 bytes, 0 = fp32 data.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "s2_internal.h"

namespace {

constexpr uint32_t kFp16Tag = 0x01306B47u;

struct Param {
    std::string type;
    int ints[32];
    float floats[32];
    bool set[32];
};

// Finds the line of layer `type` and its key=value pairs (keys 0..31).
s2_status read_param(const char *path, const char *type, Param &p)
{
    std::ifstream f(path);
    if (!f) return s2::set_error(S2_INVALID_ARGUMENT, "cannot open %s", path);
    std::string magic;
    f >> magic;
    if (magic != "7767517") return s2::set_error(S2_INVALID_ARGUMENT, "%s: not an ncnn param file", path);
    int layers = 0, blobs = 0;
    f >> layers >> blobs;
    std::string line;
    std::getline(f, line);
    for (int i = 0; i < layers && std::getline(f, line); ++i) {
        std::istringstream ls(line);
        std::string t, name;
        int nin = 0, nout = 0;
        ls >> t >> name >> nin >> nout;
        if (t != type) continue;
        for (int k = 0; k < nin + nout; ++k) {
            std::string blob;
            ls >> blob;
        }
        p.type = t;
        for (int k = 0; k < 32; ++k) p.set[k] = false;
        std::string kv;
        while (ls >> kv) {
            const size_t eq = kv.find('=');
            if (eq == std::string::npos) return s2::set_error(S2_INVALID_ARGUMENT, "%s: bad pair '%s'", path, kv.c_str());
            const int key = std::atoi(kv.substr(0, eq).c_str());
            if (key < 0 || key >= 32)
                return s2::set_error(S2_UNSUPPORTED, "%s: parameter key %d not supported", path, key);
            const std::string v = kv.substr(eq + 1);
            p.floats[key] = std::strtof(v.c_str(), nullptr);
            p.ints[key] = std::atoi(v.c_str());
            p.set[key] = true;
        }
        return S2_OK;
    }
    return s2::set_error(S2_INVALID_ARGUMENT, "%s: no %s layer", path, type);
}

int geti(const Param &p, int k, int dflt) { return p.set[k] ? p.ints[k] : dflt; }
float getf(const Param &p, int k, float dflt) { return p.set[k] ? p.floats[k] : dflt; }

float half_to_float(uint16_t h)
{
    const uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: renormalise
            int e = -1;
            uint32_t m = man;
            do {
                m <<= 1;
                ++e;
            } while ((m & 0x400u) == 0);
            bits = sign | ((112u - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// Decodes blobs of the given (count, type) schedule from a .bin file.
struct BinReader {
    FILE *f = nullptr;
    const char *path;
    std::vector<float> *out;
    explicit BinReader(const char *p, std::vector<float> *o) : path(p), out(o) { f = std::fopen(p, "rb"); }
    ~BinReader()
    {
        if (f) std::fclose(f);
    }
    s2_status raw(size_t n)
    {
        const size_t at = out->size();
        out->resize(at + n);
        if (std::fread(out->data() + at, 4, n, f) != n)
            return s2::set_error(S2_INVALID_ARGUMENT, "%s: truncated (raw fp32 blob of %zu)", path, n);
        return S2_OK;
    }
    s2_status tagged(size_t n)
    {
        uint32_t tag = 0;
        if (std::fread(&tag, 4, 1, f) != 1) return s2::set_error(S2_INVALID_ARGUMENT, "%s: truncated (tag)", path);
        if (tag == 0) return raw(n);
        if (tag != kFp16Tag)
            return s2::set_error(S2_UNSUPPORTED, "%s: weight tag 0x%08x (fp16 0x%08x and fp32 0 are supported)", path,
                                 tag, kFp16Tag);
        std::vector<uint16_t> h(n);
        if (std::fread(h.data(), 2, n, f) != n)
            return s2::set_error(S2_INVALID_ARGUMENT, "%s: truncated (fp16 blob of %zu)", path, n);
        if ((n * 2) % 4) {
            uint16_t pad;
            if (std::fread(&pad, 2, 1, f) != 1) return s2::set_error(S2_INVALID_ARGUMENT, "%s: truncated padding", path);
        }
        const size_t at = out->size();
        out->resize(at + n);
        for (size_t i = 0; i < n; ++i) (*out)[at + i] = half_to_float(h[i]);
        return S2_OK;
    }
    s2_status finish()
    {
        if (std::fgetc(f) != EOF) return s2::set_error(S2_INVALID_ARGUMENT, "%s: trailing bytes after the last blob", path);
        return S2_OK;
    }
};

s2_status copy_out(const std::vector<float> &w, float *weights, size_t cap, size_t *n)
{
    *n = w.size();
    if (!weights) return S2_OK;
    if (cap < w.size()) return s2::set_error(S2_INVALID_ARGUMENT, "weight buffer holds %zu floats, %zu needed", cap, w.size());
    std::memcpy(weights, w.data(), w.size() * 4);
    return S2_OK;
}

}  // namespace

extern "C" s2_status s2_ncnn_read_block(const char *param_path, const char *bin_path, s2_block_params *bp,
                                        float *weights, size_t cap, size_t *n)
{
    s2::clear_error();
    if (!param_path || !bin_path || !bp || !n) return s2::set_error(S2_INVALID_ARGUMENT, "s2_ncnn_read_block: null argument");
    Param p;
    s2_status s = read_param(param_path, "SeedVR2DiTBlock", p);
    if (s != S2_OK) return s;
    // ParamDict keys 0..8 and their defaults (seedvr2_dit_block.cpp:643-655)
    bp->block_index = geti(p, 0, 0);
    bp->shared = geti(p, 1, 0);
    bp->last = geti(p, 2, 0);
    bp->shifted = geti(p, 3, 0);
    bp->dim = geti(p, 4, 2560);
    bp->heads = geti(p, 5, 20);
    bp->head_dim = geti(p, 6, 128);
    bp->mlp_hidden = geti(p, 7, 6912);
    bp->eps = getf(p, 8, 1e-5f);
    if (bp->dim <= 0 || bp->dim != bp->heads * bp->head_dim || bp->mlp_hidden <= 0)
        return s2::set_error(S2_INVALID_ARGUMENT, "%s: inconsistent block parameters", param_path);
    std::vector<float> w;
    BinReader r(bin_path, &w);
    if (!r.f) return s2::set_error(S2_INVALID_ARGUMENT, "cannot open %s", bin_path);
    const size_t d = bp->dim, h = bp->mlp_hidden, hd = bp->head_dim;
    for (int br = 0; br < (bp->shared ? 1 : 2); ++br) {  // load_branch (:657-680)
        if ((s = r.raw(6 * d)) != S2_OK || (s = r.tagged(3 * d * d)) != S2_OK || (s = r.tagged(d * d)) != S2_OK ||
            (s = r.raw(d)) != S2_OK || (s = r.raw(hd)) != S2_OK || (s = r.raw(hd)) != S2_OK ||
            (s = r.tagged(h * d)) != S2_OK || (s = r.tagged(h * d)) != S2_OK || (s = r.tagged(d * h)) != S2_OK)
            return s;
    }
    if ((s = r.raw(S2_ROPE_PAIRS)) != S2_OK || (s = r.finish()) != S2_OK) return s;
    return copy_out(w, weights, cap, n);
}

extern "C" s2_status s2_ncnn_read_input(const char *param_path, const char *bin_path, s2_head_params *hp,
                                        float *weights, size_t cap, size_t *n)
{
    s2::clear_error();
    if (!param_path || !bin_path || !hp || !n) return s2::set_error(S2_INVALID_ARGUMENT, "s2_ncnn_read_input: null argument");
    Param p;
    s2_status s = read_param(param_path, "SeedVR2DiTInput", p);
    if (s != S2_OK) return s;
    // seedvr2_dit_input.cpp:207-214
    hp->dim = geti(p, 0, 2560);
    hp->video_channels = geti(p, 1, 33);
    hp->text_channels = geti(p, 2, 5120);
    hp->sinusoidal_dim = geti(p, 3, 256);
    hp->embedding_dim = geti(p, 4, 15360);
    hp->out_channels = 0;
    hp->eps = 0.f;
    std::vector<float> w;
    BinReader r(bin_path, &w);
    if (!r.f) return s2::set_error(S2_INVALID_ARGUMENT, "cannot open %s", bin_path);
    const size_t d = hp->dim;
    const size_t io[5][2] = {{static_cast<size_t>(4 * hp->video_channels), d},
                             {static_cast<size_t>(hp->text_channels), d},
                             {static_cast<size_t>(hp->sinusoidal_dim), d},
                             {d, d},
                             {d, static_cast<size_t>(hp->embedding_dim)}};
    for (const auto &x : io)  // each InnerProduct: weight (tagged) then bias (raw), :217-224
        if ((s = r.tagged(x[0] * x[1])) != S2_OK || (s = r.raw(x[1])) != S2_OK) return s;
    if ((s = r.finish()) != S2_OK) return s;
    return copy_out(w, weights, cap, n);
}

extern "C" s2_status s2_ncnn_read_output(const char *param_path, const char *bin_path, s2_head_params *hp,
                                         float *weights, size_t cap, size_t *n)
{
    s2::clear_error();
    if (!param_path || !bin_path || !hp || !n) return s2::set_error(S2_INVALID_ARGUMENT, "s2_ncnn_read_output: null argument");
    Param p;
    s2_status s = read_param(param_path, "SeedVR2DiTOutput", p);
    if (s != S2_OK) return s;
    // seedvr2_dit_output.cpp:256-270
    hp->dim = geti(p, 0, 2560);
    hp->out_channels = geti(p, 1, 16);
    hp->eps = getf(p, 2, 1e-5f);
    hp->video_channels = hp->text_channels = hp->sinusoidal_dim = hp->embedding_dim = 0;
    std::vector<float> w;
    BinReader r(bin_path, &w);
    if (!r.f) return s2::set_error(S2_INVALID_ARGUMENT, "cannot open %s", bin_path);
    const size_t d = hp->dim, no = 4 * static_cast<size_t>(hp->out_channels);
    if ((s = r.raw(3 * d)) != S2_OK || (s = r.tagged(no * d)) != S2_OK || (s = r.raw(no)) != S2_OK ||
        (s = r.finish()) != S2_OK)
        return s;
    return copy_out(w, weights, cap, n);
}

extern "C" s2_status s2_dit_load_dir(s2_dit *model, const char *dir)
{
    s2::clear_error();
    if (!model || !dir) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_load_dir: null argument");
    const std::string root(dir);
    auto path = [&](const char *stem, const char *ext) { return root + "/" + stem + ".ncnn." + ext; };
    std::vector<float> w;
    size_t n = 0;
    s2_head_params hp;
    s2_status s = s2_ncnn_read_input(path("seedvr2_dit_input", "param").c_str(), path("seedvr2_dit_input", "bin").c_str(),
                                     &hp, nullptr, 0, &n);
    if (s != S2_OK) return s;
    w.resize(n);
    if ((s = s2_ncnn_read_input(path("seedvr2_dit_input", "param").c_str(), path("seedvr2_dit_input", "bin").c_str(),
                                &hp, w.data(), w.size(), &n)) != S2_OK ||
        (s = s2_dit_load_input(model, w.data(), n)) != S2_OK)
        return s;
    if ((s = s2_ncnn_read_output(path("seedvr2_dit_output", "param").c_str(), path("seedvr2_dit_output", "bin").c_str(),
                                 &hp, nullptr, 0, &n)) != S2_OK)
        return s;
    w.resize(n);
    if ((s = s2_ncnn_read_output(path("seedvr2_dit_output", "param").c_str(), path("seedvr2_dit_output", "bin").c_str(),
                                 &hp, w.data(), w.size(), &n)) != S2_OK ||
        (s = s2_dit_load_output(model, w.data(), n)) != S2_OK)
        return s;
    for (int i = 0;; ++i) {
        char stem[64];
        std::snprintf(stem, sizeof(stem), "seedvr2_dit_block_%02d", i);
        const std::string pp = path(stem, "param"), bp = path(stem, "bin");
        FILE *probe = std::fopen(pp.c_str(), "r");
        if (!probe) {
            if (i == 0) return s2::set_error(S2_INVALID_ARGUMENT, "s2_dit_load_dir: %s missing", pp.c_str());
            break;
        }
        std::fclose(probe);
        s2_block_params blk;
        if ((s = s2_ncnn_read_block(pp.c_str(), bp.c_str(), &blk, nullptr, 0, &n)) != S2_OK) return s;
        w.resize(n);
        if ((s = s2_ncnn_read_block(pp.c_str(), bp.c_str(), &blk, w.data(), w.size(), &n)) != S2_OK) return s;
        if (blk.block_index != i)
            return s2::set_error(S2_INVALID_ARGUMENT, "%s: block_index %d in block file %d", pp.c_str(), blk.block_index, i);
        if ((s = s2_dit_load_block(model, i, blk.shared, blk.last, blk.shifted, w.data(), n)) != S2_OK) return s;
    }
    return S2_OK;
}
