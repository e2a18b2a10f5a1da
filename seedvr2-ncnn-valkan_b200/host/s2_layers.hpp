// C++ host mirror of the reference's ncnn custom-layer interface for the B200
// path, over the C ABI in s2_b200.h (header-only, C++17).
//
// The two layers this path replaces keep their names, their load_param /
// load_model / set_runtime_shape / forward calls, the meaning of every
// argument and the reference's return codes:
//
//   SeedVR2DiTBlock                   src/layers/seedvr2_dit_block.h:38-170
//       load_param  keys 0-8         seedvr2_dit_block.cpp:643-655
//       load_model  ModelBin order    seedvr2_dit_block.cpp:657-688
//       forward     vid, txt, emb, vid_shape -> vid_out, txt_out
//                                     seedvr2_dit_block.cpp:1114-1267
//   DynamicFramewiseSpatialAttention  src/layers/dynamic_framewise_spatial_attention.h
//       load_param  key 10 = channel count array   .cpp:50-59
//       load_model  norm_bias .. v_weight          .cpp:61-77
//       forward     one 4-D blob (w=W, h=H, d=T, c=C) -> same shape  .cpp:106-210
//
// Return codes follow the reference: 0 ok, -1 bad parameters, shapes or blob
// counts (seedvr2_dit_block.cpp:1119-1138), -100 allocation or device failure
// (the reference's sub-layer / allocation failures). last_error() holds the
// library's message of the last failure.
//
// The ncnn types the contract uses are stood in for by the small classes
// below (Mat, ParamDict, ModelBin, Option): the subset of ncnn's API the two
// layers read, with ncnn's layout rules (4-D blobs channel-major with each
// channel padded to 16 bytes, cstep).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "s2_b200.h"

namespace s2b200
{

// ---- ncnn stand-ins ---------------------------------------------------------

// A host blob: 1-D (w), 2-D (w x h rows) or 4-D (w x h x d per channel, c
// channels). Copies share storage, as ncnn's refcounted Mat does.
class Mat
{
public:
    int dims = 0, w = 0, h = 0, d = 0, c = 0;
    size_t elemsize = 0, cstep = 0;
    void *data = nullptr;

    Mat() = default;
    explicit Mat(int _w, size_t _elemsize = 4u) { create(_w, _elemsize); }
    Mat(int _w, int _h, size_t _elemsize = 4u) { create(_w, _h, _elemsize); }
    Mat(int _w, int _h, int _d, int _c, size_t _elemsize = 4u) { create(_w, _h, _d, _c, _elemsize); }

    void create(int _w, size_t _elemsize = 4u) { alloc(1, _w, 1, 1, 1, _elemsize, static_cast<size_t>(_w)); }
    void create(int _w, int _h, size_t _elemsize = 4u)
    {
        alloc(2, _w, _h, 1, 1, _elemsize, static_cast<size_t>(_w) * _h);
    }
    void create(int _w, int _h, int _d, int _c, size_t _elemsize = 4u)
    {
        const size_t plane = static_cast<size_t>(_w) * _h * _d * _elemsize;
        alloc(4, _w, _h, _d, _c, _elemsize, ((plane + 15) & ~static_cast<size_t>(15)) / _elemsize);
    }

    bool empty() const { return data == nullptr || total() == 0; }
    size_t total() const { return cstep * static_cast<size_t>(c); }
    float *row(int y) { return static_cast<float *>(data) + static_cast<size_t>(w) * y; }
    const float *row(int y) const { return static_cast<const float *>(data) + static_cast<size_t>(w) * y; }
    float *channel(int q) { return static_cast<float *>(data) + cstep * q; }
    const float *channel(int q) const { return static_cast<const float *>(data) + cstep * q; }
    template <typename T>
    operator T *()
    {
        return static_cast<T *>(data);
    }
    template <typename T>
    operator const T *() const
    {
        return static_cast<const T *>(data);
    }

private:
    std::shared_ptr<std::vector<unsigned char>> store_;

    void alloc(int _dims, int _w, int _h, int _d, int _c, size_t _elemsize, size_t _cstep)
    {
        dims = _dims, w = _w, h = _h, d = _d, c = _c, elemsize = _elemsize, cstep = _cstep;
        const size_t bytes = cstep * static_cast<size_t>(c) * elemsize;
        store_ = std::make_shared<std::vector<unsigned char>>(bytes > 0 ? bytes : 1, 0);
        data = store_->data();
    }
};

// Integer / float / blob parameters by id, as ncnn::ParamDict.
class ParamDict
{
public:
    int get(int id, int def) const { return kind(id) == 1 ? e_[id].i : def; }
    float get(int id, float def) const { return kind(id) == 2 ? e_[id].f : def; }
    Mat get(int id, const Mat &def) const { return kind(id) == 3 ? e_[id].m : def; }
    void set(int id, int v) { grow(id).kind = 1, e_[id].i = v; }
    void set(int id, float v) { grow(id).kind = 2, e_[id].f = v; }
    void set(int id, const Mat &v) { grow(id).kind = 3, e_[id].m = v; }

private:
    struct Entry
    {
        int kind = 0, i = 0;
        float f = 0.f;
        Mat m;
    };
    std::vector<Entry> e_;
    int kind(int id) const { return id >= 0 && id < static_cast<int>(e_.size()) ? e_[id].kind : 0; }
    Entry &grow(int id)
    {
        if (id >= static_cast<int>(e_.size())) e_.resize(id + 1);
        return e_[id];
    }
};

// Sequential weight arrays, as ncnn::ModelBin (load(w, type) returns the next
// w values as fp32; an empty Mat once the stream is exhausted).
class ModelBin
{
public:
    virtual ~ModelBin() = default;
    virtual Mat load(int w, int type) const = 0;
};

// A ModelBin over one flat fp32 array in load order.
class ModelBinFromFloats : public ModelBin
{
public:
    ModelBinFromFloats(const float *data, size_t count) : data_(data), count_(count) {}
    Mat load(int w, int) const override
    {
        if (w <= 0 || pos_ + static_cast<size_t>(w) > count_) return Mat();
        Mat m(w);
        std::memcpy(m.data, data_ + pos_, static_cast<size_t>(w) * sizeof(float));
        pos_ += static_cast<size_t>(w);
        return m;
    }
    size_t consumed() const { return pos_; }

private:
    const float *data_;
    size_t count_;
    mutable size_t pos_ = 0;
};

// The options forward() reads: the CUDA device and the stream the call runs on
// (the host-buffer forward synchronises it before returning, as the reference's
// CPU forward returns with its outputs written).
struct Option
{
    int num_threads = 1;  // kept for signature parity; the B200 path does not use host threads
    int device = 0;
    void *stream = nullptr;
};

// ---- status mapping -------------------------------------------------------------

// The reference's codes for a library status: -1 for invalid arguments and
// shape mismatches, -100 for everything that failed on the device or in allocation.
inline int reference_code(s2_status s)
{
    if (s == S2_OK) return 0;
    if (s == S2_INVALID_ARGUMENT) return -1;
    return -100;
}

// ---- SeedVR2DiTBlock ------------------------------------------------------------

// The reference's debug capture (seedvr2_dit_block.h:20-36): [rows][channels]
// fp32 Mats of one forward, filled when set with set_debug_tensors.
struct SeedVR2DiTBlockDebugTensors {
    Mat qkv_vid, qkv_txt;
    Mat norm_q_vid, norm_q_txt, norm_k_vid, norm_k_txt;
    Mat attention_q, attention_k, attention_v, attention_output;
    Mat projected_vid, projected_txt;
    Mat output_vid, output_txt;
};

class SeedVR2DiTBlock
{
public:
    explicit SeedVR2DiTBlock(int device = 0) : device_(device) {}
    ~SeedVR2DiTBlock() { release(); }
    SeedVR2DiTBlock(const SeedVR2DiTBlock &) = delete;
    SeedVR2DiTBlock &operator=(const SeedVR2DiTBlock &) = delete;

    // keys 0 block_index, 1 shared_weights, 2 last_layer, 3 shifted, 4 dim,
    // 5 heads, 6 head_dim, 7 mlp_hidden, 8 eps; -1 unless dim == heads * head_dim.
    int load_param(const ParamDict &pd)
    {
        block_index = pd.get(0, 0);
        shared_weights = pd.get(1, 0) != 0;
        last_layer = pd.get(2, 0) != 0;
        shifted = pd.get(3, 0) != 0;
        dim = pd.get(4, 2560);
        heads = pd.get(5, 20);
        head_dim = pd.get(6, 128);
        mlp_hidden = pd.get(7, 6912);
        eps = pd.get(8, 1e-5f);
        if (dim != heads * head_dim) return -1;
        release();
        return track(s2_dit_block_create(device_, block_index, shared_weights, last_layer, shifted, dim, heads,
                                         head_dim, mlp_hidden, eps, 0, 0, 0, &block_));
    }

    // Per branch (video, then text unless shared): attn shift / scale / gate,
    // mlp shift / scale / gate [dim]; qkv W [3 dim x dim]; proj W [dim x dim] + b
    // [dim]; norm_q, norm_k [head_dim]; SwiGLU gate W, in W [mlp x dim]; out W
    // [dim x mlp]; then the 21 RoPE frequencies. -100 if the stream runs out.
    int load_model(const ModelBin &mb)
    {
        if (!block_) return -1;
        std::vector<float> stream;
        stream.reserve(s2_dit_block_weight_count(block_));
        auto take = [&](int n) {
            const Mat m = mb.load(n, 0);
            if (m.empty()) return false;
            const float *p = m;
            stream.insert(stream.end(), p, p + n);
            return true;
        };
        const int branches = shared_weights ? 1 : 2;
        for (int b = 0; b < branches; ++b) {
            for (int k = 0; k < 6; ++k)
                if (!take(dim)) return -100;
            if (!take(3 * dim * dim) || !take(dim * dim) || !take(dim) || !take(head_dim) || !take(head_dim) ||
                !take(mlp_hidden * dim) || !take(mlp_hidden * dim) || !take(dim * mlp_hidden))
                return -100;
        }
        if (!take(21)) return -100;
        return track(s2_dit_block_load(block_, stream.data(), stream.size()));
    }

    void set_runtime_shape(int frames, int height, int width)
    {
        if (block_) track(s2_dit_block_set_runtime_shape(block_, frames, height, width));
    }

    // bottom = {vid [L x dim], txt [Lt x dim], emb [6 dim], vid_shape int32 [3]},
    // top = 2 blobs, filled with vid_out [L x dim] and txt_out [Lt x dim].
    int forward(const std::vector<Mat> &bottom, std::vector<Mat> &top, const Option &opt) const
    {
        if (!block_) return -1;
        if (bottom.size() != 4 || top.size() != 2) return fail(-1, "blob count mismatch");
        const Mat &vid = bottom[0], &txt = bottom[1], &emb = bottom[2], &shape = bottom[3];
        if (vid.dims != 2 || txt.dims != 2 || vid.w != dim || txt.w != dim ||
            static_cast<int>(emb.total()) != dim * 6 || shape.dims != 1 || shape.w != 3)
            return fail(-1, "invalid input shapes");
        top[0].create(dim, vid.h);
        top[1].create(dim, txt.h);
        if (debug_) {
            // set_debug_tensors: size the capture Mats for this forward and hand them to the library
            const int32_t *sh = static_cast<const int32_t *>(shape);
            int rows = 0;
            s2_status s = s2_dit_block_set_runtime_shape(block_, sh[0], sh[1], sh[2]);
            if (s == S2_OK) s = s2_dit_block_debug_rows(block_, txt.h, &rows);
            if (s != S2_OK) return track(s);
            SeedVR2DiTBlockDebugTensors &t = *debug_;
            const int L = vid.h, Lt = txt.h;
            Mat *m[14] = {&t.qkv_vid, &t.qkv_txt, &t.norm_q_vid, &t.norm_q_txt, &t.norm_k_vid, &t.norm_k_txt,
                          &t.attention_q, &t.attention_k, &t.attention_v, &t.attention_output, &t.projected_vid,
                          &t.projected_txt, &t.output_vid, &t.output_txt};
            const int h[14] = {L, Lt, L, Lt, L, Lt, rows, rows, rows, rows, L, Lt, L, Lt};
            s2_block_debug dbg;
            float **p = reinterpret_cast<float **>(&dbg);
            for (int i = 0; i < 14; ++i) {
                m[i]->create(i < 2 ? 3 * dim : dim, h[i]);
                p[i] = static_cast<float *>(*m[i]);
            }
            s2_dit_block_set_debug_tensors_host(block_, &dbg);
        }
        const int rc = track(s2_dit_block_forward_host(block_, opt.stream, vid, vid.h, txt, txt.h, emb,
                                                       static_cast<const int32_t *>(shape), top[0], top[1]));
        if (debug_) s2_dit_block_set_debug_tensors_host(block_, nullptr);
        return rc;
    }

    // Only for stage-by-stage numerical comparison; the tensors must outlive the
    // forwards that fill them (seedvr2_dit_block.h:58).
    void set_debug_tensors(SeedVR2DiTBlockDebugTensors *tensors) { debug_ = tensors; }

    // The same on device buffers (fp32, row-major), stream-ordered.
    int forward_device(const float *vid, int L, const float *txt, int Lt, const float *emb, float *vid_out,
                       float *txt_out, const Option &opt) const
    {
        if (!block_) return -1;
        return track(s2_dit_block_forward(block_, opt.stream, vid, L, txt, Lt, emb, vid_out, txt_out));
    }

    const std::string &last_error() const { return error_; }

    int block_index = 0;
    bool shared_weights = false, last_layer = false, shifted = false;
    int dim = 2560, heads = 20, head_dim = 128, mlp_hidden = 6912;
    float eps = 1e-5f;

private:
    int device_;
    s2_dit_block *block_ = nullptr;
    SeedVR2DiTBlockDebugTensors *debug_ = nullptr;
    mutable std::string error_;

    int track(s2_status s) const
    {
        if (s != S2_OK) error_ = s2_last_error();
        return reference_code(s);
    }
    int fail(int code, const char *msg) const
    {
        error_ = msg;
        return code;
    }
    void release()
    {
        if (block_) s2_dit_block_destroy(block_);
        block_ = nullptr;
    }
};

// ---- DynamicFramewiseSpatialAttention ----------------------------------------------

class DynamicFramewiseSpatialAttention
{
public:
    explicit DynamicFramewiseSpatialAttention(int device = 0) : device_(device) {}
    ~DynamicFramewiseSpatialAttention() { release(); }
    DynamicFramewiseSpatialAttention(const DynamicFramewiseSpatialAttention &) = delete;
    DynamicFramewiseSpatialAttention &operator=(const DynamicFramewiseSpatialAttention &) = delete;

    // key 10: an int array whose first value is the channel count (a multiple
    // of 32, the GroupNorm's groups); -1 otherwise.
    int load_param(const ParamDict &pd)
    {
        const Mat shape = pd.get(10, Mat());
        if (shape.empty()) return -1;
        channels = static_cast<const int *>(shape)[0];
        if (channels <= 0 || channels % 32 != 0) return -1;
        release();
        return track(s2_vae_attention_create(device_, channels, &layer_));
    }

    // norm_bias, norm_weight, k_bias, k_weight, out_bias, out_weight, q_bias,
    // q_weight, v_bias, v_weight (weights [out][in] = C x C); -100 if the stream
    // runs out.
    int load_model(const ModelBin &mb)
    {
        if (!layer_) return -1;
        const int m = channels * channels;
        Mat w[10];
        const int sizes[10] = {channels, channels, channels, m, channels, m, channels, m, channels, m};
        for (int i = 0; i < 10; ++i) {
            w[i] = mb.load(sizes[i], 1);
            if (w[i].empty()) return -100;
        }
        return track(s2_vae_attention_load(layer_, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7], w[8], w[9]));
    }

    // bottom: w = W, h = H, d = T frames, c = channels (cstep-padded channels);
    // top gets the same shape: x + out_proj(attention(GroupNorm(x))).
    int forward(const Mat &bottom, Mat &top, const Option &opt) const
    {
        if (!layer_) return -1;
        if (bottom.dims != 4 || bottom.c != channels) return fail(-1, "invalid input blob");
        top.create(bottom.w, bottom.h, bottom.d, bottom.c);
        if (top.cstep != bottom.cstep) return fail(-1, "unexpected channel step");
        return track(s2_vae_attention_forward_host(layer_, opt.stream, bottom, bottom.d, bottom.h, bottom.w,
                                                   static_cast<long long>(bottom.cstep), top));
    }

    const std::string &last_error() const { return error_; }

    int channels = 0;

private:
    int device_;
    s2_vae_attention *layer_ = nullptr;
    mutable std::string error_;

    int track(s2_status s) const
    {
        if (s != S2_OK) error_ = s2_last_error();
        return reference_code(s);
    }
    int fail(int code, const char *msg) const
    {
        error_ = msg;
        return code;
    }
    void release()
    {
        if (layer_) s2_vae_attention_destroy(layer_);
        layer_ = nullptr;
    }
};

}  // namespace s2b200
