// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// Minimal stand-in for ncnn's `layer.h` (Layer base class, layer creator
// macro, create_layer) so the reference's CPU layer sources compile unmodified.
// `create_layer("InnerProduct")` returns the shim's own fp32 InnerProduct
// (y = W x + b, W stored [out][in]); its results are NOT ncnn's and are
// therefore parity-unpinned.
#pragma once

#include <string>
#include <vector>

#include "mat.h"

namespace ncnn {

class Layer
{
public:
    Layer() : one_blob_only(false), support_inplace(false), support_vulkan(false), support_packing(false),
              support_bf16_storage(false), support_fp16_storage(false), support_vulkan_packing(false) {}
    virtual ~Layer() {}

    virtual int load_param(const ParamDict&) { return 0; }
    virtual int load_model(const ModelBin&) { return 0; }
    virtual int create_pipeline(const Option&) { return 0; }
    virtual int destroy_pipeline(const Option&) { return 0; }

    virtual int forward(const std::vector<Mat>& bottom_blobs, std::vector<Mat>& top_blobs, const Option& opt) const
    {
        if (!one_blob_only || bottom_blobs.size() != 1 || top_blobs.size() != 1) return -1;
        return forward(bottom_blobs[0], top_blobs[0], opt);
    }
    virtual int forward(const Mat&, Mat&, const Option&) const { return -1; }

    bool one_blob_only;
    bool support_inplace;
    bool support_vulkan;
    bool support_packing;
    bool support_bf16_storage;
    bool support_fp16_storage;
    bool support_vulkan_packing;
    std::string type;
    std::string name;
};

typedef Layer* (*layer_creator_func)(void*);

// Only "InnerProduct" is provided.
Layer* create_layer(const char* type);

} // namespace ncnn

#define DEFINE_LAYER_CREATOR(name)                          \
    ::ncnn::Layer* name##_layer_creator(void* /*userdata*/) \
    {                                                       \
        return new name;                                    \
    }
