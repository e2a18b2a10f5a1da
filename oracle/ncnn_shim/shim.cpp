// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// The shim's InnerProduct: ncnn's documented semantics (param 0 = num_output,
// 1 = bias_term, 2 = weight_data_size; weights [out][in] then bias; a 2-D input
// whose width equals num_input is processed row by row). Accumulation is fp32
// in input order; ncnn's own GEMM kernels differ, so results through this
// layer are parity-unpinned against real ncnn.
#include "layer.h"

#include <cstring>

namespace ncnn {
namespace {

class ShimInnerProduct : public Layer
{
public:
    ShimInnerProduct() { one_blob_only = true; }

    int load_param(const ParamDict& pd) override
    {
        num_output = pd.get(0, 0);
        bias_term = pd.get(1, 0);
        weight_data_size = pd.get(2, 0);
        return num_output > 0 && weight_data_size % num_output == 0 ? 0 : -1;
    }

    int load_model(const ModelBin& mb) override
    {
        weight = mb.load(weight_data_size, 0);
        if (weight.empty()) return -100;
        if (bias_term)
        {
            bias = mb.load(num_output, 1);
            if (bias.empty()) return -100;
        }
        // Keep a transposed copy [in][out] so the inner loop runs over
        // contiguous outputs; the per-output summation order stays i = 0..in-1.
        const int num_input = weight_data_size / num_output;
        weight_t.create(num_output, num_input);
        const float* w = weight;
        for (int o = 0; o < num_output; o++)
            for (int i = 0; i < num_input; i++)
                weight_t.row(i)[o] = w[(size_t)o * num_input + i];
        return 0;
    }

    int forward(const Mat& in, Mat& out, const Option& opt) const override
    {
        const int num_input = weight_data_size / num_output;
        int rows = 1;
        if (in.dims == 2 && in.w == num_input)
            rows = in.h;
        else if ((int)(in.w * in.h) != num_input)
            return -1;
        if (in.dims == 2 && in.w == num_input)
            out.create(num_output, rows, 4u, opt.blob_allocator);
        else
            out.create(num_output, 4u, opt.blob_allocator);
        if (out.empty()) return -100;
        const float* b = bias_term ? (const float*)bias : nullptr;
#pragma omp parallel for num_threads(opt.num_threads)
        for (int y = 0; y < rows; y++)
        {
            const float* x = (const float*)in.data + (size_t)y * num_input;
            float* o = (float*)out.data + (size_t)y * num_output;
            for (int k = 0; k < num_output; k++) o[k] = b ? b[k] : 0.f;
            for (int i = 0; i < num_input; i++)
            {
                const float xi = x[i];
                const float* wt = weight_t.row(i);
                for (int k = 0; k < num_output; k++) o[k] += wt[k] * xi;
            }
        }
        return 0;
    }

private:
    int num_output = 0;
    int bias_term = 0;
    int weight_data_size = 0;
    Mat weight;
    Mat weight_t;
    Mat bias;
};

} // namespace

Layer* create_layer(const char* type)
{
    if (type && std::strcmp(type, "InnerProduct") == 0) return new ShimInnerProduct;
    return nullptr;
}

} // namespace ncnn
