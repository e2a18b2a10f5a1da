// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// The shim's InnerProduct: ncnn's documented semantics (param 0 = num_output,
// 1 = bias_term, 2 = weight_data_size; weights [out][in] then bias; a 2-D input
// whose width equals num_input is processed row by row). Accumulation is fp32
// in input order; ncnn's own GEMM kernels differ, so results through this
// layer are parity-unpinned against real ncnn.
#include "layer.h"

#include <immintrin.h>

#include <algorithm>
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
        // A packed copy for the tiled loop: [num_output / 32][in][32], so that one
        // 32-output block streams contiguously over the inputs.
        const int num_input = weight_data_size / num_output;
        const int col_blocks = num_output / 32;
        weight_p.create(32 * num_input * (col_blocks > 0 ? col_blocks : 1));
        const float* w = weight;
        for (int cb = 0; cb < col_blocks; cb++)
            for (int i = 0; i < num_input; i++)
                for (int k = 0; k < 32; k++)
                    ((float*)weight_p.data)[((size_t)cb * num_input + i) * 32 + k] = w[(size_t)(cb * 32 + k) * num_input + i];
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
        const float* xin = (const float*)in.data;
        float* yout = (float*)out.data;
        // Tiles of kRows rows x 32 outputs whose partial sums stay in registers
        // over the whole input loop. Each output starts from its bias and adds
        // wt[i][k] * x[i] for i = 0 .. in-1 in order with one rounded multiply
        // and one rounded add per term (no FMA), the same arithmetic as a plain
        // row-at-a-time loop, bit for bit.
        const int kRows = 3, kCols = 32, kChunk = 24;  // kChunk rows per task (a multiple of kRows)
        const int col_blocks = num_output / kCols, row_chunks = (rows + kChunk - 1) / kChunk;
#pragma omp parallel for num_threads(opt.num_threads) schedule(dynamic)
        for (int t = 0; t < col_blocks * row_chunks; t++)
        {
            const int k0 = (t % col_blocks) * kCols, y_end = std::min(rows, (t / col_blocks) * kChunk + kChunk);
            int y = (t / col_blocks) * kChunk;
            for (; y + kRows <= y_end; y += kRows)
                tile<kRows>(xin + (size_t)y * num_input, num_input, k0, b, yout + (size_t)y * num_output, num_output);
            for (; y < y_end; y++)
                tile<1>(xin + (size_t)y * num_input, num_input, k0, b, yout + (size_t)y * num_output, num_output);
        }
        // outputs past the last full 32-column block (num_output % 32)
        const int kt = col_blocks * kCols;
        if (kt < num_output)
        {
#pragma omp parallel for num_threads(opt.num_threads)
            for (int y = 0; y < rows; y++)
            {
                const float* x = xin + (size_t)y * num_input;
                float* o = yout + (size_t)y * num_output;
                for (int k = kt; k < num_output; k++)
                {
                    const float* wk = (const float*)weight + (size_t)k * num_input;
                    float s = b ? b[k] : 0.f;
                    for (int i = 0; i < num_input; i++) s += wk[i] * x[i];
                    o[k] = s;
                }
            }
        }
        return 0;
    }

private:
    // R rows x 32 outputs starting at column k0: 4R vectors of 8 partial sums
    // held in registers across the input loop (AVX2 multiply, then add).
    template <int R>
    void tile(const float* x, int num_input, int k0, const float* b, float* y, int num_output) const
    {
        __m256 acc[R][4];
        for (int r = 0; r < R; r++)
            for (int v = 0; v < 4; v++) acc[r][v] = b ? _mm256_loadu_ps(b + k0 + 8 * v) : _mm256_setzero_ps();
        for (int i = 0; i < num_input; i++)
        {
            const float* wt = (const float*)weight_p.data + ((size_t)(k0 / 32) * num_input + i) * 32;
            const __m256 w0 = _mm256_loadu_ps(wt), w1 = _mm256_loadu_ps(wt + 8), w2 = _mm256_loadu_ps(wt + 16),
                         w3 = _mm256_loadu_ps(wt + 24);
            for (int r = 0; r < R; r++)
            {
                const __m256 xi = _mm256_broadcast_ss(x + (size_t)r * num_input + i);
                acc[r][0] = _mm256_add_ps(acc[r][0], _mm256_mul_ps(w0, xi));
                acc[r][1] = _mm256_add_ps(acc[r][1], _mm256_mul_ps(w1, xi));
                acc[r][2] = _mm256_add_ps(acc[r][2], _mm256_mul_ps(w2, xi));
                acc[r][3] = _mm256_add_ps(acc[r][3], _mm256_mul_ps(w3, xi));
            }
        }
        for (int r = 0; r < R; r++)
            for (int v = 0; v < 4; v++) _mm256_storeu_ps(y + (size_t)r * num_output + k0 + 8 * v, acc[r][v]);
    }

    int num_output = 0;
    int bias_term = 0;
    int weight_data_size = 0;
    Mat weight;
    Mat weight_p;
    Mat bias;
};

} // namespace

Layer* create_layer(const char* type)
{
    if (type && std::strcmp(type, "InnerProduct") == 0) return new ShimInnerProduct;
    return nullptr;
}

} // namespace ncnn
