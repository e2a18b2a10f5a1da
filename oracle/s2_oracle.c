/* TEST INFRASTRUCTURE ONLY -- CPU oracle (plain C restatement) of the
 * reference's hot path. See s2_oracle.h for the function-by-function map to
 * the reference sources. Never part of the product path. */
#include "s2_oracle.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define S2O_HEAD_DIM 128
#define S2O_ROPE_PAIRS 21

static int ceil_div_i(int a, int b) { return (a + b - 1) / b; }
static int min_i(int a, int b) { return a < b ? a : b; }
static int max_i(int a, int b) { return a > b ? a : b; }

float s2o_round_bf16(float x)
{
    /* round-to-nearest-even on the upper 16 bits (seedvr2_dit_block.cpp:68-79) */
    uint32_t bits;
    memcpy(&bits, &x, sizeof bits);
    bits += 0x7fffu + ((bits >> 16) & 1u);
    bits &= 0xffff0000u;
    memcpy(&x, &bits, sizeof x);
    return x;
}

/* seedvr2_dit_block.cpp:827-868 */
int s2o_make_windows(int frames, int height, int width, int shifted,
                     int wt, int wh, int ww, int *out, int cap)
{
    if (frames <= 0 || height <= 0 || width <= 0) return 0;
    int win_t, win_h, win_w;
    if (wt > 0 && wh > 0 && ww > 0) {
        win_t = wt; win_h = wh; win_w = ww;
    } else {
        /* grid resized to a ~3600-token footprint, split into thirds; the
         * temporal window is a quarter of (at most 30) frames */
        const double scale = sqrt(3600.0 / (double)(height * width));
        const int rh = (int)nearbyint(height * scale);
        const int rw = (int)nearbyint(width * scale);
        win_h = ceil_div_i(rh, 3);
        win_w = ceil_div_i(rw, 3);
        win_t = ceil_div_i(min_i(frames, 30), 4);
    }
    const double st = shifted && win_t < frames ? 0.5 : 0.0;
    const double sh = shifted && win_h < height ? 0.5 : 0.0;
    const double sw = shifted && win_w < width ? 0.5 : 0.0;
    const int nt = shifted ? (st > 0.0 ? (int)ceil((frames - st) / win_t) + 1 : 1) : ceil_div_i(frames, win_t);
    const int nh = shifted ? (sh > 0.0 ? (int)ceil((height - sh) / win_h) + 1 : 1) : ceil_div_i(height, win_h);
    const int nw = shifted ? (sw > 0.0 ? (int)ceil((width - sw) / win_w) + 1 : 1) : ceil_div_i(width, win_w);

    int count = 0;
    /* w outermost, t innermost */
    for (int iw = 0; iw < nw; iw++)
        for (int ih = 0; ih < nh; ih++)
            for (int it = 0; it < nt; it++) {
                const int t0 = max_i((int)((it - st) * win_t), 0);
                const int t1 = min_i((int)((it - st + 1.0) * win_t), frames);
                const int h0 = max_i((int)((ih - sh) * win_h), 0);
                const int h1 = min_i((int)((ih - sh + 1.0) * win_h), height);
                const int w0 = max_i((int)((iw - sw) * win_w), 0);
                const int w1 = min_i((int)((iw - sw + 1.0) * win_w), width);
                if (t1 > t0 && h1 > h0 && w1 > w0) {
                    if (count < cap && out) {
                        int *o = out + 6 * count;
                        o[0] = t0; o[1] = t1; o[2] = h0; o[3] = h1; o[4] = w0; o[5] = w1;
                    }
                    count++;
                }
            }
    return count;
}

/* Per-head QK-RMSNorm * gamma, then MM-RoPE over 3 axes x 21 pairs (dims
 * 0..125), then bf16 rounding (seedvr2_dit_block.cpp:942-974). */
static void norm_rope_round(const float *src, const float *gamma, float *dst,
                            int pt, int ph, int pw, float eps, const float *freqs)
{
    double ss = 0.0;
    for (int d = 0; d < S2O_HEAD_DIM; d++) ss += (double)src[d] * src[d];
    const float inv = 1.f / sqrtf((float)(ss / S2O_HEAD_DIM) + eps);
    for (int d = 0; d < S2O_HEAD_DIM; d++) dst[d] = src[d] * inv * gamma[d];
    const int pos[3] = {pt, ph, pw};
    for (int axis = 0; axis < 3; axis++)
        for (int p = 0; p < S2O_ROPE_PAIRS; p++) {
            const int d = axis * 2 * S2O_ROPE_PAIRS + 2 * p;
            const float angle = pos[axis] * freqs[p];
            const float c = cosf(angle);
            const float s = sinf(angle);
            const float a = dst[d];
            const float b = dst[d + 1];
            dst[d] = a * c - b * s;
            dst[d + 1] = b * c + a * s;
        }
    for (int d = 0; d < S2O_HEAD_DIM; d++) dst[d] = s2o_round_bf16(dst[d]);
}

int s2o_window_attention(const float *vid_qkv, int L, const float *txt_qkv, int Lt,
                         int frames, int height, int width, int heads, int shifted,
                         int wt, int wh, int ww, float eps,
                         const float *norm_q_vid, const float *norm_k_vid,
                         const float *norm_q_txt, const float *norm_k_txt,
                         const float *freqs21, int round_out,
                         int head_begin, int head_end, const unsigned char *window_mask,
                         int num_threads,
                         float *vid_out, float *txt_out,
                         float *packed_q, float *packed_k, float *packed_v, float *packed_o)
{
    const int hd = S2O_HEAD_DIM;
    const int dim = heads * hd;
    if (frames * height * width != L || L <= 0 || Lt < 0 || heads <= 0) return -1;
    if (head_begin < 0) head_begin = 0;
    if (head_end <= 0 || head_end > heads) head_end = heads;
    const int nwin = s2o_make_windows(frames, height, width, shifted, wt, wh, ww, NULL, 0);
    if (nwin <= 0) return -1;
    int *win = (int *)malloc(sizeof(int) * 6 * (size_t)nwin);
    int *seq_off = (int *)malloc(sizeof(int) * (size_t)nwin);
    s2o_make_windows(frames, height, width, shifted, wt, wh, ww, win, nwin);
    int total_rows = 0;
    for (int w = 0; w < nwin; w++) {
        const int *b = win + 6 * w;
        seq_off[w] = total_rows;
        total_rows += (b[1] - b[0]) * (b[3] - b[2]) * (b[5] - b[4]) + Lt;
    }
    memset(vid_out, 0, sizeof(float) * (size_t)L * dim);
    memset(txt_out, 0, sizeof(float) * (size_t)Lt * dim);
    const float scale = 1.f / sqrtf((float)hd);
    const float inv_nwin = 1.f / (float)nwin;

#pragma omp parallel for num_threads(num_threads > 0 ? num_threads : 1) schedule(dynamic, 1)
    for (int head = head_begin; head < head_end; head++) {
        float *txt_acc = (float *)calloc((size_t)(Lt > 0 ? Lt : 1) * hd, sizeof(float));
        for (int w = 0; w < nwin; w++) {
            if (window_mask && !window_mask[w]) continue;
            const int *b = win + 6 * w;
            const int lt = b[1] - b[0], lh = b[3] - b[2], lw = b[5] - b[4];
            const int Lw = lt * lh * lw;
            const int S = Lw + Lt;
            float *q = (float *)malloc(sizeof(float) * (size_t)S * hd);
            float *k = (float *)malloc(sizeof(float) * (size_t)S * hd);
            float *v = (float *)malloc(sizeof(float) * (size_t)S * hd);
            float *sc = (float *)malloc(sizeof(float) * (size_t)S);
            int *vidx = (int *)malloc(sizeof(int) * (size_t)(Lw > 0 ? Lw : 1));
            int row = 0;
            /* video tokens in t, y, x order; RoPE position (Lt + t - t0, y - h0, x - w0) */
            for (int t = b[0]; t < b[1]; t++)
                for (int y = b[2]; y < b[3]; y++)
                    for (int x = b[4]; x < b[5]; x++, row++) {
                        const int g = (t * height + y) * width + x;
                        vidx[row] = g;
                        const float *src = vid_qkv + (size_t)g * 3 * dim;
                        norm_rope_round(src + head * hd, norm_q_vid, q + (size_t)row * hd,
                                        Lt + (t - b[0]), y - b[2], x - b[4], eps, freqs21);
                        norm_rope_round(src + dim + head * hd, norm_k_vid, k + (size_t)row * hd,
                                        Lt + (t - b[0]), y - b[2], x - b[4], eps, freqs21);
                        for (int d = 0; d < hd; d++)
                            v[(size_t)row * hd + d] = s2o_round_bf16(src[2 * dim + head * hd + d]);
                    }
            /* text tokens at RoPE position (l, l, l) */
            for (int l = 0; l < Lt; l++, row++) {
                const float *src = txt_qkv + (size_t)l * 3 * dim;
                norm_rope_round(src + head * hd, norm_q_txt, q + (size_t)row * hd, l, l, l, eps, freqs21);
                norm_rope_round(src + dim + head * hd, norm_k_txt, k + (size_t)row * hd, l, l, l, eps, freqs21);
                for (int d = 0; d < hd; d++)
                    v[(size_t)row * hd + d] = s2o_round_bf16(src[2 * dim + head * hd + d]);
            }
            if (packed_q || packed_k || packed_v)
                for (int r = 0; r < S; r++) {
                    const size_t o = (size_t)(seq_off[w] + r) * dim + (size_t)head * hd;
                    if (packed_q) memcpy(packed_q + o, q + (size_t)r * hd, sizeof(float) * hd);
                    if (packed_k) memcpy(packed_k + o, k + (size_t)r * hd, sizeof(float) * hd);
                    if (packed_v) memcpy(packed_v + o, v + (size_t)r * hd, sizeof(float) * hd);
                }
            /* softmax(q k^T * scale) v with double dots (seedvr2_dit_block.cpp:1045-1079) */
            for (int qi = 0; qi < S; qi++) {
                const float *qr = q + (size_t)qi * hd;
                float mx = -INFINITY;
                for (int ki = 0; ki < S; ki++) {
                    const float *kr = k + (size_t)ki * hd;
                    double dot = 0.0;
                    for (int d = 0; d < hd; d++) dot += (double)qr[d] * kr[d];
                    sc[ki] = (float)dot * scale;
                    if (sc[ki] > mx) mx = sc[ki];
                }
                float den = 0.f;
                for (int ki = 0; ki < S; ki++) {
                    sc[ki] = expf(sc[ki] - mx);
                    den += sc[ki];
                }
                float *dst = qi < Lw ? vid_out + (size_t)vidx[qi] * dim + (size_t)head * hd
                                     : txt_acc + (size_t)(qi - Lw) * hd;
                for (int d = 0; d < hd; d++) {
                    double acc = 0.0;
                    for (int ki = 0; ki < S; ki++) acc += (double)(sc[ki] / den) * v[(size_t)ki * hd + d];
                    const float o = round_out ? s2o_round_bf16((float)acc) : (float)acc;
                    dst[d] += o;
                    if (packed_o) packed_o[(size_t)(seq_off[w] + qi) * dim + (size_t)head * hd + d] = o;
                }
            }
            free(q); free(k); free(v); free(sc); free(vidx);
        }
        /* text output = window sum x 1/nwin (seedvr2_dit_block.cpp:1081-1088) */
        for (int l = 0; l < Lt; l++)
            for (int d = 0; d < hd; d++)
                txt_out[(size_t)l * dim + (size_t)head * hd + d] = txt_acc[(size_t)l * hd + d] * inv_nwin;
        free(txt_acc);
    }
    free(win);
    free(seq_off);
    return 0;
}

/* dynamic_framewise_spatial_attention.cpp:79-104: y = W x + b, double accumulation */
static void vae_linear(const float *in, float *out, const float *w, const float *b, int tokens, int c,
                       int num_threads)
{
#pragma omp parallel for num_threads(num_threads > 0 ? num_threads : 1)
    for (int t = 0; t < tokens; t++) {
        const float *xr = in + (size_t)t * c;
        float *yr = out + (size_t)t * c;
        for (int o = 0; o < c; o++) {
            const float *wr = w + (size_t)o * c;
            double acc = b[o];
            for (int i = 0; i < c; i++) acc += (double)xr[i] * wr[i];
            yr[o] = (float)acc;
        }
    }
}

/* dynamic_framewise_spatial_attention.cpp:106-210 */
int s2o_vae_attention(int channels, int frames, int height, int width,
                      const float *norm_bias, const float *norm_weight,
                      const float *k_bias, const float *k_weight,
                      const float *out_bias, const float *out_weight,
                      const float *q_bias, const float *q_weight,
                      const float *v_bias, const float *v_weight,
                      const float *x, int frame_begin, int frame_end, int num_threads, float *y)
{
    if (channels <= 0 || channels % 32 != 0 || frames <= 0 || height <= 0 || width <= 0) return -1;
    if (frame_begin < 0) frame_begin = 0;
    if (frame_end <= 0 || frame_end > frames) frame_end = frames;
    const int tokens = height * width;
    const int cpg = channels / 32;
    const float scale = 1.f / sqrtf((float)channels);
    const size_t plane = (size_t)frames * tokens; /* per-channel stride of x/y */
    const size_t n = (size_t)tokens * channels;
    float *nrm = (float *)malloc(sizeof(float) * n);
    float *qm = (float *)malloc(sizeof(float) * n);
    float *km = (float *)malloc(sizeof(float) * n);
    float *vm = (float *)malloc(sizeof(float) * n);
    float *att = (float *)malloc(sizeof(float) * n);
    float *prj = (float *)malloc(sizeof(float) * n);
    for (int f = frame_begin; f < frame_end; f++) {
        /* GroupNorm(32, eps 1e-6) per frame into token-major rows */
        for (int g = 0; g < 32; g++) {
            double sum = 0.0, sq = 0.0;
            for (int lc = 0; lc < cpg; lc++) {
                const float *in = x + plane * (size_t)(g * cpg + lc) + (size_t)f * tokens;
                for (int t = 0; t < tokens; t++) {
                    sum += in[t];
                    sq += (double)in[t] * in[t];
                }
            }
            const int count = cpg * tokens;
            const float mean = (float)(sum / count);
            const float var = (float)(sq / count - (double)mean * mean);
            const float inv_std = 1.f / sqrtf((var > 0.f ? var : 0.f) + 1e-6f);
            for (int lc = 0; lc < cpg; lc++) {
                const int c = g * cpg + lc;
                const float *in = x + plane * (size_t)c + (size_t)f * tokens;
                const float sc = norm_weight[c] * inv_std;
                const float off = norm_bias[c] - mean * sc;
                for (int t = 0; t < tokens; t++) nrm[(size_t)t * channels + c] = in[t] * sc + off;
            }
        }
        vae_linear(nrm, qm, q_weight, q_bias, tokens, channels, num_threads);
        vae_linear(nrm, km, k_weight, k_bias, tokens, channels, num_threads);
        vae_linear(nrm, vm, v_weight, v_bias, tokens, channels, num_threads);
        memset(att, 0, sizeof(float) * n);
#pragma omp parallel for num_threads(num_threads > 0 ? num_threads : 1)
        for (int qt = 0; qt < tokens; qt++) {
            float *sc = (float *)malloc(sizeof(float) * (size_t)tokens);
            float mx = -INFINITY;
            for (int kt = 0; kt < tokens; kt++) {
                double s = 0.0;
                for (int c = 0; c < channels; c++)
                    s += (double)qm[(size_t)qt * channels + c] * km[(size_t)kt * channels + c];
                sc[kt] = (float)s * scale;
                if (sc[kt] > mx) mx = sc[kt];
            }
            double den = 0.0;
            for (int kt = 0; kt < tokens; kt++) {
                sc[kt] = expf(sc[kt] - mx);
                den += sc[kt];
            }
            float *orow = att + (size_t)qt * channels;
            for (int kt = 0; kt < tokens; kt++) {
                const float p = (float)(sc[kt] / den);
                const float *vr = vm + (size_t)kt * channels;
                for (int c = 0; c < channels; c++) orow[c] += p * vr[c];
            }
            free(sc);
        }
        vae_linear(att, prj, out_weight, out_bias, tokens, channels, num_threads);
        for (int c = 0; c < channels; c++) {
            const float *res = x + plane * (size_t)c + (size_t)f * tokens;
            float *o = y + plane * (size_t)c + (size_t)f * tokens;
            for (int t = 0; t < tokens; t++) o[t] = prj[(size_t)t * channels + c] + res[t];
        }
    }
    free(nrm); free(qm); free(km); free(vm); free(att); free(prj);
    return 0;
}

/* The same layer evaluated for a subset of query tokens of one frame
 * (dynamic_framewise_spatial_attention.cpp:115-194 restricted to the output
 * rows `tokens_sel`): GroupNorm statistics and the K/V projections cover the
 * whole frame, Q, attention, output projection and residual only the listed
 * tokens. x is dense [C][T][H][W]; y_sel receives [n_sel][C] (token-major).
 * Exists so that full-size frames (14,400 tokens at C = 512) can be checked
 * in seconds. */
int s2o_vae_attention_tokens(int channels, int frames, int height, int width,
                             const float *norm_bias, const float *norm_weight,
                             const float *k_bias, const float *k_weight,
                             const float *out_bias, const float *out_weight,
                             const float *q_bias, const float *q_weight,
                             const float *v_bias, const float *v_weight,
                             const float *x, int frame, const int *tokens_sel, int n_sel, int num_threads,
                             float *y_sel)
{
    if (channels <= 0 || channels % 32 != 0 || frame < 0 || frame >= frames || n_sel <= 0) return -1;
    const int tokens = height * width;
    const int cpg = channels / 32;
    const float scale = 1.f / sqrtf((float)channels);
    const size_t plane = (size_t)frames * tokens;
    const size_t n = (size_t)tokens * channels;
    for (int i = 0; i < n_sel; i++)
        if (tokens_sel[i] < 0 || tokens_sel[i] >= tokens) return -1;
    float *nrm = (float *)malloc(sizeof(float) * n);
    float *km = (float *)malloc(sizeof(float) * n);
    float *vm = (float *)malloc(sizeof(float) * n);
    float *qs = (float *)malloc(sizeof(float) * (size_t)n_sel * channels);
    float *as = (float *)calloc((size_t)n_sel * channels, sizeof(float));
    float *nsel = (float *)malloc(sizeof(float) * (size_t)n_sel * channels);
    float *ps = (float *)malloc(sizeof(float) * (size_t)n_sel * channels);
    for (int g = 0; g < 32; g++) {
        double sum = 0.0, sq = 0.0;
        for (int lc = 0; lc < cpg; lc++) {
            const float *in = x + plane * (size_t)(g * cpg + lc) + (size_t)frame * tokens;
            for (int t = 0; t < tokens; t++) {
                sum += in[t];
                sq += (double)in[t] * in[t];
            }
        }
        const int count = cpg * tokens;
        const float mean = (float)(sum / count);
        const float var = (float)(sq / count - (double)mean * mean);
        const float inv_std = 1.f / sqrtf((var > 0.f ? var : 0.f) + 1e-6f);
        for (int lc = 0; lc < cpg; lc++) {
            const int c = g * cpg + lc;
            const float *in = x + plane * (size_t)c + (size_t)frame * tokens;
            const float sc = norm_weight[c] * inv_std;
            const float off = norm_bias[c] - mean * sc;
            for (int t = 0; t < tokens; t++) nrm[(size_t)t * channels + c] = in[t] * sc + off;
        }
    }
    vae_linear(nrm, km, k_weight, k_bias, tokens, channels, num_threads);
    vae_linear(nrm, vm, v_weight, v_bias, tokens, channels, num_threads);
    for (int i = 0; i < n_sel; i++)
        memcpy(nsel + (size_t)i * channels, nrm + (size_t)tokens_sel[i] * channels, sizeof(float) * channels);
    vae_linear(nsel, qs, q_weight, q_bias, n_sel, channels, num_threads);
#pragma omp parallel for num_threads(num_threads > 0 ? num_threads : 1)
    for (int i = 0; i < n_sel; i++) {
        float *sc = (float *)malloc(sizeof(float) * (size_t)tokens);
        float mx = -INFINITY;
        for (int kt = 0; kt < tokens; kt++) {
            double s = 0.0;
            for (int c = 0; c < channels; c++)
                s += (double)qs[(size_t)i * channels + c] * km[(size_t)kt * channels + c];
            sc[kt] = (float)s * scale;
            if (sc[kt] > mx) mx = sc[kt];
        }
        double den = 0.0;
        for (int kt = 0; kt < tokens; kt++) {
            sc[kt] = expf(sc[kt] - mx);
            den += sc[kt];
        }
        float *orow = as + (size_t)i * channels;
        for (int kt = 0; kt < tokens; kt++) {
            const float p = (float)(sc[kt] / den);
            const float *vr = vm + (size_t)kt * channels;
            for (int c = 0; c < channels; c++) orow[c] += p * vr[c];
        }
        free(sc);
    }
    vae_linear(as, ps, out_weight, out_bias, n_sel, channels, num_threads);
    for (int i = 0; i < n_sel; i++)
        for (int c = 0; c < channels; c++)
            y_sel[(size_t)i * channels + c] =
                ps[(size_t)i * channels + c] + x[plane * (size_t)c + (size_t)frame * tokens + tokens_sel[i]];
    free(nrm); free(km); free(vm); free(qs); free(as); free(nsel); free(ps);
    return 0;
}


/* ---- sampler (src/model/sampler.cpp) ---------------------------------------- */

/* EulerSampler::EulerSampler (sampler.cpp:181-187) */
void s2o_sampler_timesteps(int steps, float *timesteps)
{
    if (steps < 1) steps = 1;
    for (int i = 0; i < steps; i++) timesteps[i] = 1000.0f * (1.0f - (float)i / steps);
}

/* standard_deviation (sampler.cpp:41-62): sequential fp64 sum and sum of squares */
static double sampler_std(const float *v, size_t n)
{
    double sum = 0.0, square_sum = 0.0;
    for (size_t i = 0; i < n; i++) {
        sum += v[i];
        square_sum += (double)v[i] * v[i];
    }
    if (n <= 1) return 0.0;
    double variance = (square_sum - sum * sum / n) / (n - 1);
    if (variance < 0.0) variance = 0.0;
    return sqrt(variance);
}

/* EulerSampler::apply_cfg (sampler.cpp:200-238) */
void s2o_apply_cfg(const float *positive, const float *negative, size_t n, float scale, float rescale, float *output)
{
    for (size_t i = 0; i < n; i++) output[i] = negative[i] + scale * (positive[i] - negative[i]);
    if (rescale != 0.0f) {
        const double cfg_std = sampler_std(output, n);
        if (cfg_std > 0.0) {
            const float factor = (float)(rescale * sampler_std(positive, n) / cfg_std + (1.0f - rescale));
            for (size_t i = 0; i < n; i++) output[i] *= factor;
        }
    }
}

/* EulerSampler::step_to (sampler.cpp:240-265) */
void s2o_euler_step_to(const float *prediction, const float *current, size_t n, float timestep, float next_timestep,
                       float *output)
{
    const float bt = timestep / 1000.0f;
    const float at = 1.0f - bt;
    float bs = next_timestep / 1000.0f;
    bs = bs < 0.0f ? 0.0f : (bs > 1.0f ? 1.0f : bs);
    const float as = 1.0f - bs;
    for (size_t i = 0; i < n; i++) {
        const float x0 = current[i] - bt * prediction[i];
        const float xT = current[i] + at * prediction[i];
        output[i] = as * x0 + bs * xT;
    }
}

/* EulerSampler::endpoint (sampler.cpp:267-286) */
void s2o_euler_endpoint(const float *prediction, const float *current, size_t n, float timestep, float *output)
{
    const float bt = timestep / 1000.0f;
    for (size_t i = 0; i < n; i++) output[i] = current[i] - bt * prediction[i];
}

/* transformed_condition_timestep(noise_scale, latent) / 1000 (engine.cpp:79-92, 108) */
float s2o_condition_ratio(float noise_scale, int latent_frames, int latent_height, int latent_width)
{
    const float timestep = noise_scale * 1000.0f;
    if (timestep == 0.0f) return 0.0f;
    const float frames = (float)((latent_frames - 1) * 4 + 1);
    const float height = (float)(latent_height * 8);
    const float width = (float)(latent_width * 8);
    const float x1 = 256.0f * 256.0f * 37.0f;
    const float x2 = 1280.0f * 720.0f * 145.0f;
    const float shift = 1.0f + (height * width * frames - x1) * (5.0f - 1.0f) / (x2 - x1);
    const float normalized = timestep / 1000.0f;
    return 1000.0f * shift * normalized / (1.0f + (shift - 1.0f) * normalized) / 1000.0f;
}

/* make_condition_latent (engine.cpp:106-121) */
void s2o_make_condition(const float *encoded, const float *noise, size_t n, float ratio, float *output)
{
    for (size_t i = 0; i < n; i++) output[i] = (1.0f - ratio) * encoded[i] + ratio * noise[i];
}

/* ---- VAE layers -------------------------------------------------------- */

/* dynamic_framewise_group_norm.cpp:63-121: per (frame, group of C/32
 * channels) double sums in channel-then-position order, mean and variance
 * rounded to float as there, y = x * scale + offset without contraction. */
int s2o_group_norm(int channels, int frames, int height, int width, const float *bias, const float *weight,
                   const float *x, int num_threads, float *y)
{
    const int groups = 32;
    if (channels <= 0 || channels % groups != 0 || frames <= 0 || height <= 0 || width <= 0) return -1;
    const int cpg = channels / groups;
    const size_t hw = (size_t)height * width, plane = hw * (size_t)frames;
#pragma omp parallel for collapse(2) num_threads(num_threads > 0 ? num_threads : 1)
    for (int f = 0; f < frames; f++)
        for (int g = 0; g < groups; g++) {
            double sum = 0.0, sq = 0.0;
            for (int lc = 0; lc < cpg; lc++) {
                const float *in = x + (size_t)(g * cpg + lc) * plane + (size_t)f * hw;
                for (size_t i = 0; i < hw; i++) {
                    const float v = in[i];
                    sum += v;
                    sq += (double)v * v;
                }
            }
            const int count = cpg * (int)hw;
            const float mean = (float)(sum / count);
            const float var = (float)(sq / count - (double)mean * mean);
            const float inv_std = 1.f / sqrtf((var > 0.f ? var : 0.f) + 1e-6f);
            for (int lc = 0; lc < cpg; lc++) {
                const int c = g * cpg + lc;
                const float *in = x + (size_t)c * plane + (size_t)f * hw;
                float *out = y + (size_t)c * plane + (size_t)f * hw;
                const float scale = weight[c] * inv_std;
                const float offset = bias[c] - mean * scale;
                for (size_t i = 0; i < hw; i++) out[i] = in[i] * scale + offset;
            }
        }
    return 0;
}

/* dynamic_space_time_shuffle.cpp:65-130: 1x1x1 projection accumulated in
 * double from the bias, then projected channel
 * ((oy * 2 + ox) * tr + ot) * Cin + c goes to output channel c at frame
 * f * tr + ot (the duplicated raw frame 1 dropped when tr > 1), row
 * 2 y + oy, column 2 x + ox. */
int s2o_space_time_shuffle(int in_channels, int projected_channels, int frames, int height, int width,
                           const float *bias, const float *weight, const float *x, int num_threads, float *y)
{
    const int sr = 2;
    if (in_channels <= 0 || projected_channels % (in_channels * sr * sr) != 0) return -1;
    const int tr = projected_channels / in_channels / (sr * sr);
    if (tr <= 0) return -1;
    const int out_frames = tr > 1 ? frames * tr - 1 : frames, ow = width * sr, oh = height * sr;
    const size_t hw = (size_t)height * width, in_plane = hw * (size_t)frames;
    const size_t out_plane = (size_t)ow * oh * (size_t)out_frames;
#pragma omp parallel for num_threads(num_threads > 0 ? num_threads : 1)
    for (int oc = 0; oc < in_channels; oc++)
        for (int f = 0; f < frames; f++)
            for (int yy = 0; yy < height; yy++)
                for (int xx = 0; xx < width; xx++)
                    for (int oy = 0; oy < sr; oy++)
                        for (int ox = 0; ox < sr; ox++)
                            for (int ot = 0; ot < tr; ot++) {
                                const int p = ((oy * sr + ox) * tr + ot) * in_channels + oc;
                                const int raw = f * tr + ot;
                                if (tr > 1 && raw == 1) continue;
                                const int of = tr > 1 && raw > 1 ? raw - 1 : raw;
                                const float *wr = weight + (size_t)p * in_channels;
                                double v = bias[p];
                                for (int ic = 0; ic < in_channels; ic++)
                                    v += (double)x[(size_t)ic * in_plane + (size_t)f * hw + (size_t)yy * width + xx] *
                                         wr[ic];
                                y[(size_t)oc * out_plane + (size_t)of * oh * ow + (size_t)(yy * sr + oy) * ow +
                                  (size_t)(xx * sr + ox)] = (float)v;
                            }
    return 0;
}

/* Convolution3D (patch 0001 :17-25): out[p][z][i][j] = bias[p] + sum over
 * input channels q, then taps (kd, kh, kw) in that order, of
 * in[q][z*sd + kd*dd - pad_front][i*sh + kh*dh - pad_top][j*sw + kw*dw - pad_left]
 * * weight[p][q][kd][kh][kw], out-of-range positions reading pad_value; fp32
 * accumulation as the shader's afp sum. */
int s2o_conv3d(int in_channels, int frames, int height, int width, int out_channels, int kd, int kh, int kw,
               int sd, int sh, int sw, int dd, int dh, int dw, int pad_front, int pad_top, int pad_left,
               int pad_behind, int pad_bottom, int pad_right, float pad_value, const float *bias,
               const float *weight, const float *x, int num_threads, float *y, int *od, int *oh, int *ow)
{
    if (in_channels <= 0 || out_channels <= 0 || kd <= 0 || kh <= 0 || kw <= 0 || sd <= 0 || sh <= 0 || sw <= 0 ||
        dd <= 0 || dh <= 0 || dw <= 0 || pad_front < 0 || pad_top < 0 || pad_left < 0 || pad_behind < 0 ||
        pad_bottom < 0 || pad_right < 0)
        return -1;
    const int ed = dd * (kd - 1) + 1, eh = dh * (kh - 1) + 1, ew = dw * (kw - 1) + 1;
    const int D = (frames + pad_front + pad_behind - ed) / sd + 1;
    const int Hh = (height + pad_top + pad_bottom - eh) / sh + 1;
    const int Ww = (width + pad_left + pad_right - ew) / sw + 1;
    if (D <= 0 || Hh <= 0 || Ww <= 0) return -1;
    if (od) *od = D;
    if (oh) *oh = Hh;
    if (ow) *ow = Ww;
    if (!y) return 0;
    const size_t in_plane = (size_t)frames * height * width, out_plane = (size_t)D * Hh * Ww;
    const int maxk = kd * kh * kw;
#pragma omp parallel for num_threads(num_threads > 0 ? num_threads : 1)
    for (int p = 0; p < out_channels; p++)
        for (int z = 0; z < D; z++)
            for (int i = 0; i < Hh; i++)
                for (int j = 0; j < Ww; j++) {
                    float sum = bias ? bias[p] : 0.f;
                    for (int q = 0; q < in_channels; q++) {
                        const float *wq = weight + ((size_t)p * in_channels + q) * maxk;
                        for (int a = 0; a < kd; a++)
                            for (int b = 0; b < kh; b++)
                                for (int c = 0; c < kw; c++) {
                                    const int iz = z * sd + a * dd - pad_front;
                                    const int ih = i * sh + b * dh - pad_top;
                                    const int iw = j * sw + c * dw - pad_left;
                                    float v = pad_value;
                                    if (iz >= 0 && iz < frames && ih >= 0 && ih < height && iw >= 0 && iw < width)
                                        v = x[(size_t)q * in_plane + ((size_t)iz * height + ih) * width + iw];
                                    sum += v * wq[(a * kh + b) * kw + c];
                                }
                    }
                    y[(size_t)p * out_plane + ((size_t)z * Hh + i) * Ww + j] = sum;
                }
    return 0;
}
