/* TEST INFRASTRUCTURE ONLY -- the CPU oracle for the SeedVR2 windowed
 * MM-attention hot path. Used by tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg as the checker; never linked into or called by the product.
 *
 * A plain-C restatement of the reference's CPU algorithm (czwdysj/seedvr2-ncnn-valkan):
 *   s2o_make_windows      <- SeedVR2DiTBlock::make_windows  src/layers/seedvr2_dit_block.cpp:827-868
 *   s2o_window_attention  <- SeedVR2DiTBlock::attention     src/layers/seedvr2_dit_block.cpp:870-1091
 *                            (bf16 RNE helper :68-79)
 *   s2o_vae_attention     <- DynamicFramewiseSpatialAttention::forward
 *                            src/layers/dynamic_framewise_spatial_attention.cpp:79-210
 *   s2o_sampler_*         <- EulerSampler (timesteps, apply_cfg, step_to, endpoint)
 *                            src/model/sampler.cpp:19-62, 181-286
 *   s2o_group_norm        <- DynamicFramewiseGroupNorm::forward
 *                            src/layers/dynamic_framewise_group_norm.cpp:63-121
 *   s2o_space_time_shuffle<- DynamicSpaceTimeShuffle::forward
 *                            src/layers/dynamic_space_time_shuffle.cpp:65-130
 *   s2o_conv3d            <- ncnn's Convolution3D as the reference patches it
 *                            (patches/0001-feat-Convolution3D-Vulkan-pack1.patch:
 *                            the shader's stated formula and loop order, :17-25,
 *                            :87-127, SAME padding :240-265). ncnn itself is not
 *                            vendored, so this one is a restatement only.
 *   s2o_condition_ratio / s2o_make_condition
 *                         <- transformed_condition_timestep / make_condition_latent
 *                            src/core/engine.cpp:79-121 (restated only: engine.cpp
 *                            is not part of the reference build under oracle/_ref)
 * Every float/double conversion point follows the reference so that, built with
 * the same flags as oracle/_ref (the reference's own code), results match bit
 * for bit; tests/test_oracle.py pins this against tests/golden/.
 */
#ifndef S2_ORACLE_H
#define S2_ORACLE_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Window boxes {t0,t1,h0,h1,w0,w1}. wt/wh/ww > 0 override the reference's
 * resolution-adaptive window size (an extension used for BASELINE.json's
 * explicit geometries); 0,0,0 = reference rule. Returns the window count;
 * writes at most `cap` windows. */
int s2o_make_windows(int frames, int height, int width, int shifted,
                     int wt, int wh, int ww, int *out, int cap);

/* bf16 round-to-nearest-even, kept in fp32 (reference :68-79). */
float s2o_round_bf16(float x);

/* The attention() path. vid_qkv [L][3*heads*128], txt_qkv [Lt][3*heads*128].
 *   round_out   1 = bf16-round each window output (reference CPU, :1074);
 *               0 = keep fp32 (reference Vulkan shader, :416-436).
 *   head_begin/head_end: compute heads [head_begin, head_end) only.
 *   window_mask: NULL = all windows, else nonzero entries select windows
 *               (text is then summed over the selected windows only, still
 *               divided by the total window count).
 *   vid_out [L][dim] and txt_out [Lt][dim] are fully overwritten (zeros where
 *   not computed). packed_{q,k,v,o} (optional) receive the reference's debug
 *   capture layout [sum_w (L_w+Lt)][dim]. Returns 0, or -1 on bad shapes. */
int s2o_window_attention(const float *vid_qkv, int L, const float *txt_qkv, int Lt,
                         int frames, int height, int width, int heads, int shifted,
                         int wt, int wh, int ww, float eps,
                         const float *norm_q_vid, const float *norm_k_vid,
                         const float *norm_q_txt, const float *norm_k_txt,
                         const float *freqs21, int round_out,
                         int head_begin, int head_end, const unsigned char *window_mask,
                         int num_threads,
                         float *vid_out, float *txt_out,
                         float *packed_q, float *packed_k, float *packed_v, float *packed_o);

/* VAE mid-block spatial attention; x, y dense [C][T][H][W]. Weights as the
 * reference's load_model order. frame_begin/frame_end select frames (others
 * of y untouched). Returns 0 or -1. */
int s2o_vae_attention(int channels, int frames, int height, int width,
                      const float *norm_bias, const float *norm_weight,
                      const float *k_bias, const float *k_weight,
                      const float *out_bias, const float *out_weight,
                      const float *q_bias, const float *q_weight,
                      const float *v_bias, const float *v_weight,
                      const float *x, int frame_begin, int frame_end, int num_threads, float *y);

/* The same layer for the query tokens tokens_sel[0..n_sel) of one frame only
 * (full GroupNorm statistics and K/V); y_sel [n_sel][C]. Returns 0 or -1. */
int s2o_vae_attention_tokens(int channels, int frames, int height, int width,
                             const float *norm_bias, const float *norm_weight,
                             const float *k_bias, const float *k_weight,
                             const float *out_bias, const float *out_weight,
                             const float *q_bias, const float *q_weight,
                             const float *v_bias, const float *v_weight,
                             const float *x, int frame, const int *tokens_sel, int n_sel, int num_threads,
                             float *y_sel);

/* Sampler on fp32 tensors of n elements, summed / transformed in storage
 * order (the reference walks channel, frame, row, x of a dense 4D Mat, which is
 * the same order). */
void s2o_sampler_timesteps(int steps, float *timesteps);
void s2o_apply_cfg(const float *positive, const float *negative, size_t n, float scale, float rescale, float *output);
void s2o_euler_step_to(const float *prediction, const float *current, size_t n, float timestep, float next_timestep,
                       float *output);
void s2o_euler_endpoint(const float *prediction, const float *current, size_t n, float timestep, float *output);
float s2o_condition_ratio(float noise_scale, int latent_frames, int latent_height, int latent_width);
void s2o_make_condition(const float *encoded, const float *noise, size_t n, float ratio, float *output);

/* VAE layers on [C][T][H][W] fp32 blobs (no cstep padding). */
int s2o_group_norm(int channels, int frames, int height, int width, const float *bias, const float *weight,
                   const float *x, int num_threads, float *y);
/* y: [in_channels][T'][2H][2W], T' = T * tr - 1 when tr = projected / in / 4 > 1, else T. */
int s2o_space_time_shuffle(int in_channels, int projected_channels, int frames, int height, int width,
                           const float *bias, const float *weight, const float *x, int num_threads, float *y);
/* Convolution3D: weight [out][in][kd][kh][kw], bias [out] or NULL; pads
 * (front, top, left, behind, bottom, right) >= 0; out-of-range taps read
 * pad_value. Returns the output extents in *od, *oh, *ow (y may be NULL to
 * query them), or -1 on bad arguments. */
int s2o_conv3d(int in_channels, int frames, int height, int width, int out_channels, int kd, int kh, int kw,
               int sd, int sh, int sw, int dd, int dh, int dw, int pad_front, int pad_top, int pad_left,
               int pad_behind, int pad_bottom, int pad_right, float pad_value, const float *bias,
               const float *weight, const float *x, int num_threads, float *y, int *od, int *oh, int *ow);

#ifdef __cplusplus
}
#endif
#endif
