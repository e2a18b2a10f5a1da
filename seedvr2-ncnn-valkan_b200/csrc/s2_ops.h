// Internal helpers shared between the layer objects of libs2b200 (not part of
// the C ABI).
#pragma once

#include <cuda_runtime.h>

#include "s2_b200.h"

namespace s2 {

// Let `dst` use the same activation scratch (packed Q/K/V, text partials /
// block activations) as `src`. Only for objects whose forwards run one after
// another on one stream, like the blocks of one DiT forward.
void share_attention_scratch(s2_attention_layer *dst, const s2_attention_layer *src);
void share_block_scratch(s2_dit_block *dst, const s2_dit_block *src);

// Reduction of a block's text attention output across ranks (a sharded DiT
// step): called between the attention and the output projection with the
// rank's partial text mean [Lt][dim] fp32, stream-ordered on `st`.
struct TextReduce {
    s2_status (*fn)(void *ctx, float *buf, size_t n, cudaStream_t st) = nullptr;
    void *ctx = nullptr;
};

// Where a sharded step's block writes its video output rows instead of vid_out:
// row r to base[dest[r].x] + dest[r].y * dim (the next block's input on the row's
// next owner; bases of other ranks are peer mappings). The stores are plain, so
// the caller orders them with the destination's readers.
struct RowScatter {
    const int2 *dest = nullptr;
    float *base[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
};

// s2_dit_block_forward with an optional text reduction and an optional scatter of
// the video output rows (not with debug captures).
s2_status dit_block_forward_ex(s2_dit_block *b, void *stream, const float *vid, int L, const float *txt, int Lt,
                               const float *emb, float *vid_out, float *txt_out, const TextReduce *reduce,
                               const RowScatter *scatter = nullptr);
s2_attention_layer *dit_block_attention(s2_dit_block *b);

// Debug capture of the attention stage the layer just ran (the block's
// set_debug_tensors): packed Q/K/V and the per-window outputs as [rows][dim]
// fp32, the pre-RoPE normalised q/k of the video and text rows; NULL outputs
// are skipped. attention_debug_rows: the packed row count of the current plan.
int attention_debug_rows(const s2_attention_layer *l);
s2_status attention_debug_capture(s2_attention_layer *l, cudaStream_t st, const void *vid_qkv, s2_dtype in_dtype,
                                  int L, const void *txt_qkv, int Lt, const void *vid_out, float *att_q, float *att_k,
                                  float *att_v, float *att_o, float *nq_vid, float *nk_vid, float *nq_txt,
                                  float *nk_txt);

// Attention prologue fused into the block's Q|K|V projection: the layer's
// current plan as the targets of GEMM_EPI_QKV_PACK (the packed Q/K/V workspace,
// the row map of the layer's L video rows followed by its Lt text rows, the
// per-window text rows, gammas, RoPE table, eps), plan and workspace set up for
// (L, Lt); then attention_forward_packed runs the attention core and the text
// mean on the packed operands the projection wrote.
struct GemmArgs;
// (cos, sin) of pos * freqs[pair] as [pair][max_pos] (s2_prologue.cu)
s2_status rope_table_pairs(cudaStream_t st, const float *freqs21, int max_pos, void *table);
s2_status attention_pack_target(s2_attention_layer *l, cudaStream_t st, int L, int Lt, GemmArgs *g);
s2_status attention_forward_packed(s2_attention_layer *l, cudaStream_t st, int L, int Lt, void *vid_out,
                                   float *txt_out);

// y = fp16( (x * inv_rms(x) [* gamma]) * mul + add0 + add1 ) per row
// (s2_block.cu); gamma and mul may be null (no gamma / no modulation).
s2_status rms_ada(cudaStream_t st, const float *x, int rows, int dim, float eps, const float *gamma,
                  const float *mul, const float *add0, const float *add1, void *y_f16);
// out [8][dim] modulation vectors of one branch (see modulation_kernel).
s2_status modulation_vectors(cudaStream_t st, const float *emb, const float *mod6, int dim, float *out);
s2_status f32_to_f16(cudaStream_t st, const float *x, long long n, void *y_f16);
// fp32 copy of n 16-bit values: bf16 for S2_MODE_BF16_REF, fp16 otherwise (s2_prologue.cu).
s2_status to_f32(cudaStream_t st, s2_mode mode, const void *src, long long n, float *dst);

// Sampler pieces (s2_sampler.cu). Guidance rescale factor of (pos, neg) into
// device memory inside `workspace` (cfg_workspace_bytes(), 16-byte aligned);
// *factor points at it.
size_t cfg_workspace_bytes();
s2_status cfg_factor(cudaStream_t st, const float *pos, const float *neg, long long n, float scale, float rescale,
                     void *workspace, float **factor);
// out = step_to / endpoint of x with the prediction pos, guided by neg when
// neg != null and scaled by *factor when factor != null.
s2_status sampler_update(cudaStream_t st, const float *x, const float *pos, const float *neg, float scale,
                         const float *factor, long long n, float timestep, float next_timestep, int final_step,
                         float *out);

}  // namespace s2
