/*
 * s2_b200.h -- C ABI of the B200 (sm_100a) SeedVR2 windowed MM-attention path.
 *
 * This is the drop-in boundary for the hot path of czwdysj/seedvr2-ncnn-valkan:
 * the body of SeedVR2DiTBlock::attention (src/layers/seedvr2_dit_block.cpp:870-1091),
 * i.e. window partition, per-head QK-RMSNorm, 3-axis MM-RoPE, bf16 rounding,
 * joint (video window || shared text) attention, video scatter and the
 * cross-window text mean. Everything else in the block stays with the caller.
 *
 * Conventions
 *  - Every entry point returns an s2_status (values mirror seedvr2::Status,
 *    include/seedvr2/engine.h:20-31). On failure s2_last_error() (thread-local)
 *    holds a one-line diagnostic, like the reference's stderr lines.
 *  - Device entry points are stream-ordered on the cudaStream_t passed as
 *    `void* stream` (NULL = legacy default stream) and never synchronise the
 *    host, except the *_host variants, which copy host buffers in and out.
 *  - Device pointers are caller-owned. Layer objects own only their weights,
 *    cached window plans and workspaces. A call with another shape rebuilds
 *    the cached plans (in place, or reallocated when larger) and may grow the
 *    workspaces, so a caller that captures an object's forward into its own
 *    CUDA graph may replay it only while every call on that object uses the
 *    captured shapes; after any other call it captures again. The DiT's own
 *    Euler-step graph handles this itself.
 *  - head_dim is 128 (the reference's MM-RoPE covers dims 0..125 and assumes
 *    128, seedvr2_dit_block.cpp:956-971).
 */
#ifndef S2_B200_H
#define S2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported entry points (the library is built with hidden visibility). */
#if defined(__GNUC__)
#define S2_API __attribute__((visibility("default")))
#else
#define S2_API
#endif

#define S2_HEAD_DIM 128
#define S2_ROPE_PAIRS 21

typedef enum s2_status {
    S2_OK = 0,                  /* seedvr2::Status::Ok */
    S2_INVALID_ARGUMENT = -1,   /* bad shape / blob count (reference returns -1) */
    S2_NOT_LOADED = -2,         /* weights not loaded / runtime shape not set */
    S2_INFERENCE_FAILED = -5,   /* a CUDA launch or device-side check failed */
    S2_UNSUPPORTED = -6,        /* no sm_100 device, or unsupported dtype/mode */
    S2_OUT_OF_MEMORY = -7       /* workspace allocation failed (reference -100) */
} s2_status;

typedef enum s2_dtype {
    S2_F32 = 0,
    S2_F16 = 1,
    S2_BF16 = 2
} s2_dtype;

/* Output rounding of the attention core. In both modes the packed Q/K/V hold
 * the reference's bf16-rounded values (RNE, the .bfloat16() before SDPA),
 * stored as fp16 -- exact for |x| in fp16's normal range [6.1e-5, 65504),
 * absolute error < 3e-8 below it -- both GEMMs run f16 x f16 on tcgen05 with
 * fp32 accumulation in TMEM, and P is fp16.
 *  S2_MODE_BF16_REF: outputs rounded to bf16 (RNE) and stored as bf16, as the
 *    reference CPU path rounds each window output (seedvr2_dit_block.cpp:1074).
 *  S2_MODE_F16: outputs stored as fp16 without the bf16 rounding (the
 *    reference's Vulkan shader keeps its fp32 result, :416-436). */
/*  S2_MODE_BF16_F16: outputs rounded to bf16 like S2_MODE_BF16_REF but stored
 *    as fp16 (exact for |x| in fp16's normal range), so that a following
 *    f16 x f16 tensor-core GEMM (the block's output projection) reads the
 *    reference's rounded values directly. */
typedef enum s2_mode {
    S2_MODE_BF16_REF = 0,
    S2_MODE_F16 = 1,
    S2_MODE_BF16_F16 = 2
} s2_mode;

/* One 3-D window box, half-open ranges on the (T, H, W) token grid.
 * Same fields as SeedVR2DiTBlock::Window (seedvr2_dit_block.h:98-106). */
typedef struct s2_window {
    int32_t t0, t1, h0, h1, w0, w1;
} s2_window;

/* One packed attention row. src >= 0: video token (t*H + y)*W + x;
 * src < 0: text token -(src+1). (pt, ph, pw) is its MM-RoPE position:
 * video (Lt + t - t0, y - h0, x - w0), text (l, l, l)
 * (seedvr2_dit_block.cpp:988, :1011). */
typedef struct s2_row {
    int32_t src, pt, ph, pw;
} s2_row;

/* ---- host-side planning ------------------------------------------------ */

/* Replaces SeedVR2DiTBlock::make_windows (seedvr2_dit_block.cpp:827-868),
 * bit-identical. wt/wh/ww > 0 override the resolution-adaptive window size
 * (explicit geometries); pass 0,0,0 for the reference rule. Writes up to
 * `cap` windows to `out` (may be NULL) and the full count to *count. */
S2_API s2_status s2_make_windows(int frames, int height, int width, int shifted,
                          int wt, int wh, int ww,
                          s2_window *out, int cap, int *count);

/* Packs windows into a varlen sequence list: window w occupies rows
 * [cu_seqlens[w], cu_seqlens[w+1]) = its L_w video tokens in (t, y, x) order
 * followed by the Lt text tokens -- the reference's per-window sequence
 * (seedvr2_dit_block.cpp:976-1028) and debug-capture row order (:899-907).
 * cu_seqlens has n+1 entries; rows has cu_seqlens[n] entries (either may be
 * NULL to query *total_rows only). */
S2_API s2_status s2_build_varlen(int frames, int height, int width,
                          const s2_window *windows, int n, int text_len,
                          int32_t *cu_seqlens, s2_row *rows, int *total_rows);

/* Multi-GPU ownership of a layer's windows: owner[i] = rank of window i, by a
 * deterministic longest-processing-time rule on cost S_w^2 (S_w = L_w +
 * text_len). Every window has one owner, so every video token has one. */
S2_API s2_status s2_shard_windows(const s2_window *windows, int n, int text_len, int n_ranks, int32_t *owner);

/* The sharded DiT step's ownership of BOTH window kinds of a grid, chosen
 * together so that few rows change owner at the plain <-> shifted layer
 * boundaries. A window's cost is a block's work on it: its video rows L_w (the
 * projections, MLP and norms, which dominate) + 1e-4 * S_w^2 (its attention,
 * S_w = L_w + text_len), in units of one row's per-row work. The plain windows
 * (owner_plain, s2_make_windows order) go in contiguous runs of their order with
 * the smallest largest run cost; each shifted window (owner_shifted), costliest
 * first, to the rank holding most of its rows whose load stays within 2 % of
 * the mean (else the least loaded).
 * Per-kind s2_shard_windows ownership is returned instead when it moves fewer
 * rows at no worse balance (small grids whose tilings split along frames). */
S2_API s2_status s2_shard_windows_joint(int frames, int height, int width, int wt, int wh, int ww, int text_len,
                                        int n_ranks, int32_t *owner_plain, int32_t *owner_shifted);
/* Rank `rank`'s view of that ownership for window kind `kind` (0 plain, 1
 * shifted) and the row exchange to the other kind, as the sharded step runs
 * it: the windows it owns (window_ids, *n_windows); its local rows
 * (local_tokens: the patched-grid token of each, window by window, (t, y, x)
 * inside a window; *n_local); send_rows: its local rows to send, destination
 * by destination (send_counts[n_ranks]), each in the destination's local order
 * of the other kind; recv_rows: where the rows received from each source
 * (recv_counts[n_ranks]) go in its local order of the other kind; its own
 * rows are among both (a local copy). *moved_rows: tokens of the grid whose
 * owner changes. Arrays may be NULL; their sizes are at most frames*height*width
 * (windows: the kind's window count). */
S2_API s2_status s2_shard_exchange(int frames, int height, int width, int wt, int wh, int ww, int text_len,
                                   int n_ranks, int rank, int kind, int32_t *window_ids, int *n_windows,
                                   int32_t *local_tokens, int *n_local, int32_t *send_counts, int32_t *send_rows,
                                   int32_t *recv_counts, int32_t *recv_rows, long long *moved_rows);
/* Where each of rank `rank`'s kind-`kind` local rows goes at the boundary to
 * the other kind, as the sharded step's exchange kernel writes it: the rank
 * holding the row's token under the other kind (dest_rank) and the row's index
 * in that rank's local order of the other kind (dest_row). *n_local = the
 * rank's kind-`kind` local row count; arrays may be NULL. */
S2_API s2_status s2_shard_row_destinations(int frames, int height, int width, int wt, int wh, int ww,
                                           int text_len, int n_ranks, int rank, int kind, int32_t *dest_rank,
                                           int32_t *dest_row, int *n_local);

/* ---- device kernels (explicit buffers) ---------------------------------- */

/* Fused prologue: per (packed row, head) RMSNorm over 128 dims (eps) times
 * gamma, MM-RoPE (3 axes x 21 pairs, angle = pos * freqs[p]), bf16 RNE
 * rounding; V rounded only. Replaces normalize_and_rotate and the V copy
 * (seedvr2_dit_block.cpp:942-1028) and the Vulkan qkv_prepare shader (:192-330).
 *   vid_qkv [L][3*heads*128], txt_qkv [Lt][3*heads*128] in `in_dtype`
 *   gammas: device fp32 [4][128] = norm_q_vid, norm_k_vid, norm_q_txt, norm_k_txt
 *   rows: device s2_row [n_rows]
 *   q, k, v: device fp16 [heads][n_rows][128] (bf16-rounded values).
 *   rope_table: device table from s2_rope_table for positions [0, max_pos)
 *   (every rows[].pt/ph/pw must be < max_pos). */
S2_API size_t s2_rope_table_bytes(int max_pos);
S2_API s2_status s2_rope_table(void *stream, const float *freqs21, int max_pos, void *rope_table);
S2_API s2_status s2_qk_norm_rope(void *stream,
                          const void *vid_qkv, const void *txt_qkv, s2_dtype in_dtype,
                          int heads, float eps, const float *gammas, const void *rope_table,
                          const s2_row *rows, int n_rows, s2_mode mode, void *q, void *k, void *v);

/* Varlen window attention on sm_100a (tcgen05 MMA into TMEM, TMA-fed
 * shared-memory ring, warp-specialised online softmax). For window w with
 * sequence rows [cu[w], cu[w+1]) and text_len trailing text rows:
 * O = softmax(Q K^T / sqrt(128)) V over the window's own rows, non-causal.
 * Video rows are scattered to vid_out[rows[r].src][h*128 + d] ([L][heads*128],
 * bf16 for S2_MODE_BF16_REF, fp16 for S2_MODE_F16); text rows go to
 * txt_partial[w][l][h*128 + d] ([n_windows][text_len][heads*128], same type). Replaces the attention core
 * (seedvr2_dit_block.cpp:1045-1079; Vulkan block_attention :339-438 plus
 * zero_buffer/window_sum scatter :442-457, :541-572).
 *   cu_seqlens: device int32 [n_windows+1]; rows: device s2_row.
 *   work: device int32 [n_work] of (window << 16 | q_block) items, one per
 *   256 query rows, costliest first (s2_plan_work); n_work * heads CTAs are
 *   launched.
 *   err: device int32 error word (0 = ok), set on a device-side timeout. */
S2_API s2_status s2_window_attention(void *stream, s2_mode mode,
                              const void *q, const void *k, const void *v, int heads, int n_rows,
                              const int32_t *cu_seqlens, int n_windows, int text_len,
                              const s2_row *rows, const int32_t *work, int n_work,
                              void *vid_out, void *txt_partial, int32_t *err);

/* Host helper: the (window, q_block) work list for s2_window_attention,
 * sorted by descending cost. Returns the item count in *n_work; `work` may be
 * NULL to query. cu_seqlens is the host copy. */
S2_API s2_status s2_plan_work(const int32_t *cu_seqlens, int n_windows, int32_t *work, int cap, int *n_work);

/* Text mean: txt_out[l][c] = (sum over w of txt_partial[w][l][c], in window
 * order, fp32) * scale (scale = 1/total windows; reference :1081-1088).
 * accumulate != 0 adds into txt_out instead of overwriting. */
S2_API s2_status s2_text_window_sum(void *stream, s2_mode mode, const void *txt_partial,
                             int n_windows, int text_len, int dim, float scale, int accumulate,
                             float *txt_out);

/* ---- layer object: mirror of SeedVR2DiTBlock's attention stage ---------- */

typedef struct s2_attention_layer s2_attention_layer;

/* load_param subset (seedvr2_dit_block.cpp:643-655): heads, head_dim (must be
 * 128), eps, shifted; window override wt/wh/ww (0 = reference rule); mode. */
S2_API s2_status s2_attention_layer_create(int device, int heads, int head_dim, float eps, int shifted,
                                    int wt, int wh, int ww, s2_mode mode,
                                    s2_attention_layer **out);
S2_API s2_status s2_attention_layer_destroy(s2_attention_layer *layer);

/* load_model subset (:657-688): host fp32 norm_q/norm_k of the video branch,
 * of the text branch (pass the video ones again for shared blocks), and
 * rope freqs [21]. */
S2_API s2_status s2_attention_layer_load(s2_attention_layer *layer,
                                  const float *norm_q_vid, const float *norm_k_vid,
                                  const float *norm_q_txt, const float *norm_k_txt,
                                  const float *freqs21);

/* set_runtime_shape (seedvr2_dit_block.h:55). */
S2_API s2_status s2_attention_layer_set_runtime_shape(s2_attention_layer *layer, int frames, int height, int width);

/* Restrict this layer to a subset of its windows (window sharding across
 * GPUs). ids NULL / n 0 = all windows. */
S2_API s2_status s2_attention_layer_set_window_subset(s2_attention_layer *layer, const int32_t *ids, int n);

/* With a window subset, let the layer read and write only the subset's video
 * tokens, compacted in packed order (window by window, (t, y, x) inside a
 * window): vid_qkv [n][3*dim] and vid_out [n][dim] with n from
 * s2_attention_layer_local_rows (after load and set_runtime_shape). Used by
 * the sharded DiT step, where each GPU keeps only its windows' rows. */
S2_API s2_status s2_attention_layer_set_local_rows(s2_attention_layer *layer, int enable);
S2_API s2_status s2_attention_layer_local_rows(s2_attention_layer *layer, int Lt, int *n_video);

/* attention() on device buffers: vid_qkv [L][3*dim], txt_qkv [Lt][3*dim] in
 * in_dtype; vid_out [L][dim] in the mode dtype (rows of windows outside the
 * subset are left untouched); txt_out [Lt][dim] fp32 = sum over this layer's
 * windows of the text outputs times 1/(total windows), or, with accumulate,
 * added into txt_out. Returns -1 on shape mismatch like the reference. */
S2_API s2_status s2_attention_layer_forward(s2_attention_layer *layer, void *stream,
                                     const void *vid_qkv, s2_dtype in_dtype, int L,
                                     const void *txt_qkv, int Lt,
                                     void *vid_out, float *txt_out);

/* Same on HOST buffers (the ncnn::Mat contract: vid_shape int32[3], inputs
 * [rows][3*dim], outputs [rows][dim]); copies in, runs, copies out and
 * synchronises `stream`. io_dtype is the element type of all four host
 * buffers except txt_out, which is fp32. */
S2_API s2_status s2_attention_layer_forward_host(s2_attention_layer *layer, void *stream,
                                          const void *vid_qkv, const void *txt_qkv,
                                          s2_dtype io_dtype, int L, int Lt, const int32_t *vid_shape,
                                          void *vid_out, float *txt_out);

/* Number of s2 kernels the last forward launched (for launch accounting). */
S2_API int s2_attention_layer_last_launches(const s2_attention_layer *layer);

/* Synchronises the layer's last stream and reports the device-side error word
 * (0 = ok; nonzero = a bounded wait inside the attention kernel timed out).
 * Returns S2_INFERENCE_FAILED when the word is set or the stream failed. */
S2_API s2_status s2_attention_layer_device_error(s2_attention_layer *layer, int *code);

/* ---- the whole DiT block (SeedVR2DiTBlock::forward) ----------------------- */

typedef struct s2_dit_block s2_dit_block;

/* load_param (seedvr2_dit_block.cpp:643-655): block_index, shared, last,
 * shifted, dim, heads, head_dim (128), mlp_hidden (a multiple of 128), eps;
 * wt/wh/ww override the window size (0,0,0 = the reference rule). */
S2_API s2_status s2_dit_block_create(int device, int block_index, int shared, int last, int shifted, int dim,
                                     int heads, int head_dim, int mlp_hidden, float eps, int wt, int wh, int ww,
                                     s2_dit_block **out);
S2_API s2_status s2_dit_block_destroy(s2_dit_block *block);

/* load_model (:657-688): the layer's host fp32 weight stream in the
 * reference's order -- per branch (video, then text unless shared): attn
 * shift, scale, gate, mlp shift, scale, gate [dim]; qkv W [3 dim][dim]; proj
 * W [dim][dim], proj b [dim]; norm_q, norm_k [128]; mlp gate W, in W
 * [hidden][dim]; out W [dim][hidden] -- then rope freqs [21].
 * n_floats must equal s2_dit_block_weight_count(block). */
S2_API size_t s2_dit_block_weight_count(const s2_dit_block *block);
S2_API s2_status s2_dit_block_load(s2_dit_block *block, const float *weights, size_t n_floats);

/* set_runtime_shape (seedvr2_dit_block.h:55) and window sharding. */
S2_API s2_status s2_dit_block_set_runtime_shape(s2_dit_block *block, int frames, int height, int width);
S2_API s2_status s2_dit_block_set_window_subset(s2_dit_block *block, const int32_t *ids, int n);
/* With a window subset: video rows are the subset's tokens only (see
 * s2_attention_layer_set_local_rows); vid / vid_out then have that many rows. */
S2_API s2_status s2_dit_block_set_local_rows(s2_dit_block *block, int enable);

/* forward (:1114-1267) on DEVICE buffers: vid [L][dim], txt [Lt][dim], emb
 * [6 dim] (emb[6c + slot]), all fp32 -> vid_out [L][dim], txt_out [Lt][dim]
 * fp32. RMSNorm + adaLN, QKV / output / SwiGLU MLP projections on the tensor
 * cores (fp16 operands, fp32 accumulation and residual stream), the windowed
 * attention of this header, gated residuals, the last block's text rule.
 * Stream-ordered; outputs must not alias inputs. */
S2_API s2_status s2_dit_block_forward(s2_dit_block *block, void *stream, const float *vid, int L, const float *txt,
                                      int Lt, const float *emb, float *vid_out, float *txt_out);

/* Same on HOST buffers with the vid_shape blob (int32 [3]), the ncnn::Mat
 * contract; synchronises `stream`. */
S2_API s2_status s2_dit_block_forward_host(s2_dit_block *block, void *stream, const float *vid, int L,
                                           const float *txt, int Lt, const float *emb, const int32_t *vid_shape,
                                           float *vid_out, float *txt_out);
S2_API int s2_dit_block_last_launches(const s2_dit_block *block);

/* set_debug_tensors (seedvr2_dit_block.h:20-36, 58): the reference's 14
 * capture points of one forward, written to DEVICE fp32 buffers the caller
 * owns (NULL members are skipped; tensors = NULL switches capturing off), in
 * the reference's [rows][channels] layouts:
 *   qkv_vid [L][3 dim], qkv_txt [Lt][3 dim] -- the QKV projections (kept in
 *     fp16 by this build: the captured values are those fp16 numbers);
 *   norm_q_vid, norm_k_vid [L][dim], norm_q_txt, norm_k_txt [Lt][dim] -- per
 *     head x * rsqrt(mean x^2 + eps) * gamma, before RoPE and rounding;
 *   attention_q, attention_k, attention_v [rows][dim] -- the packed window
 *     sequences (window by window, video (t, y, x) then text), bf16-rounded;
 *   attention_output [rows][dim] -- each packed row's window output (video
 *     rows as written to the attention output, text rows per window);
 *   projected_vid [L][dim], projected_txt [Lt][dim] -- output projection +
 *     bias, before the gate and residual;
 *   output_vid [L][dim], output_txt [Lt][dim] -- the block outputs.
 * rows = s2_dit_block_debug_rows (after set_runtime_shape). Capturing adds
 * conversion kernels and two projection GEMMs to each forward. */
typedef struct s2_block_debug {
    float *qkv_vid, *qkv_txt;
    float *norm_q_vid, *norm_q_txt, *norm_k_vid, *norm_k_txt;
    float *attention_q, *attention_k, *attention_v, *attention_output;
    float *projected_vid, *projected_txt;
    float *output_vid, *output_txt;
} s2_block_debug;
S2_API s2_status s2_dit_block_set_debug_tensors(s2_dit_block *block, const s2_block_debug *tensors);
/* The same for s2_dit_block_forward_host with HOST fp32 buffers (the
 * reference's host Mats): the captures are staged on the device and copied
 * out with the outputs. */
S2_API s2_status s2_dit_block_set_debug_tensors_host(s2_dit_block *block, const s2_block_debug *tensors);
S2_API s2_status s2_dit_block_debug_rows(s2_dit_block *block, int Lt, int *rows);
S2_API s2_status s2_dit_block_device_error(s2_dit_block *block, int *code);

/* ---- the block's projections (ncnn InnerProduct replacement) ------------- */

/* y = x W^T (+ b) as the block runs its InnerProduct layers (created at
 * seedvr2_dit_block.cpp:28-56, applied :1114-1267) on sm_100a tcgen05:
 * a [M][K] and b [N][K] fp16 row-major (K contiguous, K a multiple of 64,
 * rows 16-byte aligned), fp32 accumulation in TMEM, fused epilogues:
 *  S2_GEMM_SPLIT_F16: fp16 out[n / split][m * split + n % split] (out0..2;
 *    the fused Q|K|V projection with split = dim);
 *  S2_GEMM_GATED_RESID_F32: fp32 y[m][n] = ((acc + bias[n]) * gmul[n] +
 *    resid[m][n]) * out_scale (gmul / resid may be NULL: no gate / no
 *    residual); with split_row > 0, rows m >= split_row read resid2 and write
 *    y2 at row m - split_row (apply_ada_output_and_residual :807-825);
 *  S2_GEMM_SWIGLU_F16: every 256 columns of W hold 128 gate rows then the
 *    matching 128 "in" rows; fp16 out0[m][(n / 256) * 128 + j] =
 *    silu(gate_j) * in_j (apply_mlp :1093-1112).
 * workspace (device fp32, workspace_floats) lets a GEMM of at most 128 rows
 * that would fill less than half the GPU split K over up to 8 CTAs per tile
 * (deterministic: partial sums added in split order by a second kernel);
 * NULL = never split. A split result differs from the unsplit one within
 * fp32 rounding (another summation order). *extra_launches (may be NULL)
 * receives the kernels launched beyond the GEMM itself. err (required):
 * device int32 error word, set when a bounded wait inside the kernel gives
 * up. row_dest (S2_GEMM_GATED_RESID_F32 only, may be NULL): device int32
 * pairs {0, r'} per row r below split_row (or M): row r is written to y at
 * row r' instead of row r (the row scatter the sharded Euler step uses with
 * other ranks' buffers, here within y; every destination row written once;
 * no split-K). Stream-ordered. */
typedef enum s2_gemm_epilogue {
    S2_GEMM_SPLIT_F16 = 0,
    S2_GEMM_GATED_RESID_F32 = 2,
    S2_GEMM_SWIGLU_F16 = 3
} s2_gemm_epilogue;
typedef struct s2_gemm_desc {
    int epilogue, M, N, K;
    const void *a, *b;
    const float *bias, *gmul, *resid, *resid2;
    void *out0, *out1, *out2;
    float *y, *y2;
    int split, split_row;
    float out_scale;
    float *workspace;
    size_t workspace_floats;
    int32_t *err;
    const int32_t *row_dest;
} s2_gemm_desc;
S2_API s2_status s2_gemm(void *stream, const s2_gemm_desc *desc, int *extra_launches);

/* ---- multi-GPU communicator (no counterpart in the reference) ------------ */

/* One rank per GPU; NCCL over NVLink / NVSwitch, loaded on first use
 * (libnccl.so.2). Rank 0 creates the id, every rank passes the same bytes
 * (e.g. broadcast through torch.distributed) to s2_comm_init. */
#define S2_COMM_ID_BYTES 128
typedef struct s2_comm s2_comm;
S2_API s2_status s2_comm_unique_id(char *id /* [S2_COMM_ID_BYTES] */);
S2_API s2_status s2_comm_init(int device, int nranks, int rank, const char *id, s2_comm **out);
/* The same with an explicit deadline (s2_comm_init uses $S2_COMM_TIMEOUT_MS,
 * else 300 s): the ranks' rendezvous runs on a non-blocking NCCL communicator
 * polled against the deadline, so a rank that never joins ends in
 * ncclCommAbort and S2_INFERENCE_FAILED instead of blocking the host. Every
 * later NCCL call's result and the communicator's asynchronous state are
 * checked; after an abort the communicator refuses further work (destroy it). */
S2_API s2_status s2_comm_init_timeout(int device, int nranks, int rank, const char *id, long long timeout_ms,
                                      s2_comm **out);
S2_API s2_status s2_comm_set_timeout(s2_comm *comm, long long timeout_ms);
/* Waits on the host for `stream` (which holds this communicator's collectives)
 * under the same watchdog: returns S2_OK when the stream's work finished, or
 * aborts the communicator on an asynchronous NCCL error or at the deadline. */
S2_API s2_status s2_comm_wait(s2_comm *comm, void *stream);
S2_API s2_status s2_comm_destroy(s2_comm *comm);
S2_API int s2_comm_size(const s2_comm *comm);
S2_API int s2_comm_rank(const s2_comm *comm);

/* ---- the DiT model and one Euler step ------------------------------------ */

typedef struct s2_dit s2_dit;

/* SeedVR2DiT (src/model/dit.cpp:277-383): input head, n_blocks blocks, output
 * head. Reference values: n_blocks 32, dim 2560, heads 20, head_dim 128,
 * mlp_hidden 6912, eps 1e-5, video_channels 33, text_channels 5120,
 * sinusoidal_dim 256, out_channels 16 (the embedding is 6 * dim). */
S2_API s2_status s2_dit_create(int device, int n_blocks, int dim, int heads, int head_dim, int mlp_hidden, float eps,
                               int video_channels, int text_channels, int sinusoidal_dim, int out_channels, int wt,
                               int wh, int ww, s2_dit **out);
S2_API s2_status s2_dit_destroy(s2_dit *model);

/* Weight streams (host fp32) in the reference's load_model orders:
 * SeedVR2DiTInput (seedvr2_dit_input.cpp:217-224: video, text, time-in,
 * time-hidden, time-out projections, each W [out][in] then b),
 * SeedVR2DiTBlock (see s2_dit_block_load; the flags come from the block's
 * exported param file: shared for index >= 10, shifted for odd index, last
 * for the final block) and SeedVR2DiTOutput (seedvr2_dit_output.cpp:264-270:
 * norm weight, shift, scale [dim], projection W [4 oc][dim] then b). */
S2_API size_t s2_dit_input_weight_count(const s2_dit *model);
S2_API size_t s2_dit_output_weight_count(const s2_dit *model);
S2_API s2_status s2_dit_load_input(s2_dit *model, const float *weights, size_t n_floats);
S2_API s2_status s2_dit_load_block(s2_dit *model, int index, int shared, int last, int shifted, const float *weights,
                                   size_t n_floats);
S2_API s2_status s2_dit_load_output(s2_dit *model, const float *weights, size_t n_floats);

/* SeedVR2DiT::forward on DEVICE buffers: latent fp32 [video_channels][T][H][W]
 * (H, W even), text fp32 [Lt][text_channels], timestep -> prediction fp32
 * [out_channels][T][H][W]. Stream-ordered, no host synchronisation. */
S2_API s2_status s2_dit_forward(s2_dit *model, void *stream, const float *latent, int T, int H, int W,
                                const float *text, int Lt, float timestep, float *prediction);

/* One Euler sampling step as the engine runs it with one step and cfg 1
 * (src/core/engine.cpp:125-149, 308-343; EulerSampler::endpoint,
 * src/model/sampler.cpp:276-286): latent = noise || condition || ones,
 * prediction = DiT(latent, text, timestep), x0 = noise - (timestep/1000) *
 * prediction. noise, condition, x0: fp32 [out_channels][T][H][W]. */
S2_API s2_status s2_dit_euler_step(s2_dit *model, void *stream, const float *noise, const float *condition, int T,
                                   int H, int W, const float *text, int Lt, float timestep, float *x0);
/* Same on HOST buffers (copies in and out, synchronises `stream`). */
S2_API s2_status s2_dit_euler_step_host(s2_dit *model, void *stream, const float *noise, const float *condition,
                                        int T, int H, int W, const float *text, int Lt, float timestep, float *x0);
/* The engine's sampling loop on the device (src/core/engine.cpp:308-347 with
 * EulerSampler, src/model/sampler.cpp:181-286): x = noise; for each of
 * `steps` timesteps t_i = 1000 (1 - i/steps): prediction = DiT(x || condition
 * || ones, positive_text, t_i); when cfg_scale != 1 also the negative
 * prediction, guided = neg + cfg_scale (pos - neg), rescaled by cfg_rescale *
 * std(pos) / std(guided) + (1 - cfg_rescale) when cfg_rescale != 0; then
 * x = step_to(x, t_i, t_{i+1}), or the endpoint x - (t/1000) prediction at the
 * last step. noise, condition, out: DEVICE fp32 [out_channels][T][H][W]
 * (out may alias noise); texts fp32 [Lt][text_channels] (negative_text may be
 * NULL when cfg_scale == 1). Stream-ordered; runs the forwards eagerly (no
 * graph), so it also works on a sharded model (s2_dit_set_comm). */
S2_API s2_status s2_dit_sample(s2_dit *model, void *stream, const float *noise, const float *condition, int T, int H,
                               int W, const float *positive_text, const float *negative_text, int Lt, int steps,
                               float cfg_scale, float cfg_rescale, float *out);

/* The same loop with positive and negative texts of their own token counts
 * (the reference's default embeddings are 58 and 64 tokens; each DiT
 * forward takes any text length, dit.cpp:277-383). s2_dit_sample is this
 * call with both lengths Lt. */
S2_API s2_status s2_dit_sample_texts(s2_dit *model, void *stream, const float *noise, const float *condition, int T,
                                     int H, int W, const float *positive_text, int positive_len,
                                     const float *negative_text, int negative_len, int steps, float cfg_scale,
                                     float cfg_rescale, float *out);

/* Sampler pieces on DEVICE fp32 tensors of n elements (sampler.cpp):
 * timesteps of an n-step schedule (host; :181-187); classifier-free guidance
 * (:200-238; workspace of s2_apply_cfg_workspace_bytes(), 16-byte aligned,
 * needed only when rescale != 0); Euler step_to (:240-265) and endpoint
 * (:267-286). Outputs may alias inputs. */
S2_API s2_status s2_sampler_timesteps(int steps, float *timesteps);
S2_API size_t s2_apply_cfg_workspace_bytes(void);
S2_API s2_status s2_apply_cfg(void *stream, const float *positive, const float *negative, long long n, float scale,
                              float rescale, void *workspace, float *output);
S2_API s2_status s2_euler_step_to(void *stream, const float *prediction, const float *current, long long n,
                                  float timestep, float next_timestep, float *output);
S2_API s2_status s2_euler_endpoint(void *stream, const float *prediction, const float *current, long long n,
                                   float timestep, float *output);
/* Condition latent from the VAE encoding and augmentation noise
 * (make_condition_latent, src/core/engine.cpp:79-121): condition =
 * (1 - r) encoded + r noise with r = s2_condition_ratio(noise_scale, T, H, W)
 * (the shifted condition timestep / 1000 of a latent of T frames, H x W). */
S2_API float s2_condition_ratio(float noise_scale, int latent_frames, int latent_height, int latent_width);
S2_API s2_status s2_make_condition(void *stream, const float *encoded, const float *noise, int C, int T, int H, int W,
                                   float noise_scale, float *condition);

/* From the second call with the same shapes, buffers and timestep,
 * s2_dit_euler_step replays the step as one CUDA graph (captured on an
 * internal stream); enable = 0 keeps every call eager. On by default; a call
 * on a stream that is itself being captured always runs eagerly. A call of
 * s2_dit_forward or s2_dit_sample(_texts) on the model drops the graph (it may
 * grow the workspaces the graph points at): the next Euler step runs eagerly
 * and captures again. */
S2_API s2_status s2_dit_set_graph(s2_dit *model, int enable);

/* Shard the DiT step over the communicator's ranks (NULL = one GPU). Every
 * block's windows are split by s2_shard_windows; each rank keeps only its
 * windows' video rows (text rows replicated), all-reduces each block's text
 * attention mean, exchanges rows between the plain and shifted window
 * ownerships of consecutive blocks, and all ranks end with the full output
 * (disjoint per-rank parts summed). All ranks call forward / euler_step with
 * the same inputs, in the same order (the graph of a sharded step holds the
 * NCCL calls: destroy the model before the communicator). At the first call
 * for a grid the ranks gather each other's grid and window sizes and all
 * return S2_INVALID_ARGUMENT when they differ. */
S2_API s2_status s2_dit_set_comm(s2_dit *model, s2_comm *comm);
S2_API int s2_dit_last_launches(const s2_dit *model);
S2_API s2_status s2_dit_device_error(s2_dit *model, int *code);

/* ---- the reference's exported model files (host only) -------------------- */

/* Readers for the model directory written by the reference's exporter
 * (tools/export_seedvr2_dit_ncnn.py; loaded by SeedVR2DiT::load,
 * src/model/dit.cpp:119-214): per layer an ncnn .param text graph and a .bin
 * of weight blobs (raw fp32 vectors; InnerProduct weights tagged fp16
 * 0x01306B47 or fp32 0). Each reader parses the layer's ParamDict and decodes
 * the .bin into the fp32 stream that layer's s2_*_load takes; weights NULL
 * returns the float count in *n. */
typedef struct s2_block_params {
    int block_index, shared, last, shifted, dim, heads, head_dim, mlp_hidden;
    float eps;
} s2_block_params;
typedef struct s2_head_params {
    int dim, video_channels, text_channels, sinusoidal_dim, embedding_dim, out_channels;
    float eps;
} s2_head_params;
S2_API s2_status s2_ncnn_read_block(const char *param_path, const char *bin_path, s2_block_params *params,
                                    float *weights, size_t cap, size_t *n);
S2_API s2_status s2_ncnn_read_input(const char *param_path, const char *bin_path, s2_head_params *params,
                                    float *weights, size_t cap, size_t *n);
S2_API s2_status s2_ncnn_read_output(const char *param_path, const char *bin_path, s2_head_params *params,
                                     float *weights, size_t cap, size_t *n);
/* Loads seedvr2_dit_input / seedvr2_dit_output / seedvr2_dit_block_NN
 * (.ncnn.param + .ncnn.bin) from `dir` into the model (block flags from the
 * block files). */
S2_API s2_status s2_dit_load_dir(s2_dit *model, const char *dir);

/* ---- VAE mid-block spatial attention ------------------------------------ */

/* Single-head attention per frame, the core of the VAE mid-block attention
 * (DynamicFramewiseSpatialAttention::forward,
 * src/layers/dynamic_framewise_spatial_attention.cpp:149-180; Vulkan
 * attention pipeline :599-775): for every frame f and query token t,
 * out[f*tokens + t] = softmax_k(q[f*tokens + t] . k[f*tokens + k] / sqrt(channels)) v.
 * q, k, v, out: device fp16 [frames*tokens][head_dim] row-major, head_dim =
 * channels padded to 128, 256 or 512 with zero columns (the padded output
 * columns come out zero). tcgen05 MMA into TMEM, fp32 accumulation, P fp16.
 * err: device int32 error word, set on a device-side timeout. */
S2_API s2_status s2_spatial_attention(void *stream, const void *q, const void *k, const void *v, int channels,
                                      int head_dim, int frames, int tokens, void *out, int32_t *err);

typedef struct s2_vae_attention s2_vae_attention;

/* load_param (dynamic_framewise_spatial_attention.cpp:50-59): channels must
 * be a positive multiple of 32 (GroupNorm with 32 groups); this build
 * supports channels <= 512. */
S2_API s2_status s2_vae_attention_create(int device, int channels, s2_vae_attention **out);
S2_API s2_status s2_vae_attention_destroy(s2_vae_attention *layer);

/* load_model (:61-77): host fp32 arrays in the reference's load order;
 * weights are [out][in] = channels x channels. */
S2_API s2_status s2_vae_attention_load(s2_vae_attention *layer, const float *norm_bias, const float *norm_weight,
                                       const float *k_bias, const float *k_weight, const float *out_bias,
                                       const float *out_weight, const float *q_bias, const float *q_weight,
                                       const float *v_bias, const float *v_weight);

/* forward (:106-210) on DEVICE buffers in ncnn's 4-D layout: x and y are fp32
 * [channels][cstep], channel plane = frames x height x width (cstep >=
 * frames*height*width). GroupNorm(32, eps 1e-6) per frame, Q/K/V 1x1
 * projections, attention, output projection + residual: y = x + proj(attn).
 * Stream-ordered, no host synchronisation; x and y must not alias. */
S2_API s2_status s2_vae_attention_forward(s2_vae_attention *layer, void *stream, const float *x, int frames,
                                          int height, int width, long long cstep, float *y);

/* Same on HOST buffers (the ncnn::Mat contract); copies in and out and
 * synchronises `stream`. */
S2_API s2_status s2_vae_attention_forward_host(s2_vae_attention *layer, void *stream, const float *x, int frames,
                                               int height, int width, long long cstep, float *y);

/* Kernels launched by the last forward, and the device error word (0 = ok). */
S2_API int s2_vae_attention_last_launches(const s2_vae_attention *layer);
S2_API s2_status s2_vae_attention_device_error(s2_vae_attention *layer, int *code);

/* ---- the VAE's other layers: GroupNorm, space-time shuffle, Conv3D ------- */

/* All three work on ncnn 4-D blobs, fp32 [channels][cstep] whose channel
 * plane holds frames x height x width values (x and y may have different
 * csteps, each at least its plane); x and y must not alias. Device forwards
 * are stream-ordered with no host synchronisation; the *_host variants copy
 * packed host blobs [channels][plane] in and out and synchronise `stream`.
 *
 * DynamicFramewiseGroupNorm (src/layers/dynamic_framewise_group_norm.cpp):
 * load_param :43-53 (channels from param key 10, a positive multiple of the
 * 32 groups), load_model :55-61 (bias, then weight, [channels] each), forward
 * :63-121 -- per frame and group of channels/32 channels, the mean and
 * variance of its values (double sums), y = x * w / sqrt(var + 1e-6) +
 * (b - mean * w / sqrt(var + 1e-6)). */
typedef struct s2_vae_group_norm s2_vae_group_norm;
S2_API s2_status s2_vae_group_norm_create(int device, int channels, s2_vae_group_norm **out);
S2_API s2_status s2_vae_group_norm_destroy(s2_vae_group_norm *layer);
S2_API s2_status s2_vae_group_norm_load(s2_vae_group_norm *layer, const float *bias, const float *weight);
S2_API s2_status s2_vae_group_norm_forward(s2_vae_group_norm *layer, void *stream, const float *x, int frames,
                                           int height, int width, long long cstep, float *y, long long y_cstep);
S2_API s2_status s2_vae_group_norm_forward_host(s2_vae_group_norm *layer, void *stream, const float *x, int frames,
                                                int height, int width, float *y);
S2_API int s2_vae_group_norm_last_launches(const s2_vae_group_norm *layer);

/* DynamicSpaceTimeShuffle (src/layers/dynamic_space_time_shuffle.cpp):
 * load_param :41-55 (projected channels P from param key 10, in channels from
 * key 11's [P, in]; P = in x 4 x temporal ratio), load_model :57-63 (bias [P],
 * weight [P][in]), forward :65-130 -- a 1x1x1 projection whose channel
 * ((oy * 2 + ox) * tr + ot) * in + c lands in output channel c at frame
 * f * tr + ot (raw frame 1 dropped when tr > 1: T' = T * tr - 1), row
 * 2 y + oy, column 2 x + ox. This build needs in channels % 32 == 0. */
typedef struct s2_vae_space_time_shuffle s2_vae_space_time_shuffle;
S2_API s2_status s2_vae_space_time_shuffle_create(int device, int in_channels, int projected_channels,
                                                  s2_vae_space_time_shuffle **out);
S2_API s2_status s2_vae_space_time_shuffle_destroy(s2_vae_space_time_shuffle *layer);
S2_API s2_status s2_vae_space_time_shuffle_load(s2_vae_space_time_shuffle *layer, const float *bias,
                                                const float *weight);
S2_API s2_status s2_vae_space_time_shuffle_output_shape(const s2_vae_space_time_shuffle *layer, int frames, int height,
                                                        int width, int *out_frames, int *out_height, int *out_width);
S2_API s2_status s2_vae_space_time_shuffle_forward(s2_vae_space_time_shuffle *layer, void *stream, const float *x,
                                                   int frames, int height, int width, long long cstep, float *y,
                                                   long long y_cstep);
S2_API s2_status s2_vae_space_time_shuffle_forward_host(s2_vae_space_time_shuffle *layer, void *stream,
                                                        const float *x, int frames, int height, int width, float *y);
S2_API int s2_vae_space_time_shuffle_last_launches(const s2_vae_space_time_shuffle *layer);
S2_API s2_status s2_vae_space_time_shuffle_device_error(s2_vae_space_time_shuffle *layer, int *code);

/* ncnn's Convolution3D as the VAE uses it (the layer the reference patches,
 * patches/0001-feat-Convolution3D-Vulkan-pack1.patch): ParamDict fields of
 * the layer -- num_output, kernel d/h/w, dilation, stride, pads (front, top,
 * left, behind, bottom, right; all -233 = SAME_UPPER, all -234 = SAME_LOWER,
 * resolved per input as :240-265), pad_value (0 in this build), bias_term;
 * weights [out][in][kd][kh][kw] then bias [out]. out[p][z][i][j] = bias[p] +
 * sum over q, kd, kh, kw of in[q][z sd + kd dd - front][i sh + kh dh -
 * top][j sw + kw dw - left] * w[p][q][kd][kh][kw] (the patch's :17-25), as
 * an implicit GEMM on tcgen05: fp16 operands, fp32 accumulation. This build
 * needs stride_w <= 4. */
typedef struct s2_vae_conv3d s2_vae_conv3d;
S2_API s2_status s2_vae_conv3d_create(int device, int in_channels, int out_channels, int kernel_d, int kernel_h,
                                      int kernel_w, int dilation_d, int dilation_h, int dilation_w, int stride_d,
                                      int stride_h, int stride_w, int pad_front, int pad_top, int pad_left,
                                      int pad_behind, int pad_bottom, int pad_right, float pad_value, int bias_term,
                                      s2_vae_conv3d **out);
S2_API s2_status s2_vae_conv3d_destroy(s2_vae_conv3d *layer);
S2_API s2_status s2_vae_conv3d_load(s2_vae_conv3d *layer, const float *weight, const float *bias);
S2_API s2_status s2_vae_conv3d_output_shape(const s2_vae_conv3d *layer, int frames, int height, int width,
                                            int *out_frames, int *out_height, int *out_width);
S2_API s2_status s2_vae_conv3d_forward(s2_vae_conv3d *layer, void *stream, const float *x, int frames, int height,
                                       int width, long long cstep, float *y, long long y_cstep);
S2_API s2_status s2_vae_conv3d_forward_host(s2_vae_conv3d *layer, void *stream, const float *x, int frames,
                                            int height, int width, float *y);
S2_API int s2_vae_conv3d_last_launches(const s2_vae_conv3d *layer);
S2_API s2_status s2_vae_conv3d_device_error(s2_vae_conv3d *layer, int *code);

/* ---- allocation-free variant -------------------------------------------- */

/* Limits of the fixed scratch used by s2_dit_window_attention_noalloc
 * (about 29 MiB of device memory in total). */
#define S2_NOALLOC_MAX_ROW_HEADS 32768       /* packed rows (sum of L_w + Lt) x heads */
#define S2_NOALLOC_MAX_TEXT_ELEMS 2097152    /* windows x text_len x heads*128 */
#define S2_NOALLOC_MAX_WINDOWS 512
#define S2_NOALLOC_MAX_ROPE_POS 1024         /* largest RoPE position + 1 */

/* No counterpart in the reference. The whole attention stage (what
 * s2_attention_layer_forward does) for callers that must not allocate device
 * memory while they run -- e.g. code executing inside another framework's
 * memory pool or allocator callbacks, or a host that has reserved all HBM up
 * front -- so it never calls cudaMalloc, cudaFree or an allocating library
 * routine. Instead of workspaces it uses one fixed device array that belongs
 * to this library (the S2_NOALLOC_* limits above): every GPU that loads the
 * library's module holds that array until the process exits. Inputs and
 * outputs are the caller's: vid_qkv [L][3*heads*128] and txt_qkv
 * [text_len][3*heads*128] in in_dtype, gammas device fp32 [4][128] (norm_q_vid,
 * norm_k_vid, norm_q_txt, norm_k_txt), freqs21 device fp32 [21], vid_out
 * [L][heads*128] (bf16 or fp16 by mode), txt_out fp32 [text_len][heads*128];
 * err (device int32, may be NULL) receives the kernel's error word (cleared
 * at the start of every call).
 * Sizes beyond the limits return S2_INVALID_ARGUMENT with a message naming
 * the limit. The first call on each device resolves the array's device
 * address (cudaGetSymbolAddress with that device current), so make the first
 * call on a device before any stream capture. All calls share the array and
 * it keeps the last call's contents: calls whose GPU work overlaps (other
 * streams or threads without ordering) race on it. */
S2_API s2_status s2_dit_window_attention_noalloc(void *stream, s2_mode mode,
                                                 const void *vid_qkv, const void *txt_qkv, s2_dtype in_dtype,
                                                 int frames, int height, int width, int text_len,
                                                 int heads, float eps, int shifted, int wt, int wh, int ww,
                                                 const float *gammas, const float *freqs21,
                                                 void *vid_out, float *txt_out, int32_t *err);

/* ---- failure injection (tests only; no counterpart in the reference) ----- */

/* The next n device allocations made by this library's layer objects fail as
 * if the GPU were out of memory (their calls return S2_OUT_OF_MEMORY); 0 clears
 * it. For exercising callers' out-of-memory paths. */
S2_API s2_status s2_debug_fail_allocations(int n);
/* One shot, for the next s2_window_attention launch in the process (layer
 * forwards included): every bounded wait of that launch gives up after
 * wait_ns (0 = the default 1 s), and with skip_k_tile >= 0 the load producer of
 * its first CTA leaves out that K tile (counted from the CTA's first), so the
 * tensor-core role's wait for it runs out. The launch then ends on its own with
 * its error word set (2, 3 or 5: the K wait, the producer's wait for a slot
 * that role never released, or a softmax wait for the S tile that was never
 * computed, whichever gives up first), the layer's
 * device-error query returns S2_INFERENCE_FAILED, its TMEM is freed, and
 * launches after it are unaffected. */
S2_API s2_status s2_debug_attention_fault(int skip_k_tile, unsigned long long wait_ns);

/* ---- misc ---------------------------------------------------------------- */

S2_API const char *s2_last_error(void);
/* 0 if device `device` is an sm_100 part this build can run on. */
S2_API s2_status s2_device_check(int device);
S2_API int s2_version(void);

#ifdef __cplusplus
}
#endif
#endif /* S2_B200_H */
