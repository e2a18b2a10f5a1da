// Internal interface of the tcgen05 GEMM (s2_gemm.cu) and the shared
// tensor-map encoder. Not part of the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "s2_b200.h"

namespace s2 {

// 2-D fp16 tensor map over a row-major [rows][inner] matrix (row pitch
// row_bytes), box = box_inner x box_rows elements, 128-byte swizzle.
bool make_map_2d(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_rows);
// Maps for TMA stores from a staging tile: fp16 without swizzle, fp32 with
// 128-byte swizzle (box inner extent 32 floats).
bool make_map_2d_plain(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                       uint32_t box_inner, uint32_t box_rows);
bool make_map_2d_plain_f32(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                           uint32_t box_inner, uint32_t box_rows);

// Epilogues of D = A B^T (+ bias).
enum GemmEpilogue : int {
    // fp16 row-major outputs split by column blocks of `split`: column n goes to
    // out[n / split][row * split + n % split] (the fused Q|K|V projection).
    GEMM_EPI_SPLIT_F16 = 0,
    // fp32 channel-major output with residual: for n < n_valid,
    // y[n * ldt + row] = acc + bias[n] + resid[n * ldt + row] (1x1 conv back
    // into an ncnn [C][cstep] blob; no residual when resid is null).
    GEMM_EPI_RESID_T_F32 = 1,
    // fp32 row-major output with the DiT block's gated residual
    // (apply_ada_output_and_residual, seedvr2_dit_block.cpp:807-825):
    // y[row * N + n] = ((acc + bias[n]) * gmul[n] + resid[row * N + n]) * out_scale,
    // gmul[n] = emb[6 n + slot] + gate[n] precomputed (no multiply when gmul
    // is null; no residual when resid is null: the plain "+ bias" projection).
    GEMM_EPI_GATED_RESID_F32 = 2,
    // SwiGLU (apply_mlp, :1093-1112): every 256-column tile holds 128 gate
    // columns then the 128 matching "in" columns; out[0] is fp16
    // [row][N / 2], hidden column (n / 256) * 128 + j = silu(gate_j) * in_j.
    GEMM_EPI_SWIGLU_F16 = 3,
    // Space-time shuffle (DynamicSpaceTimeShuffle, dynamic_space_time_shuffle.cpp:65-130):
    // row = input token (f * sh_h + y) * sh_w + x, column n = ((oy * sh_tr + ot) * sh_cin
    // + c) * 2 + ox (the projected channels permuted so that ox is innermost);
    // y[c * ldt + (t' * 2 sh_h + 2 y + oy) * 2 sh_w + 2 x + ox] = acc + bias[n] with
    // t' = f * sh_tr + ot, less one past the dropped raw frame 1 when sh_tr > 1.
    // Needs sh_cin % 16 == 0, ldt even and y 8-byte aligned (float2 stores).
    GEMM_EPI_SHUFFLE_F32 = 4,
    // Convolution output: row = position (z * geom.oh + i) * geom.owp + j of the
    // output grid padded to geom.owp columns; for j < geom.ow,
    // y[n * ldt + (z * geom.oh + i) * geom.ow + j] = acc + bias[n] (n < n_valid).
    GEMM_EPI_CONV_F32 = 5,
    // The DiT block's fused Q|K|V projection with the attention prologue applied
    // to the fp32 accumulator (normalize_and_rotate, seedvr2_dit_block.cpp:942-974):
    // per row and head of the Q and K column blocks, RMS normalisation over the
    // 128 head dims (squares summed in fp32, four chains), times the branch
    // gamma, 3-axis RoPE on dims 0..125; V unchanged; every value rounded to
    // bf16 (RNE) and stored as fp16 into the window-packed, head-major operands
    // of the attention core at the row's packed row (text rows: into every
    // window's text rows). See PackArgs. N = 3 * dim, dim a multiple of 128.
    GEMM_EPI_QKV_PACK = 6,
};

// GEMM_EPI_QKV_PACK targets.
struct PackArgs {
    // per GEMM row: {packed row, pt, ph, pw}, {-1 - l, l, l, l} for text row l, or
    // {-0x7fffffff, ...} for a row that has no packed row (nothing is stored)
    const int4 *map = nullptr;
    const int32_t *text_dst = nullptr;  // per window: packed row of its text row 0
    int n_windows = 0;
    void *q = nullptr, *k = nullptr, *v = nullptr;  // fp16 [dim / 128][n_rows][128]
    int n_rows = 0;
    int dim = 0;                        // heads * 128
    const float *gammas = nullptr;      // [q video, k video, q text, k text][128]
    const float2 *rope = nullptr;       // (cos, sin) pair-major: [21][max_pos]
    int max_pos = 0;
    float eps = 0.f;
};

// Implicit-GEMM 3-D convolution: A is not a matrix but the im2col of a
// token-major fp16 input [D][H][W][Cp] (Cp a multiple of 64) read through a
// 4-D tensor map in boxes of 64 channels x 32 output columns; K slice kc is tap
// kc / (Cp / 64) (taps in (kd, kh, kw) order) and channels 64 * (kc % (Cp / 64)).
// Out-of-range taps read zeros (the TMA fill): zero padding.
struct ConvGeom {
    int od = 0, oh = 0, ow = 0, owp = 0;  // output extents; owp = ow rounded up to 32
    int kd = 1, kh = 1, kw = 1;
    int sd = 1, sh = 1, sw = 1;
    int dd = 1, dh = 1, dw = 1;
    int pf = 0, pt = 0, pl = 0;  // front / top / left padding
    int cslices = 1;             // Cp / 64
    int in_d = 0, in_h = 0, in_w = 0;  // input extents
};

struct GemmArgs {
    int M = 0, N = 0, K = 0;      // K a multiple of 64
    const float *bias = nullptr;  // [N] or null
    int epilogue = GEMM_EPI_SPLIT_F16;
    void *out[3] = {nullptr, nullptr, nullptr};
    int split = 0;
    const float *resid = nullptr;
    float *y = nullptr;
    long long ldt = 0;
    int n_valid = 0;
    const float *gmul = nullptr;  // GEMM_EPI_GATED_RESID_F32 gate vector [N] or null
    // GEMM_EPI_GATED_RESID_F32 row split (0 = none): rows >= split_row read
    // resid2 and write y2 at row - split_row (video and text rows of a block
    // with shared weights in one GEMM)
    int split_row = 0;
    const float *resid2 = nullptr;
    float *y2 = nullptr;
    float out_scale = 1.f;
    int bn = 0;                   // tile width 256 or 128 (0: chosen from the wave fill)
    int pair = -1;                // CTA pairs (256 x 256 tiles on two SMs): 1 on, 0 off, -1 chosen by shape
    // Split-K workspace: with `partial` set, a GEMM of at most 128 rows whose tiles
    // fill less than half of the grid splits K over up to 8 CTAs per tile; each writes
    // fp32 partial sums [split][M][N] here (capacity `partial_floats`) and a second
    // kernel adds them in split order and applies the epilogue. Set by gemm_f16.
    float *partial = nullptr;
    size_t partial_floats = 0;
    int ksplit = 0;
    int *extra_launches = nullptr;  // if set, incremented per kernel launched beyond the GEMM itself
    int32_t *err = nullptr;       // device error word (bounded waits)
    int sh_cin = 0, sh_tr = 1, sh_h = 0, sh_w = 0;  // GEMM_EPI_SHUFFLE_F32 geometry
    int conv = 0;                 // 1: A is the im2col of the convolution `geom`
    ConvGeom geom;
    PackArgs pk;                  // GEMM_EPI_QKV_PACK
    // GEMM_EPI_GATED_RESID_F32 row scatter: with row_dest set, row r (< split_row, or
    // < M) goes to dest_base[row_dest[r].x] + row_dest[r].y * N instead of y -- any
    // rank's buffer mapped into this process (peer stores over NVLink), each thread
    // fencing its stores at system scope before the kernel ends. No split-K.
    const int2 *row_dest = nullptr;
    float *dest_base[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
};

// D[M][N] = A[M][K] B[N][K]^T on sm_100a: A and B fp16, K-major (row-major
// with K contiguous, rows 16-byte aligned), fp32 accumulation in TMEM.
s2_status gemm_f16(cudaStream_t st, const void *A, const void *B, const GemmArgs &args);

// 3-D convolution as an implicit GEMM (args.conv = 1, args.geom set): A is the
// token-major fp16 input [geom.in_d][geom.in_h][geom.in_w][Cp] (Cp = cslices *
// 64, zero channels past the real ones), B the fp16 weights [N][taps * Cp]
// (tap-major, K contiguous); args.M = od * oh * owp, args.K = taps * Cp,
// args.epilogue = GEMM_EPI_CONV_F32. Same entry point: gemm_f16.

}  // namespace s2
