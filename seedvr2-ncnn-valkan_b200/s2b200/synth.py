"""Seeded synthetic inputs for the windowed MM-attention path.

No public dataset exists for this path; these stand in for real activations
with the shapes and distributions the reference's benchmarks use: QKV rows
drawn N(0, 1) and stored as fp16-representable values, 58 text tokens (the
shipped default positive embedding length), QK-norm gammas ``1 + 0.1 N(0,1)``
and the model's RoPE frequencies ``1 / 10000^(2p/42)``, p < 21
(tools/diagnose_seedvr2_rope.py:36-37 of the reference).
"""
from __future__ import annotations

import numpy as np

HEAD_DIM = 128
TEXT_LEN = 58

# Grids (T, H, W) of BASELINE.json's configs after VAE compression + patchify.
GRIDS = {
    "cfg0": (2, 16, 30),      # 480x256x5f
    "cfg2": (6, 45, 80),      # 720p x 21f
    "cfg3": (12, 67, 120),    # 1080p x 45f
}
# VAE mid-block attention (config 4): channels, latent frames, height, width.
VAE_CFG4 = (512, 6, 90, 160)
# BASELINE.json's explicit window geometries (the reference computes its own).
OVERRIDES = {"cfg0": (2, 8, 10), "cfg2": (6, 15, 20), "cfg3": (4, 17, 20)}


def rope_freqs() -> np.ndarray:
    return (1.0 / 10000.0 ** (np.arange(21, dtype=np.float64) * 2.0 / 42.0)).astype(np.float32)


def layer_inputs(grid, heads=20, text_len=TEXT_LEN, seed=666):
    """(vid_qkv [L, 3*dim] f32, txt_qkv [Lt, 3*dim] f32, gammas [4][128] f32, freqs [21] f32).

    QKV values are exactly representable in fp16, so the fp32 and fp16 copies
    of the same draw feed identical numbers to the oracle and the GPU."""
    T, H, W = grid
    L = T * H * W
    dim = heads * HEAD_DIM
    rng = np.random.default_rng(seed)
    vid = rng.standard_normal((L, 3 * dim), dtype=np.float32).astype(np.float16).astype(np.float32)
    txt = rng.standard_normal((text_len, 3 * dim), dtype=np.float32).astype(np.float16).astype(np.float32)
    gam = (1.0 + 0.1 * rng.standard_normal((4, HEAD_DIM))).astype(np.float32)
    return vid, txt, gam, rope_freqs()


def attention_flops(windows: np.ndarray, text_len: int, heads: int) -> float:
    """Algorithmic FLOPs of one attention layer: sum_w 4 * S_w^2 * 128 * heads."""
    s = (windows[:, 1] - windows[:, 0]) * (windows[:, 3] - windows[:, 2]) * (windows[:, 5] - windows[:, 4]) + text_len
    return float(np.sum(4.0 * s.astype(np.float64) ** 2 * HEAD_DIM * heads))


def prologue_bytes(L: int, text_len: int, heads: int, in_bytes: int) -> float:
    """Algorithmic HBM bytes of the prologue: read each QKV row once (video and
    text), write each row's packed q/k/v once in 16-bit (text rows once, not per
    window)."""
    dim = heads * HEAD_DIM
    return float((L + text_len) * 3 * dim * in_bytes + (L + text_len) * 3 * dim * 2)


def prologue_bytes_moved(L: int, text_len: int, n_rows: int, heads: int, in_bytes: int) -> float:
    """Bytes the prologue moves: the algorithmic read, and the packed rows it
    writes, the text rows once per window (n_rows packed rows)."""
    dim = heads * HEAD_DIM
    return float((L + text_len) * 3 * dim * in_bytes + n_rows * 3 * dim * 2)


def vae_inputs(shape=VAE_CFG4, seed=666):
    """(x [C, T, H, W] f32, weights dict) for the VAE mid-block attention.

    x ~ N(0, 1) stored fp16-representable; projection weights and biases
    N(0, 0.02); GroupNorm gamma 1 + 0.1 N(0, 1), beta 0.1 N(0, 1)."""
    C, T, H, W = shape
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((C, T, H, W), dtype=np.float32).astype(np.float16).astype(np.float32)
    w = {"norm_weight": (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32),
         "norm_bias": (0.1 * rng.standard_normal(C)).astype(np.float32)}
    for name in ("q", "k", "v", "out"):
        w[f"{name}_weight"] = (0.02 * rng.standard_normal(C * C)).astype(np.float32)
        w[f"{name}_bias"] = (0.02 * rng.standard_normal(C)).astype(np.float32)
    return x, w


def vae_attention_flops(shape) -> float:
    """Algorithmic FLOPs of the per-frame attention: T * 4 * (H*W)^2 * C."""
    C, T, H, W = shape
    return float(T) * 4.0 * float(H * W) ** 2 * C


def vae_projection_flops(shape) -> float:
    """FLOPs of the four 1x1 projections: 4 * 2 * T*H*W * C^2."""
    C, T, H, W = shape
    return 8.0 * T * H * W * float(C) * C


def block_weights(dim, heads, mlp_hidden, shared=False, seed=666):
    """Flat fp32 weight stream of one SeedVR2DiTBlock in the reference's
    load_model order (seedvr2_dit_block.cpp:657-688): per branch the six adaLN
    vectors N(0, 0.02), qkv W, proj W + b, mlp gate/in/out W ~ N(0, 0.02),
    QK-norm gammas 1 + 0.1 N(0, 1); then the RoPE freqs."""
    rng = np.random.default_rng(seed)

    def branch():
        parts = [0.02 * rng.standard_normal(dim, dtype=np.float32) for _ in range(6)]
        parts += [0.02 * rng.standard_normal(3 * dim * dim, dtype=np.float32),
                  0.02 * rng.standard_normal(dim * dim, dtype=np.float32),
                  0.02 * rng.standard_normal(dim, dtype=np.float32),
                  (1.0 + 0.1 * rng.standard_normal(HEAD_DIM)).astype(np.float32),
                  (1.0 + 0.1 * rng.standard_normal(HEAD_DIM)).astype(np.float32),
                  0.02 * rng.standard_normal(mlp_hidden * dim, dtype=np.float32),
                  0.02 * rng.standard_normal(mlp_hidden * dim, dtype=np.float32),
                  0.02 * rng.standard_normal(dim * mlp_hidden, dtype=np.float32)]
        return parts

    stream = branch() if shared else branch() + branch()
    stream.append(rope_freqs())
    return np.concatenate([p.astype(np.float32).ravel() for p in stream])


def block_activations(grid, dim, text_len=TEXT_LEN, seed=667):
    """(vid [L, dim], txt [Lt, dim]) ~ N(0, 1) and emb [6 dim] ~ N(0, 0.02)."""
    T, H, W = grid
    rng = np.random.default_rng(seed)
    vid = rng.standard_normal((T * H * W, dim), dtype=np.float32)
    txt = rng.standard_normal((text_len, dim), dtype=np.float32)
    emb = (0.02 * rng.standard_normal(6 * dim)).astype(np.float32)
    return vid, txt, emb


def block_gemm_flops(L, text_len, dim, mlp_hidden, last=False):
    """FLOPs of a block's projections: qkv, proj, SwiGLU (gate + in), out."""
    per_row = 2.0 * dim * (3 * dim + dim + 2 * mlp_hidden + mlp_hidden)
    txt_rows = text_len if not last else 0
    return per_row * L + per_row * txt_rows + (2.0 * dim * 4 * dim * text_len if last else 0.0)


# DiT heads (SeedVR2DiTInput / SeedVR2DiTOutput) and the config-2 latent.
DIT_CFG2_LATENT = (6, 90, 160)   # T, H, W of the 16-channel latent (720p x 21 frames)
DIT_HEADS = dict(video_channels=33, text_channels=5120, sinusoidal_dim=256, out_channels=16)


def dit_input_weights(dim, video_channels=33, text_channels=5120, sinusoidal_dim=256, seed=668):
    """SeedVR2DiTInput weight stream (load_model order, seedvr2_dit_input.cpp:217-224):
    video, text, time-in, time-hidden, time-out projections, each W [out][in]
    ~ N(0, 0.02) then b ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    ed = 6 * dim
    parts = []
    for n_in, n_out in ((4 * video_channels, dim), (text_channels, dim), (sinusoidal_dim, dim), (dim, dim),
                        (dim, ed)):
        parts += [0.02 * rng.standard_normal(n_in * n_out, dtype=np.float32),
                  0.02 * rng.standard_normal(n_out, dtype=np.float32)]
    return np.concatenate(parts).astype(np.float32)


def dit_output_weights(dim, out_channels=16, seed=669):
    """SeedVR2DiTOutput weight stream (seedvr2_dit_output.cpp:264-270): norm
    weight 1 + 0.1 N, shift and scale N(0, 0.02), projection W, b ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    n = 4 * out_channels
    return np.concatenate([(1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32),
                           0.02 * rng.standard_normal(dim, dtype=np.float32),
                           0.02 * rng.standard_normal(dim, dtype=np.float32),
                           0.02 * rng.standard_normal(n * dim, dtype=np.float32),
                           0.02 * rng.standard_normal(n, dtype=np.float32)]).astype(np.float32)


def dit_latents(latent_shape, out_channels=16, text_len=TEXT_LEN, text_channels=5120, seed=670):
    """(noise, condition [oc, T, H, W] ~ N(0, 1), text [Lt, text_channels] ~ N(0, 1))."""
    T, H, W = latent_shape
    rng = np.random.default_rng(seed)
    noise = rng.standard_normal((out_channels, T, H, W), dtype=np.float32)
    cond = rng.standard_normal((out_channels, T, H, W), dtype=np.float32)
    text = rng.standard_normal((text_len, text_channels), dtype=np.float32)
    return noise, cond, text


def block_weights_device(dim, heads, mlp_hidden, shared=False, seed=666, device="cuda"):
    """The block_weights layout and distributions drawn with torch's device RNG
    (identical on every GPU for the same seed), returned as a host fp32 numpy
    array -- fast enough to build a 32-block model on each of several ranks."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)

    def nrm(n, std, mean=0.0):
        return (torch.randn(n, generator=g, device=device) * std + mean)

    def branch():
        parts = [nrm(dim, 0.02) for _ in range(6)]
        parts += [nrm(3 * dim * dim, 0.02), nrm(dim * dim, 0.02), nrm(dim, 0.02), nrm(HEAD_DIM, 0.1, 1.0),
                  nrm(HEAD_DIM, 0.1, 1.0), nrm(mlp_hidden * dim, 0.02), nrm(mlp_hidden * dim, 0.02),
                  nrm(dim * mlp_hidden, 0.02)]
        return parts

    parts = branch() if shared else branch() + branch()
    parts.append(torch.from_numpy(rope_freqs()).to(device))
    return torch.cat(parts).float().cpu().numpy()
