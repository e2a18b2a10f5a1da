"""Deterministic inputs of the reference's own layer test runners, restated.

* tests/dit_block_vulkan_runner.cpp of the reference: fill() :43-53, weight
  stream write_vec / write_ip / write_branch :80-119, the 4 cases :213-218.
* tests/attention_vulkan_runner.cpp: make_input() :83-95, weights :50-68 in
  load_model order :73-75, the 4 cases :155-160. Its fill() evaluates
  ``(i % 7) - 3`` in size_t, which wraps to ~1.8e19 for i % 7 < 3; the
  evidently intended signed value is used here.
"""
from __future__ import annotations

import numpy as np

# (dim, heads, head_dim, mlp_hidden, T, H, W, text_len, shared, last, shifted)
BLOCK_CASES = [
    (128, 1, 128, 128, 2, 2, 2, 3, False, False, False),
    (128, 1, 128, 128, 2, 2, 2, 3, False, False, True),
    (128, 1, 128, 128, 1, 1, 1, 2, True, True, False),
    (256, 2, 128, 128, 3, 2, 2, 4, False, False, False),
]

# (C, T, H, W)
VAE_CASES = [(32, 2, 4, 4), (64, 3, 5, 5), (32, 1, 8, 8), (64, 2, 3, 5)]


def fill(cols: int, rows: int, off: int) -> np.ndarray:
    idx = np.arange(rows * cols, dtype=np.int64)
    return (((idx + off) % 11 - 5).astype(np.float32) * np.float32(0.1)).reshape(rows, cols)


def vec(n: int, seed: int) -> np.ndarray:
    i = np.arange(n, dtype=np.int64)
    return np.float32(0.01) * ((i + seed) % 9 - 4).astype(np.float32)


def ip(n_in: int, n_out: int, bias: bool, seed: int) -> list[np.ndarray]:
    i = np.arange(n_in * n_out, dtype=np.int64)
    out = [np.float32(0.005) * ((i + seed) % 7 - 3).astype(np.float32)]
    if bias:
        j = np.arange(n_out, dtype=np.int64)
        out.append(np.float32(0.01) * ((j + seed) % 5 - 2).astype(np.float32))
    return out


def branch(dim: int, head_dim: int, mlp: int, base: int) -> dict[str, np.ndarray]:
    b = {}
    for k, name in enumerate(["attn_shift", "attn_scale", "attn_gate", "mlp_shift", "mlp_scale", "mlp_gate"]):
        b[name] = vec(dim, base + k)
    b["qkv"] = ip(dim, 3 * dim, False, base + 6)[0]
    b["proj_w"], b["proj_b"] = ip(dim, dim, True, base + 7)
    b["norm_q"] = vec(head_dim, base + 8)
    b["norm_k"] = vec(head_dim, base + 9)
    b["gate_w"] = ip(dim, mlp, False, base + 10)[0]
    b["in_w"] = ip(dim, mlp, False, base + 11)[0]
    b["out_w"] = ip(mlp, dim, False, base + 12)[0]
    return b


BRANCH_ORDER = ["attn_shift", "attn_scale", "attn_gate", "mlp_shift", "mlp_scale", "mlp_gate", "qkv", "proj_w",
                "proj_b", "norm_q", "norm_k", "gate_w", "in_w", "out_w"]


def block_case(case):
    """Returns (params, weight stream, vid, txt, emb, shape, gammas[4], freqs) of one block case."""
    dim, heads, hd, mlp, T, H, W, lt, shared, last, shifted = case
    vb = branch(dim, hd, mlp, 0)
    tb = vb if shared else branch(dim, hd, mlp, 50)
    stream = [vb[k] for k in BRANCH_ORDER]
    if not shared:
        stream += [tb[k] for k in BRANCH_ORDER]
    freqs = vec(21, 100)
    stream.append(freqs)
    weights = np.concatenate([s.ravel() for s in stream]).astype(np.float32)
    params = dict(block_index=0, shared=shared, last=last, shifted=shifted, dim=dim, heads=heads, head_dim=hd,
                  mlp_hidden=mlp, eps=1e-5)
    vid = fill(dim, T * H * W, 0)
    txt = fill(dim, lt, 100)
    emb = fill(dim * 6, 1, 200).ravel()
    gammas = np.stack([vb["norm_q"], vb["norm_k"], tb["norm_q"], tb["norm_k"]])
    return params, weights, vid, txt, emb, (T, H, W), gammas, freqs


def attention_case(case):
    """The same case at the attention stage: QKV rows from fill(), runner gammas and freqs."""
    dim, heads, hd, mlp, T, H, W, lt, shared, last, shifted = case
    _, _, _, _, _, shape, gammas, freqs = block_case(case)
    vid_qkv = fill(3 * dim, T * H * W, 0)
    txt_qkv = fill(3 * dim, lt, 100)
    return vid_qkv, txt_qkv, gammas, freqs, shape, heads, shifted


def vae_case(case):
    """(x [C,T,H,W], weights dict, flat weight stream in load_model order)."""
    C, T, H, W = case

    def f(n, base, step):
        i = np.arange(n, dtype=np.int64)
        return (np.float32(base) + np.float32(step) * ((i % 7) - 3).astype(np.float32)).astype(np.float32)

    m = C * C
    w = {"norm_bias": f(C, 0, 0.02), "norm_weight": f(C, 1, 0.02), "q_bias": f(C, 0, 0.01),
         "q_weight": f(m, 0, 0.005), "k_bias": f(C, 0, 0.01), "k_weight": f(m, 0, 0.005),
         "v_bias": f(C, 0, 0.01), "v_weight": f(m, 0, 0.005), "out_bias": f(C, 0, 0.01),
         "out_weight": f(m, 0, 0.005)}
    order = ["norm_bias", "norm_weight", "k_bias", "k_weight", "out_bias", "out_weight", "q_bias", "q_weight",
             "v_bias", "v_weight"]
    flat = np.concatenate([w[k] for k in order])
    idx = np.arange(C * T * H * W, dtype=np.int64)
    x = ((idx % 11 - 5).astype(np.float32) * np.float32(0.1)).reshape(C, T, H, W)
    return x, w, flat
