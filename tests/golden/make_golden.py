"""Generates tests/golden/*.npz from the reference's OWN CPU code.

Run in the build container (needs oracle/_ref/libs2ref.so, i.e. the reference
tree at build time):  python tests/golden/make_golden.py
The fixtures pin the C restatement (tests/test_oracle.py) and are the
committed parity targets of the GPU path (tests/test_gpu_attention.py).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "seedvr2-ncnn-valkan_b200"))

import oracle  # noqa: E402
import refcases  # noqa: E402
from s2b200 import synth  # noqa: E402

WINDOW_GRIDS = [(2, 16, 30), (6, 45, 80), (12, 67, 120), (2, 2, 2), (1, 1, 1), (3, 2, 2), (5, 64, 64),
                (9, 80, 96), (5, 240, 320), (21, 90, 160), (1, 7, 3), (4, 33, 33), (31, 17, 5), (45, 134, 240),
                (2, 30, 40), (1, 60, 60), (30, 1, 1), (8, 16, 16)]


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 values that are exactly bf16 -> their upper 16 bits."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    assert np.all((u & 0xFFFF) == 0), "value not bf16-representable"
    return (u >> 16).astype(np.uint16)


def main():
    ref = oracle.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libs2ref.so missing: build it with `make -C oracle ref`")

    # 1. window boxes, reference rule
    win = {}
    for g in WINDOW_GRIDS:
        for s in (0, 1):
            win[f"{g[0]}x{g[1]}x{g[2]}_s{s}"] = ref.make_windows(*g, s)
    np.savez_compressed(os.path.join(HERE, "windows.npz"), **win)

    # 2. config-0 grid, one head, seeded N(0,1) fp16-representable inputs
    grid = synth.GRIDS["cfg0"]
    vid, txt, gam, freqs = synth.layer_inputs(grid, heads=1, seed=666)
    out = dict(grid=np.array(grid, np.int32), vid_qkv=vid.astype(np.float16), txt_qkv=txt.astype(np.float16),
               gammas=gam, freqs=freqs)
    for s in (0, 1):
        vo, to, pk = ref.attention(vid, txt, grid, 1, list(gam), freqs, s, packed=True)
        out[f"vid_out_s{s}"] = bf16_bits(vo)
        out[f"txt_out_s{s}"] = to
        out[f"packed_o_s{s}"] = bf16_bits(pk["o"])
        if s == 0:
            for k in "qkv":
                out[f"packed_{k}_s0"] = bf16_bits(pk[k])
    np.savez_compressed(os.path.join(HERE, "attn_cfg0_h1.npz"), **out)

    # 3. the reference runner's block cases at the attention stage
    att = {}
    for i, case in enumerate(refcases.BLOCK_CASES):
        vq, tq, g4, fr, shape, heads, shifted = refcases.attention_case(case)
        vo, to, pk = ref.attention(vq, tq, shape, heads, list(g4), fr, shifted, packed=True)
        att[f"c{i}_vid_out"] = vo
        att[f"c{i}_txt_out"] = to
        att[f"c{i}_packed_o"] = pk["o"]
    np.savez_compressed(os.path.join(HERE, "attn_runner_cases.npz"), **att)

    # 4. the same cases through the full block forward (shim InnerProduct; see oracle/ncnn_shim)
    blk = {}
    for i, case in enumerate(refcases.BLOCK_CASES):
        params, weights, vid_b, txt_b, emb, shape, _, _ = refcases.block_case(case)
        vo, to = ref.block_forward(params, weights, vid_b, txt_b, emb, shape)
        blk[f"c{i}_vid_out"] = vo
        blk[f"c{i}_txt_out"] = to
    np.savez_compressed(os.path.join(HERE, "block_runner_cases.npz"), **blk)

    # 5. the reference VAE-attention runner cases
    vae = {}
    for i, case in enumerate(refcases.VAE_CASES):
        x, _, flat = refcases.vae_case(case)
        vae[f"c{i}_y"] = ref.vae_attention(x, flat)
    np.savez_compressed(os.path.join(HERE, "vae_runner_cases.npz"), **vae)

    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
