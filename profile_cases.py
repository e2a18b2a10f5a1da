"""Single-layer cases at the production shapes, run on cuda:0 for profiling one
kernel in isolation (an ncu capture with several passes needs a program that
holds a few GB at most; the 32-block Euler step holds far more).

    python profile_cases.py block720p
    python profile_cases.py vae_cfg4

block720p: one unshared, plain-window DiT block (dim 2560, 20 heads, SwiGLU
    6912) over the 720p token grid 6x45x80 plus 58 text rows, random-init
    weights, three forwards (kernel order per forward: RMSNorm+adaLN, video
    QKV GEMM, text QKV GEMM, prologue, window attention, text mean, ...).
vae_cfg4: the VAE mid-block attention layer at 512 channels x 6 frames of
    90x160, three forwards.

Each case prints one JSON line with its device ms per forward (CUDA events)
and exits non-zero on a device error.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "seedvr2-ncnn-valkan_b200"))

from s2b200 import DynamicFramewiseSpatialAttention, SeedVR2DiTBlock, synth  # noqa: E402

CASES = ("block720p", "vae_cfg4")


def _time(torch, fn, reps):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def block720p(torch, reps=3):
    grid, dim = synth.GRIDS["cfg2"], 2560
    b = SeedVR2DiTBlock(device=0)
    b.load_param(block_index=0, shared=False, last=False, shifted=False, dim=dim, heads=20, mlp_hidden=6912)
    b.load_model(synth.block_weights_device(dim, 20, 6912, shared=False, seed=100, device="cuda:0"))
    b.set_runtime_shape(*grid)
    vid, txt, emb = (torch.from_numpy(a).cuda() for a in synth.block_activations(grid, dim))
    vo, to = torch.empty_like(vid), torch.empty_like(txt)
    ms = _time(torch, lambda: b.forward(vid, txt, emb, vo, to), reps)
    err = b.device_error()
    b.close()
    return {"case": "block720p", "ms_per_forward": ms, "device_error": err,
            "finite": bool(torch.isfinite(vo).all().item())}


def vae_cfg4(torch, reps=3):
    shape = synth.VAE_CFG4
    x, w = synth.vae_inputs(shape)
    lay = DynamicFramewiseSpatialAttention(device=0)
    lay.load_param(shape[0])
    lay.load_model(w)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty_like(xd)
    ms = _time(torch, lambda: lay.forward(xd, y), reps)
    err = lay.device_error()
    lay.close()
    return {"case": "vae_cfg4", "ms_per_forward": ms, "device_error": err,
            "finite": bool(torch.isfinite(y).all().item())}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=CASES)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    import torch
    assert torch.cuda.is_available(), "the cases run on a CUDA device"
    torch.cuda.set_device(0)
    out = {"block720p": block720p, "vae_cfg4": vae_cfg4}[args.case](torch, args.reps)
    print(json.dumps(out), flush=True)
    if out["device_error"] != 0 or not out["finite"]:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
