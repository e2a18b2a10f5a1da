"""Writes model files in the layout of the reference's exporter
(tools/export_seedvr2_dit_ncnn.py): an ncnn .param graph of Input layers plus
the custom layer with its ParamDict, and a .bin of weight blobs in load_model
order -- raw fp32 vectors, and InnerProduct weights behind a 4-byte tag
(0x01306B47: fp16, padded to 4 bytes; 0: fp32). Test infrastructure: builds
synthetic model directories for the library's readers.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

FP16_TAG = 0x01306B47


def write_param(path: Path, layer: str, inputs, outputs, params: dict):
    lines = [f"Input input_{b} 0 1 {b}" for b in inputs]
    kv = " ".join(f"{k}={v:e}" if isinstance(v, float) else f"{k}={int(v)}" for k, v in params.items())
    lines.append(" ".join([layer, path.name.split(".")[0], str(len(inputs)), str(len(outputs)), *inputs, *outputs, kv]))
    blobs = len(set(inputs) | set(outputs))
    path.write_text(f"7767517\n{len(lines)} {blobs}\n" + "\n".join(lines) + "\n")


def write_bin(path: Path, stream: np.ndarray, schedule, storage="fp16") -> np.ndarray:
    """schedule: (count, tagged) blobs covering `stream`. Returns the values a
    reader must produce (tagged blobs rounded to fp16 when stored as fp16)."""
    out, expect, at = [], [], 0
    for count, tagged in schedule:
        v = np.asarray(stream[at:at + count], np.float32)
        at += count
        if tagged and storage == "fp16":
            h = v.astype("<f2")
            raw = h.tobytes()
            out += [struct.pack("<I", FP16_TAG), raw, b"\0" * ((-len(raw)) % 4)]
            expect.append(h.astype(np.float32))
        else:
            if tagged:
                out.append(struct.pack("<I", 0))
            out.append(v.astype("<f4").tobytes())
            expect.append(v)
    assert at == stream.size
    path.write_bytes(b"".join(out))
    return np.concatenate(expect)


def block_schedule(dim, mlp, shared, head_dim=128):
    br = [(6 * dim, False), (3 * dim * dim, True), (dim * dim, True), (dim, False), (head_dim, False),
          (head_dim, False), (mlp * dim, True), (mlp * dim, True), (dim * mlp, True)]
    return br * (1 if shared else 2) + [(21, False)]


def input_schedule(dim, vc=33, tc=5120, sd=256):
    s = []
    for n_in, n_out in ((4 * vc, dim), (tc, dim), (sd, dim), (dim, dim), (dim, 6 * dim)):
        s += [(n_in * n_out, True), (n_out, False)]
    return s


def output_schedule(dim, oc=16):
    return [(3 * dim, False), (4 * oc * dim, True), (4 * oc, False)]


def write_block(root: Path, index, stream, dim, heads, mlp, shared, last, shifted, storage="fp16", eps=1e-5):
    stem = root / f"seedvr2_dit_block_{index:02d}.ncnn"
    write_param(Path(f"{stem}.param"), "SeedVR2DiTBlock", ("vid", "txt", "emb", "vid_shape"), ("vid_out", "txt_out"),
                {0: index, 1: shared, 2: last, 3: shifted, 4: dim, 5: heads, 6: 128, 7: mlp, 8: float(eps)})
    return write_bin(Path(f"{stem}.bin"), stream, block_schedule(dim, mlp, shared), storage)


def write_input(root: Path, stream, dim, tc=5120, storage="fp16"):
    write_param(root / "seedvr2_dit_input.ncnn.param", "SeedVR2DiTInput", ("vid", "txt", "timestep", "vid_shape"),
                ("vid_out", "txt_out", "emb", "patched_shape"), {0: dim, 1: 33, 2: tc, 3: 256, 4: 6 * dim})
    return write_bin(root / "seedvr2_dit_input.ncnn.bin", stream, input_schedule(dim, tc=tc), storage)


def write_output(root: Path, stream, dim, storage="fp16"):
    write_param(root / "seedvr2_dit_output.ncnn.param", "SeedVR2DiTOutput", ("vid", "emb", "vid_shape"),
                ("vid_out", "output_shape"), {0: dim, 1: 16, 2: 1e-5})
    return write_bin(root / "seedvr2_dit_output.ncnn.bin", stream, output_schedule(dim), storage)
