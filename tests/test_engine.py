"""seedvr2::SeedVR2Engine (include/seedvr2/engine.h, libseedvr2.so) through its
C++ runner, tests/cpp/engine_runner.cpp -- a caller that includes only the
public engine header, like the reference's install-consumer program.

CPU: the header and runner compile (-Wall -Werror), the library exports the
engine, and the status paths that need no GPU return the reference's codes
(option checks of src/core/vulkan_context.cpp:62-69, missing backends,
process before load).
GPU: a small exported model directory (the reference exporter's layout, with
default_pos_emb.bin / default_neg_emb.bin of different token counts) is
loaded, and process_latent runs a guided, rescaled 2-step sample from VAE
moments. The expected latent comes from the reference's own code: its
sampler loop and DiT layers (oracle/_ref) on the same weights, fed with the
engine's random draws and the condition latent. Gate: the reference's full-DiT
gate (tools/test_seedvr2_dit_ncnn.py:248-250) on the displacement noise - x0.
"""
from __future__ import annotations

import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "seedvr2-ncnn-valkan_b200", "lib")
SRC = os.path.join(ROOT, "tests", "cpp", "engine_runner.cpp")
FLAGS = ["-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I" + os.path.join(ROOT, "include")]


def gxx():
    exe = shutil.which("g++")
    if exe is None:
        pytest.skip("g++ not available")
    return exe


@pytest.fixture(scope="module")
def runner(tmp_path_factory):
    assert os.path.exists(os.path.join(LIBDIR, "libseedvr2.so")), "build the library first"
    exe = str(tmp_path_factory.mktemp("engine") / "engine_runner")
    r = subprocess.run([gxx(), *FLAGS, SRC, "-L" + LIBDIR, "-lseedvr2", "-ls2b200", "-Wl,-rpath," + LIBDIR,
                        "-o", exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return exe


def _lines(out):
    return [ln for ln in out.splitlines() if ln.startswith("[")]


def test_engine_library_exports():
    r = subprocess.run(["nm", "-D", "--defined-only", "-C", os.path.join(LIBDIR, "libseedvr2.so")],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    for sym in ("seedvr2::SeedVR2Engine::load(", "seedvr2::SeedVR2Engine::process(",
                "seedvr2::SeedVR2Engine::process_latent(", "seedvr2::SeedVR2Engine::last_error",
                "seedvr2::SeedVR2Engine::loaded", "seedvr2::status_message", "seedvr2::Video::valid",
                "seedvr2::TextEmbedding::valid"):
        assert sym in r.stdout, sym


def test_status_paths_without_gpu(runner):
    r = subprocess.run([runner, "errors"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = _lines(r.stdout)
    assert len(lines) == 13 and all(" PASS" in ln for ln in lines), r.stdout


def _write_embedding(path, emb):
    with open(path, "wb") as f:
        f.write(np.array(emb.shape, np.int32).tobytes())
        f.write(np.ascontiguousarray(emb, np.float32).tobytes())


@pytest.mark.gpu
def test_process_latent_guided_vs_reference(runner, ref, tmp_path):
    import ncnn_files
    import oracle
    import parity
    import s2b200
    from s2b200 import synth

    dim, heads, mlp, tc, n_blocks = 256, 2, 256, 256, 4
    model = tmp_path / "model"
    dit_dir = model / "dit_full_fp16"
    dit_dir.mkdir(parents=True)
    wi = ncnn_files.write_input(dit_dir, synth.dit_input_weights(dim, 33, tc, 256), dim, tc)
    wo = ncnn_files.write_output(dit_dir, synth.dit_output_weights(dim), dim)
    bws, bps = [], []
    for i in range(n_blocks):
        f = s2b200.block_flags(i, n_blocks)
        bws.append(ncnn_files.write_block(dit_dir, i, synth.block_weights(dim, heads, mlp, f["shared"], seed=60 + i),
                                          dim, heads, mlp, f["shared"], f["last"], f["shifted"]))
        bps.append(dict(block_index=i, dim=dim, heads=heads, head_dim=128, mlp_hidden=mlp, eps=1e-5, **f))
    rng = np.random.default_rng(77)
    pos = rng.standard_normal((7, tc)).astype(np.float32)
    neg = rng.standard_normal((9, tc)).astype(np.float32)
    _write_embedding(model / "default_pos_emb.bin", pos)
    _write_embedding(model / "default_neg_emb.bin", neg)
    T, H, W = 2, 12, 20
    moments = np.concatenate([rng.standard_normal((16, T, H, W)), rng.uniform(-4, 1, (16, T, H, W))])
    moments = moments.astype(np.float32)
    moments.tofile(tmp_path / "moments.bin")
    steps, cfg, rescale, noise_scale, seed = 2, 2.5, 0.5, 0.1, 1234
    r = subprocess.run([runner, "run", str(model), str(tmp_path / "moments.bin"), str(tmp_path), "32", str(T), str(H),
                        str(W), str(steps), str(cfg), str(rescale), str(noise_scale), str(seed), "1"],
                       capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert all(" PASS" in ln for ln in _lines(r.stdout)), r.stdout

    def load(name):
        return np.fromfile(tmp_path / name, np.float32).reshape(16, T, H, W)

    x0, encoded, noise, augment = (load(n) for n in ("x0.bin", "encoded.bin", "noise.bin", "augment.bin"))
    condition = oracle.SamplerPort(oracle.port().lib).make_condition(encoded, augment, noise_scale)
    hp = dict(dim=dim, text_channels=tc, sinusoidal_dim=256, embedding_dim=6 * dim, out_channels=16, eps=1e-5)
    want = ref.sample(hp, wi, bps, bws, wo, noise, condition, pos, neg, steps, cfg, rescale)
    m = parity.metrics(noise - x0, noise - want)
    assert m["finite"] and m["nrmse"] <= 0.02 and m["cosine"] >= 0.9998, m
