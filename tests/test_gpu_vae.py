"""GPU parity of the VAE mid-block attention (DynamicFramewiseSpatialAttention)
through the C ABI: GroupNorm + fused Q|K|V projection + per-frame tcgen05
attention + output projection with residual.

References: the reference's own CPU outputs for its runner cases (golden
fixtures), the C restatement oracle on identical seeded inputs, its
token-subset variant for full 90x160 frames at C = 512, and a plain PyTorch
fp32 attention for the attention core alone.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import parity
import refcases
import s2b200
from s2b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert s2b200.device_check(0) == 0, s2b200.last_error()
    return torch


def make_layer(C, weights):
    layer = s2b200.DynamicFramewiseSpatialAttention(device=0)
    assert layer.load_param(C) == 0
    layer.load_model(weights)
    return layer


def run_gpu(torch, x, weights):
    layer = make_layer(x.shape[0], weights)
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = layer.forward(xd)
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    assert layer.last_launches() == 5
    return y.cpu().numpy()


def check_vae(y, expected, x, what):
    """y within max-abs 2e-3 of the reference, and the attention branch
    (y - x) itself at cosine >= 0.9999."""
    m = parity.metrics(y, expected)
    assert m["finite"], f"{what}: non-finite {m}"
    assert m["max_abs"] <= parity.MAX_ABS, f"{what}: {m}"
    mb = parity.metrics(y - x, expected - x)
    assert mb["cosine"] >= parity.COSINE, f"{what} (attention branch): {mb}"
    return m, mb


@pytest.mark.parametrize("i", range(len(refcases.VAE_CASES)))
def test_runner_cases_vs_reference(torch_cuda, golden, i):
    x, w, _ = refcases.vae_case(refcases.VAE_CASES[i])
    y = run_gpu(torch_cuda, x, w)
    check_vae(y, golden("vae_runner_cases.npz")[f"c{i}_y"], x, f"runner case {i}")


def test_flat_weight_stream_matches_dict(torch_cuda):
    x, w, flat = refcases.vae_case(refcases.VAE_CASES[0])
    layer = make_layer(x.shape[0], flat)
    y0 = layer.forward(torch_cuda.from_numpy(x).cuda()).cpu().numpy()
    y1 = run_gpu(torch_cuda, x, w)
    assert np.array_equal(y0, y1)


@pytest.mark.parametrize("shape", [(512, 2, 12, 20), (96, 3, 9, 23), (320, 1, 16, 17), (256, 2, 8, 16)])
def test_random_shapes_vs_oracle(torch_cuda, port, shape):
    """Ragged token counts (tails of the last key/query tile), channel
    padding to 128 / 512, several frames, d = 256 and d = 512."""
    x, w = synth.vae_inputs(shape, seed=shape[0] + shape[2])
    y = run_gpu(torch_cuda, x, w)
    check_vae(y, port.vae_attention(x, w), x, f"shape {shape}")


def test_cfg4_full_frames_sampled(torch_cuda, port):
    """Config 4 at full size (C 512, 6 frames of 90x160 = 14,400 tokens):
    every output checked for finiteness, 96 seeded query tokens of the first
    and last frame against the oracle (query-tile edges included)."""
    x, w = synth.vae_inputs(synth.VAE_CFG4)
    C, T, H, W = x.shape
    y = run_gpu(torch_cuda, x, w)
    assert np.isfinite(y).all()
    rng = np.random.default_rng(7)
    N = H * W
    for f in (0, T - 1):
        sel = np.unique(np.concatenate([[0, 127, 128, N - 1, N - 64], rng.choice(N, 91, replace=False)]))
        exp = port.vae_attention_tokens(x, w, f, sel)
        got = y[:, f].reshape(C, N)[:, sel].T
        xs = x[:, f].reshape(C, N)[:, sel].T
        check_vae(got, exp, xs, f"cfg4 frame {f}")


def test_host_forward_and_determinism(torch_cuda):
    x, w = synth.vae_inputs((128, 2, 10, 30), seed=3)
    layer = make_layer(128, w)
    y_host = layer.forward_host(x)
    y_host2 = layer.forward_host(x)
    y_dev = run_gpu(torch_cuda, x, w)
    assert np.array_equal(y_host, y_host2)
    assert np.array_equal(y_host, y_dev)


@pytest.mark.parametrize("shape", [(96, 5, 9, 14), (256, 3, 12, 20)])
def test_host_forward_frame_pipeline(torch_cuda, shape):
    """The host-buffer forward runs frame by frame (upload, forward and download of
    consecutive frames overlapped on three streams). It must equal the device
    forward bit for bit, for a dense blob and for a channel step padded past
    T*H*W, whose padding in y it leaves untouched."""
    x, w = synth.vae_inputs(shape, seed=21)
    C, T, H, W = x.shape
    n = T * H * W
    layer = make_layer(C, w)
    y_dev = run_gpu(torch_cuda, x, w)
    assert np.array_equal(layer.forward_host(x), y_dev)
    cstep = n + 37
    blob = np.full((C, cstep), 7.0, np.float32)
    blob[:, :n] = x.reshape(C, n)
    yb = np.full((C, cstep), -3.0, np.float32)
    for _ in range(2):
        rc = s2b200.lib().s2_vae_attention_forward_host(layer.handle, None, ctypes.c_void_p(blob.ctypes.data), T, H, W,
                                                        cstep, ctypes.c_void_p(yb.ctypes.data))
        assert rc == 0, s2b200.last_error()
        assert np.array_equal(yb[:, :n].reshape(x.shape), y_dev)
        assert np.all(yb[:, n:] == -3.0)


def test_cstep_padded_blob(torch_cuda, port):
    """An ncnn blob whose channel stride exceeds T*H*W (cstep alignment)."""
    torch = torch_cuda
    x, w = synth.vae_inputs((64, 1, 5, 7), seed=11)
    C, T, H, W = x.shape
    cstep = 40
    blob = np.full((C, cstep), 7.0, np.float32)
    blob[:, :T * H * W] = x.reshape(C, -1)
    layer = make_layer(C, w)
    yd = torch.full((C, cstep), -3.0, device="cuda")
    layer.forward(torch.from_numpy(blob).cuda(), y=yd, shape=(T, H, W))
    y = yd.cpu().numpy()
    assert np.all(y[:, T * H * W:] == -3.0)
    check_vae(y[:, :T * H * W].reshape(x.shape), port.vae_attention(x, w), x, "cstep blob")


@pytest.mark.parametrize("channels,frames,tokens", [(512, 2, 1000), (256, 1, 300), (128, 3, 129)])
def test_spatial_attention_core_vs_torch_fp32(torch_cuda, channels, frames, tokens):
    torch = torch_cuda
    P = s2b200.padded_channels(channels)
    g = torch.Generator().manual_seed(channels + tokens)
    q, k, v = [torch.zeros((frames * tokens, P), dtype=torch.float16) for _ in range(3)]
    for t in (q, k, v):
        t[:, :channels] = torch.randn((frames * tokens, channels), generator=g).half()
    out = torch.empty((frames * tokens, P), dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s2b200.spatial_attention(q.cuda(), k.cuda(), v.cuda(), channels, frames, tokens, out, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.float().cpu().reshape(frames, tokens, P)
    qf, kf, vf = (t.float().reshape(frames, tokens, P) for t in (q, k, v))
    ref = torch.softmax(qf @ kf.transpose(1, 2) / channels ** 0.5, dim=-1) @ vf
    assert torch.all(got[..., channels:] == 0)
    parity.check(got.numpy(), ref.numpy(), False, f"core C{channels}")
