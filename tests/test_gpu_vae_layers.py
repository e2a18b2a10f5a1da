"""GPU parity of the VAE's GroupNorm, space-time shuffle and Conv3D layers
(s2_vae_group_norm_*, s2_vae_space_time_shuffle_*, s2_vae_conv3d_*) through
the C ABI.

References: the reference's own DynamicFramewiseGroupNorm and
DynamicSpaceTimeShuffle (oracle/_ref, built from its sources) and, for
Convolution3D -- ncnn's layer, which the reference only patches -- the C
restatement of the patch's formula (oracle/s2_oracle.c, pinned against
PyTorch's conv3d in tests/test_oracle.py). Full config-4 sizes are checked
on sampled output positions recomputed here in float64.

Tolerances: GroupNorm keeps the reference's float arithmetic (its double sums
are only re-associated), so it is gated at 1e-5 absolute with >= 99.9 % of
elements bit-equal. The projection and the convolution take fp16 operands
with fp32 accumulation (the reference: fp32 operands, double / fp32
accumulation): max-abs <= 2e-3 and cosine >= 0.9999, on inputs and weights
scaled so outputs are O(1).
"""
from __future__ import annotations

import numpy as np
import pytest

import parity
import s2b200

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert s2b200.device_check(0) == 0, s2b200.last_error()
    return torch


def _x(shape, seed):
    """N(0, 1) inputs, fp16-representable (both sides read the same numbers)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal(shape, dtype=np.float32).astype(np.float16).astype(np.float32)


def _check_fp16_path(got, want, what):
    m = parity.metrics(got, want)
    assert m["finite"] and m["max_abs"] <= parity.MAX_ABS and m["cosine"] >= parity.COSINE, f"{what}: {m}"
    return m


# ---- GroupNorm -----------------------------------------------------------------

@pytest.mark.parametrize("shape", [(32, 2, 4, 4), (64, 3, 5, 7), (128, 1, 16, 16), (512, 6, 90, 160)])
def test_group_norm_vs_reference(torch_cuda, ref, shape):
    torch = torch_cuda
    rng = np.random.default_rng(shape[0])
    x = (_x(shape, 1) * 1.5 + 0.25).astype(np.float32)
    b = (0.1 * rng.standard_normal(shape[0])).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(shape[0])).astype(np.float32)
    layer = s2b200.DynamicFramewiseGroupNorm()
    layer.load_param(shape[0])
    layer.load_model(b, w)
    y = layer.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    want = ref.group_norm(x, b, w)
    m = parity.metrics(y.cpu().numpy(), want)
    assert m["max_abs"] <= 1e-5 and m["exact_frac"] >= 0.999, m
    assert layer.last_launches() == 2
    # host-buffer call: same bytes
    assert np.array_equal(layer.forward_host(x), y.cpu().numpy())


def test_group_norm_on_padded_blobs(torch_cuda, ref):
    """ncnn blobs carry a channel stride (cstep) past the plane; input and
    output strides may differ."""
    torch = torch_cuda
    C, T, H, W = 64, 2, 5, 7
    plane = T * H * W
    x = _x((C, T, H, W), 2)
    b = np.linspace(-0.1, 0.1, C).astype(np.float32)
    w = np.linspace(0.9, 1.1, C).astype(np.float32)
    xb = np.full((C, plane + 6), np.nan, np.float32)
    xb[:, :plane] = x.reshape(C, plane)
    layer = s2b200.DynamicFramewiseGroupNorm()
    layer.load_param(C)
    layer.load_model(b, w)
    dx = torch.from_numpy(xb).cuda()
    dy = torch.full((C, plane + 10), 7.0, device="cuda")
    rc = s2b200.lib().s2_vae_group_norm_forward(layer.handle, s2b200._stream_ptr(), s2b200._ptr(dx), T, H, W,
                                                 plane + 6, s2b200._ptr(dy), plane + 10)
    assert rc == 0, s2b200.last_error()
    torch.cuda.synchronize()
    y = dy.cpu().numpy()
    assert np.all(y[:, plane:] == 7.0), "wrote past the channel plane"
    m = parity.metrics(y[:, :plane].reshape(C, T, H, W), ref.group_norm(x, b, w))
    assert m["max_abs"] <= 1e-5, m


# ---- space-time shuffle -----------------------------------------------------------

def _sts_weights(cin, tr, seed):
    rng = np.random.default_rng(seed)
    P = cin * 4 * tr
    w = (rng.standard_normal((P, cin)) / np.sqrt(cin)).astype(np.float32)
    b = (0.1 * rng.standard_normal(P)).astype(np.float32)
    return b, w


def _sts_layer(cin, tr, b, w):
    layer = s2b200.DynamicSpaceTimeShuffle()
    layer.load_param(cin, cin * 4 * tr)
    layer.load_model(b, w)
    return layer


@pytest.mark.parametrize("cin,tr,grid", [(32, 1, (1, 3, 5)), (64, 2, (3, 4, 6)), (96, 2, (2, 5, 3)),
                                         (512, 2, (2, 16, 24))])
def test_space_time_shuffle_vs_reference(torch_cuda, ref, cin, tr, grid):
    torch = torch_cuda
    b, w = _sts_weights(cin, tr, cin + tr)
    x = _x((cin,) + grid, 3)
    layer = _sts_layer(cin, tr, b, w)
    y = layer.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    want = ref.space_time_shuffle(x, b, w)
    assert y.shape == want.shape
    _check_fp16_path(y.cpu().numpy(), want, f"space-time shuffle {cin} x{tr} {grid}")
    assert layer.last_launches() == 2
    assert np.array_equal(layer.forward_host(x), y.cpu().numpy())


def test_space_time_shuffle_config4_sampled(torch_cuda):
    """The decoder's shuffle at the config-4 latent (512 channels, 6 x 90 x 160,
    temporal ratio 2 -> 11 x 180 x 320): every output position of 200 sampled
    input tokens, recomputed in float64 from the layer's definition."""
    torch = torch_cuda
    cin, tr, (T, H, W) = 512, 2, (6, 90, 160)
    b, w = _sts_weights(cin, tr, 9)
    x = _x((cin, T, H, W), 4)
    layer = _sts_layer(cin, tr, b, w)
    y = layer.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    y = y.cpu().numpy()
    assert y.shape == (cin, 2 * T - 1, 2 * H, 2 * W) and np.isfinite(y).all()
    rng = np.random.default_rng(5)
    toks = np.stack([rng.integers(0, T, 200), rng.integers(0, H, 200), rng.integers(0, W, 200)], 1)
    toks[0] = (0, 0, 0)
    toks[1] = (T - 1, H - 1, W - 1)
    got, want = [], []
    for f, yy, xx in toks:
        proj = w.astype(np.float64) @ x[:, f, yy, xx].astype(np.float64) + b  # [P]
        for oy in range(2):
            for ox in range(2):
                for ot in range(tr):
                    raw = f * tr + ot
                    if raw == 1:
                        continue
                    of = raw - 1 if raw > 1 else raw
                    p0 = ((oy * 2 + ox) * tr + ot) * cin
                    got.append(y[:, of, 2 * yy + oy, 2 * xx + ox])
                    want.append(proj[p0:p0 + cin])
    _check_fp16_path(np.array(got), np.array(want), "config-4 shuffle (sampled)")


# ---- Convolution3D ----------------------------------------------------------------

def _conv_weights(cout, cin, k, seed, bias=True):
    rng = np.random.default_rng(seed)
    fan_in = cin * k[0] * k[1] * k[2]
    w = (rng.standard_normal((cout, cin) + tuple(k)) * (0.5 / np.sqrt(fan_in))).astype(np.float32)
    b = (0.1 * rng.standard_normal(cout)).astype(np.float32) if bias else None
    return w, b


def _conv_layer(cin, cout, w, b, k, s, d, p):
    layer = s2b200.Convolution3D()
    layer.load_param(cin, cout, kernel=k, dilation=d, stride=s, pad=p, bias_term=b is not None)
    layer.load_model(w, b)
    return layer


CONV_CASES = [
    # (cin, cout, input T,H,W, kernel, stride, dilation, pad (front, top, left, behind, bottom, right))
    (64, 64, (3, 6, 40), (3, 3, 3), (1, 1, 1), (1, 1, 1), (0, 1, 1, 0, 1, 1)),   # the causal 3x3x3 conv
    (32, 96, (4, 5, 33), (3, 3, 3), (1, 1, 1), (1, 1, 1), (0, 1, 1, 0, 1, 1)),   # ow 33: padded to 64
    (96, 40, (2, 7, 20), (1, 1, 1), (1, 1, 1), (1, 1, 1), (0, 0, 0, 0, 0, 0)),   # 1x1x1, cin not / 64
    (64, 64, (3, 9, 66), (3, 3, 3), (1, 2, 2), (1, 1, 1), (0, 1, 1, 0, 1, 1)),   # spatial stride 2
    (32, 32, (5, 8, 32), (3, 3, 3), (2, 1, 1), (1, 2, 2), (1, 2, 2, 1, 2, 2)),   # temporal stride, dilation
    (32, 64, (3, 6, 17), (3, 3, 3), (1, 1, 1), (1, 1, 1), (-233,) * 6),           # SAME_UPPER
]


@pytest.mark.parametrize("case", range(len(CONV_CASES)))
@pytest.mark.parametrize("bias", [True, False])
def test_conv3d_vs_restatement(torch_cuda, port, case, bias):
    torch = torch_cuda
    cin, cout, grid, k, s, d, p = CONV_CASES[case]
    w, b = _conv_weights(cout, cin, k, 11 + case, bias)
    x = _x((cin,) + grid, 6 + case)
    layer = _conv_layer(cin, cout, w, b, k, s, d, p)
    y = layer.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    if p[0] in (-233, -234):
        # SAME: the restatement takes the resolved pads (ncnn's rule for stride 1: total k - 1, upper half after)
        tot = [kk - 1 for kk in k]
        pp = (tot[0] // 2, tot[1] // 2, tot[2] // 2, tot[0] - tot[0] // 2, tot[1] - tot[1] // 2, tot[2] - tot[2] // 2)
    else:
        pp = p
    want = port.conv3d(x, w, b, stride=s, dilation=d, pad=pp)
    assert tuple(y.shape) == want.shape
    _check_fp16_path(y.cpu().numpy(), want, f"conv case {case} bias={bias}")
    assert layer.last_launches() == 2
    assert np.array_equal(layer.forward_host(x), y.cpu().numpy())


def test_conv3d_config4_sampled(torch_cuda):
    """A 512 -> 512 causal 3x3x3 convolution over the config-4 latent
    (6 frames of 90 x 160, two replicated leading frames as the exporter's
    causal padding): 64 sampled output positions x all 512 channels,
    recomputed in float64."""
    torch = torch_cuda
    cin = cout = 512
    T, H, W = 6, 90, 160
    x = _x((cin, T, H, W), 8)
    xc = np.concatenate([x[:, :1], x[:, :1], x], axis=1)  # causal time padding (replicated first frame)
    k = (3, 3, 3)
    w, b = _conv_weights(cout, cin, k, 21)
    layer = _conv_layer(cin, cout, w, b, k, (1, 1, 1), (1, 1, 1), (0, 1, 1, 0, 1, 1))
    y = layer.forward(torch.from_numpy(xc).cuda())
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    y = y.cpu().numpy()
    assert y.shape == (cout, T, H, W) and np.isfinite(y).all()
    xp = np.pad(xc, ((0, 0), (0, 0), (1, 1), (1, 1))).astype(np.float64)
    wf = w.reshape(cout, -1).astype(np.float64)
    rng = np.random.default_rng(12)
    pos = [(0, 0, 0), (T - 1, H - 1, W - 1), (2, 0, W - 1)] + [
        (int(rng.integers(T)), int(rng.integers(H)), int(rng.integers(W))) for _ in range(61)]
    got = np.array([y[:, z, i, j] for z, i, j in pos])
    want = np.array([wf @ xp[:, z:z + 3, i:i + 3, j:j + 3].reshape(-1) + b for z, i, j in pos])
    _check_fp16_path(got, want, "config-4 conv (sampled)")


def test_conv3d_rejects_unsupported(torch_cuda):
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.Convolution3D().load_param(8, 8, pad_value=1.0)
    assert e.value.status == s2b200.S2_UNSUPPORTED
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.Convolution3D().load_param(8, 8, pad=(-1, 0, 0, 0, 0, 0))
    assert e.value.status == s2b200.S2_INVALID_ARGUMENT
