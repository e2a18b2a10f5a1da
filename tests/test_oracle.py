"""The C restatement oracle, pinned against the reference's own outputs.

Golden fixtures come from the reference's CPU layer code built unmodified
(tests/golden/make_golden.py). Same floating-point flags on both sides, so
the restatement must match bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest

import refcases
from conftest import from_bf16_bits
from s2b200 import synth


def test_windows_match_reference(port, golden):
    g = golden("windows.npz")
    assert len(g.files) >= 30
    for key in g.files:
        dims, s = key.split("_s")
        T, H, W = map(int, dims.split("x"))
        assert np.array_equal(port.make_windows(T, H, W, int(s)), g[key]), key


@pytest.mark.parametrize("shifted", [0, 1])
def test_attention_cfg0_one_head_bit_exact(port, golden, shifted):
    g = golden("attn_cfg0_h1.npz")
    grid = tuple(int(x) for x in g["grid"])
    vo, to, pk = port.window_attention(g["vid_qkv"].astype(np.float32), g["txt_qkv"].astype(np.float32), grid, 1,
                                       list(g["gammas"]), g["freqs"], shifted, packed=True)
    assert np.array_equal(vo, from_bf16_bits(g[f"vid_out_s{shifted}"]))
    assert np.array_equal(to, g[f"txt_out_s{shifted}"])
    assert np.array_equal(pk["o"], from_bf16_bits(g[f"packed_o_s{shifted}"]))
    if shifted == 0:
        for k in "qkv":
            assert np.array_equal(pk[k], from_bf16_bits(g[f"packed_{k}_s0"])), k


@pytest.mark.parametrize("i", range(len(refcases.BLOCK_CASES)))
def test_attention_runner_cases_bit_exact(port, golden, i):
    g = golden("attn_runner_cases.npz")
    vq, tq, g4, fr, shape, heads, shifted = refcases.attention_case(refcases.BLOCK_CASES[i])
    vo, to, pk = port.window_attention(vq, tq, shape, heads, list(g4), fr, shifted, packed=True)
    assert np.array_equal(vo, g[f"c{i}_vid_out"])
    assert np.array_equal(to, g[f"c{i}_txt_out"])
    assert np.array_equal(pk["o"], g[f"c{i}_packed_o"])


@pytest.mark.parametrize("i", range(len(refcases.VAE_CASES)))
def test_vae_runner_cases_bit_exact(port, golden, i):
    g = golden("vae_runner_cases.npz")
    x, w, _ = refcases.vae_case(refcases.VAE_CASES[i])
    y = port.vae_attention(x, w)
    assert np.array_equal(y, g[f"c{i}_y"])


def test_unrounded_variant_is_close_and_round_consistent(port):
    """round_out=0 is the reference Vulkan shader's output (no bf16 rounding)."""
    vid, txt, gam, freqs = synth.layer_inputs((1, 6, 7), heads=2, text_len=5, seed=3)
    a, ta, _ = port.window_attention(vid, txt, (1, 6, 7), 2, list(gam), freqs, 0, round_out=True)
    b, tb, _ = port.window_attention(vid, txt, (1, 6, 7), 2, list(gam), freqs, 0, round_out=False)
    rounded = np.vectorize(port.lib.s2o_round_bf16, otypes=[np.float32])(b)
    assert np.array_equal(a, rounded)
    assert np.allclose(ta, tb, atol=1e-2)


def test_heads_and_window_subsets_partition_the_output(port):
    grid = (2, 9, 11)
    vid, txt, gam, freqs = synth.layer_inputs(grid, heads=3, text_len=7, seed=5)
    full, tfull, _ = port.window_attention(vid, txt, grid, 3, list(gam), freqs, 1)
    n = len(port.make_windows(*grid, 1))
    acc = np.zeros_like(full)
    tacc = np.zeros_like(tfull)
    for hb in range(3):
        for part in (np.arange(n) % 2 == 0, np.arange(n) % 2 == 1):
            v, t, _ = port.window_attention(vid, txt, grid, 3, list(gam), freqs, 1, heads_range=(hb, hb + 1),
                                            window_mask=part)
            acc += v
            tacc += t
    assert np.array_equal(acc, full)
    assert np.allclose(tacc, tfull, rtol=1e-6, atol=1e-7)


def test_restatement_matches_reference_live(port, ref):
    """Beyond the fixtures: a fresh seeded case, 2 heads, both layer kinds."""
    grid = (3, 10, 14)
    vid, txt, gam, freqs = synth.layer_inputs(grid, heads=2, seed=11)
    for s in (0, 1):
        a = port.window_attention(vid, txt, grid, 2, list(gam), freqs, s, packed=True)
        b = ref.attention(vid, txt, grid, 2, list(gam), freqs, s, packed=True)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
        for k in "qkvo":
            assert np.array_equal(a[2][k], b[2][k])


@pytest.mark.parametrize("i", range(len(refcases.VAE_CASES)))
def test_vae_token_subset_equals_full(port, i):
    x, w, _ = refcases.vae_case(refcases.VAE_CASES[i])
    C, T, H, W = x.shape
    y = port.vae_attention(x, w)
    for f in range(T):
        sel = np.arange(H * W)[::-1].copy()
        assert np.array_equal(port.vae_attention_tokens(x, w, f, sel), y[:, f].reshape(C, -1)[:, sel].T)


# ---- the VAE's GroupNorm, space-time shuffle and Conv3D ----------------------

@pytest.mark.parametrize("shape", [(32, 1, 4, 4), (64, 3, 10, 12), (96, 2, 5, 7)])
def test_group_norm_restatement_matches_reference(port, ref, shape):
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape) * 2 + 0.5).astype(np.float32)
    b = rng.standard_normal(shape[0]).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(shape[0])).astype(np.float32)
    assert np.array_equal(port.group_norm(x, b, w), ref.group_norm(x, b, w))


@pytest.mark.parametrize("cin,tr,grid", [(32, 1, (1, 3, 5)), (64, 2, (3, 4, 6)), (32, 2, (1, 2, 2))])
def test_space_time_shuffle_restatement_matches_reference(port, ref, cin, tr, grid):
    rng = np.random.default_rng(cin + tr)
    P = cin * 4 * tr
    x = rng.standard_normal((cin,) + grid).astype(np.float32)
    b = (0.02 * rng.standard_normal(P)).astype(np.float32)
    w = (0.05 * rng.standard_normal((P, cin))).astype(np.float32)
    a, r = port.space_time_shuffle(x, b, w), ref.space_time_shuffle(x, b, w)
    assert a.shape == (cin, grid[0] * tr - 1 if tr > 1 else grid[0], 2 * grid[1], 2 * grid[2])
    assert np.array_equal(a, r)


@pytest.mark.parametrize("case", [
    dict(k=(3, 3, 3), s=(1, 1, 1), d=(1, 1, 1), p=(0, 1, 1, 0, 1, 1)),
    dict(k=(3, 3, 3), s=(1, 2, 2), d=(1, 1, 1), p=(0, 1, 1, 0, 1, 1)),
    dict(k=(1, 1, 1), s=(1, 1, 1), d=(1, 1, 1), p=(0, 0, 0, 0, 0, 0)),
    dict(k=(3, 3, 3), s=(1, 1, 1), d=(1, 2, 2), p=(1, 2, 2, 1, 2, 2)),
    dict(k=(2, 3, 1), s=(2, 1, 1), d=(1, 1, 1), p=(1, 0, 0, 0, 2, 0)),
])
def test_conv3d_restatement_matches_torch(port, case):
    """The Convolution3D restatement (the formula of the reference's patch)
    against PyTorch's conv3d on the same fp32 data, with explicit zero pads."""
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 4, 9, 11)).astype(np.float32)
    w = (0.2 * rng.standard_normal((6, 5) + case["k"])).astype(np.float32)
    b = rng.standard_normal(6).astype(np.float32)
    got = port.conv3d(x, w, b, stride=case["s"], dilation=case["d"], pad=case["p"])
    pf, pt, pl, pb, pbo, pr = case["p"]
    xp = np.pad(x, ((0, 0), (pf, pb), (pt, pbo), (pl, pr)))
    want = torch.nn.functional.conv3d(torch.from_numpy(xp)[None].double(), torch.from_numpy(w).double(),
                                      torch.from_numpy(b).double(), stride=case["s"], dilation=case["d"])[0].numpy()
    assert got.shape == want.shape
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
