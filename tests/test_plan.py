"""Host side of the product library (no GPU needed): the C ABI loads and
exports every declared symbol, and the window / varlen / work planning is
bit-exact against the reference (golden) and the oracle."""
from __future__ import annotations

import os
import re

import numpy as np
import pytest

import s2b200
from conftest import ROOT
from s2b200 import synth


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "s2_b200.h")).read()
    return sorted(set(re.findall(r"^S2_API\s+[\w\s\*]*?\b(s2_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    import ctypes
    lib = ctypes.CDLL(s2b200.LIB_PATH)
    declared = _declared_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(declared) == sorted(s2b200.exported_symbols())
    assert s2b200.lib().s2_version() >= 1


def test_make_windows_bit_exact_vs_reference(golden):
    g = golden("windows.npz")
    for key in g.files:
        dims, s = key.split("_s")
        T, H, W = map(int, dims.split("x"))
        assert np.array_equal(s2b200.make_windows(T, H, W, int(s)), g[key]), key


@pytest.mark.parametrize("seed", range(4))
def test_make_windows_random_grids_vs_oracle(port, seed):
    rng = np.random.default_rng(seed)
    for _ in range(200):
        T, H, W = int(rng.integers(1, 50)), int(rng.integers(1, 200)), int(rng.integers(1, 300))
        for s in (0, 1):
            assert np.array_equal(s2b200.make_windows(T, H, W, s), port.make_windows(T, H, W, s)), (T, H, W, s)


def test_window_override_vs_oracle_and_baseline_geometry(port):
    for name, grid in synth.GRIDS.items():
        ov = synth.OVERRIDES[name]
        for s in (0, 1):
            a = s2b200.make_windows(*grid, s, ov)
            assert np.array_equal(a, port.make_windows(*grid, s, ov))
    # 2x8x10 windows on the 2x16x30 grid -> 6 windows of 160 tokens
    w = s2b200.make_windows(2, 16, 30, 0, (2, 8, 10))
    sizes = (w[:, 1] - w[:, 0]) * (w[:, 3] - w[:, 2]) * (w[:, 5] - w[:, 4])
    assert len(w) == 6 and np.all(sizes == 160)


@pytest.mark.parametrize("grid,shifted", [((2, 16, 30), 0), ((2, 16, 30), 1), ((6, 45, 80), 1), ((1, 1, 1), 0)])
def test_windows_disjoint_cover(grid, shifted):
    T, H, W = grid
    cover = np.zeros(grid, np.int32)
    for t0, t1, h0, h1, w0, w1 in s2b200.make_windows(T, H, W, shifted):
        cover[t0:t1, h0:h1, w0:w1] += 1
    assert np.all(cover == 1)


def test_build_varlen_matches_reference_sequence_layout():
    T, H, W, Lt = 2, 16, 30, 58
    wins = s2b200.make_windows(T, H, W, 1)
    cu, rows = s2b200.build_varlen(T, H, W, wins, Lt)
    assert cu[0] == 0 and cu[-1] == rows.shape[0] == T * H * W + len(wins) * Lt
    seen = []
    for w, (t0, t1, h0, h1, w0, w1) in enumerate(wins):
        seq = rows[cu[w]:cu[w + 1]]
        n_vid = (t1 - t0) * (h1 - h0) * (w1 - w0)
        vid, txt = seq[:n_vid], seq[n_vid:]
        exp = [((t * H + y) * W + x, Lt + t - t0, y - h0, x - w0) for t in range(t0, t1) for y in range(h0, h1)
               for x in range(w0, w1)]
        assert np.array_equal(vid, np.array(exp, np.int32).reshape(-1, 4))
        assert np.array_equal(txt[:, 0], -(np.arange(Lt) + 1))
        assert np.array_equal(txt[:, 1], np.arange(Lt)) and np.array_equal(txt[:, 3], np.arange(Lt))
        seen.extend(vid[:, 0].tolist())
    assert sorted(seen) == list(range(T * H * W))


def test_plan_work_covers_tiles_costliest_first():
    wins = s2b200.make_windows(6, 45, 80, 1)
    cu, _ = s2b200.build_varlen(6, 45, 80, wins, 58)
    work = s2b200.plan_work(cu)
    S = np.diff(cu)
    tiles = -(-S // 256)  # one CTA per 256 query rows (two 128-row Q tiles)
    assert len(work) == tiles.sum()
    w, qt = work >> 16, work & 0xFFFF
    cost = S[w]
    assert np.all(np.diff(cost) <= 0)
    for win in range(len(S)):
        assert sorted(qt[w == win].tolist()) == list(range(tiles[win]))


def test_invalid_arguments_report_reference_status():
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.make_windows(0, 4, 4, 0)
    assert e.value.status == s2b200.S2_INVALID_ARGUMENT
    assert "invalid grid" in str(e.value)
    with pytest.raises(s2b200.S2Error):
        s2b200.make_windows(2, 4, 4, 0, (2, 0, 3))
    with pytest.raises(s2b200.S2Error):
        s2b200.build_varlen(2, 4, 4, np.array([[0, 3, 0, 4, 0, 4]], np.int32), 5)


def test_layer_create_without_gpu_reports_unsupported():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    layer = s2b200.SeedVR2DiTBlockAttention()
    with pytest.raises(s2b200.S2Error) as e:
        layer.load_param(heads=20, dim=2560)
    assert e.value.status == s2b200.S2_UNSUPPORTED


def test_vae_layer_channel_checks():
    """load_param rejects channel counts the reference rejects (not a multiple
    of the 32 GroupNorm groups) before touching a device."""
    for bad in (0, 48, -32):
        with pytest.raises(s2b200.S2Error) as e:
            s2b200.DynamicFramewiseSpatialAttention().load_param(bad)
        assert e.value.status == s2b200.S2_INVALID_ARGUMENT
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.DynamicFramewiseSpatialAttention().load_param(544)
    assert e.value.status == s2b200.S2_UNSUPPORTED
    assert [s2b200.padded_channels(c) for c in (32, 128, 160, 256, 288, 512)] == [128, 128, 256, 256, 512, 512]


def test_vae_layer_create_without_gpu_reports_unsupported():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(s2b200.S2Error) as e:
        s2b200.DynamicFramewiseSpatialAttention().load_param(512)
    assert e.value.status == s2b200.S2_UNSUPPORTED
