"""GPU parity of the sm_100a path, called through the C ABI (libs2b200.so).

Reference values come from the committed golden fixtures (the reference's own
CPU code) and from the C restatement oracle run here on the same inputs.
Full-size configs that the oracle cannot finish in seconds are checked on a
seeded sample of (window, head) pairs plus size-independent properties.
"""
from __future__ import annotations

import numpy as np
import pytest

import parity
import refcases
import s2b200
from conftest import from_bf16_bits
from s2b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    rc = s2b200.device_check(0)
    assert rc == 0, s2b200.last_error()
    return torch


def make_layer(heads, gammas, freqs, grid, shifted, mode=s2b200.MODE_BF16_REF, override=(0, 0, 0)):
    layer = s2b200.SeedVR2DiTBlockAttention(device=0, mode=mode, window_override=override)
    assert layer.load_param(shifted=shifted, dim=heads * 128, heads=heads) == 0
    layer.load_model(gammas[0], gammas[1], freqs, gammas[2], gammas[3])
    layer.set_runtime_shape(*grid)
    return layer


def run_gpu(torch, vid, txt, gammas, freqs, grid, heads, shifted, mode=s2b200.MODE_BF16_REF, override=(0, 0, 0),
            in_dtype=None):
    in_dtype = in_dtype or torch.float32
    layer = make_layer(heads, gammas, freqs, grid, shifted, mode, override)
    v = torch.from_numpy(np.ascontiguousarray(vid)).to("cuda", in_dtype)
    t = torch.from_numpy(np.ascontiguousarray(txt)).to("cuda", in_dtype)
    vo, to = layer.forward(v, t)
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    assert layer.last_launches() == 3
    return vo.float().cpu().numpy(), to.cpu().numpy()


@pytest.mark.parametrize("shifted", [0, 1])
def test_golden_cfg0_one_head(torch_cuda, golden, shifted):
    g = golden("attn_cfg0_h1.npz")
    grid = tuple(int(x) for x in g["grid"])
    vo, to = run_gpu(torch_cuda, g["vid_qkv"].astype(np.float32), g["txt_qkv"].astype(np.float32), g["gammas"],
                     g["freqs"], grid, 1, shifted)
    m = parity.check(vo, from_bf16_bits(g[f"vid_out_s{shifted}"]), True, "vid")
    parity.check(to, g[f"txt_out_s{shifted}"], True, "txt")
    assert m["exact_frac"] > 0.9


def test_prologue_packed_qkv_vs_golden(torch_cuda, golden):
    torch = torch_cuda
    g = golden("attn_cfg0_h1.npz")
    T, H, W = (int(x) for x in g["grid"])
    wins = s2b200.make_windows(T, H, W, 0)
    cu, rows = s2b200.build_varlen(T, H, W, wins, 58)
    d_rows = torch.from_numpy(rows.copy()).cuda()
    gam = torch.from_numpy(np.ascontiguousarray(g["gammas"])).cuda()
    fr = torch.from_numpy(np.ascontiguousarray(g["freqs"])).cuda()
    tab = s2b200.rope_table(fr, int(rows[:, 1:].max()) + 1)
    v = torch.from_numpy(g["vid_qkv"]).cuda()
    t = torch.from_numpy(g["txt_qkv"]).cuda()
    q, k, vv = s2b200.qk_norm_rope(v, t, 1, gam, tab, d_rows)
    torch.cuda.synchronize()
    for name, got in zip("qkv", (q, k, vv)):
        exp = from_bf16_bits(g[f"packed_{name}_s0"])
        a = got[0].float().cpu().numpy()
        m = parity.metrics(a, exp)
        # Bit-exact except where the fp64 summation order or sincosf moves a
        # value across a bf16 rounding boundary: one ulp, or for tiny results
        # of the rotation's a*c - b*s cancellation a few 1e-7 absolute.
        assert m["exact_frac"] > 0.999, (name, m)
        assert np.all(np.abs(a - exp) <= np.maximum(parity.bf16_ulp(exp), 1e-5)), (name, m)


@pytest.mark.parametrize("i", range(len(refcases.BLOCK_CASES)))
def test_reference_runner_cases(torch_cuda, golden, i):
    g = golden("attn_runner_cases.npz")
    vq, tq, g4, fr, shape, heads, shifted = refcases.attention_case(refcases.BLOCK_CASES[i])
    vo, to = run_gpu(torch_cuda, vq, tq, g4, fr, shape, heads, shifted)
    parity.check(vo, g[f"c{i}_vid_out"], True, "vid")
    parity.check(to, g[f"c{i}_txt_out"], True, "txt")


@pytest.mark.parametrize("shifted", [0, 1])
@pytest.mark.parametrize("override", [(0, 0, 0), (2, 8, 10)])
def test_cfg0_full_heads_vs_oracle(torch_cuda, port, shifted, override):
    grid = synth.GRIDS["cfg0"]
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=100 + shifted)
    vo, to = run_gpu(torch_cuda, vid, txt, gam, fr, grid, 20, shifted, override=override)
    ro, rt, _ = port.window_attention(vid, txt, grid, 20, list(gam), fr, shifted, override=override)
    parity.check(vo, ro, True, "vid")
    parity.check(to, rt, True, "txt")


@pytest.mark.parametrize("shifted", [0, 1])
def test_fp16_mode_vs_unrounded_oracle(torch_cuda, port, shifted):
    torch = torch_cuda
    grid = synth.GRIDS["cfg0"]
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=7)
    vo, to = run_gpu(torch, vid, txt, gam, fr, grid, 20, shifted, mode=s2b200.MODE_F16, in_dtype=torch.float16)
    ro, rt, _ = port.window_attention(vid, txt, grid, 20, list(gam), fr, shifted, round_out=False)
    m = parity.check(vo, ro, False, "vid")
    parity.check(to, rt, False, "txt")
    assert m["max_abs"] < 1e-3


def test_input_dtypes_agree(torch_cuda):
    torch = torch_cuda
    grid = (2, 9, 13)
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=4, seed=9)
    outs = [run_gpu(torch, vid, txt, gam, fr, grid, 4, 1, in_dtype=dt) for dt in (torch.float32, torch.float16)]
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    # bf16 inputs of bf16-representable values: same numbers again
    vb = vid.astype(np.float32)
    vb = (vb.view(np.uint32) & 0xFFFF0000).view(np.float32)
    tb = (txt.view(np.uint32) & 0xFFFF0000).view(np.float32)
    a = run_gpu(torch, vb, tb, gam, fr, grid, 4, 1, in_dtype=torch.float32)
    b = run_gpu(torch, vb, tb, gam, fr, grid, 4, 1, in_dtype=torch.bfloat16)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def _sampled(torch, port, name, shifted, override=(0, 0, 0), n_win=3, heads_pick=(0, 13)):
    grid = synth.GRIDS[name]
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=31 + shifted)
    vo, to = run_gpu(torch, vid, txt, gam, fr, grid, 20, shifted, override=override)
    wins = s2b200.make_windows(*grid, shifted, override)
    sizes = (wins[:, 1] - wins[:, 0]) * (wins[:, 3] - wins[:, 2]) * (wins[:, 5] - wins[:, 4])
    # largest, smallest and one random window
    rng = np.random.default_rng(5)
    pick = sorted({int(np.argmax(sizes)), int(np.argmin(sizes)), int(rng.integers(len(wins)))})[:n_win]
    mask = np.zeros(len(wins), np.uint8)
    mask[pick] = 1
    T, H, W = grid
    for h in heads_pick:
        ro, _, _ = port.window_attention(vid, txt, grid, 20, list(gam), fr, shifted, override=override,
                                         heads_range=(h, h + 1), window_mask=mask)
        cols = slice(h * 128, (h + 1) * 128)
        for w in pick:
            t0, t1, h0, h1, w0, w1 = wins[w]
            idx = ((np.arange(t0, t1)[:, None, None] * H + np.arange(h0, h1)[None, :, None]) * W
                   + np.arange(w0, w1)[None, None, :]).ravel()
            parity.check(vo[idx, cols], ro[idx, cols], True, f"{name} window {w} head {h}")
    # every video row written exactly once (no zero rows left), text finite
    assert np.all(np.abs(vo).sum(axis=1) > 0)
    assert np.isfinite(to).all()


@pytest.mark.parametrize("shifted", [0, 1])
def test_cfg2_720p_sampled(torch_cuda, port, shifted):
    _sampled(torch_cuda, port, "cfg2", shifted)


@pytest.mark.parametrize("shifted", [0, 1])
def test_cfg3_1080p_ragged_sampled(torch_cuda, port, shifted):
    _sampled(torch_cuda, port, "cfg3", shifted, n_win=2, heads_pick=(19,))


@pytest.mark.parametrize("shifted", [0, 1])
def test_bench_path_cfg2_full_vs_unrounded_oracle(torch_cuda, port, shifted):
    """Exactly the configuration bench.py times: the 720p layer (27 plain / 64
    shifted windows) in S2_MODE_F16 with fp16 QKV in and fp16 out -- every
    window, every head and the text mean against the oracle's unrounded
    variant (the reference's Vulkan output semantics,
    seedvr2_dit_block.cpp:416-436; arithmetic :1045-1079)."""
    torch = torch_cuda
    grid = synth.GRIDS["cfg2"]
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=41 + shifted)
    vo, to = run_gpu(torch, vid, txt, gam, fr, grid, 20, shifted, mode=s2b200.MODE_F16, in_dtype=torch.float16)
    ro, rt, _ = port.window_attention(vid, txt, grid, 20, list(gam), fr, shifted, round_out=False)
    m = parity.check(vo, ro, False, f"cfg2 shifted={shifted} vid")
    parity.check(to, rt, False, f"cfg2 shifted={shifted} txt")
    assert m["max_abs"] < 1e-3, m


@pytest.mark.parametrize("shifted", [0, 1])
def test_bench_path_cfg3_sampled_all_heads(torch_cuda, port, shifted):
    """Config 3 (1080p x 45f, 96,480 tokens, 100 plain / 125 shifted windows)
    in the benchmarked mode (fp16 in, S2_MODE_F16): all 20 heads of the
    largest, the smallest and one random window, video rows of the full-layer
    run, and the text partial sum of those windows through a window-subset
    layer (the sharded path) against the oracle restricted to them."""
    torch = torch_cuda
    grid = synth.GRIDS["cfg3"]
    T, H, W = grid
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=51 + shifted)
    vo, _ = run_gpu(torch, vid, txt, gam, fr, grid, 20, shifted, mode=s2b200.MODE_F16, in_dtype=torch.float16)
    assert np.all(np.abs(vo).sum(axis=1) > 0), "a video row was not written"
    wins = s2b200.make_windows(*grid, shifted)
    sizes = (wins[:, 1] - wins[:, 0]) * (wins[:, 3] - wins[:, 2]) * (wins[:, 5] - wins[:, 4])
    rng = np.random.default_rng(17 + shifted)
    pick = sorted({int(np.argmax(sizes)), int(np.argmin(sizes)), int(rng.integers(len(wins)))})
    mask = np.zeros(len(wins), np.uint8)
    mask[pick] = 1
    ro, rt, _ = port.window_attention(vid, txt, grid, 20, list(gam), fr, shifted, round_out=False,
                                      window_mask=mask)
    for w in pick:
        t0, t1, h0, h1, w0, w1 = wins[w]
        idx = ((np.arange(t0, t1)[:, None, None] * H + np.arange(h0, h1)[None, :, None]) * W
               + np.arange(w0, w1)[None, None, :]).ravel()
        parity.check(vo[idx], ro[idx], False, f"cfg3 shifted={shifted} window {w} ({sizes[w]} tokens)")
    layer = make_layer(20, gam, fr, grid, shifted, mode=s2b200.MODE_F16)
    layer.set_window_subset(np.array(pick, np.int32))
    _, to_sub = layer.forward(torch.from_numpy(vid).to("cuda", torch.float16),
                              torch.from_numpy(txt).to("cuda", torch.float16))
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    parity.check(to_sub.cpu().numpy(), rt, False, f"cfg3 shifted={shifted} text partial")


def test_long_windows_override_cfg2(torch_cuda, port):
    """BASELINE's 6x15x20 windows: S = 1858 keys -> 15 key tiles per CTA."""
    _sampled(torch_cuda, port, "cfg2", 1, override=synth.OVERRIDES["cfg2"], n_win=2, heads_pick=(4,))


def test_tiny_windows_and_single_text_token(torch_cuda, port):
    for grid, lt, shifted in [((1, 1, 1), 1, 0), ((1, 1, 1), 3, 1), ((2, 2, 2), 2, 1), ((1, 3, 130), 1, 0),
                              ((5, 7, 300), 5, 1)]:
        vid, txt, gam, fr = synth.layer_inputs(grid, heads=2, text_len=lt, seed=lt)
        vo, to = run_gpu(torch_cuda, vid, txt, gam, fr, grid, 2, shifted)
        ro, rt, _ = port.window_attention(vid, txt, grid, 2, list(gam), fr, shifted)
        parity.check(vo, ro, True, f"vid {grid}")
        parity.check(to, rt, True, f"txt {grid}")


def test_deterministic(torch_cuda):
    grid = (2, 16, 30)
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=1)
    a = run_gpu(torch_cuda, vid, txt, gam, fr, grid, 20, 1)
    b = run_gpu(torch_cuda, vid, txt, gam, fr, grid, 20, 1)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_window_subsets_partition_the_layer(torch_cuda):
    """Window sharding: disjoint subsets write disjoint video rows and their
    text partial sums (each pre-scaled by 1/total windows) add to the mean."""
    torch = torch_cuda
    grid = (6, 45, 80)
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=4)
    full_v, full_t = run_gpu(torch, vid, txt, gam, fr, grid, 20, 1)
    n = len(s2b200.make_windows(*grid, 1))
    v = torch.from_numpy(vid).cuda()
    t = torch.from_numpy(txt).cuda()
    acc_v = torch.zeros((vid.shape[0], 2560), dtype=torch.bfloat16, device="cuda")
    acc_t = torch.zeros((txt.shape[0], 2560), dtype=torch.float32, device="cuda")
    for r in range(3):
        layer = make_layer(20, gam, fr, grid, 1)
        layer.set_window_subset(np.arange(r, n, 3))
        vo, to = layer.forward(v, t)
        acc_v += vo
        acc_t += to
        assert layer.device_error() == 0
    torch.cuda.synchronize()
    assert np.array_equal(acc_v.float().cpu().numpy(), full_v)
    np.testing.assert_allclose(acc_t.cpu().numpy(), full_t, rtol=0, atol=1e-6)


def test_host_buffer_forward_matches_device(torch_cuda):
    grid = (2, 16, 30)
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=20, seed=2)
    dv, dt = run_gpu(torch_cuda, vid, txt, gam, fr, grid, 20, 0)
    layer = make_layer(20, gam, fr, grid, 0)
    hv, ht = layer.forward_host(vid, txt, np.array(grid, np.int32), io_dtype=s2b200.S2_F32)
    assert np.array_equal(hv, dv) and np.array_equal(ht, dt)
    # fp16 host I/O in fp16 mode
    layer16 = make_layer(20, gam, fr, grid, 0, mode=s2b200.MODE_F16)
    hv16, ht16 = layer16.forward_host(vid.astype(np.float16), txt.astype(np.float16), np.array(grid, np.int32),
                                      io_dtype=s2b200.S2_F16)
    assert hv16.dtype == np.float16 and np.isfinite(hv16).all()
    np.testing.assert_allclose(hv16.astype(np.float32), dv, atol=8e-3)


@pytest.mark.parametrize("grid,shifted", [((6, 24, 40), 0), ((6, 24, 40), 1), ((5, 16, 30), 1)])
@pytest.mark.parametrize("io", ["f32", "f16"])
def test_pipelined_host_forward_matches_device(torch_cuda, grid, shifted, io):
    """The host-buffer forward overlaps uploads, compute and downloads slab by
    slab of frames; its outputs must equal the device-buffer forward's exactly,
    and a window-subset layer (serial host path) must agree too."""
    torch = torch_cuda
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=4, seed=9)
    mode = s2b200.MODE_F16 if io == "f16" else s2b200.MODE_BF16_REF
    io_dtype = s2b200.S2_F16 if io == "f16" else s2b200.S2_F32
    cast = (lambda a: a.astype(np.float16)) if io == "f16" else (lambda a: a)
    dev_layer = make_layer(4, gam, fr, grid, shifted, mode=mode)
    dvo, dto = dev_layer.forward(torch.from_numpy(cast(vid)).cuda(), torch.from_numpy(cast(txt)).cuda())
    torch.cuda.synchronize()
    dvo, dto = dvo.float().cpu().numpy(), dto.cpu().numpy()
    layer = make_layer(4, gam, fr, grid, shifted, mode=mode)
    for _ in range(2):  # the second call reuses the pipeline's streams and events
        hv, ht = layer.forward_host(cast(vid), cast(txt), np.array(grid, np.int32), io_dtype=io_dtype)
        assert np.array_equal(hv.astype(np.float32), dvo) and np.array_equal(ht, dto)
    n = len(s2b200.make_windows(*grid, shifted))
    acc_v = np.zeros_like(dvo)
    for r in range(2):
        sub = make_layer(4, gam, fr, grid, shifted, mode=mode)
        sub.set_window_subset(np.arange(r, n, 2))
        sv, _ = sub.forward_host(cast(vid), cast(txt), np.array(grid, np.int32), io_dtype=io_dtype)
        acc_v += sv.astype(np.float32)
    assert np.array_equal(acc_v, dvo)


def test_shape_mismatch_returns_invalid_argument(torch_cuda):
    torch = torch_cuda
    grid = (2, 4, 4)
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=1, seed=0)
    layer = make_layer(1, gam, fr, (2, 4, 5), 0)
    with pytest.raises(s2b200.S2Error) as e:
        layer.forward(torch.from_numpy(vid).cuda(), torch.from_numpy(txt).cuda())
    assert e.value.status == s2b200.S2_INVALID_ARGUMENT
