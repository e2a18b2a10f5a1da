"""The allocation-free entry point, s2_dit_window_attention_noalloc.

It exists for callers that must not allocate device memory while they run
(code inside another framework's memory pool or allocator callbacks, or a
host that reserved all HBM up front): it runs the whole attention stage out
of one fixed scratch array that belongs to the library. These tests call it
through the C ABI, twice in a row with different windows and inputs, and
compare each result with the regular layer entry point
(s2_attention_layer_forward) on the same inputs, within the tolerance the
other parity tests use. The file name sorts last so a stop-at-first-failure
run has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest

import parity
import s2b200
from s2b200 import synth


def _call(torch, vid, txt, gam_d, fr_d, grid, heads, shifted, err, mode=s2b200.MODE_BF16_REF):
    T, H, W = grid
    dim = heads * 128
    vid_out = torch.zeros((vid.shape[0], dim), dtype=s2b200.mode_dtype(mode), device="cuda")
    txt_out = torch.zeros((txt.shape[0], dim), dtype=torch.float32, device="cuda")
    rc = s2b200.lib().s2_dit_window_attention_noalloc(
        s2b200._stream_ptr(), mode, s2b200._ptr(vid), s2b200._ptr(txt), s2b200._dtype_code(vid), T, H, W,
        txt.shape[0], heads, ctypes.c_float(1e-5), int(shifted), 0, 0, 0, s2b200._ptr(gam_d), s2b200._ptr(fr_d),
        s2b200._ptr(vid_out), s2b200._ptr(txt_out), s2b200._ptr(err))
    assert rc == 0, s2b200.last_error()
    return vid_out, txt_out


def _layer(torch, vid, txt, gam, fr, grid, heads, shifted):
    layer = s2b200.SeedVR2DiTBlockAttention(device=0, mode=s2b200.MODE_BF16_REF)
    layer.load_param(shifted=shifted, dim=heads * 128, heads=heads)
    layer.load_model(gam[0], gam[1], fr, gam[2], gam[3])
    layer.set_runtime_shape(*grid)
    vo, to = layer.forward(vid, txt)
    torch.cuda.synchronize()
    assert layer.device_error() == 0
    return vo.float().cpu().numpy(), to.cpu().numpy()


@pytest.mark.gpu
def test_noalloc_matches_layer_entry_point_on_consecutive_calls():
    import torch
    assert torch.cuda.is_available()
    assert s2b200.device_check(0) == 0, s2b200.last_error()
    err = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    grid = synth.GRIDS["cfg0"]
    cases = [(0, 41), (1, 42)]  # plain then shifted windows, different inputs
    for shifted, seed in cases:
        vid_np, txt_np, gam, fr = synth.layer_inputs(grid, heads=20, seed=seed)
        vid = torch.from_numpy(vid_np).cuda()
        txt = torch.from_numpy(txt_np).cuda()
        gam_d = torch.from_numpy(gam).cuda()
        fr_d = torch.from_numpy(fr).cuda()
        vo, to = _call(torch, vid, txt, gam_d, fr_d, grid, 20, shifted, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        ref_v, ref_t = _layer(torch, vid, txt, gam, fr, grid, 20, shifted)
        parity.check(vo.float().cpu().numpy(), ref_v, True, f"noalloc vid (shifted={shifted})")
        parity.check(to.cpu().numpy(), ref_t, True, f"noalloc txt (shifted={shifted})")

    # A further call changes no device memory (it only reuses the fixed array).
    vid_np, txt_np, gam, fr = synth.layer_inputs(grid, heads=20, seed=43)
    vid = torch.from_numpy(vid_np).cuda()
    txt = torch.from_numpy(txt_np).cuda()
    gam_d = torch.from_numpy(gam).cuda()
    fr_d = torch.from_numpy(fr).cuda()
    vout = torch.zeros((vid.shape[0], 2560), dtype=torch.bfloat16, device="cuda")
    tout = torch.zeros((txt.shape[0], 2560), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    rc = s2b200.lib().s2_dit_window_attention_noalloc(
        s2b200._stream_ptr(), s2b200.MODE_BF16_REF, s2b200._ptr(vid), s2b200._ptr(txt), s2b200.S2_F32, *grid, 58,
        20, ctypes.c_float(1e-5), 1, 0, 0, 0, s2b200._ptr(gam_d), s2b200._ptr(fr_d), s2b200._ptr(vout),
        s2b200._ptr(tout), None)
    torch.cuda.synchronize()
    assert rc == 0, s2b200.last_error()
    assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch():
    """The 720p grid needs far more than the fixed scratch; the call must say so
    before touching the GPU."""
    dummy = ctypes.c_void_p(256)
    T, H, W = synth.GRIDS["cfg2"]
    rc = s2b200.lib().s2_dit_window_attention_noalloc(
        None, s2b200.MODE_F16, dummy, dummy, s2b200.S2_F16, T, H, W, 58, 20, ctypes.c_float(1e-5), 0, 0, 0, 0,
        dummy, dummy, dummy, dummy, None)
    assert rc == s2b200.S2_INVALID_ARGUMENT
    msg = s2b200.last_error()
    assert "limit" in msg and "32768" in msg
