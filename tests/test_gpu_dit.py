"""GPU parity of the DiT and one Euler step (SeedVR2DiT::forward with the
engine's one-step sampling) through the C ABI: input head (patchify, video and
text projections, timestep MLP), the block stack, output head (RMSNorm, adaLN,
projection, unpatchify) fused with the Euler endpoint.

The reference is its own CPU code run layer by layer (SeedVR2DiTInput, each
SeedVR2DiTBlock, SeedVR2DiTOutput built from its sources, oracle/_ref) plus
the restated make_dit_input / endpoint arithmetic (oracle.euler_step).
Gate (the reference's own full-DiT gate, tools/test_seedvr2_dit_ncnn.py:
248-250): prediction NRMSE <= 0.02 and cosine >= 0.9998, plus x0 within
max-abs 2e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

import parity
import s2b200
from s2b200 import synth

pytestmark = pytest.mark.gpu

NRMSE_MAX = 0.02
COS_MIN = 0.9998


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert s2b200.device_check(0) == 0, s2b200.last_error()
    return torch


def build_case(n_blocks, dim, heads, mlp, tc, flags):
    wi = synth.dit_input_weights(dim, 33, tc, 256)
    wo = synth.dit_output_weights(dim)
    bws, bps = [], []
    for i in range(n_blocks):
        f = flags(i)
        bws.append(synth.block_weights(dim, heads, mlp, f["shared"], seed=100 + i))
        bps.append(dict(block_index=i, dim=dim, heads=heads, head_dim=128, mlp_hidden=mlp, eps=1e-5, **f))
    head_params = dict(dim=dim, text_channels=tc, sinusoidal_dim=256, embedding_dim=6 * dim, out_channels=16, eps=1e-5)
    return head_params, wi, wo, bps, bws


def make_model(n_blocks, dim, heads, mlp, tc, wi, wo, bps, bws):
    m = s2b200.SeedVR2DiT(n_blocks=n_blocks, dim=dim, heads=heads, mlp_hidden=mlp, text_channels=tc)
    m.load_input(wi)
    m.load_output(wo)
    for i in range(n_blocks):
        m.load_block(i, bws[i], **{k: bps[i][k] for k in ("shared", "last", "shifted")})
    return m


def check_step(x0, ex0, noise, what):
    m = parity.metrics(x0, ex0)
    assert m["finite"] and m["max_abs"] <= parity.MAX_ABS, f"{what} x0: {m}"
    p = parity.metrics(noise - x0, noise - ex0)  # (t/1000) * prediction at t = 1000
    assert p["nrmse"] <= NRMSE_MAX and p["cosine"] >= COS_MIN, f"{what} prediction: {p}"


def four_block_flags(i):
    return [dict(shared=False, shifted=False, last=False), dict(shared=True, shifted=True, last=False),
            dict(shared=False, shifted=False, last=False), dict(shared=True, shifted=True, last=True)][i]


@pytest.mark.parametrize("n_blocks,dim,heads,mlp,tc,lat,Lt", [
    (4, 256, 2, 256, 200, (2, 12, 20), 10),     # every branch kind; text channels padded 200 -> 256
    (32, 256, 2, 512, 512, (3, 16, 24), 20),    # 32 blocks with the export's flags
])
def test_euler_step_vs_reference(torch_cuda, ref, n_blocks, dim, heads, mlp, tc, lat, Lt):
    flags = four_block_flags if n_blocks == 4 else (lambda i: s2b200.block_flags(i, n_blocks))
    hp, wi, wo, bps, bws = build_case(n_blocks, dim, heads, mlp, tc, flags)
    noise, cond, text = synth.dit_latents(lat, 16, Lt, tc)
    ex0, _ = ref.euler_step(hp, wi, bps, bws, wo, noise, cond, text, 1000.0)
    m = make_model(n_blocks, dim, heads, mlp, tc, wi, wo, bps, bws)
    x0 = m.euler_step(*(torch_cuda.from_numpy(a).cuda() for a in (noise, cond, text)))
    torch_cuda.cuda.synchronize()
    assert m.device_error() == 0
    check_step(x0.cpu().numpy(), ex0, noise, f"{n_blocks} blocks")
    assert np.array_equal(m.euler_step_host(noise, cond, text), x0.cpu().numpy())


def test_forward_prediction_vs_reference(torch_cuda, ref):
    hp, wi, wo, bps, bws = build_case(4, 256, 2, 256, 256, four_block_flags)
    noise, cond, text = synth.dit_latents((2, 8, 10), 16, 7, 256)
    latent = np.concatenate([noise, cond, np.ones((1,) + noise.shape[1:], np.float32)])
    vid, txt, emb = ref.dit_input(hp, wi, latent, text, 1000.0)
    for bp, bw in zip(bps, bws):
        vid, txt = ref.block_forward(bp, bw, vid, txt, emb, (2, 4, 5))
    epred = ref.dit_output(hp, wo, vid, emb, (2, 4, 5))
    m = make_model(4, 256, 2, 256, 256, wi, wo, bps, bws)
    pred = m.forward(torch_cuda.from_numpy(latent).cuda(), torch_cuda.from_numpy(text).cuda(), 1000.0)
    torch_cuda.cuda.synchronize()
    p = parity.metrics(pred.cpu().numpy(), epred)
    assert p["nrmse"] <= NRMSE_MAX and p["cosine"] >= COS_MIN and p["max_abs"] <= parity.MAX_ABS, p


@pytest.mark.parametrize("shifted", [False, True])
def test_block_at_config2_token_count(torch_cuda, ref, shifted):
    """One block over config 2's 21,600 video tokens (27 plain / 64 shifted
    windows of up to 868 rows) at reduced width."""
    dim, heads, mlp, grid = 256, 2, 512, synth.GRIDS["cfg2"]
    w = synth.block_weights(dim, heads, mlp, seed=21)
    vid, txt, emb = synth.block_activations(grid, dim)
    params = dict(block_index=5, shared=False, last=False, shifted=shifted, dim=dim, heads=heads, head_dim=128,
                  mlp_hidden=mlp, eps=1e-5)
    evo, eto = ref.block_forward(params, w, vid, txt, emb, grid)
    b = s2b200.SeedVR2DiTBlock()
    b.load_param(**params)
    b.load_model(w)
    b.set_runtime_shape(*grid)
    vo, to = b.forward(*(torch_cuda.from_numpy(a).cuda() for a in (vid, txt, emb)))
    torch_cuda.cuda.synchronize()
    assert b.device_error() == 0
    for name, got, exp, inp in (("vid", vo.cpu().numpy(), evo, vid), ("txt", to.cpu().numpy(), eto, txt)):
        m = parity.metrics(got, exp)
        assert m["max_abs"] <= parity.MAX_ABS, f"{name}: {m}"
        assert parity.metrics(got - inp, exp - inp)["cosine"] >= parity.COSINE, name


def test_load_checks(torch_cuda):
    m = s2b200.SeedVR2DiT(n_blocks=2, dim=128, heads=1, mlp_hidden=128, text_channels=64)
    with pytest.raises(s2b200.S2Error) as e:
        m.load_input(np.zeros(m.input_weight_count() - 1, np.float32))
    assert e.value.status == s2b200.S2_INVALID_ARGUMENT
    m.load_input(synth.dit_input_weights(128, 33, 64, 256))
    m.load_output(synth.dit_output_weights(128))
    noise, cond, text = synth.dit_latents((1, 4, 4), 16, 3, 64)
    with pytest.raises(s2b200.S2Error) as e:  # blocks missing
        m.euler_step_host(noise, cond, text)
    assert e.value.status == s2b200.S2_NOT_LOADED


def test_graph_replay_matches_eager(torch_cuda):
    """Calls 1 (eager), 2 (captured) and 3+ (graph replay) of an Euler step on
    the same buffers give identical results, and so does a model with graphs
    switched off."""
    torch = torch_cuda
    hp, wi, wo, bps, bws = build_case(4, 256, 2, 256, 256, four_block_flags)
    noise, cond, text = synth.dit_latents((2, 8, 12), 16, 9, 256)
    n, c, t = (torch.from_numpy(a).cuda() for a in (noise, cond, text))
    m = make_model(4, 256, 2, 256, 256, wi, wo, bps, bws)
    x0 = torch.empty_like(n)
    outs = []
    for _ in range(4):
        x0.zero_()
        m.euler_step(n, c, t, 1000.0, x0)
        torch.cuda.synchronize()
        outs.append(x0.cpu().numpy().copy())
    assert m.device_error() == 0
    eager = make_model(4, 256, 2, 256, 256, wi, wo, bps, bws)
    eager.set_graph(False)
    ref_out = eager.euler_step(n, c, t, 1000.0).cpu().numpy()
    for o in outs:
        assert np.array_equal(o, ref_out)
    assert m.last_launches() == eager.last_launches()


def test_graph_dropped_by_forward_on_larger_grid(torch_cuda):
    """A captured Euler-step graph points at the step's workspaces; a plain
    forward (and a sampling loop) on a larger grid grows them, so the next Euler
    step for the first grid must run again (eager, then a new capture) and give
    the eager model's result."""
    torch = torch_cuda
    hp, wi, wo, bps, bws = build_case(4, 256, 2, 256, 256, four_block_flags)
    noise, cond, text = synth.dit_latents((2, 8, 12), 16, 9, 256)
    n, c, t = (torch.from_numpy(a).cuda() for a in (noise, cond, text))
    m = make_model(4, 256, 2, 256, 256, wi, wo, bps, bws)
    x0 = torch.empty_like(n)
    for _ in range(3):  # eager, captured, replayed
        m.euler_step(n, c, t, 1000.0, x0)
    big_n, big_c, big_t = (torch.from_numpy(a).cuda() for a in synth.dit_latents((3, 16, 20), 16, 9, 256))
    big_lat = torch.cat([big_n, big_c, torch.ones_like(big_n[:1])], 0)
    m.forward(big_lat, big_t, 1000.0)
    m.sample(big_n, big_c, big_t, steps=1)
    outs = []
    for _ in range(3):
        x0.zero_()
        m.euler_step(n, c, t, 1000.0, x0)
        torch.cuda.synchronize()
        outs.append(x0.cpu().numpy().copy())
    assert m.device_error() == 0
    eager = make_model(4, 256, 2, 256, 256, wi, wo, bps, bws)
    eager.set_graph(False)
    ref_out = eager.euler_step(n, c, t, 1000.0).cpu().numpy()
    for o in outs:
        assert np.array_equal(o, ref_out)


def test_load_exported_model_dir(torch_cuda, tmp_path):
    """A model directory in the reference's exported layout (fp16-tagged
    InnerProduct weights) loads through s2_dit_load_dir and gives exactly the
    step of the same weights loaded as streams."""
    import ncnn_files
    dim, heads, mlp, tc, n_blocks = 256, 2, 256, 256, 4
    ei = ncnn_files.write_input(tmp_path, synth.dit_input_weights(dim, 33, tc, 256), dim, tc)
    eo = ncnn_files.write_output(tmp_path, synth.dit_output_weights(dim), dim)
    ebs = []
    for i in range(n_blocks):
        f = s2b200.block_flags(i, n_blocks)
        ebs.append(ncnn_files.write_block(tmp_path, i, synth.block_weights(dim, heads, mlp, f["shared"], seed=40 + i),
                                          dim, heads, mlp, f["shared"], f["last"], f["shifted"]))
    a = s2b200.SeedVR2DiT(n_blocks=n_blocks, dim=dim, heads=heads, mlp_hidden=mlp, text_channels=tc)
    a.load_dir(str(tmp_path))
    b = s2b200.SeedVR2DiT(n_blocks=n_blocks, dim=dim, heads=heads, mlp_hidden=mlp, text_channels=tc)
    b.load_input(ei)
    b.load_output(eo)
    for i in range(n_blocks):
        b.load_block(i, ebs[i])
    noise, cond, text = synth.dit_latents((2, 8, 10), 16, 5, tc)
    assert np.array_equal(a.euler_step_host(noise, cond, text), b.euler_step_host(noise, cond, text))
