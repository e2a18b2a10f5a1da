"""GPU parity of the device sampler through the C ABI: classifier-free
guidance (with the std rescale), Euler step_to / endpoint and the condition
latent against the reference's own EulerSampler (oracle/_ref) and the C
restatement; and the whole sampling loop (s2_dit_sample: several steps, with
guidance) against the reference's code run step by step.

Elementwise updates use the reference's float operation order with no
contraction, so they are compared bit for bit; the rescale factor comes from
fp64 sums taken in a different order (parallel), so guided-and-rescaled
outputs are compared to 1e-6 relative. The sampling loop uses the reference's
full-DiT gate (tools/test_seedvr2_dit_ncnn.py:248-250) on the displacement
noise - x0: NRMSE <= 0.02 and cosine >= 0.9998."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import parity
import s2b200
from s2b200 import synth

from test_gpu_dit import build_case, four_block_flags, make_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert s2b200.device_check(0) == 0, s2b200.last_error()
    return torch


@pytest.fixture(scope="module")
def sref(ref):
    return oracle.SamplerRef(ref.lib)


def _pair(shape, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape).astype(np.float32), rng.standard_normal(shape).astype(np.float32))


def _dev(torch, *arrays):
    return [torch.from_numpy(a).cuda() for a in arrays]


@pytest.mark.parametrize("shape", [(16, 6, 90, 160), (16, 1, 3, 5), (3, 2, 7, 11)])
@pytest.mark.parametrize("scale,rescale", [(1.0, 0.0), (2.5, 0.0), (3.0, 0.7), (5.0, 1.0)])
def test_apply_cfg(torch_cuda, sref, shape, scale, rescale):
    pos, neg = _pair(shape, 21)
    want = sref.apply_cfg(pos, neg, scale, rescale)
    got = s2b200.apply_cfg(*_dev(torch_cuda, pos, neg), scale, rescale)
    torch_cuda.cuda.synchronize()
    got = got.cpu().numpy()
    if rescale == 0.0:
        assert np.array_equal(got, want)
    else:
        assert np.allclose(got, want, rtol=1e-6, atol=1e-7), np.abs(got - want).max()


@pytest.mark.parametrize("t,t_next", [(1000.0, 750.0), (750.0, 500.0), (333.33, 0.0), (1000.0, 1200.0)])
def test_step_to_and_endpoint(torch_cuda, sref, t, t_next):
    pred, cur = _pair((16, 6, 90, 160), 31)
    dp, dc = _dev(torch_cuda, pred, cur)
    a = s2b200.euler_step_to(dp, dc, t, t_next)
    b = s2b200.euler_endpoint(dp, dc, t)
    inplace = dc.clone()
    s2b200.euler_step_to(dp, inplace, t, t_next, out=inplace)  # output may alias the current latent
    torch_cuda.cuda.synchronize()
    assert np.array_equal(a.cpu().numpy(), sref.step_to(pred, cur, t, t_next))
    assert np.array_equal(b.cpu().numpy(), sref.endpoint(pred, cur, t))
    assert np.array_equal(inplace.cpu().numpy(), a.cpu().numpy())


def test_make_condition(torch_cuda):
    enc, noise = _pair((16, 6, 90, 160), 41)
    got = s2b200.make_condition(*_dev(torch_cuda, enc, noise), 0.1)
    torch_cuda.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), oracle.SamplerPort(oracle.port().lib).make_condition(enc, noise, 0.1))


@pytest.mark.parametrize("steps,cfg,rescale,neg_len", [(1, 1.0, 0.0, 7), (3, 1.0, 0.0, 7), (2, 2.0, 0.0, 7),
                                                       (2, 3.0, 0.7, 7), (2, 2.5, 0.5, 9)])
def test_sample_vs_reference(torch_cuda, ref, steps, cfg, rescale, neg_len):
    """neg_len != 7: the negative text has its own token count, as the
    reference's default embeddings do (58 positive, 64 negative tokens)."""
    hp, wi, wo, bps, bws = build_case(4, 256, 2, 256, 256, four_block_flags)
    noise, cond, text = synth.dit_latents((2, 8, 10), 16, 7, 256)
    neg_text = np.random.default_rng(5).standard_normal((neg_len, text.shape[1])).astype(np.float32)
    want = ref.sample(hp, wi, bps, bws, wo, noise, cond, text, neg_text if cfg != 1.0 else None, steps, cfg, rescale)
    m = make_model(4, 256, 2, 256, 256, wi, wo, bps, bws)
    dn, dc, dt, dnt = _dev(torch_cuda, noise, cond, text, neg_text)
    got = m.sample(dn, dc, dt, dnt if cfg != 1.0 else None, steps, cfg, rescale)
    torch_cuda.cuda.synchronize()
    assert m.device_error() == 0
    got = got.cpu().numpy()
    p = parity.metrics(noise - got, noise - want)
    assert p["finite"] and p["nrmse"] <= 0.02 and p["cosine"] >= 0.9998, p
    if steps == 1 and cfg == 1.0:
        # one unguided step is the Euler step of s2_dit_euler_step
        x0 = m.euler_step(dn, dc, dt, 1000.0)
        torch_cuda.cuda.synchronize()
        assert np.array_equal(x0.cpu().numpy(), got)
    # again, in place on a copy of the noise: the same result
    x = dn.clone()
    m.sample(x, dc, dt, dnt if cfg != 1.0 else None, steps, cfg, rescale, out=x)
    torch_cuda.cuda.synchronize()
    assert np.array_equal(x.cpu().numpy(), got)
