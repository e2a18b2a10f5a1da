"""Euler sampler and classifier-free guidance: the C restatement
(oracle/s2_oracle.c) against the reference's own EulerSampler
(src/model/sampler.cpp compiled into oracle/_ref), bit for bit, plus the
reference's known answers (tests/runtime_unit_test.cpp:62-82) and the host
helpers of the library (timesteps, condition ratio) that need no GPU."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import s2b200


@pytest.fixture(scope="module")
def sport():
    return oracle.SamplerPort(oracle.port().lib)


@pytest.fixture(scope="module")
def sref():
    r = oracle.ref()
    if r is None:
        pytest.skip("reference build (oracle/_ref) not available")
    return oracle.SamplerRef(r.lib)


def _pair(shape, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape).astype(np.float32), rng.standard_normal(shape).astype(np.float32))


def test_known_answers(sport, sref):
    # runtime_unit_test.cpp:62-82: cfg(2, 0, 1.5) = 3; endpoint(1, 0.25, t=1000) = 0.75
    pos, neg = np.full((1, 1, 1, 2), 2.0, np.float32), np.zeros((1, 1, 1, 2), np.float32)
    for s in (sport, sref):
        assert np.allclose(s.apply_cfg(pos, neg, 1.5, 0.0), 3.0, atol=1e-6)
        cur, pred = np.ones((1, 1, 1, 2), np.float32), np.full((1, 1, 1, 2), 0.25, np.float32)
        assert np.allclose(s.endpoint(pred, cur, 1000.0), 0.75, atol=1e-6)


@pytest.mark.parametrize("steps", [1, 2, 3, 4, 7, 50])
def test_timesteps(sport, sref, steps):
    t = sport.timesteps(steps)
    assert np.array_equal(t, sref.timesteps(steps))
    assert np.array_equal(t, s2b200.sampler_timesteps(steps))
    assert t[0] == 1000.0 and np.all(np.diff(t) < 0)


@pytest.mark.parametrize("shape", [(16, 2, 6, 10), (16, 1, 1, 1), (3, 5, 7, 11)])
@pytest.mark.parametrize("scale,rescale", [(1.0, 0.0), (2.5, 0.0), (3.0, 0.7), (5.0, 1.0), (0.5, 0.3)])
def test_cfg_matches_reference(sport, sref, shape, scale, rescale):
    pos, neg = _pair(shape, 7)
    a, b = sport.apply_cfg(pos, neg, scale, rescale), sref.apply_cfg(pos, neg, scale, rescale)
    assert np.array_equal(a, b)


def test_cfg_rescale_degenerate(sport, sref):
    # guided std == 0 (pos == neg constant): no rescale, as the reference's cfg_std > 0 guard
    pos = np.full((2, 1, 2, 2), 0.5, np.float32)
    for s in (sport, sref):
        assert np.array_equal(s.apply_cfg(pos, pos, 4.0, 0.7), pos)


@pytest.mark.parametrize("t,t_next", [(1000.0, 750.0), (750.0, 500.0), (333.33, 0.0), (1000.0, 1200.0),
                                      (100.0, -5.0)])
def test_step_to_and_endpoint_match_reference(sport, sref, t, t_next):
    pred, cur = _pair((16, 2, 6, 10), 11)
    assert np.array_equal(sport.step_to(pred, cur, t, t_next), sref.step_to(pred, cur, t, t_next))
    assert np.array_equal(sport.endpoint(pred, cur, t), sref.endpoint(pred, cur, t))


def test_step_to_final_timestep_zero_is_endpoint(sport):
    # t_next = 0: as = 1, bs = 0 -> 1 * x0 + 0 * xT = x0 exactly
    pred, cur = _pair((4, 2, 3, 5), 3)
    assert np.array_equal(sport.step_to(pred, cur, 250.0, 0.0), sport.endpoint(pred, cur, 250.0))


@pytest.mark.parametrize("noise_scale,T,H,W", [(0.0, 6, 90, 160), (0.1, 6, 90, 160), (0.25, 2, 16, 30),
                                               (1.0, 12, 134, 240)])
def test_condition_ratio(sport, noise_scale, T, H, W):
    r = sport.condition_ratio(noise_scale, T, H, W)
    assert np.float32(r) == np.float32(s2b200.condition_ratio(noise_scale, T, H, W))
    assert (r == 0.0) == (noise_scale == 0.0)
    if noise_scale > 0:
        assert 0.0 < r <= 1.0


def test_make_condition(sport):
    enc, noise = _pair((16, 2, 4, 6), 5)
    r = np.float32(sport.condition_ratio(0.2, 2, 4, 6))
    want = (np.float32(1.0) - r) * enc + r * noise
    assert np.array_equal(sport.make_condition(enc, noise, 0.2), want.astype(np.float32))
