"""Rectified-flow math: the noising path, timestep draws inside (0, T), and the fixed / dynamic time
shift (monotone, endpoints fixed, the calibration points of the dynamic rule)."""
import math

import pytest
import torch

from pan2_b200.diffusion.flow_matching import draw_timesteps, interpolate, shift_timesteps


def test_interpolate_is_the_straight_path():
    x0, eps = torch.randn(3, 4, 5), torch.randn(3, 4, 5)
    t = torch.tensor([0.0, 250.0, 1000.0])
    x = interpolate(x0, eps, t, dim=0, T=1000)
    assert torch.allclose(x[0], x0[0]) and torch.allclose(x[2], eps[2])
    assert torch.allclose(x[1], 0.75 * x0[1] + 0.25 * eps[1])
    # the velocity target noise - x0 is the derivative of the path in t / T
    h = 1e-3
    d = (interpolate(x0, eps, t + h * 1000, T=1000) - x) / h
    assert torch.allclose(d[1], (eps - x0)[1], atol=1e-3)


@pytest.mark.parametrize("dist", ["uniform", "lognorm"])
def test_draws_stay_inside_the_interval(dist):
    g = torch.Generator().manual_seed(0)
    t = draw_timesteps(10000, "cpu", g, distribution=dist, T=1000)
    assert t.min() > 0 and t.max() < 1000
    if dist == "lognorm":  # sigmoid of N(0, 1): median at T / 2
        assert abs(t.median().item() - 500) < 20


def test_fixed_shift_is_monotone_with_fixed_endpoints():
    t = torch.linspace(0, 1000, 101)
    s = shift_timesteps(t, 1000, 9.0)
    assert s[0] == 0 and s[-1] == pytest.approx(1000)
    assert torch.all(s[1:] >= s[:-1]) and torch.all(s[1:-1] > t[1:-1])  # shift > 1 moves toward noise
    assert s[50].item() == pytest.approx(9 * 0.5 / (1 + 8 * 0.5) * 1000)
    assert torch.equal(shift_timesteps(t, 1000, 1.0), t)


def test_dynamic_shift_calibration():
    t = torch.full((2,), 500.0)
    # latent grids (frames, h, w): 121 frames of 1024 x 1024 pixels, and one 256 x 256 image
    shapes = torch.tensor([[31, 64, 64], [1, 16, 16]])
    out = shift_timesteps(t, 1000, mode="dynamic", latent_shapes=shapes, rescale_factor=1.0)
    s_video = math.exp(1.15 + 1.64)
    s_image = math.exp(0.5 + 0.0)
    for got, s in zip(out.tolist(), (s_video, s_image)):
        assert got == pytest.approx(s * 0.5 / (1 + (s - 1) * 0.5) * 1000, rel=1e-5)
    with pytest.raises(ValueError):
        shift_timesteps(t, 1000, mode="dynamic")
