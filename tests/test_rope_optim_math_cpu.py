"""Plain-math checks of the RoPE tables, patchify and the optimizer's element-wise CPU paths (the
CUDA kernels are tested against these same paths on the GPU)."""
import math

import torch

from pan2_b200.data.patching import packed_rope_tables, patchify, unpatchify
from pan2_b200.models.rope import apply_rope, rope_tables_for_grid, rotate_half
from pan2_b200.optim import flat_ops as F


def test_rope_preserves_norms_and_relative_angles():
    axes = (16, 24, 24)
    cos, sin = rope_tables_for_grid(axes, (2, 3, 4), theta=256.0)
    assert cos.shape == (24, 64) and torch.allclose(cos ** 2 + sin ** 2, torch.ones_like(cos))
    q = torch.randn(24, 2, 64)
    k = torch.randn(24, 2, 64)
    qr, kr = apply_rope(q, k, (cos, sin))
    assert torch.allclose(qr.norm(dim=-1), q.norm(dim=-1), atol=1e-4)  # rotations
    # the same vector at two positions: the dot product depends only on the position difference
    v = torch.randn(64)
    x = v.expand(24, 1, 64).contiguous()
    xr, _ = apply_rope(x, x, (cos, sin))
    d01 = (xr[0, 0] * xr[1, 0]).sum()
    d12 = (xr[1, 0] * xr[2, 0]).sum()  # positions (0,0,0)->(0,0,1) and (0,0,1)->(0,0,2)
    assert torch.allclose(d01, d12, atol=1e-4)
    assert torch.equal(rotate_half(torch.tensor([1.0, 2.0, 3.0, 4.0])), torch.tensor([-2.0, 1.0, -4.0, 3.0]))


def test_packed_rope_tables_leave_text_rows_unrotated():
    axes = (16, 24, 24)
    cos, sin = packed_rope_tables(axes, 256.0, (1.0, 1.0, 1.0), [(1, 2, 2), (2, 1, 2)], [3, 5], 20)
    c0, s0 = rope_tables_for_grid(axes, (1, 2, 2), theta=256.0)
    assert torch.equal(cos[:4], c0) and torch.equal(sin[:4], s0)
    assert torch.all(cos[4:7] == 1) and torch.all(sin[4:7] == 0)       # caption of sample 0
    assert torch.all(cos[11:] == 1) and torch.all(sin[11:] == 0)       # caption of sample 1 + padding


def test_patchify_round_trip():
    lat = torch.randn(5, 4, 6, 8)
    tok = patchify(lat, (1, 2, 2))
    assert tok.shape == (5 * 4, 4 * 3 * 4)
    assert torch.equal(unpatchify(tok.t(), (4, 3, 4), (1, 2, 2), 5), lat)


def test_master_halves_are_exact():
    x = torch.randn(1000) * 10
    hi = torch.empty(1000, dtype=torch.bfloat16)
    lo = torch.empty(1000, dtype=torch.int16)
    F.split_master(x, hi, lo)
    assert torch.equal(F.join_master(hi, lo), x)
    # hi is x truncated toward zero to bf16
    assert torch.all(hi.float().abs() <= x.abs()) and torch.all((hi.float() - x).abs() <= x.abs() * 2 ** -7)


def test_muon_and_adamw_element_math():
    n = 64
    g = torch.randn(n)
    clip = torch.tensor([0.5])
    buf = torch.randn(n)
    buf0 = buf.clone()
    out = torch.empty(n)
    F.muon_momentum(buf, g, clip, 0.95, out)
    gi = g * 0.5
    assert torch.allclose(buf, 0.95 * buf0 + 0.05 * gi)
    assert torch.allclose(out, 0.05 * gi + 0.95 * buf)           # Nesterov look-ahead
    x = torch.randn(n)
    hi, lo = torch.empty(n, dtype=torch.bfloat16), torch.empty(n, dtype=torch.int16)
    F.split_master(x, hi, lo)
    u = torch.randn(n)
    F.muon_update(hi, lo, u, torch.tensor([1e-2]), 0.2, 0.1)
    assert torch.allclose(F.join_master(hi, lo), x * (1 - 1e-2 * 0.1) - 1e-2 * 0.2 * u, atol=1e-6)
    F.split_master(x, hi, lo)
    m, v = torch.zeros(n), torch.zeros(n)
    F.adamw_update(hi, lo, g, m, v, None, torch.tensor([1e-3]), 0.9, 0.95, 1e-8, 0.05, 1)
    # first step: m / (sqrt(v) / sqrt(bc2)) / bc1 = sign(g) (up to eps)
    expect = x * (1 - 1e-3 * 0.05) - 1e-3 * g.sign()
    assert torch.allclose(F.join_master(hi, lo), expect, atol=1e-5)


def test_global_norm_clip_factor():
    parts = torch.tensor([9.0, 16.0, 0.0])
    out = torch.empty(2)
    F.norm_and_clip(parts, 1.0, out)
    assert out[0].item() == 5.0 and math.isclose(out[1].item(), 1.0 / (5.0 + 1e-6), rel_tol=1e-6)
    F.norm_and_clip(parts, 10.0, out)
    assert out[1].item() == 1.0
