"""Wan VAE adapter with a stand-in ``diffusers.models.AutoencoderKLWan`` (diffusers and the VAE weights
are not in this image): resize-to-cover + centre crop, [-1, 1] pixels, latent (de)normalisation with
the VAE's per-channel mean / std, and the [-1, 1] -> [0, 1] decode mapping."""
import sys
import types

import torch

C = 4  # latent channels of the stand-in (the real VAE has 48)


class _Dist:
    def __init__(self, z):
        self._z = z

    def mode(self):
        return self._z


class _FakeVAE(torch.nn.Module):
    """Latent = the 3 pixel channels plus a copy of the first: an invertible toy mapping."""

    def __init__(self):
        super().__init__()
        self.config = types.SimpleNamespace(latents_mean=[0.5, -0.25, 1.0, 0.0], latents_std=[2.0, 0.5, 1.0, 4.0])

    @classmethod
    def from_pretrained(cls, *a, **k):
        return cls()

    def encode(self, pix):  # [1, 3, 1, H, W] -> [1, C, 1, H, W]
        z = torch.cat([pix, pix[:, :1]], dim=1)
        return types.SimpleNamespace(latent_dist=_Dist(z))

    def decode(self, lat, return_dict=False):
        return (lat[:, :3],)


def test_encode_normalises_and_decode_inverts(monkeypatch):
    from PIL import Image
    mod = types.ModuleType("diffusers.models")
    mod.AutoencoderKLWan = _FakeVAE
    pkg = types.ModuleType("diffusers")
    pkg.models = mod
    monkeypatch.setitem(sys.modules, "diffusers", pkg)
    monkeypatch.setitem(sys.modules, "diffusers.models", mod)
    from pan2_b200.models.vae import WanVAE
    vae = WanVAE(device="cpu", dtype=torch.float32)
    # a 40 x 20 image covers a 16 x 16 target after a 0.8 zoom (32 x 16), then a centre crop
    img = Image.new("RGB", (40, 20), (255, 0, 128))
    z = vae.encode_image(img, 16, 16)
    assert z.shape == (1, C, 1, 16, 16)
    mean = torch.tensor([0.5, -0.25, 1.0, 0.0]).view(1, -1, 1, 1, 1)
    std = torch.tensor([2.0, 0.5, 1.0, 4.0]).view(1, -1, 1, 1, 1)
    pix = z * std + mean  # undo the normalisation: the stand-in latent is the [-1, 1] pixels
    assert torch.allclose(pix[0, 0], torch.ones(1, 16, 16), atol=1e-2)        # red 255 -> +1
    assert torch.allclose(pix[0, 1], -torch.ones(1, 16, 16), atol=1e-2)       # green 0 -> -1
    assert torch.allclose(pix[0, 2], torch.full((1, 16, 16), 128 / 127.5 - 1), atol=1e-2)
    video = vae.decode(z)
    assert video.shape == (1, 3, 1, 16, 16) and video.dtype == torch.float32
    assert torch.allclose(video[0, :, 0, 0, 0], torch.tensor([1.0, 0.0, 128 / 255]), atol=1e-2)
