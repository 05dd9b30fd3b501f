"""Wan 2.2 VAE adapter for the generation pipeline.

The DiT works in the normalised latent space of the Wan 2.2 TI2V VAE (48 channels, 16x spatial and 4x
temporal compression, the first frame in its own latent frame).  The VAE itself is a third-party
model (``diffusers.AutoencoderKLWan``, weights ``Wan-AI/Wan2.2-TI2V-5B-Diffusers``); this adapter loads
it when diffusers and the weights are present and exposes the two calls the pipeline makes
(reference: pan/pipelines/pan_video_pipeline.py:150-185, 536-546):

* ``encode_image(image, height, width)`` -- scale (Lanczos) to cover, centre-crop, map to [-1, 1],
  posterior mode, normalise with the VAE's latent mean / std -> ``[1, 48, 1, h, w]``;
* ``decode(latents)`` -- de-normalise, decode, map [-1, 1] -> [0, 1] -> float ``[B, 3, F, H, W]`` on CPU.
"""
from __future__ import annotations

from typing import Optional

import torch

WAN22_REPO = "Wan-AI/Wan2.2-TI2V-5B-Diffusers"


class WanVAE:
    def __init__(self, checkpoint: Optional[str] = None, device="cuda", dtype=torch.bfloat16):
        try:
            from diffusers.models import AutoencoderKLWan
        except ImportError as e:  # pragma: no cover - optional dependency
            raise ImportError("the Wan 2.2 VAE needs the diffusers package; without it run the pipeline with "
                              "output_type='latent' and reference latents") from e
        self.device = torch.device(device)
        self.dtype = dtype
        self.vae = AutoencoderKLWan.from_pretrained(checkpoint or WAN22_REPO, subfolder="vae",
                                                    torch_dtype=dtype).to(self.device).eval()
        cfg = self.vae.config
        self.mean = torch.tensor(cfg.latents_mean, device=self.device, dtype=dtype).view(1, -1, 1, 1, 1)
        self.std = torch.tensor(cfg.latents_std, device=self.device, dtype=dtype).view(1, -1, 1, 1, 1)

    def to(self, device) -> "WanVAE":
        """Move the VAE and its latent statistics (generation offloading parks it on the CPU)."""
        self.device = torch.device(device)
        self.vae.to(self.device)
        self.mean, self.std = self.mean.to(self.device), self.std.to(self.device)
        return self

    @torch.no_grad()
    def encode_image(self, image, height: int, width: int) -> torch.Tensor:
        import torchvision.transforms.functional as TF
        from PIL import Image
        from torchvision.transforms import InterpolationMode
        if isinstance(image, str):
            image = Image.open(image).convert("RGB")
        w0, h0 = image.size
        zoom = max(width / w0, height / h0)
        image = TF.resize(image, [int(round(h0 * zoom)), int(round(w0 * zoom))], interpolation=InterpolationMode.LANCZOS)
        pix = TF.normalize(TF.to_tensor(TF.center_crop(image, [height, width])), [0.5], [0.5])
        pix = pix[None, :, None].to(self.device, self.dtype)
        lat = self.vae.encode(pix).latent_dist.mode()
        return (lat - self.mean.to(lat.dtype)) / self.std.to(lat.dtype)

    @torch.no_grad()
    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        lat = latents.to(self.device, self.dtype) * self.std + self.mean
        pix = self.vae.decode(lat, return_dict=False)[0]
        return pix.mul(0.5).add(0.5).clamp(0, 1).float().cpu()
