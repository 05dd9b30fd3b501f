"""Write a small synthetic dataset in the formats the packing loader reads.

Same output layout as the reference's scripts/make_sample_data.py (videos.csv with ``latent_path``
and ``caption`` columns, one ``latent`` [48, T, H, W] safetensors file per clip, and an
``images.tar`` of ``<key>.safetensors`` / ``<key>.txt`` pairs).  Latents are Gaussian noise and
captions are placeholder JSON documents with the structured-caption fields (multi-line, so the CSV
reader's quoted-field handling is exercised).  For format checks and smoke tests, not for training.

    python -m pan2_b200.data.make_sample_data --output sample_data
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import tarfile
from pathlib import Path
from typing import Sequence, Tuple

import torch

LATENT_CHANNELS = 48
IMAGE_GRIDS: Tuple[Tuple[int, int], ...] = ((44, 78), (78, 44), (48, 28), (32, 32), (40, 60))


def placeholder_video_caption(index: int, seconds: float) -> str:
    mid = round(seconds / 2, 1)
    end = round(seconds, 1)
    events = []
    for k, (a, b) in enumerate(((0.0, mid), (mid, end))):
        events.append({"event_index": k, "timestamp": f"{a} - {b}", "event_description": f"Placeholder event {k}.",
                       "camera_motion": [{"timestamp": f"{a} - {b}", "camera_motion": ["static"]}],
                       "contained_actions": [{"timestamp": f"{a} - {b}",
                                              "action": "<|Subject1|> placeholder action"}]})
    doc = {"video_style": "Placeholder", "lighting": "Placeholder", "perspective_view": "Placeholder",
           "subjects_lifecycle": [{"subject_id": "<|Subject1|>", "display_name": f"Placeholder subject {index}",
                                   "subject_attribute": "Placeholder"}],
           "init_frame_visual_description": f"Synthetic sample {index} (random-noise latent).",
           "events": events, "quality": "Placeholder"}
    return json.dumps(doc, indent=2)


def placeholder_image_caption(index: int) -> str:
    return json.dumps({"events": [{"init_frame_visual_description": f"Synthetic image {index}; random latent."}]})


def write_sample_data(output: str, num_videos: int = 10, num_images: int = 10, latent_frames: int = 31,
                      height: int = 44, width: int = 78, fps: float = 24.0, seed: int = 0,
                      image_grids: Sequence[Tuple[int, int]] = IMAGE_GRIDS,
                      channels: int = LATENT_CHANNELS) -> Path:
    from safetensors.torch import save, save_file
    out = Path(output).resolve()
    (out / "latents").mkdir(parents=True, exist_ok=True)
    g = torch.Generator().manual_seed(seed)
    seconds = ((latent_frames - 1) * 4 + 1) / fps
    with open(out / "videos.csv", "w", newline="", encoding="utf-8") as f:
        w = csv.writer(f, quoting=csv.QUOTE_ALL)
        w.writerow(["latent_path", "caption"])
        for i in range(num_videos):
            path = out / "latents" / f"video_{i:02d}.safetensors"
            lat = torch.randn((channels, latent_frames, height, width), generator=g).to(torch.bfloat16)
            save_file({"latent": lat}, str(path))
            w.writerow([str(path), placeholder_video_caption(i, seconds)])
    with tarfile.open(out / "images.tar", "w") as tar:
        for i in range(num_images):
            h, wd = image_grids[i % len(image_grids)]
            lat = torch.randn((channels, 1, h, wd), generator=g).to(torch.bfloat16)
            for name, data in ((f"{i:08d}.safetensors", save({"latent": lat})),
                               (f"{i:08d}.txt", placeholder_image_caption(i).encode())):
                info = tarfile.TarInfo(name)
                info.size = len(data)
                tar.addfile(info, io.BytesIO(data))
    return out


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--output", default="sample_data")
    p.add_argument("--num_videos", type=int, default=10)
    p.add_argument("--num_images", type=int, default=10)
    p.add_argument("--latent_frames", type=int, default=31, help="latent T; 31 latent frames = 121 video frames")
    p.add_argument("--height", type=int, default=44, help="latent H (44 = 704 px)")
    p.add_argument("--width", type=int, default=78, help="latent W (78 = 1248 px)")
    p.add_argument("--fps", type=float, default=24.0)
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    out = write_sample_data(a.output, a.num_videos, a.num_images, a.latent_frames, a.height, a.width, a.fps, a.seed)
    print(f"wrote {a.num_videos} videos and {a.num_images} images to {out}")


if __name__ == "__main__":
    main()
