"""Per-item reading: precomputed Wan-2.2 latents and captions, task draws and token-budget checks.

Formats (reference dataset/video_item_processor.py and image_item_processor.py):

* video: one ``.safetensors`` file per CSV row (column ``latent_path``) holding ``latent``
  ``[C, T, H, W]`` (a leading batch dim of 1 is dropped); caption in column ``caption``;
* image: WebDataset-style tar shards of ``<key>.safetensors`` (``latent`` ``[C, 1, H, W]``) +
  ``<key>.txt`` caption pairs.

Each video item draws its task from an RNG seeded by its position (so a resumed run draws the same):
video continuation with ``video_cond_prob`` (a random prefix of latent frames is clean context),
image-to-video with ``image_cond_prob`` (first latent frame), otherwise text-to-video; captions are
dropped (the classifier-free-guidance empty caption) with ``cfg_drop_prob``.  Items that exceed any
budget (joint, video, caption, text-encoder tokens, per-sequence limits) are skipped.

Captions reach the model as text-encoder embeddings ``[n, 4096]``; :class:`CaptionCodec` is the
interface (tokenize to a length, embed a batch).  The Qwen implementation lives in
:mod:`pan2_b200.models.text_encoder`; :class:`HashCaptionCodec` is a deterministic stand-in for
offline tests and synthetic runs.
"""
from __future__ import annotations

import hashlib
import io
import logging
import random
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

log = logging.getLogger("pan2_b200.data")


def decode_latent(raw: bytes, where: str = "") -> torch.Tensor:
    from safetensors.torch import load as st_load
    tensors = st_load(raw)
    if "latent" not in tensors:
        raise KeyError(f"expected a 'latent' tensor{(' in ' + where) if where else ''}, got {list(tensors)}")
    lat = tensors["latent"]
    if lat.dim() == 5 and lat.shape[0] == 1:
        lat = lat[0]
    if lat.dim() != 4:
        raise ValueError(f"expected a [C, T, H, W] latent{(' in ' + where) if where else ''}, got {tuple(lat.shape)}")
    return lat.contiguous()


def load_latent(path: str) -> torch.Tensor:
    with open(path, "rb") as f:
        return decode_latent(f.read(), path)


@dataclass
class ItemRef:
    """JSON-serialisable locator of one item (video CSV row or image tar member)."""
    global_index: int
    modality: str = "video"
    csv_index: int = -1
    local_index: int = -1
    local_file_pos: int = -1
    local_line_num: int = -1
    epoch_index: int = 0
    shard_index: int = -1
    sample_index: int = -1
    cycle: int = 0
    # image members' byte ranges in an uncompressed tar: [latent offset, latent size, caption
    # offset, caption size], so a resumed loader reads a buffered image back without a tar scan
    tar_members: Optional[List[int]] = None


@dataclass
class Caption:
    """A caption as the text encoder sees it: ``full_length`` templated tokens of which the last
    ``cropped_length`` (after ``prefix_len``) become caption rows."""
    text: str
    full_length: int
    prefix_len: int
    cropped_length: int
    token_ids: Optional[torch.Tensor] = None


class CaptionCodec:
    """Text -> tokens -> embeddings."""
    embed_dim: int = 4096

    def tokenize(self, text: str, limit: int) -> Caption:
        raise NotImplementedError

    def empty(self, limit: int) -> Caption:
        return self.tokenize("", limit)

    def embed(self, captions: Sequence[Caption], device) -> torch.Tensor:
        """``[sum(cropped_length), embed_dim]`` caption rows, packed in order."""
        raise NotImplementedError


class HashCaptionCodec(CaptionCodec):
    """Deterministic stand-in: whitespace tokens, each embedded by a hash-seeded Gaussian vector.
    Used when no text encoder is available (tests, synthetic smoke runs)."""

    def __init__(self, embed_dim: int = 4096, prefix_len: int = 4):
        self.embed_dim = embed_dim
        self.prefix_len = prefix_len

    def tokenize(self, text: str, limit: int) -> Caption:
        words = text.split()[: max(0, limit - 1)] + ["<eos>"]
        ids = torch.tensor([int(hashlib.md5(w.encode()).hexdigest()[:8], 16) for w in words], dtype=torch.long)
        n = len(words)
        return Caption(text=text, full_length=n + self.prefix_len, prefix_len=self.prefix_len, cropped_length=n,
                       token_ids=ids)

    def embed(self, captions: Sequence[Caption], device) -> torch.Tensor:
        rows = []
        for c in captions:
            for tid in c.token_ids.tolist():
                g = torch.Generator().manual_seed(tid % (2 ** 31))
                rows.append(torch.randn(self.embed_dim, generator=g))
        if not rows:
            return torch.zeros(0, self.embed_dim, device=device)
        return torch.stack(rows).to(device)


@dataclass
class Budgets:
    joint: int
    video: int
    caption: int
    text_encoder: int
    joint_segment: int
    caption_segment: int
    text_encoder_segment: int = 1 << 30
    max_num_seq: int = 8


@dataclass
class Item:
    """A decoded sample ready for packing."""
    ref: ItemRef
    latent: torch.Tensor                 # [C, T, H, W]
    caption: Caption
    prefix_frames: int                   # clean latent frames given as context (i2v / v2v)
    n_video_tokens: int
    grid: Tuple[int, int, int]           # token grid (t, h, w)
    modality: str = "video"
    resume: Any = None


def draw_task(seed: int, ref: ItemRef, latent_steps: int, video_cond_prob: float, image_cond_prob: float,
              cfg_drop_prob: float) -> Tuple[int, bool]:
    """``(prefix latent frames, drop caption)`` from an RNG seeded by the item's position: with
    ``video_cond_prob`` a continuation prefix of 1 .. T // 2 latent frames, with ``image_cond_prob``
    the first frame; clips of fewer than 2 latent frames get no prefix (reference:
    dataset/video_item_processor.py:239-250)."""
    rng = random.Random(hash((seed, ref.epoch_index, ref.global_index, ref.local_index, ref.local_file_pos)))
    u = rng.random()
    if latent_steps < 2:
        prefix = 0
    elif u < video_cond_prob:
        prefix = rng.randint(1, max(1, latent_steps // 2))
    elif u < video_cond_prob + image_cond_prob:
        prefix = 1
    else:
        prefix = 0
    drop = rng.random() < cfg_drop_prob
    return prefix, drop


def finalize_item(latent: torch.Tensor, text: str, ref: ItemRef, *, prefix_frames: int, drop_caption: bool,
                  codec: CaptionCodec, budgets: Budgets, patch_size, modality: str) -> Optional[Item]:
    """Tokenise and apply every budget check; None when the item cannot be packed."""
    pt, ph, pw = patch_size
    _, T, H, W = latent.shape
    if H % ph or W % pw or T % pt:
        log.warning(f"skipping {modality} item {ref.global_index}/{ref.shard_index}:{ref.sample_index}: latent grid "
                    f"{(T, H, W)} not divisible by patch {tuple(patch_size)}")
        return None
    grid = (T // pt, H // ph, W // pw)
    n_video = grid[0] * grid[1] * grid[2]
    cap = codec.empty(budgets.caption_segment) if drop_caption else codec.tokenize(text, budgets.caption_segment)
    c = cap.cropped_length
    for needed, limit, what in ((n_video + c, budgets.joint, "joint tokens (packed_joint_token_budget)"),
                                (cap.full_length, budgets.text_encoder, "templated text tokens (text-encoder budget)"),
                                (n_video, budgets.video, "video tokens (packed_video_token_budget)"),
                                (c, budgets.caption, "caption tokens (packed_caption_token_budget)"),
                                (cap.full_length, budgets.text_encoder_segment, "templated text tokens per item"),
                                (n_video + c, budgets.joint_segment, "joint tokens (packed_joint_segment_limit)"),
                                (c, budgets.caption_segment, "caption tokens (packed_caption_segment_limit)")):
        if needed > limit:
            log.warning(f"skipping {modality} item {ref.global_index}/{ref.shard_index}:{ref.sample_index}: "
                        f"needs {needed} {what} > {limit}")
            return None
    return Item(ref=ref, latent=latent, caption=cap, prefix_frames=prefix_frames, n_video_tokens=n_video, grid=grid,
                modality=modality)


def _plain_tar(path: str) -> bool:
    """True for an uncompressed tar, whose member data sit at fixed byte offsets of the file."""
    with open(path, "rb") as f:
        magic = f.read(6)
    return not (magic[:2] == b"\x1f\x8b" or magic[:3] == b"BZh" or magic == b"\xfd7zXZ\x00")


def iter_tar_samples(path: str, start: int = 0):
    """Yield ``(sample_index, key, latent_bytes, caption, members)`` from a WebDataset-style tar:
    every key with a ``.safetensors`` and a ``.txt`` member is one sample, numbered in tar order,
    from sample ``start`` on (the data of earlier samples is not read).  ``members`` is ``[latent
    offset, latent size, caption offset, caption size]`` in an uncompressed tar (``None`` in a
    compressed one); :func:`read_tar_sample` reads them back."""
    import tarfile
    plain = _plain_tar(path)
    pending: Dict[str, Dict[str, Any]] = {}
    idx = 0
    with tarfile.open(path, "r") as tf:
        for m in tf:
            if not m.isfile():
                continue
            key, _, ext = m.name.rpartition(".")
            entry = pending.setdefault(key, {})
            # plain tars are read at the recorded offsets once a sample is wanted; a compressed one
            # is read as it streams past (seeking back in it would decompress from the start)
            entry[ext] = (m, None if plain else tf.extractfile(m).read())
            if "safetensors" in entry and "txt" in entry:
                (lat, lat_b), (txt, txt_b) = entry["safetensors"], entry["txt"]
                del pending[key]
                if idx >= start:
                    if plain:
                        lat_b, txt_b = tf.extractfile(lat).read(), tf.extractfile(txt).read()
                    members = [lat.offset_data, lat.size, txt.offset_data, txt.size] if plain else None
                    yield idx, key, lat_b, txt_b.decode("utf-8", "ignore"), members
                idx += 1


def read_tar_sample(path: str, members: Sequence[int]) -> Tuple[bytes, str]:
    """``(latent_bytes, caption)`` of one sample from its member byte ranges (uncompressed tar)."""
    lat_off, lat_n, txt_off, txt_n = (int(v) for v in members)
    with open(path, "rb") as f:
        f.seek(lat_off)
        raw = f.read(lat_n)
        f.seek(txt_off)
        txt = f.read(txt_n)
    if len(raw) != lat_n or len(txt) != txt_n:
        raise ValueError(f"{path} is shorter than the recorded sample ranges {list(members)}")
    return raw, txt.decode("utf-8", "ignore")
