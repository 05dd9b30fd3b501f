"""Packed-sequence metadata shared by the dataloader, the model and the kernels.

Two token layouts are used for one packed batch of ``k`` samples (video ``v_i`` + caption ``t_i``),
matching the reference's ``PackedSequenceParams`` (pan/models/transformers/pan_transformer.py:622-668):

* concat layout ``[v_1 .. v_k, t_1 .. t_k, pad]``: the per-modality GEMMs see two contiguous row
  segments (video rows, then text rows);
* interleave layout ``[v_1, t_1, .., v_k, t_k, pad]``: attention sees one contiguous joint
  segment per sample.

``concat = interleave[interleave_to_concat]`` and ``interleave = concat[concat_to_interleave]``;
padding rows map to themselves.

Unlike the reference, every boundary is ALSO kept as a host-side Python int/list.  The batch is
assembled on the host anyway, so kernels get exact grids without a device read-back.
"""
from __future__ import annotations

from dataclasses import dataclass, field, fields, replace
from typing import List, Optional, Sequence

import torch


@dataclass
class PackedSequenceParams:
    caption_cu_seqlens: torch.Tensor          # [k+1] int32, caption rows (text block, concat order)
    video_cu_seqlens: torch.Tensor            # [k+1] int32, video rows
    caption_segment_limit: int
    joint_cu_seqlens: torch.Tensor            # [k+1] int32, interleave layout (full sequence under CP)
    indices_interleave_to_concat: torch.Tensor  # [L] int32
    indices_concat_to_interleave: torch.Tensor  # [L] int32
    cu_seqlens_concat: torch.Tensor           # [k+2] int32: k video segments + 1 merged text segment
    cu_seqlens_matmul: torch.Tensor           # [3] int32: [0, n_video, n_video + n_text]
    joint_segment_limit: int
    freqs_cos: torch.Tensor                   # [L, 1, D] fp32, interleave layout
    freqs_sin: torch.Tensor
    active_sequence_count: torch.Tensor       # [] int32
    joint_packed_length: int
    # Host copies of the boundaries (local coordinates).
    video_lens: List[int] = field(default_factory=list)
    caption_lens: List[int] = field(default_factory=list)
    joint_lens: List[int] = field(default_factory=list)   # full-sequence lengths under CP
    # Context parallelism (strided shard of the joint sequence).
    cp_text_index: Optional[torch.Tensor] = None
    cp_joint_total: Optional[int] = None
    cp_caption_lens: Optional[List[int]] = None   # full per-sample caption lengths (caption encoder)
    cp_group: Optional[object] = None             # the cp process group of this shard

    @property
    def num_samples(self) -> int:
        return len(self.video_lens)

    @property
    def n_video(self) -> int:
        return int(sum(self.video_lens))

    @property
    def n_text(self) -> int:
        return int(sum(self.caption_lens))

    @property
    def n_active(self) -> int:
        return self.n_video + self.n_text

    @property
    def concat_bounds(self) -> List[int]:
        """Host copy of ``cu_seqlens_concat``."""
        out = [0]
        for n in self.video_lens:
            out.append(out[-1] + n)
        out.append(out[-1] + self.n_text)
        return out

    @property
    def max_joint_len(self) -> int:
        return max(self.joint_lens) if self.joint_lens else 0

    def to(self, device, non_blocking: bool = False) -> "PackedSequenceParams":
        kw = {}
        for f in fields(self):
            v = getattr(self, f.name)
            if isinstance(v, torch.Tensor):
                kw[f.name] = v.to(device, non_blocking=non_blocking)
        return replace(self, **kw)

    def tensors(self):
        return {f.name: getattr(self, f.name) for f in fields(self) if isinstance(getattr(self, f.name), torch.Tensor)}


def _cu(lens: Sequence[int]) -> List[int]:
    out = [0]
    for n in lens:
        out.append(out[-1] + int(n))
    return out


def layout_permutations(video_lens: Sequence[int], caption_lens: Sequence[int], total: int):
    """``(interleave_to_concat, concat_to_interleave)`` as int64 CPU tensors of length ``total``.

    concat position ``p`` holds the token stored at interleave position ``interleave_to_concat[p]``.
    """
    k = len(video_lens)
    n_video = sum(video_lens)
    n_active = n_video + sum(caption_lens)
    if total < n_active:
        raise ValueError(f"total length {total} < active tokens {n_active}")
    itc = torch.empty(total, dtype=torch.int64)
    pos_inter = 0
    vstart = 0
    tstart = n_video
    for i in range(k):
        v, t = int(video_lens[i]), int(caption_lens[i])
        itc[vstart:vstart + v] = torch.arange(pos_inter, pos_inter + v)
        pos_inter += v
        itc[tstart:tstart + t] = torch.arange(pos_inter, pos_inter + t)
        pos_inter += t
        vstart += v
        tstart += t
    itc[n_active:] = torch.arange(n_active, total)
    cti = torch.empty_like(itc)
    cti[itc] = torch.arange(total)
    return itc, cti


def build_packed_params(video_lens: Sequence[int], caption_lens: Sequence[int], total: int,
                        freqs_cos: torch.Tensor, freqs_sin: torch.Tensor,
                        joint_segment_limit: Optional[int] = None,
                        caption_segment_limit: Optional[int] = None) -> PackedSequenceParams:
    """Build CPU packed metadata from per-sample lengths.

    ``freqs_cos``/``freqs_sin`` are ``[total, D]`` (or ``[total, 1, D]``) in interleave layout.
    """
    video_lens = [int(v) for v in video_lens]
    caption_lens = [int(t) for t in caption_lens]
    joint_lens = [v + t for v, t in zip(video_lens, caption_lens)]
    itc, cti = layout_permutations(video_lens, caption_lens, total)
    n_video = sum(video_lens)
    concat = _cu(video_lens) + [n_video + sum(caption_lens)]
    i32 = lambda xs: torch.tensor(xs, dtype=torch.int32)
    if freqs_cos.ndim == 2:
        freqs_cos, freqs_sin = freqs_cos.unsqueeze(1), freqs_sin.unsqueeze(1)
    return PackedSequenceParams(
        caption_cu_seqlens=i32(_cu(caption_lens)),
        video_cu_seqlens=i32(_cu(video_lens)),
        caption_segment_limit=int(caption_segment_limit or max(caption_lens or [1])),
        joint_cu_seqlens=i32(_cu(joint_lens)),
        indices_interleave_to_concat=itc.to(torch.int32),
        indices_concat_to_interleave=cti.to(torch.int32),
        cu_seqlens_concat=i32(concat),
        cu_seqlens_matmul=i32([0, n_video, n_video + sum(caption_lens)]),
        joint_segment_limit=int(joint_segment_limit or max(joint_lens or [1])),
        freqs_cos=freqs_cos.float().contiguous(),
        freqs_sin=freqs_sin.float().contiguous(),
        active_sequence_count=torch.tensor(len(video_lens), dtype=torch.int32),
        joint_packed_length=int(total),
        video_lens=video_lens,
        caption_lens=caption_lens,
        joint_lens=joint_lens,
    )
