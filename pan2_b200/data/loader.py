"""Packed latent loader: a background packing thread feeding GPU batch assembly.

Behaviour of the reference's PackedIterator (dataset/packed_dataloader.py:84-468): a producer packs
items into :class:`~pan2_b200.data.packing.PackedPlan` objects (CPU; latents read by a thread pool);
the consumer copies each plan's latents to the GPU from pinned memory, draws one timestep per sample
(logit-normal or uniform, then the fixed or resolution-dependent shift), noises every frame, builds
the channel-concat model input ``[x_t (C), clean prefix (C), prefix mask (1)]``, patchifies it to
``[C_in, n_video, 1, 1]``, computes the velocity target ``noise - x_0`` ``[n_video, C*pt*ph*pw]``, embeds
the captions and builds :class:`~pan2_b200.models.packed.PackedSequenceParams`.  The yielded
:class:`LoaderMeta` carries the dataloader state that resumes exactly after this batch.
"""
from __future__ import annotations

import queue
import threading
from dataclasses import dataclass
from typing import Dict, Iterator, Optional, Tuple

import torch

from ..diffusion.flow_matching import draw_timesteps, interpolate, shift_timesteps
from ..models.packed import build_packed_params
from .packing import DataloaderState, PackedPlan, PackingDataset
from .patching import patchify


@dataclass
class LoaderMeta:
    active_sequence_count: int
    active_joint_length: int
    active_video_length: int
    active_caption_length: int
    active_image_count: int
    dataloader_state: DataloaderState


CONDITIONING_SCHEMAS = ("token_concat", "channel_concat")


def _producer(it: Iterator[PackedPlan], q: "queue.Queue", stop: threading.Event):
    try:
        for plan in it:
            # pin the latents here so the consumer's H2D copies are asynchronous
            if torch.cuda.is_available():
                for item in plan.items:
                    item.latent = item.latent.pin_memory()
            if not _put_until_stopped(q, plan, stop):
                return
        _put_until_stopped(q, None, stop)
    except BaseException as e:  # surfaced on the consumer side
        _put_until_stopped(q, e, stop)


def _put_until_stopped(q: "queue.Queue", obj, stop: threading.Event) -> bool:
    """Put ``obj`` into ``q``, giving up once ``stop`` is set; True when it was put."""
    while not stop.is_set():
        try:
            q.put(obj, timeout=0.5)
            return True
        except queue.Full:
            continue
    return False


class PackedLoader:
    """Iterator of ``(batch dict, LoaderMeta)``; the batch dict has the trainer's keys
    ``hidden_states, timestep, text_states, target, packed_seq_params``."""

    def __init__(self, dataset: PackingDataset, *, device, dtype=torch.bfloat16, prefetch: int = 2, seed: int = 0,
                 T: int = 1000, timestep_distribution: str = "lognorm", timestep_loc: float = 0.0,
                 timestep_scale: float = 1.0, shift: float = 1.0, shift_mode: str = "fixed",
                 shift_kwargs: Optional[Dict] = None, start_index: int = 0,
                 conditioning_schema: str = "channel_concat"):
        if conditioning_schema not in CONDITIONING_SCHEMAS:
            raise ValueError(f"conditioning_schema must be one of {CONDITIONING_SCHEMAS}, got {conditioning_schema!r}")
        # channel_concat: every frame noised, [clean prefix frames | prefix mask] appended as 49 extra
        # channels (2 * 48 + 1 = 97 inputs); token_concat: the 48 noised channels alone
        # (reference: dataset/packed_dataloader.py:388-418)
        self.channel_concat = conditioning_schema == "channel_concat"
        self.dataset = dataset
        self.device = torch.device(device)
        self.dtype = dtype
        self.prefetch = prefetch
        # every batch reseeds both generators from (seed, batch index), so a resumed run that starts
        # at batch ``start_index`` draws exactly what the uninterrupted run drew
        self.seed = seed
        self.batch_index = start_index
        self.cpu_rng = torch.Generator()
        self.dev_rng = torch.Generator(device=self.device)
        self.T, self.dist, self.loc, self.scale = T, timestep_distribution, timestep_loc, timestep_scale
        self.shift, self.shift_mode, self.shift_kwargs = shift, shift_mode, dict(shift_kwargs or {})
        # the dynamic shift reads each item's token grid; these strides turn it back into frames and
        # pixels (Wan 2.2: 4 frames and 16 x 16 pixels per latent, times the patch; reference:
        # train.py:1349-1358)
        pt, ph, pw = tuple(getattr(dataset, "patch_size", (1, 2, 2)))
        self.shift_kwargs.setdefault("frame_stride", 4 * pt)
        self.shift_kwargs.setdefault("pixel_stride_h", 16 * ph)
        self.shift_kwargs.setdefault("pixel_stride_w", 16 * pw)
        self._stop = threading.Event()
        self._thread = None
        self._q = None

    def __iter__(self):
        # a second iter() stops the previous producer first (each producer gets its own stop event,
        # so the old one cannot keep filling a queue that nobody reads)
        self.close()
        self._q = queue.Queue(maxsize=self.prefetch)
        self._stop = threading.Event()
        self._thread = threading.Thread(target=_producer, args=(iter(self.dataset), self._q, self._stop), daemon=True)
        self._thread.start()
        return self

    def __next__(self) -> Tuple[Dict, LoaderMeta]:
        if self._q is None:
            iter(self)
        plan = self._q.get()
        if plan is None:
            raise StopIteration
        if isinstance(plan, BaseException):
            raise plan
        return self.assemble(plan)

    def close(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    @torch.no_grad()
    def assemble(self, plan: PackedPlan) -> Tuple[Dict, LoaderMeta]:
        dev = self.device
        pt, ph, pw = self.dataset.patch_size
        n = len(plan.items)
        self.cpu_rng.manual_seed((self.seed * 1000003 + self.batch_index) % (2 ** 62))
        self.dev_rng.manual_seed((self.seed * 1000003 + self.batch_index + 7) % (2 ** 62))
        self.batch_index += 1
        t = draw_timesteps(n, "cpu", self.cpu_rng, distribution=self.dist, T=self.T, loc=self.loc, scale=self.scale)
        t = shift_timesteps(t, self.T, self.shift, self.shift_mode,
                            latent_shapes=torch.tensor([list(g) for g in plan.grids], dtype=torch.float32),
                            **self.shift_kwargs)
        # rounded to the batch dtype (bf16 in bf16 runs) before the noising and the timestep
        # embedding read it, as the reference loader does (dataset/packed_dataloader.py:370-374)
        t = t.to(self.dtype).float()
        t_dev = t.to(dev, non_blocking=True)
        inputs, targets = [], []
        for i, item in enumerate(plan.items):
            x0 = item.latent.to(dev, non_blocking=True).float()
            noise = torch.randn(x0.shape, device=dev, generator=self.dev_rng)
            xt = interpolate(x0.unsqueeze(0), noise.unsqueeze(0), t_dev[i:i + 1], dim=0, T=self.T)[0]
            C, Tl, H, W = x0.shape
            if self.channel_concat:
                cond = x0.new_zeros(C + 1, Tl, H, W)
                k = min(item.prefix_frames, Tl)
                if k > 0:
                    cond[:C, :k] = x0[:, :k]
                    cond[C, :k] = 1.0
                xt = torch.cat([xt, cond], 0)
            inputs.append(patchify(xt, (pt, ph, pw)))
            targets.append(patchify(noise - x0, (pt, ph, pw)).t())
        hidden = torch.cat(inputs, 1).to(self.dtype)[:, :, None, None].contiguous()
        target = torch.cat(targets, 0).to(self.dtype).contiguous()
        text = self.dataset.codec.embed([it.caption for it in plan.items], dev).to(self.dtype)
        meta = build_packed_params(plan.video_lens, plan.caption_lens, plan.total, plan.freqs_cos, plan.freqs_sin)
        meta = meta.to(dev, non_blocking=True)
        batch = dict(hidden_states=hidden, timestep=t_dev.float(), text_states=text.contiguous(), target=target,
                     packed_seq_params=meta)
        lm = LoaderMeta(n, sum(plan.video_lens) + sum(plan.caption_lens), sum(plan.video_lens),
                        sum(plan.caption_lens), plan.num_images, plan.state)
        return batch, lm
