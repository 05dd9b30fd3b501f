"""Host offloading for generation: models parked on the CPU between uses, DiT blocks streamed.

The reference pipeline has three runtime modes (pan/pipelines/pan_video_pipeline.py:111-158,
generate.py:391-423): ``none`` keeps every model on the GPU; ``models`` keeps the text encoder, the
DiT and the VAE on the CPU and moves each to the GPU only while it runs; ``blocks`` additionally
leaves the DiT's joint blocks in host memory and streams them to the GPU while the DiT runs.
``auto`` picks ``blocks`` when the DiT's weights do not fit in the GPU's free memory, else
``none``.  A B200 holds the bf16 29B DiT (58 GB) with room to spare, so ``auto`` resolves to
``none`` unless the GPU is shared.

:class:`BlockStreamer` is this framework's block streaming.  Every block's parameters and buffers
are packed, 256-byte aligned, into one flat host buffer per block (pinned when prefetching), and
two device slots of the largest block's size are allocated once.  Before block ``i`` runs its
tensors are re-pointed into a slot; with ``prefetch`` a copy stream loads the next block of the
run order into the other slot while block ``i`` computes (the copy waits for an event recorded
after the slot's previous block finished), so the transfer of one block overlaps the compute of
the one before it.  Without ``prefetch`` the host buffers stay pageable and each block is copied
on the compute stream right before it runs.  After a block runs its tensors point back at their
host buffers, so nothing outside the streamer holds slot memory.
"""
from __future__ import annotations

import itertools
from contextlib import contextmanager
from typing import Iterable, Iterator, List, Sequence, Tuple

import torch
from torch import nn

OFFLOAD_MODES = ("none", "models", "blocks")
_ALIGN = 256


def module_bytes(module: nn.Module) -> int:
    return sum(t.numel() * t.element_size() for t in itertools.chain(module.parameters(), module.buffers()))


def choose_offload(mode: str, dit_bytes: int, device) -> str:
    """Resolve ``auto``: ``blocks`` when ``dit_bytes`` do not fit in the free memory of ``device``."""
    if mode != "auto":
        if mode not in OFFLOAD_MODES:
            raise ValueError(f"offload must be one of {('auto',) + OFFLOAD_MODES}, got {mode!r}")
        return mode
    device = torch.device(device)
    if device.type != "cuda":
        return "none"
    free, _ = torch.cuda.mem_get_info(device)
    return "none" if dit_bytes < free else "blocks"


def _to(obj, device) -> None:
    """Move a model (an ``nn.Module`` or a wrapper with a ``to(device)`` method) to ``device``."""
    if obj is not None and hasattr(obj, "to"):
        obj.to(device)


@contextmanager
def resident(enabled: bool, device, *models) -> Iterator[None]:
    """With ``enabled``, keep ``models`` on ``device`` inside the block and on the CPU after it."""
    if not enabled:
        yield
        return
    for m in models:
        _to(m, device)
    try:
        yield
    finally:
        for m in models:
            _to(m, torch.device("cpu"))


class BlockStreamer:
    """Runs a sequence of blocks whose weights live in host memory (see the module docstring)."""

    def __init__(self, blocks: Sequence[nn.Module], device, prefetch: bool = True):
        self.device = torch.device(device)
        cuda = self.device.type == "cuda"
        self.prefetch = bool(prefetch) and cuda
        self.layouts: List[List[Tuple[torch.Tensor, int, int]]] = []
        self.host: List[torch.Tensor] = []
        largest = 0
        for blk in blocks:
            entries, off = [], 0
            for t in itertools.chain(blk.parameters(), blk.buffers()):
                n = t.numel() * t.element_size()
                entries.append((t, off, n))
                off += (n + _ALIGN - 1) // _ALIGN * _ALIGN
            host = torch.empty(max(off, _ALIGN), dtype=torch.uint8, pin_memory=self.prefetch)
            for t, o, n in entries:
                view = self._view(host, t, o, n)
                view.copy_(t.data)
                t.data = view
            self.layouts.append(entries)
            self.host.append(host)
            largest = max(largest, off)
        n_slots = 2 if self.prefetch else 1
        self.slots = [torch.empty(max(largest, _ALIGN), dtype=torch.uint8, device=self.device) for _ in range(n_slots)]
        if self.prefetch:
            self.copy_stream = torch.cuda.Stream(self.device)
            self.loaded = [torch.cuda.Event() for _ in range(n_slots)]
            self.free = [torch.cuda.Event() for _ in range(n_slots)]

    @staticmethod
    def _view(flat: torch.Tensor, t: torch.Tensor, off: int, n: int) -> torch.Tensor:
        return flat[off:off + n].view(t.dtype).view(t.shape)

    def _point(self, i: int, flat: torch.Tensor) -> None:
        for t, o, n in self.layouts[i]:
            t.data = self._view(flat, t, o, n)

    def _copy_in(self, i: int, slot: int) -> None:
        n = self.host[i].numel()
        self.slots[slot][:n].copy_(self.host[i], non_blocking=self.prefetch)

    def _prefetch(self, i: int, slot: int) -> None:
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.free[slot])  # the slot's previous block has finished
            self._copy_in(i, slot)
            self.loaded[slot].record(self.copy_stream)

    def run(self, blocks: Sequence[nn.Module], order: Iterable[int]) -> Iterator[Tuple[int, nn.Module]]:
        """Yield ``(i, blocks[i])`` for ``i`` in ``order`` with block ``i``'s tensors on the device
        while the caller runs it."""
        order = list(order)
        if not order:
            return
        compute = torch.cuda.current_stream(self.device) if self.prefetch else None
        if self.prefetch:
            self._prefetch(order[0], 0)
        for k, i in enumerate(order):
            s = k % len(self.slots)
            if self.prefetch:
                compute.wait_event(self.loaded[s])
            else:
                self._copy_in(i, s)
            self._point(i, self.slots[s])
            if self.prefetch and k + 1 < len(order):
                self._prefetch(order[k + 1], 1 - s)
            try:
                yield i, blocks[i]
            finally:
                self._point(i, self.host[i])
                if self.prefetch:
                    self.free[s].record(compute)


def enable_block_streaming(transformer: nn.Module, device, prefetch: bool = True) -> BlockStreamer:
    """Move ``transformer``'s blocks to host memory and stream them during ``predict_packed``; every
    other submodule goes to ``device``."""
    device = torch.device(device)
    for name, child in transformer.named_children():
        if name != "blocks":
            child.to(device)
    streamer = BlockStreamer(transformer.blocks, device, prefetch=prefetch)  # copies each block to host memory
    transformer.block_streamer = streamer
    return streamer


class NonBlockParts:
    """The DiT's submodules other than its blocks, moved as one (``blocks`` mode keeps the blocks
    in the streamer's host buffers)."""

    def __init__(self, transformer: nn.Module):
        self.transformer = transformer

    def to(self, device) -> "NonBlockParts":
        for name, child in self.transformer.named_children():
            if name != "blocks":
                child.to(device)
        for prm in self.transformer.parameters(recurse=False):
            prm.data = prm.data.to(device)
        for name, buf in list(self.transformer.named_buffers(recurse=False)):
            setattr(self.transformer, name, buf.to(device))
        return self
