"""Uninitialised-memory and determinism checks for the CUDA kernels (no compute-sanitizer needed).

The packed layout leaves padding rows after the last segment, and several kernels write only the
valid rows of a freshly allocated output.  A kernel that reads such a row before anything wrote it
reads whatever the caching allocator handed out.  :func:`poison_free_memory` fills the allocator's
free blocks with a byte pattern (``0xFF`` makes every bf16 / fp32 word a NaN), so a later
``torch.empty`` returns NaN-filled memory and any read of an unwritten element shows up as a NaN in
the result.  Running the same step after poisoning with ``0xFF`` and with ``0x00`` and comparing the
outputs checks that no kernel depends on memory it never wrote: the hazards the reference guards
with comments and zero-inits around its padding rows (``mlp_ops.py:88-103``, ``mlp_ops.py:136-144``)
and its Ulysses index_copy note (``ulysses.py:99-106``).

:func:`device_errors` reads and clears every device error flag of the extension (kernel-side bounds,
alignment and bounded-wait failures record a code there instead of faulting).
"""
from __future__ import annotations

from typing import Callable, Dict

import torch


def poison_free_memory(byte: int = 0xFF, device=None, headroom: int = 2 << 30, chunk: int = 4 << 30,
                       small_blocks: int = 512) -> int:
    """Fill the caching allocator's free memory on ``device`` with ``byte``; returns bytes filled.

    Large-pool memory is poisoned by allocating blocks of ``chunk`` bytes (halving the block size
    when one does not fit) until all but ``headroom`` bytes of the device's free memory are taken,
    filling them and freeing them back to the cache, so that later allocations are carved from
    poisoned blocks.  The small pool (requests up to 1 MiB, served from 2 MiB segments) is
    poisoned with ``small_blocks`` 1 MiB tensors.
    """
    dev = torch.device(device if device is not None else torch.cuda.current_device())
    torch.cuda.synchronize(dev)
    free, _ = torch.cuda.mem_get_info(dev)
    remaining = max(0, free - headroom)
    blocks, filled = [], 0
    while remaining >= (64 << 20) and chunk >= (64 << 20):
        size = min(chunk, remaining)
        try:
            t = torch.empty(size, dtype=torch.uint8, device=dev)
        except torch.cuda.OutOfMemoryError:
            chunk //= 2
            continue
        t.fill_(byte)
        blocks.append(t)
        filled += size
        remaining -= size
    smalls = [torch.empty(1 << 20, dtype=torch.uint8, device=dev) for _ in range(small_blocks)]
    for t in smalls:
        t.fill_(byte)
    filled += small_blocks << 20
    torch.cuda.synchronize(dev)
    del blocks, smalls
    return filled


def device_errors() -> int:
    """The extension's device error flag (0 when clear), cleared after reading."""
    from ..ops._ext import ext
    return int(ext().error_flag(True))


def run_poisoned(fn: Callable[[], Dict[str, torch.Tensor]], byte: int) -> Dict[str, torch.Tensor]:
    """Run ``fn`` after poisoning free device memory with ``byte``; returns host copies of its
    results.  ``fn`` must allocate its working tensors itself (inside the call)."""
    torch.cuda.empty_cache()
    poison_free_memory(byte)
    out = fn()
    torch.cuda.synchronize()
    return {k: v.detach().float().cpu() for k, v in out.items()}
