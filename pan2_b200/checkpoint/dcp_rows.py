"""Torch distributed checkpoints (DCP) written and read as row ranges, one tensor at a time.

The reference trainer saves ``checkpoint-N/transformer`` and ``optimizer`` with ``dcp.save`` of FSDP2
state dicts (train.py:1089-1093): every parameter is a ``Shard(0)`` DTensor, so the folder holds, per
rank, the rank's rows of every tensor, and ``.metadata`` lists the chunks.  This module produces the
same on-disk format from this framework's flat units without building a state dict:

* :func:`save_row_chunks` runs ``dcp.save`` with a planner whose write items are declared from
  ``(name, global shape, first row, row count)`` and whose data are produced only when the storage
  writer asks for them (``resolve_data``), so host memory holds one tensor's rows at a time and no
  DTensor or process-group machinery is needed beyond DCP's own plan exchange;
* :func:`load_row_chunks` runs ``dcp.load`` (without collectives) with a planner that requests
  exactly the given row range of each named tensor, whatever chunking the writer used, so a
  checkpoint written by any number of ranks -- this framework's or the reference's -- loads on any
  other number.

Row ranges follow ``torch.chunk`` along dim 0 (``ceil(rows / world)`` rows per rank), the layout FSDP2's
``Shard(0)`` uses.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.api import CheckpointException
from torch.distributed.checkpoint.default_planner import DefaultLoadPlanner, DefaultSavePlanner
from torch.distributed.checkpoint.metadata import (ChunkStorageMetadata, MetadataIndex, TensorProperties,
                                                   TensorStorageMetadata)
from torch.distributed.checkpoint.planner import (LoadPlan, SavePlan, TensorWriteData, WriteItem,
                                                  WriteItemType)
from torch.distributed.checkpoint.planner_helpers import create_read_items_for_chunk_list


@dataclass
class RowChunk:
    """Rows ``[row0, row0 + rows)`` of tensor ``name`` (global ``shape``), produced on demand."""
    name: str
    shape: Sequence[int]
    row0: int
    rows: int
    dtype: torch.dtype
    produce: Callable[[], torch.Tensor]  # -> contiguous CPU tensor [rows, *shape[1:]]

    def offsets(self) -> torch.Size:
        return torch.Size([self.row0] + [0] * (len(self.shape) - 1))

    def sizes(self) -> torch.Size:
        return torch.Size([self.rows] + list(self.shape[1:]))


class _RowChunkSavePlanner(DefaultSavePlanner):
    def __init__(self, chunks: List[RowChunk]):
        super().__init__(flatten_state_dict=False, flatten_sharded_tensors=False)
        self._chunks = {c.name: c for c in chunks if c.rows > 0}

    def create_local_plan(self) -> SavePlan:
        items = []
        for c in self._chunks.values():
            items.append(WriteItem(
                index=MetadataIndex(c.name, c.offsets()), type=WriteItemType.SHARD,
                tensor_data=TensorWriteData(chunk=ChunkStorageMetadata(offsets=c.offsets(), sizes=c.sizes()),
                                            properties=TensorProperties(dtype=c.dtype), size=torch.Size(c.shape))))
        self.plan = SavePlan(items)
        return self.plan

    def resolve_data(self, write_item: WriteItem) -> torch.Tensor:
        c = self._chunks[write_item.index.fqn]
        t = c.produce()
        if tuple(t.shape) != tuple(c.sizes()) or t.dtype != c.dtype:
            raise ValueError(f"{c.name}: produced {tuple(t.shape)} {t.dtype}, declared {tuple(c.sizes())} {c.dtype}")
        return t.contiguous()


def save_row_chunks(folder: str, chunks: List[RowChunk], process_group=None, no_dist: bool = False) -> None:
    """Every rank calls this with its own chunks (ranks may own no rows of a tensor)."""
    try:
        dcp.save({}, storage_writer=dcp.FileSystemWriter(folder, thread_count=1),
                 planner=_RowChunkSavePlanner(chunks), process_group=process_group, no_dist=no_dist)
    except CheckpointException as err:
        raise RuntimeError(f"writing {folder} failed: {err}") from None


class _RowChunkLoadPlanner(DefaultLoadPlanner):
    def __init__(self, dest: Dict[str, tuple]):
        super().__init__(flatten_state_dict=False, flatten_sharded_tensors=False)
        self._dest = dest  # name -> (row0, tensor [rows, *rest])

    def set_up_planner(self, state_dict, metadata=None, is_coordinator: bool = False) -> None:
        self.state_dict, self.metadata, self.is_coordinator = state_dict, metadata, is_coordinator

    def create_local_plan(self) -> LoadPlan:
        items = []
        for name, (row0, t) in self._dest.items():
            md = self.metadata.state_dict_metadata.get(name)
            if not isinstance(md, TensorStorageMetadata):
                raise KeyError(f"{name} is not a tensor of this checkpoint")
            if t.shape[0] == 0:
                continue
            local = ChunkStorageMetadata(offsets=torch.Size([row0] + [0] * (t.dim() - 1)), sizes=t.shape)
            items += create_read_items_for_chunk_list(name, md, [local])
        return LoadPlan(items)

    def resolve_tensor(self, read_item):
        _, t = self._dest[read_item.dest_index.fqn]
        view = t
        for d, (o, n) in enumerate(zip(read_item.dest_offsets, read_item.lengths)):
            view = view.narrow(d, o, n)
        return view

    def commit_tensor(self, read_item, tensor) -> None:
        pass  # the reader copied into the view of the destination


def tensor_specs(folder: str) -> Dict[str, tuple]:
    """``name -> (shape, dtype)`` of every tensor of a DCP folder."""
    try:
        md = dcp.FileSystemReader(folder).read_metadata()
    except CheckpointException as err:
        raise RuntimeError(f"reading {folder} failed: {err}") from None
    return {k: (tuple(m.size), m.properties.dtype) for k, m in md.state_dict_metadata.items()
            if isinstance(m, TensorStorageMetadata)}


def load_row_chunks(folder: str, dest: Dict[str, tuple]) -> None:
    """Fill ``dest[name] = (row0, tensor)`` with rows ``[row0, row0 + tensor.shape[0])`` of each
    named tensor (the destination dtype may differ from the stored one; values are cast)."""
    if not dest:
        return
    same, cast = {}, {}
    specs = tensor_specs(folder)
    for name, (row0, t) in dest.items():
        if name not in specs:
            raise KeyError(f"{folder} has no tensor {name}")
        if specs[name][1] == t.dtype and t.is_contiguous():
            same[name] = (row0, t)
        else:
            cast[name] = (row0, t, torch.empty(t.shape, dtype=specs[name][1]))
    plan = dict(same)
    plan.update({n: (r0, tmp) for n, (r0, _, tmp) in cast.items()})
    try:
        dcp.load({}, storage_reader=dcp.FileSystemReader(folder), planner=_RowChunkLoadPlanner(plan), no_dist=True)
    except CheckpointException as err:  # a BaseException: turned into an ordinary, catchable error
        raise RuntimeError(f"reading {folder} failed: {err}") from None
    for _, (_, t, tmp) in cast.items():
        t.copy_(tmp)


def is_dcp_folder(folder: str) -> bool:
    import os
    return os.path.isfile(os.path.join(folder, ".metadata"))
