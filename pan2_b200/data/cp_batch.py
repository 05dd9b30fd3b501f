"""Context-parallel batch distribution: cp-rank 0 loads, the group shares, each rank keeps its shard.

Reference: dataset/cp_batch.py:46-241.  Only cp-rank 0 runs the packing loader; each step it
broadcasts the batch (host metadata as one object broadcast on the CPU group, tensors as device
broadcasts on the cp group) and every rank takes its strided shard of the joint sequence -- joint
token ``j`` lives on cp-rank ``j % cp``, the layout of :mod:`pan2_b200.parallel.ulysses`.  Within a
sample the shard is an in-order subset of its video tokens followed by an in-order subset of its
caption tokens, so the local batch is an ordinary packed batch with shorter segments:

* sharded: ``hidden_states`` columns / ``target`` rows (video tokens), RoPE tables (joint order);
* local: per-sample video / caption counts (a sample may keep zero rows of one modality), the
  concat layout and its interleave<->concat permutations;
* full (replicated): ``text_states`` and the caption segments (the caption encoder attends over
  whole captions; its output is then gathered down to this rank's rows with ``cp_text_index``),
  ``timestep`` and the joint segments (attention runs on the gathered full sequence).

The loss needs no special handling: the engine all-reduces ``(sum, count)`` over every rank.
"""
from __future__ import annotations

from dataclasses import replace
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from ..models.packed import PackedSequenceParams, build_packed_params
from ..parallel.ulysses import shard_sizes

_TENSOR_KEYS = ("hidden_states", "timestep", "text_states", "target")


def _strided_count(length: int, offset: int, cp: int) -> int:
    return -(-(length - offset) // cp) if offset < length else 0


def shard_rows(video_lens: List[int], caption_lens: List[int], cp: int, rank: int):
    """Rows of cp-rank ``rank``: ``(video rows, caption rows, local video lens, local caption lens)``,
    video / caption rows indexing the full batch's concat-order video / caption blocks."""
    n = len(video_lens)
    vcu, ccu = [0], [0]
    for a, b in zip(video_lens, caption_lens):
        vcu.append(vcu[-1] + a)
        ccu.append(ccu[-1] + b)
    jcu = [a + b for a, b in zip(vcu, ccu)]
    vrows: List[int] = []
    trows: List[int] = []
    lv, lc = [], []
    for i in range(n):
        v_off = (rank - jcu[i]) % cp
        t_off = (rank - jcu[i] - video_lens[i]) % cp
        vrows += range(vcu[i] + v_off, vcu[i + 1], cp)
        trows += range(ccu[i] + t_off, ccu[i + 1], cp)
        lv.append(_strided_count(video_lens[i], v_off, cp))
        lc.append(_strided_count(caption_lens[i], t_off, cp))
    assert sum(lv) + sum(lc) == shard_sizes(jcu[-1], cp)[rank], (lv, lc, jcu[-1], cp, rank)
    return vrows, trows, lv, lc


def local_params(P: PackedSequenceParams, cp: int, rank: int, group, device) -> Tuple[PackedSequenceParams, torch.Tensor]:
    """Local packed metadata of cp-rank ``rank`` for the full ``P``; also returns the video row index."""
    vlen, clen = list(P.video_lens), list(P.caption_lens)
    vrows, trows, lv, lc = shard_rows(vlen, clen, cp, rank)
    S = sum(vlen) + sum(clen)
    if sum(lv) == 0:
        raise ValueError(f"with cp={cp}, context-parallel rank {rank} gets no video token of the {S}-token batch; lower cp_size")
    s_local = sum(lv) + sum(lc)
    idx_v = torch.tensor(vrows, dtype=torch.long, device=device)
    idx_t = torch.tensor(trows, dtype=torch.long, device=device)
    cos = P.freqs_cos[:S][rank::cp]
    sin = P.freqs_sin[:S][rank::cp]
    local = build_packed_params(lv, lc, s_local, cos.reshape(s_local, -1), sin.reshape(s_local, -1),
                                joint_segment_limit=P.joint_segment_limit,
                                caption_segment_limit=P.caption_segment_limit).to(device, non_blocking=True)
    local = replace(local, joint_cu_seqlens=P.joint_cu_seqlens, joint_lens=list(P.joint_lens),
                    caption_cu_seqlens=P.caption_cu_seqlens, cp_caption_lens=list(clen), cp_text_index=idx_t,
                    cp_joint_total=S, cp_group=group, active_sequence_count=P.active_sequence_count)
    return local, idx_v


def strided_split(batch: Dict, cp: int, rank: int, group=None) -> Dict:
    """This cp-rank's shard of a FULL batch (``packed_seq_params`` with host lengths)."""
    dev = batch["hidden_states"].device
    local, idx_v = local_params(batch["packed_seq_params"], cp, rank, group, dev)
    return dict(hidden_states=batch["hidden_states"].index_select(1, idx_v).contiguous(),
                timestep=batch["timestep"], text_states=batch["text_states"],
                target=batch["target"].index_select(0, idx_v).contiguous(), packed_seq_params=local)


def broadcast_batch(batch: Optional[Dict], meta, cp_group, cpu_group, device) -> Tuple[Dict, object]:
    """Broadcast ``(batch, meta)`` from cp-rank 0 of ``cp_group``; the others pass ``(None, None)``.
    ``cpu_group`` is a gloo group with the same members as ``cp_group`` (host metadata).
    ``meta.dataloader_state`` stays on the source rank (only it resumes a loader)."""
    src = dist.get_global_rank(cp_group, 0)
    is_src = dist.get_rank() == src
    if is_src:
        P: PackedSequenceParams = batch["packed_seq_params"]
        host = dict(video_lens=list(P.video_lens), caption_lens=list(P.caption_lens), total=int(P.joint_packed_length),
                    jlim=P.joint_segment_limit, clim=P.caption_segment_limit,
                    specs={k: (tuple(batch[k].shape), batch[k].dtype) for k in _TENSOR_KEYS},
                    rope=(tuple(P.freqs_cos.shape),),
                    meta=replace(meta, dataloader_state=None) if meta is not None else None)
        obj = [host]
    else:
        obj = [None]
    dist.broadcast_object_list(obj, src=src, group=cpu_group)
    host = obj[0]
    if is_src:
        tensors = [batch[k].contiguous() for k in _TENSOR_KEYS]
        tensors += [P.freqs_cos.contiguous(), P.freqs_sin.contiguous()]
    else:
        tensors = [torch.empty(s, dtype=d, device=device) for s, d in (host["specs"][k] for k in _TENSOR_KEYS)]
        tensors += [torch.empty(host["rope"][0], dtype=torch.float32, device=device) for _ in range(2)]
    works = [dist.broadcast(t, src=src, group=cp_group, async_op=True) for t in tensors]
    for w in works:
        w.wait()
    if is_src:
        return batch, meta
    out = {k: t for k, t in zip(_TENSOR_KEYS, tensors)}
    P = build_packed_params(host["video_lens"], host["caption_lens"], host["total"], tensors[4].reshape(host["total"], -1),
                            tensors[5].reshape(host["total"], -1), joint_segment_limit=host["jlim"],
                            caption_segment_limit=host["clim"]).to(device)
    out["packed_seq_params"] = P
    return out, host["meta"]


def broadcast_and_split(batch: Optional[Dict], meta, layout, device) -> Tuple[Dict, object]:
    """The two steps the train loop runs per micro-batch under context parallelism."""
    batch, meta = broadcast_batch(batch, meta, layout.cp_group, layout.cp_cpu_group, device)
    return strided_split(batch, layout.cp_size, layout.cp_rank, layout.cp_group), meta
