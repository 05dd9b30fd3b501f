"""Token-budget bin packing of mixed video / image items with exact resume state.

Same packing contract as the reference (dataset/packing_dataset.py:348-891): items stream from the
video CSVs (byte-offset cursor, so a resumed run continues at the next row) and the image tars,
mixed by a counter-seeded draw with ``image_sample_prob``; each item goes best-fit into one of
``num_buffers`` virtual bins under five budgets (joint tokens, video tokens, caption tokens,
text-encoder tokens, sequences); when an item fits nowhere the fullest bin is flushed into a
:class:`PackedPlan`.  :class:`DataloaderState` (JSON) records the in-flight bin contents as item
references plus the stream cursors and the draw counter.
"""
from __future__ import annotations

import csv
import glob
import io
import json
import logging
import os
import random
from concurrent.futures import ThreadPoolExecutor
from dataclasses import asdict, dataclass, field
from typing import Iterator, List, Optional, Sequence, Tuple

import torch

from .items import (Budgets, CaptionCodec, Item, ItemRef, decode_latent, draw_task, finalize_item, iter_tar_samples,
                    load_latent, read_tar_sample)
from .patching import packed_rope_tables

log = logging.getLogger("pan2_b200.data")

MIX_SALT = 0x51C3A7E1


@dataclass
class ImageCursor:
    shard_index: int = 0
    sample_index: int = 0
    cycle: int = 0


@dataclass
class DataloaderState:
    buffer_items: List[List[ItemRef]]
    next_stream_ref: Optional[ItemRef]
    image_cursor: Optional[ImageCursor] = None
    draw_count: int = 0

    def to_json(self) -> str:
        return json.dumps({
            "buffer_items": [[asdict(r) for r in b] for b in self.buffer_items],
            "next_stream_ref": asdict(self.next_stream_ref) if self.next_stream_ref else None,
            "image_cursor": asdict(self.image_cursor) if self.image_cursor else None,
            "draw_count": self.draw_count,
        })

    @classmethod
    def from_json(cls, s: str) -> "DataloaderState":
        d = json.loads(s)
        return cls(buffer_items=[[ItemRef(**r) for r in b] for b in d["buffer_items"]],
                   next_stream_ref=ItemRef(**d["next_stream_ref"]) if d.get("next_stream_ref") else None,
                   image_cursor=ImageCursor(**d["image_cursor"]) if d.get("image_cursor") else None,
                   draw_count=d.get("draw_count", 0))

    def reset_video_stream(self) -> "DataloaderState":
        """Drop the video cursor and in-flight video refs; keep images and the draw counter."""
        return DataloaderState([[r for r in b if r.modality == "image"] for b in self.buffer_items], None,
                               self.image_cursor, self.draw_count)


@dataclass
class PackedPlan:
    """CPU output of one flushed bin."""
    items: List[Item]
    video_lens: List[int]
    caption_lens: List[int]
    grids: List[Tuple[int, int, int]]
    total: int
    freqs_cos: torch.Tensor
    freqs_sin: torch.Tensor
    state: DataloaderState
    num_images: int


@dataclass
class _Bin:
    budgets: Budgets
    items: List[Item] = field(default_factory=list)
    joint: int = 0
    video: int = 0
    caption: int = 0
    text: int = 0

    def fits(self, it: Item) -> bool:
        c = it.caption.cropped_length
        b = self.budgets
        return (self.joint + it.n_video_tokens + c <= b.joint and self.text + it.caption.full_length <= b.text_encoder
                and self.video + it.n_video_tokens <= b.video and self.caption + c <= b.caption
                and len(self.items) < b.max_num_seq)

    def add(self, it: Item):
        c = it.caption.cropped_length
        self.items.append(it)
        self.joint += it.n_video_tokens + c
        self.video += it.n_video_tokens
        self.caption += c
        self.text += it.caption.full_length

    def remaining(self) -> int:
        return self.budgets.joint - self.joint

    def flush(self) -> List[Item]:
        out = self.items
        self.items = []
        self.joint = self.video = self.caption = self.text = 0
        return out


def expand_csv_paths(paths: Sequence[str]) -> List[str]:
    out = []
    for p in paths:
        if os.path.isdir(p):
            out += sorted(glob.glob(os.path.join(p, "*.csv")))
        else:
            out.append(p)
    return out


def expand_tar_paths(paths: Sequence[str]) -> List[str]:
    """Tar shards of ``paths``: folders (every ``.tar`` below them, recursively), ``.tar`` files,
    and text files listing more of either, one per line; absolute, de-duplicated and sorted
    (reference: dataset/image_item_processor.py:76-108)."""
    out = set()
    for p in paths:
        p = p.strip()
        if not p:
            continue
        if os.path.isdir(p):
            out.update(os.path.abspath(t) for t in glob.glob(os.path.join(p, "**", "*.tar"), recursive=True))
        elif p.endswith(".tar"):
            out.add(os.path.abspath(p))
        elif os.path.isfile(p):
            with open(p) as f:
                out.update(expand_tar_paths([ln.strip() for ln in f if ln.strip()]))
        else:
            raise ValueError(f"image tar path {p!r} is neither a folder, a .tar file nor a list file")
    return sorted(out)


def _read_record(f) -> bytes:
    """One CSV record from a binary file: lines are joined while a quoted field is open."""
    line = f.readline()
    while line and line.count(b'"') % 2 == 1:
        nxt = f.readline()
        if not nxt:
            break
        line += nxt
    return line


def _parse_record(raw: bytes) -> List[str]:
    return next(csv.reader([raw.decode("utf-8")]))


def read_csv_row(path: str, pos: int) -> dict:
    """The row of ``path`` whose record starts at byte ``pos``."""
    with open(path, "rb") as f:
        header = _parse_record(_read_record(f))
        f.seek(pos)
        return dict(zip(header, _parse_record(_read_record(f))))


class CsvStream:
    """Rows of a list of CSV files, each with its byte offset, cycling through the files forever
    (one pass = one epoch).  Quoted fields may span lines."""

    def __init__(self, paths: Sequence[str]):
        self.paths = list(paths)
        if not self.paths:
            raise ValueError("no video CSV files")

    def rows(self, last: Optional[ItemRef]) -> Iterator[Tuple[dict, ItemRef]]:
        """Rows after ``last`` (the last row consumed), or from the start."""
        csv_i = last.csv_index if last else 0
        epoch = last.epoch_index if last else 0
        gidx = (last.global_index + 1) if last else 0
        resume = last
        # a whole pass that starts at the first file and yields nothing means every CSV is empty:
        # fail instead of cycling through empty files forever
        full_pass, yielded = resume is None and csv_i == 0, 0
        while True:
            with open(self.paths[csv_i], "rb") as f:
                header = _parse_record(_read_record(f))
                local = 0
                if resume is not None:
                    f.seek(resume.local_file_pos)
                    _read_record(f)
                    local = resume.local_index + 1
                    resume = None
                while True:
                    pos = f.tell()
                    raw = _read_record(f)
                    if not raw:
                        break
                    if not raw.strip():
                        continue
                    row = dict(zip(header, _parse_record(raw)))
                    yield row, ItemRef(global_index=gidx, csv_index=csv_i, local_index=local, local_file_pos=pos,
                                       epoch_index=epoch)
                    gidx += 1
                    local += 1
                    yielded += 1
            csv_i += 1
            if csv_i == len(self.paths):
                if full_pass and yielded == 0:
                    raise ValueError(f"the video CSVs ({len(self.paths)} file(s)) contain no rows")
                csv_i = 0
                epoch += 1
                full_pass, yielded = True, 0


class PackingDataset:
    """Iterator of :class:`PackedPlan` objects."""

    def __init__(self, csv_paths: Sequence[str], codec: CaptionCodec, budgets: Budgets, *, patch_size=(1, 2, 2),
                 rope_axes=(16, 56, 56), rope_theta: float = 256.0, rope_scale=(16 / 24, 1.0, 1.0),
                 num_buffers: int = 4, seed: int = 0, image_tars: Sequence[str] = (), image_sample_prob: float = 0.0,
                 video_cond_prob: float = 0.0, image_cond_prob: float = 0.3, cfg_drop_prob: float = 0.1,
                 num_workers: int = 4, resume: Optional[DataloaderState] = None, pad_multiple: int = 128):
        self.stream = CsvStream(expand_csv_paths(csv_paths)) if csv_paths else None
        self.tars = expand_tar_paths(image_tars)
        self.codec, self.budgets = codec, budgets
        self.patch_size, self.rope_axes, self.rope_theta, self.rope_scale = tuple(patch_size), rope_axes, rope_theta, rope_scale
        self.num_buffers, self.seed = num_buffers, seed
        self.image_sample_prob = image_sample_prob if self.tars else 0.0
        self.video_cond_prob, self.image_cond_prob, self.cfg_drop_prob = video_cond_prob, image_cond_prob, cfg_drop_prob
        self.num_workers = max(1, num_workers)
        self.resume = resume
        self.pad_multiple = pad_multiple

    # ------------------------------------------------------------------ item production
    def _video_item(self, row_ref) -> Optional[Item]:
        row, ref = row_ref
        path = (row.get("latent_path") or "").strip()
        text = row.get("caption")
        if not path or not isinstance(text, str) or not text.strip():
            return None
        # lone UTF-16 surrogates (broken emoji from data preparation) cannot be encoded as UTF-8
        # and would fail the tokenizer: drop them
        text = text.encode("utf-8", "ignore").decode("utf-8")
        try:
            lat = load_latent(path)
        except Exception as e:  # a missing or unreadable latent skips the row, as in the reference
            log.warning(f"skipping row {ref.local_index} of csv[{ref.csv_index}]: cannot load {path!r}: {e}")
            return None
        prefix, drop = draw_task(self.seed, ref, int(lat.shape[1]), self.video_cond_prob, self.image_cond_prob,
                                 self.cfg_drop_prob)
        return finalize_item(lat, text, ref, prefix_frames=prefix, drop_caption=drop, codec=self.codec,
                             budgets=self.budgets, patch_size=self.patch_size, modality="video")

    def _image_stream(self, cur: ImageCursor):
        shard, sample, cycle = cur.shard_index % len(self.tars), cur.sample_index, cur.cycle
        # shards read from their first sample in a row that yielded nothing; once that covers every
        # tar, all of them are empty: fail instead of cycling through empty tars forever
        empty_run = 0
        while True:
            yielded = 0
            for idx, key, raw, text, members in iter_tar_samples(self.tars[shard], start=sample):
                yielded += 1
                ref = ItemRef(global_index=-1, modality="image", shard_index=shard, sample_index=idx, cycle=cycle,
                              tar_members=members)
                yield raw, text, ref, ImageCursor(shard, idx + 1, cycle)
            empty_run = empty_run + 1 if (yielded == 0 and sample == 0) else 0
            if empty_run == len(self.tars):
                raise ValueError(f"the image tars ({len(self.tars)} file(s)) contain no complete samples")
            shard, sample = shard + 1, 0
            if shard == len(self.tars):
                shard, cycle = 0, cycle + 1

    def _image_item(self, raw, text, ref) -> Optional[Item]:
        try:
            lat = decode_latent(raw)
        except Exception:
            return None
        drop = random.Random(hash((self.seed, ref.shard_index, ref.sample_index, ref.cycle))).random() < self.cfg_drop_prob
        return finalize_item(lat, text, ref, prefix_frames=0, drop_caption=drop, codec=self.codec,
                             budgets=self.budgets, patch_size=self.patch_size, modality="image")

    def _mixed(self) -> Iterator[Tuple[Optional[Item], ItemRef, Optional[ImageCursor], int]]:
        if self.stream is None and not self.tars:
            raise ValueError("no video CSVs and no image tars")
        st = self.resume
        video_rows = self.stream.rows(st.next_stream_ref if st else None) if self.stream else None
        img_cur = (st.image_cursor if st and st.image_cursor else ImageCursor())
        images = self._image_stream(img_cur) if self.tars else None
        draws = st.draw_count if st else 0
        last_video_ref = st.next_stream_ref if st else None
        pool = ThreadPoolExecutor(self.num_workers)
        try:
            pending = []
            while True:
                rng = random.Random(hash((self.seed, MIX_SALT, draws)))
                draws += 1
                use_image = images is not None and (video_rows is None or rng.random() < self.image_sample_prob)
                if use_image:
                    raw, text, ref, img_cur = next(images)
                    fut = pool.submit(self._image_item, raw, text, ref)
                else:
                    row_ref = next(video_rows)
                    last_video_ref = row_ref[1]
                    fut = pool.submit(self._video_item, row_ref)
                pending.append((fut, last_video_ref, img_cur, draws))
                if len(pending) >= 2 * self.num_workers:
                    f, vref, icur, dc = pending.pop(0)
                    yield f.result(), vref, icur, dc
        finally:
            pool.shutdown(wait=False, cancel_futures=True)

    # ------------------------------------------------------------------ packing
    def _plan(self, items: List[Item], state: DataloaderState) -> PackedPlan:
        vlen = [it.n_video_tokens for it in items]
        clen = [it.caption.cropped_length for it in items]
        grids = [it.grid for it in items]
        n_active = sum(vlen) + sum(clen)
        total = (n_active + self.pad_multiple - 1) // self.pad_multiple * self.pad_multiple
        cos, sin = packed_rope_tables(self.rope_axes, self.rope_theta, self.rope_scale, grids, clen, total)
        return PackedPlan(items, vlen, clen, grids, total, cos, sin, state,
                          sum(1 for it in items if it.modality == "image"))

    def _restore_bins(self, bins: List[_Bin]):
        st = self.resume
        if not st:
            return
        for b, refs in zip(bins, st.buffer_items):
            for ref in refs:
                it = None
                if ref.modality == "video" and self.stream:
                    row = read_csv_row(self.stream.paths[ref.csv_index], ref.local_file_pos)
                    it = self._video_item((row, ref))
                elif ref.modality == "image" and self.tars:
                    tar = self.tars[ref.shard_index % len(self.tars)]
                    if ref.tar_members is not None:  # byte ranges recorded: no scan of the tar
                        it = self._image_item(*read_tar_sample(tar, ref.tar_members), ref)
                    else:
                        for idx, key, raw, text, _ in iter_tar_samples(tar, start=ref.sample_index):
                            it = self._image_item(raw, text, ref)
                            break
                if it is not None and b.fits(it):  # items that no longer fit are dropped
                    b.add(it)

    def __iter__(self) -> Iterator[PackedPlan]:
        bins = [_Bin(self.budgets) for _ in range(self.num_buffers)]
        self._restore_bins(bins)
        for item, vref, icur, draws in self._mixed():
            if item is None:
                continue
            flushed = []
            while True:
                cands = [b for b in bins if b.fits(item)]
                if cands:
                    min(cands, key=lambda b: b.remaining()).add(item)
                    break
                full = max(bins, key=lambda b: b.joint)
                if not full.items:
                    break  # fits no empty bin either; unreachable after the item-level budget checks
                flushed.append(full.flush())
            for out in flushed:
                # the state names everything still in flight, the item just placed included
                state = DataloaderState([[it.ref for it in b.items] for b in bins], vref, icur, draws)
                yield self._plan(out, state)
