"""Checkpoints of the flat-unit engine: torch distributed checkpoint (DCP) folders, streamed per tensor,
resharded on load.

Directory layout of ``checkpoint-<step>/`` (the reference's, train.py:455-458 and 1060-1151):

* ``transformer/`` -- a DCP folder (``.metadata`` + one ``__<rank>_0.distcp`` per rank) holding every
  parameter under its model name as fp32, each rank writing the ``Shard(0)`` rows it owns
  (``ceil(rows / W)`` rows per rank, FSDP2's rule).  The reference's converter and loaders read it
  as they read the reference trainer's own ``transformer/`` folder;
* ``optimizer/`` -- a DCP folder with the same rows of ``state.<name>.momentum_buffer`` (Muon) or
  ``state.<name>.exp_avg`` / ``state.<name>.exp_avg_sq`` (AdamW), plus ``pan2_state.json`` (step
  count, optimizer choice);
* ``training_state.pt`` -- ``{"lr_schedulers": {name: state}, "global_step": N}``;
* ``dataloader/<dp_rank>.json`` -- the packing loader's cursor;
* ``COMPLETE`` -- written by rank 0 after every rank finished; a folder without it is unreadable and
  resume falls back to the previous checkpoint (train.py:1256-1279).

Saving declares each tensor's rows to DCP and produces them only when the writer asks for them
(:mod:`pan2_b200.checkpoint.dcp_rows`), so a rank holds one tensor's host copy at a time and there is
no gather.  Loading requests, per unit, exactly the rows the loading rank owns, so a checkpoint loads
on any world size.  Folders of the earlier per-rank safetensors format (``meta.json`` beside
``<unit>.rank<r>-of-<W>.safetensors``) still load.  :func:`consolidate` writes a plain state dict
(5 GB safetensors shards + index).
"""
from __future__ import annotations

import glob
import json
import os
import re
import shutil
from typing import Callable, Dict, Iterable, List, Optional, Tuple

import torch
import torch.distributed as dist

FORMAT = "pan2_b200-sharded-v1"
COMPLETE = "COMPLETE"


def checkpoint_layout(root: str) -> Tuple[str, str, str]:
    return os.path.join(root, "transformer"), os.path.join(root, "optimizer"), os.path.join(root, "training_state.pt")


def _fname(unit: str, rank: int, world: int) -> str:
    return f"{unit}.rank{rank:05d}-of-{world:05d}.safetensors"


def rows_owned(rows: int, world: int, rank: int) -> Tuple[int, int]:
    per = -(-rows // world)
    a = min(rows, rank * per)
    return a, min(rows, a + per)


def _slot_rows(x: torch.Tensor, s, k: int) -> torch.Tensor:
    return x[s.shard_off:s.shard_off + k * s.cols].view(k, s.cols)


def _opt_names(engine, s) -> List[Tuple[str, str]]:
    if engine._is_muon(s):
        return [("mom", "momentum_buffer")]
    return [("m", "exp_avg"), ("v", "exp_avg_sq")]


def _state_rows(engine, u, s, key: str, k: int) -> torch.Tensor:
    buf = u.state[key]
    off = engine._soff[id(s)]
    return buf[off:off + k * s.cols].view(k, s.cols)


def _barrier(group):
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.barrier(group=group)


def _slot_producer(u, s, k: int, which: str, key: Optional[str] = None, engine=None):
    """Producer of rows ``[0, k)`` of slot ``s`` (this rank's rows) as a CPU fp32 tensor shaped like
    the parameter: the joined fp32 master (``which == "w"``) or optimizer state ``key``."""
    from ..optim.flat_ops import join_master
    rest = tuple(s.shape[1:]) if len(s.shape) > 1 else ()

    def produce():
        n = k * s.cols
        if which == "w":
            x = join_master(u.hi[s.shard_off:s.shard_off + n], u.lo[s.shard_off:s.shard_off + n])
        else:
            x = _state_rows(engine, u, s, key, k).reshape(-1).float()
        return x.cpu().reshape((k,) + rest)
    return produce


def save_engine(engine, root: str, *, group=None, save_optimizer: bool = True) -> None:
    """Every rank calls this (collectively over ``group``, default: the default process group).
    Writes ``transformer/`` (and ``optimizer/``) of ``root`` as DCP folders."""
    from .dcp_rows import RowChunk, save_row_chunks
    model_dir, optim_dir, _ = checkpoint_layout(root)
    world, rank = engine.world, engine.rank
    if hasattr(engine, "flush_updates"):
        engine.flush_updates()
    if engine.device.type == "cuda":
        torch.cuda.synchronize(engine.device)
    no_dist = not (dist.is_initialized() and dist.get_world_size(group) > 1)
    weights, states = [], []
    for u in engine.sharded.units:
        for s in u.slots:
            a, b = rows_owned(s.rows, world, rank)
            shape = tuple(s.shape) if len(s.shape) > 0 else (s.rows,)
            weights.append(RowChunk(s.name, shape, a, b - a, torch.float32, _slot_producer(u, s, b - a, "w")))
            if save_optimizer:
                for key, label in _opt_names(engine, s):
                    states.append(RowChunk(f"state.{s.name}.{label}", shape, a, b - a, torch.float32,
                                           _slot_producer(u, s, b - a, "state", key, engine)))
    save_row_chunks(model_dir, weights, process_group=group, no_dist=no_dist)
    if save_optimizer:
        save_row_chunks(optim_dir, states, process_group=group, no_dist=no_dist)
        if rank == 0:
            with open(os.path.join(optim_dir, "pan2_state.json"), "w") as f:
                json.dump({"step": engine.step_count, "use_muon": engine.optim.use_muon}, f)


class ShardedReader:
    """Row-range reads of one saved folder (``transformer/`` or ``optimizer/``)."""

    def __init__(self, folder: str, meta_folder: Optional[str] = None):
        meta_path = os.path.join(meta_folder or folder, "meta.json")
        with open(meta_path) as f:
            meta = json.load(f)
        if meta.get("format") != FORMAT:
            raise ValueError(f"{meta_path}: unknown checkpoint format {meta.get('format')!r}")
        self.folder = folder
        self.world = int(meta["world_size"])
        self.where: Dict[str, Tuple[str, int, int]] = {}   # param name -> (unit, rows, cols)
        for u in meta["units"]:
            for p in u["params"]:
                self.where[p["name"]] = (u["name"], int(p["rows"]), int(p["cols"]))
        self._open: Dict[str, object] = {}

    def _handle(self, unit: str, q: int):
        from safetensors import safe_open
        fn = os.path.join(self.folder, _fname(unit, q, self.world))
        h = self._open.get(fn)
        if h is None:
            if not os.path.exists(fn):
                raise FileNotFoundError(fn)
            h = safe_open(fn, framework="pt", device="cpu")
            self._open[fn] = h
        return h

    def has(self, param: str) -> bool:
        return param in self.where

    def read_rows(self, param: str, a: int, b: int, suffix: str = "") -> torch.Tensor:
        """Rows ``[a, b)`` of ``param`` (+``suffix`` for optimizer entries) as fp32 ``[b-a, cols]``."""
        unit, rows, cols = self.where[param]
        out = torch.empty(max(0, b - a), cols, dtype=torch.float32)
        per = -(-rows // self.world)
        r = a
        while r < b:
            q = r // per
            qa, qb = rows_owned(rows, self.world, q)
            hi = min(b, qb)
            t = self._handle(unit, q).get_slice(param + suffix)[r - qa:hi - qa]
            out[r - a:hi - a] = t.float()
            r = hi
        return out

    def full(self, param: str, suffix: str = "") -> torch.Tensor:
        unit, rows, cols = self.where[param]
        return self.read_rows(param, 0, rows, suffix)


def load_engine(engine, root: str, *, load_optimizer: bool = True, strict: bool = True) -> List[str]:
    """Load ``root``'s transformer (and optimizer) rows this rank owns; works across world sizes.
    Returns parameter names absent from the checkpoint (raises when ``strict``)."""
    from .dcp_rows import is_dcp_folder
    model_dir, optim_dir, _ = checkpoint_layout(root)
    if hasattr(engine, "flush_updates"):
        engine.flush_updates()
    if engine.device.type == "cuda":
        torch.cuda.synchronize(engine.device)
    if load_optimizer and not os.path.isdir(optim_dir):
        raise ValueError(f"no optimizer state found under {root}")
    if is_dcp_folder(model_dir):
        missing = _load_dcp(engine, model_dir, optim_dir if load_optimizer else None)
    else:
        missing = _load_safetensors_shards(engine, model_dir, optim_dir if load_optimizer else None)
    if strict and missing:
        raise ValueError(f"{len(missing)} transformer tensors absent from {model_dir} (first: {missing[:5]})")
    return missing


def _load_dcp(engine, model_dir: str, optim_dir: Optional[str]) -> List[str]:
    from .dcp_rows import load_row_chunks, tensor_specs
    from ..parallel.sharded import set_master
    from ..optim.flat_ops import join_master
    world, rank = engine.world, engine.rank
    have_w = tensor_specs(model_dir)
    have_o = tensor_specs(optim_dir) if optim_dir is not None else {}
    missing = []
    for u in engine.sharded.units:
        x = join_master(u.hi, u.lo).cpu().clone()
        want_w, want_o = {}, {}
        for s in u.slots:
            if s.name not in have_w:
                missing.append(s.name)
                continue
            a, b = rows_owned(s.rows, world, rank)
            want_w[s.name] = (a, torch.empty((b - a,) + tuple(have_w[s.name][0][1:]), dtype=torch.float32))
            if optim_dir is not None:
                for key, label in _opt_names(engine, s):
                    name = f"state.{s.name}.{label}"
                    if name in have_o:
                        want_o[name] = (a, torch.empty((b - a,) + tuple(have_o[name][0][1:]), dtype=torch.float32))
        load_row_chunks(model_dir, want_w)
        load_row_chunks(optim_dir, want_o) if optim_dir is not None else None
        for s in u.slots:
            if s.name not in want_w:
                continue
            a, rows = want_w[s.name]
            _slot_rows(x, s, rows.shape[0]).copy_(rows.reshape(rows.shape[0], -1))
            for key, label in (_opt_names(engine, s) if optim_dir is not None else ()):
                got = want_o.get(f"state.{s.name}.{label}")
                if got is not None:
                    dst = _state_rows(engine, u, s, key, got[1].shape[0])
                    dst.copy_(got[1].reshape(dst.shape).to(dst.device, dst.dtype))
        set_master(u, x.to(engine.device))
        if world == 1:
            engine.sharded.bind_weights(u, u.hi)
    if optim_dir is not None:
        meta_path = os.path.join(optim_dir, "pan2_state.json")
        if os.path.exists(meta_path):
            with open(meta_path) as f:
                engine.step_count = int(json.load(f).get("step", engine.step_count))
    return missing


def _load_safetensors_shards(engine, model_dir: str, optim_dir: Optional[str]) -> List[str]:
    """The earlier per-rank safetensors format (``meta.json`` + ``<unit>.rank<r>-of-<W>``)."""
    from ..parallel.sharded import set_master
    from ..optim.flat_ops import join_master
    wr = ShardedReader(model_dir)
    orr, ometa = None, {}
    if optim_dir is not None:
        orr = ShardedReader(optim_dir, meta_folder=model_dir)
        with open(os.path.join(optim_dir, "meta.json")) as f:
            ometa = json.load(f)
    world, rank = engine.world, engine.rank
    missing = []
    for u in engine.sharded.units:
        x = join_master(u.hi, u.lo).cpu().clone()
        for s in u.slots:
            if not wr.has(s.name):
                missing.append(s.name)
                continue
            a, b = rows_owned(s.rows, world, rank)
            _slot_rows(x, s, b - a).copy_(wr.read_rows(s.name, a, b))
            if orr is not None:
                for key, label in _opt_names(engine, s):
                    dst = _state_rows(engine, u, s, key, b - a)
                    dst.copy_(orr.read_rows(s.name, a, b, "." + label).to(dst.device, dst.dtype))
        set_master(u, x.to(engine.device))
        if world == 1:
            engine.sharded.bind_weights(u, u.hi)
    if orr is not None:
        engine.step_count = int(ometa.get("step", engine.step_count))
    return missing


# ------------------------------------------------------------------ plain state dicts
def strip_wrapper_prefix(name: str) -> str:
    """Parameter name without the ``module.`` / ``model.`` prefixes that DDP / FSDP wrappers and
    trainer state dicts add (the reference's loaders strip the same two)."""
    for pre in ("module.", "model."):
        if name.startswith(pre):
            name = name[len(pre):]
    return name


class LazyStateDict:
    """Read-on-demand view of a plain state dict: safetensors shards (a folder, an index json or one
    file), a ``.pt``/``.bin`` file, a torch distributed checkpoint (DCP) folder -- the reference
    trainer's ``checkpoint-N/transformer`` -- or this framework's sharded checkpoint folder.
    ``get(name)`` loads one tensor.  Names are reported without ``module.`` / ``model.`` prefixes
    unless ``key_map`` says otherwise."""

    def __init__(self, path: str, key_map: Optional[Callable[[str], str]] = None):
        self.key_map = key_map or strip_wrapper_prefix
        path = str(path)
        self._files: Dict[str, str] = {}
        self._eager: Optional[Dict[str, torch.Tensor]] = None
        self._sharded: Optional[ShardedReader] = None
        self._dcp = None
        p = os.path.normpath(path)
        if os.path.isdir(p) and os.path.exists(os.path.join(p, "transformer", "meta.json")):
            p = os.path.join(p, "transformer")
        if os.path.isdir(p) and os.path.exists(os.path.join(p, "meta.json")):
            self._sharded = ShardedReader(p)
            self._names = {self.key_map(k): k for k in self._sharded.where}
            return
        if os.path.isdir(p) and not os.path.exists(os.path.join(p, ".metadata")) and \
                os.path.exists(os.path.join(p, "transformer", ".metadata")):
            p = os.path.join(p, "transformer")
        if os.path.isdir(p) and os.path.exists(os.path.join(p, ".metadata")):
            import torch.distributed.checkpoint as dcp
            from torch.distributed.checkpoint.metadata import TensorStorageMetadata
            reader = dcp.FileSystemReader(p)
            meta = reader.read_metadata()
            self._dcp = (p, {k: (tuple(m.size), m.properties.dtype) for k, m in meta.state_dict_metadata.items()
                             if isinstance(m, TensorStorageMetadata)})
            self._names = {self.key_map(k): k for k in self._dcp[1]}
            return
        files = []
        if os.path.isdir(p):
            files = sorted(glob.glob(os.path.join(p, "*.safetensors")))
            if not files:
                pts = sorted(glob.glob(os.path.join(p, "*.pt")) + glob.glob(os.path.join(p, "*.bin")))
                if pts:
                    p = pts[0]
        elif p.endswith(".json"):
            with open(p) as f:
                idx = json.load(f)["weight_map"]
            files = sorted({os.path.join(os.path.dirname(p), v) for v in idx.values()})
        elif p.endswith(".safetensors"):
            files = [p]
        if files:
            from safetensors import safe_open
            for fn in files:
                with safe_open(fn, framework="pt", device="cpu") as h:
                    for k in h.keys():
                        self._files[k] = fn
            self._names = {self.key_map(k): k for k in self._files}
        else:
            sd = torch.load(p, map_location="cpu", weights_only=True)
            for wrapper in ("state_dict", "model"):
                if isinstance(sd, dict) and isinstance(sd.get(wrapper), dict):
                    sd = sd[wrapper]
            self._eager = {k: v for k, v in sd.items() if isinstance(v, torch.Tensor)}
            self._names = {self.key_map(k): k for k in self._eager}

    def keys(self) -> Iterable[str]:
        return self._names.keys()

    def __contains__(self, name: str) -> bool:
        return name in self._names

    def get(self, name: str, default=None):
        raw = self._names.get(name)
        if raw is None:
            return default
        if self._sharded is not None:
            return self._sharded.full(raw)
        if self._dcp is not None:
            import torch.distributed.checkpoint as dcp
            folder, specs = self._dcp
            size, dtype = specs[raw]
            out = {raw: torch.empty(size, dtype=dtype)}
            dcp.load(out, storage_reader=dcp.FileSystemReader(folder), no_dist=True)
            return out[raw]
        if self._eager is not None:
            return self._eager[raw]
        from safetensors import safe_open
        with safe_open(self._files[raw], framework="pt", device="cpu") as h:
            return h.get_tensor(raw)


def consolidate(src: str, out_dir: str, dtype=torch.bfloat16, max_shard_bytes: int = 5 * 1024 ** 3,
                prefix: str = "diffusion_pytorch_model") -> List[str]:
    """Write a sharded checkpoint (``checkpoint-N`` or its ``transformer/``) as plain safetensors
    shards plus ``<prefix>.safetensors.index.json``; returns the shard paths."""
    from safetensors.torch import save_file
    sd = LazyStateDict(src)
    os.makedirs(out_dir, exist_ok=True)
    names = sorted(sd.keys())
    groups, cur, size = [], [], 0
    esize = torch.empty(0, dtype=dtype).element_size()
    for n in names:
        _, rows, cols = sd._sharded.where[n] if sd._sharded is not None else (None, 0, 0)
        nbytes = rows * cols * esize if sd._sharded is not None else sd.get(n).numel() * esize
        if cur and size + nbytes > max_shard_bytes:
            groups.append(cur)
            cur, size = [], 0
        cur.append(n)
        size += nbytes
    if cur:
        groups.append(cur)
    shapes = {}
    if sd._sharded is not None:
        with open(os.path.join(sd._sharded.folder, "meta.json")) as f:
            for u in json.load(f)["units"]:
                for p in u["params"]:
                    shapes[p["name"]] = tuple(p["shape"])
    paths, weight_map, total = [], {}, 0
    for i, grp in enumerate(groups):
        fn = f"{prefix}-{i + 1:05d}-of-{len(groups):05d}.safetensors"
        tensors = {}
        for n in grp:
            t = sd.get(n)
            if n in shapes:
                t = t.reshape(shapes[n])
            tensors[n] = t.to(dtype).contiguous()
            total += tensors[n].numel() * esize
            weight_map[n] = fn
        save_file(tensors, os.path.join(out_dir, fn), metadata={"format": "pt"})
        paths.append(os.path.join(out_dir, fn))
    with open(os.path.join(out_dir, f"{prefix}.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)
    return paths


def load_plain_into_engine(engine, path: str, strict: bool = True) -> List[str]:
    """Warm start from a plain state dict (any :class:`LazyStateDict` source), one unit at a time.
    Legacy per-modality block keys are converted per block (``convert_legacy_block_keys``)."""
    from .keys import convert_legacy_block_keys
    from ..parallel.sharded import set_master
    from ..optim.flat_ops import join_master
    sd = LazyStateDict(path)
    all_keys = list(sd.keys())
    tmtd = bool(engine.arch.get("text_modulation_timestep_dependent", False))
    missing = []
    world, rank = engine.world, engine.rank
    if hasattr(engine, "flush_updates"):
        engine.flush_updates()
    if engine.device.type == "cuda":
        torch.cuda.synchronize(engine.device)
    for u in engine.sharded.units:
        if u.name.startswith("blocks."):
            pre = u.name + "."
            local = {k: sd.get(k) for k in all_keys if k.startswith(pre)}
            lw = next((s for s in u.slots if s.name == pre + "text_modulation.linear.weight"), None)
            convert_legacy_block_keys(local, pre, tmtd, torch.Size(lw.shape) if lw is not None else None)
            getter = local.get
        else:
            getter = sd.get
        x = join_master(u.hi, u.lo).cpu().clone()
        for s in u.slots:
            t = getter(s.name)
            if t is None:
                missing.append(s.name)
                continue
            a, b = rows_owned(s.rows, world, rank)
            _slot_rows(x, s, b - a).copy_(t.reshape(s.rows, s.cols)[a:b].float())
        set_master(u, x.to(engine.device))
        if world == 1:
            engine.sharded.bind_weights(u, u.hi)
    if strict and missing:
        raise ValueError(f"{len(missing)} transformer tensors absent from {path} (first: {missing[:5]})")
    return missing


# ------------------------------------------------------------------ folders
_CKPT_RE = re.compile(r"checkpoint-(\d+)$")


def list_checkpoints(output_dir: str) -> List[Tuple[int, str]]:
    if not os.path.isdir(output_dir):
        return []
    out = []
    for d in os.listdir(output_dir):
        m = _CKPT_RE.match(d)
        if m:
            out.append((int(m.group(1)), os.path.join(output_dir, d)))
    return sorted(out)


def is_complete(root: str) -> bool:
    return os.path.exists(os.path.join(root, COMPLETE))


def mark_complete(root: str, step: int) -> None:
    with open(os.path.join(root, COMPLETE), "w") as f:
        f.write(f"{step}\n")


def clear_complete(root: str) -> None:
    """Drop the marker before a folder is rewritten, so an interrupted rewrite reads as incomplete."""
    try:
        os.remove(os.path.join(root, COMPLETE))
    except FileNotFoundError:
        pass


def cleanup_old(output_dir: str, keep: int) -> List[str]:
    """Keep the ``keep`` most recent complete checkpoints; returns the removed folders.

    Only complete checkpoints count toward ``keep``.  Incomplete folders older than the newest
    complete one (left by interrupted saves) are removed too; incomplete folders newer than it (an
    interrupted save of a run that was rolled back to an earlier step) are left in place, since a
    resumed run skips them and rewrites them when it reaches their step again."""
    if keep <= 0:
        return []
    ck = list_checkpoints(output_dir)
    complete = [(s, d) for s, d in ck if is_complete(d)]
    if not complete:
        return []
    kept = {d for _, d in complete[-keep:]}
    newest = complete[-1][0]
    removed = []
    for s, d in ck:
        if d in kept or s > newest:
            continue
        shutil.rmtree(d, ignore_errors=True)
        removed.append(d)
    return removed


def main(argv=None) -> None:
    """``python -m pan2_b200.checkpoint.io consolidate --input checkpoint-N --output DIR [--dtype]``:
    write a checkpoint (any form :class:`LazyStateDict` reads) as one plain safetensors state dict."""
    import argparse
    ap = argparse.ArgumentParser(description="Checkpoint tools")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("consolidate", help="sharded / distributed checkpoint -> plain safetensors shards + index")
    c.add_argument("--input", required=True, help="checkpoint-N, its transformer/ folder, or any state dict")
    c.add_argument("--output", required=True)
    c.add_argument("--dtype", default="bf16", choices=("bf16", "fp32"))
    c.add_argument("--max_shard_gb", type=float, default=5.0)
    args = ap.parse_args(argv)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    paths = consolidate(args.input, args.output, dtype=dtype, max_shard_bytes=int(args.max_shard_gb * 1024 ** 3))
    print(f"wrote {len(paths)} shard(s) to {args.output}")


if __name__ == "__main__":
    main()
