"""Prompt files for generation: entry parsing, frame counts, negative prompts and resume checks.

Accepts the reference's prompt-file format and follows its rules (inference/inputs.py:1-189 of the
reference), implemented here as a per-entry reader:

* the file is a JSON list of entries, or an object holding that list under exactly one of
  ``entries`` / ``prompts`` / ``data``;
* an entry's task is its ``task`` / ``type`` field, else ``i2v`` when it names a reference image
  (``image_path`` / ``image`` / ``ref_image``), else ``t2v``; its prompt is the first non-empty of
  ``refined_prompt``, ``refined_prompts``, ``prompt``, ``caption``;
* frames: ``4 * ceil(duration_sec * fps / 4) + 1`` (frame counts the Wan VAE encodes), else
  ``frames`` / ``num_target_frames``, else the fallback; computed in exact rational arithmetic;
* output: ``<task>_<sanitised id>.mp4``, else ``relative_path``, else ``<task>_<index>.mp4``; paths
  that leave the output folder or repeat are errors; with task ``auto`` each task gets a subfolder;
* a negative prompt that is a JSON object has every ``time_range_sec`` set to the clip's span;
* :func:`is_complete` lets a run skip an output only when the video and its ``_config.json`` exist
  and every generation argument matches; a finished output with other settings is an error.
"""
from __future__ import annotations

import json
import math
import re
from fractions import Fraction
from pathlib import Path, PurePosixPath
from typing import Dict, List, Optional

GUIDANCE_KEYS = ("cfg_start_step", "cfg_end_step", "stg_scale", "stg_skip_layers")
# arguments that only choose where an output goes; every other argument must match to resume
ROUTING_ARGS = frozenset({"prompt_json", "output_dir", "prompt_shard_index", "prompt_shard_count",
                          "skip_existing", "output_path", "task", "image_root"})
TASKS = ("t2v", "i2v")
IMAGE_KEYS = ("image_path", "image", "ref_image")
PROMPT_KEYS = ("refined_prompt", "refined_prompts", "prompt", "caption")
NEGATIVE_KEYS = ("negative_prompt", "negative_prompts", "neg_prompt")
WRAPPER_KEYS = ("entries", "prompts", "data")


def _exact_positive(value, what: str, whole: bool = False) -> Fraction:
    """``value`` as an exact positive rational (a whole number when ``whole``)."""
    problem = f"{what} must be a positive finite {'integer' if whole else 'number'}, got {value!r}"
    if isinstance(value, bool):
        raise ValueError(problem)
    try:
        q = Fraction(str(value).strip())
    except (ValueError, ZeroDivisionError):
        raise ValueError(problem) from None
    if q <= 0 or (whole and q.denominator != 1):
        raise ValueError(problem)
    return q


def resolve_frames(entry: Dict, fps=24, fallback=121) -> int:
    rate = _exact_positive(fps, "fps")
    default = _exact_positive(fallback, "video_length", whole=True)
    if entry.get("duration_sec") is not None:
        seconds = _exact_positive(entry["duration_sec"], "duration_sec")
        return 4 * math.ceil(seconds * rate / 4) + 1
    for key in ("frames", "num_target_frames"):
        if entry.get(key) is not None:
            return int(_exact_positive(entry[key], key, whole=True))
    return int(default)


def _stamp_time_ranges(node, span: str):
    if isinstance(node, list):
        return [_stamp_time_ranges(v, span) for v in node]
    if isinstance(node, dict):
        return {k: span if k == "time_range_sec" else _stamp_time_ranges(v, span) for k, v in node.items()}
    return node


def render_negative_duration(text, video_length: int, fps=24):
    """A structured (JSON object) negative prompt with its time ranges set to this clip's duration;
    any other text unchanged."""
    try:
        parsed = json.loads(text)
    except (TypeError, json.JSONDecodeError):
        return text
    if not isinstance(parsed, dict):
        return text
    span = "0 to " + format((int(video_length) - 1) / float(fps), "g")
    return json.dumps(_stamp_time_ranges(parsed, span), ensure_ascii=False, separators=(",", ":"))


def _entry_list(payload) -> list:
    if isinstance(payload, dict):
        present = [k for k in WRAPPER_KEYS if k in payload]
        if len(present) != 1:
            raise ValueError(f"a prompt-file object must hold its entries under exactly one of {WRAPPER_KEYS}; "
                             f"found {present}")
        payload = payload[present[0]]
    if not isinstance(payload, list):
        raise ValueError("a prompt file holds a list of entries")
    return payload


def _single_alias(entry: Dict, keys, what: str, truthy: bool = True) -> Optional[str]:
    """The one alias of ``keys`` the entry uses (all present aliases must agree)."""
    used = [k for k in keys if (entry.get(k) if truthy else k in entry)]
    if len({json.dumps(entry[k], sort_keys=True) for k in used}) > 1:
        raise ValueError(f"entry gives different values for the {what} aliases {used}")
    return used[0] if used else None


class _EntryReader:
    """Turns one prompt-file entry into a generation record."""

    def __init__(self, entry, index: int, out_root: Path, mode: str, image_root: Optional[Path],
                 check_images: bool):
        if not isinstance(entry, dict):
            raise ValueError(f"prompt entry {index} is not a JSON object")
        self.entry, self.index, self.out_root, self.mode = entry, index, out_root, mode
        self.image_root, self.check_images = image_root, check_images

    def task(self) -> str:
        named = {str(self.entry[k]).strip().lower() for k in ("task", "type") if self.entry.get(k)}
        if len(named) > 1:
            raise ValueError(f"entry {self.index}: task and type disagree ({sorted(named)})")
        t = named.pop() if named else ("i2v" if any(self.entry.get(k) for k in IMAGE_KEYS) else "t2v")
        if t not in TASKS:
            raise ValueError(f"entry {self.index}: task {t!r} is not one of {TASKS}")
        return t

    def image(self, task: str) -> Optional[str]:
        key = _single_alias(self.entry, IMAGE_KEYS, "reference image")
        if task == "t2v":
            if key:
                raise ValueError(f"entry {self.index}: a text-to-video entry names a reference image ({key})")
            return None
        if key is None:
            raise ValueError(f"entry {self.index}: an image-to-video entry needs one of {IMAGE_KEYS}")
        raw = self.entry[key]
        if not isinstance(raw, str) or not raw.strip():
            raise ValueError(f"entry {self.index}: the reference image path is empty")
        p = Path(raw)
        if self.image_root is not None:
            if p.name in ("", ".", ".."):
                raise ValueError(f"entry {self.index}: {raw!r} has no file name to look up under image_root")
            p = self.image_root / p.name
        resolved = p.resolve()
        if self.check_images and not resolved.is_file():
            raise ValueError(f"entry {self.index}: reference image {resolved} is not a file")
        return str(resolved)

    def prompt(self, task: str) -> str:
        text = next((self.entry[k] for k in PROMPT_KEYS if self.entry.get(k)), None)
        if not isinstance(text, str) or not text.strip():
            raise ValueError(f"entry {self.index} ({task}): no prompt text in any of {PROMPT_KEYS}")
        return text

    def output(self, task: str, n_before: int) -> Path:
        ident = self.entry.get("id")
        ident = "" if ident is None else str(ident).strip()
        if ident:
            safe = re.sub(r"[^A-Za-z0-9._-]+", "_", ident).strip("._-")
            if not safe:
                raise ValueError(f"entry {self.index}: id {ident!r} leaves no usable file name")
            name = f"{task}_{safe}.mp4"
        else:
            name = str(self.entry.get("relative_path") or "").strip() or f"{task}_{n_before:04d}.mp4"
        rel = PurePosixPath(name)
        folder = self.out_root / task if self.mode == "auto" else self.out_root
        target = (folder / name).resolve()
        if (rel.is_absolute() or ".." in rel.parts or "\\" in name or rel.suffix.lower() != ".mp4"
                or not target.is_relative_to(self.out_root)):
            raise ValueError(f"entry {self.index}: output path {name!r} is not a .mp4 inside the output folder")
        return target

    def negative(self, frames: int, fps, default_negative: str):
        key = _single_alias(self.entry, NEGATIVE_KEYS, "negative prompt", truthy=False)
        if key is not None:
            return self.entry[key]
        return render_negative_duration(default_negative, frames, fps)


def load_inference_inputs(path, output_dir, *, task: str = "t2v", fps=24, fallback=121, shard_index: int = 0,
                          shard_count: int = 1, default_negative: str = "", validate_images: bool = True,
                          image_root=None) -> List[Dict]:
    """Generation records of this shard (every ``shard_count``-th record from ``shard_index``)."""
    if task not in TASKS + ("auto",):
        raise ValueError(f"task {task!r} is not t2v, i2v or auto")
    if not isinstance(validate_images, bool):
        raise ValueError("validate_images takes True or False")
    if not (type(shard_index) is int and type(shard_count) is int and 0 <= shard_index < shard_count):
        raise ValueError(f"prompt shard {shard_index!r} of {shard_count!r} is not a valid shard")
    root_images = None
    if image_root is not None:
        if not str(image_root).strip():
            raise ValueError("image_root is empty")
        root_images = Path(image_root).resolve()
        if validate_images and not root_images.is_dir():
            raise ValueError(f"image_root {root_images} is not a folder")
    out_root = Path(output_dir).resolve()
    records: List[Dict] = []
    taken = set()
    for i, entry in enumerate(_entry_list(json.loads(Path(path).read_text(encoding="utf-8")))):
        r = _EntryReader(entry, i, out_root, task, root_images, validate_images)
        t = r.task()
        if task != "auto" and t != task:
            continue
        image = r.image(t)
        prompt = r.prompt(t)
        target = r.output(t, len(records))
        if target in taken:
            raise ValueError(f"entry {i}: output {target} is produced by an earlier entry too")
        taken.add(target)
        frames = resolve_frames(entry, fps, fallback)
        rec = dict(prompt=prompt, negative_prompt=r.negative(frames, fps, default_negative), video_length=frames,
                   output_path=str(target))
        if task == "auto":
            rec["task"] = t
        if image is not None:
            rec["image_path"] = image
        records.append(rec)
    if not records:
        raise ValueError(f"{path} has no entries for task {task}")
    return records[shard_index::shard_count]


def is_complete(args) -> bool:
    """True when this output exists with the same generation settings (skip it); False when it is
    missing or half written (generate it); an error when it exists with other settings."""
    video = Path(args.output_path)
    settings = video.with_name(video.stem + "_config.json")
    if not all(p.is_file() and p.stat().st_size > 0 for p in (video, settings)):
        return False
    try:
        saved = json.loads(settings.read_text(encoding="utf-8"))["arguments"]
    except (OSError, ValueError, KeyError, TypeError):
        return False
    if not isinstance(saved, dict):
        return False
    changed = sorted(k for k, v in vars(args).items()
                     if not k.startswith("_") and k not in ROUTING_ARGS and saved.get(k, _MISSING) != v)
    if changed:
        raise ValueError(f"{video} was generated with other settings ({', '.join(changed)}); "
                         "use another output folder or turn off skip_existing")
    return True


_MISSING = object()
