"""Prompt-file parsing for generation, frame counts, negative-prompt rendering and resume checks.

Behaviour of the reference's inference/inputs.py:1-189:

* a prompt file is a JSON list of entries, or an object with exactly one of ``entries`` / ``prompts`` /
  ``data`` holding that list;
* an entry's task is ``task`` / ``type``, else ``i2v`` when it names a reference image (``image_path``,
  ``image`` or ``ref_image``), else ``t2v``; its prompt is the first non-empty of ``refined_prompt``,
  ``refined_prompts``, ``prompt``, ``caption``;
* the frame count is ``4 * ceil(duration_sec * fps / 4) + 1`` (the counts the Wan VAE encodes), else
  ``frames`` / ``num_target_frames``, else the fallback;
* the output is ``<task>_<sanitised id>.mp4`` or ``relative_path``; unsafe or duplicate paths are
  rejected; with task ``auto`` outputs are namespaced by task;
* a structured (JSON) negative prompt has every ``time_range_sec`` rewritten to the clip's duration;
* :func:`is_complete` skips an output only when the video and its ``_config.json`` exist and every
  generation argument matches; a mismatch is an error (fail closed).
"""
from __future__ import annotations

import json
import re
from decimal import ROUND_CEILING, Decimal, InvalidOperation
from pathlib import Path, PurePosixPath
from typing import Dict, List

GUIDANCE_KEYS = ("cfg_start_step", "cfg_end_step", "stg_scale", "stg_skip_layers")
ROUTING_ARGS = {"prompt_json", "output_dir", "prompt_shard_index", "prompt_shard_count", "skip_existing",
                "output_path", "task", "image_root"}


def _positive(value, name: str, integer: bool = False) -> Decimal:
    if isinstance(value, bool):
        raise ValueError(f"{name} must be positive and finite")
    try:
        d = Decimal(str(value))
    except (InvalidOperation, ValueError):
        raise ValueError(f"{name} must be positive and finite") from None
    if not d.is_finite() or d <= 0 or (integer and d != d.to_integral_value()):
        raise ValueError(f"{name} must be positive and finite" + (" integer" if integer else ""))
    return d


def resolve_frames(entry: Dict, fps=24, fallback=121) -> int:
    fps_d = _positive(fps, "fps")
    fb = _positive(fallback, "video_length", integer=True)
    if entry.get("duration_sec") is not None:
        dur = _positive(entry["duration_sec"], "duration_sec")
        return int((dur * fps_d / 4).to_integral_value(rounding=ROUND_CEILING)) * 4 + 1
    for key in ("frames", "num_target_frames"):
        if entry.get(key) is not None:
            return int(_positive(entry[key], key, integer=True))
    return int(fb)


def render_negative_duration(text, video_length: int, fps=24):
    try:
        doc = json.loads(text)
    except (TypeError, json.JSONDecodeError):
        return text
    if not isinstance(doc, dict):
        return text
    span = f"0 to {(int(video_length) - 1) / float(fps):g}"

    def walk(node):
        if isinstance(node, dict):
            return {k: (span if k == "time_range_sec" else walk(v)) for k, v in node.items()}
        if isinstance(node, list):
            return [walk(v) for v in node]
        return node

    return json.dumps(walk(doc), ensure_ascii=False, separators=(",", ":"))


def _entries(payload):
    if isinstance(payload, dict):
        keys = [k for k in ("entries", "prompts", "data") if k in payload]
        if len(keys) != 1:
            raise ValueError("a prompt wrapper object needs exactly one entries/prompts/data list")
        payload = payload[keys[0]]
    if not isinstance(payload, list):
        raise ValueError("the prompt JSON must contain a list of entries")
    return payload


def load_inference_inputs(path, output_dir, *, task: str = "t2v", fps=24, fallback=121, shard_index: int = 0,
                          shard_count: int = 1, default_negative: str = "", validate_images: bool = True,
                          image_root=None) -> List[Dict]:
    if task not in ("t2v", "i2v", "auto"):
        raise ValueError("task must be t2v, i2v or auto")
    if type(validate_images) is not bool:
        raise ValueError("validate_images must be a boolean")
    if image_root is not None:
        if not str(image_root).strip():
            raise ValueError("image_root must be a nonempty local directory path")
        image_root = Path(image_root).resolve()
        if validate_images and not image_root.is_dir():
            raise ValueError(f"image_root must be an existing local directory: {image_root}")
    if type(shard_count) is not int or type(shard_index) is not int or not 0 <= shard_index < shard_count:
        raise ValueError("require 0 <= prompt_shard_index < prompt_shard_count")
    root = Path(output_dir).resolve()
    records: List[Dict] = []
    seen = set()
    for entry in _entries(json.loads(Path(path).read_text(encoding="utf-8"))):
        if not isinstance(entry, dict):
            raise ValueError("prompt entries must be objects")
        declared = {str(entry[k]).strip().lower() for k in ("task", "type") if entry.get(k)}
        if len(declared) > 1:
            raise ValueError("conflicting task/type fields")
        img_keys = [k for k in ("image_path", "image", "ref_image") if entry.get(k)]
        etask = declared.pop() if declared else ("i2v" if img_keys else "t2v")
        if etask not in ("t2v", "i2v"):
            raise ValueError(f"unsupported task: {etask}")
        if task != "auto" and etask != task:
            continue
        image_path = None
        if etask == "i2v":
            if not img_keys:
                raise ValueError("an I2V entry requires image_path (or image / ref_image)")
            if len({json.dumps(entry[k]) for k in img_keys}) > 1:
                raise ValueError("conflicting reference image aliases")
            image_path = entry[img_keys[0]]
            if not isinstance(image_path, str) or not image_path.strip():
                raise ValueError("the I2V reference image must be an existing local file")
            if image_root is not None:
                base = Path(image_path).name
                if base in ("", ".", ".."):
                    raise ValueError("the I2V reference image needs a file name for image_root remapping")
                image_path = image_root / base
            image_path = str(Path(image_path).resolve())
            if validate_images and not Path(image_path).is_file():
                raise ValueError(f"the I2V reference image must be an existing local file: {image_path}")
        elif img_keys:
            raise ValueError("a T2V entry cannot name a reference image")
        prompt = next((entry[k] for k in ("refined_prompt", "refined_prompts", "prompt", "caption") if entry.get(k)),
                      None)
        if not isinstance(prompt, str) or not prompt.strip():
            raise ValueError(f"{etask.upper()} entry needs a nonempty positive prompt")
        eid = "" if entry.get("id") is None else str(entry["id"]).strip()
        if eid:
            name = re.sub(r"[^A-Za-z0-9._-]+", "_", eid).strip("._-")
            if not name:
                raise ValueError("empty output id after sanitisation")
            relative = f"{etask}_{name}.mp4"
        else:
            relative = str(entry.get("relative_path") or "").strip() or f"{etask}_{len(records):04d}.mp4"
        rel = PurePosixPath(relative)
        base_dir = root / etask if task == "auto" else root
        target = (base_dir / relative).resolve()
        if (rel.is_absolute() or ".." in rel.parts or "\\" in relative or rel.suffix.lower() != ".mp4"
                or not target.is_relative_to(root)):
            raise ValueError(f"unsafe output path: {relative}")
        if target in seen:
            raise ValueError(f"duplicate output path: {relative}")
        seen.add(target)
        frames = resolve_frames(entry, fps, fallback)
        neg_keys = [k for k in ("negative_prompt", "negative_prompts", "neg_prompt") if k in entry]
        if len({json.dumps(entry[k]) for k in neg_keys}) > 1:
            raise ValueError("conflicting negative prompt aliases")
        negative = entry[neg_keys[0]] if neg_keys else render_negative_duration(default_negative, frames, fps)
        rec = dict(prompt=prompt, negative_prompt=negative, video_length=frames, output_path=str(target))
        if task == "auto":
            rec["task"] = etask
        if etask == "i2v":
            rec["image_path"] = image_path
        records.append(rec)
    if not records:
        raise ValueError(f"the prompt JSON contains no {task.upper()} entries")
    return records[shard_index::shard_count]


def is_complete(args) -> bool:
    video = Path(args.output_path)
    cfg = video.with_name(video.stem + "_config.json")
    if not (video.is_file() and video.stat().st_size and cfg.is_file() and cfg.stat().st_size):
        return False
    try:
        saved = json.loads(cfg.read_text(encoding="utf-8"))["arguments"]
    except (OSError, ValueError, KeyError, TypeError):
        return False
    if not isinstance(saved, dict):
        return False
    diff = [k for k, v in vars(args).items()
            if not k.startswith("_") and k not in ROUTING_ARGS and (k not in saved or saved[k] != v)]
    if diff:
        raise ValueError(f"existing output settings differ for {video}: {', '.join(diff)}")
    return True
