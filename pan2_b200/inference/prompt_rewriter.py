"""Structured-caption tooling for generation prompts: rewrite, assemble, validate, count tokens.

The DiT was trained on structured JSON captions (style, lighting, perspective, subject declarations,
an initial-frame description, timed events with camera motion and subject actions, quality notes).
Free text is rewritten into that form by a local instruction-tuned model, then paired with a fixed
negative caption.  Same workflow as the reference's inference/prompts_rewritter.py:1-940 and its
pan-prompt-rewriter helpers (scripts/prompt_tools.py:1-286, scripts/production_tokens.py:1-28):

* ``rewrite``: batches of prompts (plain text, JSON records or lists; optional first-frame image
  for image-to-video) through a local model with a user-supplied system prompt, one worker process
  per GPU; every record gains ``refined_prompt``;
* ``assemble``: attaches the negative caption to each record -- the fixed template with its three
  ``time_range_sec`` placeholders set to ``0 to D`` and nothing else changed -- after validating the
  positive caption against the schema (:func:`validate_positive`);
* ``validate``: re-assembles and compares, and with the deployed tokenizer checks the token budgets
  the text encoder will see (positive soft limit 1,480, hard limit 1,536 caption tokens).

The system prompt, the negative template and the model are inputs (paths); nothing is downloaded.
"""
from __future__ import annotations

import argparse
import json
import os
import re
from copy import deepcopy
from decimal import Decimal
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple

POSITIVE_SOFT_LIMIT = 1480
HARD_LIMIT = 1536
DEFAULT_DURATION = 13
TOP_KEYS = ["video_style", "lighting", "perspective_view", "subjects_lifecycle", "init_frame_visual_description",
            "events", "quality"]
EVENT_KEYS = ["event_index", "time_range_sec", "event_description", "camera_motion", "contained_actions"]
CAMERA_TAGS = frozenset({"static", "pan_left", "pan_right", "tilt_up", "tilt_down", "track_left", "track_right",
                         "dolly_forward", "dolly_backward", "dolly_up", "dolly_down", "zoom_in", "zoom_out",
                         "roll_clockwise", "roll_counterclockwise", "unstable"})
SUBJECT_TOKEN = re.compile(r"<\|Subject[1-9][0-9]*\|>")
INTERVAL = re.compile(r"(\d+(?:\.\d)?) to (\d+(?:\.\d)?)")
PLACEHOLDER = re.compile(r'("time_range_sec"\s*:\s*")0 to \{duration_sec\}(")')


class CaptionError(ValueError):
    pass


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise CaptionError(msg)


def strict_loads(text) -> Any:
    """JSON without duplicate keys or non-finite numbers."""
    def pairs(kv):
        out = {}
        for k, v in kv:
            _need(k not in out, f"duplicate JSON key: {k}")
            out[k] = v
        return out

    def bad(x):
        raise CaptionError(f"non-finite JSON number: {x}")
    return json.loads(text, object_pairs_hook=pairs, parse_constant=bad)


def duration_of(value) -> Decimal:
    _need(type(value) in (int, float), "duration must be a JSON number")
    d = Decimal(str(value))
    _need(d.is_finite() and d > 0 and (d * 10) == (d * 10).to_integral_value(),
          "duration must be positive with at most one decimal place")
    return d


def _text(v, label: str) -> None:
    _need(isinstance(v, str) and bool(v.strip()), f"{label}: expected nonempty text")


def _keys(v, keys: List[str], label: str) -> None:
    _need(isinstance(v, dict) and list(v) == keys, f"{label}: keys must be {keys}")


def _interval(v) -> Tuple[Decimal, Decimal]:
    m = INTERVAL.fullmatch(v) if isinstance(v, str) else None
    _need(m is not None, f"invalid time interval {v!r}")
    a, b = Decimal(m.group(1)), Decimal(m.group(2))
    _need(0 <= a < b, f"empty or reversed interval {v!r}")
    return a, b


def validate_positive(text: str, duration: Decimal) -> Dict:
    """Parse and check one positive caption against the structured schema; returns the object."""
    _text(text, "refined_prompt")
    cap = strict_loads(text)
    _keys(cap, TOP_KEYS, "caption")
    for k in ("video_style", "lighting", "perspective_view", "init_frame_visual_description"):
        _text(cap[k], k)
        _need(not SUBJECT_TOKEN.search(cap[k]), f"{k}: subject tokens belong in declarations and actions only")
    _need(len(cap["init_frame_visual_description"].split()) <= 200, "initial description exceeds 200 words")
    subjects = cap["subjects_lifecycle"]
    _need(isinstance(subjects, list), "subjects_lifecycle must be a list")
    ids = set()
    for i, s in enumerate(subjects, 1):
        _keys(s, ["subject_id", "display_name", "subject_attribute"], "subject")
        _need(s["subject_id"] == f"<|Subject{i}|>", "subject ids must be <|Subject1|>, <|Subject2|>, ... in order")
        for k in ("display_name", "subject_attribute"):
            _text(s[k], k)
            _need(not SUBJECT_TOKEN.search(s[k]), f"{k}: unexpected subject token")
        ids.add(s["subject_id"])
    events = cap["events"]
    _need(isinstance(events, list) and bool(events), "events must be a nonempty list")
    t = Decimal(0)
    for i, ev in enumerate(events):
        _keys(ev, EVENT_KEYS, "event")
        _need(type(ev["event_index"]) is int and ev["event_index"] == i, "event indices must count from 0")
        a, b = _interval(ev["time_range_sec"])
        _need(a == t and b <= duration, "events must tile the duration contiguously")
        t = b
        _text(ev["event_description"], "event_description")
        _need(len(ev["event_description"].split()) <= 200, "event description exceeds 200 words")
        _need(not SUBJECT_TOKEN.search(ev["event_description"]), "no subject tokens in event prose")
        cam = ev["camera_motion"]
        _need(isinstance(cam, list) and bool(cam), "camera_motion must be a nonempty list")
        pos = a
        for row in cam:
            _keys(row, ["time_range_sec", "camera_motion"], "camera entry")
            ca, cb = _interval(row["time_range_sec"])
            _need(ca == pos and cb <= b, "camera entries must tile their event contiguously")
            pos = cb
            tags = row["camera_motion"]
            _need(isinstance(tags, list) and bool(tags) and all(isinstance(x, str) and x in CAMERA_TAGS for x in tags),
                  f"unknown camera tag in {tags}")
            _need(len(set(tags)) == len(tags) and ("static" not in tags or len(tags) == 1),
                  "duplicate or conflicting camera tags")
        _need(pos == b, "camera entries leave part of the event uncovered")
        acts = ev["contained_actions"]
        _need(isinstance(acts, list), "contained_actions must be a list")
        for act in acts:
            _keys(act, ["time_range_sec", "action"], "action")
            aa, ab = _interval(act["time_range_sec"])
            _need(a <= aa < ab <= b, "action outside its event")
            _text(act["action"], "action")
            toks = SUBJECT_TOKEN.findall(act["action"])
            _need(bool(toks) and act["action"].startswith(toks[0]) and set(toks) <= ids,
                  "an action starts with its performer and names only declared subjects")
    _need(t == duration, "events do not cover the requested duration exactly")
    q = cap["quality"]
    _keys(q, ["video_quality", "text_logos_overlays", "artifacts"], "quality")
    _text(q["video_quality"], "video_quality")
    _need(q["artifacts"] is None, "positive artifacts must be null")
    _need(q["text_logos_overlays"] is None or isinstance(q["text_logos_overlays"], str),
          "text_logos_overlays must be text or null")
    _need(not SUBJECT_TOKEN.search(json.dumps(q)), "no subject tokens in quality")
    return cap


def render_negative(template: str, duration) -> str:
    """The negative template with exactly its three ``0 to {duration_sec}`` spans set to the duration."""
    d = duration_of(duration) if not isinstance(duration, Decimal) else duration
    end = format(d.normalize(), "f")
    text = template.strip()
    out, n = PLACEHOLDER.subn(lambda m: m.group(1) + "0 to " + end + m.group(2), text)
    _need(n == 3, f"expected 3 duration placeholders in the negative template, found {n}")
    _keys(strict_loads(out), TOP_KEYS, "negative template")
    return out


def normalize_request(req) -> Tuple[Dict, Decimal]:
    _need(isinstance(req, dict), "a request must be an object")
    _need(isinstance(req.get("original_prompt"), str) and req["original_prompt"].strip(),
          "original_prompt must be nonempty text")
    _need(not ({"refined_prompt", "negative_prompt"} & set(req)), "requests must not carry captions already")
    row = deepcopy(req)
    vals = [duration_of(row[k]) for k in ("duration_sec", "target_duration_sec") if k in row]
    _need(len(set(vals)) <= 1, "conflicting duration fields")
    if not vals:
        row["duration_sec"] = DEFAULT_DURATION
        return row, Decimal(DEFAULT_DURATION)
    return row, vals[0]


def _as_list(x) -> List:
    if isinstance(x, list):
        _need(bool(x), "empty batches are not supported")
        return x
    _need(isinstance(x, dict), "expected an object or a nonempty list")
    return [x]


def assemble(request, positive, negative_template: str):
    """Records = clean request + validated ``refined_prompt`` + rendered ``negative_prompt``."""
    _need(type(request) is type(positive), "request and positive must both be objects or both lists")
    reqs, poss = _as_list(request), _as_list(positive)
    _need(len(reqs) == len(poss), "request / positive batch lengths differ")
    out = []
    for raw, pos in zip(reqs, poss):
        _keys(pos, ["refined_prompt"], "authored positive")
        row, d = normalize_request(raw)
        validate_positive(pos["refined_prompt"], d)
        row["refined_prompt"] = pos["refined_prompt"]
        row["negative_prompt"] = render_negative(negative_template, d)
        out.append(row)
    return out if isinstance(request, list) else out[0]


class EncoderTokenCounter:
    """Caption tokens the DiT receives (chat template minus the template prefix), with the same
    crop as :class:`pan2_b200.models.text_encoder.QwenCaptionCodec`."""

    def __init__(self, tokenizer=None, tokenizer_dir: Optional[str] = None):
        if tokenizer is None:
            from transformers import AutoTokenizer
            tokenizer = AutoTokenizer.from_pretrained(tokenizer_dir, local_files_only=True)
        from ..models.text_encoder import QwenCaptionCodec
        self.codec = QwenCaptionCodec.__new__(QwenCaptionCodec)
        self.codec.tokenizer = tokenizer
        self.codec._prefix = None
        self.codec.max_caption_tokens = 1 << 30

    def __call__(self, text: str) -> int:
        return int(self.codec._ids(text, None).numel()) - self.codec.prefix_len


def validate_records(records, counter: Optional[EncoderTokenCounter] = None) -> Dict:
    """Schema + budget check of assembled records; returns a report dict (``ok`` is the verdict)."""
    report = {"ok": True, "errors": [], "checks": [], "token_verified": counter is not None}
    for i, row in enumerate(_as_list(records)):
        try:
            _, d = normalize_request({k: v for k, v in row.items() if k not in ("refined_prompt", "negative_prompt")})
            validate_positive(row["refined_prompt"], d)
            _keys(strict_loads(row["negative_prompt"]), TOP_KEYS, "negative")
            if counter is not None:
                p, n = counter(row["refined_prompt"]), counter(row["negative_prompt"])
                ok = p <= POSITIVE_SOFT_LIMIT and max(p, n) <= HARD_LIMIT
                report["checks"].append({"index": i, "positive_tokens": p, "negative_tokens": n, "ok": ok})
                if not ok:
                    report["ok"] = False
                    report["errors"].append(f"record {i}: token budget exceeded ({p} / {n})")
        except (CaptionError, KeyError) as e:
            report["ok"] = False
            report["errors"].append(f"record {i}: {e}")
    return report


# ---------------------------------------------------------------------------------------------- rewriting
def _records_from(path_or_text: str) -> Tuple[List[Dict], bool]:
    p = Path(path_or_text)
    if p.exists() and p.suffix == ".json":
        doc = json.loads(p.read_text(encoding="utf-8"))
        if isinstance(doc, dict) and any(k in doc for k in ("entries", "prompts", "data")):
            doc = doc[next(k for k in ("entries", "prompts", "data") if k in doc)]
        items = doc if isinstance(doc, list) else [doc]
        recs = []
        for it in items:
            if isinstance(it, str):
                recs.append({"original_prompt": it})
            else:
                rec = dict(it)
                rec.setdefault("original_prompt", rec.get("prompt") or rec.get("caption") or "")
                recs.append(rec)
        return recs, True
    return [{"original_prompt": path_or_text}], False


def _rewrite_worker(gpu: int, model_path: str, system_prompt: str, items: List[Tuple[int, Dict]], max_new_tokens: int,
                    out_path: str) -> None:
    import torch
    from transformers import AutoModelForImageTextToText, AutoProcessor
    dev = f"cuda:{gpu}" if torch.cuda.is_available() else "cpu"
    proc = AutoProcessor.from_pretrained(model_path, local_files_only=True)
    model = AutoModelForImageTextToText.from_pretrained(model_path, local_files_only=True, dtype=torch.bfloat16,
                                                        device_map=dev).eval()
    results = {}
    for idx, rec in items:
        content = []
        if rec.get("image_path"):
            from PIL import Image
            content.append({"type": "image", "image": Image.open(rec["image_path"]).convert("RGB")})
        dur = rec.get("duration_sec", rec.get("target_duration_sec", DEFAULT_DURATION))
        content.append({"type": "text", "text": json.dumps({"original_prompt": rec["original_prompt"],
                                                            "duration_sec": dur}, ensure_ascii=False)})
        msgs = [{"role": "system", "content": [{"type": "text", "text": system_prompt}]},
                {"role": "user", "content": content}]
        inputs = proc.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True, return_dict=True,
                                          return_tensors="pt").to(dev)
        with torch.no_grad():
            ids = model.generate(**inputs, max_new_tokens=max_new_tokens, do_sample=False)
        text = proc.decode(ids[0, inputs["input_ids"].shape[1]:], skip_special_tokens=True).strip()
        try:
            text = strict_loads(text).get("refined_prompt", text)
        except (ValueError, AttributeError):
            pass
        results[idx] = text if isinstance(text, str) else json.dumps(text, ensure_ascii=False, separators=(",", ":"))
    with open(out_path, "w", encoding="utf-8") as f:
        json.dump(results, f)


def rewrite(records: List[Dict], model_path: str, system_prompt: str, gpus: Sequence[int],
            max_new_tokens: int = 4096, workdir: str = ".") -> List[str]:
    """Refined prompts for ``records`` (one worker per GPU, round-robin split, order preserved)."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    gpus = list(gpus) or [0]
    procs, outs = [], []
    for w, g in enumerate(gpus):
        items = [(i, r) for i, r in enumerate(records) if i % len(gpus) == w]
        if not items:
            continue
        out = os.path.join(workdir, f".rewrite_part{w}.json")
        outs.append(out)
        p = ctx.Process(target=_rewrite_worker, args=(g, model_path, system_prompt, items, max_new_tokens, out))
        p.start()
        procs.append(p)
    for p in procs:
        p.join()
        if p.exitcode != 0:
            raise RuntimeError(f"rewrite worker exited with {p.exitcode}")
    merged = {}
    for out in outs:
        with open(out) as f:
            merged.update({int(k): v for k, v in json.load(f).items()})
        os.remove(out)
    return [merged[i] for i in range(len(records))]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("rewrite", help="free text / prompt JSON -> records with refined_prompt")
    r.add_argument("--input", required=True, help="a prompt, or a .json file of records")
    r.add_argument("--output", required=True)
    r.add_argument("--model", required=True, help="local instruction model folder")
    r.add_argument("--system_prompt", required=True, help="text file with the authoring policy")
    r.add_argument("--negative_template", default=None, help="assemble negatives too (template file)")
    r.add_argument("--gpus", default="0", help="comma-separated GPU ids")
    r.add_argument("--max_new_tokens", type=int, default=4096)
    a = sub.add_parser("assemble", help="request + authored positive -> final records")
    a.add_argument("--request", required=True)
    a.add_argument("--positive", required=True)
    a.add_argument("--negative_template", required=True)
    a.add_argument("--output", required=True)
    v = sub.add_parser("validate", help="schema and token-budget check of final records")
    v.add_argument("--records", required=True)
    v.add_argument("--tokenizer", default=None, help="deployed text-encoder tokenizer folder")
    v.add_argument("--report", required=True)
    args = ap.parse_args(argv)
    if args.cmd == "rewrite":
        recs, _ = _records_from(args.input)
        system = Path(args.system_prompt).read_text(encoding="utf-8")
        refined = rewrite(recs, args.model, system, [int(x) for x in args.gpus.split(",") if x.strip()],
                          args.max_new_tokens, os.path.dirname(os.path.abspath(args.output)))
        for rec, txt in zip(recs, refined):
            rec["refined_prompt"] = txt
        if args.negative_template:
            tmpl = Path(args.negative_template).read_text(encoding="utf-8")
            for rec in recs:
                _, d = normalize_request({k: v for k, v in rec.items() if k != "refined_prompt"})
                rec["negative_prompt"] = render_negative(tmpl, d)
        Path(args.output).write_text(json.dumps(recs, ensure_ascii=False, indent=2) + "\n", encoding="utf-8")
        return 0
    if args.cmd == "assemble":
        out = assemble(strict_loads(Path(args.request).read_text(encoding="utf-8")),
                       strict_loads(Path(args.positive).read_text(encoding="utf-8")),
                       Path(args.negative_template).read_text(encoding="utf-8"))
        Path(args.output).write_text(json.dumps(out, ensure_ascii=False, indent=2) + "\n", encoding="utf-8")
        return 0
    counter = EncoderTokenCounter(tokenizer_dir=args.tokenizer) if args.tokenizer else None
    rep = validate_records(strict_loads(Path(args.records).read_text(encoding="utf-8")), counter)
    Path(args.report).write_text(json.dumps(rep, indent=2) + "\n", encoding="utf-8")
    print(json.dumps({k: rep[k] for k in ("ok", "token_verified", "errors")}))
    return 0 if rep["ok"] and rep["token_verified"] else (2 if rep["ok"] else 1)


if __name__ == "__main__":
    raise SystemExit(main())
